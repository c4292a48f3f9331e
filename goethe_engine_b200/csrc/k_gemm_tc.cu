// Quantized weight GEMM on the 5th-generation tensor cores: tcgen05.mma (kind::f16, f16 x f16 -> f32) with the
// accumulator in tensor memory.
//
//   y[t, n] = sum_k act[t, k] * W[n, k]          (the reference's `w @ h`, ref.py:51-59, for all token rows at once)
//
// One CTA computes a 128-row band of W (the MMA's M) against a tile of NT token rows (the MMA's N) over a fixed range
// of K (split-K, fixed per weight). Warp roles:
//   warp 0       producer of raw weight tiles: one 1-D bulk copy per tile (128 rows x 256 K, the GGUF blocks as relaid
//                at load), up to 3-4 tiles ahead;
//   warp 10      producer of activations: one 2-D tensor-map copy per 64-K stage (NT rows, 128-byte swizzle);
//   warp 1       TMEM allocation; one elected thread issues 4 tcgen05.mma (K = 16 each, weights from TMEM,
//                activations from shared memory) per 64-K stage and commits each stage back to the producers;
//   warps 2-9    dequantize each 64-K stage of the raw tile (two threads per weight row; f16 arithmetic, one rounding)
//                straight into tensor memory (tcgen05.st): the MMA reads its weight operand from TMEM, so shared
//                memory carries only the raw tiles and the activations;
//   warps 11-14  epilogue: tcgen05.ld of the accumulator (two buffers, so it overlaps the next unit's MMAs) and the
//                store, residual add, SwiGLU or split-K partial.
// Every output element accumulates its K range in one order whatever NT is, so a row's result does not depend on the
// rest of the batch. Every copy here reads this GPU's global memory into this CTA's own shared memory.
//
// Every mbarrier wait is bounded (about 2 s on the global timer); a timeout writes a code to the error word, the CTA
// drains what it issued (again bounded), frees its tensor memory and returns; gc_step reports GC_E_DEVICE.
#include <cuda.h>

#include "common.cuh"
#include "kernels.h"

namespace gck {
namespace {

constexpr int kKS = 128;                   // K per stage: two 128-byte swizzle rows of f16 (8 MMAs of K = 16)
constexpr int kSub = kBK / kKS;            // stages per raw tile (2)
constexpr int kThreads = 480;              // 15 warps
constexpr int kDeqWarps = 8;               // warps 2-9: two threads per weight row
constexpr int kEpiWarp0 = 11;              // warps 11-14: epilogue (TMEM lane quarters 3, 0, 1, 2)
constexpr unsigned long long kTimeoutNs = 2000000000ull;

enum ErrCode { kErrRawFull = 1, kErrRawEmpty, kErrStageEmpty, kErrAFull, kErrBFull, kErrAcc };

template <int TYPE>
struct TileFmt;
template <>
struct TileFmt<kQ4_K> {
  static constexpr int BYTES = kBM * 144;   // 128 x 16 B headers, then [4 stages][2 pieces][128 rows][16 B]
  static constexpr int PIECES = 2;
};
template <>
struct TileFmt<kQ8_0> {
  static constexpr int BYTES = kBM * 272;   // 128 x 16 B (8 fp16 d), then [4 stages][4 pieces][128 rows][16 B]
  static constexpr int PIECES = 4;
};

// ---------------------------------------------------------------------------------------------------- PTX wrappers
GCK_DEV void mbar_init(uint64_t *b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(b)), "r"(count));
}
GCK_DEV void mbar_expect_tx(uint64_t *b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
GCK_DEV void mbar_arrive(uint64_t *b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(b)) : "memory");
}
GCK_DEV bool mbar_try(uint64_t *b, uint32_t parity) {
  // suspends the thread (up to ~1 us) until the phase completes instead of returning at once, so waiting warps leave
  // the issue slots to the dequantizing warps
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 1000;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
GCK_DEV unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;\n" : "=l"(t));
  return t;
}
// Bounded wait for the phase of the given parity; false (and the error word set) on timeout. Each try suspends the
// thread until the phase completes (or ~1 us); the global timer is read every 64 tries.
GCK_DEV bool mbar_wait(uint64_t *b, uint32_t parity, int *err, int code) {
  if (mbar_try(b, parity)) return true;
  const unsigned long long t0 = now_ns();
  for (uint32_t n = 1;; n++) {
    if (mbar_try(b, parity)) return true;
    if ((n & 63u) == 0 && now_ns() - t0 > kTimeoutNs) {
      atomicCAS(err, 0, code);
      return false;
    }
  }
}
// the same for waits expected to be long (the epilogue waiting for a unit's accumulator): back off between tries
GCK_DEV bool mbar_wait_sleep(uint64_t *b, uint32_t parity, int *err, int code) {
  if (mbar_try(b, parity)) return true;
  const unsigned long long t0 = now_ns();
  for (uint32_t n = 1;; n++) {
    __nanosleep(256);
    if (mbar_try(b, parity)) return true;
    if ((n & 63u) == 0 && now_ns() - t0 > kTimeoutNs) {
      atomicCAS(err, 0, code);
      return false;
    }
  }
}

GCK_DEV void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
GCK_DEV void tma_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
GCK_DEV void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }
GCK_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
GCK_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

// K-major operand in the 128-byte swizzle: rows of 128 B, 8-row atoms 1024 B apart (SBO), version 1
GCK_DEV uint64_t umma_desc(const void *p) {
  uint64_t a = smem_u32(p);
  return ((a >> 4) & 0x3FFFull) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}
GCK_DEV void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
GCK_DEV void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(smem_u32(bar))
               : "memory");
}
GCK_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}

// ---------------------------------------------------------------------------------------------------- dequant
GCK_DEV uint32_t hsub2_u(uint32_t a, uint32_t b) {
  __half2 r = __hsub2(*reinterpret_cast<__half2 *>(&a), *reinterpret_cast<__half2 *>(&b));
  return *reinterpret_cast<uint32_t *>(&r);
}
GCK_DEV uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
  __half2 r = __hfma2(*reinterpret_cast<__half2 *>(&a), *reinterpret_cast<__half2 *>(&b), *reinterpret_cast<__half2 *>(&c));
  return *reinterpret_cast<uint32_t *>(&r);
}
GCK_DEV uint32_t hmul2_u(uint32_t a, uint32_t b) {
  __half2 r = __hmul2(*reinterpret_cast<__half2 *>(&a), *reinterpret_cast<__half2 *>(&b));
  return *reinterpret_cast<uint32_t *>(&r);
}
GCK_DEV uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;\n" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
// 4 byte values 0..255 in x -> two half2 (1024 + b0, 1024 + b1), (1024 + b2, 1024 + b3): exact
GCK_DEV void bytes_to_h2(uint32_t x, uint32_t &lo, uint32_t &hi) {
  lo = prmt(x, 0x64646464u, 0x5140u);
  hi = prmt(x, 0x64646464u, 0x5342u);
}

// Q4_K super-block header words (bytes 4..15 of the block) -> the 8 six-bit scales and mins, one per byte:
// scales 0-3 / mins 0-3 are the low 6 bits of bytes 0-3 / 4-7; scales 4-7 / mins 4-7 take their low 4 bits from the
// low / high nibbles of bytes 8-11 and their top 2 bits from the top 2 bits of bytes 0-3 / 4-7.
struct Q4kScales {
  uint32_t sc_lo, sc_hi, m_lo, m_hi;
};
GCK_DEV Q4kScales q4k_scales(uint32_t w0, uint32_t w1, uint32_t w2) {
  Q4kScales q;
  q.sc_lo = w0 & 0x3F3F3F3Fu;
  q.m_lo = w1 & 0x3F3F3F3Fu;
  q.sc_hi = (w2 & 0x0F0F0F0Fu) | ((w0 >> 2) & 0x30303030u);
  q.m_hi = ((w2 >> 4) & 0x0F0F0F0Fu) | ((w1 >> 2) & 0x30303030u);
  return q;
}

// Q4_K: stage j (64 K) of row r, half h: quant bytes 16h .. 16h+15 of the stage's 32 (one piece, read by this thread
// only). Low nibbles are k = 16h .. 16h+15 (sub-block 2j), high nibbles k = 32 + 16h .. (sub-block 2j+1).
// out[0..7] = TMEM columns 8h .. 8h+7, out[8..15] = columns 16 + 8h .. (two f16 per column, lower k in the low half).
GCK_DEV void dequant_q4k(const uint8_t *raw, int r, int j, int h, uint32_t d_dm, const Q4kScales &qs, uint32_t (&out)[16]) {
  const uint32_t scw = j < 2 ? qs.sc_lo : qs.sc_hi, mw = j < 2 ? qs.m_lo : qs.m_hi;
  const int sh = 16 * (j & 1);
  const int sc0 = (scw >> sh) & 0xFF, sc1 = (scw >> (sh + 8)) & 0xFF;
  const int m0 = (mw >> sh) & 0xFF, m1 = (mw >> (sh + 8)) & 0xFF;
  __half2 dd = *reinterpret_cast<__half2 *>(&d_dm);
  float d = __low2float(dd), dm = __high2float(dd);
  __half2 s0 = __float2half2_rn(d * static_cast<float>(sc0)), o0 = __float2half2_rn(-dm * static_cast<float>(m0));
  __half2 s1 = __float2half2_rn(d * static_cast<float>(sc1)), o1 = __float2half2_rn(-dm * static_cast<float>(m1));
  const uint32_t S0 = *reinterpret_cast<uint32_t *>(&s0), O0 = *reinterpret_cast<uint32_t *>(&o0);
  const uint32_t S1 = *reinterpret_cast<uint32_t *>(&s1), O1 = *reinterpret_cast<uint32_t *>(&o1);
  const uint32_t K1024 = 0x64006400u;
  const uint4 q = *reinterpret_cast<const uint4 *>(raw + kBM * 16 + (j * 2 + h) * (kBM * 16) + r * 16);
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; i++) {
    uint32_t a0, a1, b0, b1;
    bytes_to_h2(w[i] & 0x0F0F0F0Fu, a0, a1);
    bytes_to_h2((w[i] >> 4) & 0x0F0F0F0Fu, b0, b1);
    out[2 * i] = hfma2_u(hsub2_u(a0, K1024), S0, O0);
    out[2 * i + 1] = hfma2_u(hsub2_u(a1, K1024), S0, O0);
    out[8 + 2 * i] = hfma2_u(hsub2_u(b0, K1024), S1, O1);
    out[8 + 2 * i + 1] = hfma2_u(hsub2_u(b1, K1024), S1, O1);
  }
}

// Q8_0: stage j of row r, half h: block 2j + h (k = 32h .. 32h+31) -> TMEM columns 16h .. 16h+15
GCK_DEV void dequant_q80(const uint8_t *raw, int r, int j, int h, const uint4 &hdr, uint32_t (&out)[16]) {
  const uint32_t K1152 = 0x64806480u;   // 1024 + 128
  const uint32_t dw = j == 0 ? hdr.x : j == 1 ? hdr.y : j == 2 ? hdr.z : hdr.w;
  const uint32_t D = (h ? (dw >> 16) : (dw & 0xFFFFu)) * 0x10001u;
#pragma unroll
  for (int pp = 0; pp < 2; pp++) {
    const uint4 q = *reinterpret_cast<const uint4 *>(raw + kBM * 16 + (j * 4 + 2 * h + pp) * (kBM * 16) + r * 16);
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
      uint32_t a0, a1;
      bytes_to_h2(w[i] ^ 0x80808080u, a0, a1);
      out[8 * pp + 2 * i] = hmul2_u(hsub2_u(a0, K1152), D);
      out[8 * pp + 2 * i + 1] = hmul2_u(hsub2_u(a1, K1152), D);
    }
  }
}

GCK_DEV void tmem_st8(uint32_t taddr, const uint32_t *v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};\n" ::"r"(taddr), "r"(v[0]), "r"(v[1]),
               "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}
GCK_DEV void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }
GCK_DEV void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(
          tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// One ring of R stages. Stage s: 64 TMEM columns of dequantized weights (128 rows x 128 K, two f16 per column) after
// the ACC accumulator buffers, and two shared-memory activation tiles of NT rows x 64 K (128-byte swizzle). Raw
// weight tiles (HBM lookahead: 4 Q4_K = 72 KB or 3 Q8_0 = 102 KB per SM) have their own ring.
template <int TYPE, int NT>
struct Shape {
  static constexpr int STAGE_B = 2 * NT * 128;
  static constexpr int NCOLS = NT <= 32 ? 32 : NT <= 64 ? 64 : NT <= 128 ? 128 : 256;
  static constexpr int ACC = NT <= 128 ? 2 : 1;
  static constexpr int RAW = TYPE == kQ4_K ? 4 : (NT >= 256 ? 2 : 3);
  static constexpr int R_TMEM = (512 - ACC * NCOLS) / 64;
  static constexpr int R_SMEM = (216 * 1024 - RAW * TileFmt<TYPE>::BYTES) / STAGE_B;
  static constexpr int R0 = R_TMEM < R_SMEM ? R_TMEM : R_SMEM;
  static constexpr int R = R0 > 8 ? 8 : R0;
  static_assert(R >= 2, "stage ring too shallow");
};

constexpr int kXchg = 64 * 17 * 4;         // SwiGLU hand-off: 64 rows x 16 columns (+1 pad) of f32

template <int TYPE, int NT>
constexpr int smem_total() {
  using S = Shape<TYPE, NT>;
  // at least 120 KB: one CTA per SM, since each takes all 512 TMEM columns
  constexpr int need = 1024 + S::R * S::STAGE_B + S::RAW * TileFmt<TYPE>::BYTES + kXchg + 512;
  return need > 120 * 1024 ? need : 120 * 1024;
}

// Work unit w (0 .. units-1) = (token tile, weight tile, K split); a CTA takes units blockIdx.x, + gridDim.x, ...
struct Unit {
  int nt, split, tt, kt0, per;
};
GCK_DEV Unit unit_of(int w, int NTW, int KT, int splits) {
  Unit u;
  u.tt = w / (NTW * splits);
  int rem = w % (NTW * splits);
  u.nt = rem / splits;
  u.split = rem % splits;
  const int base = KT / splits, extra = KT % splits;   // the first KT % splits splits take one more raw tile
  u.per = base + (u.split < extra ? 1 : 0);
  u.kt0 = u.split * base + min(u.split, extra);
  return u;
}

template <int TYPE, int NT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const uint8_t *__restrict__ W, int NTW, int KT, int splits, int units,
                   const __grid_constant__ CUtensorMap tmap, int T, Epi epi, float *part, int Npad, int *err) {
  using F = TileFmt<TYPE>;
  using S = Shape<TYPE, NT>;
  constexpr int RS = S::RAW, SR = S::R, ACC = S::ACC;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sB = smem;
  uint8_t *sRaw = sB + SR * S::STAGE_B;
  float *xchg = reinterpret_cast<float *>(sRaw + RS * F::BYTES);
  uint64_t *bars = reinterpret_cast<uint64_t *>(reinterpret_cast<uint8_t *>(xchg) + kXchg);
  uint64_t *raw_full = bars, *raw_empty = raw_full + RS;
  uint64_t *a_full = raw_empty + RS, *st_empty = a_full + SR, *b_full = st_empty + SR;
  uint64_t *acc_full = b_full + SR, *acc_empty = acc_full + 2, *mma_done = acc_empty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int i = 0; i < RS; i++) { mbar_init(&raw_full[i], 1); mbar_init(&raw_empty[i], kDeqWarps); }
    for (int i = 0; i < SR; i++) { mbar_init(&a_full[i], kDeqWarps); mbar_init(&st_empty[i], 1); mbar_init(&b_full[i], 1); }
    for (int i = 0; i < 2; i++) { mbar_init(&acc_full[i], 1); mbar_init(&acc_empty[i], 4); }
    mbar_init(mma_done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    fence_async_smem();
  }
  if (warp == 1) {   // all 512 columns: ACC accumulator buffers, then the weight stages (one CTA per SM)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_a = tmem + ACC * S::NCOLS;   // weight stage s at columns tmem_a + 64 * s

  if (warp == 0) {
    if (lane == 0) {
      // ---- raw weight tiles: one bulk copy each, up to RS tiles ahead, across unit boundaries
      long c = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < units && ok; w += gridDim.x) {
        const Unit un = unit_of(w, NTW, KT, splits);
        for (int u = 0; u < un.per; u++, c++) {
          const int rs = static_cast<int>(c % RS);
          if (!(ok = mbar_wait(&raw_empty[rs], static_cast<uint32_t>((c / RS) & 1) ^ 1, err, kErrRawEmpty))) break;
          mbar_expect_tx(&raw_full[rs], F::BYTES);
          bulk_g2s(sRaw + rs * F::BYTES, W + (static_cast<size_t>(un.nt) * KT + un.kt0 + u) * F::BYTES, F::BYTES,
                   &raw_full[rs]);
        }
      }
      // every issued copy has landed before the CTA may exit (the last phase of each slot; bounded)
      for (long i = c > RS ? c - RS : 0; i < c; i++) mbar_wait(&raw_full[i % RS], static_cast<uint32_t>((i / RS) & 1), err, kErrRawFull);
    }
  } else if (warp == 10) {
    if (lane == 0) {
      // ---- activation stages: two tensor-map copies (64 K each) per 128-K stage, up to SR stages ahead
      long c = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < units && ok; w += gridDim.x) {
        const Unit un = unit_of(w, NTW, KT, splits);
        for (int i = 0; i < un.per * kSub; i++, c++) {
          const int s = static_cast<int>(c % SR);
          if (!(ok = mbar_wait(&st_empty[s], static_cast<uint32_t>((c / SR) & 1) ^ 1, err, kErrStageEmpty))) break;
          mbar_expect_tx(&b_full[s], S::STAGE_B);
          const int x = (un.kt0 + i / kSub) * kBK + (i % kSub) * kKS;
          tma_2d(sB + s * S::STAGE_B, &tmap, x, un.tt * NT, &b_full[s]);
          tma_2d(sB + s * S::STAGE_B + NT * 128, &tmap, x + 64, un.tt * NT, &b_full[s]);
        }
      }
      for (long i = c > SR ? c - SR : 0; i < c; i++) mbar_wait(&b_full[i % SR], static_cast<uint32_t>((i / SR) & 1), err, kErrBFull);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer: accumulator buffer (local unit index) % 2
      const uint32_t idesc = (1u << 4) | (static_cast<uint32_t>(NT >> 3) << 17) | (static_cast<uint32_t>(kBM >> 4) << 24);
      long ca = 0;
      int lu = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < units && ok; w += gridDim.x, lu++) {
        const Unit un = unit_of(w, NTW, KT, splits);
        const int ab = ACC == 2 ? (lu & 1) : 0;
        const uint32_t ph = ACC == 2 ? static_cast<uint32_t>((lu >> 1) & 1) : static_cast<uint32_t>(lu & 1);
        if (!(ok = mbar_wait(&acc_empty[ab], ph ^ 1, err, kErrAcc))) break;
        tc_fence_after();
        const uint32_t dt = tmem + ab * S::NCOLS;
        for (int i = 0; i < un.per * kSub; i++, ca++) {
          const int s = static_cast<int>(ca % SR);
          // a_full covers both operands: the dequant warps signal it only after the stage's activations landed
          if (!(ok = mbar_wait(&a_full[s], static_cast<uint32_t>((ca / SR) & 1), err, kErrAFull))) break;
          tc_fence_after();
          const uint64_t bd0 = umma_desc(sB + s * S::STAGE_B), bd1 = umma_desc(sB + s * S::STAGE_B + NT * 128);
          const uint32_t at = tmem_a + 64 * s;
#pragma unroll
          for (int k = 0; k < kKS / 16; k++)
            umma_f16_ts(dt, at + 8 * k, (k < 4 ? bd0 : bd1) + 2 * (k & 3), idesc, (i | k) != 0);
          umma_commit(&st_empty[s]);
        }
        umma_commit(&acc_full[ab]);   // arrives once every MMA of this unit has completed
      }
      // completes once every MMA issued above has: the exit below never frees tensor memory still being written
      umma_commit(mma_done);
    }
  } else if (warp < kEpiWarp0) {
    // ---- dequant: two threads per weight row, one 32-element half each, into the TMEM stage ring. Software
    // pipelined: stage i's TMEM stores are in flight while stage i+1 is computed, and only then waited for and
    // signalled, so the store latency hides behind arithmetic.
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const int hsel = (warp - 2) >> 2;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    long cr = 0, ca = 0;
    int prev = -1;              // stage slot whose stores are in flight, not yet signalled
    bool ok = true;
    long prev_c = 0;
    auto signal_prev = [&]() {
      if (prev < 0) return;
      tmem_st_wait();
      tc_fence_before();
      // the stage's activation tiles must have landed too: then one barrier tells the MMA thread both are ready
      if (!mbar_wait(&b_full[prev], static_cast<uint32_t>((prev_c / SR) & 1), err, kErrBFull)) ok = false;
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[prev]);
      prev = -1;
    };
    for (int w = blockIdx.x; w < units && ok; w += gridDim.x) {
      const Unit un = unit_of(w, NTW, KT, splits);
      for (int u = 0; u < un.per && ok; u++, cr++) {
        const int rs = static_cast<int>(cr % RS);
        if (!(ok = mbar_wait(&raw_full[rs], static_cast<uint32_t>((cr / RS) & 1), err, kErrRawFull))) break;
        const uint8_t *raw = sRaw + rs * F::BYTES;
        const uint4 hdr = *reinterpret_cast<const uint4 *>(raw + r * 16);
        const Q4kScales qsc = q4k_scales(hdr.y, hdr.z, hdr.w);
        for (int j = 0; j < kSub; j++, ca++) {
          const int s = static_cast<int>(ca % SR);
          // 128 K = two 64-K halves (quarters 2j, 2j+1 of the raw tile) -> 4 runs of 8 TMEM columns
          uint32_t v0[16], v1[16];
          if (TYPE == kQ4_K) {
            dequant_q4k(raw, r, 2 * j, hsel, hdr.x, qsc, v0);
            dequant_q4k(raw, r, 2 * j + 1, hsel, hdr.x, qsc, v1);
          } else {
            dequant_q80(raw, r, 2 * j, hsel, hdr, v0);
            dequant_q80(raw, r, 2 * j + 1, hsel, hdr, v1);
          }
          if (j == kSub - 1) {       // every byte of this raw tile is in registers: release the slot
            __syncwarp();
            if (lane == 0) mbar_arrive(&raw_empty[rs]);
          }
          signal_prev();
          if (!(ok = mbar_wait(&st_empty[s], static_cast<uint32_t>((ca / SR) & 1) ^ 1, err, kErrStageEmpty))) break;
          tc_fence_after();
          const uint32_t col = tmem_a + 64 * s + lane_base;
#pragma unroll
          for (int t = 0; t < 2; t++) {
            const uint32_t *v = t ? v1 : v0;
            const uint32_t c0 = col + 32 * t;
            if (TYPE == kQ4_K) {
              tmem_st8(c0 + 8 * hsel, v);
              tmem_st8(c0 + 16 + 8 * hsel, v + 8);
            } else {
              tmem_st8(c0 + 16 * hsel, v);
              tmem_st8(c0 + 16 * hsel + 8, v + 8);
            }
          }
          prev = s;
          prev_c = ca;
        }
      }
    }
    signal_prev();
  } else {
    // ---- epilogue: TMEM lane quarter q = weight rows 32q .. 32q+31 of the tile
    const int q = warp & 3;
    const int r = q * 32 + lane;
    int lu = 0;
    for (int w = blockIdx.x; w < units; w += gridDim.x, lu++) {
      const Unit un = unit_of(w, NTW, KT, splits);
      const int ab = ACC == 2 ? (lu & 1) : 0;
      const uint32_t ph = ACC == 2 ? static_cast<uint32_t>((lu >> 1) & 1) : static_cast<uint32_t>(lu & 1);
      const bool good = mbar_wait_sleep(&acc_full[ab], ph, err, kErrAcc);
      tc_fence_after();
      const uint32_t tbase = tmem + ab * S::NCOLS + (static_cast<uint32_t>(q * 32) << 16);
      const int row = un.nt * kBM + r, t0 = un.tt * NT;
      if (splits > 1) {
        if (good) {
          float *p = part + static_cast<size_t>(un.split) * T * Npad;
          for (int c0 = 0; c0 < NT; c0 += 16) {
            uint32_t v[16];
            tmem_ld16(tbase + c0, v);
#pragma unroll
            for (int c = 0; c < 16; c++) {
              int t = t0 + c0 + c;
              if (t < T) p[static_cast<size_t>(t) * Npad + row] = __uint_as_float(v[c]);
            }
          }
        }
      } else if (epi.kind == kEpiSwiGLU) {
        // rows 64..127 (up) hand 16 columns at a time to rows 0..63 (gate); all four warps reach every barrier
        const int f = un.nt * 64 + r;
        for (int c0 = 0; c0 < NT; c0 += 16) {
          uint32_t v[16];
          if (good) tmem_ld16(tbase + c0, v);
          if (good && r >= 64) {
#pragma unroll
            for (int c = 0; c < 16; c++) xchg[(r - 64) * 17 + c] = __uint_as_float(v[c]);
          }
          asm volatile("bar.sync 1, 128;\n" ::: "memory");
          if (good && r < 64) {
#pragma unroll
            for (int c = 0; c < 16; c++) {
              int t = t0 + c0 + c;
              if (t < T && f < epi.n) {
                float g = __uint_as_float(v[c]), uu = xchg[r * 17 + c];
                epi.out_h[static_cast<size_t>(t) * epi.ld + f] = __float2half_rn(g / (1.f + expf(-g)) * uu);
              }
            }
          }
          asm volatile("bar.sync 1, 128;\n" ::: "memory");
        }
      } else if (good) {
        for (int c0 = 0; c0 < NT; c0 += 16) {
          uint32_t v[16];
          tmem_ld16(tbase + c0, v);
#pragma unroll
          for (int c = 0; c < 16; c++) {
            int t = t0 + c0 + c;
            if (t < T && row < epi.n) {
              float *o = epi.out_f + static_cast<size_t>(t) * epi.ld + row;
              if (epi.kind == kEpiAdd) *o += __uint_as_float(v[c]);
              else *o = __uint_as_float(v[c]);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[ab]);
      if (!good) break;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    // no MMA may still write the accumulators when they are freed (bounded; returns at once after a normal run)
    if (lane == 0) mbar_wait(mma_done, 0, err, kErrAcc);
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(512));
  }
}

template <int TYPE, int NT>
void launch_nt(const QWeight &w, const CUtensorMap *map, int T, const Epi &epi, float *part, int *err, int sms,
               cudaStream_t s) {
  const int units = w.NT * w.splits * ((T + NT - 1) / NT);
  const int grid = units < sms ? units : sms;
  gemm_tc_kernel<TYPE, NT><<<grid, kThreads, smem_total<TYPE, NT>(), s>>>(w.data, w.NT, w.KT, w.splits, units, *map, T,
                                                                          epi, part, w.NT * kBM, err);
}

template <int TYPE>
void launch_type(const QWeight &w, const TmaSet &ts, int T, const Epi &epi, float *part, int *err, int sms,
                 cudaStream_t s) {
  int nt = tc_token_tile(T);
  const CUtensorMap *m = ts.map(nt);
  switch (nt) {
    case 16: launch_nt<TYPE, 16>(w, m, T, epi, part, err, sms, s); break;
    case 32: launch_nt<TYPE, 32>(w, m, T, epi, part, err, sms, s); break;
    case 64: launch_nt<TYPE, 64>(w, m, T, epi, part, err, sms, s); break;
    case 128: launch_nt<TYPE, 128>(w, m, T, epi, part, err, sms, s); break;
    default: launch_nt<TYPE, 256>(w, m, T, epi, part, err, sms, s); break;
  }
}

template <int TYPE, int NT>
void set_attr() {
  cudaFuncSetAttribute(gemm_tc_kernel<TYPE, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_total<TYPE, NT>());
}

}  // namespace

int tc_token_tile(int T) {
  if (T <= 16) return 16;
  if (T <= 32) return 32;
  if (T <= 64) return 64;
  if (T <= 128) return 128;
  return 256;
}

void gemm_tc_init() {
  set_attr<kQ4_K, 16>(); set_attr<kQ4_K, 32>(); set_attr<kQ4_K, 64>(); set_attr<kQ4_K, 128>(); set_attr<kQ4_K, 256>();
  set_attr<kQ8_0, 16>(); set_attr<kQ8_0, 32>(); set_attr<kQ8_0, 64>(); set_attr<kQ8_0, 128>(); set_attr<kQ8_0, 256>();
}

size_t tc_tile_bytes(int type) { return type == kQ4_K ? TileFmt<kQ4_K>::BYTES : TileFmt<kQ8_0>::BYTES; }

void launch_gemm_tc(const QWeight &w, const TmaSet &ts, int T, const Epi &epi, float *part, int *err, int sms,
                    cudaStream_t s) {
  if (T <= 0) return;
  if (w.type == kQ4_K) launch_type<kQ4_K>(w, ts, T, epi, part, err, sms, s);
  else launch_type<kQ8_0>(w, ts, T, epi, part, err, sms, s);
  if (w.splits > 1) launch_splitk_reduce(part, w.splits, T, w.NT * kBM, epi, s);
}

}  // namespace gck
