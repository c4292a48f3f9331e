// Quantized weight GEMM on the 5th-generation tensor cores: tcgen05.mma (kind::f16, f16 x f16 -> f32) with the
// accumulator in tensor memory.
//
//   y[t, n] = sum_k act[t, k] * W[n, k]          (the reference's `w @ h`, ref.py:51-59, for all token rows at once)
//
// One CTA computes a 128-row band of W (the MMA's M) against a tile of NT token rows (the MMA's N) over a fixed range
// of K (split-K, fixed per weight). Warp roles:
//   warp 0       producer: one 1-D bulk copy per raw weight tile (128 rows x 256 K, the GGUF blocks as relaid at load)
//                and one 2-D tensor-map copy per K stage of activations (NT rows x 64 K, 128-byte swizzle);
//   warp 1       TMEM allocation; one elected thread issues 4 tcgen05.mma (K = 16 each) per 64-K stage and commits
//                each stage back to the producers;
//   warps 2-5    dequantize each stage of the raw tile (one weight row per thread; f16 arithmetic with one rounding)
//                into the UMMA K-major 128-byte-swizzled layout, then read the accumulator with tcgen05.ld and apply
//                the epilogue (store, residual add, SwiGLU, or the split-K partial).
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

constexpr int kStages = 3;                 // A/B stage ring
constexpr int kRawSlots = 2;               // raw weight tile ring
constexpr int kKS = 64;                    // K per stage: one 128-byte swizzle row of f16
constexpr int kSub = kBK / kKS;            // stages per raw tile (4)
constexpr int kThreads = 192;
constexpr int kStageA = kBM * 128;         // 16 KB
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
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
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
// bounded wait for the phase of the given parity; false (and the error word set) on timeout
GCK_DEV bool mbar_wait(uint64_t *b, uint32_t parity, int *err, int code) {
  if (mbar_try(b, parity)) return true;
  unsigned long long t0 = now_ns();
  while (true) {
    if (mbar_try(b, parity)) return true;
    if (now_ns() - t0 > kTimeoutNs) {
      atomicCAS(err, 0, code);
      return false;
    }
    if (*reinterpret_cast<volatile int *>(err)) return false;   // another CTA already failed: give up early
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

// Q4_K: stage j of row r -> 64 f16 into the swizzled A row
GCK_DEV void dequant_q4k(const uint8_t *raw, int r, int j, uint32_t d_dm, const Q4kScales &qs, uint8_t *arow, int sw) {
  // sub-blocks 2j (low nibbles) and 2j+1 (high nibbles) of quant bytes 32j .. 32j+31
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
#pragma unroll
  for (int p = 0; p < 2; p++) {
    uint4 q = *reinterpret_cast<const uint4 *>(raw + kBM * 16 + (j * 2 + p) * (kBM * 16) + r * 16);
    uint32_t w[4] = {q.x, q.y, q.z, q.w};
    uint32_t lo[8], hi[8];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      uint32_t l4 = w[i] & 0x0F0F0F0Fu, h4 = (w[i] >> 4) & 0x0F0F0F0Fu;
      uint32_t a0, a1, b0, b1;
      bytes_to_h2(l4, a0, a1);
      bytes_to_h2(h4, b0, b1);
      lo[2 * i] = hfma2_u(hsub2_u(a0, K1024), S0, O0);
      lo[2 * i + 1] = hfma2_u(hsub2_u(a1, K1024), S0, O0);
      hi[2 * i] = hfma2_u(hsub2_u(b0, K1024), S1, O1);
      hi[2 * i + 1] = hfma2_u(hsub2_u(b1, K1024), S1, O1);
    }
    // piece p holds bytes 16p .. 16p+15: k = 16p .. 16p+15 (low) and 32 + 16p .. (high): chunks 2p, 2p+1, 4+2p, 5+2p
    int c0 = 2 * p, c1 = 4 + 2 * p;
    *reinterpret_cast<uint4 *>(arow + (((c0) ^ sw) << 4)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    *reinterpret_cast<uint4 *>(arow + (((c0 + 1) ^ sw) << 4)) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
    *reinterpret_cast<uint4 *>(arow + (((c1) ^ sw) << 4)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4 *>(arow + (((c1 + 1) ^ sw) << 4)) = make_uint4(hi[4], hi[5], hi[6], hi[7]);
  }
}

// Q8_0: stage j of row r (blocks 2j, 2j+1) -> 64 f16
GCK_DEV void dequant_q80(const uint8_t *raw, int r, int j, const uint4 &hdr, uint8_t *arow, int sw) {
  const uint32_t K1152 = 0x64806480u;   // 1024 + 128
  // the row's 8 block scales: d[2j] and d[2j+1] are the two halves of header word j
  const uint32_t dw = j == 0 ? hdr.x : j == 1 ? hdr.y : j == 2 ? hdr.z : hdr.w;
  const uint32_t D0 = (dw & 0xFFFFu) * 0x10001u, D1 = (dw >> 16) * 0x10001u;
#pragma unroll
  for (int p = 0; p < 4; p++) {
    uint4 q = *reinterpret_cast<const uint4 *>(raw + kBM * 16 + (j * 4 + p) * (kBM * 16) + r * 16);
    uint32_t w[4] = {q.x, q.y, q.z, q.w};
    uint32_t o[8];
    const uint32_t D = p < 2 ? D0 : D1;
#pragma unroll
    for (int i = 0; i < 4; i++) {
      uint32_t a0, a1;
      bytes_to_h2(w[i] ^ 0x80808080u, a0, a1);
      o[2 * i] = hmul2_u(hsub2_u(a0, K1152), D);
      o[2 * i + 1] = hmul2_u(hsub2_u(a1, K1152), D);
    }
    *reinterpret_cast<uint4 *>(arow + (((2 * p) ^ sw) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<uint4 *>(arow + (((2 * p + 1) ^ sw) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

template <int NT>
struct Shape {
  static constexpr int STAGE_B = NT * 128;
  static constexpr int NCOLS = NT <= 32 ? 32 : NT <= 64 ? 64 : NT <= 128 ? 128 : 256;
};

template <int TYPE, int NT>
constexpr int smem_total() {
  return 1024 + kStages * kStageA + kStages * Shape<NT>::STAGE_B + kRawSlots * TileFmt<TYPE>::BYTES + 256;
}

template <int TYPE, int NT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const uint8_t *__restrict__ W, int KT, int splits, const __grid_constant__ CUtensorMap tmap, int T,
                   Epi epi, float *part, int Npad, int *err) {
  using F = TileFmt<TYPE>;
  using S = Shape<NT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sA = smem;
  uint8_t *sB = sA + kStages * kStageA;
  uint8_t *sRaw = sB + kStages * S::STAGE_B;
  uint64_t *bars = reinterpret_cast<uint64_t *>(sRaw + kRawSlots * F::BYTES);
  uint64_t *raw_full = bars, *raw_empty = bars + kRawSlots, *a_full = bars + 2 * kRawSlots;
  uint64_t *b_full = a_full + kStages, *st_empty = b_full + kStages, *acc_full = st_empty + kStages;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_full + 1);

  const int nt = blockIdx.x, split = blockIdx.y, t0 = blockIdx.z * NT;
  const int per = KT / splits, kt0 = split * per, nstage = per * kSub;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kRawSlots; i++) { mbar_init(&raw_full[i], 1); mbar_init(&raw_empty[i], 4); }
    for (int i = 0; i < kStages; i++) { mbar_init(&a_full[i], 4); mbar_init(&b_full[i], 1); mbar_init(&st_empty[i], 1); }
    mbar_init(acc_full, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    fence_async_smem();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                 "r"(S::NCOLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---- producer
      int issued_raw = 0, issued_b = 0;
      bool ok = true;
      for (int u = 0; u < per && ok; u++) {
        int rs = u % kRawSlots;
        ok = mbar_wait(&raw_empty[rs], ((u / kRawSlots) & 1) ^ 1, err, kErrRawEmpty);
        if (!ok) break;
        mbar_expect_tx(&raw_full[rs], F::BYTES);
        bulk_g2s(sRaw + rs * F::BYTES, W + (static_cast<size_t>(nt) * KT + kt0 + u) * F::BYTES, F::BYTES, &raw_full[rs]);
        issued_raw++;
        for (int j = 0; j < kSub; j++) {
          int i = u * kSub + j, s = i % kStages;
          ok = mbar_wait(&st_empty[s], ((i / kStages) & 1) ^ 1, err, kErrStageEmpty);
          if (!ok) break;
          mbar_expect_tx(&b_full[s], S::STAGE_B);
          tma_2d(sB + s * S::STAGE_B, &tmap, (kt0 + u) * kBK + j * kKS, t0, &b_full[s]);
          issued_b++;
        }
      }
      // drain: every copy issued has landed before the CTA may exit (bounded)
      for (int u = 0; u < issued_raw; u++) {
        if (u + kRawSlots < issued_raw) continue;
        mbar_wait(&raw_full[u % kRawSlots], (u / kRawSlots) & 1, err, kErrRawFull);
      }
      for (int i = (issued_b > kStages ? issued_b - kStages : 0); i < issued_b; i++)
        mbar_wait(&b_full[i % kStages], (i / kStages) & 1, err, kErrBFull);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer
      const uint32_t idesc = (1u << 4) | (static_cast<uint32_t>(NT >> 3) << 17) | (static_cast<uint32_t>(kBM >> 4) << 24);
      for (int i = 0; i < nstage; i++) {
        int s = i % kStages;
        uint32_t ph = (i / kStages) & 1;
        if (!mbar_wait(&a_full[s], ph, err, kErrAFull)) break;
        if (!mbar_wait(&b_full[s], ph, err, kErrBFull)) break;
        tc_fence_after();
        uint64_t ad = umma_desc(sA + s * kStageA), bd = umma_desc(sB + s * S::STAGE_B);
#pragma unroll
        for (int k = 0; k < kKS / 16; k++) umma_f16(tmem, ad + 2 * k, bd + 2 * k, idesc, (i | k) != 0);
        umma_commit(&st_empty[s]);
      }
      umma_commit(acc_full);   // arrives once every MMA issued above has completed
    }
  } else {
    // ---- dequant (one weight row per thread) then epilogue
    const int q = warp & 3;                 // TMEM lane quarter of this warp
    const int r = q * 32 + lane;            // weight row in the tile = accumulator lane
    const int sw = r & 7;
    bool ok = true;
    for (int u = 0; u < per && ok; u++) {
      int rs = u % kRawSlots;
      ok = mbar_wait(&raw_full[rs], (u / kRawSlots) & 1, err, kErrRawFull);
      if (!ok) break;
      const uint8_t *raw = sRaw + rs * F::BYTES;
      const uint4 hdr = *reinterpret_cast<const uint4 *>(raw + r * 16);
      const Q4kScales qsc = q4k_scales(hdr.y, hdr.z, hdr.w);
      for (int j = 0; j < kSub; j++) {
        int i = u * kSub + j, s = i % kStages;
        ok = mbar_wait(&st_empty[s], ((i / kStages) & 1) ^ 1, err, kErrStageEmpty);
        if (!ok) break;
        uint8_t *arow = sA + s * kStageA + r * 128;
        if (TYPE == kQ4_K) dequant_q4k(raw, r, j, hdr.x, qsc, arow, sw);
        else dequant_q80(raw, r, j, hdr, arow, sw);
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[s]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&raw_empty[rs]);
    }
    // epilogue: the accumulator's lane r = weight row nt*128 + r, column c = token t0 + c
    bool done = mbar_wait(acc_full, 0, err, kErrAcc);
    tc_fence_after();
    const bool good = done && ok;
    const int row = nt * kBM + r;
    const uint32_t tbase = tmem + (static_cast<uint32_t>(q * 32) << 16);
    if (splits > 1) {
      if (good) {
        float *p = part + static_cast<size_t>(split) * T * Npad;
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
      // rows 64..127 (up) hand their values to rows 0..63 (gate) through shared memory (the finished stage ring);
      // all four warps reach the named barrier whatever happened before it
      float *xu = reinterpret_cast<float *>(sA);      // [64][NT + 1]
      if (good && r >= 64) {
        for (int c0 = 0; c0 < NT; c0 += 16) {
          uint32_t v[16];
          tmem_ld16(tbase + c0, v);
#pragma unroll
          for (int c = 0; c < 16; c++) xu[(r - 64) * (NT + 1) + c0 + c] = __uint_as_float(v[c]);
        }
      }
      asm volatile("bar.sync 1, 128;\n" ::: "memory");
      if (good && r < 64) {
        const int f = nt * 64 + r;
        for (int c0 = 0; c0 < NT; c0 += 16) {
          uint32_t v[16];
          tmem_ld16(tbase + c0, v);
#pragma unroll
          for (int c = 0; c < 16; c++) {
            int t = t0 + c0 + c;
            if (t < T && f < epi.n) {
              float g = __uint_as_float(v[c]), uu = xu[r * (NT + 1) + c0 + c];
              epi.out_h[static_cast<size_t>(t) * epi.ld + f] = __float2half_rn(g / (1.f + expf(-g)) * uu);
            }
          }
        }
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
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    // no MMA may still write the accumulator when it is freed (bounded; returns at once after a normal run)
    if (lane == 0) mbar_wait(acc_full, 0, err, kErrAcc);
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(S::NCOLS));
  }
}

template <int TYPE, int NT>
void launch_nt(const QWeight &w, const CUtensorMap *maps, const __half *, int T, const Epi &epi, float *part, int *err,
               cudaStream_t s) {
  (void)maps;
  dim3 grid(w.NT, w.splits, (T + NT - 1) / NT);
  gemm_tc_kernel<TYPE, NT><<<grid, kThreads, smem_total<TYPE, NT>(), s>>>(w.data, w.KT, w.splits, *maps, T, epi, part,
                                                                          w.NT * kBM, err);
}

template <int TYPE>
void launch_type(const QWeight &w, const TmaSet &ts, const __half *act, int T, const Epi &epi, float *part, int *err,
                 cudaStream_t s) {
  int nt = tc_token_tile(T);
  const CUtensorMap *m = ts.map(nt);
  switch (nt) {
    case 16: launch_nt<TYPE, 16>(w, m, act, T, epi, part, err, s); break;
    case 32: launch_nt<TYPE, 32>(w, m, act, T, epi, part, err, s); break;
    case 64: launch_nt<TYPE, 64>(w, m, act, T, epi, part, err, s); break;
    case 128: launch_nt<TYPE, 128>(w, m, act, T, epi, part, err, s); break;
    default: launch_nt<TYPE, 256>(w, m, act, T, epi, part, err, s); break;
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

void launch_gemm_tc(const QWeight &w, const TmaSet &ts, const __half *act, int T, const Epi &epi, float *part,
                    int *err, cudaStream_t s) {
  if (T <= 0) return;
  if (w.type == kQ4_K) launch_type<kQ4_K>(w, ts, act, T, epi, part, err, s);
  else launch_type<kQ8_0>(w, ts, act, T, epi, part, err, s);
  if (w.splits > 1) launch_splitk_reduce(part, w.splits, T, w.NT * kBM, epi, s);
}

}  // namespace gck
