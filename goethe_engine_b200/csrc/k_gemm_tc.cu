// Quantized weight GEMM on the 5th-generation tensor cores: tcgen05.mma (kind::f16, f16 x f16 -> f32) with both
// operands in shared memory and the accumulator in tensor memory.
//
//   y[t, n] = sum_k act[t, k] * W[n, k]          (the reference's `w @ h`, ref.py:51-59, for all token rows at once)
//
// A persistent CTA per SM walks work units: a 128-row band of W (the MMA's M) against a tile of NT token rows (the
// MMA's N) over a fixed range of K (split-K, fixed per weight). Each 128 x 256 weight tile (the GGUF blocks as relaid
// at load) is two stages of 128 K. Warp roles:
//   warp 0       producer of activations: 64-K x NT-row tensor-map copies (128-byte swizzle), up to R stages ahead;
//   warp 1       TMEM allocation; one elected thread issues the stage's 8 tcgen05.mma (K = 16 each, A = the stage's
//                dequantized weights, B = its activations, both from shared memory) and one commit per stage;
//   warps 2-5    epilogue: tcgen05.ld of the accumulator (two buffers, so it overlaps the next unit's MMAs) and the
//                store, residual add, SwiGLU or split-K partial;
//   warps 6-21   dequantize, in two groups of 8 warps: group g takes the g-th 128-K half of every tile, so one group's
//                waits overlap the other's arithmetic. A thread owns one weight row and one 64-K swizzle atom of the
//                stage: it loads its row's raw bytes straight from global memory (a stage ahead, into registers),
//                makes exact f16 weights (one rounding) and stores them into the stage's A operand in the 128-byte
//                swizzled K-major layout the MMA reads (conflict-free: 32 rows, eight distinct 16-byte slots per
//                eight rows).
// Why shared memory and not tensor memory for the weights: measured on this part, 16 warps storing into TMEM
// (tcgen05.st) slow a concurrent M128 x N64 x K16 MMA from about 62-69 to 137-143 cycles, whether its A operand is in
// TMEM or in shared memory (the accumulator is in TMEM), while the same warps storing into shared memory leave it at
// 63-71 cycles.
// Every output element accumulates its K range in one order whatever NT is, so a row's result does not depend on the
// rest of the batch. Every copy here reads this GPU's own global memory into this CTA's own shared memory.
//
// Every mbarrier wait is bounded (about 2 s on the global timer); a timeout writes a code to the error word, the CTA
// drains what it issued (again bounded), frees its tensor memory and returns; gc_step reports GC_E_DEVICE.
#include <cuda.h>

#include "common.cuh"
#include "dequant.cuh"
#include "kernels.h"

namespace gck {
namespace {

constexpr int kThreads = 704;              // 22 warps
constexpr int kEpiWarp0 = 2;               // warps 2-5: epilogue (TMEM lane quarters 2, 3, 0, 1)
constexpr int kDeqWarp0 = 6;               // warps 6-21: dequant, two groups
constexpr int kGroupWarps = 8;             // per group: two threads per weight row (one per 64-K atom of a stage)
constexpr int kKS = 128;                   // K of a stage: two stages per 256-K weight tile, one per dequant group
constexpr int kAStage = kBM * kKS * 2;     // a stage's A operand: 128 rows x 128 K f16 (two 16 KB swizzle atoms)
constexpr unsigned long long kTimeoutNs = 2000000000ull;

enum ErrCode { kErrStageEmpty = 3, kErrAFull, kErrBFull, kErrAcc };

template <int TYPE>
struct TileFmt;
template <>
struct TileFmt<kQ4_K> {
  static constexpr int BYTES = kBM * 144;   // 128 x 16 B headers, then [8 sub-blocks][128 rows][16 B]
};
template <>
struct TileFmt<kQ8_0> {
  static constexpr int BYTES = kBM * 272;   // 128 x 16 B (8 fp16 d), then [8 blocks][2 halves][128 rows][16 B]
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

GCK_DEV void umma_f16_ss(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Stage geometry: a stage is 128 K, its A operand (kAStage) and KS / 64 activation boxes of NT rows x 64 K, both in
// the 128-byte swizzle; R stages in flight (the shared memory left for them, at most 4, even). Two accumulator buffers
// of NCOLS TMEM columns.
template <int TYPE, int NT>
struct Shape {
  static constexpr int BOX_B = NT * 128;                // one 64-K activation box
  static constexpr int STAGE_B = (kKS / 64) * BOX_B;
  static constexpr int STAGE = kAStage + STAGE_B;
  static constexpr int NCOLS = NT <= 32 ? 32 : NT <= 64 ? 64 : NT <= 128 ? 128 : 256;
  static constexpr int R0 = (200 * 1024) / STAGE;
  static constexpr int R = R0 >= 4 ? 4 : R0 >= 2 ? 2 : R0;
  static_assert(R >= 2, "stage ring too shallow");
  // the two dequant groups take alternate stages (the two halves of every tile): an even ring gives every slot one
  // group, which waits on it in order, so a parity wait never passes on a phase two behind
  static_assert(R % 2 == 0, "stage slots must each belong to one dequant group");
};

template <int TYPE, int NT>
constexpr int smem_total() {
  using S = Shape<TYPE, NT>;
  return 1024 + S::R * S::STAGE + 512;
}

// The raw bytes one dequant thread turns into one 64-K atom of a stage (its row's header and quant pieces in the
// relaid tile formats above), loaded from global memory a stage ahead.
template <int TYPE>
struct RawRow;
template <>
struct RawRow<kQ4_K> {
  static constexpr int NP = 2;                          // two 32-K sub-blocks
  uint4 hdr, p[NP];
};
template <>
struct RawRow<kQ8_0> {
  static constexpr int NP = 4;                          // two 32-K blocks, two 16-quant halves each
  uint4 hdr, p[NP];
};

GCK_DEV uint4 ldg_stream(const uint8_t *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
GCK_DEV void sts128(uint32_t addr, const uint32_t *v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};\n" ::"r"(addr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3])
               : "memory");
}

// Row r's raw bytes for atom `atom` (0..3: 64-K quarter of the 256-K tile) of the tile at `tile`.
template <int TYPE>
GCK_DEV void load_raw(RawRow<TYPE> &x, const uint8_t *tile, int r, int atom) {
  x.hdr = ldg_stream(tile + r * 16);
#pragma unroll
  for (int i = 0; i < RawRow<TYPE>::NP; i++) {
    // Q4_K: sub-block 2 * atom + i at [g][row]; Q8_0: piece 2 * (2 * atom + i / 2) + i % 2 = 4 * atom + i at [piece][row]
    const int piece = TYPE == kQ4_K ? 2 * atom + i : 4 * atom + i;
    x.p[i] = ldg_stream(tile + kBM * 16 + (piece * kBM + r) * 16);
  }
}

// Row r's f16 weights of one 64-K atom into the stage's A operand: eight 16-byte chunks (8 consecutive K each), chunk j
// of row r at row offset 128 * (r % 8) + 16 * (j ^ (r % 8)) in its 8-row group (the 128-byte swizzle).
template <int TYPE>
GCK_DEV void dequant_atom(const RawRow<TYPE> &x, int atom, uint32_t row_addr, int r) {
  const uint32_t sw = static_cast<uint32_t>(r & 7);
  if (TYPE == kQ4_K) {
    const uint32_t dd = prmt(x.hdr.x, 0, 0x1010u);                 // (d, d)
    const uint32_t mm = prmt(x.hdr.x, 0, 0x3232u) ^ 0x80008000u;   // (-dmin, -dmin)
    uint32_t S01, O01;
    q4k_pair_scales(x.hdr, 2 * atom, dd, mm, S01, O01);
#pragma unroll
    for (int e = 0; e < 2; e++) {
      const uint32_t Sg = prmt(S01, 0, e ? 0x3232u : 0x1010u), Og = prmt(O01, 0, e ? 0x3232u : 0x1010u);
      uint32_t v[16];
      q4_word(x.p[e].x, Sg, Og, v);
      q4_word(x.p[e].y, Sg, Og, v + 4);
      q4_word(x.p[e].z, Sg, Og, v + 8);
      q4_word(x.p[e].w, Sg, Og, v + 12);
#pragma unroll
      for (int c = 0; c < 4; c++) sts128(row_addr + 16u * ((static_cast<uint32_t>(4 * e + c)) ^ sw), v + 4 * c);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 2; e++) {
      const int g = 2 * atom + e;                                    // 32-K block of the tile
      const uint32_t dw2 = (g >> 1) == 0 ? x.hdr.x : (g >> 1) == 1 ? x.hdr.y : (g >> 1) == 2 ? x.hdr.z : x.hdr.w;
      const uint32_t D = prmt(dw2, 0, (g & 1) ? 0x3232u : 0x1010u);
      const uint4 q0 = x.p[2 * e], q1 = x.p[2 * e + 1];
      uint32_t v[16];
      q8_word(q0.x, D, v); q8_word(q0.y, D, v + 2); q8_word(q0.z, D, v + 4); q8_word(q0.w, D, v + 6);
      q8_word(q1.x, D, v + 8); q8_word(q1.y, D, v + 10); q8_word(q1.z, D, v + 12); q8_word(q1.w, D, v + 14);
#pragma unroll
      for (int c = 0; c < 4; c++) sts128(row_addr + 16u * ((static_cast<uint32_t>(4 * e + c)) ^ sw), v + 4 * c);
    }
  }
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
                   const __grid_constant__ CUtensorMap tmap, int T, Epi epi, float *part, int Npad, int *err, Signal sig) {
  using F = TileFmt<TYPE>;
  using S = Shape<TYPE, NT>;
  constexpr int SR = S::R;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned (the 128-byte swizzle atom) by an offset into the __shared__ array, so that every pointer derived
  // from it stays a shared-memory pointer to the compiler (shared loads, not generic ones)
  uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t *sA = smem;                              // [SR][kAStage]
  uint8_t *sB = sA + SR * kAStage;                 // [SR][STAGE_B]
  uint64_t *bars = reinterpret_cast<uint64_t *>(sB + SR * S::STAGE_B);
  uint64_t *a_full = bars, *st_empty = a_full + SR, *b_full = st_empty + SR;
  uint64_t *acc_full = b_full + SR, *acc_empty = acc_full + 2, *mma_done = acc_empty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // the next kernel may start as this one's CTAs run; the weight stream depends on no earlier kernel, so only the
  // activation producer and the epilogue wait for the previous kernels (dep_wait)
  dep_launch();

  if (threadIdx.x == 0) {
    for (int i = 0; i < SR; i++) { mbar_init(&a_full[i], kGroupWarps); mbar_init(&st_empty[i], 1); mbar_init(&b_full[i], 1); }
    for (int i = 0; i < 2; i++) { mbar_init(&acc_full[i], 1); mbar_init(&acc_empty[i], 4); }
    mbar_init(mma_done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    fence_async_smem();
  }
  if (warp == 1) {   // the two accumulator buffers
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                 "r"(2 * S::NCOLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---- activation stages: two tensor-map copies (64 K each) per stage, up to SR stages ahead
      dep_wait();
      long c = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < units && ok; w += gridDim.x) {
        const Unit un = unit_of(w, NTW, KT, splits);
        for (int i = 0; i < un.per * 2; i++, c++) {
          const int s = static_cast<int>(c % SR);
          if (!(ok = mbar_wait(&st_empty[s], static_cast<uint32_t>((c / SR) & 1) ^ 1, err, kErrStageEmpty))) break;
          mbar_expect_tx(&b_full[s], S::STAGE_B);
          const int x = (un.kt0 + i / 2) * kBK + (i % 2) * kKS;
#pragma unroll
          for (int b = 0; b < kKS / 64; b++) tma_2d(sB + s * S::STAGE_B + b * S::BOX_B, &tmap, x + 64 * b, un.tt * NT, &b_full[s]);
        }
      }
      for (long i = c > SR ? c - SR : 0; i < c; i++) mbar_wait(&b_full[i % SR], static_cast<uint32_t>((i / SR) & 1), err, kErrBFull);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer: accumulator buffer (local unit index) % 2; per stage 8 MMAs of K 16, both operands in shared
      // memory (A: the stage's weights, two 16 KB atoms; B: its two activation boxes)
      const uint32_t idesc = (1u << 4) | (static_cast<uint32_t>(NT >> 3) << 17) | (static_cast<uint32_t>(kBM >> 4) << 24);
      int s = 0;                 // stage slot and the parity of its current use
      uint32_t par = 0;
      int lu = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < units && ok; w += gridDim.x, lu++) {
        const Unit un = unit_of(w, NTW, KT, splits);
        const int ab = lu & 1;
        const uint32_t ph = static_cast<uint32_t>((lu >> 1) & 1);
        if (!(ok = mbar_wait(&acc_empty[ab], ph ^ 1, err, kErrAcc))) break;
        tc_fence_after();
        const uint32_t dt = tmem + ab * S::NCOLS;
        for (int i = 0; i < un.per * 2; i++) {
          // a_full covers both operands: the dequant group signals it only after the stage's activations landed
          if (!(ok = mbar_wait(&a_full[s], par, err, kErrAFull))) break;
          tc_fence_after();
          const uint64_t ad = umma_desc(sA + s * kAStage), bd = umma_desc(sB + s * S::STAGE_B);
#pragma unroll
          for (int k = 0; k < kKS / 16; k++)
            umma_f16_ss(dt, ad + static_cast<uint64_t>((k >> 2) * ((kBM * 128) >> 4) + 2 * (k & 3)),
                        bd + static_cast<uint64_t>((k >> 2) * (S::BOX_B >> 4) + 2 * (k & 3)), idesc, (i | k) != 0);
          umma_commit(&st_empty[s]);
          if (++s == SR) {
            s = 0;
            par ^= 1u;
          }
        }
        umma_commit(&acc_full[ab]);   // arrives once every MMA of this unit has completed
      }
      // completes once every MMA issued above has: the exit below never frees tensor memory still being written
      umma_commit(mma_done);
    }
  } else if (warp >= kDeqWarp0) {
    // ---- dequant: group grp takes the grp-th 128-K half of every tile (global stage c = 2 * tile + grp); in the group
    // thread (row r, atom half hsel) writes 64 K of row r: atom 2 * grp + hsel of the tile, atom hsel of the stage
    const int dw = warp - kDeqWarp0;
    const int grp = dw / kGroupWarps;
    const int hsel = (dw / 4) & 1;
    const int r = (warp & 3) * 32 + lane;
    const int atom = 2 * grp + hsel;
    const uint32_t row_off = static_cast<uint32_t>(hsel * (kBM * 128) + (r >> 3) * 1024 + (r & 7) * 128);
    const uint32_t sA0 = smem_u32(sA);
    // the tile sequence of this CTA, one step ahead: (w, u) = unit and tile within it
    int w = blockIdx.x, u = 0;
    Unit un = unit_of(w < units ? w : 0, NTW, KT, splits);
    auto tile_ptr = [&](const Unit &x, int uu) {
      return W + (static_cast<size_t>(x.nt) * KT + x.kt0 + uu) * F::BYTES;
    };
    RawRow<TYPE> cur, nxt;
    bool have = w < units;
    if (have) load_raw<TYPE>(cur, tile_ptr(un, 0), r, atom);
    long t = 0;                                  // tiles done: global stage 2 * t + grp
    bool ok = true;
    while (have && ok) {
      // the next tile of the sequence, its raw bytes loaded now (they land while this tile is dequantized)
      int w2 = w, u2 = u + 1;
      Unit un2 = un;
      if (u2 == un.per) {
        w2 += gridDim.x;
        u2 = 0;
        if (w2 < units) un2 = unit_of(w2, NTW, KT, splits);
      }
      const bool have2 = w2 < units;
      if (have2) load_raw<TYPE>(nxt, tile_ptr(un2, u2), r, atom);
      const long c = 2 * t + grp;
      const int s = static_cast<int>(c % SR);
      // every lane waits; the warp leaves together if any lane's wait ran out (the arrive below is per warp)
      ok = mbar_wait(&st_empty[s], static_cast<uint32_t>((c / SR) & 1) ^ 1, err, kErrStageEmpty);
      if (!(ok = __all_sync(0xffffffffu, ok))) break;
      dequant_atom<TYPE>(cur, atom, sA0 + static_cast<uint32_t>(s * kAStage) + row_off, r);
      // the generic-proxy stores become visible to the tensor core's (async-proxy) reads
      fence_async_smem();
      // the stage's activation tiles must have landed too: then a_full alone tells the MMA thread both are ready
      ok = mbar_wait(&b_full[s], static_cast<uint32_t>((c / SR) & 1), err, kErrBFull);
      if (!(ok = __all_sync(0xffffffffu, ok))) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[s]);
      cur = nxt;
      w = w2;
      u = u2;
      un = un2;
      have = have2;
      t++;
    }
  } else if (warp >= kEpiWarp0) {
    // ---- epilogue: TMEM lane quarter q = weight rows 32q .. 32q+31 of the tile
    dep_wait();
    const int q = warp & 3;
    const int r = q * 32 + lane;
    int lu = 0;
    for (int w = blockIdx.x; w < units; w += gridDim.x, lu++) {
      const Unit un = unit_of(w, NTW, KT, splits);
      const int ab = lu & 1;
      const uint32_t ph = static_cast<uint32_t>((lu >> 1) & 1);
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
              if (t < T) p[static_cast<size_t>(t) * Npad + row] = __uint_as_float(v[c]) * epi_scale(epi, t);
            }
          }
        }
      } else if (epi.kind == kEpiSwiGLU) {
        // even rows are gate rows, the odd row after each its up row (feature un.nt * 64 + r / 2): the two lanes swap
        // values and each takes half the token columns (the gate lane the even ones)
        const int f = un.nt * 64 + (r >> 1);
        const int odd = r & 1;
        for (int c0 = 0; c0 < NT; c0 += 16) {
          uint32_t v[16];
          if (good) tmem_ld16(tbase + c0, v);
#pragma unroll
          for (int c = 0; c < 16; c++) {
            const int t = t0 + c0 + c;
            const float mine = __uint_as_float(v[c]) * (epi.scale && t < T ? epi.scale[t] : 1.f);
            const float other = __shfl_xor_sync(0xffffffffu, mine, 1);
            if (good && (c & 1) == odd && t < T && f < epi.n) {
              const float g = odd ? other : mine, uu = odd ? mine : other;
              epi.out_h[static_cast<size_t>(t) * epi.ld + f] = __float2half_rn(silu_mul(g, uu));
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
              const float y = __uint_as_float(v[c]) * epi_scale(epi, t);
              if (epi.kind == kEpiAdd) *o += y;
              else *o = y;
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
  // with a signal: every thread's stores are made visible system-wide; the last CTA to get here publishes the flag
  if (sig.flag) __threadfence_system();
  tc_fence_before();
  __syncthreads();
  if (sig.flag && threadIdx.x == 0) signal_if_last(sig);
  if (warp == 1) {
    // no MMA may still write the accumulators when they are freed (bounded; returns at once after a normal run)
    if (lane == 0) mbar_wait(mma_done, 0, err, kErrAcc);
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(2 * S::NCOLS));
  }
}

template <int TYPE, int NT>
void launch_nt(const QWeight &w, const CUtensorMap *map, int T, const Epi &epi, float *part, int *err, int sms,
               const Signal &sig, cudaStream_t s) {
  const int units = w.NT * w.splits * ((T + NT - 1) / NT);
  const int grid = units < sms ? units : sms;
  launch_pdl(gemm_tc_kernel<TYPE, NT>, grid, kThreads, smem_total<TYPE, NT>(), s, w.data, w.NT, w.KT, w.splits, units,
             *map, T, epi, part, w.NT * kBM, err, sig);
}

template <int TYPE>
void launch_type(const QWeight &w, const TmaSet &ts, int T, const Epi &epi, float *part, int *err, int sms,
                 const Signal &sig, cudaStream_t s) {
  int nt = tc_token_tile(T);
  const CUtensorMap *m = ts.map(nt);
  switch (nt) {
    case 16: launch_nt<TYPE, 16>(w, m, T, epi, part, err, sms, sig, s); break;
    case 32: launch_nt<TYPE, 32>(w, m, T, epi, part, err, sms, sig, s); break;
    case 64: launch_nt<TYPE, 64>(w, m, T, epi, part, err, sms, sig, s); break;
    case 128: launch_nt<TYPE, 128>(w, m, T, epi, part, err, sms, sig, s); break;
    default: launch_nt<TYPE, 256>(w, m, T, epi, part, err, sms, sig, s); break;
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
                    cudaStream_t s, const Signal &sig) {
  if (T <= 0) return;
  if (w.type == kQ4_K) launch_type<kQ4_K>(w, ts, T, epi, part, err, sms, sig, s);
  else launch_type<kQ8_0>(w, ts, T, epi, part, err, sms, sig, s);
}

}  // namespace gck
