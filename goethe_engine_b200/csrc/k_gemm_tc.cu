// Quantized weight GEMM on the 5th-generation tensor cores: tcgen05.mma (kind::f16, f16 x f16 -> f32) with the
// accumulator in tensor memory.
//
//   y[t, n] = sum_k act[t, k] * W[n, k]          (the reference's `w @ h`, ref.py:51-59, for all token rows at once)
//
// A persistent CTA per SM (it takes all 512 TMEM columns) walks work units: a 128-row band of W (the MMA's M) against
// a tile of NT token rows (the MMA's N) over a fixed range of K (split-K, fixed per weight). Warp roles:
//   warp 0       producer of raw weight tiles: one 1-D bulk copy per tile (128 rows x 256 K, the GGUF blocks as relaid
//                at load), 2-4 tiles ahead, across unit boundaries;
//   warp 2       producer of activations: 64-K x NT-row tensor-map copies (128-byte swizzle), a stage ahead;
//   warp 1       TMEM allocation; one elected thread issues the stage's tcgen05.mma (K = 16 each, weights from TMEM,
//                activations from shared memory) and one commit per stage back to the producers;
//   warps 7-22   dequantize into tensor memory (tcgen05.st), in two groups of 8 warps that take alternate stages, so
//                one group's barrier waits overlap the other's arithmetic (two threads per weight row in a group; f16
//                arithmetic, one rounding): the MMA reads its weight operand from TMEM, so shared memory carries only
//                the raw tiles and the activations;
//   warps 3-6    epilogue: tcgen05.ld of the accumulator (two buffers, so it overlaps the next unit's MMAs) and the
//                store, residual add, SwiGLU or split-K partial.
// At a decode batch of 64 the M128 x N64 MMAs and the Q4_K weight stream need about the same time per tile, so the
// MMA thread is kept fed by a stage ring of whole 256-K tiles.
// For 128-row token tiles (prefill, verify) and an even band count, CTAs run in pairs (clusters of two): each streams
// and dequantizes its own band, holds half of the token tile, and the pair's first CTA issues one M = 256 MMA
// (tcgen05.mma.cta_group::2) for both, half as many MMA instructions per weight tile.
// Every output element accumulates its K range in one order whatever NT is, so a row's result does not depend on the
// rest of the batch. Every copy here reads this GPU's global memory into this CTA's own shared memory.
//
// Every mbarrier wait is bounded (about 2 s on the global timer); a timeout writes a code to the error word, the CTA
// drains what it issued (again bounded), frees its tensor memory and returns; gc_step reports GC_E_DEVICE.
#include <cuda.h>

#include <algorithm>
#include <vector>

#include "common.cuh"
#include "dequant.cuh"
#include "kernels.h"

namespace gck {
namespace {

constexpr int kThreads = 736;              // 23 warps
constexpr int kEpiWarp0 = 3;               // warps 3-6: epilogue (TMEM lane quarters 3, 0, 1, 2)
constexpr int kDeqWarp0 = 7;               // warps 7-22: dequant, two groups
constexpr int kGroupWarps = 8;             // per group: two threads per weight row
constexpr unsigned long long kTimeoutNs = 2000000000ull;

enum ErrCode { kErrRawFull = 1, kErrRawEmpty, kErrStageEmpty, kErrAFull, kErrBFull, kErrAcc, kErrChain };

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

// Bounded wait until the counter reaches need (acquire at GPU scope); false (error word set) on timeout
GCK_DEV bool wait_count(const unsigned *cnt, unsigned need, int *err, int code) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(cnt) : "memory");
  if (v >= need) return true;
  const unsigned long long t0 = now_ns();
  for (uint32_t n = 1;; n++) {
    __nanosleep(128);
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(cnt) : "memory");
    if (v >= need) return true;
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

// ---- CTA pairs (cta_group::2): one M256 MMA over two CTAs' tensor memory and shared memory
GCK_DEV uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return r;
}
GCK_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
// the cluster-window address of the variable at p's offset in the shared memory of CTA `rank` of this cluster
GCK_DEV uint32_t cluster_addr(const void *p, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
  return a;
}
// Arrive on the other CTA's barrier (a cluster-window address). Default semantics (release at CTA scope), the form
// cluster pipelines use: the data the MMA reads after this signal are tensor memory, ordered by tcgen05.wait::st and
// the tcgen05 fences around the barrier, and activations the tensor-map copy wrote (its completion seen on b_full
// first). A release at cluster scope here cost about 1600 cycles per warp and stage, the arrive stalled until then.
GCK_DEV void mbar_arrive_cluster(uint32_t addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];\n" ::"r"(addr) : "memory");
}
// A from both CTAs' tensor memory (128 rows each, same columns), B from both CTAs' shared memory (N / 2 rows each,
// same offset), D into both CTAs' tensor memory (each its own 128 rows x N)
GCK_DEV void umma_f16_ts_pair(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(
          tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrives on the barrier at bar's offset in both CTAs of the pair once the issuing thread's MMAs have completed
GCK_DEV void umma_commit_pair(uint64_t *bar) {
  asm volatile(
      "{\n .reg .b16 m;\n mov.b16 m, 3;\n"
      " tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n}\n" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Stage geometry. A stage is KS of K: KS / 2 TMEM columns of dequantized weights (128 rows, two f16 per column)
// after the ACC accumulator buffers, and KS / 64 shared-memory activation boxes of NT / P rows x 64 K (128-byte
// swizzle; P = 2 for a CTA pair, each CTA holding half of the token tile). KS is a whole raw tile (256) up to NT = 128
// and half of one at NT = 256 (so that two activation stages fit).
template <int TYPE, int NT, int P = 1>
struct Shape {
  static constexpr int KS = NT >= 256 ? 128 : 256;
  static constexpr int SPT = kBK / KS;                  // stages per raw tile
  static constexpr int BOX_B = NT / P * 128;            // one 64-K activation box
  static constexpr int STAGE_B = (KS / 64) * BOX_B;
  static constexpr int NCOLS = NT <= 32 ? 32 : NT <= 64 ? 64 : NT <= 128 ? 128 : 256;
  static constexpr int ACC = NT <= 128 ? 2 : 1;
  static constexpr int RAW = TYPE == kQ4_K ? 4 : (NT >= 128 ? 2 : 4);
  static constexpr int R_TMEM = (512 - ACC * NCOLS) / (KS / 2);
  static constexpr int R_SMEM = (204 * 1024 - RAW * TileFmt<TYPE>::BYTES) / STAGE_B;
  static constexpr int R0 = R_TMEM < R_SMEM ? R_TMEM : R_SMEM;
  static constexpr int R = R0 > 4 ? 4 : R0;
  static_assert(R >= 2, "stage ring too shallow");
  // With one stage per raw tile the two dequant groups take alternate tiles. An even raw ring gives every slot a
  // single consumer group, which waits on it in order, so a parity wait can never pass on a phase two behind (with an
  // odd ring a group could see slot s "full" while the other group's earlier tile in s was still landing).
  static_assert(SPT == 2 || RAW % 2 == 0, "raw ring slots must each belong to one dequant group");
};


template <int TYPE, int NT, int P = 1>
constexpr int smem_total() {
  using S = Shape<TYPE, NT, P>;
  // at least 120 KB: one CTA per SM, since each takes all 512 TMEM columns
  constexpr int need = 1024 + S::R * S::STAGE_B + S::RAW * TileFmt<TYPE>::BYTES + 512;
  return need > 120 * 1024 ? need : 120 * 1024;
}

// Work unit w (0 .. units-1) = (weight tile, K split, token tile), the token tile fastest; a CTA takes units
// blockIdx.x, + gridDim.x, ... With several token tiles (prefill) the CTAs that run at the same time then share row
// bands, so a band's weight tiles come from DRAM once and from L2 for the other token tiles (token tile slowest, every
// tile pass streamed all the weights again: 6.7x the weight bytes at a 2048-token step). A unit's arithmetic does not
// depend on the order.
struct Unit {
  int nt, split, tt, kt0, per;
};
GCK_DEV Unit unit_of(int w, int NTW, int KT, int splits, int TT) {
  Unit u;
  u.tt = w % TT;
  int rem = w / TT;
  u.nt = rem / splits;
  u.split = rem % splits;
  const int base = KT / splits, extra = KT % splits;   // the first KT % splits splits take one more raw tile
  u.per = base + (u.split < extra ? 1 : 0);
  u.kt0 = u.split * base + min(u.split, extra);
  return u;
}

// P = 1: one CTA per MMA (M = 128). P = 2: a cluster of two CTAs (a pair) takes two adjacent 128-row bands, band
// 2 * pair band + CTA rank, against one token tile; each CTA streams and dequantizes its own band into its own tensor
// memory and loads half of the token rows, and the pair's first CTA issues one M = 256 MMA for both
// (tcgen05.mma.cta_group::2), which costs about what an M = 128 one does. The second CTA's dequant and epilogue warps
// arrive on the first CTA's barriers (a_full, acc_empty); the MMA thread's commits arrive on both CTAs' barriers
// (st_empty, acc_full, mma_done). Every copy still reads this GPU's global memory into this CTA's own shared memory.
template <int TYPE, int NT, int P>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const uint8_t *__restrict__ W, int NTW, int KT, int splits, int units,
                   const __grid_constant__ CUtensorMap tmap, int T, Epi epi, float *part, int Npad, int *err, Signal sig,
                   const __grid_constant__ CUtensorMap tmap1, Chain ch) {
  using F = TileFmt<TYPE>;
  using S = Shape<TYPE, NT, P>;
  constexpr int RS = S::RAW, SR = S::R, ACC = S::ACC, KS = S::KS, SPT = S::SPT;
  const uint32_t rank = P == 2 ? cluster_rank() : 0;
  const int first = blockIdx.x / P, stride = gridDim.x / P;   // this CTA's pair (or CTA), the number of them
  const int TT = units / (NTW / P * splits);           // token tiles
  // this CTA's units: first, first + stride, ... of the one GEMM; or, chained (P = 1, one token tile), its list in the
  // schedule, entries with bit 31 set being units of the second GEMM
  const bool chained = P == 1 && ch.W != nullptr;
  const int s0 = chained ? ch.sched_off[blockIdx.x] : 0;
  const int n_units = chained ? ch.sched_off[blockIdx.x + 1] - s0 : (units > first ? (units - first + stride - 1) / stride : 0);
  auto job = [&](int i, int &ph) -> Unit {
    if (chained) {
      const int e = ch.sched[s0 + i];
      ph = (e >> 31) & 1;
      const int w = e & 0x7fffffff;
      return ph ? unit_of(w, ch.NTW, ch.KT, ch.splits, 1) : unit_of(w, NTW, KT, splits, 1);
    }
    ph = 0;
    return unit_of(first + i * stride, NTW / P, KT, splits, TT);
  };
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned (the 128-byte swizzle atom) by an offset into the __shared__ array, so that every pointer derived
  // from it stays a shared-memory pointer to the compiler (shared loads, not generic ones); the offset is the same in
  // both CTAs of a pair, so the MMA's shared-memory descriptors address both
  uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t *sB = smem;
  uint8_t *sRaw = sB + SR * S::STAGE_B;
  uint64_t *bars = reinterpret_cast<uint64_t *>(sRaw + RS * F::BYTES);
  uint64_t *raw_full = bars, *raw_empty = raw_full + RS;
  uint64_t *a_full = raw_empty + RS, *st_empty = a_full + SR, *b_full = st_empty + SR;
  uint64_t *acc_full = b_full + SR, *acc_empty = acc_full + 2, *mma_done = acc_empty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // the next kernel may start as this one's CTAs run; the weight stream depends on no earlier kernel, so only the
  // activation producer and the epilogue wait for the previous kernels (dep_wait)
  dep_launch();

  if (threadIdx.x == 0) {
    // a raw tile is read by one dequant group (KS = 256) or by both (KS = 128); a pair's a_full and acc_empty (used in
    // its first CTA) count both CTAs' warps
    for (int i = 0; i < RS; i++) { mbar_init(&raw_full[i], 1); mbar_init(&raw_empty[i], kGroupWarps * SPT); }
    for (int i = 0; i < SR; i++) { mbar_init(&a_full[i], P * kGroupWarps); mbar_init(&st_empty[i], 1); mbar_init(&b_full[i], 1); }
    for (int i = 0; i < 2; i++) { mbar_init(&acc_full[i], 1); mbar_init(&acc_empty[i], 4 * P); }
    mbar_init(mma_done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    fence_async_smem();
  }
  if (warp == 1) {   // all 512 columns: ACC accumulator buffers, then the weight stages (one CTA per SM)
    if constexpr (P == 2) {    // both CTAs' warps 1 together: the same columns in each
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                   "r"(512));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;\n" ::);
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                   "r"(512));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (P == 2) cluster_sync();   // both CTAs' barriers initialised before any remote arrive or multicast commit
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_a = tmem + ACC * S::NCOLS;   // weight stage s at columns tmem_a + (KS / 2) * s

  if (warp == 0) {
    if (lane == 0) {
      // ---- raw weight tiles: one bulk copy each, up to RS tiles ahead, across unit boundaries
      long c = 0;
      bool ok = true;
      for (int i = 0; i < n_units && ok; i++) {
        int g2;
        const Unit un = job(i, g2);
        const int band = P * un.nt + static_cast<int>(rank);
        const uint8_t *Wp = g2 ? ch.W : W;
        const int KTp = g2 ? ch.KT : KT;
        for (int u = 0; u < un.per; u++, c++) {
          const int rs = static_cast<int>(c % RS);
          if (!(ok = mbar_wait(&raw_empty[rs], static_cast<uint32_t>((c / RS) & 1) ^ 1, err, kErrRawEmpty))) break;
          mbar_expect_tx(&raw_full[rs], F::BYTES);
          bulk_g2s(sRaw + rs * F::BYTES, Wp + (static_cast<size_t>(band) * KTp + un.kt0 + u) * F::BYTES, F::BYTES,
                   &raw_full[rs]);
        }
      }
      // every issued copy has landed before the CTA may exit (the last phase of each slot; bounded)
      for (long i = c > RS ? c - RS : 0; i < c; i++) mbar_wait(&raw_full[i % RS], static_cast<uint32_t>((i / RS) & 1), err, kErrRawFull);
    }
  } else if (warp == 2) {
    if (lane == 0) {
      // ---- activation stages: KS / 64 tensor-map copies (64 K each) per stage, up to SR stages ahead; a pair's CTA
      // loads token rows rank * NT / 2 .. of the tile
      dep_wait();
      long c = 0;
      bool ok = true;
      for (int j = 0; j < n_units && ok; j++) {
        int g2;
        const Unit un = job(j, g2);
        const int y = un.tt * NT + static_cast<int>(rank) * (NT / P);
        const CUtensorMap *map = g2 ? &tmap1 : &tmap;
        for (int i = 0; i < un.per * SPT; i++, c++) {
          const int s = static_cast<int>(c % SR);
          const int kt = un.kt0 + i / SPT;
          if (g2 && i % SPT == 0) {
            // a chained unit's input K tile: every first-GEMM band that writes it (4 bands of 64 features; 4 epilogue
            // warps each) has stored its rows; then its tensor-map copies may read them
            const int nb = min(4, NTW - 4 * kt);
            if (!(ok = wait_count(&ch.ready[kt], 4u * static_cast<unsigned>(nb), err, kErrChain))) break;
            asm volatile("fence.proxy.async.global;\n" ::: "memory");
          }
          if (!(ok = mbar_wait(&st_empty[s], static_cast<uint32_t>((c / SR) & 1) ^ 1, err, kErrStageEmpty))) break;
          mbar_expect_tx(&b_full[s], S::STAGE_B);
          const int x = kt * kBK + (i % SPT) * KS;
#pragma unroll
          for (int b = 0; b < KS / 64; b++) tma_2d(sB + s * S::STAGE_B + b * S::BOX_B, map, x + 64 * b, y, &b_full[s]);
        }
      }
      for (long i = c > SR ? c - SR : 0; i < c; i++) mbar_wait(&b_full[i % SR], static_cast<uint32_t>((i / SR) & 1), err, kErrBFull);
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---- MMA issuer (a pair's first CTA): accumulator buffer (local unit index) % 2
      const uint32_t idesc =
          (1u << 4) | (static_cast<uint32_t>(NT >> 3) << 17) | (static_cast<uint32_t>((P * kBM) >> 4) << 24);
      int s = 0;                 // stage slot and the parity of its current use
      uint32_t par = 0;
      int lu = 0;
      bool ok = true;
      for (int j = 0; j < n_units && ok; j++, lu++) {
        int g2;
        const Unit un = job(j, g2);
        const int ab = ACC == 2 ? (lu & 1) : 0;
        const uint32_t ph = ACC == 2 ? static_cast<uint32_t>((lu >> 1) & 1) : static_cast<uint32_t>(lu & 1);
        if (!(ok = mbar_wait(&acc_empty[ab], ph ^ 1, err, kErrAcc))) break;
        tc_fence_after();
        const uint32_t dt = tmem + ab * S::NCOLS;
        for (int i = 0; i < un.per * SPT; i++) {
          // a_full covers both operands: the dequant group signals it only after the stage's activations landed
          if (!(ok = mbar_wait(&a_full[s], par, err, kErrAFull))) break;
          tc_fence_after();
          const uint32_t at = tmem_a + (KS / 2) * s;
          const uint64_t bd = umma_desc(sB + s * S::STAGE_B);
#pragma unroll
          for (int k = 0; k < KS / 16; k++) {
            const uint64_t bk = bd + static_cast<uint64_t>((k >> 2) * (S::BOX_B >> 4) + 2 * (k & 3));
            if constexpr (P == 2) umma_f16_ts_pair(dt, at + 8 * k, bk, idesc, (i | k) != 0);
            else umma_f16_ts(dt, at + 8 * k, bk, idesc, (i | k) != 0);
          }
          if constexpr (P == 2) umma_commit_pair(&st_empty[s]);
          else umma_commit(&st_empty[s]);
          if (++s == SR) {
            s = 0;
            par ^= 1u;
          }
        }
        // arrives once every MMA of this unit has completed
        if constexpr (P == 2) umma_commit_pair(&acc_full[ab]);
        else umma_commit(&acc_full[ab]);
      }
      // completes once every MMA issued above has: the exit below never frees tensor memory still being written
      if constexpr (P == 2) umma_commit_pair(mma_done);
      else umma_commit(mma_done);
    }
  } else if (warp >= kDeqWarp0) {
    // ---- dequant: two groups of 8 warps take alternate stages, so one group's waits overlap the other's arithmetic.
    // In a group, two threads per weight row (TMEM lane = row), each KS / 2 of the stage's K, straight into TMEM.
    const int dw = warp - kDeqWarp0;
    const int grp = dw / kGroupWarps;
    const int hsel = (dw / 4) & 1;
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t a_full0 = P == 2 ? cluster_addr(a_full, 0) : 0u;   // the MMA-issuing CTA's a_full
    long c = 0, cr = 0;
    bool ok = true;
    for (int j = 0; j < n_units && ok; j++) {
      int g2;
      const Unit un = job(j, g2);
      for (int u = 0; u < un.per && ok; u++, cr++) {
        const int rs = static_cast<int>(cr % RS);
        for (int sub = 0; sub < SPT; sub++, c++) {
          if ((c & 1) != grp) continue;
          const int s = static_cast<int>(c % SR);
          // every lane waits; the warp leaves together if any lane's wait ran out (the stores below are warp-wide)
          ok = mbar_wait(&raw_full[rs], static_cast<uint32_t>((cr / RS) & 1), err, kErrRawFull);
          ok = ok && mbar_wait(&st_empty[s], static_cast<uint32_t>((c / SR) & 1) ^ 1, err, kErrStageEmpty);
          if (!(ok = __all_sync(0xffffffffu, ok))) break;
          tc_fence_after();
          const uint8_t *raw = sRaw + rs * F::BYTES;
          const uint4 hdr = *reinterpret_cast<const uint4 *>(raw + r * 16);
          const uint32_t col = tmem_a + (KS / 2) * s + lane_base + (KS / 4) * hsel;
          const int g0 = (KS / 32) * sub + (KS / 64) * hsel;   // first 32-K block of this thread
          if (TYPE == kQ4_K) {
            const uint32_t dd = prmt(hdr.x, 0, 0x1010u);                 // (d, d)
            const uint32_t mm = prmt(hdr.x, 0, 0x3232u) ^ 0x80008000u;   // (-dmin, -dmin)
#pragma unroll
            for (int gp = 0; gp < KS / 128; gp++) {
              const int g = g0 + 2 * gp;
              uint32_t S01, O01;
              q4k_pair_scales(hdr, g, dd, mm, S01, O01);
#pragma unroll
              for (int e = 0; e < 2; e++) {
                const uint32_t Sg = prmt(S01, 0, e ? 0x3232u : 0x1010u), Og = prmt(O01, 0, e ? 0x3232u : 0x1010u);
                const uint4 qw = *reinterpret_cast<const uint4 *>(raw + kBM * 16 + ((g + e) * kBM + r) * 16);
                uint32_t v[16];
                q4_word(qw.x, Sg, Og, v);
                q4_word(qw.y, Sg, Og, v + 4);
                q4_word(qw.z, Sg, Og, v + 8);
                q4_word(qw.w, Sg, Og, v + 12);
                tmem_st8(col + 16 * (2 * gp + e), v);
                tmem_st8(col + 16 * (2 * gp + e) + 8, v + 8);
              }
            }
          } else {
#pragma unroll
            for (int gi = 0; gi < KS / 64; gi++) {
              const int g = g0 + gi;
              const uint32_t dw2 = (g >> 1) == 0 ? hdr.x : (g >> 1) == 1 ? hdr.y : (g >> 1) == 2 ? hdr.z : hdr.w;
              const uint32_t D = prmt(dw2, 0, (g & 1) ? 0x3232u : 0x1010u);
              const uint4 q0 = *reinterpret_cast<const uint4 *>(raw + kBM * 16 + ((2 * g) * kBM + r) * 16);
              const uint4 q1 = *reinterpret_cast<const uint4 *>(raw + kBM * 16 + ((2 * g + 1) * kBM + r) * 16);
              uint32_t v[16];
              q8_word(q0.x, D, v); q8_word(q0.y, D, v + 2); q8_word(q0.z, D, v + 4); q8_word(q0.w, D, v + 6);
              q8_word(q1.x, D, v + 8); q8_word(q1.y, D, v + 10); q8_word(q1.z, D, v + 12); q8_word(q1.w, D, v + 14);
              tmem_st8(col + 16 * gi, v);
              tmem_st8(col + 16 * gi + 8, v + 8);
            }
          }
          // this group's last read of the raw tile (each group reads a tile once)
          __syncwarp();
          if (lane == 0) mbar_arrive(&raw_empty[rs]);
          tmem_st_wait();
          tc_fence_before();
          // the stage's activation tiles must have landed too: then a_full alone tells the MMA thread both are ready
          ok = mbar_wait(&b_full[s], static_cast<uint32_t>((c / SR) & 1), err, kErrBFull);
          if (!(ok = __all_sync(0xffffffffu, ok))) break;
          if (lane == 0) {
            if (P == 2 && rank != 0) mbar_arrive_cluster(a_full0 + 8u * s);
            else mbar_arrive(&a_full[s]);
          }
        }
      }
    }
  } else if (warp >= kEpiWarp0) {
    // ---- epilogue: TMEM lane quarter q = weight rows 32q .. 32q+31 of this CTA's band
    dep_wait();
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t acc_empty0 = P == 2 ? cluster_addr(acc_empty, 0) : 0u;
    int lu = 0;
    for (int j = 0; j < n_units; j++, lu++) {
      int g2;
      const Unit un = job(j, g2);
      const int band = P * un.nt + static_cast<int>(rank);
      const int ab = ACC == 2 ? (lu & 1) : 0;
      const uint32_t ph = ACC == 2 ? static_cast<uint32_t>((lu >> 1) & 1) : static_cast<uint32_t>(lu & 1);
      const bool good = mbar_wait_sleep(&acc_full[ab], ph, err, kErrAcc);
      tc_fence_after();
      const uint32_t tbase = tmem + ab * S::NCOLS + (static_cast<uint32_t>(q * 32) << 16);
      const int row = band * kBM + r, t0 = un.tt * NT;
      if (g2) {
        // a chained second-GEMM unit: its split-K partial, or (one slice) its residual add / store
        if (good) {
          const bool sliced = ch.splits > 1;
          float *p = sliced ? ch.part + static_cast<size_t>(un.split) * T * ch.Npad : nullptr;
          for (int c0 = 0; c0 < NT; c0 += 16) {
            uint32_t v[16];
            tmem_ld16(tbase + c0, v);
#pragma unroll
            for (int c = 0; c < 16; c++) {
              const int t = t0 + c0 + c;
              if (t >= T) continue;
              const float y = __uint_as_float(v[c]) * epi_scale(ch.epi, t);
              if (sliced) p[static_cast<size_t>(t) * ch.Npad + row] = y;
              else if (row < ch.epi.n) {
                float *o = ch.epi.out_f + static_cast<size_t>(t) * ch.epi.ld + row;
                if (ch.epi.kind == kEpiAdd) *o += y;
                else *o = y;
              }
            }
          }
        }
      } else if (splits > 1) {
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
        // even rows are gate rows, the odd row after each its up row (feature band * 64 + r / 2): the two lanes swap
        // values and each takes half the token columns (the gate lane the even ones)
        const int f = band * 64 + (r >> 1);
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
      if (chained && !g2) {
        // this band's features are stored: count the warp in for the second GEMM's K tile that reads them (every
        // lane's stores made visible at GPU scope first)
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicAdd(&ch.ready[(band * 64) / kBK], 1u);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (P == 2 && rank != 0) mbar_arrive_cluster(acc_empty0 + 8u * ab);
        else mbar_arrive(&acc_empty[ab]);
      }
      if (!good) break;
    }
  }
  // with a signal: every thread's stores are made visible system-wide; the last CTA to get here publishes the flag
  if (sig.flag) __threadfence_system();
  tc_fence_before();
  __syncthreads();
  if (sig.flag && threadIdx.x == 0) signal_if_last(sig);
  if (chained && threadIdx.x == 0) {
    // every thread of this CTA is past its waits on the K-tile counters; the last CTA to get here resets them for the
    // next chained launch (which reads them only after this launch has completed)
    __threadfence();
    if (atomicAdd(ch.done, 1u) == gridDim.x - 1) {
      for (int k = 0; k < ch.KT; k++) atomicExch(&ch.ready[k], 0u);
      atomicExch(ch.done, 0u);
      __threadfence();
    }
  }
  if (warp == 1) {
    // no MMA may still write the accumulators when they are freed (bounded; returns at once after a normal run); a
    // pair's commit of mma_done reaches both CTAs
    if (lane == 0) mbar_wait(mma_done, 0, err, kErrAcc);
    __syncwarp();
  }
  if constexpr (P == 2) {
    // neither CTA frees its tensor memory or leaves (its shared memory) while the other's arrives or the pair's MMAs
    // may still reach them: every thread of both CTAs is past its loop here, and both MMA-done waits have returned
    tc_fence_before();
    cluster_sync();
  }
  if (warp == 1) {
    tc_fence_after();
    if constexpr (P == 2) asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(512));
    else asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(512));
  }
}

// the number of two-CTA clusters of the paired kernel that can be resident at once (0: none)
int g_pair_clusters = 0;

template <int TYPE, int NT, int P>
void launch_nt(const QWeight &w, const CUtensorMap *map, int T, const Epi &epi, float *part, int *err, int sms,
               int pairs, const Signal &sig, cudaStream_t s) {
  const int units = w.NT / P * w.splits * ((T + NT - 1) / NT);
  int groups = P == 2 ? pairs : sms;
  if (units < groups) groups = units;
  const int smem = smem_total<TYPE, NT, P>();
  if constexpr (P == 1) {
    launch_pdl(gemm_tc_kernel<TYPE, NT, 1>, groups, kThreads, smem, s, w.data, w.NT, w.KT, w.splits, units, *map, T,
               epi, part, w.NT * kBM, err, sig, *map, Chain{});
  } else {
    // a cluster of two CTAs per pair, with programmatic serialization as launch_pdl gives the other kernels
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * groups);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = at;
    cfg.numAttrs = g_pdl ? 2 : 1;
    cudaLaunchKernelEx(&cfg, gemm_tc_kernel<TYPE, NT, 2>, w.data, w.NT, w.KT, w.splits, units, *map, T, epi, part,
                       w.NT * kBM, err, sig, *map, Chain{});
  }
}

template <int TYPE>
void launch_type(const QWeight &w, const TmaSet &ts, int T, const Epi &epi, float *part, int *err, int sms,
                 int pairs, const Signal &sig, cudaStream_t s) {
  const int nt = tc_token_tile(T);
  // pairs for even band counts at 128-row token tiles (each CTA loads the tile's half, a 64-row box). At 32 and 64
  // rows (decode) pairs measured slower: a pair stage took as long as one CTA's (2379 vs 2292 cycles, C3 step 5.25 vs
  // 5.15 ms), the MMA issue was not the limit there once halved.
  if (pairs > 0 && w.NT % 2 == 0 && nt == 128) {
    launch_nt<TYPE, 128, 2>(w, ts.map(64), T, epi, part, err, sms, pairs, sig, s);
    return;
  }
  const CUtensorMap *m = ts.map(nt);
  switch (nt) {
    case 16: launch_nt<TYPE, 16, 1>(w, m, T, epi, part, err, sms, pairs, sig, s); break;
    case 32: launch_nt<TYPE, 32, 1>(w, m, T, epi, part, err, sms, pairs, sig, s); break;
    case 64: launch_nt<TYPE, 64, 1>(w, m, T, epi, part, err, sms, pairs, sig, s); break;
    case 128: launch_nt<TYPE, 128, 1>(w, m, T, epi, part, err, sms, pairs, sig, s); break;
    default: launch_nt<TYPE, 256, 1>(w, m, T, epi, part, err, sms, pairs, sig, s); break;
  }
}

template <int TYPE, int NT>
void launch_chain_nt(const QWeight &w0, const CUtensorMap *m0, const Epi &e0, const CUtensorMap *m1, const Chain &ch,
                     int ctas, int T, int *err, cudaStream_t s) {
  // one token tile: the first GEMM's units are its bands (no K split: its SwiGLU epilogue needs whole sums)
  launch_pdl(gemm_tc_kernel<TYPE, NT, 1>, ctas, kThreads, smem_total<TYPE, NT, 1>(), s, w0.data, w0.NT, w0.KT, 1,
             w0.NT, *m0, T, e0, static_cast<float *>(nullptr), w0.NT * kBM, err, Signal{}, *m1, ch);
}

template <int TYPE>
void launch_chain_type(const QWeight &w0, const TmaSet &ts0, const Epi &e0, const TmaSet &ts1, const Chain &ch,
                       int ctas, int T, int *err, cudaStream_t s) {
  switch (tc_token_tile(T)) {
    case 16: launch_chain_nt<TYPE, 16>(w0, ts0.map(16), e0, ts1.map(16), ch, ctas, T, err, s); break;
    case 32: launch_chain_nt<TYPE, 32>(w0, ts0.map(32), e0, ts1.map(32), ch, ctas, T, err, s); break;
    default: launch_chain_nt<TYPE, 64>(w0, ts0.map(64), e0, ts1.map(64), ch, ctas, T, err, s); break;
  }
}

template <int TYPE, int NT, int P = 1>
void set_attr() {
  cudaFuncSetAttribute(gemm_tc_kernel<TYPE, NT, P>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       smem_total<TYPE, NT, P>());
}

// how many two-CTA clusters of the pair kernel fit on the device at once (one CTA per SM); 0 if none or on error
int max_pair_clusters() {
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sms / 2 * 2);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem_total<kQ4_K, 128, 2>();
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemm_tc_kernel<kQ4_K, 128, 2>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

}  // namespace

// The token tile (the MMA's N) for a step of T token rows: the smallest of 16 .. 128 that holds them, 128 above. A
// 256-row tile takes half of TMEM for one accumulator, which leaves one accumulator (a unit's epilogue stalls the
// next unit's MMAs) and two weight stages: measured slower for prefill and verify (C4 a8 33007 vs 37287 tok/s).
int tc_token_tile(int T) {
  if (T <= 16) return 16;
  if (T <= 32) return 32;
  if (T <= 64) return 64;
  return 128;
}

void gemm_tc_init() {
  set_attr<kQ4_K, 16>(); set_attr<kQ4_K, 32>(); set_attr<kQ4_K, 64>(); set_attr<kQ4_K, 128>(); set_attr<kQ4_K, 256>();
  set_attr<kQ8_0, 16>(); set_attr<kQ8_0, 32>(); set_attr<kQ8_0, 64>(); set_attr<kQ8_0, 128>(); set_attr<kQ8_0, 256>();
  set_attr<kQ4_K, 128, 2>(); set_attr<kQ8_0, 128, 2>();
  g_pair_clusters = max_pair_clusters();
}

int tc_pair_clusters() { return g_pair_clusters; }

double chain_schedule(int NTW0, int KT0, int NTW1, int KT1, int splits1, int sms, int *ctas, int *sched_out,
                      int *off_out) {
  const int total = NTW0 + NTW1 * splits1;
  const int G = std::min(sms, total);
  std::vector<std::vector<int>> lists(G);
  std::vector<double> load(G, 0.0);
  // a unit costs its raw tiles plus about half a tile of epilogue not hidden under the next unit
  for (int u = 0; u < NTW0; u++) {
    lists[u % G].push_back(u);
    load[u % G] += KT0 + 0.5;
  }
  const int base = KT1 / splits1, extra = KT1 % splits1;
  for (int sp = 0; sp < splits1; sp++)
    for (int nt = 0; nt < NTW1; nt++) {
      const int b = static_cast<int>(std::min_element(load.begin(), load.end()) - load.begin());
      lists[b].push_back(static_cast<int>(0x80000000u | static_cast<unsigned>(nt * splits1 + sp)));
      load[b] += base + (sp < extra ? 1 : 0) + 0.5;
    }
  if (sched_out && off_out) {
    int n = 0;
    for (int b = 0; b < G; b++) {
      off_out[b] = n;
      for (int e : lists[b]) sched_out[n++] = e;
    }
    off_out[G] = n;
  }
  if (ctas) *ctas = G;
  return *std::max_element(load.begin(), load.end());
}

void launch_gemm_tc_chain(const QWeight &w0, const TmaSet &ts0, const Epi &e0, const QWeight &w1, const TmaSet &ts1,
                          const Epi &e1, float *part1, const ChainPlan &cp, int T, int *err, cudaStream_t s) {
  if (T <= 0) return;
  Chain ch;
  ch.W = w1.data;
  ch.NTW = w1.NT;
  ch.KT = w1.KT;
  ch.splits = w1.splits;
  ch.epi = e1;
  ch.part = part1;
  ch.Npad = w1.NT * kBM;
  ch.sched = cp.sched;
  ch.sched_off = cp.off;
  ch.ready = cp.ready;
  ch.done = cp.done;
  if (w0.type == kQ4_K) launch_chain_type<kQ4_K>(w0, ts0, e0, ts1, ch, cp.ctas, T, err, s);
  else launch_chain_type<kQ8_0>(w0, ts0, e0, ts1, ch, cp.ctas, T, err, s);
}

size_t tc_tile_bytes(int type) { return type == kQ4_K ? TileFmt<kQ4_K>::BYTES : TileFmt<kQ8_0>::BYTES; }

void launch_gemm_tc(const QWeight &w, const TmaSet &ts, int T, const Epi &epi, float *part, int *err, int sms,
                    int pairs, cudaStream_t s, const Signal &sig) {
  if (T <= 0) return;
  if (pairs > g_pair_clusters) pairs = g_pair_clusters;
  if (pairs > sms / 2) pairs = sms / 2;
  if (w.type == kQ4_K) launch_type<kQ4_K>(w, ts, T, epi, part, err, sms, pairs, sig, s);
  else launch_type<kQ8_0>(w, ts, T, epi, part, err, sms, pairs, sig, s);
}

}  // namespace gck
