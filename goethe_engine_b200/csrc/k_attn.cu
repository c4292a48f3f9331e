// Paged GQA attention over f16 or fp8 KV pages, for decode, prefill chunks and tree verify in one kernel.
//
// Reference math (goethe_engine/ref.py:55-57): for each query head, sc = q . K / sqrt(dh) over the visible rows,
// softmax, weighted sum of V. Visible rows (ref.py:102, abi/gc.h:139-146): the cached prefix rows 0 .. pos-1, then the
// token's ancestors (a chain: rows pos .. pos+j).
//
// Work decomposition. A warp owns up to 16 query rows: the G = H / KVH query heads of one kv head for up to 16 / G
// consecutive chain tokens of one item (a prefill chunk), or one token (decode, tree node). It walks the token's
// visible list in fixed groups of 16 entries and fixed splits of pv.split entries (kSplit in batch-invariant buckets);
// the last CTA of a (query group, kv
// head) to finish merges the splits' partials in split order. A split's groups are resolved to pages once (block
// table; a tree token's own rows through its path); groups' K and V rows are gathered with cp.async, double
// buffered (decode warps: 20 resident per SM at <= 96 registers); a CTA of several warps shares them when its warps
// serve consecutive tokens of one item. Every row's arithmetic depends only on its own list, so results are identical
// alone, batched, chunked or as tree nodes (batch invariance).
//
// Tensor cores (mma.sync m16n8k16, f16 x f16 -> f32), with the 16 entries of a group as M and the query rows as N in
// tiles of 8 (a decode warp holds one tile: its G <= 8 heads):
//   S^T[16 entries x 8 rows] = K . Q^T,      O^T[dh x 8 rows] += V^T . P^T
// P^T comes from the S^T accumulators by an 8x8 transpose in registers (movmatrix).
//
// fp8 pages: K and V codes are exact in f16; the per-page exponents (scale 2^e, see k_misc.cu) come back as a 2^-ek
// factor on each score and as a running exponent E on the accumulator (O is kept scaled by 2^E, E = the V exponent of
// the group's first entry; entries of other pages in the group carry 2^(E - ev) on their probability).
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace gck {

namespace {

template <int DH, bool FP8>
struct Cfg {
  static constexpr int ESZ = FP8 ? 1 : 2;
  static constexpr int RB = DH * ESZ;                // bytes of one KV row of one head
  static constexpr int ROWB = RB;                    // smem row, its 16-byte chunks XOR-swizzled (chunk_at)
  static constexpr int BUF = 2 * kGroup * ROWB;      // K rows then V rows
  static constexpr int CHUNKS = RB / 16;             // 16-byte chunks per row
  static constexpr int SWZ = CHUNKS >= 8 ? 7 : CHUNKS - 1;
  static constexpr int NKS = DH / 16;                // QK k-steps
  static constexpr int NMT = DH / 16;                // PV m-tiles (16 head dims each)
  static constexpr int NST = 2;                      // gather ring: double buffered (occupancy beats lookahead)
  static constexpr int NGS = kSplit / kGroup;        // groups per split
  static constexpr int PG_OFF = NST * BUF;           // [NGS] page of each group (-1: entries resolved one by one)
  static constexpr int GE_OFF = PG_OFF + NGS * 4;    // [NGS][2] page exponents (K, V) of page groups
  static constexpr int EE_OFF = GE_OFF + NGS * 2;    // [NST][16][2] per-entry exponents of resolved groups
  static constexpr int SMEM = EE_OFF + NST * kGroup * 2;
  static constexpr int TAIL_OFF = (SMEM + 15) / 16 * 16;   // per-warp tail buffers of tree CTAs: K, V rows, exponents
  static constexpr int TAIL_B = BUF + 2 * kGroup;
};

// byte offset of 16-byte chunk c of smem row `row`: chunks are XOR-swizzled by the row's low bits, so that the
// fragment reads below (8 rows at one chunk column, or one row's chunks across 8 lanes) hit distinct bank groups
template <class C>
__device__ __forceinline__ int chunk_at(int row, int c) {
  return row * C::ROWB + ((c ^ (row & C::SWZ)) << 4);
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;\n" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
// 8x8 b16 transpose across the warp: lane (g, t) gives row g, columns 2t, 2t+1 and gets row g of the transpose
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(d) : "r"(x));
  return d;
}
// four e4m3 codes (bytes 0..3 of w) -> f16x2 of bytes (0, 1) and of bytes (2, 3), the word split into its 16-bit halves
__device__ __forceinline__ void e4m3x4_to_h2x2(uint32_t w, uint32_t &lo, uint32_t &hi) {
  asm("{\n .reg .b16 l, h;\n mov.b32 {l, h}, %2;\n cvt.rn.f16x2.e4m3x2 %0, l;\n cvt.rn.f16x2.e4m3x2 %1, h;\n}\n"
      : "=r"(lo), "=r"(hi)
      : "r"(w));
}
// the CTA's barrier; a one-warp CTA needs only the warp's (which orders the lanes' shared-memory accesses, the cp.async
// rows each lane waited for included)
template <int NW>
__device__ __forceinline__ void cta_sync() {
  if constexpr (NW == 1) __syncwarp();
  else __syncthreads();
}
// the running max's starting value: finite, and so far below any score (|score| < 2^100 in the log2 domain) that
// 2^(kMaxFloor - score) is 0
constexpr float kMaxFloor = -1e30f;
// 2^e as a float for an integer e in [-126, 127], built from its bits (exact)
__device__ __forceinline__ float pow2i(int e) { return __int_as_float((127 + e) << 23); }
// 2^x by the hardware approximation (PTX ex2.approx.ftz: exactly 1 at 0 and +0 at -inf; results below 2^-126 flush
// to 0, far under what an f16 probability or the f32 row sum can hold)
__device__ __forceinline__ float ex2(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(r) : "f"(x));
  return r;
}

// One warp = up to 8 * NT query rows (row r: token r / G of the group, query head head * G + r % G) against one kv
// head. Per 16-entry group, with the entries as the MMA's M and the query rows as its N (tiles of 8 rows):
//   S^T[16 entries x 8 rows] = K[16 x dh] . Q^T           (A = K from shared memory, B = Q^T held in registers)
//   O^T[dh x 8 rows]        += V^T[dh x 16 entries] . P^T  (A = V^T from shared memory, B = P^T: S^T transposed in
//                                                           registers with movmatrix)
// A row's arithmetic does not depend on how many rows or tiles the warp holds.
// Head dims are permuted inside the MMAs so that lanes read contiguous bytes: in QK, lane t's k indices of k-step s
// are dims t*dh/4 + 4s + {0,1,2,3}; in PV, lane g's output rows of m-tile mt are dims g*dh/8 + 2mt + {0, 1}.
template <int DH, bool FP8, int NW, int NT>
__global__ void __launch_bounds__(32 * NW, NT > 1 ? 1 : (NW == 1 ? 20 : 2)) attn_kernel(PlanView pv, AttnArgs a) {
  using C = Cfg<DH, FP8>;
  constexpr int NTHR = 32 * NW;
  dep_wait();
  dep_launch();
  extern __shared__ __align__(128) uint8_t sm[];
  int *sPg = reinterpret_cast<int *>(sm + C::PG_OFF);
  int8_t *sGE = reinterpret_cast<int8_t *>(sm + C::GE_OFF);
  int8_t *sEE = reinterpret_cast<int8_t *>(sm + C::EE_OFF);

  const AttnWork w = pv.work[blockIdx.x];
  if (w.nqg == 0) return;   // an empty entry of a work list padded to a captured step's grid
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int g = lane / 4, t = lane % 4;
  const QGroup q0 = pv.qgroups[w.qg0];
  const Item it = pv.items[q0.item];
  int nvis_max = 0;
  for (int i = 0; i < w.nqg; i++) nvis_max = max(nvis_max, pv.qgroups[w.qg0 + i].nvis);
  const int lo = w.split * pv.split, hi = min(lo + pv.split, nvis_max);
  // a CTA of several tree nodes shares only the groups of plain rows below the item's own rows; each warp then walks
  // the groups that reach its own path (its tail) from a private buffer, in the same order a lone warp would
  const bool tree_cta = NW > 1 && q0.path_len > 0;
  const int shared_hi = tree_cta ? min(hi, it.pos / kGroup * kGroup) : hi;
  const int ngroups = shared_hi > lo ? (shared_hi - lo + kGroup - 1) / kGroup : 0;
  const bool active = warp < w.nqg;
  const int qgi = w.qg0 + (active ? warp : 0);
  const QGroup qg = pv.qgroups[qgi];
  const int G = a.H / a.KVH;
  const int head = w.head;
  const int nrows = active ? qg.ntok * G : 0;
  const bool page_exp = FP8 && a.exps;

  // ---- the split's groups: a group of plain rows (entry i is row i: every group of a chain, and a tree token's
  // groups below its own rows) is one page, read from the block table once; the rest are resolved entry by entry
  for (int gi = tid; gi < ngroups; gi += NTHR) {
    const int i0 = lo + gi * kGroup;
    const bool plain = !q0.path_len || i0 + kGroup <= it.pos;
    const int pg = plain ? static_cast<int>(pv.blocks[it.blk_off + i0 / kBlock]) : -1;
    sPg[gi] = pg;
    if (page_exp && plain) {
      const int8_t *pe = a.exps + (static_cast<size_t>(pg) * a.KVH + head) * 2;
      sGE[2 * gi] = pe[0];
      sGE[2 * gi + 1] = pe[1];
    }
  }
  cta_sync<NW>();

  // ---- Q^T fragments: tile nt, lane (g, t): row nt*8 + g, dims t*dh/4 + 4s + {0,1} (b0) and {2,3} (b1)
  uint32_t qb[NT][C::NKS][2];
#pragma unroll
  for (int nt = 0; nt < NT; nt++) {
    const int r = nt * 8 + g;
    uint32_t v[DH / 8];
    if (r < nrows) {
      const int tok = it.tok0 + qg.j0 + r / G, qh = head * G + r % G;
      const uint4 *src = reinterpret_cast<const uint4 *>(a.q + (static_cast<size_t>(tok) * a.H + qh) * DH + t * (DH / 4));
#pragma unroll
      for (int i = 0; i < DH / 32; i++) {
        uint4 u = src[i];
        v[4 * i] = u.x; v[4 * i + 1] = u.y; v[4 * i + 2] = u.z; v[4 * i + 3] = u.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < DH / 8; i++) v[i] = 0u;
    }
#pragma unroll
    for (int s = 0; s < C::NKS; s++) {
      qb[nt][s][0] = v[2 * s];
      qb[nt][s][1] = v[2 * s + 1];
    }
  }
  // this lane's softmax rows: r = nt*8 + 2t + c
  int nvis[NT][2];
  bool rvalid[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; nt++)
#pragma unroll
    for (int c = 0; c < 2; c++) {
      const int r = nt * 8 + 2 * t + c;
      rvalid[nt][c] = r < nrows;
      nvis[nt][c] = qg.path_len ? it.pos + (r / G == 0 ? qg.path_len : qg.path_len1) : it.pos + qg.j0 + r / G + 1;
    }
  // a group that ends at or below every row's visible count needs no position masks (warp-uniform test)
  int nvis_lo = INT_MAX;
#pragma unroll
  for (int nt = 0; nt < NT; nt++)
#pragma unroll
    for (int c = 0; c < 2; c++)
      if (rvalid[nt][c]) nvis_lo = min(nvis_lo, nvis[nt][c]);
  nvis_lo = __reduce_min_sync(0xffffffffu, nvis_lo);

  const uint8_t *kbase = static_cast<const uint8_t *>(a.kc);
  const uint8_t *vbase = static_cast<const uint8_t *>(a.vc);
  // gather group gi's K and V rows into ring slot buf (entries past the list end read real rows and are masked)
  auto issue = [&](int gi, int buf) {
    uint8_t *sK = sm + buf * C::BUF;
    uint8_t *sV = sK + kGroup * C::ROWB;
    const int pg = sPg[gi];
    if (pg >= 0) {
      const size_t pb = (static_cast<size_t>(pg) * a.KVH + head) * (kBlock * C::RB);
#pragma unroll
      for (int c = tid; c < 2 * kGroup * C::CHUNKS; c += NTHR) {
        const int isv = c / (kGroup * C::CHUNKS), rem = c % (kGroup * C::CHUNKS);
        const int e = rem / C::CHUNKS, ch = rem % C::CHUNKS;
        cp_async16((isv ? sV : sK) + chunk_at<C>(e, ch), (isv ? vbase : kbase) + pb + e * C::RB + ch * 16);
      }
    } else {
      const int i0 = lo + gi * kGroup;
#pragma unroll
      for (int c = tid; c < 2 * kGroup * C::CHUNKS; c += NTHR) {
        const int isv = c / (kGroup * C::CHUNKS), rem = c % (kGroup * C::CHUNKS);
        const int e = rem / C::CHUNKS, ch = rem % C::CHUNKS;
        const int row = list_row(pv, it, q0, min(i0 + e, hi - 1));
        const size_t off = ((static_cast<size_t>(row / kBlock) * a.KVH + head) * kBlock + row % kBlock) * C::RB + ch * 16;
        cp_async16((isv ? sV : sK) + chunk_at<C>(e, ch), (isv ? vbase : kbase) + off);
      }
      if (page_exp) {
        for (int e = tid; e < kGroup; e += NTHR) {
          const int row = list_row(pv, it, q0, min(i0 + e, hi - 1));
          const int8_t *pe = a.exps + (static_cast<size_t>(row / kBlock) * a.KVH + head) * 2;
          sEE[(buf * kGroup + e) * 2] = pe[0];
          sEE[(buf * kGroup + e) * 2 + 1] = pe[1];
        }
      }
    }
  };

  float o[NT][C::NMT][4];
#pragma unroll
  for (int nt = 0; nt < NT; nt++)
#pragma unroll
    for (int j = 0; j < C::NMT; j++) o[nt][j][0] = o[nt][j][1] = o[nt][j][2] = o[nt][j][3] = 0.f;
  float mrow[NT][2], lrow[NT][2];
#pragma unroll
  // the running max starts at a finite floor far below any score: 2^(floor - m) is 0 once a score is seen, and
  // exactly 1 (with p = 2^-inf = 0) while a row has seen only masked entries, so no -inf special cases are needed
  for (int nt = 0; nt < NT; nt++) mrow[nt][0] = mrow[nt][1] = kMaxFloor, lrow[nt][0] = lrow[nt][1] = 0.f;
  int E = 0;
  bool have_e = false;

  // ring: group gi sits in slot gi % NST; every iteration commits one cp.async group (empty past the end), so waiting
  // for all but the newest NST - 1 groups means group gi has landed
#pragma unroll
  for (int st = 0; st < C::NST - 1; st++) {
    if (st < ngroups) issue(st, st);
    cp_async_commit();
  }
  // one 16-entry group of the row list starting at list index i0, staged at sK (K rows, then V rows): page groups
  // carry their (K, V) exponents in ge, resolved groups per-entry exponents in ee
  // rmask: the rows that take part (a tree node's own tail leaves the other node's rows out: an exact no-op for them)
  auto consume = [&](const uint8_t *sK, int i0, const int8_t *ge, const int8_t *ee, uint32_t rmask) {
    const uint8_t *sV = sK + kGroup * C::ROWB;
    // ---- S^T = K Q^T: A rows g, g+8 (entries), lane t's dim slice
    constexpr int KW = C::RB / 4 / 4;   // words of a lane's K slice
    uint32_t k0[KW], k1[KW];
#pragma unroll
    for (int i = 0; i < KW / 4; i++) {
      const int c = t * (KW / 4) + i;   // the lane's chunks of the row
      uint4 u = *reinterpret_cast<const uint4 *>(sK + chunk_at<C>(g, c));
      k0[4 * i] = u.x; k0[4 * i + 1] = u.y; k0[4 * i + 2] = u.z; k0[4 * i + 3] = u.w;
      u = *reinterpret_cast<const uint4 *>(sK + chunk_at<C>(g + 8, c));
      k1[4 * i] = u.x; k1[4 * i + 1] = u.y; k1[4 * i + 2] = u.z; k1[4 * i + 3] = u.w;
    }
    // two accumulator chains (even / odd k-steps), summed at the end: half the MMA dependency chain
    float sc[NT][4], sc2[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
      sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = sc2[nt][0] = sc2[nt][1] = sc2[nt][2] = sc2[nt][3] = 0.f;
#pragma unroll
    for (int s = 0; s < C::NKS; s++) {
      uint32_t af[4];
      if (FP8) {
        e4m3x4_to_h2x2(k0[s], af[0], af[2]);
        e4m3x4_to_h2x2(k1[s], af[1], af[3]);
      } else {
        af[0] = k0[2 * s]; af[2] = k0[2 * s + 1];
        af[1] = k1[2 * s]; af[3] = k1[2 * s + 1];
      }
#pragma unroll
      for (int nt = 0; nt < NT; nt++) mma_f16((s & 1) ? sc2[nt] : sc[nt], af, qb[nt][s]);
    }
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
      for (int c = 0; c < 4; c++) sc[nt][c] += sc2[nt][c];
    // ---- page scales of entries g and g + 8: 2^-ek on the scores, 2^(E - ev) on the probabilities. O stays in one
    // exponent frame E (O is kept scaled by 2^E); E moves (and O is rescaled) only when a page's V exponent is more
    // than kRebase away, so the f16 probabilities times 2^(E - ev) neither overflow nor lose their bits
    float ks0 = a.scale_log2, ks1 = a.scale_log2, pv0 = 1.f, pv1 = 1.f, fe = 1.f;
    if (page_exp) {
      int ev0, ev1, evref;
      if (ge) {
        const float k = a.scale_log2 * pow2i(-ge[0]);
        ks0 = ks1 = k;
        evref = ev0 = ev1 = ge[1];
      } else {
        evref = ee[1];
        ks0 = a.scale_log2 * pow2i(-ee[2 * g]);
        ks1 = a.scale_log2 * pow2i(-ee[2 * (g + 8)]);
        ev0 = ee[2 * g + 1];
        ev1 = ee[2 * (g + 8) + 1];
      }
      constexpr int kRebase = 10;
      if (!have_e) {
        E = evref;
        have_e = true;
      } else if (evref - E > kRebase || E - evref > kRebase) {
        fe = pow2i(evref - E);
        E = evref;
      }
      pv0 = pow2i(E - ev0);
      pv1 = pow2i(E - ev1);
    }
    const bool full = i0 + kGroup <= nvis_lo;
    // ---- online softmax per row (log2 domain); a row's 16 entries sit in the 8 lanes of one t. The max is reduced
    // across those lanes every group; the row sum stays per lane (every lane of a row applies the same rescalings)
    // and is reduced once after the last group
    uint32_t pb[NT][2];
    float f[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
      float x[2][2];   // [entry g / g+8][row c]
#pragma unroll
      for (int c = 0; c < 2; c++) {
        const bool in = rvalid[nt][c] && ((rmask >> (nt * 8 + 2 * t + c)) & 1u);
        if (full) {
          const float bias = in ? 0.f : -INFINITY;
          x[0][c] = fmaf(sc[nt][c], ks0, bias);
          x[1][c] = fmaf(sc[nt][2 + c], ks1, bias);
        } else {
          const bool ok0 = in && i0 + g < nvis[nt][c];
          const bool ok1 = in && i0 + g + 8 < nvis[nt][c];
          x[0][c] = ok0 ? sc[nt][c] * ks0 : -INFINITY;
          x[1][c] = ok1 ? sc[nt][2 + c] * ks1 : -INFINITY;
        }
      }
      float p[2][2];
#pragma unroll
      for (int c = 0; c < 2; c++) {
        float mx = fmaxf(x[0][c], x[1][c]);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float mn = fmaxf(mrow[nt][c], mx);
        const float alpha = ex2(mrow[nt][c] - mn);
        mrow[nt][c] = mn;
        p[0][c] = ex2(x[0][c] - mn);
        p[1][c] = ex2(x[1][c] - mn);
        lrow[nt][c] = lrow[nt][c] * alpha + (p[0][c] + p[1][c]);
        f[nt][c] = alpha * fe;
      }
      // P^T as the PV B operand: (entries 2t, 2t+1 | 2t+8, 2t+9) of row g
      pb[nt][0] = movmatrix_t(pack_h2(p[0][0] * pv0, p[0][1] * pv0));
      pb[nt][1] = movmatrix_t(pack_h2(p[1][0] * pv1, p[1][1] * pv1));
    }
    // rescaling by exactly 1 changes nothing: skipped when no row of the warp needs it
    bool one = true;
#pragma unroll
    for (int nt = 0; nt < NT; nt++) one = one && f[nt][0] == 1.f && f[nt][1] == 1.f;
    if (!__all_sync(0xffffffffu, one)) {
#pragma unroll
      for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int j = 0; j < C::NMT; j++) {
          o[nt][j][0] *= f[nt][0]; o[nt][j][1] *= f[nt][1]; o[nt][j][2] *= f[nt][0]; o[nt][j][3] *= f[nt][1];
        }
    }
    // ---- O^T += V^T P^T: lane (g, t) reads entries 2t, 2t+1, 2t+8, 2t+9, dims [g*dh/8, (g+1)*dh/8)
    constexpr int VW = C::RB / 8 / 4;   // words of a lane's V slice per entry
    uint32_t vr[4][VW];
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const int e = 2 * t + (q & 1) + (q >> 1) * 8;
      if (VW >= 4) {
#pragma unroll
        for (int i = 0; i < VW / 4; i++) {
          const uint4 u = *reinterpret_cast<const uint4 *>(sV + chunk_at<C>(e, g * (VW / 4) + i));
          vr[q][4 * i] = u.x; vr[q][4 * i + 1] = u.y; vr[q][4 * i + 2] = u.z; vr[q][4 * i + 3] = u.w;
        }
      } else {   // 8 bytes: fp8 with dh 64 (half of chunk g / 2)
        const uint2 u = *reinterpret_cast<const uint2 *>(sV + chunk_at<C>(e, g >> 1) + (g & 1) * 8);
        vr[q][0] = u.x;
        vr[q][VW - 1] = u.y;
      }
    }
#pragma unroll
    for (int mt = 0; mt < C::NMT; mt++) {
      uint32_t af[4];
      if (FP8) {
        // dims 2mt (rows g) and 2mt + 1 (rows g + 8) of the slice: byte 2mt % 4 (+1) of word mt / 2; one permute
        // gathers both dims' entry pairs (low half: dim 2mt, high half: dim 2mt + 1)
        const int wi = mt / 2, b0 = 2 * (mt % 2);
        const uint32_t sel = b0 | ((4 + b0) << 4) | ((b0 + 1) << 8) | ((5 + b0) << 12);
        e4m3x4_to_h2x2(prmt(vr[0][wi], vr[1][wi], sel), af[0], af[1]);
        e4m3x4_to_h2x2(prmt(vr[2][wi], vr[3][wi], sel), af[2], af[3]);
      } else {
        af[0] = prmt(vr[0][mt], vr[1][mt], 0x5410u);
        af[1] = prmt(vr[0][mt], vr[1][mt], 0x7632u);
        af[2] = prmt(vr[2][mt], vr[3][mt], 0x5410u);
        af[3] = prmt(vr[2][mt], vr[3][mt], 0x7632u);
      }
#pragma unroll
      for (int nt = 0; nt < NT; nt++) mma_f16(o[nt][mt], af, pb[nt]);
    }
  };

  for (int gi = 0; gi < ngroups; gi++) {
    const int buf = gi % C::NST;
    if (gi + C::NST - 1 < ngroups) issue(gi + C::NST - 1, (gi + C::NST - 1) % C::NST);
    cp_async_commit();
    cp_async_wait<C::NST - 1>();
    cta_sync<NW>();
    const int i0 = lo + gi * kGroup;
    if (active && i0 < qg.nvis)
      consume(sm + buf * C::BUF, i0, sPg[gi] >= 0 ? sGE + 2 * gi : nullptr, sEE + buf * kGroup * 2, 0xFFFFFFFFu);
    cta_sync<NW>();
  }
  cp_async_wait<0>();

  if constexpr (NW > 1) {
    if (tree_cta && active) {
      // this warp's tails: for each of its tree tokens (one or two), the list entries from the item's last plain group
      // boundary, resolved through that token's path, with the other token's rows left out
      uint8_t *tK = sm + C::TAIL_OFF + warp * C::TAIL_B;
      uint8_t *tV = tK + kGroup * C::ROWB;
      int8_t *tE = reinterpret_cast<int8_t *>(tK + C::BUF);
      const int nnode = qg.path_len1 > 0 ? 2 : 1;
      for (int nd = 0; nd < nnode; nd++) {
        const int poff = nd ? qg.path_off1 : qg.path_off;
        const int hiw = min(lo + pv.split, it.pos + (nd ? qg.path_len1 : qg.path_len));
        const uint32_t rmask = nnode == 1 ? 0xFFFFFFFFu : ((1u << G) - 1u) << (nd * G);
        for (int i0 = max(lo, shared_hi); i0 < hiw; i0 += kGroup) {
          for (int c = lane; c < 2 * kGroup * C::CHUNKS; c += 32) {
            const int isv = c / (kGroup * C::CHUNKS), rem = c % (kGroup * C::CHUNKS);
            const int e = rem / C::CHUNKS, ch = rem % C::CHUNKS;
            const int row = list_row_path(pv, it, poff, min(i0 + e, hiw - 1));
            const size_t off =
                ((static_cast<size_t>(row / kBlock) * a.KVH + head) * kBlock + row % kBlock) * C::RB + ch * 16;
            cp_async16((isv ? tV : tK) + chunk_at<C>(e, ch), (isv ? vbase : kbase) + off);
          }
          if (page_exp && lane < kGroup) {
            const int row = list_row_path(pv, it, poff, min(i0 + lane, hiw - 1));
            const int8_t *pe = a.exps + (static_cast<size_t>(row / kBlock) * a.KVH + head) * 2;
            tE[2 * lane] = pe[0];
            tE[2 * lane + 1] = pe[1];
          }
          cp_async_commit();
          cp_async_wait<0>();
          __syncwarp();
          consume(tK, i0, nullptr, tE, rmask);
          __syncwarp();
        }
      }
    }
  }

  // the row sums: the 8 lanes of a row (same t) hold their entries' shares, reduced in one fixed order
#pragma unroll
  for (int nt = 0; nt < NT; nt++)
#pragma unroll
    for (int c = 0; c < 2; c++) {
      float l = lrow[nt][c];
      l += __shfl_xor_sync(0xffffffffu, l, 4);
      l += __shfl_xor_sync(0xffffffffu, l, 8);
      l += __shfl_xor_sync(0xffffffffu, l, 16);
      lrow[nt][c] = l;
    }

  if (!active || w.split >= qg.nsplit) return;
  const int rows = qg.ntok * G;
  const float inv = (page_exp && have_e) ? pow2i(-E) : 1.f;
  if (qg.nsplit == 1) {
    // the whole list in one split: out = (O 2^-E) / l, which is what the merge below computes for a single split
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
      for (int c = 0; c < 2; c++) {
        if (!rvalid[nt][c]) continue;
        const int r = nt * 8 + 2 * t + c;
        const int tok = it.tok0 + qg.j0 + r / G, qo = head * G + r % G;
        uint32_t wv[C::NMT];
#pragma unroll
        for (int mt = 0; mt < C::NMT; mt++)
          wv[mt] = pack_h2((o[nt][mt][c] * inv) / lrow[nt][c], (o[nt][mt][2 + c] * inv) / lrow[nt][c]);
        uint32_t *dst = reinterpret_cast<uint32_t *>(a.out + (static_cast<size_t>(tok) * a.H + qo) * DH + g * (DH / 8));
#pragma unroll
        for (int mt = 0; mt < C::NMT; mt++) dst[mt] = wv[mt];
      }
    return;
  }
  const int pi = qg.part_base + head * qg.nsplit + w.split;
#pragma unroll
  for (int nt = 0; nt < NT; nt++)
#pragma unroll
    for (int c = 0; c < 2; c++) {
      if (!rvalid[nt][c]) continue;
      const int r = nt * 8 + 2 * t + c;
      float2 *dst = reinterpret_cast<float2 *>(a.part_o + (static_cast<size_t>(pi) * 16 + r) * DH + g * (DH / 8));
#pragma unroll
      for (int mt = 0; mt < C::NMT; mt++) dst[mt] = make_float2(o[nt][mt][c] * inv, o[nt][mt][2 + c] * inv);
      if (g == 0) a.part_ml[static_cast<size_t>(pi) * 16 + r] = make_float2(mrow[nt][c], lrow[nt][c]);
    }
  // ---- the last split of (query group, kv head) to finish merges them all, in split order:
  // out = sum_s O_s 2^(m_s - m) / sum_s l_s 2^(m_s - m). Which split finishes last does not change the arithmetic.
  __threadfence();
  __syncwarp();
  int last = 0;
  if (lane == 0) last = atomicAdd(&a.sem[qgi * a.KVH + head], 1) == qg.nsplit - 1;
  last = __shfl_sync(0xffffffffu, last, 0);
  if (!last) return;
  __threadfence();
  // kMergeRows rows at a time: their (m, l) per split a lane each, then their O rows of kMergeChunk splits loaded
  // together (a lane's DPL consecutive dims of each, one vector load); every element still sums in split order, and
  // which split finished last does not change the arithmetic
  constexpr int kMergeChunk = 8, kMergeRows = 2, DPL = DH / 32;
  using Vec = typename std::conditional<DPL == 4, float4, float2>::type;
  const int pb0 = qg.part_base + head * qg.nsplit, S = qg.nsplit;
  for (int rb = 0; rb < rows; rb += kMergeRows) {
    float m[kMergeRows];
#pragma unroll
    for (int r = 0; r < kMergeRows; r++) m[r] = -INFINITY;
    for (int s0 = 0; s0 < S; s0 += 32)
#pragma unroll
      for (int r = 0; r < kMergeRows; r++)
        if (rb + r < rows && s0 + lane < S)
          m[r] = fmaxf(m[r], __ldcg(&a.part_ml[static_cast<size_t>(pb0 + s0 + lane) * 16 + rb + r]).x);
#pragma unroll
    for (int r = 0; r < kMergeRows; r++) m[r] = warp_max(m[r]);
    float num[kMergeRows][DPL], den[kMergeRows];
#pragma unroll
    for (int r = 0; r < kMergeRows; r++) {
      den[r] = 0.f;
#pragma unroll
      for (int k = 0; k < DPL; k++) num[r][k] = 0.f;
    }
    for (int s0 = 0; s0 < S; s0 += 32) {
      float wr[kMergeRows], lr[kMergeRows];
#pragma unroll
      for (int r = 0; r < kMergeRows; r++) {
        const float2 ml = rb + r < rows && s0 + lane < S
                              ? __ldcg(&a.part_ml[static_cast<size_t>(pb0 + s0 + lane) * 16 + rb + r])
                              : make_float2(-INFINITY, 0.f);
        wr[r] = ml.x == -INFINITY ? 0.f : exp2f(ml.x - m[r]);
        lr[r] = ml.y;
      }
      const int n = min(32, S - s0);
      for (int j0 = 0; j0 < n; j0 += kMergeChunk) {
        float po[kMergeChunk][kMergeRows][DPL];
#pragma unroll
        for (int j = 0; j < kMergeChunk; j++)
#pragma unroll
          for (int r = 0; r < kMergeRows; r++) {
            Vec v;
            if (j0 + j < n && rb + r < rows) {
              const float *src = a.part_o + (static_cast<size_t>(pb0 + s0 + j0 + j) * 16 + rb + r) * DH + lane * DPL;
              v = __ldcg(reinterpret_cast<const Vec *>(src));
            } else {
              v = Vec{};
            }
            const float *vf = reinterpret_cast<const float *>(&v);
#pragma unroll
            for (int k = 0; k < DPL; k++) po[j][r][k] = vf[k];
          }
#pragma unroll
        for (int j = 0; j < kMergeChunk; j++)
#pragma unroll
          for (int r = 0; r < kMergeRows; r++) {
            const float wj = __shfl_sync(0xffffffffu, wr[r], (j0 + j) & 31);
            const float lj = __shfl_sync(0xffffffffu, lr[r], (j0 + j) & 31);
            if (j0 + j < n) {
#pragma unroll
              for (int k = 0; k < DPL; k++) num[r][k] += po[j][r][k] * wj;
              den[r] += lj * wj;
            }
          }
      }
    }
#pragma unroll
    for (int r = 0; r < kMergeRows; r++) {
      if (rb + r >= rows) break;
      const int tok = it.tok0 + qg.j0 + (rb + r) / G, qo = head * G + (rb + r) % G;
      __half *dst = a.out + (static_cast<size_t>(tok) * a.H + qo) * DH + lane * DPL;
#pragma unroll
      for (int k = 0; k < DPL; k++) dst[k] = __float2half_rn(num[r][k] / den[r]);
    }
  }
  if (lane == 0) a.sem[qgi * a.KVH + head] = 0;   // ready for the next launch
}

template <int DH, bool FP8, int NW, int NT>
void launch_t(const PlanView &pv, const AttnArgs &a, cudaStream_t s) {
  using C = Cfg<DH, FP8>;
  constexpr int kMaxSmem = C::TAIL_OFF + NW * C::TAIL_B;
  const int smem = NW > 1 && pv.tree_cta ? kMaxSmem : C::SMEM;
  // per device (tensor-parallel ranks launch on theirs from their own threads)
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(attn_kernel<DH, FP8, NW, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (pv.n_work > 0) launch_pdl(attn_kernel<DH, FP8, NW, NT>, pv.n_work, 32 * NW, smem, s, pv, a);
}
template <int DH, bool FP8>
void launch_dh(const PlanView &pv, const AttnArgs &a, int nw, cudaStream_t s) {
  const bool wide = pv.max_rows > 8;
  if (nw > 1) {
    if (wide) launch_t<DH, FP8, 8, 2>(pv, a, s);
    else launch_t<DH, FP8, 8, 1>(pv, a, s);
  } else {
    if (wide) launch_t<DH, FP8, 1, 2>(pv, a, s);
    else launch_t<DH, FP8, 1, 1>(pv, a, s);
  }
}

}  // namespace

void launch_attention(const PlanView &pv, const AttnArgs &a, int nw, cudaStream_t s) {
  if (a.dh == 128) {
    if (a.kv_fp8) launch_dh<128, true>(pv, a, nw, s);
    else launch_dh<128, false>(pv, a, nw, s);
  } else {
    if (a.kv_fp8) launch_dh<64, true>(pv, a, nw, s);
    else launch_dh<64, false>(pv, a, nw, s);
  }
}

}  // namespace gck
