// Paged GQA attention over f16 or fp8 KV pages, for decode, prefill chunks and tree verify in one kernel.
//
// Reference math (goethe_engine/ref.py:55-57): for each query head, sc = q . K / sqrt(dh) over the visible rows,
// softmax, weighted sum of V. Visible rows (ref.py:102, abi/gc.h:139-146): the cached prefix rows 0 .. pos-1, then the
// token's ancestors (a chain: rows pos .. pos+j).
//
// Work decomposition. A warp owns 16 MMA rows: the G = H / KVH query heads of one kv head for up to 16 / G consecutive
// chain tokens of one item (a prefill chunk), or one token (decode, tree node). It walks the token's visible list in
// fixed groups of 16 entries and fixed splits of kSplit entries; splits are merged by attn_combine in split order. A
// group's K and V rows are gathered through the block table into shared memory with cp.async (double buffered); a CTA
// of several warps shares them when its warps serve consecutive tokens of one item. Every row's arithmetic depends only
// on its own list, so results are identical alone, batched, chunked or as tree nodes (batch invariance).
//
// Tensor cores (mma.sync m16n8k16, f16 x f16 -> f32):
//   S[16 rows x 8 entries] = Q[16 x dh] . K^T     (K as the B operand: one 8-entry tile per half of the group)
//   O[16 rows x dh] += P[16 x 16 entries] . V      (P straight from the S accumulators, V as the B operand)
// The head dimension is permuted inside the MMAs so that every lane reads contiguous bytes: for S, lane quad t reads
// dims [t*dh/4, (t+1)*dh/4) of its K row; for O, lane g owns output dims [g*dh/8, (g+1)*dh/8). A permutation of the
// contraction dimension does not change the dot product; the output dims are written back in their true places.
//
// fp8 pages: K and V codes are exact in f16; the per-page exponents (scale 2^e, see k_misc.cu) come back as a 2^-ek
// factor on each score and as a running exponent E on the accumulator (O is kept scaled by 2^E, E = the V exponent of
// the group's first entry; entries of other pages in the group carry 2^(E - ev) on their probability).
#include "common.cuh"
#include "kernels.h"

namespace gck {

namespace {

template <int DH, bool FP8>
struct Cfg {
  static constexpr int ESZ = FP8 ? 1 : 2;
  static constexpr int ROWB = DH * ESZ + 16;         // padded smem row: conflict-free fragment reads
  static constexpr int BUF = 2 * kGroup * ROWB;      // K rows then V rows
  static constexpr int CHUNKS = DH * ESZ / 16;       // 16-byte chunks per row
  static constexpr int NKS = DH / 16;                // QK k-steps
  static constexpr int NNT = DH / 8;                 // PV n-tiles
  static constexpr int SMEM = 2 * BUF + 2 * kGroup * 2 * 4;  // two buffers + page exponents
};

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;\n" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

template <int DH, bool FP8>
__global__ void __launch_bounds__(256) attn_kernel(PlanView pv, AttnArgs a) {
  using C = Cfg<DH, FP8>;
  extern __shared__ __align__(128) uint8_t sm[];
  int *sE = reinterpret_cast<int *>(sm + 2 * C::BUF);   // [2 bufs][16 entries][2] page exponents (K, V)

  const AttnWork w = pv.work[blockIdx.x];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, nthr = blockDim.x;
  const int g = lane / 4, t = lane % 4;
  const QGroup q0 = pv.qgroups[w.qg0];
  const Item it = pv.items[q0.item];
  int nvis_max = 0;
  for (int i = 0; i < w.nqg; i++) nvis_max = max(nvis_max, pv.qgroups[w.qg0 + i].nvis);
  const int lo = w.split * kSplit, hi = min(lo + kSplit, nvis_max);
  const int ngroups = (hi - lo + kGroup - 1) / kGroup;
  const bool active = warp < w.nqg;
  const QGroup qg = pv.qgroups[w.qg0 + (active ? warp : 0)];
  const int G = a.H / a.KVH;
  const int head = w.head;

  // rows g and g + 8 of this lane: (token, query head), validity and list length
  int tokr[2], qh[2], nvis[2];
  bool valid[2];
#pragma unroll
  for (int h = 0; h < 2; h++) {
    int r = g + 8 * h;
    int tl = r / G;
    valid[h] = active && tl < qg.ntok;
    tokr[h] = it.tok0 + qg.j0 + tl;
    qh[h] = head * G + r % G;
    nvis[h] = qg.path_len ? it.pos + qg.path_len : it.pos + qg.j0 + tl + 1;
  }

  // Q fragments: lane quad t holds dims [t*DH/4, (t+1)*DH/4) of rows g and g+8
  uint32_t qa[C::NKS][4];
#pragma unroll
  for (int h = 0; h < 2; h++) {
    uint32_t v[DH / 8];
    if (valid[h]) {
      const uint4 *src = reinterpret_cast<const uint4 *>(a.q + (static_cast<size_t>(tokr[h]) * a.H + qh[h]) * DH + t * (DH / 4));
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
      qa[s][h] = v[2 * s];
      qa[s][2 + h] = v[2 * s + 1];
    }
  }

  const uint8_t *kbase = static_cast<const uint8_t *>(a.kc);
  const uint8_t *vbase = static_cast<const uint8_t *>(a.vc);
  auto issue = [&](int gi, int buf) {
    uint8_t *sK = sm + buf * C::BUF;
    uint8_t *sV = sK + kGroup * C::ROWB;
    const int i0 = lo + gi * kGroup;
    for (int c = threadIdx.x; c < 2 * kGroup * C::CHUNKS; c += nthr) {
      int isv = c / (kGroup * C::CHUNKS), rem = c % (kGroup * C::CHUNKS);
      int e = rem / C::CHUNKS, ch = rem % C::CHUNKS;
      int i = i0 + e;
      bool ok = i < hi;
      int row = ok ? list_row(pv, it, q0, i) : 0;
      size_t off = ((static_cast<size_t>(row / kBlock) * a.KVH + head) * kBlock + row % kBlock) * (DH * C::ESZ) + ch * 16;
      uint8_t *dst = (isv ? sV : sK) + e * C::ROWB + ch * 16;
      cp_async16_pred(dst, (isv ? vbase : kbase) + off, ok);
    }
    if (FP8 && a.exps) {
      for (int e = threadIdx.x; e < kGroup; e += nthr) {
        int i = i0 + e;
        int ek = 0, ev = 0;
        if (i < hi) {
          int row = list_row(pv, it, q0, i);
          const int8_t *pe = a.exps + (static_cast<size_t>(row / kBlock) * a.KVH + head) * 2;
          ek = pe[0];
          ev = pe[1];
        }
        sE[(buf * kGroup + e) * 2] = ek;
        sE[(buf * kGroup + e) * 2 + 1] = ev;
      }
    }
    cp_async_commit();
  };

  float o[C::NNT][4];
#pragma unroll
  for (int j = 0; j < C::NNT; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  int E = 0;
  bool have_e = false;

  if (ngroups > 0) issue(0, 0);
  for (int gi = 0; gi < ngroups; gi++) {
    const int buf = gi & 1;
    if (gi + 1 < ngroups) {
      issue(gi + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const int i0 = lo + gi * kGroup;
    if (active && i0 < qg.nvis) {
      const uint8_t *sK = sm + buf * C::BUF;
      const uint8_t *sV = sK + kGroup * C::ROWB;
      // ---- S = Q K^T for entries 0..7 (tile 0) and 8..15 (tile 1)
      float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int tile = 0; tile < 2; tile++) {
        const uint8_t *kr = sK + (tile * 8 + g) * C::ROWB + t * (DH / 4) * C::ESZ;
        uint32_t kw[DH / 4 * C::ESZ / 4];
#pragma unroll
        for (int i = 0; i < DH / 4 * C::ESZ / 16; i++) {
          uint4 u = reinterpret_cast<const uint4 *>(kr)[i];
          kw[4 * i] = u.x; kw[4 * i + 1] = u.y; kw[4 * i + 2] = u.z; kw[4 * i + 3] = u.w;
        }
#pragma unroll
        for (int s = 0; s < C::NKS; s++) {
          uint32_t b[2];
          if (FP8) {
            b[0] = e4m3x2_to_h2(static_cast<uint16_t>(kw[s] & 0xffff));
            b[1] = e4m3x2_to_h2(static_cast<uint16_t>(kw[s] >> 16));
          } else {
            b[0] = kw[2 * s];
            b[1] = kw[2 * s + 1];
          }
          mma_f16(sc[tile], qa[s], b);
        }
      }
      // ---- scale, mask, online softmax (log2 domain)
      int evref = 0;
      float pscale[2][2] = {{1.f, 1.f}, {1.f, 1.f}};   // [tile][entry parity]: 2^(evref - ev)
      float kscale[2][2] = {{1.f, 1.f}, {1.f, 1.f}};
      if (FP8 && a.exps) {
        const int *ee = sE + buf * kGroup * 2;
        evref = ee[1];
#pragma unroll
        for (int tile = 0; tile < 2; tile++)
#pragma unroll
          for (int c = 0; c < 2; c++) {
            int e = tile * 8 + 2 * t + c;
            kscale[tile][c] = exp2f(-static_cast<float>(ee[2 * e]));
            pscale[tile][c] = exp2f(static_cast<float>(evref - ee[2 * e + 1]));
          }
      }
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int tile = 0; tile < 2; tile++)
#pragma unroll
        for (int c = 0; c < 4; c++) {
          int h = c / 2, e = tile * 8 + 2 * t + (c % 2);
          bool ok = valid[h] && i0 + e < nvis[h];
          float v = ok ? sc[tile][c] * a.scale_log2 * kscale[tile][c % 2] : -INFINITY;
          sc[tile][c] = v;
          mx[h] = fmaxf(mx[h], v);
        }
      float alpha[2];
#pragma unroll
      for (int h = 0; h < 2; h++) {
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
        float mn = fmaxf(mrow[h], mx[h]);
        alpha[h] = mn == -INFINITY ? 1.f : exp2f(mrow[h] - mn);
        mrow[h] = mn;
      }
      float ps[2] = {0.f, 0.f};
#pragma unroll
      for (int tile = 0; tile < 2; tile++)
#pragma unroll
        for (int c = 0; c < 4; c++) {
          int h = c / 2;
          float p = mrow[h] == -INFINITY ? 0.f : exp2f(sc[tile][c] - mrow[h]);
          ps[h] += p;
          sc[tile][c] = p * pscale[tile][c % 2];
        }
#pragma unroll
      for (int h = 0; h < 2; h++) {
        ps[h] += __shfl_xor_sync(0xffffffffu, ps[h], 1);
        ps[h] += __shfl_xor_sync(0xffffffffu, ps[h], 2);
        lrow[h] = lrow[h] * alpha[h] + ps[h];
      }
      float f0 = alpha[0], f1 = alpha[1];
      if (FP8 && a.exps) {
        float fe = have_e ? exp2f(static_cast<float>(evref - E)) : 1.f;
        f0 *= fe;
        f1 *= fe;
        E = evref;
        have_e = true;
      }
#pragma unroll
      for (int j = 0; j < C::NNT; j++) {
        o[j][0] *= f0; o[j][1] *= f0; o[j][2] *= f1; o[j][3] *= f1;
      }
      uint32_t pa[4] = {pack_h2(sc[0][0], sc[0][1]), pack_h2(sc[0][2], sc[0][3]), pack_h2(sc[1][0], sc[1][1]),
                        pack_h2(sc[1][2], sc[1][3])};
      // ---- O += P V: lane g owns output dims [g*DH/8, (g+1)*DH/8)
      constexpr int VB = DH / 8 * C::ESZ;   // bytes per entry per lane
      uint32_t vr[4][VB / 4];
#pragma unroll
      for (int q = 0; q < 4; q++) {
        int e = 2 * t + (q & 1) + (q >> 1) * 8;      // entries 2t, 2t+1, 2t+8, 2t+9
        if (VB >= 16) {
          const uint4 *src = reinterpret_cast<const uint4 *>(sV + e * C::ROWB + g * VB);
#pragma unroll
          for (int i = 0; i < VB / 16; i++) {
            uint4 u = src[i];
            vr[q][4 * i] = u.x; vr[q][4 * i + 1] = u.y; vr[q][4 * i + 2] = u.z; vr[q][4 * i + 3] = u.w;
          }
        } else {   // 8 bytes: fp8 with dh 64
          uint2 u = *reinterpret_cast<const uint2 *>(sV + e * C::ROWB + g * VB);
          vr[q][0] = u.x;
          vr[q][VB / 4 - 1] = u.y;
        }
      }
#pragma unroll
      for (int j = 0; j < C::NNT; j++) {
        uint32_t b[2];
        if (FP8) {
          // byte j of entries (2t, 2t+1) and (2t+8, 2t+9)
          uint32_t sel = (j % 4) | ((4 + j % 4) << 4);
          b[0] = e4m3x2_to_h2(static_cast<uint16_t>(prmt(vr[0][j / 4], vr[1][j / 4], sel)));
          b[1] = e4m3x2_to_h2(static_cast<uint16_t>(prmt(vr[2][j / 4], vr[3][j / 4], sel)));
        } else {
          uint32_t sel = (j % 2) ? 0x7632u : 0x5410u;
          b[0] = prmt(vr[0][j / 2], vr[1][j / 2], sel);
          b[1] = prmt(vr[2][j / 2], vr[3][j / 2], sel);
        }
        mma_f16(o[j], pa, b);
      }
    }
    __syncthreads();
  }

  if (!active || w.split >= qg.nsplit) return;
  const int pi = qg.part_base + head * qg.nsplit + w.split;
  const float inv = (FP8 && a.exps && have_e) ? exp2f(-static_cast<float>(E)) : 1.f;
#pragma unroll
  for (int h = 0; h < 2; h++) {
    if (!valid[h]) continue;
    int r = g + 8 * h;
    float *dst = a.part_o + (static_cast<size_t>(pi) * 16 + r) * DH;
#pragma unroll
    for (int j = 0; j < C::NNT; j++) {
      dst[(2 * t) * (DH / 8) + j] = o[j][2 * h] * inv;
      dst[(2 * t + 1) * (DH / 8) + j] = o[j][2 * h + 1] * inv;
    }
    if (t == 0) a.part_ml[static_cast<size_t>(pi) * 16 + r] = make_float2(mrow[h], lrow[h]);
  }
}

// out[token, head, :] = sum_s O_s 2^(m_s - m) / sum_s l_s 2^(m_s - m), splits in order
template <int DH>
__global__ void attn_combine(PlanView pv, AttnArgs a) {
  const QGroup qg = pv.qgroups[blockIdx.x];
  const Item it = pv.items[qg.item];
  const int head = blockIdx.y, G = a.H / a.KVH;
  const int rows = qg.ntok * G;
  for (int i = threadIdx.x; i < rows * DH; i += blockDim.x) {
    int r = i / DH, d = i % DH;
    const int pb = qg.part_base + head * qg.nsplit;
    float m = -INFINITY;
    for (int s = 0; s < qg.nsplit; s++) m = fmaxf(m, a.part_ml[static_cast<size_t>(pb + s) * 16 + r].x);
    float num = 0.f, den = 0.f;
    for (int s = 0; s < qg.nsplit; s++) {
      float2 ml = a.part_ml[static_cast<size_t>(pb + s) * 16 + r];
      float wgt = ml.x == -INFINITY ? 0.f : exp2f(ml.x - m);
      num += a.part_o[(static_cast<size_t>(pb + s) * 16 + r) * DH + d] * wgt;
      den += ml.y * wgt;
    }
    int tok = it.tok0 + qg.j0 + r / G, qh = head * G + r % G;
    a.out[(static_cast<size_t>(tok) * a.H + qh) * DH + d] = __float2half_rn(num / den);
  }
}

template <int DH, bool FP8>
void launch_t(const PlanView &pv, const AttnArgs &a, int nw, cudaStream_t s) {
  using C = Cfg<DH, FP8>;
  if (pv.n_work > 0) attn_kernel<DH, FP8><<<pv.n_work, 32 * nw, C::SMEM, s>>>(pv, a);
}

}  // namespace

void launch_attention(const PlanView &pv, const AttnArgs &a, int nw, cudaStream_t s) {
  if (a.dh == 128) {
    if (a.kv_fp8) launch_t<128, true>(pv, a, nw, s);
    else launch_t<128, false>(pv, a, nw, s);
  } else {
    if (a.kv_fp8) launch_t<64, true>(pv, a, nw, s);
    else launch_t<64, false>(pv, a, nw, s);
  }
}

void launch_attention_combine(const PlanView &pv, const AttnArgs &a, cudaStream_t s) {
  if (pv.n_qg <= 0) return;
  if (a.dh == 128) attn_combine<128><<<dim3(pv.n_qg, a.KVH), 128, 0, s>>>(pv, a);
  else attn_combine<64><<<dim3(pv.n_qg, a.KVH), 128, 0, s>>>(pv, a);
}

}  // namespace gck
