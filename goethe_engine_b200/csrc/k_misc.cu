// Row-wise kernels of the decoder step: embedding gather, RMSNorm, RoPE + KV write (f16 or fp8 with per-page
// scales), split-K reduction with the GEMM epilogues, argmax, and the KV block operations behind gc_copy_blocks and
// gc_commit. Each is HBM- or latency-bound and touches every byte once.
//
// Reference math (goethe_engine/ref.py): rms ref.py:14-15, RoPE ref.py:31-37 (interleaved pairs), KV write ref.py:54,
// SwiGLU ref.py:59, commit ref.py:114-120, copy_blocks ref.py:122-126.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace gck {

// ----------------------------------------------------------------------------------------------------------------
// embedding: x[t, :] = dequant(token_embd[tok[t], :])
__device__ float dequant_elem(const uint8_t *row, int type, int e) {
  switch (type) {
    case kF32: return reinterpret_cast<const float *>(row)[e];
    case kF16: return __half2float(reinterpret_cast<const __half *>(row)[e]);
    case kQ8_0: {
      const uint8_t *b = row + (e / 32) * 34;
      return __half2float(*reinterpret_cast<const __half *>(b)) * static_cast<float>(static_cast<int8_t>(b[2 + e % 32]));
    }
    default: {  // Q4_K
      const uint8_t *b = row + (e / 256) * 144;
      int w = e % 256, sub = w / 32, l = w % 32, c = sub / 2;
      const uint8_t *s = b + 4;
      int sc, m;
      if (sub < 4) { sc = s[sub] & 63; m = s[sub + 4] & 63; }
      else { sc = (s[sub + 4] & 15) | ((s[sub - 4] >> 6) << 4); m = (s[sub + 4] >> 4) | ((s[sub] >> 6) << 4); }
      int q = (sub & 1) ? (b[16 + 32 * c + l] >> 4) : (b[16 + 32 * c + l] & 15);
      float d = __half2float(*reinterpret_cast<const __half *>(b));
      float dm = __half2float(*reinterpret_cast<const __half *>(b + 2));
      return d * static_cast<float>(sc) * static_cast<float>(q) - dm * static_cast<float>(m);
    }
  }
}

__global__ void embed_kernel(PlanView pv, const uint8_t *emb, int type, size_t row_bytes, int d, float *x) {
  dep_wait();
  dep_launch();
  int t = blockIdx.x;
  const uint8_t *row = emb + static_cast<size_t>(pv.tok_id[t]) * row_bytes;
  for (int e = threadIdx.x; e < d; e += blockDim.x) x[static_cast<size_t>(t) * d + e] = dequant_elem(row, type, e);
}

void launch_embed(const PlanView &pv, const uint8_t *emb, int type, size_t row_bytes, int d, float *x,
                  cudaStream_t s) {
  launch_pdl(embed_kernel, pv.T, 256, 0, s, pv, emb, type, row_bytes, d, x);
}

// ----------------------------------------------------------------------------------------------------------------
// RMSNorm: out[r, :] = f16(x[src(r), :] * rsqrt(mean(x^2) + eps) * gain); columns d .. ld-1 are zeroed.
// With residual partials (a split-K o_proj / down_proj before it): first x[src] += sum_s part[s, src, :] (splits in
// order, from 0), written back, as that GEMM's residual-add epilogue would have.
// One CTA per row; float4 loads, all issued before the first use. The sum of squares has a fixed order (each thread's
// strided partials in index order, then a fixed shuffle tree, then the warps in index order), independent of the batch.
// ---- tensor-parallel peer-memory reduction (declared in kernels.h)
constexpr int kErrTpWait = 16;                    // error word: a peer's flag did not arrive within the limit
constexpr unsigned long long kTpTimeoutNs = 2000000000ull;

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;\n" : "=l"(t));
  return t;
}
// thread 0: until flag[k][b] >= need for ranks k in [k0, k1) (bounded: sets the error word and returns false)
__device__ bool tp_wait_flags(const TpPeers &p, int k0, int k1, int b, unsigned long long need) {
  const unsigned long long t0 = global_ns();
  for (int k = k0; k < k1; k++)
    while (ld_acquire_sys(p.flag[k] + b) < need) {
      if (global_ns() - t0 > kTpTimeoutNs) {
        atomicCAS(p.err, 0, kErrTpWait);
        return false;
      }
      __nanosleep(64);
    }
  return true;
}

__global__ void tp_signal_kernel(unsigned long long *flag, unsigned long long value) {
  // the stream's earlier kernels have completed: make their writes visible system-wide, then publish
  __threadfence_system();
  asm volatile("st.release.sys.global.u64 [%0], %1;\n" ::"l"(flag), "l"(value) : "memory");
}

// rows [r0, r1) of this rank: the sum over ranks 0 .. n-1 (in that order) of their partials, into this rank's buffer
__global__ void tp_reduce_scatter_kernel(TpPeers p, int b, unsigned long long epoch, int T, int d, int S, Signal sig) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = tp_wait_flags(p, 0, p.n, b, epoch * 4 + 1);
  __syncthreads();
  if (!ok) return;   // the flag is not published: the readers' waits run out too and the step reports the error
  int r0, r1;
  tp_rows(T, p.n, p.rank, r0, r1);
  const int nv = d / 4;
  const size_t total = static_cast<size_t>(r1 - r0) * nv;
  float4 *dst = reinterpret_cast<float4 *>(p.buf[p.rank][b]);
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t e = static_cast<size_t>(r0) * nv + i;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    const size_t slice = static_cast<size_t>(T) * nv;   // float4s of one split-K slice
    for (int k = 0; k < p.n; k++)
      for (int sp = 0; sp < S; sp++) {
        const float4 x = __ldcv(reinterpret_cast<const float4 *>(p.buf[k][b]) + sp * slice + e);
        a.x += x.x; a.y += x.y; a.z += x.z; a.w += x.w;
      }
    dst[e] = a;   // into slice 0 of this rank's rows: no other rank reads them in this phase
  }
  if (sig.flag) {
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) signal_if_last(sig);
  }
}

void launch_tp_signal(unsigned long long *flag, unsigned long long value, cudaStream_t s) {
  tp_signal_kernel<<<1, 1, 0, s>>>(flag, value);
}
void launch_tp_reduce_scatter(const TpPeers &p, int b, unsigned long long epoch, int T, int d, int S, const Signal &sig,
                              cudaStream_t s) {
  int r0, r1;
  tp_rows(T, p.n, p.rank, r0, r1);
  const size_t total = static_cast<size_t>(std::max(0, r1 - r0)) * (d / 4);
  int blocks = static_cast<int>(std::min<size_t>((total + 255) / 256, 148 * 8));
  tp_reduce_scatter_kernel<<<std::max(blocks, 1), 256, 0, s>>>(p, b, epoch, T, d, S, sig);
}

// a8: the per-token scale of a row whose largest magnitude is amax (symmetric int8: amax maps to 127); an all-zero row
// keeps scale 1 (every code 0). IEEE division, as the oracle computes it.
__device__ __forceinline__ float act_scale_of(float amax) { return amax > 0.f ? __fdiv_rn(amax, 127.f) : 1.f; }

constexpr int kNormThreads = 512;
constexpr int kNormMaxVec = 4;    // float4 loads per thread: d <= 512 * 4 * 4 = 8192
// split-K partials are read kSplitChunk slices at a time (RMSNorm: as many as keep 16 float4 loads per thread),
// all their loads in flight together, and summed in split order
constexpr int kSplitChunk = 4;

template <int NV>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(float *x, const int *rows, const float *gain, float eps,
                                                               int d, int ld, __half *out, const float *part, int S,
                                                               int pld, int T, TpPeers tp, int tpb,
                                                               unsigned long long tp_epoch, float *qscale) {
  dep_wait();
  dep_launch();
  int r = blockIdx.x;
  int src = rows ? rows[r] : r;
  const float *tpsum = nullptr;   // tensor parallelism: this row's all-reduced sum, at its owner rank
  if (tp.n > 1) {
    const int per = (T + tp.n - 1) / tp.n, owner = src / per;
    __shared__ int ok;
    if (threadIdx.x == 0) ok = tp_wait_flags(tp, owner, owner + 1, tpb, tp_epoch * 4 + 2);
    __syncthreads();
    if (!ok) return;
    tpsum = tp.buf[owner][tpb] + static_cast<size_t>(src) * d;
  }
  float4 *xr = reinterpret_cast<float4 *>(x + static_cast<size_t>(src) * d);
  const float4 *gr = reinterpret_cast<const float4 *>(gain);
  const int nv = d / 4;
  float4 v[NV];
#pragma unroll
  for (int i = 0; i < NV; i++) {
    int e = threadIdx.x + i * kNormThreads;
    v[i] = e < nv ? xr[e] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (tpsum) {
#pragma unroll
    for (int i = 0; i < NV; i++) {
      int e = threadIdx.x + i * kNormThreads;
      if (e >= nv) continue;
      const float4 a = __ldcv(reinterpret_cast<const float4 *>(tpsum) + e);
      v[i].x += a.x; v[i].y += a.y; v[i].z += a.z; v[i].w += a.w;
      xr[e] = v[i];
    }
  }
  if (part) {
    // per element: ((0 + p_0) + p_1) + ... in split order, then added to x; a chunk's loads are all issued first
    float4 a[NV];
#pragma unroll
    for (int i = 0; i < NV; i++) a[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    // a chunk of CH splits keeps 16 float4 loads in flight per thread whatever the row length
    constexpr int CH = 16 / NV;
    for (int sp0 = 0; sp0 < S; sp0 += CH) {
      float4 pp[CH][NV];
#pragma unroll
      for (int j = 0; j < CH; j++) {
        const float4 *pr = reinterpret_cast<const float4 *>(part + (static_cast<size_t>(sp0 + j) * T + src) * pld);
#pragma unroll
        for (int i = 0; i < NV; i++) {
          int e = threadIdx.x + i * kNormThreads;
          pp[j][i] = sp0 + j < S && e < nv ? pr[e] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
#pragma unroll
      for (int j = 0; j < CH; j++) {
        if (sp0 + j >= S) break;
#pragma unroll
        for (int i = 0; i < NV; i++) {
          a[i].x += pp[j][i].x; a[i].y += pp[j][i].y; a[i].z += pp[j][i].z; a[i].w += pp[j][i].w;
        }
      }
    }
#pragma unroll
    for (int i = 0; i < NV; i++) {
      int e = threadIdx.x + i * kNormThreads;
      if (e >= nv) continue;
      v[i].x += a[i].x; v[i].y += a[i].y; v[i].z += a[i].z; v[i].w += a[i].w;
      xr[e] = v[i];
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; i++) {
    ss = fmaf(v[i].x, v[i].x, ss);
    ss = fmaf(v[i].y, v[i].y, ss);
    ss = fmaf(v[i].z, v[i].z, ss);
    ss = fmaf(v[i].w, v[i].w, ss);
  }
  ss = warp_sum(ss);
  __shared__ float wsum[32];
  int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) wsum[w] = ss;
  __syncthreads();
  if (w == 0) {
    float s2 = l < kNormThreads / 32 ? wsum[l] : 0.f;
    s2 = warp_sum(s2);
    if (l == 0) wsum[0] = s2;
  }
  __syncthreads();
  float inv = rsqrtf(wsum[0] / static_cast<float>(d) + eps);
  __half2 *o = reinterpret_cast<__half2 *>(out + static_cast<size_t>(r) * ld);
  if (qscale) {
    // a8: the normalized row in float32, its amax over the block, then codes rint(y / s) with s = amax / 127
    float am = 0.f;
#pragma unroll
    for (int i = 0; i < NV; i++) {
      int e = threadIdx.x + i * kNormThreads;
      if (e < nv) {
        float4 g = gr[e];
        v[i] = make_float4(v[i].x * inv * g.x, v[i].y * inv * g.y, v[i].z * inv * g.z, v[i].w * inv * g.w);
        am = fmaxf(am, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
      }
    }
    am = warp_max(am);
    __shared__ float wmax[32];
    if (l == 0) wmax[w] = am;
    __syncthreads();
    if (w == 0) {
      float m2 = l < kNormThreads / 32 ? wmax[l] : 0.f;
      m2 = warp_max(m2);
      if (l == 0) wmax[0] = m2;
    }
    __syncthreads();
    const float sc = act_scale_of(wmax[0]);
#pragma unroll
    for (int i = 0; i < NV; i++) {
      int e = threadIdx.x + i * kNormThreads;
      if (e < nv) {
        o[2 * e] = __floats2half2_rn(rintf(__fdiv_rn(v[i].x, sc)), rintf(__fdiv_rn(v[i].y, sc)));
        o[2 * e + 1] = __floats2half2_rn(rintf(__fdiv_rn(v[i].z, sc)), rintf(__fdiv_rn(v[i].w, sc)));
      }
    }
    if (threadIdx.x == 0) qscale[r] = sc;
  } else {
#pragma unroll
    for (int i = 0; i < NV; i++) {
      int e = threadIdx.x + i * kNormThreads;
      if (e < nv) {
        float4 g = gr[e];
        o[2 * e] = __floats2half2_rn(v[i].x * inv * g.x, v[i].y * inv * g.y);
        o[2 * e + 1] = __floats2half2_rn(v[i].z * inv * g.z, v[i].w * inv * g.w);
      }
    }
  }
  for (int e = d / 2 + threadIdx.x; e < ld / 2; e += kNormThreads) o[e] = __floats2half2_rn(0.f, 0.f);
}

// ----------------------------------------------------------------------------------------------------------------
// a8 activations of a GEMM input written by another kernel (attention output, SwiGLU output): one CTA per row, the
// row's amax, then codes rint(x / s) in place (f16 integers, exact), s = amax / 127 into scale[row].
constexpr int kQuantThreads = 256;

__global__ void __launch_bounds__(kQuantThreads) act_quant_kernel(__half *buf, int n, int ld, float *scale) {
  dep_wait();
  dep_launch();
  __half2 *row = reinterpret_cast<__half2 *>(buf + static_cast<size_t>(blockIdx.x) * ld);
  const int n2 = n / 2;
  float am = 0.f;
  for (int e = threadIdx.x; e < n2; e += kQuantThreads) {
    const float2 f = __half22float2(row[e]);
    am = fmaxf(am, fmaxf(fabsf(f.x), fabsf(f.y)));
  }
  am = warp_max(am);
  __shared__ float wmax[kQuantThreads / 32];
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) wmax[w] = am;
  __syncthreads();
  float m = l < kQuantThreads / 32 ? wmax[l] : 0.f;
  m = warp_max(m);
  const float sc = act_scale_of(m);
  for (int e = threadIdx.x; e < n2; e += kQuantThreads) {
    const float2 f = __half22float2(row[e]);
    row[e] = __floats2half2_rn(rintf(__fdiv_rn(f.x, sc)), rintf(__fdiv_rn(f.y, sc)));
  }
  if (threadIdx.x == 0) scale[blockIdx.x] = sc;
}

void launch_act_quant(__half *buf, int T, int n, int ld, float *scale, cudaStream_t s) {
  if (T <= 0) return;
  launch_pdl(act_quant_kernel, T, kQuantThreads, 0, s, buf, n, ld, scale);
}

void launch_rmsnorm(float *x, const int *rows, int n, const float *gain, float eps, int d, int ld, __half *out,
                    const float *part, int S, int pld, int T, const TpPeers *tp, int tp_buf,
                    unsigned long long tp_epoch, float *qscale, cudaStream_t s) {
  TpPeers none{};
  none.n = 1;
  if (n <= 0) return;
  // float4s per thread for a row of d: 1 (d <= 2048), 2 (d <= 4096) or 4 (d <= 8192)
  const int nvec = (d / 4 + kNormThreads - 1) / kNormThreads;
  const TpPeers &tpp = tp ? *tp : none;
  if (nvec <= 1)
    launch_pdl(rmsnorm_kernel<1>, n, kNormThreads, 0, s, x, rows, gain, eps, d, ld, out, part, S, pld, T, tpp, tp_buf,
               tp_epoch, qscale);
  else if (nvec == 2)
    launch_pdl(rmsnorm_kernel<2>, n, kNormThreads, 0, s, x, rows, gain, eps, d, ld, out, part, S, pld, T, tpp, tp_buf,
               tp_epoch, qscale);
  else
    launch_pdl(rmsnorm_kernel<kNormMaxVec>, n, kNormThreads, 0, s, x, rows, gain, eps, d, ld, out, part, S, pld, T,
               tpp, tp_buf, tp_epoch, qscale);
}

// ----------------------------------------------------------------------------------------------------------------
// RoPE and KV write. qkv [T, (H + 2 KVH) * dh] f32 (or its split-K partials) -> q [T, H, dh] f16 (rotated); K (rotated) and V -> the layer's
// pages. fp8 page mode: a page's exponent e (scale 2^e) is set by the row that is its first (row % 16 == 0) from that
// row's amax (the largest e with amax * 2^e <= 64, clamped to [-8, 15]); later rows of the page use it, also within
// the same step (a token recomputes its page's first row from this step's qkv).
__device__ int page_exp(float amax) {
  if (!(amax > 0.f) || !isfinite(amax)) return 0;
  int k;
  float m = frexpf(amax, &k);
  int e = 6 - k + (m == 0.5f ? 1 : 0);
  return min(max(e, -8), 15);
}

// the q/k/v projection output: the GEMM's rows, or its split-K partials summed in split order (from 0)
struct QkvSrc {
  const float *p;
  int S;            // 1: p is [T, ld]; > 1: p is [S, T, ld] partials
  int ld, T;
  __device__ float operator()(int t, int c) const {
    if (S == 1) return p[static_cast<size_t>(t) * ld + c];
    float v = 0.f;
    for (int s0 = 0; s0 < S; s0 += kSplitChunk) {
      float x[kSplitChunk];
#pragma unroll
      for (int j = 0; j < kSplitChunk; j++) x[j] = s0 + j < S ? p[(static_cast<size_t>(s0 + j) * T + t) * ld + c] : 0.f;
#pragma unroll
      for (int j = 0; j < kSplitChunk; j++)
        if (s0 + j < S) v += x[j];
    }
    return v;
  }
  // columns c, c + 1 (c even): one 8-byte load per split
  __device__ float2 pair(int t, int c) const {
    if (S == 1) return *reinterpret_cast<const float2 *>(p + static_cast<size_t>(t) * ld + c);
    float2 v = make_float2(0.f, 0.f);
    for (int s0 = 0; s0 < S; s0 += kSplitChunk) {
      float2 x[kSplitChunk];
#pragma unroll
      for (int j = 0; j < kSplitChunk; j++)
        x[j] = s0 + j < S ? *reinterpret_cast<const float2 *>(p + (static_cast<size_t>(s0 + j) * T + t) * ld + c)
                          : make_float2(0.f, 0.f);
#pragma unroll
      for (int j = 0; j < kSplitChunk; j++)
        if (s0 + j < S) {
          v.x += x[j].x;
          v.y += x[j].y;
        }
    }
    return v;
  }
  // columns c[i], c[i] + 1 (each even) for i < N: every column's 8-byte load of a chunk of splits issued together
  // (32 / N splits: 32 float2 in flight per thread), each column summed in split order as pair() does
  template <int N>
  __device__ void pairs(int t, const int (&c)[N], float2 (&v)[N]) const {
    if (S == 1) {
#pragma unroll
      for (int i = 0; i < N; i++) v[i] = *reinterpret_cast<const float2 *>(p + static_cast<size_t>(t) * ld + c[i]);
      return;
    }
    constexpr int CH = 32 / N;
#pragma unroll
    for (int i = 0; i < N; i++) v[i] = make_float2(0.f, 0.f);
    for (int s0 = 0; s0 < S; s0 += CH) {
      float2 x[CH][N];
#pragma unroll
      for (int jj = 0; jj < CH; jj++) {
        const float *row = p + (static_cast<size_t>(s0 + jj) * T + t) * ld;
#pragma unroll
        for (int i = 0; i < N; i++)
          x[jj][i] = s0 + jj < S ? *reinterpret_cast<const float2 *>(row + c[i]) : make_float2(0.f, 0.f);
      }
#pragma unroll
      for (int jj = 0; jj < CH; jj++)
        if (s0 + jj < S) {
#pragma unroll
          for (int i = 0; i < N; i++) {
            v[i].x += x[jj][i].x;
            v[i].y += x[jj][i].y;
          }
        }
    }
  }
};

// RoPE of one (even, odd) pair, rounded step by step (no contraction), so that every kernel site that rotates a row
// gets the same bits: the writer of a page's first row and the later rows of that page agree on its exponent
__device__ __forceinline__ float2 rot(float2 x, float2 c) {
  return make_float2(__fsub_rn(__fmul_rn(x.x, c.x), __fmul_rn(x.y, c.y)),
                     __fadd_rn(__fmul_rn(x.x, c.y), __fmul_rn(x.y, c.x)));
}

// amax of row t's (rotated) k or v head at columns c0..: a warp reads it again (a page's first row from another token)
template <int DH>
__device__ float head_amax(const QkvSrc &q, int t, int c0, const float2 *cs, bool rotate) {
  float m = 0.f;
  for (int i = threadIdx.x % 32; i < DH / 2; i += 32) {
    float2 v = q.pair(t, c0 + 2 * i);
    if (rotate) v = rot(v, cs[i]);
    m = fmaxf(m, fmaxf(fabsf(v.x), fabsf(v.y)));
  }
  return warp_max(m);
}

// One warp per (token, head): q heads are rotated into q (f16); kv heads are rotated (k) and written to the token's
// page row (f16, or e4m3 with the page's exponents). Every input of the warp is loaded before its first store.
template <int DH>
__global__ void rope_kv_kernel(PlanView pv, QkvSrc qs, int H, int KVH, const float2 *rope_tab, __half *q, void *kc,
                               void *vc, int8_t *exps, int kv_fp8, int page_scale) {
  dep_wait();
  dep_launch();
  constexpr int NP = DH / 64;   // (even, odd) pairs per lane: pair i = lane + 32 p
  const int t = blockIdx.x;
  const int hh = threadIdx.x / 32 + blockIdx.y * (blockDim.x / 32);  // head slot: [0, H) q heads, [H, H + KVH) kv
  if (hh >= H + KVH) return;
  const int lane = threadIdx.x % 32;
  const bool is_q = hh < H;
  const int h = hh - H;
  const int c0 = is_q ? hh * DH : (H + h) * DH, vcol = (H + KVH + h) * DH;
  const bool fp8_page = !is_q && kv_fp8 && page_scale;
  // plan entries, the head's q/k and v columns, the rotation table: all issued together
  const int pos = pv.rope_pos[t];
  const int r = is_q ? 0 : pv.kv_row[t];
  const int ft = fp8_page ? pv.first_tok[t] : -1;
  float2 x[NP], xv[NP], c[NP];
  if (is_q) {
    int cols[NP];
#pragma unroll
    for (int p = 0; p < NP; p++) cols[p] = c0 + 2 * (lane + 32 * p);
    qs.pairs<NP>(t, cols, x);
  } else {
    // the k and v columns in one gather
    int cols[2 * NP];
    float2 kv[2 * NP];
#pragma unroll
    for (int p = 0; p < NP; p++) {
      cols[p] = c0 + 2 * (lane + 32 * p);
      cols[NP + p] = vcol + 2 * (lane + 32 * p);
    }
    qs.pairs<2 * NP>(t, cols, kv);
#pragma unroll
    for (int p = 0; p < NP; p++) {
      x[p] = kv[p];
      xv[p] = kv[NP + p];
    }
  }
  const float2 *cs = rope_tab + static_cast<size_t>(pos) * (DH / 2);
#pragma unroll
  for (int p = 0; p < NP; p++) c[p] = cs[lane + 32 * p];
#pragma unroll
  for (int p = 0; p < NP; p++) x[p] = rot(x[p], c[p]);
  if (is_q) {
    __half2 *dst = reinterpret_cast<__half2 *>(q + (static_cast<size_t>(t) * H + hh) * DH);
#pragma unroll
    for (int p = 0; p < NP; p++) dst[lane + 32 * p] = __floats2half2_rn(x[p].x, x[p].y);
    return;
  }
  const int blk = r / kBlock, rip = r % kBlock;
  const size_t off = ((static_cast<size_t>(blk) * KVH + h) * kBlock + rip) * DH;
  if (!kv_fp8) {
    __half2 *kd = reinterpret_cast<__half2 *>(static_cast<__half *>(kc) + off);
    __half2 *vd = reinterpret_cast<__half2 *>(static_cast<__half *>(vc) + off);
#pragma unroll
    for (int p = 0; p < NP; p++) {
      kd[lane + 32 * p] = __floats2half2_rn(x[p].x, x[p].y);
      vd[lane + 32 * p] = __floats2half2_rn(xv[p].x, xv[p].y);
    }
    return;
  }
  int ek = 0, ev = 0;
  if (page_scale) {
    int8_t *pe = exps + (static_cast<size_t>(blk) * KVH + h) * 2;
    if (ft == t) {
      // this token's row is its page's first: the exponents come from its own rotated k and its v
      float mk = 0.f, mv = 0.f;
#pragma unroll
      for (int p = 0; p < NP; p++) {
        mk = fmaxf(mk, fmaxf(fabsf(x[p].x), fabsf(x[p].y)));
        mv = fmaxf(mv, fmaxf(fabsf(xv[p].x), fabsf(xv[p].y)));
      }
      ek = page_exp(warp_max(mk));
      ev = page_exp(warp_max(mv));
      if (lane == 0) { pe[0] = static_cast<int8_t>(ek); pe[1] = static_cast<int8_t>(ev); }
    } else if (ft >= 0) {
      // the page's first row is written in this step by token ft: derive its exponents from that row
      const float2 *fcs = rope_tab + static_cast<size_t>(pv.rope_pos[ft]) * (DH / 2);
      ek = page_exp(head_amax<DH>(qs, ft, c0, fcs, true));
      ev = page_exp(head_amax<DH>(qs, ft, vcol, fcs, false));
    } else {
      ek = pe[0];
      ev = pe[1];
    }
  }
  const float sk = exp2f(static_cast<float>(ek)), sv = exp2f(static_cast<float>(ev));
  uint16_t *kd = reinterpret_cast<uint16_t *>(static_cast<uint8_t *>(kc) + off);
  uint16_t *vd = reinterpret_cast<uint16_t *>(static_cast<uint8_t *>(vc) + off);
#pragma unroll
  for (int p = 0; p < NP; p++) {
    const int i = lane + 32 * p;
    kd[i] = static_cast<uint16_t>(f32_to_e4m3(x[p].x * sk) | (f32_to_e4m3(x[p].y * sk) << 8));
    vd[i] = static_cast<uint16_t>(f32_to_e4m3(xv[p].x * sv) | (f32_to_e4m3(xv[p].y * sv) << 8));
  }
}

void launch_rope_kv(const PlanView &pv, const float *qkv, int S, int ld, int H, int KVH, int dh,
                    const float2 *rope_tab, __half *q, void *kc, void *vc, int8_t *exps, int kv_fp8, int page_scale,
                    cudaStream_t s) {
  int heads = H + KVH, per = 8;
  dim3 grid(pv.T, (heads + per - 1) / per);
  QkvSrc qs{qkv, S, ld, pv.T};
  if (dh == 128)
    launch_pdl(rope_kv_kernel<128>, grid, per * 32, 0, s, pv, qs, H, KVH, rope_tab, q, kc, vc, exps, kv_fp8, page_scale);
  else
    launch_pdl(rope_kv_kernel<64>, grid, per * 32, 0, s, pv, qs, H, KVH, rope_tab, q, kc, vc, exps, kv_fp8, page_scale);
}

// ----------------------------------------------------------------------------------------------------------------
// Split-K reduction: v = sum_{s=0..S-1} part[s, t, n] in that order, then the epilogue.

__global__ void splitk_reduce_kernel(const float *part, int S, int T, int Npad, Epi epi) {
  dep_wait();
  dep_launch();
  size_t total = static_cast<size_t>(T) * (epi.kind == kEpiSwiGLU ? Npad / 8 : Npad);
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    if (epi.kind == kEpiSwiGLU) {
      // four consecutive features per thread: gate and up rows alternate (row 2i of a 128-row tile is gate feature
      // tile * 64 + i, row 2i + 1 its up row), so two float4 loads hold the four (gate, up) pairs
      int q4 = Npad / 2 / 4;
      int t = static_cast<int>(i / q4), f = static_cast<int>(i % q4) * 4;
      int tile = f / 64, w = f % 64;
      int n0 = tile * 128 + 2 * w;
      float4 g = make_float4(0.f, 0.f, 0.f, 0.f), u = g;
      for (int s0 = 0; s0 < S; s0 += kSplitChunk) {
        float4 a[kSplitChunk], b[kSplitChunk];
#pragma unroll
        for (int j = 0; j < kSplitChunk; j++) {
          const float *row = part + (static_cast<size_t>(s0 + j) * T + t) * Npad;
          a[j] = s0 + j < S ? *reinterpret_cast<const float4 *>(row + n0) : make_float4(0.f, 0.f, 0.f, 0.f);
          b[j] = s0 + j < S ? *reinterpret_cast<const float4 *>(row + n0 + 4) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int j = 0; j < kSplitChunk; j++) {
          if (s0 + j >= S) break;
          g.x += a[j].x; u.x += a[j].y; g.y += a[j].z; u.y += a[j].w;
          g.z += b[j].x; u.z += b[j].y; g.w += b[j].z; u.w += b[j].w;
        }
      }
      __half *o = epi.out_h + static_cast<size_t>(t) * epi.ld + f;
      if (f < epi.n) o[0] = __float2half_rn(silu_mul(g.x, u.x));
      if (f + 1 < epi.n) o[1] = __float2half_rn(silu_mul(g.y, u.y));
      if (f + 2 < epi.n) o[2] = __float2half_rn(silu_mul(g.z, u.z));
      if (f + 3 < epi.n) o[3] = __float2half_rn(silu_mul(g.w, u.w));
    } else {
      int t = static_cast<int>(i / Npad), n = static_cast<int>(i % Npad);
      if (n >= epi.n) continue;
      float v = 0.f;
      for (int s0 = 0; s0 < S; s0 += kSplitChunk) {
        float x[kSplitChunk];
#pragma unroll
        for (int j = 0; j < kSplitChunk; j++) x[j] = s0 + j < S ? part[(static_cast<size_t>(s0 + j) * T + t) * Npad + n] : 0.f;
#pragma unroll
        for (int j = 0; j < kSplitChunk; j++)
          if (s0 + j < S) v += x[j];
      }
      float *o = epi.out_f + static_cast<size_t>(t) * epi.ld + n;
      if (epi.kind == kEpiAdd) *o += v;
      else *o = v;
    }
  }
}

void launch_splitk_reduce(const float *part, int S, int T, int Npad, const Epi &epi, cudaStream_t s) {
  size_t total = static_cast<size_t>(T) * Npad;
  int blocks = static_cast<int>((total + 255) / 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  launch_pdl(splitk_reduce_kernel, blocks, 256, 0, s, part, S, T, Npad, epi);
}

// ----------------------------------------------------------------------------------------------------------------
// argmax per row, first index of the maximum (torch.argmax); NaN never wins. With pick (a tensor-parallel rank's
// vocabulary slice starting at row `offset`): the candidate (value bits, global index) instead of the index.
__global__ void argmax_kernel(const float *logits, int V, int *out, int *pick, int offset) {
  dep_wait();
  dep_launch();
  int r = blockIdx.x;
  const float *row = logits + static_cast<size_t>(r) * V;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  for (int v = threadIdx.x; v < V; v += blockDim.x) {
    float x = row[v];
    if (x > best) { best = x; idx = v; }
  }
  for (int o = 16; o > 0; o >>= 1) {
    float b2 = __shfl_xor_sync(0xffffffffu, best, o);
    int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
    if (b2 > best || (b2 == best && i2 < idx)) { best = b2; idx = i2; }
  }
  __shared__ float sb[32];
  __shared__ int si[32];
  int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) { sb[w] = best; si[w] = idx; }
  __syncthreads();
  if (w == 0) {
    best = l < blockDim.x / 32 ? sb[l] : -INFINITY;
    idx = l < blockDim.x / 32 ? si[l] : 0x7fffffff;
    for (int o = 16; o > 0; o >>= 1) {
      float b2 = __shfl_xor_sync(0xffffffffu, best, o);
      int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
      if (b2 > best || (b2 == best && i2 < idx)) { best = b2; idx = i2; }
    }
    if (l == 0) {
      if (pick) {
        pick[2 * r] = __float_as_int(best);
        pick[2 * r + 1] = idx == 0x7fffffff ? idx : idx + offset;
      } else {
        out[r] = idx == 0x7fffffff ? 0 : idx;
      }
    }
  }
}

// the ranks' candidates [tp][R][2] -> the first index of the maximum over the whole vocabulary (slices ascend by rank)
__global__ void argmax_merge_kernel(const int *pick, int tp, int R, int *out) {
  dep_wait();
  dep_launch();
  int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= R) return;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  for (int k = 0; k < tp; k++) {
    float v = __int_as_float(pick[(static_cast<size_t>(k) * R + r) * 2]);
    int i = pick[(static_cast<size_t>(k) * R + r) * 2 + 1];
    if (i != 0x7fffffff && (v > best || (v == best && i < idx))) { best = v; idx = i; }
  }
  out[r] = idx == 0x7fffffff ? 0 : idx;
}

// a row's argmax in kArgChunks parts (one CTA each), then the first maximum of the parts (parts ascend in index)
constexpr int kArgChunks = 8;
__global__ void argmax_part_kernel(const float *logits, int V, int *pick) {
  dep_wait();
  dep_launch();
  const int r = blockIdx.x, c = blockIdx.y;
  const int per = (V + kArgChunks - 1) / kArgChunks;
  const int v0 = c * per, v1 = min(V, v0 + per);
  const float *row = logits + static_cast<size_t>(r) * V;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  for (int v = v0 + threadIdx.x; v < v1; v += blockDim.x) {
    float x = row[v];
    if (x > best) { best = x; idx = v; }
  }
  for (int o = 16; o > 0; o >>= 1) {
    float b2 = __shfl_xor_sync(0xffffffffu, best, o);
    int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
    if (b2 > best || (b2 == best && i2 < idx)) { best = b2; idx = i2; }
  }
  __shared__ float sb[32];
  __shared__ int si[32];
  int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) { sb[w] = best; si[w] = idx; }
  __syncthreads();
  if (w == 0) {
    best = l < blockDim.x / 32 ? sb[l] : -INFINITY;
    idx = l < blockDim.x / 32 ? si[l] : 0x7fffffff;
    for (int o = 16; o > 0; o >>= 1) {
      float b2 = __shfl_xor_sync(0xffffffffu, best, o);
      int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
      if (b2 > best || (b2 == best && i2 < idx)) { best = b2; idx = i2; }
    }
    if (l == 0) {
      pick[(static_cast<size_t>(c) * gridDim.x + r) * 2] = __float_as_int(best);
      pick[(static_cast<size_t>(c) * gridDim.x + r) * 2 + 1] = idx;
    }
  }
}

__global__ void table_patch_kernel(const uint2 *patches, int n, uint32_t *tables) {
  dep_wait();
  dep_launch();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) tables[patches[i].x] = patches[i].y;
}

void launch_table_patch(const uint2 *patches, int n, uint32_t *tables, cudaStream_t s) {
  if (n > 0) launch_pdl(table_patch_kernel, std::min((n + 255) / 256, 148), 256, 0, s, patches, n, tables);
}

__global__ void spec_accept_kernel(const int *chain, const int *target, int K, int *out) {
  dep_wait();
  if (threadIdx.x != 0) return;
  int j = 0;
  while (j < K && chain[j + 1] == target[j]) j++;
  for (int i = 0; i <= j; i++) out[i] = target[i];
  out[K + 1] = j + 1;
}

void launch_spec_accept(const int *chain, const int *target, int K, int *out, cudaStream_t s) {
  launch_pdl(spec_accept_kernel, 1, 32, 0, s, chain, target, K, out);
}

void launch_argmax_merge(const int *pick, int tp, int R, int *out, cudaStream_t s);
void launch_argmax(const float *logits, int R, int V, int *out, int *scratch, cudaStream_t s) {
  if (R <= 0) return;
  launch_pdl(argmax_part_kernel, dim3(R, kArgChunks), 512, 0, s, logits, V, scratch);
  launch_argmax_merge(scratch, kArgChunks, R, out, s);
}
void launch_argmax_pick(const float *logits, int R, int V, int offset, int *pick, cudaStream_t s) {
  if (R > 0) launch_pdl(argmax_kernel, R, 1024, 0, s, logits, V, static_cast<int *>(nullptr), pick, offset);
}
void launch_argmax_merge(const int *pick, int tp, int R, int *out, cudaStream_t s) {
  if (R > 0) launch_pdl(argmax_merge_kernel, (R + 127) / 128, 128, 0, s, pick, tp, R, out);
}

// ----------------------------------------------------------------------------------------------------------------
// gc_copy_blocks: page src -> dst for every layer, K and V, and the fp8 page exponents. pairs: [n][2] (src, dst).
__global__ void copy_blocks_kernel(const int *pairs, size_t page_bytes, size_t layer_bytes, uint8_t *kc, uint8_t *vc,
                                   int8_t *exps, size_t exps_layer, int exps_per_block) {
  int p = blockIdx.x, l = blockIdx.y;
  int src = pairs[2 * p], dst = pairs[2 * p + 1];
  const uint4 *ks = reinterpret_cast<const uint4 *>(kc + l * layer_bytes + src * page_bytes);
  uint4 *kd = reinterpret_cast<uint4 *>(kc + l * layer_bytes + dst * page_bytes);
  const uint4 *vs = reinterpret_cast<const uint4 *>(vc + l * layer_bytes + src * page_bytes);
  uint4 *vd = reinterpret_cast<uint4 *>(vc + l * layer_bytes + dst * page_bytes);
  for (size_t i = threadIdx.x; i < page_bytes / 16; i += blockDim.x) { kd[i] = ks[i]; vd[i] = vs[i]; }
  if (exps && threadIdx.x < exps_per_block)
    exps[l * exps_layer + static_cast<size_t>(dst) * exps_per_block + threadIdx.x] =
        exps[l * exps_layer + static_cast<size_t>(src) * exps_per_block + threadIdx.x];
}

void launch_copy_blocks(const int *pairs, int n, int L, size_t page_bytes, size_t layer_bytes, uint8_t *kc,
                        uint8_t *vc, int8_t *exps, size_t exps_layer, int exps_per_block, cudaStream_t s) {
  if (n > 0) copy_blocks_kernel<<<dim3(n, L), 256, 0, s>>>(pairs, page_bytes, layer_bytes, kc, vc, exps, exps_layer,
                                                            exps_per_block);
}

// ----------------------------------------------------------------------------------------------------------------
// gc_commit: moves[m] = (src row, dst row). Phase 1 copies every source row (all layers, heads, K and V) to tmp as
// decoded f32; phase 2 sets the exponents of pages whose first row is a destination (fp8 page mode); phase 3 writes
// every destination. Reading all sources first makes overlapping moves (a destination that is another move's source)
// behave like the reference's in-order loop, since destinations never lie after their own source.
template <typename KV>
__device__ float kv_load(const KV *p, size_t i, float inv);
template <>
__device__ float kv_load<__half>(const __half *p, size_t i, float) { return __half2float(p[i]); }
template <>
__device__ float kv_load<uint8_t>(const uint8_t *p, size_t i, float inv) { return e4m3_to_f32(p[i]) * inv; }

__global__ void commit_gather_kernel(const int *moves, int L, int KVH, int dh, const uint8_t *kc, const uint8_t *vc,
                                     const int8_t *exps, int kv_fp8, size_t layer_bytes, size_t exps_layer,
                                     float *tmp) {
  int m = blockIdx.x, l = blockIdx.y;
  int src = moves[2 * m];
  int blk = src / kBlock, rip = src % kBlock;
  for (int i = threadIdx.x; i < KVH * dh; i += blockDim.x) {
    int h = i / dh, e = i % dh;
    size_t off = ((static_cast<size_t>(blk) * KVH + h) * kBlock + rip) * dh + e;
    float kv, vv;
    if (kv_fp8) {
      float ik = 1.f, iv = 1.f;
      if (exps) {
        const int8_t *pe = exps + l * exps_layer + (static_cast<size_t>(blk) * KVH + h) * 2;
        ik = exp2f(-static_cast<float>(pe[0]));
        iv = exp2f(-static_cast<float>(pe[1]));
      }
      kv = kv_load<uint8_t>(kc + l * layer_bytes, off, ik);
      vv = kv_load<uint8_t>(vc + l * layer_bytes, off, iv);
    } else {
      kv = kv_load<__half>(reinterpret_cast<const __half *>(kc + l * layer_bytes), off, 1.f);
      vv = kv_load<__half>(reinterpret_cast<const __half *>(vc + l * layer_bytes), off, 1.f);
    }
    float *o = tmp + ((static_cast<size_t>(m) * L + l) * 2) * KVH * dh;
    o[i] = kv;
    o[KVH * dh + i] = vv;
  }
}

__global__ void commit_exps_kernel(const int *moves, int L, int KVH, int dh, int8_t *exps, size_t exps_layer,
                                   const float *tmp) {
  int m = blockIdx.x, l = blockIdx.y;
  int dst = moves[2 * m + 1];
  if (dst % kBlock) return;
  int blk = dst / kBlock;
  int h = threadIdx.x / 32;
  if (h >= KVH) return;
  const float *o = tmp + ((static_cast<size_t>(m) * L + l) * 2) * KVH * dh;
  float ak = 0.f, av = 0.f;
  for (int e = threadIdx.x % 32; e < dh; e += 32) {
    ak = fmaxf(ak, fabsf(o[h * dh + e]));
    av = fmaxf(av, fabsf(o[KVH * dh + h * dh + e]));
  }
  ak = warp_max(ak);
  av = warp_max(av);
  if (threadIdx.x % 32 == 0) {
    int8_t *pe = exps + l * exps_layer + (static_cast<size_t>(blk) * KVH + h) * 2;
    pe[0] = static_cast<int8_t>(page_exp(ak));
    pe[1] = static_cast<int8_t>(page_exp(av));
  }
}

__global__ void commit_scatter_kernel(const int *moves, int L, int KVH, int dh, uint8_t *kc, uint8_t *vc,
                                      const int8_t *exps, int kv_fp8, size_t layer_bytes, size_t exps_layer,
                                      const float *tmp) {
  int m = blockIdx.x, l = blockIdx.y;
  int dst = moves[2 * m + 1];
  int blk = dst / kBlock, rip = dst % kBlock;
  const float *o = tmp + ((static_cast<size_t>(m) * L + l) * 2) * KVH * dh;
  for (int i = threadIdx.x; i < KVH * dh; i += blockDim.x) {
    int h = i / dh, e = i % dh;
    size_t off = ((static_cast<size_t>(blk) * KVH + h) * kBlock + rip) * dh + e;
    if (kv_fp8) {
      float sk = 1.f, sv = 1.f;
      if (exps) {
        const int8_t *pe = exps + l * exps_layer + (static_cast<size_t>(blk) * KVH + h) * 2;
        sk = exp2f(static_cast<float>(pe[0]));
        sv = exp2f(static_cast<float>(pe[1]));
      }
      kc[l * layer_bytes + off] = f32_to_e4m3(o[i] * sk);
      vc[l * layer_bytes + off] = f32_to_e4m3(o[KVH * dh + i] * sv);
    } else {
      reinterpret_cast<__half *>(kc + l * layer_bytes)[off] = __float2half_rn(o[i]);
      reinterpret_cast<__half *>(vc + l * layer_bytes)[off] = __float2half_rn(o[KVH * dh + i]);
    }
  }
}

void launch_commit(const int *moves, int n, int L, int KVH, int dh, uint8_t *kc, uint8_t *vc, int8_t *exps,
                   int kv_fp8, size_t layer_bytes, size_t exps_layer, float *tmp, cudaStream_t s) {
  if (n <= 0) return;
  dim3 g(n, L);
  commit_gather_kernel<<<g, 256, 0, s>>>(moves, L, KVH, dh, kc, vc, exps, kv_fp8, layer_bytes, exps_layer, tmp);
  if (kv_fp8 && exps) commit_exps_kernel<<<g, 32 * KVH, 0, s>>>(moves, L, KVH, dh, exps, exps_layer, tmp);
  commit_scatter_kernel<<<g, 256, 0, s>>>(moves, L, KVH, dh, kc, vc, exps, kv_fp8, layer_bytes, exps_layer, tmp);
}

}  // namespace gck
