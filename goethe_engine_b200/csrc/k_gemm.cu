// Quantized weight GEMM, tensor-core path on mma.sync (m16n8k16, f16 x f16 -> f32).
//
//   y[t, n] = sum_k act[t, k] * W[n, k]        (the reference's `w @ h`, ref.py:51-59, for every token row at once)
//
// W is stored in tiles of kBM = 128 rows x kBK = 256 columns (weights.cpp relays GGUF Q8_0 / Q4_K / F16 rows into
// them). A CTA owns one 128-row tile band and a range of K tiles (split-K), and 64 token rows; per K tile it
// prefetches the next raw tile and activation tile with cp.async while it dequantizes the current one into shared
// memory (f32 math, one rounding to f16) and runs the MMAs. Every output element is reduced over K in the same order
// whatever the number of tokens (the split count is fixed per weight), so a row is bit-identical alone or batched.
#include "common.cuh"
#include "kernels.h"

namespace gck {

namespace {

constexpr int kThreads = 256;
constexpr int kLdA = kBK + 8;   // padded smem row (halves): conflict-free ldmatrix
constexpr int kSA = kBM * kLdA * 2;
constexpr int kSB = kBN * kLdA * 2;

__device__ __forceinline__ void q4k_scale_min(const uint8_t *s, int j, int &sc, int &m) {
  if (j < 4) {
    sc = s[j] & 63;
    m = s[j + 4] & 63;
  } else {
    sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
    m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

// raw tile (smem) -> sA f16 [128][kLdA]; thread = (row, half of the 256 columns)
template <int TYPE>
__device__ void dequant_tile(const uint8_t *raw, __half *sA) {
  int r = threadIdx.x >> 1, hf = threadIdx.x & 1;
  __half *dst = sA + r * kLdA + hf * 128;
  if (TYPE == kQ4_K) {
    const uint8_t *hdr = raw + r * 16;
    float d = __half2float(*reinterpret_cast<const __half *>(hdr));
    float dm = __half2float(*reinterpret_cast<const __half *>(hdr + 2));
    const uint8_t *qs = raw + kBM * 16 + r * 128 + hf * 64;
#pragma unroll
    for (int cc = 0; cc < 2; cc++) {
      int c = 2 * hf + cc;
      int sc0, m0, sc1, m1;
      q4k_scale_min(hdr + 4, 2 * c, sc0, m0);
      q4k_scale_min(hdr + 4, 2 * c + 1, sc1, m1);
      float s0 = d * static_cast<float>(sc0), o0 = dm * static_cast<float>(m0);
      float s1 = d * static_cast<float>(sc1), o1 = dm * static_cast<float>(m1);
      const uint4 *q4 = reinterpret_cast<const uint4 *>(qs + cc * 32);
#pragma unroll
      for (int v = 0; v < 2; v++) {
        uint4 u = q4[v];
        uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int b = 0; b < 16; b += 2) {
          uint32_t x0 = (w[b / 4] >> (8 * (b % 4))) & 0xff, x1 = (w[b / 4] >> (8 * (b % 4 + 1))) & 0xff;
          int l = v * 16 + b;
          *reinterpret_cast<__half2 *>(dst + cc * 64 + l) =
              __floats2half2_rn(fmaf(s0, static_cast<float>(x0 & 15), -o0), fmaf(s0, static_cast<float>(x1 & 15), -o0));
          *reinterpret_cast<__half2 *>(dst + cc * 64 + 32 + l) =
              __floats2half2_rn(fmaf(s1, static_cast<float>(x0 >> 4), -o1), fmaf(s1, static_cast<float>(x1 >> 4), -o1));
        }
      }
    }
  } else {  // Q8_0
    const __half *ds = reinterpret_cast<const __half *>(raw) + r * 8 + hf * 4;
    const uint8_t *qs = raw + kBM * 16 + r * 256 + hf * 128;
#pragma unroll
    for (int b = 0; b < 4; b++) {
      float d = __half2float(ds[b]);
      const uint4 *q4 = reinterpret_cast<const uint4 *>(qs + b * 32);
#pragma unroll
      for (int v = 0; v < 2; v++) {
        uint4 u = q4[v];
        uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 16; e += 2) {
          int8_t a0 = static_cast<int8_t>((w[e / 4] >> (8 * (e % 4))) & 0xff);
          int8_t a1 = static_cast<int8_t>((w[e / 4] >> (8 * (e % 4 + 1))) & 0xff);
          *reinterpret_cast<__half2 *>(dst + b * 32 + v * 16 + e) =
              __floats2half2_rn(d * static_cast<float>(a0), d * static_cast<float>(a1));
        }
      }
    }
  }
}

template <int TYPE>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const uint8_t *__restrict__ W, int KT, int splits, const __half *__restrict__ act, int T, Epi epi,
                float *part, int Npad) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tb = static_cast<int>(TYPE == kF16 ? 0 : tile_bytes(TYPE));
  __half *sA = reinterpret_cast<__half *>(smem);
  __half *sB0 = reinterpret_cast<__half *>(smem + kSA);
  uint8_t *raw0 = smem + kSA + 2 * kSB;

  const int nt = blockIdx.x, split = blockIdx.y, t0 = blockIdx.z * kBN;
  const int per = KT / splits, kt0 = split * per, kt1 = kt0 + per;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int wm = warp % 4, wn = warp / 4;
  const size_t tileB = TYPE == kF16 ? static_cast<size_t>(kBM) * kBK * 2 : tile_bytes(TYPE);
  const int Kpad = KT * kBK;

  auto load_stage = [&](int kt, int buf) {
    // activations: 64 rows x 256 halves
    __half *sB = sB0 + buf * (kSB / 2);
    for (int c = tid; c < kBN * (kBK / 8); c += kThreads) {
      int row = c / (kBK / 8), col = (c % (kBK / 8)) * 8;
      int t = t0 + row;
      const __half *src = act + static_cast<size_t>(t < T ? t : 0) * Kpad + kt * kBK + col;
      cp_async16_pred(sB + row * kLdA + col, src, t < T);
    }
    const uint8_t *src = W + (static_cast<size_t>(nt) * KT + kt) * tileB;
    if (TYPE == kF16) {
      for (int c = tid; c < kBM * (kBK / 8); c += kThreads) {
        int row = c / (kBK / 8), col = (c % (kBK / 8)) * 8;
        cp_async16(sA + row * kLdA + col, src + (static_cast<size_t>(row) * kBK + col) * 2);
      }
    } else {
      uint8_t *dst = raw0 + buf * tb;
      for (int c = tid; c < tb / 16; c += kThreads) cp_async16(dst + c * 16, src + c * 16);
    }
    cp_async_commit();
  };

  float acc[2][4][4];
#pragma unroll
  for (int i = 0; i < 2; i++)
#pragma unroll
    for (int j = 0; j < 4; j++)
#pragma unroll
      for (int k = 0; k < 4; k++) acc[i][j][k] = 0.f;

  if (TYPE != kF16) load_stage(kt0, 0);
  for (int kt = kt0; kt < kt1; kt++) {
    int buf = (kt - kt0) & 1;
    if (TYPE == kF16) {
      load_stage(kt, 0);
      cp_async_wait<0>();
    } else if (kt + 1 < kt1) {
      load_stage(kt + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (TYPE != kF16) {
      dequant_tile<TYPE>(raw0 + buf * tb, sA);
      __syncthreads();
    }
    const __half *sB = sB0 + (TYPE == kF16 ? 0 : buf) * (kSB / 2);
#pragma unroll 4
    for (int kk = 0; kk < kBK / 16; kk++) {
      uint32_t a[2][4], b[4][2];
#pragma unroll
      for (int mt = 0; mt < 2; mt++) {
        const __half *p = sA + (wm * 32 + mt * 16 + (lane % 16)) * kLdA + kk * 16 + (lane / 16) * 8;
        ldmatrix_x4(a[mt][0], a[mt][1], a[mt][2], a[mt][3], p);
      }
#pragma unroll
      for (int np = 0; np < 2; np++) {
        const __half *p = sB + (wn * 32 + np * 16 + (lane / 16) * 8 + (lane % 8)) * kLdA + kk * 16 + ((lane / 8) % 2) * 8;
        ldmatrix_x4(b[2 * np][0], b[2 * np][1], b[2 * np + 1][0], b[2 * np + 1][1], p);
      }
#pragma unroll
      for (int mt = 0; mt < 2; mt++)
#pragma unroll
        for (int j = 0; j < 4; j++) mma_f16(acc[mt][j], a[mt], b[j]);
    }
    __syncthreads();
  }

  const int g = lane / 4, tq = lane % 4;
  if (splits > 1) {
    float *p = part + static_cast<size_t>(split) * T * Npad;
#pragma unroll
    for (int mt = 0; mt < 2; mt++)
#pragma unroll
      for (int j = 0; j < 4; j++)
#pragma unroll
        for (int e = 0; e < 4; e++) {
          int row = nt * kBM + wm * 32 + mt * 16 + g + (e / 2) * 8;
          int t = t0 + wn * 32 + j * 8 + 2 * tq + (e % 2);
          if (t < T) p[static_cast<size_t>(t) * Npad + row] = acc[mt][j][e];
        }
    return;
  }
  if (epi.kind == kEpiSwiGLU) {
    // gate rows 0..63 and up rows 64..127 of the tile meet in shared memory
    float *sC = reinterpret_cast<float *>(smem);  // [128][kBN + 1]
#pragma unroll
    for (int mt = 0; mt < 2; mt++)
#pragma unroll
      for (int j = 0; j < 4; j++)
#pragma unroll
        for (int e = 0; e < 4; e++) {
          int row = wm * 32 + mt * 16 + g + (e / 2) * 8;
          int col = wn * 32 + j * 8 + 2 * tq + (e % 2);
          sC[row * (kBN + 1) + col] = acc[mt][j][e];
        }
    __syncthreads();
    for (int i = tid; i < 64 * kBN; i += kThreads) {
      int f = i % 64, c = i / 64;
      int t = t0 + c, feat = nt * 64 + f;
      if (t < T && feat < epi.n) {
        float gg = sC[f * (kBN + 1) + c], uu = sC[(64 + f) * (kBN + 1) + c];
        epi.out_h[static_cast<size_t>(t) * epi.ld + feat] = __float2half_rn(gg / (1.f + expf(-gg)) * uu);
      }
    }
    return;
  }
#pragma unroll
  for (int mt = 0; mt < 2; mt++)
#pragma unroll
    for (int j = 0; j < 4; j++)
#pragma unroll
      for (int e = 0; e < 4; e++) {
        int n = nt * kBM + wm * 32 + mt * 16 + g + (e / 2) * 8;
        int t = t0 + wn * 32 + j * 8 + 2 * tq + (e % 2);
        if (t < T && n < epi.n) {
          float *o = epi.out_f + static_cast<size_t>(t) * epi.ld + n;
          if (epi.kind == kEpiAdd) *o += acc[mt][j][e];
          else *o = acc[mt][j][e];
        }
      }
}

template <int TYPE>
size_t smem_bytes() {
  return TYPE == kF16 ? kSA + kSB : kSA + 2 * kSB + 2 * tile_bytes(TYPE);
}

template <int TYPE>
void launch_t(const QWeight &w, const __half *act, int T, const Epi &epi, float *part, cudaStream_t s) {
  size_t sm = smem_bytes<TYPE>();
  dim3 grid(w.NT, w.splits, (T + kBN - 1) / kBN);
  gemm_kernel<TYPE><<<grid, kThreads, sm, s>>>(w.data, w.KT, w.splits, act, T, epi, part, w.NT * kBM);
}

}  // namespace

void gemm_init() {
  cudaFuncSetAttribute(gemm_kernel<kQ4_K>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem_bytes<kQ4_K>()));
  cudaFuncSetAttribute(gemm_kernel<kQ8_0>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem_bytes<kQ8_0>()));
  cudaFuncSetAttribute(gemm_kernel<kF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem_bytes<kF16>()));
}

void launch_gemm(const QWeight &w, const __half *act, int T, const Epi &epi, float *part, cudaStream_t s) {
  if (T <= 0) return;
  switch (w.type) {
    case kQ4_K: launch_t<kQ4_K>(w, act, T, epi, part, s); break;
    case kQ8_0: launch_t<kQ8_0>(w, act, T, epi, part, s); break;
    default: launch_t<kF16>(w, act, T, epi, part, s); break;
  }
  if (w.splits > 1) launch_splitk_reduce(part, w.splits, T, w.NT * kBM, epi, s);
}

}  // namespace gck
