// F16 weight GEMM on mma.sync (m16n8k16, f16 x f16 -> f32): the path of unquantized (F16/F32) checkpoints;
// quantized weights (Q4_K, Q8_0) run on the tcgen05 kernel of k_gemm_tc.cu.
//
//   y[t, n] = sum_k act[t, k] * W[n, k]        (the reference's `w @ h`, ref.py:51-59, for every token row at once)
//
// W is stored in tiles of kBM = 128 rows x kBK = 256 columns of f16 (runtime.cu relays the GGUF rows into them). A
// CTA owns one 128-row tile band, a range of K tiles (split-K) and 64 token rows, and loads each K tile of weights and
// activations with cp.async before its MMAs. Every output element is reduced over K in the same order whatever the
// number of tokens (the split count is fixed per weight), so a row is bit-identical alone or batched.
#include "common.cuh"
#include "kernels.h"

namespace gck {

namespace {

constexpr int kThreads = 256;
constexpr int kLdA = kBK + 8;   // padded smem row (halves): conflict-free ldmatrix
constexpr int kSA = kBM * kLdA * 2;
constexpr int kSB = kBN * kLdA * 2;

template <int TYPE>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const uint8_t *__restrict__ W, int KT, int splits, const __half *__restrict__ act, int T, Epi epi,
                float *part, int Npad) {
  static_assert(TYPE == kF16, "quantized weights run on the tcgen05 kernel");
  dep_wait();
  dep_launch();
  extern __shared__ __align__(128) uint8_t smem[];
  __half *sA = reinterpret_cast<__half *>(smem);
  __half *sB = reinterpret_cast<__half *>(smem + kSA);

  const int nt = blockIdx.x, split = blockIdx.y, t0 = blockIdx.z * kBN;
  const int per = KT / splits, kt0 = split * per, kt1 = kt0 + per;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int wm = warp % 4, wn = warp / 4;
  const size_t tileB = static_cast<size_t>(kBM) * kBK * 2;
  const int Kpad = KT * kBK;

  float acc[2][4][4];
#pragma unroll
  for (int i = 0; i < 2; i++)
#pragma unroll
    for (int j = 0; j < 4; j++)
#pragma unroll
      for (int k = 0; k < 4; k++) acc[i][j][k] = 0.f;

  for (int kt = kt0; kt < kt1; kt++) {
    // activations: 64 rows x 256 halves (rows past T read as zeros); weights: 128 rows x 256 halves
    for (int c = tid; c < kBN * (kBK / 8); c += kThreads) {
      int row = c / (kBK / 8), col = (c % (kBK / 8)) * 8;
      int t = t0 + row;
      const __half *src = act + static_cast<size_t>(t < T ? t : 0) * Kpad + kt * kBK + col;
      cp_async16_pred(sB + row * kLdA + col, src, t < T);
    }
    const uint8_t *src = W + (static_cast<size_t>(nt) * KT + kt) * tileB;
    for (int c = tid; c < kBM * (kBK / 8); c += kThreads) {
      int row = c / (kBK / 8), col = (c % (kBK / 8)) * 8;
      cp_async16(sA + row * kLdA + col, src + (static_cast<size_t>(row) * kBK + col) * 2);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
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
          if (t < T) p[static_cast<size_t>(t) * Npad + row] = acc[mt][j][e] * epi_scale(epi, t);
        }
    return;
  }
  if (epi.kind == kEpiSwiGLU) {
    // gate rows (even) and their up rows (the odd row after each) of the tile meet in shared memory
    float *sC = reinterpret_cast<float *>(smem);  // [128][kBN + 1]
#pragma unroll
    for (int mt = 0; mt < 2; mt++)
#pragma unroll
      for (int j = 0; j < 4; j++)
#pragma unroll
        for (int e = 0; e < 4; e++) {
          int row = wm * 32 + mt * 16 + g + (e / 2) * 8;
          int col = wn * 32 + j * 8 + 2 * tq + (e % 2);
          sC[row * (kBN + 1) + col] = acc[mt][j][e] * (epi.scale && t0 + col < T ? epi.scale[t0 + col] : 1.f);
        }
    __syncthreads();
    for (int i = tid; i < 64 * kBN; i += kThreads) {
      int f = i % 64, c = i / 64;
      int t = t0 + c, feat = nt * 64 + f;
      if (t < T && feat < epi.n) {
        float gg = sC[(2 * f) * (kBN + 1) + c], uu = sC[(2 * f + 1) * (kBN + 1) + c];
        epi.out_h[static_cast<size_t>(t) * epi.ld + feat] = __float2half_rn(silu_mul(gg, uu));
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
          const float y = acc[mt][j][e] * epi_scale(epi, t);
          if (epi.kind == kEpiAdd) *o += y;
          else *o = y;
        }
      }
}

template <int TYPE>
size_t smem_bytes() {
  return kSA + kSB;
}

template <int TYPE>
void launch_t(const QWeight &w, const __half *act, int T, const Epi &epi, float *part, cudaStream_t s) {
  size_t sm = smem_bytes<TYPE>();
  dim3 grid(w.NT, w.splits, (T + kBN - 1) / kBN);
  launch_pdl(gemm_kernel<TYPE>, grid, kThreads, sm, s, w.data, w.KT, w.splits, act, T, epi, part, w.NT * kBM);
}

}  // namespace

void gemm_init() {
  cudaFuncSetAttribute(gemm_kernel<kF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem_bytes<kF16>()));
}

// F16 weights (checkpoints stored unquantized); Q4_K and Q8_0 run on the tcgen05 kernel of k_gemm_tc.cu
void launch_gemm(const QWeight &w, const __half *act, int T, const Epi &epi, float *part, cudaStream_t s) {
  if (T <= 0) return;
  launch_t<kF16>(w, act, T, epi, part, s);
}

}  // namespace gck
