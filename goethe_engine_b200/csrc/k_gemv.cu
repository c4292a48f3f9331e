// Quantized weight GEMV for decode steps of a few token rows (buckets whose manifest determinism is "tolerance"):
//
//   y[t, n] = sum_k act[t, k] * W[n, k]        t < T <= kGemvMaxT       (ref.py:51-59, the reference's `w @ h`)
//
// At one to four token rows a step's linear layers are a stream of the quantized weights (Q4_K 0.5625 B, Q8_0
// 1.0625 B per weight) with a handful of multiply-adds per byte, so this runs on the CUDA cores at the HBM roofline
// instead of feeding 16-token tiles to the tensor cores. A CTA takes one unit = a 128-row band of the relaid weight
// (the tcgen05 GEMM's tiles: 256 K per tile, rows' 16-byte chunks adjacent) over a fixed slice of its K tiles. The
// tiles stream through a ring in shared memory, one 1-D bulk copy per tile issued by one thread, the first ones before
// the kernel waits for its activations (the weights depend on no earlier kernel): a CTA keeps the whole ring in flight
// (about 70 KB, two CTAs per SM), where a register double buffer held one tile of its threads' bytes and left HBM
// half idle at batch 1. Two threads per row split each tile's eight 32-K sub-blocks: a thread takes its row's 16-byte
// pieces of the tile from shared memory (rows adjacent: conflict-free), dequantizes them (the shared f16 helpers:
// every weight rounded once, as in the GEMM) and multiplies them with the step's activations, staged once per CTA in
// shared memory. Each 32-K sub-block accumulates in packed f16, then in f32; the two halves of a row add in a fixed
// order. Every wait on the ring is bounded (about 2 s): a timeout sets the error word and the CTA returns.
//
// Numerics: the f16 sub-block sums make this path differ from the tcgen05 one in the last bits, and the library uses
// it only for a few rows, so a row's result depends on the batch width: the manifest's "tolerance" determinism (a
// batch-invariant bucket never runs it). Slices of K write split-K partials [slice][T][Npad] that the next kernel sums
// in slice order (RMSNorm, RoPE) or a reduce launch does (SwiGLU, the head), exactly as for the GEMM.
#include <algorithm>

#include "common.cuh"
#include "dequant.cuh"
#include "kernels.h"

namespace gck {
namespace {

constexpr int kGemvThreads = 256;   // two threads per row of the 128-row band

constexpr unsigned long long kRingWaitNs = 2000000000ull;
constexpr int kErrGemvRing = 17;    // error word: a tile of the ring did not land within the limit

template <int TYPE>
struct Raw;
template <>
struct Raw<kQ4_K> {                 // a thread's bytes of one tile: the row's header, sub-blocks 4h .. 4h+3
  static constexpr int TILE = kBM * 144;
  static constexpr int N = 5;
  static constexpr int RING = 4;    // tiles in flight per CTA (73.7 KB)
};
template <>
struct Raw<kQ8_0> {                 // the row's scales, blocks 4h .. 4h+3 (two 16-byte halves each)
  static constexpr int TILE = kBM * 272;
  static constexpr int N = 9;
  static constexpr int RING = 2;    // 69.6 KB
};
// dynamic shared memory: the ring's barriers (128 B), the ring, then the activations [T][nk] f16
constexpr int kRingOff = 128;

GCK_DEV void ring_init(uint64_t *b) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(smem_u32(b)));
}
// one 1-D bulk copy of a tile into its ring slot; the slot's barrier completes when the bytes have landed
GCK_DEV void ring_fill(uint8_t *dst, const uint8_t *src, uint32_t bytes, uint64_t *b) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(b))
               : "memory");
}
GCK_DEV bool ring_try(uint64_t *b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 1000;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// bounded wait for the phase of the given parity; false (and the error word set) on timeout
GCK_DEV bool ring_wait(uint64_t *b, uint32_t parity, int *err) {
  if (ring_try(b, parity)) return true;
  unsigned long long t0, t;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t0));
  for (uint32_t n = 1;; n++) {
    if (ring_try(b, parity)) return true;
    if ((n & 63u) == 0) {
      asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
      if (t - t0 > kRingWaitNs) {
        atomicCAS(err, 0, kErrGemvRing);
        return false;
      }
    }
  }
}

// a thread's 16-byte pieces of the tile in shared memory (row r, half hs)
template <int TYPE>
GCK_DEV void load_raw(const uint8_t *tile, int r, int hs, uint4 (&v)[Raw<TYPE>::N]) {
  const uint4 *t = reinterpret_cast<const uint4 *>(tile);
  v[0] = t[r];
  if (TYPE == kQ4_K) {
#pragma unroll
    for (int i = 0; i < 4; i++) v[1 + i] = t[kBM + (4 * hs + i) * kBM + r];
  } else {
#pragma unroll
    for (int i = 0; i < 8; i++) v[1 + i] = t[kBM + (8 * hs + i) * kBM + r];
  }
}

// the 32-K sub-block's 16 f16 pairs times the activations of T rows: f16 partial sums, then into acc (f32)
template <int T>
GCK_DEV void dot32(const uint32_t (&w)[16], const __half2 *xs, int ldx2, float (&acc)[T]) {
#pragma unroll
  for (int t = 0; t < T; t++) {
    const uint4 *x4 = reinterpret_cast<const uint4 *>(xs + t * ldx2);
    __half2 s = __float2half2_rn(0.f);
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const uint4 xv = x4[j];
      s = __hfma2(*reinterpret_cast<const __half2 *>(&w[4 * j]), *reinterpret_cast<const __half2 *>(&xv.x), s);
      s = __hfma2(*reinterpret_cast<const __half2 *>(&w[4 * j + 1]), *reinterpret_cast<const __half2 *>(&xv.y), s);
      s = __hfma2(*reinterpret_cast<const __half2 *>(&w[4 * j + 2]), *reinterpret_cast<const __half2 *>(&xv.z), s);
      s = __hfma2(*reinterpret_cast<const __half2 *>(&w[4 * j + 3]), *reinterpret_cast<const __half2 *>(&xv.w), s);
    }
    const float2 f = __half22float2(s);
    acc[t] += f.x + f.y;
  }
}

template <int TYPE, int T>
GCK_DEV void tile_dot(const uint4 (&v)[Raw<TYPE>::N], int hs, const __half2 *xs, int ldx2, float (&acc)[T]) {
  const uint4 hdr = v[0];
  if (TYPE == kQ4_K) {
    const uint32_t dd = prmt(hdr.x, 0, 0x1010u);                 // (d, d)
    const uint32_t mm = prmt(hdr.x, 0, 0x3232u) ^ 0x80008000u;   // (-dmin, -dmin)
#pragma unroll
    for (int gp = 0; gp < 2; gp++) {
      const int g = 4 * hs + 2 * gp;
      uint32_t S01, O01;
      q4k_pair_scales(hdr, g, dd, mm, S01, O01);
#pragma unroll
      for (int e = 0; e < 2; e++) {
        const uint32_t Sg = prmt(S01, 0, e ? 0x3232u : 0x1010u), Og = prmt(O01, 0, e ? 0x3232u : 0x1010u);
        const uint4 qw = v[1 + 2 * gp + e];
        uint32_t w[16];
        q4_word(qw.x, Sg, Og, w);
        q4_word(qw.y, Sg, Og, w + 4);
        q4_word(qw.z, Sg, Og, w + 8);
        q4_word(qw.w, Sg, Og, w + 12);
        dot32<T>(w, xs + (g + e) * 16, ldx2, acc);
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int b = 4 * hs + i;
      const uint32_t dw2 = (b >> 1) == 0 ? hdr.x : (b >> 1) == 1 ? hdr.y : (b >> 1) == 2 ? hdr.z : hdr.w;
      const uint32_t D = prmt(dw2, 0, (b & 1) ? 0x3232u : 0x1010u);
      const uint4 q0 = v[1 + 2 * i], q1 = v[2 + 2 * i];
      uint32_t w[16];
      q8_word(q0.x, D, w); q8_word(q0.y, D, w + 2); q8_word(q0.z, D, w + 4); q8_word(q0.w, D, w + 6);
      q8_word(q1.x, D, w + 8); q8_word(q1.y, D, w + 10); q8_word(q1.z, D, w + 12); q8_word(q1.w, D, w + 14);
      dot32<T>(w, xs + b * 16, ldx2, acc);
    }
  }
}

// unit blockIdx.x = (band nt, K slice sl); activations staged as [T][nk] f16 (nk = the slice's tiles x 256, zero past K)
template <int TYPE, int T>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const uint8_t *__restrict__ W, int KT, int gs,
                                                            const __half *__restrict__ x, int ldx, int K, int Tn,
                                                            Epi epi, float *part, int Npad, int *err) {
  constexpr int TILE = Raw<TYPE>::TILE, RING = Raw<TYPE>::RING;
  extern __shared__ __align__(128) uint8_t gsm[];
  uint64_t *full = reinterpret_cast<uint64_t *>(gsm);
  uint8_t *ring = gsm + kRingOff;
  const int nt = blockIdx.x / gs, sl = blockIdx.x % gs;
  const int base = KT / gs, extra = KT % gs;
  const int per = base + (sl < extra ? 1 : 0), kt0 = sl * base + min(sl, extra);
  const int nk = per * kBK;
  const int r = threadIdx.x & (kBM - 1), hs = threadIdx.x / kBM;
  const uint8_t *tiles = W + (static_cast<size_t>(nt) * KT + kt0) * TILE;
  // the weights depend on no earlier kernel: the ring's first tiles are requested before waiting for the activations
  if (threadIdx.x == 0) {
    for (int i = 0; i < RING; i++) ring_init(&full[i]);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    for (int i = 0; i < RING && i < per; i++) ring_fill(ring + i * TILE, tiles + static_cast<size_t>(i) * TILE, TILE, &full[i]);
  }
  dep_wait();
  dep_launch();
  __half *sx = reinterpret_cast<__half *>(gsm + kRingOff + RING * TILE);
  const int k0 = kt0 * kBK, chunks = nk / 8;
  for (int i = threadIdx.x; i < T * chunks; i += kGemvThreads) {
    const int t = i / chunks, c = i % chunks, k = k0 + 8 * c;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (t < Tn) {
      if (k + 8 <= K) {
        v = *reinterpret_cast<const uint4 *>(x + static_cast<size_t>(t) * ldx + k);
      } else {
        __half h8[8];
#pragma unroll
        for (int j = 0; j < 8; j++) h8[j] = k + j < K ? x[static_cast<size_t>(t) * ldx + k + j] : __float2half(0.f);
        v = *reinterpret_cast<const uint4 *>(h8);
      }
    }
    reinterpret_cast<uint4 *>(sx + static_cast<size_t>(t) * nk)[c] = v;
  }
  __syncthreads();   // the activations staged, the ring's barriers initialised

  float acc[T];
#pragma unroll
  for (int t = 0; t < T; t++) acc[t] = 0.f;
  const __half2 *xs = reinterpret_cast<const __half2 *>(sx);
  int u = 0;
  for (; u < per; u++) {
    // tile u sits in slot u % RING, phase (u / RING) & 1 of its barrier; every thread waits for it
    const int slot = u % RING;
    const bool ok = ring_wait(&full[slot], static_cast<uint32_t>((u / RING) & 1), err);
    uint4 cur[Raw<TYPE>::N];
    load_raw<TYPE>(ring + slot * TILE, r, hs, cur);
    // every thread holds its bytes of the slot; a timeout anywhere ends the loop for the whole CTA
    if (__syncthreads_or(ok ? 0 : 1)) break;
    if (threadIdx.x == 0 && u + RING < per) {
      // the generic-proxy reads of the slot above are ordered before the bulk copy's writes into it
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
      ring_fill(ring + slot * TILE, tiles + static_cast<size_t>(u + RING) * TILE, TILE, &full[slot]);
    }
    tile_dot<TYPE, T>(cur, hs, xs + u * (kBK / 2), nk / 2, acc);
  }
  if (u < per) {
    // a tile did not land in time: the copies this CTA issued land before it exits (bounded), then it returns
    if (threadIdx.x == 0)
      for (int i = u; i < per && i < u + RING; i++) ring_wait(&full[i % RING], static_cast<uint32_t>((i / RING) & 1), err);
    return;
  }

  // the row's two halves, in order (sub-blocks 0-3, then 4-7)
  __shared__ float sred[T][kBM];
  if (hs == 1) {
#pragma unroll
    for (int t = 0; t < T; t++) sred[t][r] = acc[t];
  }
  __syncthreads();
  const int row = nt * kBM + r;
  if (hs == 0) {
#pragma unroll
    for (int t = 0; t < T; t++) acc[t] += sred[t][r];
    if (epi.scale)     // a8: every product of token row t times its activation scale
#pragma unroll
      for (int t = 0; t < T; t++)
        if (t < Tn) acc[t] *= epi.scale[t];
  }
  if (gs > 1) {
    if (hs == 0)
#pragma unroll
      for (int t = 0; t < T; t++)
        if (t < Tn) part[(static_cast<size_t>(sl) * Tn + t) * Npad + row] = acc[t];
    return;
  }
  if (epi.kind == kEpiSwiGLU) {
    // even rows are gate rows, the odd row after each its up row (feature nt * 64 + r / 2): the up value comes from
    // the neighbouring lane (warps 0-3 hold whole rows here)
    if (hs == 0) {
      const int f = nt * 64 + (r >> 1);
#pragma unroll
      for (int t = 0; t < T; t++) {
        const float uu = __shfl_xor_sync(0xffffffffu, acc[t], 1);
        if ((r & 1) == 0 && t < Tn && f < epi.n)
          epi.out_h[static_cast<size_t>(t) * epi.ld + f] = __float2half_rn(silu_mul(acc[t], uu));
      }
    }
    return;
  }
  if (hs == 0 && row < epi.n) {
#pragma unroll
    for (int t = 0; t < T; t++)
      if (t < Tn) {
        float *o = epi.out_f + static_cast<size_t>(t) * epi.ld + row;
        if (epi.kind == kEpiAdd) *o += acc[t];
        else *o = acc[t];
      }
  }
}

template <int TYPE, int T>
void launch_tt(const QWeight &w, int gs, const __half *x, int ldx, int Tn, const Epi &epi, float *part, int *err,
               cudaStream_t s) {
  const int per_max = (w.KT + gs - 1) / gs;
  const size_t smem = kRingOff + static_cast<size_t>(Raw<TYPE>::RING) * Raw<TYPE>::TILE +
                      static_cast<size_t>(T) * per_max * kBK * 2;
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(gemv_kernel<TYPE, T>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  launch_pdl(gemv_kernel<TYPE, T>, w.NT * gs, kGemvThreads, smem, s, w.data, w.KT, gs, x, ldx, w.K, Tn, epi, part,
             w.NT * kBM, err);
}

template <int TYPE>
void launch_type(const QWeight &w, int gs, const __half *x, int ldx, int Tn, const Epi &epi, float *part, int *err,
                 cudaStream_t s) {
  if (Tn <= 1) launch_tt<TYPE, 1>(w, gs, x, ldx, Tn, epi, part, err, s);
  else if (Tn == 2) launch_tt<TYPE, 2>(w, gs, x, ldx, Tn, epi, part, err, s);
  else launch_tt<TYPE, 4>(w, gs, x, ldx, Tn, epi, part, err, s);
}

}  // namespace

int gemv_slices(int NTW, int KT, int sms, bool reader_sums) {
  // one wave: as many units as fit two CTAs per SM (the ring's shared memory admits two), so every unit streams at
  // once with the same share of tiles; at most 16 tiles (4096 K) of activations per CTA, at most 16 slices; a weight
  // whose partials would need a reduce launch keeps one slice when its bands alone fill the SMs
  const int lo = (KT + 15) / 16;
  if (!reader_sums && NTW >= sms) return lo;
  int gs = std::max(1, 2 * sms / NTW);
  gs = std::min(gs, std::min(16, KT));
  return std::max(gs, lo);
}

void launch_gemv(const QWeight &w, int gs, const __half *x, int ldx, int T, const Epi &epi, float *part, int *err,
                 cudaStream_t s) {
  if (T <= 0) return;
  if (w.type == kQ4_K) launch_type<kQ4_K>(w, gs, x, ldx, T, epi, part, err, s);
  else launch_type<kQ8_0>(w, gs, x, ldx, T, epi, part, err, s);
}

}  // namespace gck
