// Device helpers shared by the kernels: PTX wrappers for sm_100a (cp.async, ldmatrix, mma.sync, fp8 conversion,
// mbarrier with bounded waits) and small numeric utilities.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "plan.h"

namespace gck {

#define GCK_DEV __device__ __forceinline__

GCK_DEV uint32_t smem_u32(const void *p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// SwiGLU of one feature, silu(g) * u = g / (1 + e^-g) * u (ref.py's F.silu(g) * u), with the fast exponential and
// division intrinsics (a few ulp in f32, far below the f16 rounding of the result); every kernel uses this one
GCK_DEV float silu_mul(float g, float u) { return __fdividef(g, 1.f + __expf(-g)) * u; }

// Programmatic dependent launch. A forward kernel started by launch_pdl may begin while the kernel before it in the
// stream still runs: it calls dep_wait() before its first access of memory that an earlier kernel writes or reads
// (dep_wait returns once the earlier kernels have completed and their writes are visible), and dep_launch() so that
// the next kernel's CTAs may start early (its prologue, or a weight stream that depends on nothing, overlaps this
// kernel's tail). Launched without the attribute, both return at once.
GCK_DEV void dep_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
GCK_DEV void dep_launch() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

extern bool g_pdl;   // programmatic dependent launch of the forward kernels (on unless GCK_PDL=0)
template <typename... P, typename... A>
inline void launch_pdl(void (*k)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, A... args) {
  if (!g_pdl) {
    k<<<grid, block, smem, s>>>(args...);
    return;
  }
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, k, args...);
}

GCK_DEV void cp_async16(void *smem, const void *gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(smem)), "l"(gmem));
}
// 16-byte copy that writes zeros when pred is false (src-size 0)
GCK_DEV void cp_async16_pred(void *smem, const void *gmem, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem), "r"(pred ? 16 : 0));
}
GCK_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
GCK_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

GCK_DEV void ldmatrix_x4(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3, const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}

// D = A(16x16, row) * B(16x8, col) + D, f16 inputs, f32 accumulators
GCK_DEV void mma_f16(float *d, const uint32_t *a, const uint32_t *b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// two e4m3 codes (low byte -> low half) to a half2, exact
GCK_DEV uint32_t e4m3x2_to_h2(uint16_t v) {
  uint32_t r;
  asm volatile("cvt.rn.f16x2.e4m3x2 %0, %1;\n" : "=r"(r) : "h"(v));
  return r;
}

// float to e4m3 code, round to nearest even, saturating at +-448
GCK_DEV uint8_t f32_to_e4m3(float x) {
  uint16_t r;
  asm volatile("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;\n" : "=h"(r) : "f"(0.f), "f"(x));
  return static_cast<uint8_t>(r & 0xff);
}

GCK_DEV float e4m3_to_f32(uint8_t c) {
  uint32_t h2 = e4m3x2_to_h2(static_cast<uint16_t>(c));
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h2 & 0xffff)));
}

GCK_DEV uint32_t pack_h2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&h);
}

GCK_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
GCK_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Physical KV row of list entry `i` for token `j` of item `it` (see plan.h): the prefix and chain rows map to
// themselves, tree rows through the token's path.
GCK_DEV int list_row(const PlanView &pv, const Item &it, const QGroup &qg, int i) {
  int r = i;
  if (qg.path_len && i >= it.pos) r = it.pos + pv.paths[qg.path_off + (i - it.pos)];
  return static_cast<int>(pv.blocks[it.blk_off + r / kBlock]) * kBlock + (r % kBlock);
}
// the same for a tree token given by its path (offset, length) in plan.paths
GCK_DEV int list_row_path(const PlanView &pv, const Item &it, int path_off, int i) {
  const int r = i >= it.pos ? it.pos + pv.paths[path_off + (i - it.pos)] : i;
  return static_cast<int>(pv.blocks[it.blk_off + r / kBlock]) * kBlock + (r % kBlock);
}

}  // namespace gck
