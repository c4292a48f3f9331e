/* gck_ext.h — entry points of this library beyond the gc.h ABI. None has a counterpart in the reference's abi/gc.h;
 * the engine never calls them. They serve measurement: device-side timing of gc_step with CUDA events recorded on
 * the handle's own stream, and a count of the kernels a step launched. */
#ifndef GOETHE_B200_GCK_EXT_H
#define GOETHE_B200_GCK_EXT_H

#include "gc.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Kernel classes of a step, for gck_stats.class_ms / class_launches (bit i of a mask = class i). */
enum {
  GCK_K_EMBED = 0,      /* token embedding gather */
  GCK_K_NORM = 1,       /* RMSNorm (every layer's two, and the final one) */
  GCK_K_QKV = 2,        /* fused q/k/v projection GEMM */
  GCK_K_ROPE = 3,       /* RoPE + KV page write */
  GCK_K_ATTN = 4,       /* paged attention (splits) */
  GCK_K_COMBINE = 5,    /* attention split merge */
  GCK_K_O = 6,          /* o_proj GEMM + residual */
  GCK_K_GATEUP = 7,     /* gate/up GEMM + SwiGLU */
  GCK_K_DOWN = 8,       /* down_proj GEMM + residual */
  GCK_K_HEAD = 9,       /* LM head GEMM */
  GCK_K_ARGMAX = 10,    /* device argmax */
  GCK_K_REDUCE = 11,    /* split-K reduction + epilogue of a GEMM with K splits */
  GCK_K_ALLREDUCE = 12, /* tensor parallelism: all-reduce of o_proj / down_proj, argmax gather */
  GCK_K_QUANT = 13,     /* a8 buckets: per-token int8 quantization of the attention and SwiGLU outputs */
  GCK_K_CLASSES = 16
};

typedef struct gck_stats {
  uint32_t size;
  uint32_t steps;                         /* gc_step calls since gck_stats_enable */
  uint64_t launches;                      /* kernels those steps launched */
  double forward_ms;                      /* device time from a step's first kernel to its last, summed over steps */
  double class_ms[GCK_K_CLASSES];         /* device time of the masked classes' launches, summed */
  uint64_t class_launches[GCK_K_CLASSES]; /* launches of each masked class */
  uint64_t h2d_bytes;                     /* host-to-device bytes those steps copied (plans, block-table patches) */
  uint32_t graph_steps;                   /* steps replayed from a captured CUDA graph (class_mask 0 only) */
  uint32_t graph_captures;                /* steps captured into a new graph */
  uint32_t gemm_pairs;                    /* two-CTA clusters the tcgen05 GEMM runs on (0: one CTA per MMA) */
} gck_stats;

/* Starts (and resets) step statistics on h; class_mask picks the classes whose launches are each bracketed by a
 * pair of events (0: only the whole-step events). Returns GC_OK or GC_E_ARG. */
GC_API int gck_stats_enable(gc_handle *h, uint32_t class_mask);

/* Stops recording and copies the statistics (up to out->size bytes). */
GC_API int gck_stats_read(gc_handle *h, gck_stats *out);

/* gc_commit without device allocation. No counterpart in the reference's abi/gc.h (an addition of this library).
 *
 * Some callers cannot allocate device memory while they run: a serving process that reserves all of the GPU's memory
 * at start-up and treats any later cudaMalloc as a failure, or one that shares the GPU under a fixed memory budget
 * enforced by an allocator it does not control. gc_commit grows its staging buffers with cudaMalloc on first use; this entry point does the
 * same commit (row base + path[j] becomes row base + j in every layer, K and V; fp8 rows re-encoded into their new
 * page's scale) with its scratch in a fixed 16 MiB device array inside the library instead, and allocates nothing.
 *
 * Limits and rules:
 *  - the scratch holds the move list and every moved row of every layer as float32: (path entries that move) times
 *    layers x 2 x kv_heads x head_dim x 4 bytes must fit 16 MiB less 256 bytes (an 8B-shaped model: about 63 rows;
 *    a 70B-shaped one: about 25); a longer path returns GC_E_ARG and a text giving the limit;
 *  - gc_open looks the array's address up (cudaGetSymbolAddress) on every device it opens, with that device current;
 *    under CUDA's lazy module loading that is when the array is committed on the device, so it counts toward the
 *    handle's memory at open and a commit allocates nothing, its first one included. A device that opened a handle
 *    holds the 16 MiB until the process exits;
 *  - all callers on one device share the array and it keeps the last call's contents; calls that overlap on the GPU
 *    (two handles of one device committing from different threads at once) race, so serialize them. The call itself
 *    returns only after its work on the handle's stream has finished. */
GC_API int gck_commit_static(gc_handle *h, uint64_t sid, uint32_t base, const uint32_t *path, uint32_t n);

#ifdef __cplusplus
}
#endif
#endif
