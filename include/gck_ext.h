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
  GCK_K_CLASSES = 16
};

typedef struct gck_stats {
  uint32_t size;
  uint32_t steps;                         /* gc_step calls since gck_stats_enable */
  uint64_t launches;                      /* kernels those steps launched */
  double forward_ms;                      /* device time from a step's first kernel to its last, summed over steps */
  double class_ms[GCK_K_CLASSES];         /* device time of the masked classes' launches, summed */
  uint64_t class_launches[GCK_K_CLASSES]; /* launches of each masked class */
} gck_stats;

/* Starts (and resets) step statistics on h; class_mask picks the classes whose launches are each bracketed by a
 * pair of events (0: only the whole-step events). Returns GC_OK or GC_E_ARG. */
GC_API int gck_stats_enable(gc_handle *h, uint32_t class_mask);

/* Stops recording and copies the statistics (up to out->size bytes). */
GC_API int gck_stats_read(gc_handle *h, gck_stats *out);

#ifdef __cplusplus
}
#endif
#endif
