/* gc.h — the C ABI this library exports: goethe-engine's pack runtime interface (runtime kind "gc-c"), version 1.2.
 *
 * This header restates, in this project's own words, the interface of the reference's abi/gc.h. Struct layouts,
 * constants and signatures are kept identical, because the engine's ctypes binding (goethe_engine/gc_c.py:27-77)
 * binds them by position and size. Each declaration names the abi/gc.h line it corresponds to.
 *
 * Conventions (abi/gc.h:7-22):
 *  - gc_abi_version() = MAJOR << 16 | MINOR; a caller needs an equal major and a minor at least its own.
 *  - Every in/out struct starts with `size`, set by the caller to the size it was compiled with. The library reads
 *    and writes only the fields that lie inside min(size, its own size); fields beyond are treated as zero and never
 *    written.
 *  - Each gc_open returns an independent handle with its own CUDA stream, weights, KV pool, sequence slots and
 *    scratch. A handle is not thread safe; handles on different threads are independent.
 *  - Functions return GC_OK or a negative GC_E_* code; gc_last_error(h) describes the last failure on h,
 *    gc_last_error(NULL) the last gc_open failure on the calling thread. An out-of-memory failure says
 *    "out of memory" (the engine retries a narrower batch ladder on that text, gc_c.py:222-227). */
#ifndef GOETHE_B200_GC_H
#define GOETHE_B200_GC_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GC_ABI_MAJOR 1
#define GC_ABI_MINOR 2
#define GC_ABI_VERSION ((GC_ABI_MAJOR << 16) | GC_ABI_MINOR)

#if defined(__GNUC__)
#define GC_API __attribute__((visibility("default")))
#else
#define GC_API
#endif

typedef struct gc_handle gc_handle;

/* Return codes (abi/gc.h:44-53). */
enum {
  GC_OK = 0,
  GC_E_ARG = -1,          /* a malformed argument or struct size, a block id outside the pool */
  GC_E_MANIFEST = -2,     /* manifest.json missing or unreadable, or a requested bucket absent */
  GC_E_WEIGHTS = -3,      /* a weight file missing or unreadable, or a tensor missing or of an unsupported type */
  GC_E_DEVICE = -4,       /* no such device, not sm_100, out of device memory, a CUDA failure */
  GC_E_UNSUPPORTED = -5,  /* a request this library does not run (spec pairs, embeddings, encoders) */
  GC_E_STATE = -6,        /* unknown sequence, no free sequence slot */
  GC_E_CAPACITY = -7      /* an output buffer is too small; the needed size is reported in the out struct */
};

/* gc_open_params.flags (abi/gc.h:56-59). */
enum { GC_OPEN_SPEC = 1u << 0, GC_OPEN_NO_CHECK = 1u << 1 };

/* abi/gc.h:61-74 */
typedef struct gc_open_params {
  uint32_t size;
  uint32_t flags;
  const char *pack_dir;          /* directory holding manifest.json */
  const char *const *weights;    /* GGUF files; tensors are found by name across all of them */
  uint32_t n_weights;
  int32_t device;                /* CUDA ordinal, -1 = the current device */
  const char *const *buckets;    /* manifest bucket ids to open (a batch ladder: the widest sets max_seqs) */
  uint32_t n_buckets;
  uint32_t pool_blocks;          /* KV blocks to allocate; 0 = the bucket's tune.pool_blocks, else what fits */
  const char *spec_policy;
  const char *scratch_dir;
  uint32_t state_pages;          /* ABI 1.1; a paged pack without bounded state reports 0 */
} gc_open_params;

/* abi/gc.h:77 */
GC_API uint32_t gc_abi_version(void);

/* abi/gc.h:79-82: loads and relays out the weights on the device, allocates the KV pool and scratch. */
GC_API int gc_open(const gc_open_params *p, gc_handle **out);

/* gc_layout.kv_dtype (abi/gc.h:85) */
enum { GC_KV_F16 = 0, GC_KV_FP8 = 1 };

/* gc_layout.flags (abi/gc.h:88-100) */
enum {
  GC_L_PAGED = 1u << 0,
  GC_L_DEVICE_ARGMAX = 1u << 1,
  GC_L_SPEC = 1u << 2,
  GC_L_BOUNDED = 1u << 3,
  GC_L_EMBED = 1u << 4,
  GC_L_SEQ2SEQ = 1u << 5
};

/* abi/gc.h:105-129 */
typedef struct gc_layout {
  uint32_t size;
  uint32_t flags;
  uint32_t vocab;
  uint32_t max_cols;             /* most tokens one gc_step takes over all its items */
  uint32_t max_seqs;             /* live sequences */
  uint32_t max_ctx;              /* longest sequence */
  uint32_t block_size;           /* KV rows per block (16) */
  uint32_t num_blocks;
  uint32_t layers;
  uint32_t kv_heads;
  uint32_t head_dim;
  uint32_t kv_dtype;
  uint32_t spec_width;
  uint32_t feat_width;
  uint64_t kv_bytes;             /* device bytes of the KV pool, fp8 page scales included */
  uint64_t state_bytes;
  uint64_t device_bytes;         /* all device bytes the handle holds */
  uint32_t state_pages;
  uint32_t pad1;
  uint32_t embd_dim;
  uint32_t embd_pool;
  uint32_t enc_frames;
  uint32_t enc_feat;
} gc_layout;

/* abi/gc.h:131 */
GC_API int gc_layout_get(gc_handle *h, gc_layout *out);

/* gc_work.flags (abi/gc.h:134-138) */
enum { GC_W_GREEDY = 1u << 0, GC_W_SPEC = 1u << 1, GC_W_FEATS = 1u << 2 };

/* abi/gc.h:145-157. Token i writes KV row pos + i and runs RoPE and attention at pos + depth(i); it attends to rows
 * < pos and to its ancestors' rows (a chain: rows pos .. pos + i). Rows do not depend on the rest of the batch. */
typedef struct gc_work {
  uint32_t size;
  uint32_t flags;
  uint64_t sid;
  uint32_t pos;
  uint32_t n_tokens;
  const int32_t *tokens;
  const int32_t *parents;        /* NULL: a chain */
  const uint32_t *blocks;        /* block table covering rows 0 .. pos + n_tokens - 1 */
  uint32_t n_blocks;
  uint32_t want;                 /* logits / argmax of the last `want` tokens */
} gc_work;

/* gc_step_in.flags (abi/gc.h:160-162) */
enum { GC_S_HOST_LOGITS = 1u << 0, GC_S_NORMALIZE = 1u << 1 };

/* abi/gc.h:164-170 */
typedef struct gc_step_in {
  uint32_t size;
  uint32_t flags;
  const gc_work *const *work;
  uint32_t n_work;
  uint32_t pad;
} gc_step_in;

/* abi/gc.h:172-190 */
typedef struct gc_step_out {
  uint32_t size;
  uint32_t n_rows;
  int32_t *tokens;
  uint32_t tokens_cap;
  uint32_t pad0;
  uint32_t *counts;
  float *logits;
  uint64_t logits_cap;
  uint64_t logits_dev;
  float *feats;
  uint64_t feats_cap;
} gc_step_out;

/* abi/gc.h:192-193: one step over the items (decode, prefill chunk, tree verify, mixed). Synchronous: host outputs
 * are written when it returns; logits_dev stays valid until the next step on the handle. */
GC_API int gc_step(gc_handle *h, const gc_step_in *in, gc_step_out *out);

/* abi/gc.h:195-208 (gc_embed, gc_encode) are exported only by embedding and encoder-decoder libraries; this
 * decoder library exports neither. */

/* abi/gc.h:210-212: after a tree verify of sid, row base + path[j] becomes row base + j (all layers, K and V). */
GC_API int gc_commit(gc_handle *h, uint64_t sid, uint32_t base, const uint32_t *path, uint32_t n);

/* abi/gc.h:214-216: block src[i] is copied into block dst[i], in order. */
GC_API int gc_copy_blocks(gc_handle *h, const uint32_t *src, const uint32_t *dst, uint32_t n);

/* abi/gc.h:218-222: bounded-state snapshots; without GC_L_BOUNDED both answer GC_E_ARG. */
GC_API int gc_state_save(gc_handle *h, uint64_t sid, uint32_t snap);
GC_API int gc_state_restore(gc_handle *h, uint32_t snap, uint64_t sid);

/* abi/gc.h:224-225: frees the sequence slot; an unknown sid is not an error. */
GC_API int gc_release(gc_handle *h, uint64_t sid);

/* abi/gc.h:227 */
GC_API const char *gc_last_error(gc_handle *h);

/* abi/gc.h:229-230: frees everything; NULL is accepted. */
GC_API void gc_close(gc_handle *h);

/* Pricing (optional in the ABI, abi/gc.h:232-237, bound by goethe_engine/pack.py lib_price:928-961). gc_probe measures a
 * device's cost constants once into an opaque blob (it times bounded probe kernels; no handle, KV or weights are
 * touched); a too-small cap gives GC_E_CAPACITY with *size set. gc_price is host math only: the predicted step time of
 * a bucket on the device the blob describes. */
GC_API int gc_probe(int device, void *constants, uint64_t cap, uint64_t *size);
GC_API int gc_price(const void *constants, uint64_t size, const char *bucket_id, double *step_us);

#ifdef __cplusplus
}
#endif
#endif
