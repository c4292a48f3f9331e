// Launch wrappers of the decoder-step kernels (host-callable; all run on the caller's stream).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "plan.h"

namespace gck {

enum WType { kF32 = 0, kF16 = 1, kQ8_0 = 8, kQ4_K = 12 };  // GGUF type ids

// GEMM tiles: a weight matrix [N, K] is stored as tiles of kBM rows x kBK columns, tile (nt, kt) at
// (nt * KT + kt) * tile_bytes. Inside a tile, scales/headers come first, then the quants (runtime.cu relayout).
constexpr int kBM = 128;
constexpr int kBK = 256;
constexpr int kBN = 64;   // tokens per CTA tile

__host__ __device__ inline size_t tile_bytes(int type) {
  switch (type) {
    case kQ4_K: return static_cast<size_t>(kBM) * 144;               // 128 x (16 B header + 128 B quants)
    case kQ8_0: return static_cast<size_t>(kBM) * (8 * 2 + 256);     // 128 x (8 fp16 scales + 256 int8)
    default: return static_cast<size_t>(kBM) * kBK * 2;              // f16
  }
}
// Q4_K and Q8_0 tiles: the 128 rows' 16-byte headers (Q4_K: d, dmin, 12 scale bytes; Q8_0: the 8 block scales), then
// the quants as [32-K block][pieces][128 rows][16 B] (Q4_K: one piece, the block's 32 nibbles reordered so that
// masks give f16 pairs of consecutive k; Q8_0: two pieces of 16 quants stored as q + 128), so that thread r of the
// dequant warps reads rows 16 B apart (runtime.cu relayout, k_gemm_tc.cu).

enum EpiKind { kEpiStore = 0, kEpiAdd = 1, kEpiSwiGLU = 2 };
struct Epi {
  int kind;
  int n;          // real output columns (features); SwiGLU: real FFN width
  int ld;         // leading dimension of the output
  float *out_f;   // Store / Add: f32 [T, ld]
  __half *out_h;  // SwiGLU: f16 [T, ld]
  // a8 activations: the input rows hold integers (per-token int8 codes, exact in f16) and row t's products are
  // multiplied by scale[t] before anything else (split-K partials included); null: a16, nothing is multiplied
  const float *scale = nullptr;
};
#ifdef __CUDACC__
// the a8 scale of token row t (1 for a16); multiplying by it is exact for a16
__device__ __forceinline__ float epi_scale(const Epi &e, int t) { return e.scale ? e.scale[t] : 1.f; }
#endif

struct QWeight {            // a relaid-out weight on the device
  const uint8_t *data = nullptr;
  int type = 0;
  int N = 0, K = 0;         // logical rows (outputs) and columns (inputs)
  int NT = 0, KT = 0;       // tiles
  int splits = 1;           // split-K factor (fixed per weight: batch invariant)
  int gslices = 1;          // K slices of the GEMV (tolerance buckets, a few token rows)
};

// Tensor parallelism: a deterministic all-reduce of the ranks' [T, d] f32 partials over peer memory (NVLink), in two
// phases on a pair of buffers (one per alternate reduction). Every rank sums the rows it owns from all ranks in rank order
// (reduce-scatter, into its own buffer), then every reader takes each row's sum from its owner; the order of the f32 adds
// never depends on T. Flags are 64-bit epoch * 4 + phase, written by the owner, polled by the peers (bounded waits).
constexpr int kMaxTp = 8;
struct TpPeers {
  int n, rank;
  float *buf[kMaxTp][2];        // every rank's two partial buffers (peer pointers; this rank's own at [rank])
  unsigned long long *flag[kMaxTp];   // every rank's flags [2] (one per buffer)
  int *err;                     // this rank's error word (a wait that ran out)
};
// rows [r0, r1) of T owned by rank k
__host__ __device__ inline void tp_rows(int T, int n, int k, int &r0, int &r1) {
  const int per = (T + n - 1) / n;
  r0 = min(T, k * per);
  r1 = min(T, r0 + per);
}
// A kernel's completion published to other GPUs: the last CTA to finish (counter, reset by it) fences system-wide and
// stores value to flag with release semantics. flag null: no signal.
struct Signal {
  unsigned long long *flag = nullptr;
  unsigned long long value = 0;
  unsigned *counter = nullptr;   // zero between launches
};
#ifdef __CUDACC__
// thread 0 of a CTA, after the CTA's threads fenced their stores system-wide and synchronized
__device__ __forceinline__ void signal_if_last(const Signal &sg) {
  const unsigned total = gridDim.x * gridDim.y * gridDim.z;
  if (atomicAdd(sg.counter, 1u) == total - 1) {
    __threadfence_system();
    *sg.counter = 0;
    asm volatile("st.release.sys.global.u64 [%0], %1;\n" ::"l"(sg.flag), "l"(sg.value) : "memory");
  }
}
#endif
void launch_tp_signal(unsigned long long *flag, unsigned long long value, cudaStream_t s);
// sig: published when every row of this rank is summed (phase 2)
// S: split-K slices per rank ([S][T][d] in each buffer); sums over ranks, then slices, in order
void launch_tp_reduce_scatter(const TpPeers &p, int b, unsigned long long epoch, int T, int d, int S, const Signal &sig,
                              cudaStream_t s);

void launch_embed(const PlanView &pv, const uint8_t *emb, int type, size_t row_bytes, int d, float *x, cudaStream_t s);
// part (nullable): S split-K partials [S, T, pld] of a residual-add GEMM, added into x before the norm.
// tp (nullable): instead, the tensor-parallel sum of buffer tp_buf for this epoch, gathered from the rows' owners.
// qscale (nullable): a8 activations. Each output row is quantized per token, symmetric int8: s = amax / 127 of the
// row's normalized values (1 for an all-zero row), code = rint(value / s), written as f16 (exact); qscale[r] = s.
void launch_rmsnorm(float *x, const int *rows, int n, const float *gain, float eps, int d, int ld, __half *out,
                    const float *part, int S, int pld, int T, const TpPeers *tp, int tp_buf,
                    unsigned long long tp_epoch, float *qscale, cudaStream_t s);
// a8 activations of a GEMM input computed elsewhere (attention output, SwiGLU output): rows [T, ld] f16, the first n
// columns quantized in place the same way, scale[t] = s of row t
void launch_act_quant(__half *buf, int T, int n, int ld, float *scale, cudaStream_t s);
// qkv: [T, ld] rows (S == 1) or [S, T, ld] split-K partials
void launch_rope_kv(const PlanView &pv, const float *qkv, int S, int ld, int H, int KVH, int dh,
                    const float2 *rope_tab, __half *q, void *kc, void *vc, int8_t *exps, int kv_fp8, int page_scale,
                    cudaStream_t s);
void launch_splitk_reduce(const float *part, int S, int T, int Npad, const Epi &epi, cudaStream_t s);
// scratch: [8][R][2] ints (the parts' candidates)
void launch_argmax(const float *logits, int R, int V, int *out, int *scratch, cudaStream_t s);
// A speculative round's acceptance: chain[0] is the anchor and chain[1..K] the drafts; target[i] the target's argmax
// after chain[0..i]. j = the longest prefix of drafts with chain[i + 1] == target[i]; out[0..j] = target[0..j] (the
// accepted drafts, then the target's own next token) and out[K + 1] = j + 1.
// The step's block-table patches: tables[p.x] = p.y for each of the n pairs.
void launch_table_patch(const uint2 *patches, int n, uint32_t *tables, cudaStream_t s);
void launch_spec_accept(const int *chain, const int *target, int K, int *out, cudaStream_t s);
// tensor parallelism: a rank's candidates (value bits, global index) of its vocabulary slice, and their merge
void launch_argmax_pick(const float *logits, int R, int V, int offset, int *pick, cudaStream_t s);
void launch_argmax_merge(const int *pick, int tp, int R, int *out, cudaStream_t s);
void launch_copy_blocks(const int *pairs, int n, int L, size_t page_bytes, size_t layer_bytes, uint8_t *kc,
                        uint8_t *vc, int8_t *exps, size_t exps_layer, int exps_per_block, cudaStream_t s);
void launch_commit(const int *moves, int n, int L, int KVH, int dh, uint8_t *kc, uint8_t *vc, int8_t *exps,
                   int kv_fp8, size_t layer_bytes, size_t exps_layer, float *tmp, cudaStream_t s);

// y = act[T, Kpad] (f16, row-major, Kpad = KT * kBK) times W^T, with the epilogue; part: split-K scratch
// [splits, T, NT * kBM] f32 (unused when splits == 1). With splits > 1 the GEMM writes only the partials: the
// reader sums them in split order (launch_splitk_reduce, or the next RMSNorm / RoPE kernel). With splits > 1 the GEMM writes only the partials and the caller
// launches launch_splitk_reduce (the sum in split order and the epilogue) after it.
// F16 weights: mma.sync kernel (k_gemm.cu). Q4_K / Q8_0 weights: tcgen05 kernel (k_gemm_tc.cu), whose activation
// tiles come through TMA tensor maps over the activation buffer, one map per token tile size.
void gemm_init();   // once per device, before the first launch_gemm
void launch_gemm(const QWeight &w, const __half *act, int T, const Epi &epi, float *part, cudaStream_t s);

// GEMV over Q4_K / Q8_0 tiles for T <= kGemvMaxT token rows: x [T, ldx] f16; gs K slices (partials [gs][T][Npad] when
// gs > 1, else the epilogue)
constexpr int kGemvMaxT = 4;
int gemv_slices(int NTW, int KT, int sms, bool reader_sums);
void launch_gemv(const QWeight &w, int gs, const __half *x, int ldx, int T, const Epi &epi, float *part, int *err,
                 cudaStream_t s);

struct TmaSet {            // tensor maps over one activation buffer [rows, K] f16, boxes of 64 K x {16..256} rows
  CUtensorMap m[5];
  const CUtensorMap *map(int nt) const { return &m[nt <= 16 ? 0 : nt <= 32 ? 1 : nt <= 64 ? 2 : nt <= 128 ? 3 : 4]; }
};
int tc_token_tile(int T);
size_t tc_tile_bytes(int type);
void gemm_tc_init();      // once per device
int tc_pair_clusters();   // two-CTA clusters of the paired GEMM that fit on the device at once (0: none)
// A chained launch: the gate/up GEMM (SwiGLU epilogue) and, in the same persistent launch, the down projection that
// reads its output, for steps of one token tile (T <= 64). Each CTA runs its units in the order of a host schedule
// (first-GEMM units first); a down unit's activation producer waits, per 256-K tile of its input, until the four
// gate/up bands that write that tile have stored it (ready[kt] counts their epilogue warps); the launch's last CTA
// resets the counters. The results are those of the two launches, bit for bit.
struct Chain {
  const uint8_t *W = nullptr;   // the second weight's tiles (null: a launch of one GEMM)
  int NTW = 0, KT = 0, splits = 1;
  Epi epi{};                    // the second GEMM's epilogue (split-K partials when splits > 1)
  float *part = nullptr;
  int Npad = 0;
  const int *sched = nullptr;      // per CTA its units in order; bit 31: a unit of the second GEMM
  const int *sched_off = nullptr;  // [grid + 1]
  unsigned *ready = nullptr;       // [KT of the second weight]
  unsigned *done = nullptr;        // CTAs finished (reset with ready)
};
struct ChainPlan {               // a chained launch's schedule on the device
  const int *sched = nullptr, *off = nullptr;
  int ctas = 0;
  unsigned *ready = nullptr, *done = nullptr;
};
// the schedule (host): the first GEMM's NTW0 bands round-robin, then the second GEMM's units (split-major, so those
// whose inputs complete first come first) each to the least-loaded CTA; returns the busiest CTA's load in tile times
double chain_schedule(int NTW0, int KT0, int NTW1, int KT1, int splits1, int sms, int *ctas, int *sched_out,
                      int *off_out);
void launch_gemm_tc_chain(const QWeight &w0, const TmaSet &ts0, const Epi &e0, const QWeight &w1, const TmaSet &ts1,
                          const Epi &e1, float *part1, const ChainPlan &cp, int T, int *err, cudaStream_t s);
// pairs: two-CTA clusters for the paired kernel (0: one CTA per MMA throughout; capped at tc_pair_clusters())
// sig (optional): the GEMM's completion published to other GPUs (tensor parallelism, phase 1 of the all-reduce)
void launch_gemm_tc(const QWeight &w, const TmaSet &ts, int T, const Epi &epi, float *part, int *err, int sms,
                    int pairs, cudaStream_t s, const Signal &sig = Signal{});


// Paged attention over the plan's work list: q [T, H, dh] f16 -> out [T, H, dh] f16. part_o / part_ml: split partials,
// merged by the last split to finish.
struct AttnArgs {
  const __half *q;
  const void *kc, *vc;       // this layer's pages [nblk][KVH][16][dh]
  const int8_t *exps;        // this layer's page exponents [nblk][KVH][2] (fp8 page mode) or null
  __half *out;
  float *part_o;             // [n_parts, 16, dh]
  float2 *part_ml;           // [n_parts, 16] (running max in log2 units, sum)
  int *sem;                  // [n_qg, KVH] finished splits (zero between launches)
  int H, KVH, dh, kv_fp8;
  float scale_log2;          // log2(e) / sqrt(dh)
};
void launch_attention(const PlanView &pv, const AttnArgs &a, int nw, cudaStream_t s);

}  // namespace gck
