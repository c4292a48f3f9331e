// libgck: the gc.h C ABI (runtime kind gc-c) over the sm_100a decoder-step kernels.
//
// The boundary follows the reference's abi/gc.h and its mock runtime (tests/mock/gck_mock.c:28-194): size-prefixed
// structs read and written up to min(caller size, own size); negative GC_E_* codes with a per-handle error text; a
// thread-local gc_open error; block ids checked against the pool (GC_E_ARG); an unknown sid in gc_release accepted.
// What happens inside a step follows goethe_engine/ref.py (RefModel.token, TorchBackend.step/commit/copy_blocks).
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <fstream>
#include <memory>
#include <mutex>
#include <sstream>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "gc.h"
#include "gck_ext.h"
#include "hostio.h"
#include "kernels.h"

using namespace gck;

namespace gck {
bool g_pdl = true;
}

namespace {

thread_local std::string g_open_err;

struct GcError {
  int code;
  std::string msg;
};

[[noreturn]] void fail(int code, const char *fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  throw GcError{code, buf};
}

void ck(cudaError_t e, const char *what) {
  if (e != cudaSuccess) {
    cudaGetLastError();
    if (e == cudaErrorMemoryAllocation) fail(GC_E_DEVICE, "%s: out of memory", what);
    fail(GC_E_DEVICE, "%s: CUDA error %s", what, cudaGetErrorString(e));
  }
}

struct Layer {
  QWeight qkv, o, gu, dn;
  const float *attn_norm = nullptr, *ffn_norm = nullptr;
};

struct Slot {
  uint64_t sid = 0;
  bool used = false;
  std::vector<uint32_t> blocks;   // the table of the sequence's last step (gc_commit addresses rows through it)
  uint32_t last_pos = 0, last_n = 0;
};

template <typename T>
size_t vbytes(const std::vector<T> &v) { return v.size() * sizeof(T); }

}  // namespace

struct gc_handle {
  int dev = 0, sms = 148;
  // tensor parallelism: a group handle (tp > 1, ranks filled) drives one rank handle per device and holds no device
  // state of its own; a rank handle holds its slices (H, KVH, F, head rows) and an NCCL communicator
  int tp = 1, rank = 0;
  std::vector<gc_handle *> ranks;
  void *comm = nullptr;              // ncclComm_t of a rank handle
  float *tp_y = nullptr;             // rank: o_proj / down_proj output, all-reduced [T, d] (NCCL path)
  float *tp_bufs[2] = {nullptr, nullptr};   // rank: partial / summed rows of alternate reductions (peer-memory path)
  unsigned long long *tp_flags = nullptr;   // rank: the two buffers' flags (epoch * 4 + phase), read by the peers
  unsigned long long tp_epoch = 0;          // reductions so far (the same on every rank)
  bool tp_p2p = false;                      // all ranks reach each other's memory: the peer-memory reduction
  unsigned *sig_counter = nullptr;          // rank: finished CTAs of a signalling kernel (zero between launches)
  int tp_splits = 1;                        // rank: most split-K slices of o_proj / down_proj (buffer depth)
  TpPeers peers{};
  int *tp_pick = nullptr;            // rank: argmax candidates (value bits, index) of every rank [tp][T][2]
  int vocab0 = 0, vocab_rows = 0;    // head rows held here: [vocab0, vocab0 + vocab_rows)
  cudaStream_t st = nullptr;
  std::string err;
  // model
  int vocab = 0, d = 0, L = 0, H = 0, KVH = 0, dh = 0, F = 0;
  float eps = 1e-5f, theta = 1e4f;
  std::vector<Layer> layers;
  const uint8_t *emb = nullptr;
  int emb_type = 0;
  size_t emb_row_bytes = 0;
  QWeight head;
  const float *out_norm = nullptr;
  float2 *rope = nullptr;
  // KV
  int kv_fp8 = 0, page_scale = 0, nblk = 0;
  uint8_t *kc = nullptr, *vc = nullptr;
  int8_t *exps = nullptr;
  size_t page_bytes = 0, layer_bytes = 0, exps_layer = 0;
  // limits
  int max_seqs = 0, max_cols = 0, max_ctx = 0, qg_tokens = 1;
  int gemv_max_t = 0;                       // tolerance buckets: steps of up to this many token rows run the GEMV
  // a8 buckets: every GEMM input is quantized per token to int8 codes (held as f16 integers) with a float scale per
  // row; the scales of the RMSNorm outputs, of the attention output and of the SwiGLU output [max_cols] each
  bool a8 = false;
  float *h_scale = nullptr, *att_scale = nullptr, *act_scale = nullptr;
  // speculative pair (GC_OPEN_SPEC): this handle is the target of one linear stream; `drafter` a second handle on the
  // same device that runs on this handle's stream; a round drafts spec_k tokens. The stream's tokens so far (row i of
  // both KV caches holds hist[i]) and how many rows of the drafter's cache hold them (it lags after prefill steps).
  gc_handle *drafter = nullptr;
  int spec_k = 0;
  std::vector<int> hist;
  int draft_rows = 0;
  std::vector<uint32_t> spec_table;          // the stream's block table: blocks 0 .. max_ctx / 16 of both pools
  int *spec_out = nullptr, *spec_out_host = nullptr;   // [spec_k + 2]: a round's accepted tokens, then their count
  // scratch
  float *x = nullptr, *qkv = nullptr, *logits = nullptr, *part = nullptr, *attn_o = nullptr, *commit_tmp = nullptr;
  __half *h = nullptr, *q = nullptr, *att = nullptr, *act = nullptr;
  float2 *attn_ml = nullptr;
  int *argmax = nullptr, *pairs = nullptr, *arg_scratch = nullptr;
  int *kerr = nullptr, *kerr_host = nullptr;   // device error word of bounded waits, and its pinned mirror
  TmaSet tma_h, tma_att, tma_act;               // activation tiles of the tcgen05 GEMMs
  size_t part_cap = 0, attn_parts_cap = 0, attn_sem_cap = 0, commit_cap = 0, pairs_cap = 0;
  int *attn_sem = nullptr;
  uint8_t *plan_dev = nullptr, *plan_host = nullptr;
  size_t plan_cap = 0;
  int *tok_host = nullptr;
  std::vector<Slot> slots;
  // block tables resident on the device: row i (tab_stride entries) is slot i's table, mirrored by slots[i].blocks;
  // a step uploads only the entries that differ from the mirror (patches)
  uint32_t *tables = nullptr;
  int tab_stride = 0;
  // captured steps (CUDA graphs): a step whose shape (plan sizes, scratch generation) repeats replays its graph; a
  // shape is captured the second time it is seen. Off under tensor parallelism, statistics and tree items.
  struct Graph { std::vector<int64_t> key; cudaGraphExec_t exec; uint64_t launches; };
  bool graphs_on = true;
  // two-CTA clusters for the paired tcgen05 GEMM (GCK_PAIR=0 at open: none, one CTA per MMA throughout)
  int tc_pairs = 0;
  // gate/up and down_proj as one chained launch at steps of one token tile (GCK_CHAIN=0 at open: two launches)
  ChainPlan chain{};
  bool chain_ok = false, chain_on = true;
  std::vector<Graph> graphs;                 // most recent last
  std::vector<std::vector<int64_t>> seen;   // shapes run once without a graph
  uint64_t scratch_gen = 0;                  // bumped whenever a scratch buffer a kernel argument points to moves
  std::vector<void *> allocs;
  size_t device_bytes = 0;
  // step statistics (gck_ext.h)
  bool stats_on = false;
  uint32_t stats_mask = 0;
  gck_stats stats{};
  std::vector<cudaEvent_t> ev_pool;
  size_t ev_used = 0;
  struct Mark { int cls; cudaEvent_t a, b; };
  std::vector<Mark> marks;
  uint64_t step_launches = 0;

  cudaEvent_t event() {
    if (ev_used == ev_pool.size()) {
      cudaEvent_t e;
      ck(cudaEventCreate(&e), "event");
      ev_pool.push_back(e);
    }
    return ev_pool[ev_used++];
  }

  void *dalloc(size_t n, const char *what) {
    void *p = nullptr;
    ck(cudaMalloc(&p, n ? n : 16), what);
    allocs.push_back(p);
    device_bytes += n;
    return p;
  }
  void dfree(void *p, size_t n) {
    if (!p) return;
    cudaFree(p);
    allocs.erase(std::remove(allocs.begin(), allocs.end(), p), allocs.end());
    device_bytes -= n;
  }
  ~gc_handle() {
    if (st) cudaStreamSynchronize(st);
    if (drafter) {
      drafter->st = nullptr;                 // the target's stream, destroyed below
      delete drafter;
      cudaSetDevice(dev);
    }
    for (void *p : allocs) cudaFree(p);
    if (plan_host) cudaFreeHost(plan_host);
    if (tok_host) cudaFreeHost(tok_host);
    if (kerr_host) cudaFreeHost(kerr_host);
    if (spec_out_host) cudaFreeHost(spec_out_host);
    for (auto &g : graphs) cudaGraphExecDestroy(g.exec);
    for (auto e : ev_pool) cudaEventDestroy(e);
    if (st) cudaStreamDestroy(st);
  }
};

namespace {

// -------------------------------------------------------------------------------------------- weights and relayout
const GgufTensor &tensor(const std::vector<std::unique_ptr<GgufFile>> &files, const std::string &name) {
  for (auto &f : files) {
    auto it = f->tensors.find(name);
    if (it != f->tensors.end()) return it->second;
  }
  fail(GC_E_WEIGHTS, "tensor %s not found in the weight files", name.c_str());
}

long long meta_int(const std::vector<std::unique_ptr<GgufFile>> &files, const std::string &k, long long dflt) {
  for (auto &f : files) {
    auto it = f->meta.find(k);
    if (it != f->meta.end()) return it->second.i;
  }
  return dflt;
}
double meta_f(const std::vector<std::unique_ptr<GgufFile>> &files, const std::string &k, double dflt) {
  for (auto &f : files) {
    auto it = f->meta.find(k);
    if (it != f->meta.end()) return it->second.f;
  }
  return dflt;
}

struct RowSrc {               // one source matrix of a (possibly concatenated / interleaved) weight
  const GgufTensor *t;
  int rows, cols;
};

// f32 -> f16 on the host (round to nearest even), for F32 checkpoints relaid to the F16 tile format
uint16_t h_f32_to_f16(float f) {
  __half h = __float2half_rn(f);
  return *reinterpret_cast<uint16_t *>(&h);
}

// Split-K of a tcgen05 weight (one persistent CTA per SM takes units b, b + sms, ...; a unit is a 128-row band over one
// K slice, slices differing by at most one 256-K tile). Chosen once per weight from its shape, never from the batch
// (batch invariance), to minimise the estimated time of a decode step's launch in tile times (about 1 us each): the
// busiest CTA's tiles, half a tile per unit (epilogue), and per slice the partials' write and read at 64 token rows
// (64 x N x 8 B at about 5 TB/s), plus a reduce launch (about 4 tiles) when no later kernel sums the slices.
int tc_splits(int NTW, int KT, int N, int sms, bool reader_sums) {
  int best = 1;
  double best_cost = 1e30;
  for (int sp = 1; sp <= std::min(16, KT); sp++) {
    const long units = static_cast<long>(NTW) * sp;
    const int base = KT / sp, extra = KT % sp;
    long max_tiles = 0, max_units = 0;
    for (int b = 0; b < sms && b < units; b++) {
      long tiles = 0, n = 0;
      for (long u = b; u < units; u += sms, n++) tiles += base + ((u % sp) < extra ? 1 : 0);
      max_tiles = std::max(max_tiles, tiles);
      max_units = std::max(max_units, n);
    }
    double cost = static_cast<double>(max_tiles) + 0.5 * static_cast<double>(max_units);
    if (sp > 1) cost += sp * (64.0 * N * 8.0 / 5e12 / 1.05e-6) + (reader_sums ? 0.0 : 4.0);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = sp;
    }
  }
  return best;
}

// Steps of one token tile (T <= 64) can run gate/up and down_proj as one chained launch (launch_gemm_tc_chain). Where
// the model allows it (a16, one GPU, gate/up and down_proj of one tcgen05 type in every layer), down_proj's split-K is
// chosen for the chained schedule: the busiest CTA's tiles in tile times, plus each slice's partials written and read
// at 64 rows. It is fixed for every step size alike (batch invariance), whether chaining is on or not.
void setup_chain(gc_handle *h) {
  if (h->layers.empty() || h->a8 || h->tp > 1) return;
  const Layer &l0 = h->layers[0];
  if ((l0.gu.type != kQ4_K && l0.gu.type != kQ8_0) || l0.dn.type != l0.gu.type) return;
  for (const Layer &ly : h->layers)
    if (ly.gu.type != l0.gu.type || ly.dn.type != l0.gu.type || ly.gu.splits != 1 || ly.gu.NT != l0.gu.NT ||
        ly.gu.KT != l0.gu.KT || ly.dn.NT != l0.dn.NT || ly.dn.KT != l0.dn.KT)
      return;
  int best = l0.dn.splits;
  double best_cost = 1e30;
  for (int sp = 1; sp <= std::min(16, l0.dn.KT); sp++) {
    double c = chain_schedule(l0.gu.NT, l0.gu.KT, l0.dn.NT, l0.dn.KT, sp, h->sms, nullptr, nullptr, nullptr);
    if (sp > 1) c += sp * (64.0 * l0.dn.N * 8.0 / 5e12 / 1.05e-6);
    if (c < best_cost - 1e-9) {
      best_cost = c;
      best = sp;
    }
  }
  for (Layer &ly : h->layers) ly.dn.splits = best;
  const int total = l0.gu.NT + l0.dn.NT * best;
  std::vector<int> sched(total), off(h->sms + 1);
  int ctas = 0;
  chain_schedule(l0.gu.NT, l0.gu.KT, l0.dn.NT, l0.dn.KT, best, h->sms, &ctas, sched.data(), off.data());
  int *d = static_cast<int *>(h->dalloc(static_cast<size_t>(total + ctas + 1) * 4, "chained launch schedule"));
  ck(cudaMemcpy(d, sched.data(), static_cast<size_t>(total) * 4, cudaMemcpyHostToDevice), "chained launch schedule");
  ck(cudaMemcpy(d + total, off.data(), static_cast<size_t>(ctas + 1) * 4, cudaMemcpyHostToDevice),
     "chained launch schedule");
  auto *cnt = static_cast<unsigned *>(h->dalloc(static_cast<size_t>(l0.dn.KT + 1) * 4, "chained launch counters"));
  ck(cudaMemset(cnt, 0, static_cast<size_t>(l0.dn.KT + 1) * 4), "chained launch counters");
  h->chain = ChainPlan{d, d + total, ctas, cnt, cnt + l0.dn.KT};
  h->chain_ok = true;
  if (const char *e = std::getenv("GCK_CHAIN")) h->chain_on = std::atoi(e) != 0;
}

// Build the tiled layout of a weight whose logical row n maps to (source, source row) by `rowmap`, on the host, and
// upload it. Tile (nt, kt) of kBM x kBK: Q4_K = 128 x 16 B headers then 128 x 128 B quants; Q8_0 = 128 x 8 fp16
// scales then 128 x 256 int8; F16 = 128 x 256 halves. Rows past N and columns past K are zero (weights of 0).
// k0: first source column (a tensor-parallel rank's slice of the input dimension; a multiple of 256 for Q4_K).
// reader_sums: the kernel after this weight's GEMM sums its split-K partials (RoPE after q/k/v, RMSNorm after o_proj
// and down_proj), so slices cost no reduce launch.
template <typename RowMap>
QWeight relayout(gc_handle *h, int type, int N, int K, RowMap rowmap, const char *what, int k0 = 0,
                 bool reader_sums = true) {
  QWeight w;
  w.type = type == kF32 ? kF16 : type;
  w.N = N;
  w.K = K;
  w.NT = (N + kBM - 1) / kBM;
  w.KT = (K + kBK - 1) / kBK;
  size_t tb = w.type == kF16 ? tile_bytes(kF16) : tc_tile_bytes(w.type);
  size_t total = tb * w.NT * w.KT;
  std::vector<uint8_t> host(total, 0);
  auto work = [&](int nt0, int nt1) {
    for (int nt = nt0; nt < nt1; nt++)
      for (int r = 0; r < kBM; r++) {
        int n = nt * kBM + r;
        if (n >= N) break;
        const GgufTensor *t = nullptr;
        int sr = 0;
        rowmap(n, t, sr);
        if (!t) continue;   // a padding row: zeros
        const uint8_t *row = t->data;
        const int Ksrc = static_cast<int>(t->dims[0]);   // the source row's full length
        for (int kt = 0; kt < w.KT; kt++) {
          uint8_t *tile = host.data() + (static_cast<size_t>(nt) * w.KT + kt) * tb;
          if (type == kQ4_K) {
            // header (d, dmin, 12 scale bytes) at r*16; then per 32-K sub-block g the row's 32 nibbles as 16 bytes at
            // [g][row r]: four words of 8 consecutive k, k = 0..7 at nibble positions 0, 4, 1, 5, 2, 6, 3, 7 (so the
            // kernel masks out f16 pairs of consecutive k). GGUF order: element 64j + l is the low nibble of quant byte
            // 32j + l for l < 32 (sub-block 2j), else the high nibble of byte 32j + l - 32 (sub-block 2j + 1).
            static const int kPos[8] = {0, 4, 1, 5, 2, 6, 3, 7};
            int nsb = K / 256;
            if (kt >= nsb) continue;
            const uint8_t *src = row + (static_cast<size_t>(sr) * (Ksrc / 256) + k0 / 256 + kt) * 144;
            std::memcpy(tile + r * 16, src, 16);
            const uint8_t *qs = src + 16;
            for (int g = 0; g < 8; g++) {
              uint32_t words[4] = {0, 0, 0, 0};
              for (int e = 0; e < 32; e++) {
                int j = g / 2;
                uint8_t byte = qs[32 * j + e];
                uint32_t nib = (g & 1) ? (byte >> 4) : (byte & 15);
                words[e / 8] |= nib << (4 * kPos[e % 8]);
              }
              std::memcpy(tile + kBM * 16 + (g * kBM + r) * 16, words, 16);
            }
          } else if (type == kQ8_0) {
            // the 8 block scales at r*16; block b's 32 quants as q + 128 (unsigned), 16 bytes each at [2b + half][row r]
            int nb = K / 32;
            for (int i = 0; i < 8; i++) {
              int b = kt * 8 + i;
              if (b >= nb) break;
              const uint8_t *src = row + (static_cast<size_t>(sr) * (Ksrc / 32) + k0 / 32 + b) * 34;
              std::memcpy(tile + r * 16 + i * 2, src, 2);
              for (int h2 = 0; h2 < 2; h2++) {
                uint8_t *dst = tile + kBM * 16 + ((2 * i + h2) * kBM + r) * 16;
                for (int e = 0; e < 16; e++) dst[e] = static_cast<uint8_t>(src[2 + 16 * h2 + e] ^ 0x80);
              }
            }
          } else {
            uint16_t *dst = reinterpret_cast<uint16_t *>(tile) + r * kBK;
            for (int c = 0; c < kBK; c++) {
              int k = kt * kBK + c;
              if (k >= K) break;
              const size_t si = static_cast<size_t>(sr) * Ksrc + k0 + k;
              if (type == kF16) dst[c] = reinterpret_cast<const uint16_t *>(row)[si];
              else dst[c] = h_f32_to_f16(reinterpret_cast<const float *>(row)[si]);
            }
          }
        }
      }
  };
  int nth = std::max(1, std::min(32, static_cast<int>(std::thread::hardware_concurrency())));
  std::vector<std::thread> th;
  int per = (w.NT + nth - 1) / nth;
  for (int i = 0; i < nth; i++) {
    int a = i * per, b = std::min(w.NT, a + per);
    if (a < b) th.emplace_back(work, a, b);
  }
  for (auto &x : th) x.join();
  uint8_t *dev = static_cast<uint8_t *>(h->dalloc(total, what));
  ck(cudaMemcpy(dev, host.data(), total, cudaMemcpyHostToDevice), what);
  w.data = dev;
  if (w.type == kF16) {
    // split-K (mma.sync kernel): the fewest K slices (a divisor of KT, at most 8) that give at least one CTA per SM
    w.splits = 1;
    for (int sp = 1; sp <= std::min(8, w.KT); sp++) {
      if (w.KT % sp) continue;
      w.splits = sp;
      if (w.NT * sp >= 148) break;
    }
  } else {
    w.splits = tc_splits(w.NT, w.KT, N, h->sms, reader_sums);
    w.gslices = gemv_slices(w.NT, w.KT, h->sms, reader_sums);
  }
  return w;
}

void check_type(const GgufTensor &t, int K) {
  if (t.type != kF32 && t.type != kF16 && t.type != kQ8_0 && t.type != kQ4_K)
    fail(GC_E_WEIGHTS, "tensor %s: ggml type %u is not supported (F32, F16, Q8_0, Q4_K)", t.name.c_str(), t.type);
  if ((t.type == kQ4_K && K % 256) || (t.type == kQ8_0 && K % 32))
    fail(GC_E_WEIGHTS, "tensor %s: row length %d does not fit its blocks", t.name.c_str(), K);
  if (t.dims.size() < 2 || static_cast<int>(t.dims[0]) != K)
    fail(GC_E_WEIGHTS, "tensor %s: row length %llu, expected %d", t.name.c_str(),
         static_cast<unsigned long long>(t.dims.empty() ? 0 : t.dims[0]), K);
}

const float *upload_f32(gc_handle *h, const GgufTensor &t, int n, const char *what) {
  std::vector<float> v(n);
  for (int i = 0; i < n; i++) {
    if (t.type == kF32) v[i] = reinterpret_cast<const float *>(t.data)[i];
    else if (t.type == kF16) v[i] = __half2float(reinterpret_cast<const __half *>(t.data)[i]);
    else fail(GC_E_WEIGHTS, "tensor %s: norm weights must be F32 or F16", t.name.c_str());
  }
  float *p = static_cast<float *>(h->dalloc(n * 4, what));
  ck(cudaMemcpy(p, v.data(), n * 4, cudaMemcpyHostToDevice), what);
  return p;
}

void load_model(gc_handle *h, const std::vector<std::unique_ptr<GgufFile>> &files) {
  std::string arch;
  for (auto &f : files) {
    auto it = f->meta.find("general.architecture");
    if (it != f->meta.end()) arch = it->second.s;
  }
  if (arch != "llama") fail(GC_E_WEIGHTS, "architecture '%s': this library runs llama-architecture GGUF", arch.c_str());
  h->L = static_cast<int>(meta_int(files, "llama.block_count", 0));
  h->d = static_cast<int>(meta_int(files, "llama.embedding_length", 0));
  h->F = static_cast<int>(meta_int(files, "llama.feed_forward_length", 0));
  h->H = static_cast<int>(meta_int(files, "llama.attention.head_count", 0));
  h->KVH = static_cast<int>(meta_int(files, "llama.attention.head_count_kv", h->H));
  h->eps = static_cast<float>(meta_f(files, "llama.attention.layer_norm_rms_epsilon", 1e-5));
  h->theta = static_cast<float>(meta_f(files, "llama.rope.freq_base", 1e4));
  if (h->L <= 0 || h->d <= 0 || h->H <= 0 || h->KVH <= 0 || h->F <= 0 || h->H % h->KVH)
    fail(GC_E_WEIGHTS, "llama metadata incomplete or inconsistent");
  h->dh = h->d / h->H;
  int G = h->H / h->KVH;
  if (h->dh != 64 && h->dh != 128) fail(GC_E_UNSUPPORTED, "head dim %d: this library runs 64 and 128", h->dh);
  if (16 % G) fail(GC_E_UNSUPPORTED, "GQA group %d: must divide 16", G);
  if (h->d % kBK || (h->H * h->dh) % kBK || h->d > 8192)
    fail(GC_E_UNSUPPORTED, "model width %d: must be a multiple of %d, at most 8192", h->d, kBK);
  h->qg_tokens = 16 / G;
  // tensor parallelism: this handle holds rank `rank` of `tp`: heads, kv heads and FFN columns split evenly, o_proj and
  // down_proj by their input columns (on 256-column super-block bounds), the head by vocabulary rows
  const int N = h->tp, rk = h->rank;
  if (N > 1) {
    if (h->KVH % N || h->H % N)
      fail(GC_E_UNSUPPORTED, "tensor parallelism %d: heads %d and kv heads %d must divide evenly", N, h->H, h->KVH);
    if ((h->H / N * h->dh) % kBK || (h->F / N) % kBK || h->F % N)
      fail(GC_E_UNSUPPORTED, "tensor parallelism %d: per-rank o_proj and down_proj inputs must be multiples of %d", N, kBK);
  }
  const GgufTensor &emb = tensor(files, "token_embd.weight");
  if (emb.dims.size() < 2 || static_cast<int>(emb.dims[0]) != h->d) fail(GC_E_WEIGHTS, "token_embd.weight shape");
  h->vocab = static_cast<int>(emb.dims[1]);
  check_type(emb, h->d);
  h->emb_type = static_cast<int>(emb.type);
  h->emb_row_bytes = emb.bytes / h->vocab;
  uint8_t *e = static_cast<uint8_t *>(h->dalloc(emb.bytes, "token_embd"));
  ck(cudaMemcpy(e, emb.data, emb.bytes, cudaMemcpyHostToDevice), "token_embd");
  h->emb = e;
  const int dq_all = h->H * h->dh, F_all = h->F;
  const int dq = h->H / N * h->dh, dkv = h->KVH / N * h->dh, Fr = h->F / N;   // this rank's slices
  for (int l = 0; l < h->L; l++) {
    std::string b = "blk." + std::to_string(l) + ".";
    Layer ly;
    const GgufTensor &tq = tensor(files, b + "attn_q.weight"), &tk = tensor(files, b + "attn_k.weight"),
                     &tv = tensor(files, b + "attn_v.weight"), &to = tensor(files, b + "attn_output.weight"),
                     &tg = tensor(files, b + "ffn_gate.weight"), &tu = tensor(files, b + "ffn_up.weight"),
                     &td = tensor(files, b + "ffn_down.weight");
    for (auto *t : {&tq, &tk, &tv, &tg, &tu}) check_type(*t, h->d);
    check_type(to, dq_all);
    check_type(td, F_all);
    if (tq.type != tk.type || tq.type != tv.type || tg.type != tu.type)
      fail(GC_E_WEIGHTS, "layer %d: q/k/v (and gate/up) must share one type", l);
    ly.qkv = relayout(h, static_cast<int>(tq.type), dq + 2 * dkv, h->d, [&](int n, const GgufTensor *&t, int &r) {
      if (n < dq) { t = &tq; r = rk * dq + n; }
      else if (n < dq + dkv) { t = &tk; r = rk * dkv + n - dq; }
      else { t = &tv; r = rk * dkv + n - dq - dkv; }
    }, "attn_qkv");
    ly.o = relayout(h, static_cast<int>(to.type), h->d, dq, [&](int n, const GgufTensor *&t, int &r) { t = &to; r = n; },
                    "attn_output", rk * dq);
    // gate/up rows interleaved: row 2i of a 128-row tile is gate feature tile * 64 + i, row 2i + 1 its up row, so a
    // SwiGLU epilogue finds a feature's two values in neighbouring lanes of one warp
    int Fp = (Fr + 63) / 64 * 64;
    ly.gu = relayout(h, static_cast<int>(tg.type), 2 * Fp, h->d, [&](int n, const GgufTensor *&t, int &r) {
      int tile = n / 128, w = n % 128;
      int f = tile * 64 + w / 2;
      t = (w & 1) == 0 ? &tg : &tu;
      r = rk * Fr + std::min(f, Fr - 1);
      if (f >= Fr) t = nullptr;
    }, "ffn_gate_up", 0, false);
    ly.gu.N = 2 * Fp;
    ly.dn = relayout(h, static_cast<int>(td.type), h->d, Fr, [&](int n, const GgufTensor *&t, int &r) { t = &td; r = n; },
                     "ffn_down", rk * Fr);
    ly.attn_norm = upload_f32(h, tensor(files, b + "attn_norm.weight"), h->d, "attn_norm");
    ly.ffn_norm = upload_f32(h, tensor(files, b + "ffn_norm.weight"), h->d, "ffn_norm");
    h->layers.push_back(ly);
  }
  h->out_norm = upload_f32(h, tensor(files, "output_norm.weight"), h->d, "output_norm");
  const GgufTensor &th = tensor(files, "output.weight");
  check_type(th, h->d);
  const int Vr = (h->vocab + N - 1) / N;
  h->vocab0 = rk * Vr;
  h->vocab_rows = std::max(0, std::min(h->vocab, h->vocab0 + Vr) - h->vocab0);
  h->head = relayout(h, static_cast<int>(th.type), h->vocab_rows, h->d,
                     [&](int n, const GgufTensor *&t, int &r) { t = &th; r = h->vocab0 + n; }, "output", 0, false);
  // tensor parallelism: o_proj and down_proj in one K slice each. Their split-K partials would cross NVLink in the
  // all-reduce (splits times the bytes), and a rank's slice of K is already N times shorter.
  if (N > 1)
    for (auto &ly : h->layers) ly.o.splits = ly.dn.splits = 1;
  // from here on the handle's head counts and FFN width are its own slices
  h->H /= N;
  h->KVH /= N;
  h->F = Fr;
}

}  // namespace

namespace {

// TMA tensor maps over an activation buffer [rows, K] f16 row-major: boxes of 64 K (128 B, swizzled) x nt rows
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

void build_tma(TmaSet &ts, void *buf, int rows, int K) {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    ck(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q), "cuTensorMapEncodeTiled");
    if (!p || q != cudaDriverEntryPointSuccess) fail(GC_E_DEVICE, "cuTensorMapEncodeTiled is not available");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  const int nts[5] = {16, 32, 64, 128, 256};
  for (int i = 0; i < 5; i++) {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
    cuuint32_t box[2] = {64, static_cast<cuuint32_t>(nts[i])};
    cuuint32_t es[2] = {1, 1};
    CUresult r = fn(&ts.m[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, buf, dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail(GC_E_DEVICE, "tensor map of an activation buffer: CUresult %d", static_cast<int>(r));
  }
}

void build_rope(gc_handle *h) {
  // ref.py:31: inv = theta ** (-arange(0, dh, 2) / dh) in float32; angle = inv * p in float32
  int half = h->dh / 2;
  std::vector<float2> tab(static_cast<size_t>(h->max_ctx) * half);
  std::vector<float> inv(half);
  for (int i = 0; i < half; i++)
    inv[i] = std::pow(h->theta, -(static_cast<float>(2 * i) / static_cast<float>(h->dh)));
  for (int p = 0; p < h->max_ctx; p++)
    for (int i = 0; i < half; i++) {
      float a = inv[i] * static_cast<float>(p);
      tab[static_cast<size_t>(p) * half + i] = make_float2(static_cast<float>(std::cos(static_cast<double>(a))),
                                                           static_cast<float>(std::sin(static_cast<double>(a))));
    }
  h->rope = static_cast<float2 *>(h->dalloc(vbytes(tab), "rope table"));
  ck(cudaMemcpy(h->rope, tab.data(), vbytes(tab), cudaMemcpyHostToDevice), "rope table");
}

template <typename T>
T *grow(gc_handle *h, T *p, size_t &cap, size_t need, const char *what) {
  if (need <= cap) return p;
  if (p) {
    cudaStreamSynchronize(h->st);
    h->dfree(p, cap);
  }
  size_t n = std::max(need, cap * 3 / 2);
  p = static_cast<T *>(h->dalloc(n, what));
  cap = n;
  return p;
}

std::string read_file(const std::string &path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) fail(GC_E_MANIFEST, "%s: cannot read", path.c_str());
  std::stringstream ss;
  ss << f.rdbuf();
  return ss.str();
}

}  // namespace

// ============================================================================================== static commit scratch
// gck_commit_static keeps its scratch (the move list and the staged rows) in this fixed device array instead of
// memory the handle allocates, so that callers that may not allocate device memory can commit tree paths. In host
// code the name is only a stand-in: the device address comes from cudaGetSymbolAddress, once per device, with that
// device current. gc_open looks it up for every device it opens (open_device): under CUDA's lazy module loading that
// lookup is what loads this file's module and commits its 16 MiB on the device, so it happens at open, where the
// handle allocates anyway, and never inside a commit. The device holds the array until the process exits.
constexpr size_t kCommitStaticBytes = static_cast<size_t>(16) << 20;
static __device__ __align__(256) unsigned char g_commit_static[kCommitStaticBytes];

namespace {
std::mutex g_static_mu;
void *g_static_addr[256] = {};

void *commit_static_address(int dev) {
  std::lock_guard<std::mutex> lk(g_static_mu);
  if (dev < 0 || dev >= 256) fail(GC_E_DEVICE, "device ordinal %d", dev);
  if (!g_static_addr[dev]) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_commit_static);
    if (e != cudaSuccess || !p) {
      cudaGetLastError();
      fail(GC_E_DEVICE, "cudaGetSymbolAddress of the static commit scratch: %s", cudaGetErrorString(e));
    }
    g_static_addr[dev] = p;
  }
  return g_static_addr[dev];
}
}  // namespace

// ============================================================================================== exported ABI
namespace {

struct OpenCfg {
  int ncol = 0, maxctx = 0, max_cols = 0, pool_tune = 0, tp = 1;
  bool tolerance = true;   // every opened bucket's determinism is "tolerance" (the GEMV for a few token rows)
  uint32_t pool_blocks = 0;
  std::string kv, kv_scale, act;   // act: "a16" (f16 activations) or "a8" (per-token int8 activations)
  int spec_k = 0;                  // a speculative pair's target: drafts per round
};

// The configuration of the buckets ids[0 .. n) of the manifest's bucket list: the widest columns and context, and the
// KV dtype, activation type and tensor-parallel degree they must agree on.
OpenCfg bucket_cfg(const Json &bl, const char *const *ids, uint32_t n, uint32_t pool_blocks) {
  OpenCfg c;
  c.pool_blocks = pool_blocks;
  for (uint32_t i = 0; i < n; i++) {
    if (!ids[i]) fail(GC_E_ARG, "gc_open: null bucket id");
    const Json *b = nullptr;
    for (auto &x : bl.arr)
      if (x.str_or("id", "") == ids[i]) b = &x;
    if (!b) fail(GC_E_MANIFEST, "bucket %s is not in the manifest", ids[i]);
    c.ncol = std::max(c.ncol, static_cast<int>(b->num_or("ncol", 1)));
    c.maxctx = std::max(c.maxctx, static_cast<int>(b->num_or("maxctx", 4096)));
    std::string bkv = b->str_or("kv", "f16");
    if (!c.kv.empty() && bkv != c.kv) fail(GC_E_MANIFEST, "buckets disagree on the KV dtype");
    c.kv = bkv;
    std::string bact = b->str_or("act", "a16");
    if (!c.act.empty() && bact != c.act) fail(GC_E_MANIFEST, "buckets disagree on the activation type (act)");
    c.act = bact;
    c.tolerance = c.tolerance && b->str_or("determinism", "batch_invariant") == "tolerance";
    const int btp = static_cast<int>(b->num_or("tp", 1));
    if (i && btp != c.tp) fail(GC_E_MANIFEST, "buckets disagree on the tensor-parallel degree");
    c.tp = btp;
    if (const Json *t = b->get("tune")) {
      c.max_cols = std::max(c.max_cols, static_cast<int>(t->num_or("max_cols", 0)));
      c.pool_tune = std::max(c.pool_tune, static_cast<int>(t->num_or("pool_blocks", 0)));
      c.kv_scale = t->str_or("kv_scale", c.kv_scale);
    }
  }
  if (c.kv != "f16" && c.kv != "fp8") fail(GC_E_MANIFEST, "kv dtype %s: f16 or fp8", c.kv.c_str());
  if (c.act != "a16" && c.act != "a8") fail(GC_E_MANIFEST, "act %s: a16 or a8", c.act.c_str());
  if (c.act == "a8" && c.tp > 1)
    fail(GC_E_UNSUPPORTED, "a8 activations under tensor parallelism: a rank sees only its slice of a row, so the "
         "per-token scale would differ from one GPU's");
  if (c.tp != 1 && c.tp != 2 && c.tp != 4 && c.tp != 8) fail(GC_E_MANIFEST, "tensor-parallel degree %d: 1, 2, 4 or 8", c.tp);
  return c;
}

// One device's state: checks the device, loads (this rank's slices of) the weights, allocates scratch and the KV pool.
void open_device(gc_handle *h, int dev, const std::vector<std::unique_ptr<GgufFile>> &files, const OpenCfg &c, int rank) {
  cudaDeviceProp prop;
  ck(cudaGetDeviceProperties(&prop, dev), "cudaGetDeviceProperties");
  if (prop.major != 10 || prop.minor != 0)
    fail(GC_E_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a (B200)", dev, prop.major, prop.minor);
  ck(cudaSetDevice(dev), "cudaSetDevice");
  h->dev = dev;
  h->rank = rank;
  h->tp = c.tp;
  h->sms = prop.multiProcessorCount;
  ck(cudaStreamCreateWithFlags(&h->st, cudaStreamNonBlocking), "stream");
  // the static commit array's address on this device (loads its module and commits the array now, not in a commit)
  commit_static_address(dev);
  gemm_init();
  gemm_tc_init();
  load_model(h, files);
  h->max_seqs = std::max(1, c.ncol);
  h->max_ctx = std::max(kBlock, c.maxctx);
  h->max_cols = c.max_cols > 0 ? c.max_cols : 2048;
  h->kv_fp8 = c.kv == "fp8";
  h->page_scale = h->kv_fp8 && c.kv_scale != "unit";
  // batch-invariant buckets run the tcgen05 GEMM at every width (a row's arithmetic never depends on the batch)
  h->gemv_max_t = c.tolerance && c.tp == 1 ? kGemvMaxT : 0;
  h->a8 = c.act == "a8";
  setup_chain(h);
  build_rope(h);
  // KV pool: [L][nblk][KVH][16][dh] for K and for V, plus fp8 page exponents [L][nblk][KVH][2]
  const size_t esz = h->kv_fp8 ? 1 : 2;
  h->page_bytes = static_cast<size_t>(h->KVH) * kBlock * h->dh * esz;
  size_t per_block = 2 * h->page_bytes * h->L + (h->kv_fp8 ? static_cast<size_t>(h->L) * h->KVH * 2 : 0);
  size_t nblk = c.pool_blocks ? c.pool_blocks : c.pool_tune;
  // scratch first, so that "what fits" is measured after it
  const int T = h->max_cols, d = h->d;
  const int wq = (h->H + 2 * h->KVH) * h->dh;
  int Fpad = h->layers[0].dn.KT * kBK;
  h->x = static_cast<float *>(h->dalloc(static_cast<size_t>(T) * d * 4, "x"));
  h->h = static_cast<__half *>(h->dalloc(static_cast<size_t>(T) * d * 2, "h"));
  h->qkv = static_cast<float *>(h->dalloc(static_cast<size_t>(T) * wq * 4, "qkv"));
  h->q = static_cast<__half *>(h->dalloc(static_cast<size_t>(T) * h->H * h->dh * 2, "q"));
  h->att = static_cast<__half *>(h->dalloc(static_cast<size_t>(T) * h->H * h->dh * 2, "att"));
  h->act = static_cast<__half *>(h->dalloc(static_cast<size_t>(T) * Fpad * 2, "act"));
  ck(cudaMemset(h->act, 0, static_cast<size_t>(T) * Fpad * 2), "act");
  h->logits = static_cast<float *>(h->dalloc(static_cast<size_t>(T) * std::max(1, h->vocab_rows) * 4, "logits"));
  h->argmax = static_cast<int *>(h->dalloc(static_cast<size_t>(T) * 4, "argmax"));
  if (h->a8) {
    h->h_scale = static_cast<float *>(h->dalloc(static_cast<size_t>(T) * 4, "a8 scales"));
    h->att_scale = static_cast<float *>(h->dalloc(static_cast<size_t>(T) * 4, "a8 scales"));
    h->act_scale = static_cast<float *>(h->dalloc(static_cast<size_t>(T) * 4, "a8 scales"));
  }
  h->arg_scratch = static_cast<int *>(h->dalloc(static_cast<size_t>(T) * 8 * 2 * 4, "argmax parts"));
  if (h->tp > 1) {
    h->tp_y = static_cast<float *>(h->dalloc(static_cast<size_t>(T) * d * 4, "tensor-parallel partial sums"));
    // o_proj / down_proj split-K partials of this rank go straight into the buffer: [splits][T][d]
    for (auto &ly : h->layers) h->tp_splits = std::max({h->tp_splits, ly.o.splits, ly.dn.splits});
    for (int b = 0; b < 2; b++)
      h->tp_bufs[b] = static_cast<float *>(
          h->dalloc(static_cast<size_t>(h->tp_splits) * T * d * 4, "tensor-parallel partials"));
    h->tp_flags = static_cast<unsigned long long *>(h->dalloc(2 * sizeof(unsigned long long), "tensor-parallel flags"));
    ck(cudaMemset(h->tp_flags, 0, 2 * sizeof(unsigned long long)), "tensor-parallel flags");
    h->sig_counter = static_cast<unsigned *>(h->dalloc(16, "signal counter"));
    ck(cudaMemset(h->sig_counter, 0, 16), "signal counter");
    h->tp_pick = static_cast<int *>(h->dalloc(static_cast<size_t>(h->tp + 1) * T * 2 * 4, "tensor-parallel argmax"));
  }
  ck(cudaMallocHost(&h->tok_host, static_cast<size_t>(T) * 4), "pinned tokens");
  h->kerr = static_cast<int *>(h->dalloc(16, "error word"));
  ck(cudaMemset(h->kerr, 0, 16), "error word");
  ck(cudaMallocHost(&h->kerr_host, 16), "pinned error word");
  build_tma(h->tma_h, h->h, T, d);
  build_tma(h->tma_att, h->att, T, h->H * h->dh);
  build_tma(h->tma_act, h->act, T, Fpad);
  if (!nblk) {
    size_t fr = 0, tot = 0;
    ck(cudaMemGetInfo(&fr, &tot), "cudaMemGetInfo");
    size_t reserve = static_cast<size_t>(4) << 30;
    nblk = fr > reserve ? (fr - reserve) / per_block : 0;
    nblk = std::min<size_t>(nblk, static_cast<size_t>(h->max_seqs) * ((h->max_ctx + kBlock - 1) / kBlock) + 64);
  }
  if (nblk < 1 || nblk > (1u << 26)) fail(GC_E_DEVICE, "KV pool of %zu blocks: out of memory", nblk);
  h->nblk = static_cast<int>(nblk);
  h->layer_bytes = h->page_bytes * nblk;
  h->kc = static_cast<uint8_t *>(h->dalloc(h->layer_bytes * h->L, "KV pool K"));
  h->vc = static_cast<uint8_t *>(h->dalloc(h->layer_bytes * h->L, "KV pool V"));
  ck(cudaMemset(h->kc, 0, h->layer_bytes * h->L), "KV pool");
  ck(cudaMemset(h->vc, 0, h->layer_bytes * h->L), "KV pool");
  if (h->kv_fp8) {
    h->exps_layer = nblk * h->KVH * 2;
    h->exps = static_cast<int8_t *>(h->dalloc(h->exps_layer * h->L, "KV page exponents"));
    ck(cudaMemset(h->exps, 0, h->exps_layer * h->L), "KV page exponents");
  }
  h->slots.resize(h->max_seqs);
  h->tab_stride = (h->max_ctx + kBlock - 1) / kBlock;
  h->tables = static_cast<uint32_t *>(h->dalloc(static_cast<size_t>(h->max_seqs) * h->tab_stride * 4, "block tables"));
  ck(cudaMemset(h->tables, 0, static_cast<size_t>(h->max_seqs) * h->tab_stride * 4), "block tables");
  if (const char *e = std::getenv("GCK_GRAPH")) h->graphs_on = std::atoi(e) != 0;
  h->tc_pairs = tc_pair_clusters();
  if (const char *e = std::getenv("GCK_PAIR")) h->tc_pairs = std::atoi(e) != 0 ? h->tc_pairs : 0;
  ck(cudaStreamSynchronize(h->st), "open");
}

// NCCL, loaded when a handle first needs it (tensor parallelism): the library does not link it
struct Nccl {
  decltype(&ncclCommInitAll) init_all = nullptr;
  decltype(&ncclCommDestroy) destroy = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
};
const Nccl &nccl() {
  static Nccl n;
  static std::once_flag once;
  static std::string why;
  std::call_once(once, [] {
    void *lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!lib) {
      why = dlerror();
      return;
    }
    n.init_all = reinterpret_cast<decltype(&ncclCommInitAll)>(dlsym(lib, "ncclCommInitAll"));
    n.destroy = reinterpret_cast<decltype(&ncclCommDestroy)>(dlsym(lib, "ncclCommDestroy"));
    n.all_reduce = reinterpret_cast<decltype(&ncclAllReduce)>(dlsym(lib, "ncclAllReduce"));
    n.all_gather = reinterpret_cast<decltype(&ncclAllGather)>(dlsym(lib, "ncclAllGather"));
    n.error_string = reinterpret_cast<decltype(&ncclGetErrorString)>(dlsym(lib, "ncclGetErrorString"));
  });
  if (!n.init_all || !n.destroy || !n.all_reduce || !n.all_gather || !n.error_string)
    fail(GC_E_DEVICE, "tensor parallelism needs NCCL (libnccl.so.2): %s", why.empty() ? "symbols missing" : why.c_str());
  return n;
}
void nck(ncclResult_t r, const char *what) {
  if (r != ncclSuccess) fail(GC_E_DEVICE, "%s: NCCL error %d (%s)", what, static_cast<int>(r), nccl().error_string(r));
}

// one communicator per rank, all in this process
void init_tp(gc_handle *g) {
  const Nccl &n = nccl();
  std::vector<ncclComm_t> comms(g->tp);
  std::vector<int> devs(g->tp);
  for (int r = 0; r < g->tp; r++) devs[r] = g->ranks[r]->dev;
  nck(n.init_all(comms.data(), g->tp, devs.data()), "ncclCommInitAll");
  for (int r = 0; r < g->tp; r++) g->ranks[r]->comm = comms[r];
  if (g->tp > kMaxTp) fail(GC_E_UNSUPPORTED, "tensor parallelism above %d", kMaxTp);
  // peer access between every pair: the all-reduce reads the other ranks' buffers over NVLink (plain loads, no multicast)
  bool p2p = true;
  for (int i = 0; i < g->tp && p2p; i++)
    for (int j = 0; j < g->tp && p2p; j++) {
      if (i == j) continue;
      int can = 0;
      ck(cudaDeviceCanAccessPeer(&can, devs[i], devs[j]), "cudaDeviceCanAccessPeer");
      if (!can) {
        p2p = false;
        break;
      }
      ck(cudaSetDevice(devs[i]), "cudaSetDevice");
      cudaError_t e = cudaDeviceEnablePeerAccess(devs[j], 0);
      if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
      else ck(e, "cudaDeviceEnablePeerAccess");
    }
  for (int r = 0; r < g->tp; r++) {
    gc_handle *h = g->ranks[r];
    h->tp_p2p = p2p;
    h->peers.n = g->tp;
    h->peers.rank = r;
    h->peers.err = h->kerr;
    for (int k = 0; k < g->tp; k++) {
      h->peers.buf[k][0] = g->ranks[k]->tp_bufs[0];
      h->peers.buf[k][1] = g->ranks[k]->tp_bufs[1];
      h->peers.flag[k] = g->ranks[k]->tp_flags;
    }
  }
}

}  // namespace

extern "C" {

GC_API uint32_t gc_abi_version(void) { return GC_ABI_VERSION; }

GC_API const char *gc_last_error(gc_handle *h) { return h ? h->err.c_str() : g_open_err.c_str(); }

GC_API int gc_open(const gc_open_params *p, gc_handle **out) {
  if (out) *out = nullptr;
  gc_handle *h = nullptr;
  try {
    if (!p || !out) fail(GC_E_ARG, "gc_open: null argument");
    // fields read: up to n_buckets and pool_blocks; anything the caller's struct does not have reads as zero
    gc_open_params P{};
    std::memcpy(&P, p, std::min<size_t>(p->size, sizeof P));
    if (p->size < offsetof(gc_open_params, pool_blocks) + sizeof(uint32_t)) fail(GC_E_ARG, "gc_open: struct size %u", p->size);
    const bool spec = (P.flags & GC_OPEN_SPEC) != 0;
    if (const char *e = std::getenv("GCK_PDL")) g_pdl = std::atoi(e) != 0;
    if (!P.pack_dir) fail(GC_E_ARG, "gc_open: no pack_dir");
    if (!P.n_buckets || !P.buckets) fail(GC_E_ARG, "gc_open: no bucket ids");
    if (spec && P.n_buckets != 2) fail(GC_E_ARG, "gc_open: a speculative pair opens two buckets {target, drafter}");
    // manifest: the requested buckets
    Json m;
    try {
      std::string txt = read_file(std::string(P.pack_dir) + "/manifest.json");
      m = JsonParser(txt).parse();
    } catch (const std::runtime_error &e) {
      fail(GC_E_MANIFEST, "manifest.json: %s", e.what());
    }
    const Json *bl = m.get("buckets");
    if (!bl || bl->kind != Json::Arr) fail(GC_E_MANIFEST, "manifest.json has no buckets");
    // a speculative pair's target and drafter buckets each configure their own model; a ladder's buckets one
    OpenCfg c = bucket_cfg(*bl, P.buckets, spec ? 1 : P.n_buckets, P.pool_blocks);
    OpenCfg cd;
    if (spec) {
      cd = bucket_cfg(*bl, P.buckets + 1, 1, 0);
      std::string pol = P.spec_policy ? P.spec_policy : "";
      if (pol.empty()) {
        // the pack's pair: manifest spec[] entry {target, drafter, policy {kind, K}}
        if (const Json *sp = m.get("spec"))
          for (auto &x : sp->arr)
            if (x.str_or("target", "") == P.buckets[0] && x.str_or("drafter", "") == P.buckets[1])
              if (const Json *po = x.get("policy")) {
                const Json *K = po->get("K");
                pol = po->str_or("kind", "") + ":" +
                      (K ? (K->kind == Json::Str ? K->str : std::to_string(static_cast<int>(K->num))) : "");
              }
      }
      if (pol.rfind("ar:", 0) != 0)
        fail(GC_E_UNSUPPORTED, "speculative policy '%s': this library runs ar:K (a draft model, K greedy drafts a round)",
             pol.c_str());
      c.spec_k = std::atoi(pol.c_str() + 3);
      if (c.spec_k < 1 || c.spec_k > 15) fail(GC_E_ARG, "speculative policy '%s': K must be 1 .. 15", pol.c_str());
      if (c.tp != 1 || cd.tp != 1) fail(GC_E_UNSUPPORTED, "a speculative pair runs on one GPU");
      // one linear stream: each model gets a pool of one whole context (every position a round can reach)
      c.ncol = cd.ncol = 1;
      cd.maxctx = c.maxctx;
      c.pool_blocks = cd.pool_blocks = static_cast<uint32_t>((c.maxctx + kBlock - 1) / kBlock + 1);
      c.tolerance = cd.tolerance = false;     // rounds verify against chain rows: the batch-invariant path only
    }
    // weights: the target's files, then (a speculative pair) a NULL entry and the drafter's
    std::vector<std::unique_ptr<GgufFile>> files, dfiles;
    if (!P.weights || !P.n_weights) fail(GC_E_WEIGHTS, "no weight files");
    bool after_null = false;
    for (uint32_t i = 0; i < P.n_weights; i++) {
      if (!P.weights[i]) {
        after_null = true;
        if (!spec) break;
        continue;
      }
      try {
        (after_null ? dfiles : files).emplace_back(new GgufFile(P.weights[i]));
      } catch (const std::runtime_error &e) {
        fail(GC_E_WEIGHTS, "%s", e.what());
      }
    }
    if (files.empty()) fail(GC_E_WEIGHTS, "no weight files");
    if (spec && dfiles.empty()) fail(GC_E_WEIGHTS, "a speculative pair needs the drafter's weight files after a NULL entry");
    // devices: `device` (or the current one) and, with tensor parallelism, the next tp - 1
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
      cudaGetLastError();
      fail(GC_E_DEVICE, "no CUDA device");
    }
    int dev = P.device;
    if (dev < 0) ck(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev + c.tp > ndev)
      fail(GC_E_DEVICE, "devices %d .. %d: only %d present", dev, dev + c.tp - 1, ndev);
    h = new gc_handle();
    if (c.tp == 1) {
      open_device(h, dev, files, c, 0);
      if (spec) {
        // the drafter: a second model on the same device, run on the target's stream (a round's launches are one
        // ordered sequence); its own weights, KV pool and scratch
        h->drafter = new gc_handle();
        open_device(h->drafter, dev, dfiles, cd, 0);
        ck(cudaSetDevice(dev), "cudaSetDevice");
        ck(cudaStreamDestroy(h->drafter->st), "stream");
        h->drafter->st = h->st;
        if (h->drafter->vocab != h->vocab)
          fail(GC_E_WEIGHTS, "drafter vocabulary %d differs from the target's %d", h->drafter->vocab, h->vocab);
        h->spec_k = c.spec_k;
        h->max_seqs = 1;
        h->slots.assign(1, Slot{});
        for (int b = 0; b < (h->max_ctx + kBlock - 1) / kBlock; b++) h->spec_table.push_back(static_cast<uint32_t>(b));
        h->spec_out = static_cast<int *>(h->dalloc(static_cast<size_t>(h->spec_k + 2) * 4, "speculative round"));
        ck(cudaMallocHost(&h->spec_out_host, static_cast<size_t>(h->spec_k + 2) * 4), "pinned speculative round");
      }
    } else {
      h->tp = c.tp;
      h->dev = dev;
      for (int r = 0; r < c.tp; r++) {
        h->ranks.push_back(new gc_handle());
        h->ranks.back()->tp = c.tp;
        h->ranks.back()->rank = r;
      }
      // the ranks load in parallel (each relays its own slices out)
      std::vector<std::thread> th;
      std::vector<std::string> errs(c.tp);
      std::vector<int> codes(c.tp, GC_OK);
      for (int r = 0; r < c.tp; r++)
        th.emplace_back([&, r] {
          try {
            open_device(h->ranks[r], dev + r, files, c, r);
          } catch (const GcError &e) {
            codes[r] = e.code;
            errs[r] = e.msg;
          } catch (const std::exception &e) {
            codes[r] = GC_E_DEVICE;
            errs[r] = e.what();
          }
        });
      for (auto &t : th) t.join();
      for (int r = 0; r < c.tp; r++)
        if (codes[r] != GC_OK) fail(codes[r], "rank %d (device %d): %s", r, dev + r, errs[r].c_str());
      init_tp(h);
      gc_handle *r0 = h->ranks[0];
      h->vocab = r0->vocab;
      h->max_seqs = r0->max_seqs;
      h->max_cols = r0->max_cols;
      h->max_ctx = r0->max_ctx;
      h->nblk = r0->nblk;
      h->L = r0->L;
      h->KVH = r0->KVH * c.tp;
      h->dh = r0->dh;
      h->kv_fp8 = r0->kv_fp8;
      for (gc_handle *r : h->ranks) {
        h->layer_bytes += r->layer_bytes;
        h->exps_layer += r->exps_layer;
        h->device_bytes += r->device_bytes;
      }
      h->slots.resize(h->max_seqs);
    }
    files.clear();
    *out = h;
    return GC_OK;
  } catch (const GcError &e) {
    g_open_err = e.msg;
    gc_close(h);
    return e.code;
  } catch (const std::exception &e) {
    g_open_err = e.what();
    gc_close(h);
    return GC_E_DEVICE;
  }
}

GC_API int gc_layout_get(gc_handle *h, gc_layout *o) {
  if (!h || !o || o->size < 8) return GC_E_ARG;
  gc_layout l{};
  l.size = sizeof l;
  l.flags = GC_L_PAGED | GC_L_DEVICE_ARGMAX;
  if (h->drafter) {
    // a speculative pair: one linear stream whose single page is the whole context (gc.h:87-131); a round of a step
    // verifies spec_k drafts and the anchor
    l.flags = GC_L_SPEC | GC_L_DEVICE_ARGMAX;
    l.vocab = h->vocab;
    l.max_cols = h->max_cols;
    l.max_seqs = 1;
    l.max_ctx = h->max_ctx;
    l.block_size = h->max_ctx;
    l.num_blocks = 1;
    l.layers = h->L;
    l.kv_heads = h->KVH;
    l.head_dim = h->dh;
    l.kv_dtype = h->kv_fp8 ? GC_KV_FP8 : GC_KV_F16;
    l.spec_width = h->spec_k + 1;
    l.kv_bytes = 2 * h->layer_bytes * h->L + h->exps_layer * h->L + 2 * h->drafter->layer_bytes * h->drafter->L +
                 h->drafter->exps_layer * h->drafter->L;
    l.device_bytes = h->device_bytes + h->drafter->device_bytes;
    uint32_t n = std::min<uint32_t>(o->size, sizeof l);
    std::memcpy(o, &l, n);
    o->size = n;
    return GC_OK;
  }
  l.vocab = h->vocab;
  l.max_cols = h->max_cols;
  l.max_seqs = h->max_seqs;
  l.max_ctx = h->max_ctx;
  l.block_size = kBlock;
  l.num_blocks = h->nblk;
  l.layers = h->L;
  l.kv_heads = h->KVH;
  l.head_dim = h->dh;
  l.kv_dtype = h->kv_fp8 ? GC_KV_FP8 : GC_KV_F16;
  l.kv_bytes = 2 * h->layer_bytes * h->L + h->exps_layer * h->L;
  l.device_bytes = h->device_bytes;
  uint32_t n = std::min<uint32_t>(o->size, sizeof l);
  std::memcpy(o, &l, n);
  o->size = n;
  return GC_OK;
}

}  // extern "C"

// ============================================================================================== the step
namespace {

struct HostPlan {
  std::vector<int> tok_id, rope_pos, kv_row, first_tok, want_tok, paths;
  std::vector<Item> items;
  std::vector<QGroup> qgroups;
  std::vector<AttnWork> work;
  std::vector<uint2> patches;      // (entry of the device block tables, block id): where a table differs from its mirror
  int n_parts = 0, nw = 1, tree_cta = 0, split = kSplit;
};

struct WorkIn {
  uint32_t flags;
  uint64_t sid;
  uint32_t pos, n;
  const int32_t *tokens, *parents;
  const uint32_t *blocks;
  uint32_t nblocks, want;
};

Slot *find_slot(gc_handle *h, uint64_t sid, bool make) {
  Slot *fr = nullptr;
  for (auto &s : h->slots) {
    if (s.used && s.sid == sid) return &s;
    if (!s.used && !fr) fr = &s;
  }
  if (make && fr) {
    fr->used = true;
    fr->sid = sid;
    return fr;
  }
  return nullptr;
}

void build_plan(gc_handle *h, const std::vector<WorkIn> &ws, HostPlan &pl) {
  const int G = h->H / h->KVH, QG = h->qg_tokens;
  int T = 0;
  bool multi = false;
  for (auto &w : ws) {
    Item it{};
    it.pos = static_cast<int>(w.pos);
    it.ntok = static_cast<int>(w.n);
    it.tok0 = T;
    // the item's table: its slot's row of the device tables, patched where it differs from the slot's mirror
    Slot *sl = find_slot(h, w.sid, true);
    if (!sl) fail(GC_E_STATE, "no free sequence slot (%d in use)", h->max_seqs);
    const int slot = static_cast<int>(sl - h->slots.data());
    const uint32_t nb = std::min<uint32_t>(w.nblocks, static_cast<uint32_t>(h->tab_stride));
    it.blk_off = slot * h->tab_stride;
    it.nblk = static_cast<int>(nb);
    for (uint32_t b = 0; b < nb; b++)
      if (b >= sl->blocks.size() || sl->blocks[b] != w.blocks[b])
        pl.patches.push_back(make_uint2(static_cast<unsigned>(it.blk_off) + b, w.blocks[b]));
    sl->blocks.assign(w.blocks, w.blocks + w.nblocks);
    it.tree = w.parents != nullptr;
    it.path_off = static_cast<int>(pl.paths.size());
    std::vector<int> depth(w.n), poff(w.n), plen(w.n);
    for (uint32_t j = 0; j < w.n; j++) {
      int par = w.parents ? w.parents[j] : static_cast<int>(j) - 1;
      depth[j] = w.parents ? (par < 0 ? 0 : depth[par] + 1) : static_cast<int>(j);
      if (w.parents) {
        std::vector<int> p;
        for (int a = static_cast<int>(j); a >= 0; a = w.parents[a]) p.push_back(a);
        std::reverse(p.begin(), p.end());
        poff[j] = static_cast<int>(pl.paths.size());
        plen[j] = static_cast<int>(p.size());
        pl.paths.insert(pl.paths.end(), p.begin(), p.end());
      }
      int row = static_cast<int>(w.pos + j);
      pl.tok_id.push_back(w.tokens[j]);
      pl.rope_pos.push_back(static_cast<int>(w.pos) + depth[j]);
      pl.kv_row.push_back(static_cast<int>(w.blocks[row / kBlock]) * kBlock + row % kBlock);
      int p0 = row - row % kBlock;
      pl.first_tok.push_back(p0 >= static_cast<int>(w.pos) ? T + (p0 - static_cast<int>(w.pos)) : -1);
      if (j + w.want >= w.n) pl.want_tok.push_back(T + static_cast<int>(j));
    }
    int item = static_cast<int>(pl.items.size());
    pl.items.push_back(it);
    // query groups, then the attention work over kv heads and splits
    int qfirst = static_cast<int>(pl.qgroups.size());
    if (w.parents) {
      // f16 KV: two tree tokens per query group (their 2G rows fill the MMA's 8-row tile; each token's tail is walked
      // with the other's rows left out, so a token's arithmetic is unchanged); fp8 KV keeps one (the exponent frame is
      // per warp)
      const int per = !h->kv_fp8 && 2 * G <= 8 ? 2 : 1;
      for (uint32_t j = 0; j < w.n; j += per) {
        QGroup q{};
        q.item = item; q.j0 = static_cast<int>(j); q.ntok = std::min<int>(per, static_cast<int>(w.n - j));
        q.path_off = poff[j]; q.path_len = plen[j];
        q.nvis = static_cast<int>(w.pos) + plen[j];
        if (q.ntok == 2) {
          q.path_off1 = poff[j + 1];
          q.path_len1 = plen[j + 1];
          q.nvis = std::max(q.nvis, static_cast<int>(w.pos) + plen[j + 1]);
        }
        pl.qgroups.push_back(q);
      }
      if (w.n > 1) multi = true;
    } else {
      for (uint32_t j = 0; j < w.n; j += QG) {
        QGroup q{};
        q.item = item; q.j0 = static_cast<int>(j); q.ntok = static_cast<int>(std::min<uint32_t>(QG, w.n - j));
        q.nvis = static_cast<int>(w.pos + j) + q.ntok;
        pl.qgroups.push_back(q);
      }
      if (pl.qgroups.size() - qfirst > 1) multi = true;
    }
    T += static_cast<int>(w.n);
  }
  // splits: kSplit entries; a tolerance bucket's step with little attention work (fewer than two single-warp CTAs per
  // SM) takes shorter splits, down to 64 entries, so that one sequence still spreads over the SMs
  pl.split = kSplit;
  if (h->gemv_max_t > 0) {
    auto ctas = [&](int sp) {
      long n = 0;
      for (const QGroup &q : pl.qgroups) n += (q.nvis + sp - 1) / sp;
      return n * h->KVH;
    };
    while (pl.split > 64 && ctas(pl.split) < 2L * h->sms) pl.split /= 2;
  }
  for (QGroup &q : pl.qgroups) {
    q.nsplit = (q.nvis + pl.split - 1) / pl.split;
    q.part_base = pl.n_parts;
    pl.n_parts += h->KVH * q.nsplit;
  }
  pl.nw = multi ? 8 : 1;
  // work: per item, kv head, split: the item's query groups (chain token groups or tree nodes) packed nw to a CTA, from
  // the first that reaches the split (a tree node that does not idles in its CTA)
  for (size_t i = 0; i < pl.items.size(); i++) {
    int q0 = -1, q1 = -1;
    for (size_t k = 0; k < pl.qgroups.size(); k++)
      if (pl.qgroups[k].item == static_cast<int>(i)) {
        if (q0 < 0) q0 = static_cast<int>(k);
        q1 = static_cast<int>(k) + 1;
      }
    int maxs = 0;
    for (int k = q0; k < q1; k++) maxs = std::max(maxs, pl.qgroups[k].nsplit);
    for (int head = 0; head < h->KVH; head++)
      for (int s = 0; s < maxs; s++) {
        int k = q0;
        while (k < q1) {
          while (k < q1 && pl.qgroups[k].nsplit <= s) k++;
          if (k == q1) break;
          int n = std::min(pl.nw, q1 - k);
          pl.work.push_back(AttnWork{k, n, head, s});
          if (pl.items[i].tree && pl.nw > 1) pl.tree_cta = 1;   // the kernel's tree warps use private tail buffers
          k += n;
        }
      }
  }
}

// A plan's parts in a buffer, each 256-byte aligned: their offsets, and the total bytes.
size_t plan_layout(const HostPlan &pl, std::vector<size_t> &off) {
  // the table patches last: every part a kernel argument points to has an offset fixed by the step's shape alone
  const size_t sizes[10] = {vbytes(pl.tok_id), vbytes(pl.rope_pos), vbytes(pl.kv_row), vbytes(pl.first_tok),
                            vbytes(pl.items), vbytes(pl.qgroups), vbytes(pl.work), vbytes(pl.paths),
                            vbytes(pl.want_tok), vbytes(pl.patches)};
  size_t total = 0;
  off.clear();
  for (size_t n : sizes) {
    off.push_back(total);
    total += (n + 255) / 256 * 256;
  }
  return total;
}

// the plan's parts copied to host memory at `host` (its layout `off`)
void plan_copy(const HostPlan &pl, uint8_t *host, const std::vector<size_t> &off) {
  const std::pair<const void *, size_t> parts[10] = {
      {pl.tok_id.data(), vbytes(pl.tok_id)},   {pl.rope_pos.data(), vbytes(pl.rope_pos)},
      {pl.kv_row.data(), vbytes(pl.kv_row)},   {pl.first_tok.data(), vbytes(pl.first_tok)},
      {pl.items.data(), vbytes(pl.items)},     {pl.qgroups.data(), vbytes(pl.qgroups)},
      {pl.work.data(), vbytes(pl.work)},       {pl.paths.data(), vbytes(pl.paths)},
      {pl.want_tok.data(), vbytes(pl.want_tok)}, {pl.patches.data(), vbytes(pl.patches)}};
  for (int i = 0; i < 10; i++)
    if (parts[i].second) std::memcpy(host + off[i], parts[i].first, parts[i].second);
}

// the device view of a plan uploaded at `dev` (its layout `off`)
PlanView plan_view(gc_handle *h, const HostPlan &pl, uint8_t *b, const std::vector<size_t> &off) {
  PlanView pv;
  pv.tok_id = reinterpret_cast<const int *>(b + off[0]);
  pv.rope_pos = reinterpret_cast<const int *>(b + off[1]);
  pv.kv_row = reinterpret_cast<const int *>(b + off[2]);
  pv.first_tok = reinterpret_cast<const int *>(b + off[3]);
  pv.items = reinterpret_cast<const Item *>(b + off[4]);
  pv.qgroups = reinterpret_cast<const QGroup *>(b + off[5]);
  pv.work = reinterpret_cast<const AttnWork *>(b + off[6]);
  pv.blocks = h->tables;
  pv.paths = reinterpret_cast<const int *>(b + off[7]);
  pv.want_tok = reinterpret_cast<const int *>(b + off[8]);
  pv.T = static_cast<int>(pl.tok_id.size());
  pv.n_items = static_cast<int>(pl.items.size());
  pv.n_qg = static_cast<int>(pl.qgroups.size());
  pv.n_work = static_cast<int>(pl.work.size());
  pv.R = static_cast<int>(pl.want_tok.size());
  pv.n_parts = pl.n_parts;
  pv.tree_cta = pl.tree_cta;
  pv.split = pl.split;
  pv.max_rows = 0;
  for (const QGroup &q : pl.qgroups) pv.max_rows = std::max(pv.max_rows, q.ntok * (h->H / h->KVH));
  return pv;
}

// Several plans packed one after another into the handle's pinned buffer and uploaded with one copy on its stream;
// returns their device views. The previous step's upload has finished: every step ends with a stream synchronize.
std::vector<PlanView> upload_plans(gc_handle *h, const std::vector<const HostPlan *> &pls) {
  std::vector<std::vector<size_t>> offs(pls.size());
  std::vector<size_t> base(pls.size());
  size_t total = 0;
  for (size_t i = 0; i < pls.size(); i++) {
    base[i] = total;
    total += plan_layout(*pls[i], offs[i]);
  }
  if (total > h->plan_cap) {
    cudaStreamSynchronize(h->st);
    if (h->plan_host) cudaFreeHost(h->plan_host);
    h->plan_host = nullptr;
    size_t cap = std::max<size_t>(total * 2, 1 << 20);
    if (h->plan_dev) h->dfree(h->plan_dev, h->plan_cap);
    h->plan_dev = static_cast<uint8_t *>(h->dalloc(cap, "plan"));
    h->scratch_gen++;
    ck(cudaMallocHost(&h->plan_host, cap), "pinned plan");
    h->plan_cap = cap;
  }
  for (size_t i = 0; i < pls.size(); i++) plan_copy(*pls[i], h->plan_host + base[i], offs[i]);
  ck(cudaMemcpyAsync(h->plan_dev, h->plan_host, total, cudaMemcpyHostToDevice, h->st), "plan upload");
  if (h->stats_on) h->stats.h2d_bytes += total;
  for (size_t i = 0; i < pls.size(); i++)
    if (!pls[i]->patches.empty())
      launch_table_patch(reinterpret_cast<const uint2 *>(h->plan_dev + base[i] + offs[i][9]),
                         static_cast<int>(pls[i]->patches.size()), h->tables, h->st);
  std::vector<PlanView> out;
  for (size_t i = 0; i < pls.size(); i++) out.push_back(plan_view(h, *pls[i], h->plan_dev + base[i], offs[i]));
  return out;
}

PlanView upload_plan(gc_handle *h, HostPlan &pl) { return upload_plans(h, {&pl})[0]; }

// a GEMM of `rows` token rows: the GEMV (tolerance buckets, a few rows, quantized weights) or the tensor-core GEMM;
// its split-K slices (partials for the next kernel) either way
bool gemv_rows(const gc_handle *h, const QWeight &w, int rows) {
  return rows > 0 && rows <= h->gemv_max_t && w.type != kF16;
}

// Split-K and attention scratch for a step's sizes (grown, never shrunk): before the step's launches, and outside any
// stream capture. Bumps scratch_gen when a buffer moves.
void forward_scratch(gc_handle *h, const PlanView &pv) {
  const int T = pv.T;
  cudaStream_t s = h->st;
  float *part0 = h->part;
  auto use_gemv = [&](const QWeight &w, int rows) { return gemv_rows(h, w, rows); };
  auto slices = [&](const QWeight &w, int rows) { return use_gemv(w, rows) ? w.gslices : w.splits; };
  size_t need = 0;
  for (auto &ly : h->layers)
    for (const QWeight *w : {&ly.qkv, &ly.o, &ly.gu, &ly.dn})
      if (slices(*w, T) > 1) need = std::max(need, static_cast<size_t>(slices(*w, T)) * T * w->NT * kBM * 4);
  if (slices(h->head, pv.R) > 1)
    need = std::max(need, static_cast<size_t>(slices(h->head, pv.R)) * pv.R * h->head.NT * kBM * 4);
  h->part = grow(h, h->part, h->part_cap, need, "split-K scratch");
  if (static_cast<size_t>(pv.n_parts) > h->attn_parts_cap) {
    cudaStreamSynchronize(s);
    if (h->attn_o) h->dfree(h->attn_o, h->attn_parts_cap * 16 * h->dh * 4);
    if (h->attn_ml) h->dfree(h->attn_ml, h->attn_parts_cap * 16 * 8);
    size_t cap = std::max<size_t>(pv.n_parts, h->attn_parts_cap * 3 / 2);
    h->attn_o = static_cast<float *>(h->dalloc(cap * 16 * h->dh * 4, "attention partials"));
    h->attn_ml = static_cast<float2 *>(h->dalloc(cap * 16 * 8, "attention partials"));
    h->attn_parts_cap = cap;
    h->scratch_gen++;
  }
  // per (query group, kv head): splits finished so far; zero between launches (the merging split resets it)
  const size_t nsem = static_cast<size_t>(pv.n_qg) * h->KVH;
  if (nsem > h->attn_sem_cap) {
    cudaStreamSynchronize(s);
    if (h->attn_sem) h->dfree(h->attn_sem, h->attn_sem_cap * 4);
    size_t cap = std::max<size_t>(nsem, h->attn_sem_cap * 3 / 2);
    h->attn_sem = static_cast<int *>(h->dalloc(cap * 4, "attention split counters"));
    ck(cudaMemsetAsync(h->attn_sem, 0, cap * 4, s), "attention split counters");
    h->attn_sem_cap = cap;
    h->scratch_gen++;
  }
  if (h->part != part0) h->scratch_gen++;
}

// A step's launches on the handle's stream (no allocation, no synchronization: a stream capture may record them)
void forward_launch(gc_handle *h, const PlanView &pv, int nw) {
  const int T = pv.T;
  cudaStream_t s = h->st;
  auto use_gemv = [&](const QWeight &w, int rows) { return gemv_rows(h, w, rows); };
  auto slices = [&](const QWeight &w, int rows) { return use_gemv(w, rows) ? w.gslices : w.splits; };
  h->step_launches = 0;
  // run(cls, kernels, fn): launch fn on the stream, bracketed by events when the class is being timed
  auto run = [&](int cls, int nk, auto fn) {
    bool rec = h->stats_on && ((h->stats_mask >> cls) & 1u);
    cudaEvent_t a = nullptr, b = nullptr;
    if (rec) {
      a = h->event();
      b = h->event();
      cudaEventRecord(a, s);
    }
    fn();
    if (rec) {
      cudaEventRecord(b, s);
      h->marks.push_back({cls, a, b});
    }
    h->step_launches += nk;
  };
  // A GEMM under class cls. With split-K it writes partials; their reader sums them in split order: the RMSNorm after
  // a residual-add projection (o_proj, down_proj), the RoPE kernel after q/k/v, else a reduce launch (GCK_K_REDUCE).
  auto gemm = [&](int cls, const QWeight &w, const TmaSet &ts, const __half *act, int ldx, int rows, const Epi &e,
                  bool reader_reduces) {
    run(cls, 1, [&] {
      if (use_gemv(w, rows)) launch_gemv(w, w.gslices, act, ldx, rows, e, h->part, h->kerr, s);
      else if (w.type == kF16) launch_gemm(w, act, rows, e, h->part, s);
      else launch_gemm_tc(w, ts, rows, e, h->part, h->kerr, h->sms, h->tc_pairs, s);
    });
    const int sl = slices(w, rows);
    if (sl > 1 && rows > 0 && !reader_reduces)
      run(GCK_K_REDUCE, 1, [&] { launch_splitk_reduce(h->part, sl, rows, w.NT * kBM, e, s); });
  };
  // residual contributions waiting for the next RMSNorm: the split-K partials of the last o_proj / down_proj, or (tensor
  // parallelism) its all-reduced output
  const float *pend = nullptr;
  int pend_s = 0, pend_ld = 0;
  bool pend_tp = false;              // the peer-memory reduction of buffer pend_b, epoch pend_ep
  int pend_b = 0;
  unsigned long long pend_ep = 0;
  auto norm = [&](const int *rows, int n, const float *gain) {
    const float *pp = pend;
    const int ps = pend_s, pl = pend_ld;
    const TpPeers *tp = pend_tp ? &h->peers : nullptr;
    run(GCK_K_NORM, 1, [&] {
      launch_rmsnorm(h->x, rows, n, gain, h->eps, h->d, h->d, h->h, pp, ps, pl, T, tp, pend_b, pend_ep, h->h_scale, s);
    });
    pend = nullptr;
    pend_s = 0;
    pend_tp = false;
  };
  // a8: the input rows of the next GEMM quantized in place (attention output, SwiGLU output); a16: nothing
  auto quant = [&](__half *buf, int n, int ld, float *scale) {
    if (h->a8) run(GCK_K_QUANT, 1, [&] { launch_act_quant(buf, T, n, ld, scale, s); });
  };
  auto residual = [&](int cls, const QWeight &w, const TmaSet &ts, const __half *act, int ldx, const float *scale) {
    if (h->tp > 1 && h->tp_p2p) {
      // this rank's share of the projection into buffer b; then the ranks' deterministic sum over peer memory: flag,
      // reduce-scatter of the rows this rank owns, flag; the next RMSNorm gathers each row's sum from its owner
      const unsigned long long ep = ++h->tp_epoch;
      const int b = static_cast<int>(ep & 1);
      const Epi e{kEpiStore, h->d, h->d, h->tp_bufs[b], nullptr, scale};
      Signal s1{h->tp_flags + b, ep * 4 + 1, h->sig_counter}, s2{h->tp_flags + b, ep * 4 + 2, h->sig_counter};
      if (w.type != kF16) {
        // the rank's split-K partials [splits][T][d] (or its output) straight into buffer b; publishes phase 1
        run(cls, 1, [&] { launch_gemm_tc(w, ts, T, e, h->tp_bufs[b], h->kerr, h->sms, h->tc_pairs, s, s1); });
      } else {
        gemm(cls, w, ts, act, ldx, T, e, false);
        run(GCK_K_ALLREDUCE, 1, [&] { launch_tp_signal(s1.flag, s1.value, s); });
      }
      const int sp = w.type != kF16 ? w.splits : 1;
      run(GCK_K_ALLREDUCE, 1, [&] { launch_tp_reduce_scatter(h->peers, b, ep, T, h->d, sp, s2, s); });   // phase 2
      pend_tp = true;
      pend_b = b;
      pend_ep = ep;
      return;
    }
    if (h->tp > 1) {
      // this rank's share of the projection (its input columns), summed over the ranks in place
      gemm(cls, w, ts, act, ldx, T, Epi{kEpiStore, h->d, h->d, h->tp_y, nullptr, scale}, false);
      run(GCK_K_ALLREDUCE, 1, [&] {
        nck(nccl().all_reduce(h->tp_y, h->tp_y, static_cast<size_t>(T) * h->d, ncclFloat, ncclSum,
                              static_cast<ncclComm_t>(h->comm), s), "all-reduce");
      });
      pend = h->tp_y;
      pend_s = 1;
      pend_ld = h->d;
      return;
    }
    gemm(cls, w, ts, act, ldx, T, Epi{kEpiAdd, h->d, h->d, h->x, nullptr, scale}, true);
    if (slices(w, T) > 1) {
      pend = h->part;
      pend_s = slices(w, T);
      pend_ld = w.NT * kBM;
    }
  };

  run(GCK_K_EMBED, 1, [&] { launch_embed(pv, h->emb, h->emb_type, h->emb_row_bytes, h->d, h->x, s); });
  const int wq = (h->H + 2 * h->KVH) * h->dh;
  AttnArgs aa{};
  aa.q = h->q;
  aa.out = h->att;
  aa.part_o = h->attn_o;
  aa.part_ml = h->attn_ml;
  aa.sem = h->attn_sem;
  aa.H = h->H;
  aa.KVH = h->KVH;
  aa.dh = h->dh;
  aa.kv_fp8 = h->kv_fp8;
  aa.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(h->dh)));
  // one token tile on the tcgen05 GEMM (not the GEMV of tolerance buckets): gate/up and down_proj chained
  const bool chain = h->chain_ok && h->chain_on && T > 0 && T <= 64 && !h->layers.empty() &&
                     !use_gemv(h->layers[0].gu, T) && !use_gemv(h->layers[0].dn, T);
  for (int l = 0; l < h->L; l++) {
    const Layer &ly = h->layers[l];
    norm(nullptr, T, ly.attn_norm);
    gemm(GCK_K_QKV, ly.qkv, h->tma_h, h->h, h->d, T, Epi{kEpiStore, wq, wq, h->qkv, nullptr, h->h_scale}, true);
    uint8_t *kc = h->kc + l * h->layer_bytes, *vc = h->vc + l * h->layer_bytes;
    int8_t *ex = h->exps ? h->exps + l * h->exps_layer : nullptr;
    const int qs = slices(ly.qkv, T);
    const bool qsplit = qs > 1;
    run(GCK_K_ROPE, 1, [&] {
      launch_rope_kv(pv, qsplit ? h->part : h->qkv, qs, qsplit ? ly.qkv.NT * kBM : wq, h->H, h->KVH, h->dh,
                     h->rope, h->q, kc, vc, ex, h->kv_fp8, h->page_scale, s);
    });
    aa.kc = kc;
    aa.vc = vc;
    aa.exps = h->page_scale ? ex : nullptr;
    run(GCK_K_ATTN, 1, [&] { launch_attention(pv, aa, nw, s); });
    quant(h->att, h->H * h->dh, h->H * h->dh, h->att_scale);
    residual(GCK_K_O, ly.o, h->tma_att, h->att, h->H * h->dh, h->att_scale);
    norm(nullptr, T, ly.ffn_norm);
    if (chain) {
      // gate/up (SwiGLU) and down_proj (its split-K partials for the next RMSNorm) in one launch
      const Epi e0{kEpiSwiGLU, h->F, ly.dn.KT * kBK, nullptr, h->act, h->h_scale};
      const Epi e1{kEpiAdd, h->d, h->d, h->x, nullptr, h->act_scale};
      run(GCK_K_GATEUP, 1, [&] {
        launch_gemm_tc_chain(ly.gu, h->tma_h, e0, ly.dn, h->tma_act, e1, h->part, h->chain, T, h->kerr, s);
      });
      if (ly.dn.splits > 1) {
        pend = h->part;
        pend_s = ly.dn.splits;
        pend_ld = ly.dn.NT * kBM;
      }
      continue;
    }
    gemm(GCK_K_GATEUP, ly.gu, h->tma_h, h->h, h->d, T,
         Epi{kEpiSwiGLU, h->F, ly.dn.KT * kBK, nullptr, h->act, h->h_scale}, false);
    quant(h->act, h->F, ly.dn.KT * kBK, h->act_scale);
    residual(GCK_K_DOWN, ly.dn, h->tma_act, h->act, ly.dn.KT * kBK, h->act_scale);
  }
  if (pv.R > 0) {
    norm(pv.want_tok, pv.R, h->out_norm);
    gemm(GCK_K_HEAD, h->head, h->tma_h, h->h, h->d, pv.R,
         Epi{kEpiStore, h->vocab_rows, h->vocab_rows, h->logits, nullptr, h->h_scale}, false);
  }
}

void forward(gc_handle *h, const PlanView &pv, int nw) {
  forward_scratch(h, pv);
  forward_launch(h, pv, nw);
}

// after the step's synchronize: fold the recorded events into the statistics
void collect_stats(gc_handle *h, cudaEvent_t f0, cudaEvent_t f1) {
  if (!h->stats_on) return;
  float ms = 0.f;
  if (f0 && cudaEventElapsedTime(&ms, f0, f1) == cudaSuccess) h->stats.forward_ms += ms;
  for (auto &m : h->marks)
    if (cudaEventElapsedTime(&ms, m.a, m.b) == cudaSuccess) {
      h->stats.class_ms[m.cls] += ms;
      h->stats.class_launches[m.cls] += 1;
    }
  h->marks.clear();
  h->ev_used = 0;
  h->stats.steps += 1;
  h->stats.launches += h->step_launches;
}


// The device part of a step on one handle (or one tensor-parallel rank): slots, plan, forward, argmax, outputs. o (may be
// null for ranks other than 0) receives logits_dev; O holds the caller's host buffers.
// A step's launches (and its device argmax over R rows, R > 0) from a captured graph: replayed when the step's shape has
// a graph, captured when the shape is seen the second time, else left to the caller (false). Every kernel argument of
// a step is a function of the key: plan sizes (the plan's part offsets and the launches' grids), the plan buffer and
// the scratch generation (the buffers the arguments point to).
bool run_graph(gc_handle *h, const PlanView &pv, int nw, int R) {
  const std::vector<int64_t> key = {pv.T, pv.n_items, pv.n_qg, pv.n_work, pv.R, pv.split, pv.max_rows, pv.tree_cta, nw,
                                    R, static_cast<int64_t>(reinterpret_cast<uintptr_t>(h->plan_dev)),
                                    static_cast<int64_t>(h->scratch_gen)};
  for (size_t i = 0; i < h->graphs.size(); i++)
    if (h->graphs[i].key == key) {
      ck(cudaGraphLaunch(h->graphs[i].exec, h->st), "graph launch");
      h->step_launches = h->graphs[i].launches;
      if (h->stats_on) h->stats.graph_steps++;
      std::rotate(h->graphs.begin() + i, h->graphs.begin() + i + 1, h->graphs.end());
      return true;
    }
  if (std::find(h->seen.begin(), h->seen.end(), key) == h->seen.end()) {
    h->seen.push_back(key);
    if (h->seen.size() > 32) h->seen.erase(h->seen.begin());
    return false;
  }
  cudaGraph_t g = nullptr;
  uint64_t launches = 0;
  ck(cudaStreamBeginCapture(h->st, cudaStreamCaptureModeRelaxed), "graph capture");
  try {
    forward_launch(h, pv, nw);
    launches = h->step_launches;
    if (R) {
      launch_argmax(h->logits, R, h->vocab_rows, h->argmax, h->arg_scratch, h->st);
      launches += 2;
    }
  } catch (...) {
    cudaStreamEndCapture(h->st, &g);
    if (g) cudaGraphDestroy(g);
    cudaGetLastError();
    throw;
  }
  cudaError_t e = cudaStreamEndCapture(h->st, &g);
  cudaGraphExec_t ex = nullptr;
  if (e == cudaSuccess) e = cudaGraphInstantiate(&ex, g, 0);
  if (g) cudaGraphDestroy(g);
  if (e != cudaSuccess) fail(GC_E_DEVICE, "step capture: %s", cudaGetErrorString(e));
  if (h->graphs.size() >= 8) {
    cudaGraphExecDestroy(h->graphs.front().exec);
    h->graphs.erase(h->graphs.begin());
  }
  h->graphs.push_back({key, ex, launches});
  ck(cudaGraphLaunch(ex, h->st), "graph launch");
  h->step_launches = launches;
  if (h->stats_on) h->stats.graph_captures++;
  return true;
}

void step_device(gc_handle *h, const std::vector<WorkIn> &ws, bool greedy, uint64_t R, uint32_t flags,
                 const gc_step_out &O, gc_step_out *o) {
  for (auto &w : ws) {
    Slot *sl = find_slot(h, w.sid, true);
    if (!sl) fail(GC_E_STATE, "no free sequence slot (%d in use)", h->max_seqs);
    sl->last_pos = w.pos;
    sl->last_n = w.n;
  }
  ck(cudaSetDevice(h->dev), "cudaSetDevice");
  HostPlan pl;
  build_plan(h, ws, pl);
  // a step that may run as a graph (not under per-class statistics, whose events bracket single launches): its
  // attention work list padded (with empty entries) to a multiple of 512, so that the attention grid, part of the
  // step's shape, changes only every few hundred splits
  const bool graphable = h->graphs_on && h->tp == 1 && !(h->stats_on && h->stats_mask) && pl.paths.empty() &&
                         !pl.work.empty();
  if (graphable) pl.work.resize((pl.work.size() + 511) / 512 * 512, AttnWork{0, 0, 0, 0});
  PlanView pv = upload_plan(h, pl);
  cudaEvent_t f0 = nullptr, f1 = nullptr;
  if (h->stats_on) {
    f0 = h->event();
    f1 = h->event();
    cudaEventRecord(f0, h->st);
  }
  forward_scratch(h, pv);
  if (graphable && run_graph(h, pv, pl.nw, greedy ? static_cast<int>(R) : 0)) {
    // launched
  } else {
    forward_launch(h, pv, pl.nw);
    if (greedy && R) {
    bool rec = h->stats_on && ((h->stats_mask >> GCK_K_ARGMAX) & 1u);
    cudaEvent_t a = rec ? h->event() : nullptr, b = rec ? h->event() : nullptr;
    if (rec) cudaEventRecord(a, h->st);
    if (h->tp > 1) {
      // each rank's best of its vocabulary slice, gathered, then the first maximum overall
      int *mine = h->tp_pick + static_cast<size_t>(h->tp) * h->max_cols * 2;
      launch_argmax_pick(h->logits, static_cast<int>(R), h->vocab_rows, h->vocab0, mine, h->st);
      nck(nccl().all_gather(mine, h->tp_pick, R * 2, ncclInt32, static_cast<ncclComm_t>(h->comm), h->st), "argmax gather");
      launch_argmax_merge(h->tp_pick, h->tp, static_cast<int>(R), h->argmax, h->st);
      h->step_launches += 2;
    } else {
      launch_argmax(h->logits, static_cast<int>(R), h->vocab_rows, h->argmax, h->arg_scratch, h->st);
      h->step_launches += 1;
    }
    if (rec) {
      cudaEventRecord(b, h->st);
      h->marks.push_back({GCK_K_ARGMAX, a, b});
    }
    h->step_launches += 1;
    }
  }
  if (f1) cudaEventRecord(f1, h->st);
  ck(cudaMemcpyAsync(h->kerr_host, h->kerr, 4, cudaMemcpyDeviceToHost, h->st), "error word");
  if (greedy) {
    if (R && h->rank == 0) ck(cudaMemcpyAsync(h->tok_host, h->argmax, R * 4, cudaMemcpyDeviceToHost, h->st), "tokens");
    ck(cudaStreamSynchronize(h->st), "step");
    if (h->rank == 0) std::memcpy(O.tokens, h->tok_host, R * 4);
  } else if (flags & GC_S_HOST_LOGITS) {
    // this handle's vocabulary rows [vocab0, vocab0 + vocab_rows) of every wanted row
    if (R)
      ck(cudaMemcpy2DAsync(O.logits + h->vocab0, static_cast<size_t>(h->vocab) * 4, h->logits,
                           static_cast<size_t>(h->vocab_rows) * 4, static_cast<size_t>(h->vocab_rows) * 4, R,
                           cudaMemcpyDeviceToHost, h->st), "logits");
    ck(cudaStreamSynchronize(h->st), "step");
  } else {
    ck(cudaStreamSynchronize(h->st), "step");
    if (o && o->size >= offsetof(gc_step_out, logits_dev) + 8) o->logits_dev = reinterpret_cast<uint64_t>(h->logits);
  }
  ck(cudaGetLastError(), "step");
  if (*h->kerr_host) {
    int code = *h->kerr_host;
    *h->kerr_host = 0;
    ck(cudaMemset(h->kerr, 0, 16), "error word");
    h->marks.clear();
    h->ev_used = 0;
    fail(GC_E_DEVICE, "a kernel's wait ran out of time (code %d); the step's results are invalid", code);
  }
  collect_stats(h, f0, f1);
}

// A speculative pair's step (GC_L_SPEC: one linear stream, gc.h:57,93,117,136,174-190). A prefill chunk or a plain
// decode runs the target only; the drafter catches up at the next round. A decode with GC_W_SPEC runs a round: the
// drafter drafts spec_k tokens greedily after the anchor (its first pass also takes the stream's tokens it has not
// seen), the target verifies anchor and drafts as one chain, and the longest prefix of drafts equal to the target's
// argmax is accepted and returned with the target's own next token (1 .. spec_k + 1 tokens). The drafts never leave
// the device: each draft pass's argmax writes its token where the next pass and the verify read it, and one copy
// brings the round back. In batch-invariant numerics a verify row equals a plain decode of the same token (chunk
// invariance), so a round returns exactly the tokens the target alone would decode greedily.
int spec_step(gc_handle *h, const gc_step_in *in, gc_step_out *o) {
  if (in->n_work != 1) fail(GC_E_UNSUPPORTED, "a speculative pair runs one sequence a step (%u items)", in->n_work);
  const gc_work *wp = in->work[0];
  if (!wp) fail(GC_E_ARG, "work item 0 is null");
  if (wp->size < offsetof(gc_work, want) + 4) fail(GC_E_ARG, "work item 0: struct size %u", wp->size);
  gc_work W{};
  std::memcpy(&W, wp, std::min<size_t>(wp->size, sizeof W));
  if (!(W.flags & GC_W_GREEDY)) fail(GC_E_UNSUPPORTED, "a speculative pair runs greedy sequences (device argmax)");
  if (W.parents) fail(GC_E_UNSUPPORTED, "a speculative pair verifies its own drafts: no tree items");
  if (W.flags & GC_W_FEATS) fail(GC_E_UNSUPPORTED, "this pack has no tap features");
  if (!W.n_tokens || !W.tokens || W.want > W.n_tokens) fail(GC_E_ARG, "work item 0: bad token count or want");
  if (!W.blocks || W.n_blocks != 1 || W.blocks[0] != 0)
    fail(GC_E_ARG, "work item 0: a speculative pair's sequence has the one page 0");
  for (uint32_t j = 0; j < W.n_tokens; j++)
    if (W.tokens[j] < 0 || W.tokens[j] >= h->vocab) fail(GC_E_ARG, "work item 0: token %d outside the vocabulary", W.tokens[j]);
  const bool round = (W.flags & GC_W_SPEC) && W.want > 0;
  if (round && W.n_tokens != 1) fail(GC_E_ARG, "a speculative round starts from one anchor token (%u given)", W.n_tokens);
  const int K = h->spec_k;
  const uint64_t end = static_cast<uint64_t>(W.pos) + W.n_tokens + (round ? K : 0);
  if (end > static_cast<uint64_t>(h->max_ctx))
    fail(GC_E_ARG, "work item 0: position %llu past the context %d", static_cast<unsigned long long>(end), h->max_ctx);
  gc_step_out O{};
  std::memcpy(&O, o, std::min<size_t>(o->size, sizeof O));
  const uint32_t rows = round ? static_cast<uint32_t>(K + 1) : W.want;
  o->n_rows = rows;
  if (O.tokens_cap < rows || (rows && !O.tokens) || !O.counts) fail(GC_E_CAPACITY, "tokens buffer too small (%u rows)", rows);
  const bool fresh = find_slot(h, W.sid, false) == nullptr;
  if (!find_slot(h, W.sid, true)) fail(GC_E_STATE, "no free sequence slot (a speculative pair runs one)");
  if (fresh) {
    h->hist.clear();
    h->draft_rows = 0;
    // a pair runs one stream: a drafter slot an earlier sequence still holds (not released) is the new stream's
    for (Slot &s : h->drafter->slots)
      if (s.used && s.sid != W.sid) s = Slot{};
  }
  if (W.pos > h->hist.size())
    fail(GC_E_STATE, "position %u not contiguous: the stream holds %zu tokens", W.pos, h->hist.size());
  h->hist.resize(W.pos);                                  // a rewind drops the rows past pos
  h->draft_rows = std::min(h->draft_rows, static_cast<int>(W.pos));
  h->hist.insert(h->hist.end(), W.tokens, W.tokens + W.n_tokens);
  const uint32_t *table = h->spec_table.data();
  const uint32_t ntab = static_cast<uint32_t>(h->spec_table.size());
  if (!round) {
    const WorkIn wi{W.flags, W.sid, W.pos, W.n_tokens, W.tokens, nullptr, table, ntab, W.want};
    step_device(h, {wi}, true, W.want, in->flags, O, o);
    O.counts[0] = W.want;
    return GC_OK;
  }
  gc_handle *d = h->drafter;
  const int pos = static_cast<int>(W.pos);
  // the drafter's backlog beyond what one pass takes runs as plain prefill chunks first
  while (pos - h->draft_rows + 1 > d->max_cols) {
    const int n = std::min(d->max_cols, pos - h->draft_rows);
    const WorkIn wi{0, W.sid, static_cast<uint32_t>(h->draft_rows), static_cast<uint32_t>(n),
                    h->hist.data() + h->draft_rows, nullptr, table, ntab, 0};
    step_device(d, {wi}, false, 0, 0, O, nullptr);
    h->draft_rows += n;
  }
  // the plans: draft passes 1 .. K (the first over the backlog and the anchor), then the verify of anchor + drafts
  std::vector<HostPlan> dp(K);
  std::vector<int> first(h->hist.begin() + h->draft_rows, h->hist.begin() + pos + 1), zero(1, 0), chain(K + 1, 0);
  build_plan(d, {WorkIn{GC_W_GREEDY, W.sid, static_cast<uint32_t>(h->draft_rows), static_cast<uint32_t>(first.size()),
                        first.data(), nullptr, table, ntab, 1}}, dp[0]);
  for (int k = 1; k < K; k++)
    build_plan(d, {WorkIn{GC_W_GREEDY, W.sid, static_cast<uint32_t>(pos + k), 1, zero.data(), nullptr, table, ntab, 1}},
               dp[k]);
  chain[0] = W.tokens[0];
  HostPlan vp;
  build_plan(h, {WorkIn{GC_W_GREEDY, W.sid, W.pos, static_cast<uint32_t>(K + 1), chain.data(), nullptr, table, ntab,
                        static_cast<uint32_t>(K + 1)}}, vp);
  ck(cudaSetDevice(h->dev), "cudaSetDevice");
  std::vector<const HostPlan *> dptr;
  for (auto &x : dp) dptr.push_back(&x);
  std::vector<PlanView> dv = upload_plans(d, dptr);
  const PlanView vv = upload_plan(h, vp);
  int *chain_dev = const_cast<int *>(vv.tok_id);          // the verify's tokens: the anchor, then each draft as made
  cudaEvent_t f0 = nullptr, f1 = nullptr;
  if (h->stats_on) {
    f0 = h->event();
    f1 = h->event();
    cudaEventRecord(f0, h->st);
  }
  h->step_launches = 0;
  uint64_t launches = 0;
  for (int k = 0; k < K; k++) {
    if (k > 0) dv[k].tok_id = chain_dev + k;                // pass k + 1 embeds draft k
    forward(d, dv[k], dp[k].nw);
    launches += d->step_launches + 1;
    launch_argmax(d->logits, 1, d->vocab_rows, chain_dev + k + 1, d->arg_scratch, h->st);
  }
  forward(h, vv, vp.nw);
  launches += h->step_launches + 2;
  launch_argmax(h->logits, K + 1, h->vocab_rows, h->argmax, h->arg_scratch, h->st);
  launch_spec_accept(chain_dev, h->argmax, K, h->spec_out, h->st);
  h->step_launches = launches;
  if (f1) cudaEventRecord(f1, h->st);
  ck(cudaMemcpyAsync(h->spec_out_host, h->spec_out, static_cast<size_t>(K + 2) * 4, cudaMemcpyDeviceToHost, h->st),
     "round");
  ck(cudaMemcpyAsync(h->kerr_host, h->kerr, 4, cudaMemcpyDeviceToHost, h->st), "error word");
  ck(cudaMemcpyAsync(d->kerr_host, d->kerr, 4, cudaMemcpyDeviceToHost, h->st), "error word");
  ck(cudaStreamSynchronize(h->st), "round");
  ck(cudaGetLastError(), "round");
  for (gc_handle *x : {h, d})
    if (*x->kerr_host) {
      const int code = *x->kerr_host;
      *x->kerr_host = 0;
      ck(cudaMemset(x->kerr, 0, 16), "error word");
      h->marks.clear();
      h->ev_used = 0;
      fail(GC_E_DEVICE, "a kernel's wait ran out of time (code %d); the round's results are invalid", code);
    }
  const int n = h->spec_out_host[K + 1];
  if (n < 1 || n > K + 1) fail(GC_E_DEVICE, "speculative round: %d tokens accepted", n);
  std::memcpy(O.tokens, h->spec_out_host, static_cast<size_t>(n) * 4);
  O.counts[0] = static_cast<uint32_t>(n);
  o->n_rows = static_cast<uint32_t>(n);
  // rows pos + 1 .. pos + n - 1 hold the accepted drafts in both caches (the drafter's only up to pos + K - 1)
  h->hist.insert(h->hist.end(), h->spec_out_host, h->spec_out_host + n - 1);
  h->draft_rows = pos + std::min(n, K);
  collect_stats(h, f0, f1);
  return GC_OK;
}

}  // namespace

extern "C" {

GC_API int gc_step(gc_handle *h, const gc_step_in *in, gc_step_out *o) {
  if (!h) return GC_E_ARG;
  try {
    if (!in || !o || in->size < offsetof(gc_step_in, n_work) + 4 || o->size < offsetof(gc_step_out, counts) + 8)
      fail(GC_E_ARG, "gc_step: null argument or struct size");
    if (h->drafter) {
      if (!in->n_work || !in->work) fail(GC_E_ARG, "gc_step: no work items");
      return spec_step(h, in, o);
    }
    if (!in->n_work || !in->work) fail(GC_E_ARG, "gc_step: no work items");
    if (in->n_work > static_cast<uint32_t>(h->max_seqs))
      fail(GC_E_ARG, "gc_step: %u items, the bucket runs %d sequences", in->n_work, h->max_seqs);
    std::vector<WorkIn> ws;
    bool greedy = true;
    uint64_t T = 0, R = 0;
    for (uint32_t i = 0; i < in->n_work; i++) {
      const gc_work *w = in->work[i];
      if (!w) fail(GC_E_ARG, "work item %u is null", i);
      gc_work W{};
      std::memcpy(&W, w, std::min<size_t>(w->size, sizeof W));
      if (w->size < offsetof(gc_work, want) + 4) fail(GC_E_ARG, "work item %u: struct size %u", i, w->size);
      if (!W.n_tokens || !W.tokens || W.want > W.n_tokens) fail(GC_E_ARG, "work item %u: bad token count or want", i);
      if (W.flags & GC_W_SPEC) fail(GC_E_UNSUPPORTED, "work item %u: speculative rounds need a spec pair", i);
      if (W.flags & GC_W_FEATS) fail(GC_E_UNSUPPORTED, "work item %u: this pack has no tap features", i);
      if (!W.blocks || static_cast<uint64_t>(W.n_blocks) * kBlock < static_cast<uint64_t>(W.pos) + W.n_tokens)
        fail(GC_E_ARG, "work item %u: block table does not cover rows 0 .. %u", i, W.pos + W.n_tokens - 1);
      if (static_cast<uint64_t>(W.pos) + W.n_tokens > static_cast<uint64_t>(h->max_ctx))
        fail(GC_E_ARG, "work item %u: position %u past the context %d", i, W.pos + W.n_tokens, h->max_ctx);
      for (uint32_t b = 0; b < W.n_blocks; b++)
        if (W.blocks[b] >= static_cast<uint32_t>(h->nblk))
          fail(GC_E_ARG, "work item %u: block %u out of pool (%d blocks)", i, W.blocks[b], h->nblk);
      for (uint32_t j = 0; j < W.n_tokens; j++) {
        if (W.tokens[j] < 0 || W.tokens[j] >= h->vocab) fail(GC_E_ARG, "work item %u: token %d outside the vocabulary", i, W.tokens[j]);
        if (W.parents && (W.parents[j] < -1 || W.parents[j] >= static_cast<int32_t>(j)))
          fail(GC_E_ARG, "work item %u: parent of token %u must be -1 or an earlier token", i, j);
      }
      for (auto &p : ws)
        if (p.sid == W.sid) fail(GC_E_ARG, "sequence %llu appears twice in one step", static_cast<unsigned long long>(W.sid));
      greedy = greedy && (W.flags & GC_W_GREEDY);
      T += W.n_tokens;
      R += W.want;
      ws.push_back(WorkIn{W.flags, W.sid, W.pos, W.n_tokens, W.tokens, W.parents, W.blocks, W.n_blocks, W.want});
    }
    if (T > static_cast<uint64_t>(h->max_cols)) fail(GC_E_ARG, "gc_step: %llu tokens, at most %d", static_cast<unsigned long long>(T), h->max_cols);
    gc_step_out O{};
    std::memcpy(&O, o, std::min<size_t>(o->size, sizeof O));
    o->n_rows = static_cast<uint32_t>(R);
    const uint32_t flags = in->flags;
    if (greedy) {
      if (O.tokens_cap < R || (R && !O.tokens) || !O.counts) fail(GC_E_CAPACITY, "tokens buffer too small (%llu rows)", static_cast<unsigned long long>(R));
    } else if (flags & GC_S_HOST_LOGITS) {
      if (O.logits_cap < R * static_cast<uint64_t>(h->vocab) || (R && !O.logits))
        fail(GC_E_CAPACITY, "logits buffer too small (%llu rows of %d)", static_cast<unsigned long long>(R), h->vocab);
    } else if (h->tp > 1) {
      fail(GC_E_UNSUPPORTED, "device logits are not gathered across tensor-parallel ranks: ask for host logits or greedy rows");
    }
    // sequence slots: the handle's table (a group's is kept for the checks, every rank holds the same one)
    for (auto &w : ws)
      if (!find_slot(h, w.sid, true)) fail(GC_E_STATE, "no free sequence slot (%d in use)", h->max_seqs);
    if (h->tp == 1) {
      step_device(h, ws, greedy, R, flags, O, o);
    } else {
      for (auto &w : ws) {
        Slot *sl = find_slot(h, w.sid, false);
        sl->blocks.assign(w.blocks, w.blocks + w.nblocks);
        sl->last_pos = w.pos;
        sl->last_n = w.n;
      }
      std::vector<std::thread> th;
      std::vector<int> codes(h->tp, GC_OK);
      std::vector<std::string> errs(h->tp);
      for (int r = 0; r < h->tp; r++)
        th.emplace_back([&, r] {
          try {
            step_device(h->ranks[r], ws, greedy, R, flags, O, r == 0 ? o : nullptr);
          } catch (const GcError &e) {
            codes[r] = e.code;
            errs[r] = e.msg;
          }
        });
      for (auto &t : th) t.join();
      for (int r = 0; r < h->tp; r++)
        if (codes[r] != GC_OK) fail(codes[r], "rank %d: %s", r, errs[r].c_str());
    }
    for (uint32_t i = 0; greedy && i < in->n_work; i++) O.counts[i] = ws[i].want;
    return GC_OK;
  } catch (const GcError &e) {
    h->err = e.msg;
    return e.code;
  }
}

}  // extern "C"

// a tensor-parallel group applies a KV operation on every rank (each holds its kv heads of the same blocks)
template <typename Fn>
static int on_ranks(gc_handle *h, Fn fn) {
  for (gc_handle *r : h->ranks) {
    int rc = fn(r);
    if (rc != GC_OK) {
      h->err = "rank " + std::to_string(r->rank) + ": " + r->err;
      return rc;
    }
  }
  return GC_OK;
}

extern "C" {

GC_API int gc_commit(gc_handle *h, uint64_t sid, uint32_t base, const uint32_t *path, uint32_t n) {
  if (!h) return GC_E_ARG;
  if (h->drafter) {
    h->err = "gc_commit: a speculative pair keeps its own rounds' rows";
    return GC_E_UNSUPPORTED;
  }
  if (!h->ranks.empty()) return on_ranks(h, [&](gc_handle *r) { return gc_commit(r, sid, base, path, n); });
  try {
    Slot *sl = find_slot(h, sid, false);
    if (!sl) fail(GC_E_STATE, "gc_commit: unknown sequence %llu", static_cast<unsigned long long>(sid));
    if (n && !path) fail(GC_E_ARG, "gc_commit: null path");
    std::vector<int> moves;
    uint64_t rows = static_cast<uint64_t>(sl->blocks.size()) * kBlock;
    for (uint32_t j = 0; j < n; j++) {
      if (path[j] < j || (j && path[j] <= path[j - 1])) fail(GC_E_ARG, "gc_commit: path must increase and path[j] >= j");
      if (static_cast<uint64_t>(base) + path[j] >= rows) fail(GC_E_ARG, "gc_commit: row %u outside the table", base + path[j]);
      if (path[j] == j) continue;
      uint32_t a = base + path[j], b = base + j;
      moves.push_back(static_cast<int>(sl->blocks[a / kBlock] * kBlock + a % kBlock));
      moves.push_back(static_cast<int>(sl->blocks[b / kBlock] * kBlock + b % kBlock));
    }
    if (moves.empty()) return GC_OK;
    ck(cudaSetDevice(h->dev), "cudaSetDevice");
    int nm = static_cast<int>(moves.size() / 2);
    h->pairs = grow(h, h->pairs, h->pairs_cap, vbytes(moves), "commit moves");
    h->commit_tmp = grow(h, h->commit_tmp, h->commit_cap, static_cast<size_t>(nm) * h->L * 2 * h->KVH * h->dh * 4, "commit rows");
    ck(cudaMemcpyAsync(h->pairs, moves.data(), vbytes(moves), cudaMemcpyHostToDevice, h->st), "commit moves");
    launch_commit(h->pairs, nm, h->L, h->KVH, h->dh, h->kc, h->vc, h->page_scale ? h->exps : nullptr, h->kv_fp8,
                  h->layer_bytes, h->exps_layer, h->commit_tmp, h->st);
    ck(cudaStreamSynchronize(h->st), "commit");
    ck(cudaGetLastError(), "commit");
    return GC_OK;
  } catch (const GcError &e) {
    h->err = e.msg;
    return e.code;
  }
}

GC_API int gc_copy_blocks(gc_handle *h, const uint32_t *src, const uint32_t *dst, uint32_t n) {
  if (!h) return GC_E_ARG;
  if (h->drafter) {
    if (!n) return GC_OK;
    h->err = "gc_copy_blocks: a speculative pair's stream has one page";
    return GC_E_UNSUPPORTED;
  }
  if (!h->ranks.empty()) return on_ranks(h, [&](gc_handle *r) { return gc_copy_blocks(r, src, dst, n); });
  try {
    if (n && (!src || !dst)) fail(GC_E_ARG, "gc_copy_blocks: null array");
    std::vector<int> pairs;
    for (uint32_t i = 0; i < n; i++) {
      if (src[i] >= static_cast<uint32_t>(h->nblk) || dst[i] >= static_cast<uint32_t>(h->nblk))
        fail(GC_E_ARG, "gc_copy_blocks: block out of pool (%u -> %u, %d blocks)", src[i], dst[i], h->nblk);
      pairs.push_back(static_cast<int>(src[i]));
      pairs.push_back(static_cast<int>(dst[i]));
    }
    if (!n) return GC_OK;
    ck(cudaSetDevice(h->dev), "cudaSetDevice");
    h->pairs = grow(h, h->pairs, h->pairs_cap, vbytes(pairs), "copy pairs");
    ck(cudaMemcpyAsync(h->pairs, pairs.data(), vbytes(pairs), cudaMemcpyHostToDevice, h->st), "copy pairs");
    // pairs run in order; a batch runs in one launch while no destination is read or written again in it
    size_t i = 0;
    while (i < n) {
      size_t j = i;
      std::vector<uint32_t> touched;
      while (j < n) {
        bool clash = false;
        for (uint32_t x : touched)
          if (x == src[j] || x == dst[j]) clash = true;
        if (clash) break;
        touched.push_back(dst[j]);
        j++;
      }
      launch_copy_blocks(h->pairs + 2 * i, static_cast<int>(j - i), h->L, h->page_bytes, h->layer_bytes, h->kc, h->vc,
                         h->exps, h->exps_layer, h->KVH * 2, h->st);
      i = j;
    }
    ck(cudaStreamSynchronize(h->st), "copy_blocks");
    ck(cudaGetLastError(), "copy_blocks");
    return GC_OK;
  } catch (const GcError &e) {
    h->err = e.msg;
    return e.code;
  }
}

GC_API int gck_commit_static(gc_handle *h, uint64_t sid, uint32_t base, const uint32_t *path, uint32_t n) {
  if (!h) return GC_E_ARG;
  if (h->drafter) {
    h->err = "gck_commit_static: a speculative pair keeps its own rounds' rows";
    return GC_E_UNSUPPORTED;
  }
  if (!h->ranks.empty()) return on_ranks(h, [&](gc_handle *r) { return gck_commit_static(r, sid, base, path, n); });
  try {
    Slot *sl = find_slot(h, sid, false);
    if (!sl) fail(GC_E_STATE, "gck_commit_static: unknown sequence %llu", static_cast<unsigned long long>(sid));
    if (n && !path) fail(GC_E_ARG, "gck_commit_static: null path");
    std::vector<int> moves;
    uint64_t rows = static_cast<uint64_t>(sl->blocks.size()) * kBlock;
    for (uint32_t j = 0; j < n; j++) {
      if (path[j] < j || (j && path[j] <= path[j - 1]))
        fail(GC_E_ARG, "gck_commit_static: path must increase and path[j] >= j");
      if (static_cast<uint64_t>(base) + path[j] >= rows)
        fail(GC_E_ARG, "gck_commit_static: row %u outside the table", base + path[j]);
      if (path[j] == j) continue;
      uint32_t a = base + path[j], b = base + j;
      moves.push_back(static_cast<int>(sl->blocks[a / kBlock] * kBlock + a % kBlock));
      moves.push_back(static_cast<int>(sl->blocks[b / kBlock] * kBlock + b % kBlock));
    }
    if (moves.empty()) return GC_OK;
    const int nm = static_cast<int>(moves.size() / 2);
    // layout in the array: the move list (256-byte aligned), then the staged rows [moves][layers][K, V][KVH * dh] f32
    const size_t list_bytes = (vbytes(moves) + 255) / 256 * 256;
    const size_t row_bytes = static_cast<size_t>(h->L) * 2 * h->KVH * h->dh * 4;
    const size_t need = list_bytes + static_cast<size_t>(nm) * row_bytes;
    if (need > kCommitStaticBytes)
      fail(GC_E_ARG, "gck_commit_static: %d moved rows need %zu bytes of scratch; the static array holds %zu (at most %zu "
           "moved rows for this model)", nm, need, kCommitStaticBytes, (kCommitStaticBytes - 256) / (row_bytes + 8));
    ck(cudaSetDevice(h->dev), "cudaSetDevice");
    // looked up at gc_open (open_device): this returns the cached address and allocates nothing
    uint8_t *base_ptr = static_cast<uint8_t *>(commit_static_address(h->dev));
    int *d_moves = reinterpret_cast<int *>(base_ptr);
    float *d_rows = reinterpret_cast<float *>(base_ptr + list_bytes);
    // nothing in the array has to start at zero: the list is copied whole and every staged row is written before read
    ck(cudaMemcpyAsync(d_moves, moves.data(), vbytes(moves), cudaMemcpyHostToDevice, h->st), "commit moves");
    launch_commit(d_moves, nm, h->L, h->KVH, h->dh, h->kc, h->vc, h->page_scale ? h->exps : nullptr, h->kv_fp8,
                  h->layer_bytes, h->exps_layer, d_rows, h->st);
    ck(cudaStreamSynchronize(h->st), "commit");
    ck(cudaGetLastError(), "commit");
    return GC_OK;
  } catch (const GcError &e) {
    h->err = e.msg;
    return e.code;
  }
}

GC_API int gc_state_save(gc_handle *h, uint64_t, uint32_t) {
  if (h) h->err = "gc_state_save: this pack has no bounded state (GC_L_BOUNDED)";
  return GC_E_ARG;
}

GC_API int gc_state_restore(gc_handle *h, uint32_t, uint64_t) {
  if (h) h->err = "gc_state_restore: this pack has no bounded state (GC_L_BOUNDED)";
  return GC_E_ARG;
}

GC_API int gc_release(gc_handle *h, uint64_t sid) {
  if (!h) return GC_E_ARG;
  Slot *sl = find_slot(h, sid, false);
  if (sl) *sl = Slot{};
  if (h->drafter) {
    gc_release(h->drafter, sid);     // the drafter's slot for the sequence
    if (sl) {                        // the stream's tokens go with its sequence
      h->hist.clear();
      h->draft_rows = 0;
    }
  }
  for (gc_handle *r : h->ranks) gc_release(r, sid);
  return GC_OK;
}

GC_API int gck_stats_enable(gc_handle *h, uint32_t class_mask) {
  if (!h) return GC_E_ARG;
  if (!h->ranks.empty()) return gck_stats_enable(h->ranks[0], class_mask);   // rank 0's device times
  h->stats = gck_stats{};
  h->stats.size = sizeof(gck_stats);
  h->stats_mask = class_mask;
  h->stats_on = true;
  h->marks.clear();
  h->ev_used = 0;
  return GC_OK;
}

GC_API int gck_stats_read(gc_handle *h, gck_stats *out) {
  if (!h || !out || out->size < 8) return GC_E_ARG;
  if (!h->ranks.empty()) return gck_stats_read(h->ranks[0], out);
  h->stats_on = false;
  uint32_t n = std::min<uint32_t>(out->size, sizeof(gck_stats));
  gck_stats st = h->stats;
  st.size = n;
  st.gemm_pairs = static_cast<uint32_t>(h->tc_pairs);
  std::memcpy(out, &st, n);
  return GC_OK;
}

GC_API void gc_close(gc_handle *h) {
  if (!h) return;
  if (!h->ranks.empty()) {
    // communicators are released by every rank at once (as their collectives run), then the ranks' memory
    std::vector<std::thread> th;
    for (gc_handle *r : h->ranks)
      th.emplace_back([r] {
        cudaSetDevice(r->dev);
        if (r->st) cudaStreamSynchronize(r->st);
        if (r->comm) nccl().destroy(static_cast<ncclComm_t>(r->comm));
        r->comm = nullptr;
      });
    for (auto &t : th) t.join();
    for (gc_handle *r : h->ranks) {
      cudaSetDevice(r->dev);
      delete r;
    }
    h->ranks.clear();
    delete h;
    return;
  }
  cudaSetDevice(h->dev);
  delete h;
}

}  // extern "C"

// ============================================================================================== pricing
// gc_probe / gc_price (abi/gc.h:232-237): the constants a device's step time follows (HBM copy bandwidth, per-launch
// latency, SMs, clock), and a roofline prediction from them. The library serves any llama GGUF, and gc_price sees only
// a bucket id, so the price is that of one reference step on the device: a single-sequence decode of the 8B Q4_K shape
// (4.221 GB of weights streamed once at the measured bandwidth, plus the step's kernel launches).
namespace {

struct PriceBlob {
  uint32_t magic = 0x45435250u;   // "PRCE"
  uint32_t version = 1;
  double hbm_gbs = 0;            // device copy bandwidth (read + write bytes / time)
  double launch_us = 0;          // back-to-back empty-kernel launch interval on one stream
  uint32_t sms = 0, clock_mhz = 0;
};

__global__ void probe_copy_kernel(const float4 *a, float4 *b, size_t n) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n; i += static_cast<size_t>(gridDim.x) * blockDim.x)
    b[i] = a[i];
}
__global__ void probe_empty_kernel() {}

constexpr double kRefWeightBytes = 4.221e9;   // 8B shape, Q4_K linear weights and head
constexpr double kRefLaunches = 292;          // kernels of one such decode step
constexpr double kRefStreamEff = 0.85;        // fraction of copy bandwidth a weight-streaming step reaches

}  // namespace

extern "C" {

GC_API int gc_probe(int device, void *constants, uint64_t cap, uint64_t *size) {
  if (!size) return GC_E_ARG;
  *size = sizeof(PriceBlob);
  if (cap < sizeof(PriceBlob) || !constants) return GC_E_CAPACITY;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
    cudaGetLastError();
    return GC_E_DEVICE;
  }
  int prev = 0;
  cudaGetDevice(&prev);
  PriceBlob b;
  int rc = GC_OK;
  float4 *x = nullptr, *y = nullptr;
  cudaStream_t st = nullptr;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  do {
    if (cudaSetDevice(device) != cudaSuccess) { rc = GC_E_DEVICE; break; }
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) { rc = GC_E_DEVICE; break; }
    b.sms = static_cast<uint32_t>(prop.multiProcessorCount);
    int clk = 0;
    cudaDeviceGetAttribute(&clk, cudaDevAttrClockRate, device);
    b.clock_mhz = static_cast<uint32_t>(clk / 1000);
    const size_t bytes = static_cast<size_t>(512) << 20;   // 512 MiB each way: well past L2
    const size_t n = bytes / sizeof(float4);
    if (cudaMalloc(&x, bytes) != cudaSuccess || cudaMalloc(&y, bytes) != cudaSuccess ||
        cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess || cudaEventCreate(&e0) != cudaSuccess ||
        cudaEventCreate(&e1) != cudaSuccess || cudaMemsetAsync(x, 0, bytes, st) != cudaSuccess) {
      rc = GC_E_DEVICE;
      break;
    }
    const int grid = static_cast<int>(b.sms) * 8;
    float best = 1e30f;
    for (int it = 0; it < 5; it++) {
      cudaEventRecord(e0, st);
      probe_copy_kernel<<<grid, 512, 0, st>>>(x, y, n);
      cudaEventRecord(e1, st);
      cudaEventSynchronize(e1);
      float ms = 0;
      cudaEventElapsedTime(&ms, e0, e1);
      if (it > 0) best = std::min(best, ms);
    }
    b.hbm_gbs = 2.0 * bytes / (best * 1e-3) / 1e9;
    const int nl = 200;
    probe_empty_kernel<<<1, 32, 0, st>>>();
    cudaEventRecord(e0, st);
    for (int i = 0; i < nl; i++) probe_empty_kernel<<<1, 32, 0, st>>>();
    cudaEventRecord(e1, st);
    cudaEventSynchronize(e1);
    float ms = 0;
    cudaEventElapsedTime(&ms, e0, e1);
    b.launch_us = ms * 1e3 / nl;
    if (cudaGetLastError() != cudaSuccess) rc = GC_E_DEVICE;
  } while (false);
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  if (st) cudaStreamDestroy(st);
  if (x) cudaFree(x);
  if (y) cudaFree(y);
  cudaSetDevice(prev);
  if (rc != GC_OK) cudaGetLastError();   // a failed probe leaves no pending error for the caller's next CUDA call
  if (rc == GC_OK) std::memcpy(constants, &b, sizeof b);
  return rc;
}

GC_API int gc_price(const void *constants, uint64_t size, const char *bucket_id, double *step_us) {
  if (!constants || !bucket_id || !step_us || size != sizeof(PriceBlob)) return GC_E_ARG;
  PriceBlob b;
  std::memcpy(&b, constants, sizeof b);
  if (b.magic != PriceBlob{}.magic || b.version != 1 || !(b.hbm_gbs > 0)) return GC_E_ARG;
  *step_us = kRefWeightBytes / (b.hbm_gbs * 1e9 * kRefStreamEff) * 1e6 + kRefLaunches * b.launch_us;
  return GC_OK;
}

}  // extern "C"
