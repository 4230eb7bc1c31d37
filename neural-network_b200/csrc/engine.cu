// Host engine and C ABI of the B200 speculative-decoding backend.
//
// One specdec_handle = one device, two decoder models (target, draft), their
// KV caches, the per-request speculative state and the activation buffers,
// all allocated once in specdec_create.  specdec_generate runs the
// reference's TransformerDecoder::generate_speculative
// (src/nn/layer.cpp:1382-1661) for B requests at once:
//
//   prefill target + draft  ->  first token  ->  WHILE(any request active) {
//     draft step 0 (catch-up + last token), draft steps 1..k-1 (+ sample),
//     verify (k+1 rows per request), accept/reject/rollback }
//
// The whole sequence is captured once per (B, S, sampling mode) into a CUDA
// graph whose round loop is a device-driven conditional WHILE node, so one
// generate call is one graph launch with no host round trips.  The same
// kernels can be launched directly (SPECDEC_NO_GRAPH=1), e.g. for per-kernel
// profiling (ncu cannot profile kernel nodes of graphs with conditional nodes).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <dlfcn.h>
#include <nccl.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <tuple>
#include <vector>

#include "../../include/specdec.h"
#include "forward.cuh"
#include "gemm.cuh"
#include "attn_tc.cuh"
#include "sample.cuh"
#include "tree.cuh"
#include "kern_table.cuh"
#include "attn_dec.cuh"
#include "gemm_w8.cuh"
#include "gemm_sk.cuh"

using namespace specdec;

namespace {

thread_local std::string g_create_err;

struct SpecErr {
  int code;
  std::string msg;
};

#define CK(x)                                                                                   \
  do {                                                                                          \
    cudaError_t e_ = (x);                                                                       \
    if (e_ != cudaSuccess)                                                                      \
      throw SpecErr{e_ == cudaErrorMemoryAllocation ? SPECDEC_ERR_OOM : SPECDEC_ERR_CUDA,       \
                    std::string(#x) + ": " + cudaGetErrorString(e_)};                         \
  } while (0)

[[noreturn]] void fail(int code, const std::string &m) { throw SpecErr{code, m}; }

// Model dimensions as this rank holds them: with tensor parallelism H, Hkv
// and F are the rank's share (heads and FFN columns), Hg, Hkvg and Fg the
// model's; dq = H * D is the rank's query width (d without parallelism).
struct Dims {
  int V, d, H, Hkv, D, F, L, max_seq, arch, kvd;
  int dq, Hg, Hkvg, Fg;
};

// A validated token tree: depth, branching, node counts per depth.
struct TreeCfg {
  int depth = 0;
  int branch[kTreeMaxDepth] = {};
  int lev[kTreeMaxDepth + 1] = {};  // lev[t]: nodes at depths 1 .. t
  int N = 0, bmax = 1;
  uint64_t sig() const {
    uint64_t g = static_cast<uint64_t>(depth);
    for (int l = 0; l < depth; ++l) g = g * 131 + static_cast<uint64_t>(branch[l]);
    return g;
  }
};

struct LayerW {
  void *wqkv = nullptr; float *sqkv = nullptr, *bqkv = nullptr;
  void *wo = nullptr; float *so = nullptr, *bo = nullptr;
  void *wgu = nullptr; float *sgu = nullptr, *bgu = nullptr;  // ref: gate/up interleaved; cfg: fc1
  void *wd = nullptr; float *sd = nullptr, *bd = nullptr;     // ref: down; cfg: fc2
  float *g1 = nullptr, *b1 = nullptr, *g2 = nullptr, *b2 = nullptr;
};

struct ModelW {
  Dims dm{};
  float *emb = nullptr, *pos = nullptr, *gf = nullptr, *bfin = nullptr;
  void *whead = nullptr; float *shead = nullptr, *bhead = nullptr;
  std::vector<LayerW> layers;
  bool loaded = false;
};

struct GraphKey {
  int B, S, k, greedy, rng_mode, catchup, max_new, u_rounds;
  float T;
  uint32_t seed;
  int top_k;
  float top_p;
  uint64_t tree_sig;  // 0: chain; else depth and branching
  int mode = 0;       // 0: a whole generation; 1: rounds of the step API
  bool operator<(const GraphKey &o) const {
    return std::tie(B, S, k, greedy, rng_mode, catchup, max_new, u_rounds, T, seed, top_k, top_p, tree_sig, mode) <
           std::tie(o.B, o.S, o.k, o.greedy, o.rng_mode, o.catchup, o.max_new, o.u_rounds, o.T, o.seed, o.top_k,
                    o.top_p, o.tree_sig, o.mode);
  }
};

struct GraphEntry {
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  int64_t fixed_kernels = 0;   // kernels outside the loop
  int64_t body_kernels = 0;    // kernels per loop iteration
};

__global__ void mt_seed_kernel(uint32_t *mt, int *mt_idx, uint32_t seed, int B) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  // std::mersenne_twister_engine::seed: x0 = seed, xi = f * (x_{i-1} ^ (x_{i-1} >> 30)) + i
  uint32_t *g = mt + static_cast<size_t>(b) * kMtN;
  uint32_t x = seed + static_cast<uint32_t>(b);
  g[0] = x;
  for (int i = 1; i < kMtN; ++i) {
    x = 1812433253u * (x ^ (x >> 30)) + static_cast<uint32_t>(i);
    g[i] = x;
  }
  mt_idx[b] = kMtN;
}

// Last kernel of a round: decides whether the WHILE node runs again and
// resets the per-round active counter.  The loop is bounded: every active
// request emits at least one token per round.
__global__ void round_cond_kernel(cudaGraphConditionalHandle hnd, int *active_count, int *iters, int max_iters,
                                  int *err) {
  const int it = *iters + 1;
  *iters = it;
  unsigned int more = (*active_count > 0) ? 1u : 0u;
  *active_count = 0;
  if (more && it >= max_iters) {
    atomicOr(err, kErrSeqLen);
    more = 0u;
  }
  cudaGraphSetConditional(hnd, more);
}

__global__ void set_int_kernel(int *p, int v) { *p = v; }

__global__ void count_iter_kernel(int *iters, int *active_count) {
  *iters = *iters + 1;
  *active_count = 0;
}

// Before the WHILE node: enter the loop only if a request is still active.
__global__ void prime_cond_kernel(cudaGraphConditionalHandle hnd, const int *active, int B) {
  int any = 0;
  for (int b = threadIdx.x; b < B; b += blockDim.x) any |= active[b];
  any = __any_sync(0xffffffffu, any);
  if (threadIdx.x == 0) cudaGraphSetConditional(hnd, any ? 1u : 0u);
}

// Head-row selection that never changes: row 2b+1 of draft step 0.
__global__ void fill_odd_kernel(int *sel, int B) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) sel[b] = 2 * b + 1;
}

// Step API (one call = a bounded number of rounds).  Before the rounds: each
// request's emitted-token count, so the call can return the tokens it added.
__global__ void step_begin_kernel(const int *n_new, int *base, int B) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) base[b] = n_new[b];
}

// Enters the round loop when a request is active and the call asked for rounds.
__global__ void step_prime_kernel(cudaGraphConditionalHandle hnd, const int *active, int B, const int *target) {
  int any = 0;
  for (int b = threadIdx.x; b < B; b += blockDim.x) any |= active[b];
  any = __any_sync(0xffffffffu, any);
  if (threadIdx.x == 0) cudaGraphSetConditional(hnd, (any && *target > 0) ? 1u : 0u);
}

// Last kernel of a step round: another round while a request is active and
// fewer than *target rounds have run in this call.
__global__ void step_cond_kernel(cudaGraphConditionalHandle hnd, int *active_count, int *iters, const int *target) {
  const int it = *iters + 1;
  *iters = it;
  const unsigned int more = (*active_count > 0 && it < *target) ? 1u : 0u;
  *active_count = 0;
  cudaGraphSetConditional(hnd, more);
}

// Rows of the attention probe: request b's last q cached positions (token 0).
__global__ void probe_rows_kernel(const int *len, int B, int q, int *tok, int *pos, int *req) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= B * q) return;
  const int b = r / q, i = r % q;
  tok[r] = 0;
  pos[r] = max(0, len[b] - q + i);
  req[r] = b;
}

// After the rounds: the tokens each request emitted in this call (at most
// cap per request; count = all it emitted).
__global__ void step_collect_kernel(const int *tokens_out, int out_len, int prompt_len, const int *n_new,
                                    const int *base, int B, int cap, int *out, int *counts) {
  const int b = blockIdx.x;
  if (b >= B) return;
  const int b0 = base[b], n = n_new[b] - b0;
  const int lim = min(max(n, 0), min(cap, out_len - prompt_len - b0));
  for (int i = threadIdx.x; i < lim; i += blockDim.x)
    out[static_cast<size_t>(b) * cap + i] = tokens_out[static_cast<size_t>(b) * out_len + prompt_len + b0 + i];
  if (threadIdx.x == 0) counts[b] = n;
}

}  // namespace

struct specdec_handle {
  specdec_config cfg{};
  int device = 0;
  cudaStream_t stream = nullptr;
  std::string err;
  ModelW tgt, dft;
  std::vector<void *> allocs;
  std::vector<void *> weight_allocs[2];
  std::map<const void *, void *> w_bf16;  // int8 weight matrix -> its bf16 image (tensor-core path)

  // caches
  void *tk = nullptr, *tv = nullptr, *dk = nullptr, *dv = nullptr;
  float *tks = nullptr, *tvs = nullptr, *dks = nullptr, *dvs = nullptr;  // int8 cache: per-row scales
  float *KVN = nullptr;                                                  // int8 cache: staged K/V rows
  size_t t_layer_stride = 0, d_layer_stride = 0;  // elements of one layer's page pool
  int t_cap = 0, d_cap = 0;                        // positions per request (the models' max_seq_len)
  // Paged KV cache: the pools hold kv_pages pages of kKvPage positions;
  // request slot b's page table is d_pt[b * ppr .. b * ppr + ppr) (shared by
  // the target and draft pools and by all layers).
  int kv_pages = 0, ppr = 0;
  int *d_pt = nullptr;
  std::vector<int> h_pt;
  float2 *rope = nullptr;
  int rope_max = 0, rope_D = 0;

  // activations: X layer input / residual stream, H projection outputs,
  // X1 normed rows, A FFN hidden, Q queries, ATT attention out
  int R_max = 0;
  int num_sms = 148;
  size_t act_elt = 4;
  void *X = nullptr, *H = nullptr, *X1 = nullptr, *A = nullptr, *Q = nullptr, *ATT = nullptr;
  float *logits = nullptr;
  RowPool pool{};
  int *sel_odd = nullptr, *sel_prefill = nullptr;

  // speculative state
  SpecState st{};
  int *d_prompts = nullptr, *d_out = nullptr;
  long long *d_stats = nullptr;
  float *d_uniforms = nullptr;
  size_t uniforms_cap = 0;
  int *d_iters = nullptr;
  int *h_pinned = nullptr;
  // step API: open after specdec_prefill; the graph key of its rounds, the
  // next round's index (host uniforms of a step go to that row), the
  // per-request counts before the current call and its round target
  bool step_open = false;
  GraphKey step_key{};
  int step_round = 0;
  int *d_step_base = nullptr, *d_step_target = nullptr, *d_step_tok = nullptr, *d_step_cnt = nullptr;
  size_t step_tok_cap = 0;

  // tensor parallelism: this rank's index, the group size and its communicator
  int tp_rank = 0, tp_world = 1;
  ncclComm_t comm = nullptr;
  int max_tree = 0, tree_base = 0;
  int logits_rows = 0;              // rows of the logits buffer  // token trees: largest tree, first pool row of the tree regions
  std::map<GraphKey, GraphEntry> graphs;
  int64_t launches = 0;        // direct mode: kernels enqueued by the last call; -1 in graph mode
  int64_t graph_fixed = 0, graph_body = 0, extra_launches = 0;
  bool src_device = false;  // the parameters being loaded are device arrays (specdec_load_params_device)
  bool use_graph = true;
  bool use_pdl = true;  // programmatic dependent launch for the kernels that support it
  int gemm_max_split = 1;  // largest split-K cluster of the tensor-core GEMM
  int gemm_clusters[kGemmMaxSplit + 1] = {};  // split-K clusters of ks CTAs resident at once
  float *gemm_ws = nullptr;  // split-K partial tiles [tile * ks + rank][column][row]
  int samp_max_cluster = 1;  // largest cluster of draft_sample_cluster_kernel
  int attn_ctas_per_sm = 2;  // attention splits the cache while the grid stays within this many CTAs per SM
  bool attn_tc = true;       // tensor-core attention for bf16 caches, head_dim 64, groups of >= attn_tc_min_q queries
  bool attn_dec = true;      // tensor-core decode attention for bf16 caches, head_dim 128, groups of <= 16 queries
  float *ad_part = nullptr;  // its split partials [groups * heads * kAdMaxSplit][kAdPartFloats]
  int *ad_ticket = nullptr;  // its per-(group, head) split counters
  int ad_groups = 0;         // groups the partial buffer holds
  int attn_tc_min_q = kAtcMinQ;
  // row batches that take the tensor-core GEMM instead of the GEMV: at least
  // gemm_min_rows rows, or gemm_wide_rows rows of a layer with at least
  // gemm_wide_elems weights
  // tensor-core GEMM on the int8 codes for row batches of at most kW8MaxRows
  // (opt-in: measured slower than the bf16-image GEMM on the large config)
  bool gemm_w8 = false;
  int w8_clusters[kW8MaxSplit + 1] = {};  // its split-K clusters of ks CTAs resident at once
  float *w8_ws = nullptr;  // its split-K partials: up to kW8WsTiles CTAs of kW8MaxRows x 128 fp32
  static constexpr int kW8WsTiles = 2 * 148;
  // persistent stream-K GEMM for row batches of at most kSkMaxRows whose
  // layers have at least sk_min_tiles 256-column tiles: the gate/up
  // projection (86 tiles) and lm_head (125) of the large config.  Measured
  // there: faster than the tile GEMM from about 80 tiles (verify gate/up 81
  // against 105 us, lm_head 105 against 122 us), slower on QKV (48 tiles:
  // 64 against 56 us), which keeps the tile GEMM with its cluster split-K
  bool gemm_sk = true;
  int sk_min_tiles = 80;
  int sk_max_ctas = 0;       // persistent CTAs of a launch (0: one per SM)
  float *sk_ws = nullptr;    // its partial tiles: two per CTA, 256 x 256 fp32
  int gemm_min_rows = kGemmMinRows;
  int gemm_wide_rows = 16;
  long long gemm_wide_elems = 2ll << 20;  // measured: the medium model's FFN down-projection (2.4M) at 32 rows

  void *dalloc(size_t bytes, std::vector<void *> *owner = nullptr) {
    void *p = nullptr;
    CK(cudaMalloc(&p, bytes ? bytes : 16));
    (owner ? *owner : allocs).push_back(p);
    return p;
  }
};

namespace {

bool act_bf16(const specdec_handle *h) { return h->cfg.act_dtype == SPECDEC_BF16; }
bool w_int8(const specdec_handle *h) { return h->cfg.weight_dtype == SPECDEC_INT8; }

Dims make_dims(const specdec_model_config &m) {
  Dims d{};
  d.V = m.vocab_size;
  d.d = m.d_model;
  d.H = m.n_heads;
  d.Hkv = m.n_kv_heads ? m.n_kv_heads : m.n_heads;
  d.D = m.n_heads ? m.d_model / m.n_heads : 0;
  d.F = m.d_ff;
  d.L = m.n_layers;
  d.max_seq = m.max_seq_len;
  d.arch = m.arch;
  d.kvd = d.Hkv * d.D;
  d.dq = d.H * d.D;
  d.Hg = d.H;
  d.Hkvg = d.Hkv;
  d.Fg = d.F;
  return d;
}

// This rank's share of a model under `world`-way tensor parallelism.
void shard_dims(Dims &d, int world, const char *who) {
  if (world <= 1) return;
  if (d.H % world || d.Hkv % world || d.F % world)
    fail(SPECDEC_ERR_INVALID, std::string(who) + ": heads, kv heads and d_ff must divide by the tensor-parallel size");
  d.H /= world;
  d.Hkv /= world;
  d.F /= world;
  d.kvd = d.Hkv * d.D;
  d.dq = d.H * d.D;
}

void check_dims(const Dims &d, const char *who) {
  auto bad = [&](const char *m) { fail(SPECDEC_ERR_INVALID, std::string(who) + ": " + m); };
  if (d.V < 1 || d.d < 2 || d.H < 1 || d.F < 1 || d.L < 0 || d.max_seq < 1) bad("non-positive dimension");
  if (d.d % d.H) bad("embed_dim must be divisible by num_heads");
  if (d.H % d.Hkv) bad("num_heads must be divisible by num_kv_heads");
  if (d.D % 2) bad("rope: head dimension D must be even");
  if (d.D > kAttnThreads) bad("head dimension above 128 is not supported");
  if (d.d > 32 * 128) bad("d_model above 4096 is not supported");
  if (d.arch != SPECDEC_ARCH_REF && d.arch != SPECDEC_ARCH_CFG) bad("unknown arch");
}

// --- weights ---------------------------------------------------------------
// Runs fn(i0, i1) over [0, n) in contiguous ranges, one per host thread (at
// most 16; one range when n is small).  The loader's passes over a 6.6 G-weight
// model take minutes on one core.
template <class F>
void parallel_ranges(size_t n, F fn) {
  const size_t hw = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
  const size_t T = std::min(hw, std::max<size_t>(1, n / 64));
  if (T <= 1) {
    fn(static_cast<size_t>(0), n);
    return;
  }
  std::vector<std::thread> th;
  const size_t per = (n + T - 1) / T;
  for (size_t t = 0; t < T; ++t) {
    const size_t a = t * per, b = std::min(n, a + per);
    if (a < b) th.emplace_back(fn, a, b);
  }
  for (auto &x : th) x.join();
}

// QuantizedDense (src/nn/quantization.cpp:40-66): per-output-column scale
// max|W[:, c]| / 127 (0 -> 1), q = clamp(round(W / s), -127, 127).  Each
// thread owns a range of columns and walks the rows in order, so the column
// maxima see the same values in the same order as a column-by-column loop.
void quantize_columns(const float *w, int K, int N, std::vector<int8_t> &q, std::vector<float> &s) {
  s.assign(N, 1.f);
  q.assign(static_cast<size_t>(K) * N, 0);
  parallel_ranges(static_cast<size_t>(N), [&](size_t c0, size_t c1) {
    std::vector<float> mx(c1 - c0, 0.f);
    for (int r = 0; r < K; ++r) {
      const float *row = w + static_cast<size_t>(r) * N;
      for (size_t c = c0; c < c1; ++c) mx[c - c0] = std::max(mx[c - c0], std::abs(row[c]));
    }
    for (size_t c = c0; c < c1; ++c) {
      const float sc = mx[c - c0] / 127.0f;
      s[c] = (sc == 0.0f) ? 1.0f : sc;
    }
    for (int r = 0; r < K; ++r)
      for (size_t c = c0; c < c1; ++c) {
        float v = std::round(w[static_cast<size_t>(r) * N + c] / s[c]);
        v = std::max(-127.0f, std::min(127.0f, v));
        q[static_cast<size_t>(r) * N + c] = static_cast<int8_t>(v);
      }
  });
}

// A set of reference Dense weights [K][N_i] (+ bias [N_i]) stacked into one
// output-major device matrix [sum N_i][K]; `interleave` stacks two equally
// wide matrices column by column (SwiGLU gate/up).
// One Dense of the reference ([K][ld] row-major, parameters() order) or the
// slice of it this rank holds: output columns col0 .. col0 + N - 1; the bias
// is replaced by zeros when !bias_on (every rank but one under tensor
// parallelism, so the bias is added once).
struct DenseSrc {
  const float *w;
  const float *b;
  int N;
  int ld = 0;    // columns of the full matrix (0: N)
  int col0 = 0;
  bool bias_on = true;
};

// Device-side loader kernels (weights that already live on the device).
// Per output column c of a Dense weight [Kfull][ld] (columns col0 .. col0 + N
// - 1): the QuantizedDense scale max|W[:, c]| / 127, 0 -> 1
// (src/nn/quantization.cpp:40-66), the same arithmetic as quantize_columns.
__global__ void col_scale_kernel(const float *__restrict__ w, int Kfull, int ld, int col0, int N,
                                 float *__restrict__ scale) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= N) return;
  float mx = 0.f;
  for (int r = 0; r < Kfull; ++r) mx = fmaxf(mx, fabsf(w[static_cast<size_t>(r) * ld + col0 + c]));
  const float sc = __fdiv_rn(mx, 127.0f);
  scale[c] = sc == 0.0f ? 1.0f : sc;
}

// The transpose to output-major rows through a 32 x 32 shared tile (both
// sides coalesced): row mul * c + add of dst [.][K] gets input rows row0 ..
// row0 + K - 1 of column col0 + c, as int8 codes q = clamp(round(w / s),
// +-127) or as fp32.
template <bool I8>
__global__ void quant_transpose_kernel(const float *__restrict__ w, int ld, int col0, int row0, int K, int N,
                                       const float *__restrict__ scale, void *__restrict__ dst, int mul, int add) {
  __shared__ float tile[32][33];
  const int c0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;
#pragma unroll
  for (int j = 0; j < 32; j += 8) {
    const int k = k0 + ty + j, c = c0 + tx;
    tile[ty + j][tx] = (k < K && c < N) ? w[static_cast<size_t>(row0 + k) * ld + col0 + c] : 0.f;
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < 32; j += 8) {
    const int c = c0 + ty + j, k = k0 + tx;
    if (c >= N || k >= K) continue;
    const float v = tile[tx][ty + j];
    const size_t o = static_cast<size_t>(mul * c + add) * K + k;
    if constexpr (I8) {
      const float q = fminf(127.0f, fmaxf(-127.0f, roundf(__fdiv_rn(v, scale[c]))));
      static_cast<int8_t *>(dst)[o] = static_cast<int8_t>(q);
    } else {
      static_cast<float *>(dst)[o] = v;
    }
  }
}

// Uploads the given Dense sources stacked (or, with `interleave`, row by row)
// as one output-major matrix [sum N][K].  K is the rank's input slice, rows
// row0 .. row0 + K - 1 of the Kfull input rows (Kfull = 0: K).  int8 scales
// are per output column over all Kfull rows, as QuantizedDense computes them
// on the whole matrix.
void upload_stacked(specdec_handle *h, int role, const std::vector<DenseSrc> &src, int K, bool interleave,
                    void **wout, float **sout, float **bout, int Kfull = 0, int row0 = 0) {
  if (Kfull == 0) Kfull = K;
  int Ntot = 0;
  for (auto &s : src) Ntot += s.N;
  std::vector<float> bias(Ntot);
  std::vector<float> scale(Ntot, 1.f);
  const bool i8 = w_int8(h);
  auto &own = h->weight_allocs[role];
  const size_t wbytes = static_cast<size_t>(Ntot) * K * (i8 ? 1 : 4);
  void *dw = h->dalloc(wbytes, &own);
  std::vector<float> wf;
  std::vector<int8_t> wq;
  if (h->src_device) {
    // the sources are device arrays: scales and the transpose on the device,
    // the (small) bias and scale vectors through the host
    float *dsc = static_cast<float *>(h->dalloc(static_cast<size_t>(std::max(1, Ntot)) * sizeof(float)));
    int base = 0;
    for (size_t m = 0; m < src.size(); ++m) {
      const DenseSrc &s = src[m];
      const int ld = s.ld ? s.ld : s.N;
      if (i8)
        col_scale_kernel<<<(s.N + 255) / 256, 256, 0, h->stream>>>(s.w, Kfull, ld, s.col0, s.N, dsc);
      const dim3 grid((s.N + 31) / 32, (K + 31) / 32), block(32, 8);
      const int mul = interleave ? 2 : 1, add = interleave ? static_cast<int>(m) : base;
      if (i8)
        quant_transpose_kernel<true><<<grid, block, 0, h->stream>>>(s.w, ld, s.col0, row0, K, s.N, dsc, dw, mul, add);
      else
        quant_transpose_kernel<false><<<grid, block, 0, h->stream>>>(s.w, ld, s.col0, row0, K, s.N, nullptr, dw, mul,
                                                                     add);
      CK(cudaGetLastError());
      std::vector<float> hb(s.N), hs(s.N, 1.f);
      CK(cudaMemcpyAsync(hb.data(), s.b + s.col0, s.N * sizeof(float), cudaMemcpyDeviceToHost, h->stream));
      if (i8) CK(cudaMemcpyAsync(hs.data(), dsc, s.N * sizeof(float), cudaMemcpyDeviceToHost, h->stream));
      CK(cudaStreamSynchronize(h->stream));
      for (int c = 0; c < s.N; ++c) {
        const int row = interleave ? (2 * c + static_cast<int>(m)) : (base + c);
        bias[row] = s.bias_on ? hb[c] : 0.f;
        scale[row] = hs[c];
      }
      base += s.N;
    }
    cudaFree(dsc);
    h->allocs.pop_back();
  } else {
    if (i8) wq.assign(static_cast<size_t>(Ntot) * K, 0);
    else wf.assign(static_cast<size_t>(Ntot) * K, 0.f);
  }
  int base = 0;
  for (size_t m = 0; m < (h->src_device ? 0 : src.size()); ++m) {
    const DenseSrc &s = src[m];
    const int ld = s.ld ? s.ld : s.N;
    std::vector<int8_t> q;
    std::vector<float> sc;
    if (i8) quantize_columns(s.w, Kfull, ld, q, sc);
    for (int c = 0; c < s.N; ++c) {
      const int gc = s.col0 + c;
      const int row = interleave ? (2 * c + static_cast<int>(m)) : (base + c);
      bias[row] = s.bias_on ? s.b[gc] : 0.f;
      if (i8) scale[row] = sc[gc];
    }
    // the transpose to output-major rows, in 32-column x 256-row blocks so the
    // strided source rows stay in cache; threads own disjoint output rows
    parallel_ranges(static_cast<size_t>(s.N), [&](size_t cb, size_t ce) {
      for (size_t c0 = cb; c0 < ce; c0 += 32) {
        const size_t c1 = std::min(ce, c0 + 32);
        for (int k0 = 0; k0 < K; k0 += 256) {
          const int k1 = std::min(K, k0 + 256);
          for (size_t c = c0; c < c1; ++c) {
            const size_t gc = static_cast<size_t>(s.col0) + c;
            const size_t row = interleave ? (2 * c + m) : (static_cast<size_t>(base) + c);
            for (int k = k0; k < k1; ++k) {
              const size_t si = static_cast<size_t>(row0 + k) * ld + gc;
              if (i8) wq[row * K + k] = q[si];
              else wf[row * K + k] = s.w[si];
            }
          }
        }
      }
    });
    base += s.N;
  }
  if (!h->src_device)
    CK(cudaMemcpy(dw, i8 ? static_cast<const void *>(wq.data()) : static_cast<const void *>(wf.data()), wbytes,
                  cudaMemcpyHostToDevice));
  float *db = static_cast<float *>(h->dalloc(Ntot * sizeof(float), &own));
  CK(cudaMemcpy(db, bias.data(), Ntot * sizeof(float), cudaMemcpyHostToDevice));
  float *ds = nullptr;
  if (i8) {
    ds = static_cast<float *>(h->dalloc(Ntot * sizeof(float), &own));
    CK(cudaMemcpy(ds, scale.data(), Ntot * sizeof(float), cudaMemcpyHostToDevice));
  }
  if (i8 && act_bf16(h)) {
    // exact bf16 image of the codes for the tensor-core GEMM (large row
    // batches), in the GEMM's tile order
    const int nkb = (K + kBK - 1) / kBK;
    const size_t n = static_cast<size_t>((Ntot + kBN - 1) / kBN) * nkb * kBN * kBK;
    void *dw16 = h->dalloc(n * 2, &own);
    i8_to_bf16_tiles_kernel<<<static_cast<unsigned>(std::min<size_t>((n + 255) / 256, 8192)), 256, 0, h->stream>>>(
        static_cast<const int8_t *>(dw), static_cast<__nv_bfloat16 *>(dw16), Ntot, K, nkb, n);
    CK(cudaGetLastError());
    CK(cudaStreamSynchronize(h->stream));
    h->w_bf16[dw] = dw16;
  }
  *wout = dw;
  *sout = ds;
  *bout = db;
}

float *upload_vec(specdec_handle *h, int role, const float *p, size_t n) {
  float *d = static_cast<float *>(h->dalloc(n * sizeof(float), &h->weight_allocs[role]));
  CK(cudaMemcpy(d, p, n * sizeof(float), h->src_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice));
  return d;
}

// Tensor shapes of TransformerDecoder::parameters() (the order load_model
// reads): Embedding [V, d] (src/nn/layer.cpp:267), Dense weight [in, out] and
// bias [1, out] (src/nn/layer.cpp:153-157), LayerNorm gamma / beta [d]
// (src/nn/layer.cpp:1063-1064).  The cfg architecture (no reference
// counterpart) adds positions [max_seq, d] and a final LayerNorm.
std::vector<std::vector<uint64_t>> param_shapes(const Dims &dm) {
  const uint64_t d = dm.d, F = dm.Fg, V = dm.V, kvd = static_cast<uint64_t>(dm.Hkvg) * dm.D;
  const bool ref = dm.arch == SPECDEC_ARCH_REF;
  std::vector<std::vector<uint64_t>> s;
  auto dense = [&](uint64_t in, uint64_t out) {
    s.push_back({in, out});
    s.push_back({1, out});
  };
  s.push_back({V, d});
  if (!ref) s.push_back({static_cast<uint64_t>(dm.max_seq), d});
  for (int l = 0; l < dm.L; ++l) {
    if (!ref) { s.push_back({d}); s.push_back({d}); }
    dense(d, d); dense(d, kvd); dense(d, kvd); dense(d, d);
    if (ref) {
      dense(d, F); dense(d, F); dense(F, d);
      for (int i = 0; i < 4; ++i) s.push_back({d});
    } else {
      s.push_back({d}); s.push_back({d});
      dense(d, F); dense(F, d);
    }
  }
  if (!ref) { s.push_back({d}); s.push_back({d}); }
  dense(d, V);
  return s;
}

void load_model(specdec_handle *h, int role, ModelW &m, int n, const float *const *P, const int64_t *numel) {
  const Dims &dm = m.dm;
  // parameter shapes are the whole model's; this rank keeps its slices
  const int d = dm.d, F = dm.Fg, V = dm.V, kvd = dm.Hkvg * dm.D;
  const int r = h->tp_rank;
  const int dq = dm.dq, kvl = dm.kvd, Fl = dm.F;
  const bool bias_rank = r == 0;  // the rank that adds the biases of the row-sliced layers
  const bool ref = dm.arch == SPECDEC_ARCH_REF;
  const int per = ref ? 18 : 16;
  const int lead = ref ? 1 : 2, tail = ref ? 2 : 4;
  const int expect = lead + per * dm.L + tail;
  if (n != expect) fail(SPECDEC_ERR_INVALID, "expected " + std::to_string(expect) + " parameters, got " + std::to_string(n));
  // shape checks (element counts) in parameters() order
  std::vector<int64_t> want;
  want.push_back(static_cast<int64_t>(V) * d);
  if (!ref) want.push_back(static_cast<int64_t>(dm.max_seq) * d);
  for (int l = 0; l < dm.L; ++l) {
    std::vector<int64_t> attn = {int64_t(d) * d, d, int64_t(d) * kvd, kvd, int64_t(d) * kvd, kvd, int64_t(d) * d, d};
    if (ref) {
      want.insert(want.end(), attn.begin(), attn.end());
      for (int64_t x : {int64_t(d) * F, int64_t(F), int64_t(d) * F, int64_t(F), int64_t(F) * d, int64_t(d)}) want.push_back(x);
      for (int i = 0; i < 4; ++i) want.push_back(d);
    } else {
      want.push_back(d); want.push_back(d);
      want.insert(want.end(), attn.begin(), attn.end());
      want.push_back(d); want.push_back(d);
      for (int64_t x : {int64_t(d) * F, int64_t(F), int64_t(F) * d, int64_t(d)}) want.push_back(x);
    }
  }
  if (!ref) { want.push_back(d); want.push_back(d); }
  want.push_back(static_cast<int64_t>(d) * V);
  want.push_back(V);
  for (int i = 0; i < n; ++i) {
    if (!P[i]) fail(SPECDEC_ERR_INVALID, "parameter " + std::to_string(i) + " is null");
    if (numel[i] != want[i])
      fail(SPECDEC_ERR_INVALID, "parameter " + std::to_string(i) + " has " + std::to_string(numel[i]) +
                                    " elements, expected " + std::to_string(want[i]));
  }
  for (void *p : h->weight_allocs[role]) cudaFree(p);
  h->weight_allocs[role].clear();

  int i = 0;
  m.emb = upload_vec(h, role, P[i++], static_cast<size_t>(V) * d);
  if (!ref) m.pos = upload_vec(h, role, P[i++], static_cast<size_t>(dm.max_seq) * d);
  m.layers.assign(dm.L, LayerW{});
  for (int l = 0; l < dm.L; ++l) {
    LayerW &L = m.layers[l];
    if (!ref) { L.g1 = upload_vec(h, role, P[i], d); L.b1 = upload_vec(h, role, P[i + 1], d); i += 2; }
    const float *qw = P[i], *qb = P[i + 1], *kw = P[i + 2], *kb = P[i + 3], *vw = P[i + 4], *vb = P[i + 5];
    const float *ow = P[i + 6], *ob = P[i + 7];
    i += 8;
    upload_stacked(h, role, {{qw, qb, dq, d, r * dq}, {kw, kb, kvl, kvd, r * kvl}, {vw, vb, kvl, kvd, r * kvl}}, d,
                   false, &L.wqkv, &L.sqkv, &L.bqkv);
    upload_stacked(h, role, {{ow, ob, d, d, 0, bias_rank}}, dq, false, &L.wo, &L.so, &L.bo, d, r * dq);
    if (ref) {
      const float *gw = P[i], *gb = P[i + 1], *uw = P[i + 2], *ub = P[i + 3], *dw = P[i + 4], *db = P[i + 5];
      i += 6;
      upload_stacked(h, role, {{gw, gb, Fl, F, r * Fl}, {uw, ub, Fl, F, r * Fl}}, d, true, &L.wgu, &L.sgu, &L.bgu);
      upload_stacked(h, role, {{dw, db, d, d, 0, bias_rank}}, Fl, false, &L.wd, &L.sd, &L.bd, F, r * Fl);
      L.g1 = upload_vec(h, role, P[i], d); L.b1 = upload_vec(h, role, P[i + 1], d);
      L.g2 = upload_vec(h, role, P[i + 2], d); L.b2 = upload_vec(h, role, P[i + 3], d);
      i += 4;
    } else {
      L.g2 = upload_vec(h, role, P[i], d); L.b2 = upload_vec(h, role, P[i + 1], d);
      i += 2;
      const float *f1w = P[i], *f1b = P[i + 1], *f2w = P[i + 2], *f2b = P[i + 3];
      i += 4;
      upload_stacked(h, role, {{f1w, f1b, Fl, F, r * Fl}}, d, false, &L.wgu, &L.sgu, &L.bgu);
      upload_stacked(h, role, {{f2w, f2b, d, d, 0, bias_rank}}, Fl, false, &L.wd, &L.sd, &L.bd, F, r * Fl);
    }
  }
  if (!ref) { m.gf = upload_vec(h, role, P[i], d); m.bfin = upload_vec(h, role, P[i + 1], d); i += 2; }
  upload_stacked(h, role, {{P[i], P[i + 1], V}}, d, false, &m.whead, &m.shead, &m.bhead);
  m.loaded = true;
}

// --- kernel launch helpers ---------------------------------------------------
template <typename... KArgs, typename... Args>
void launch(specdec_handle *h, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, Args... args) {
  kern<<<grid, block, smem, h->stream>>>(static_cast<KArgs>(args)...);
  CK(cudaGetLastError());
  ++h->launches;
}

// A launch whose CTAs form thread-block clusters of `cluster` CTAs (1 x 1 x 1:
// no cluster), with programmatic stream serialization when the kernel
// supports it (pdl_launch / pdl_wait, common.cuh) and the handle allows it.
template <typename... KArgs, typename... Args>
void launch_ex(specdec_handle *h, bool pdl, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, dim3 cluster,
               Args... args) {
  cudaLaunchConfig_t lc{};
  lc.gridDim = grid;
  lc.blockDim = block;
  lc.dynamicSmemBytes = smem;
  lc.stream = h->stream;
  cudaLaunchAttribute at[2];
  int na = 0;
  if (cluster.x * cluster.y * cluster.z > 1) {
    at[na].id = cudaLaunchAttributeClusterDimension;
    at[na].val.clusterDim.x = cluster.x;
    at[na].val.clusterDim.y = cluster.y;
    at[na].val.clusterDim.z = cluster.z;
    ++na;
  }
  if (pdl && h->use_pdl) {
    at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  lc.attrs = at;
  lc.numAttrs = na;
  CK(cudaLaunchKernelEx(&lc, kern, static_cast<KArgs>(args)...));
  ++h->launches;
}
template <typename... KArgs, typename... Args>
void launch_cluster(specdec_handle *h, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, dim3 cluster,
                    Args... args) {
  launch_ex(h, true, kern, grid, block, smem, cluster, args...);
}
template <typename... KArgs, typename... Args>
void launch_pdl(specdec_handle *h, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, Args... args) {
  launch_ex(h, true, kern, grid, block, smem, dim3(1, 1, 1), args...);
}

// Launch of a kernel given by pointer (a table entry of kern_linear.cu /
// kern_attn.cu) whose one parameter is `arg`, with clusters and programmatic
// stream serialization as launch_ex.
template <typename Arg>
void launch_fn(specdec_handle *h, bool pdl, const void *fn, dim3 grid, dim3 block, size_t smem, dim3 cluster,
               const Arg &arg) {
  if (!fn) fail(SPECDEC_ERR_UNSUPPORTED, "no kernel variant for this shape");
  cudaLaunchConfig_t lc{};
  lc.gridDim = grid;
  lc.blockDim = block;
  lc.dynamicSmemBytes = smem;
  lc.stream = h->stream;
  cudaLaunchAttribute at[2];
  int na = 0;
  if (cluster.x * cluster.y * cluster.z > 1) {
    at[na].id = cudaLaunchAttributeClusterDimension;
    at[na].val.clusterDim.x = cluster.x;
    at[na].val.clusterDim.y = cluster.y;
    at[na].val.clusterDim.z = cluster.z;
    ++na;
  }
  if (pdl && h->use_pdl) {
    at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  lc.attrs = at;
  lc.numAttrs = na;
  void *args[1] = {const_cast<Arg *>(&arg)};
  CK(cudaLaunchKernelExC(&lc, fn, args));
  ++h->launches;
}

// cuTensorMapEncodeTiled, looked up from the driver once (no link-time
// dependency on libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  if (!fn) fail(SPECDEC_ERR_CUDA, "the driver does not provide cuTensorMapEncodeTiled");
  return fn;
}

// 2-D TMA view [rows][D] of one layer's K or V cache (row = slot * Hkv * S_cap
// + kv head * S_cap + position), box = the attention kernel's tile with its
// swizzle (AttnGeom).  Rows past the end read as zeros.
template <typename KT> CUtensorMapDataType tmap_type();
template <> CUtensorMapDataType tmap_type<float>() { return CU_TENSOR_MAP_DATA_TYPE_FLOAT32; }
template <> CUtensorMapDataType tmap_type<__nv_bfloat16>() { return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; }
template <> CUtensorMapDataType tmap_type<int8_t>() { return CU_TENSOR_MAP_DATA_TYPE_UINT8; }

template <typename KT, int D>
CUtensorMap kv_tensor_map(const void *base, size_t rows) {
  using G = AttnGeom<KT, D>;
  if (rows >= (size_t(1) << 31)) fail(SPECDEC_ERR_UNSUPPORTED, "KV cache too large for 32-bit TMA row coordinates");
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(G::kRowBytes)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(G::kBoxCols), static_cast<cuuint32_t>(G::kTile)};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw = G::kSw == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                : G::kSw == 64  ? CU_TENSOR_MAP_SWIZZLE_64B
                                : G::kSw == 32  ? CU_TENSOR_MAP_SWIZZLE_32B
                                                : CU_TENSOR_MAP_SWIZZLE_NONE;
  const CUresult r = tensor_map_encoder()(&m, tmap_type<KT>(), 2, const_cast<void *>(base), dims, strides, box, estr,
                                          CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) fail(SPECDEC_ERR_CUDA, "cuTensorMapEncodeTiled failed with " + std::to_string(static_cast<int>(r)));
  return m;
}

// Columns per warp: one pair while the grid of one-pair warps fits a wave
// (two blocks per SM), else two pairs (each input vector then feeds four
// weight columns and the grid halves).  K-split: the smallest power of two (at
// most 8) that gives about one block per SM or leaves each lane at most one
// weight vector per column.
int pick_ncols(int N, int R, int K, int E, int num_sms) {
  const int row_tiles = (R + kRowTile - 1) / kRowTile;
  const long blocks2 = static_cast<long>((N + 2 * kLinWarps - 1) / (2 * kLinWarps)) * row_tiles;
  return blocks2 > 2L * num_sms ? 4 : 2;
}
int pick_ksplit(int N, int R, int K, int E, int nc, int num_sms) {
  const int row_tiles = (R + kRowTile - 1) / kRowTile;
  int ks = 1;
  while (ks < 8) {
    const int cols = nc * (kLinWarps / ks);
    const long blocks = static_cast<long>((N + cols - 1) / cols) * row_tiles;
    // stop once the grid fills the GPU, unless lanes would still stream more
    // than two weight vectors each (long K: the loop's load latency adds up)
    if ((blocks >= num_sms && K / E <= 64 * ks) || K / E <= 32 * ks) break;
    ks *= 2;
  }
  return ks;
}

constexpr size_t kLinLnSmemMax = 128 * 1024;

template <int EPI, int NC>
void launch_linear_nc(specdec_handle *h, const LinearArgs &a, dim3 grid, dim3 block) {
  const bool bf = act_bf16(h), i8 = w_int8(h);
  size_t smem = 0;
  if (a.in_g) {
    smem = static_cast<size_t>(kRowTile) * a.K * h->act_elt;
    if (smem > kLinLnSmemMax) fail(SPECDEC_ERR_UNSUPPORTED, "input rows too wide for the fused LayerNorm");
  }
  launch_fn(h, true, linear_kernel_fn(i8, bf, EPI, a.in_g ? 1 : 0, NC), grid, block, smem, dim3(1, 1, 1), a);
}

// 2-D TMA view [rows][K] of a bf16 matrix with row stride ld elements, box
// kBK x box_rows, 128-byte swizzle (the K-major operand layout of the GEMM).
CUtensorMap gemm_operand_map(const void *base, int K, int rows, int ld, int box_rows) {
  if ((ld * 2) % 16 != 0 || (reinterpret_cast<uintptr_t>(base) & 15) != 0)
    fail(SPECDEC_ERR_UNSUPPORTED, "tensor-core GEMM operands need 16-byte aligned rows");
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = tensor_map_encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims,
                                          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) fail(SPECDEC_ERR_CUDA, "cuTensorMapEncodeTiled failed with " + std::to_string(static_cast<int>(r)));
  return m;
}

// 2-D TMA view of a bf16 weight image in tile order: rows of 64 elements
// (128 bytes), block (t, kb) = rows (t nkb + kb) 256 .. + 255; box 64 x 256.
CUtensorMap weight_tiles_map(const void *base, int K, int N) {
  const int nkb = (K + kBK - 1) / kBK, nt = (N + kBN - 1) / kBN;
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(kBK), static_cast<cuuint64_t>(nt) * nkb * kBN};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(kBK) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(kBN)};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = tensor_map_encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims,
                                          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) fail(SPECDEC_ERR_CUDA, "cuTensorMapEncodeTiled failed with " + std::to_string(static_cast<int>(r)));
  return m;
}

// LayerNorm of a's input rows (bf16) into contiguous rows at dst.
bool ln_rows_ok(const LinearArgs &a) {
  return a.K % 8 == 0 && a.ldx % 8 == 0 && a.K <= 4096 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0;
}
void launch_ln_rows(specdec_handle *h, const LinearArgs &a, void *dst) {
  if (!ln_rows_ok(a)) fail(SPECDEC_ERR_UNSUPPORTED, "LayerNorm rows must be a multiple of 8 wide and 16-byte aligned");
  auto ln = a.K <= 1024 ? ln_rows_kernel<4> : a.K <= 2048 ? ln_rows_kernel<8> : ln_rows_kernel<16>;
  launch_pdl(h, ln, dim3((a.R + 1) / 2), dim3(64), 0, static_cast<const __nv_bfloat16 *>(a.x), a.ldx, a.in_rows, a.R,
         a.K, a.in_g, a.in_b, static_cast<__nv_bfloat16 *>(dst), static_cast<__nv_bfloat16 *>(nullptr));
}

// The tensor-core path: bf16 activations, int8 weights with a bf16 image, at
// least kGemmMinRows rows.  An input LayerNorm runs first as its own kernel,
// writing the normalised rows where the GEMV would have stored them
// (norm_out) or into X1, which is free whenever a LayerNorm feeds a GEMM.
template <int EPI>
bool try_launch_gemm(specdec_handle *h, LinearArgs a) {
  // >= kGemmMinRows rows, or >= 16 rows of a layer of >= 2M weights (the
  // lm_head, long FFN projections): the GEMM reads each weight once, where
  // 8-row GEMV tiles would re-read it per tile
  const bool wide = a.R >= h->gemm_wide_rows && static_cast<long long>(a.N) * a.K >= h->gemm_wide_elems;
  if (!act_bf16(h) || !w_int8(h) || (a.R < h->gemm_min_rows && !wide) || (a.K % 8) != 0) return false;
  if (a.in_g && !ln_rows_ok(a)) return false;
  // the chunked epilogue's 16-byte vectors: aligned output / residual rows,
  // and q / k / v sections and heads in whole 16-column chunks
  if (a.ldo % (a.out_f32 ? 4 : 8) != 0) return false;
  if (EPI == kEpiResid && a.ldr % 8 != 0) return false;
  if (EPI == kEpiSwiGLU && a.ldo % 8 != 0) return false;
  if (EPI == kEpiQKV && (a.qkv.d % 16 != 0 || a.qkv.kvd % 16 != 0 || a.qkv.D % 16 != 0)) return false;
  auto it = h->w_bf16.find(a.W);
  if (it == h->w_bf16.end()) return false;
  const void *A = a.x;
  int lda = a.ldx;
  if (a.in_g) {
    void *dst = a.norm_out ? a.norm_out : h->X1;
    launch_ln_rows(h, a, dst);
    A = dst;
    lda = a.K;
  } else if (a.in_rows) {
    return false;  // row gathers only come with a LayerNorm
  }
  GemmArgs g{};
  g.tma_a = gemm_operand_map(A, a.K, a.R, lda, kBM);
  g.tma_b = weight_tiles_map(it->second, a.K, a.N);
  a.in_g = a.in_b = nullptr;
  a.in_rows = nullptr;
  a.norm_out = nullptr;
  g.lin = a;
  g.err = h->st.err;
  const int gx = (a.N + kBN - 1) / kBN, gy = (a.R + kBM - 1) / kBM;
  const int nk = (a.K + kBK - 1) / kBK;
  if (h->gemm_sk && h->sk_ws && a.R <= kSkMaxRows && gx >= h->sk_min_tiles && gx <= kSkMaxTiles) {
    // row batches of a round over wide layers: the persistent stream-K GEMM
    GemmSkArgs s{};
    s.tma_a = g.tma_a;
    s.tma_b = g.tma_b;
    s.lin = a;
    s.mt = gy;
    s.nt = gx;
    s.nk = nk;
    s.ctas = std::min(h->sk_max_ctas > 0 ? std::min(h->sk_max_ctas, h->num_sms) : h->num_sms, gx * nk);
    s.ws = h->sk_ws;
    s.err = h->st.err;
    CK(gemm_sk_launch(EPI, s, h->stream, h->use_pdl));
    h->launches += 2;
    return true;
  }
  // split-K while the tiles leave most SMs idle: a power of two up to the
  // largest cluster the device schedules, each split keeping one k-block at least
  int ks = 1;
  while (h->gemm_ws && 2 * ks <= h->gemm_max_split && gx * gy * 2 * ks <= h->num_sms && 2 * ks <= nk &&
         gx * gy <= h->gemm_clusters[2 * ks])  // all clusters in one wave
    ks *= 2;
  g.ksplit = ks;
  g.ws = h->gemm_ws;
  if (ks == 1)
    launch_pdl(h, gemm_kernel<EPI>, dim3(gx, gy), dim3(kGemmThreads), static_cast<size_t>(kGemmSmem), g);
  else
    launch_ex(h, true, gemm_kernel<EPI>, dim3(gx, gy, ks), dim3(kGemmThreads), static_cast<size_t>(kGemmSmem),
              dim3(1, 1, ks), g);
  return true;
}

// 2-D TMA view [N][K] of int8 weight codes (output-major), box 64 x 128, no
// swizzle (the converter warps read it, not the tensor cores).
CUtensorMap w8_operand_map(const void *base, int K, int N) {
  if (K % 16 != 0 || (reinterpret_cast<uintptr_t>(base) & 15) != 0)
    fail(SPECDEC_ERR_UNSUPPORTED, "int8 GEMM operands need 16-byte aligned rows");
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(N)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(K)};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(kW8Feat)};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = tensor_map_encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims,
                                          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) fail(SPECDEC_ERR_CUDA, "cuTensorMapEncodeTiled failed with " + std::to_string(static_cast<int>(r)));
  return m;
}

// The int8-code tensor-core path (gemm_w8.cu): bf16 activations, int8
// weights, at most kW8MaxRows rows, the same row-count routing as the bf16
// image GEMM.  An input LayerNorm runs first as its own kernel (ln_rows), as
// for that GEMM.
template <int EPI>
bool try_launch_gemm_w8(specdec_handle *h, LinearArgs a) {
  const bool wide = a.R >= h->gemm_wide_rows && static_cast<long long>(a.N) * a.K >= h->gemm_wide_elems;
  if (!h->gemm_w8 || !act_bf16(h) || !w_int8(h) || a.R > kW8MaxRows) return false;
  if ((a.R < h->gemm_min_rows && !wide) || (a.K % 16) != 0) return false;
  if (a.in_g && !ln_rows_ok(a)) return false;
  if (EPI == kEpiSwiGLU && a.N % 2 != 0) return false;
  if (EPI == kEpiQKV && (a.qkv.D % 2 != 0)) return false;
  if (!a.in_g && a.in_rows) return false;  // row gathers only come with a LayerNorm
  const void *A = a.x;
  int lda = a.ldx;
  if (a.in_g) {
    void *dst = a.norm_out ? a.norm_out : h->X1;
    launch_ln_rows(h, a, dst);
    A = dst;
    lda = a.K;
  }
  GemmW8Args g{};
  g.np = (a.R + 15) / 16 * 16;
  g.w_bf16 = 0;  // the codes themselves (the bf16 image is in the other GEMM's tile order)
  gemm_w8_rings(g.np, g.w_bf16, &g.stages_w, &g.stages_x);
  g.tma_x = gemm_operand_map(A, a.K, a.R, lda, g.np);
  g.tma_w = w8_operand_map(a.W, a.K, a.N);
  a.in_g = a.in_b = nullptr;
  a.in_rows = nullptr;
  a.norm_out = nullptr;
  g.lin = a;
  g.err = h->st.err;
  const int tiles = (a.N + kW8Feat - 1) / kW8Feat;
  const int nk = (a.K + 63) / 64;
  // split K while the feature tiles leave SMs idle (one CTA per SM): the
  // largest power of two that keeps every CTA in one wave and at least 4
  // k-blocks per split
  int ks = 1;
  if (h->w8_ws)
    while (2 * ks <= kW8MaxSplit && tiles * 2 * ks <= std::min(h->num_sms, specdec_handle::kW8WsTiles) &&
           4 * 2 * ks <= nk && tiles <= h->w8_clusters[2 * ks])
      ks *= 2;
  g.ksplit = ks;
  g.ws = h->w8_ws;
  CK(gemm_w8_launch(EPI, g, tiles, h->stream, h->use_pdl));
  ++h->launches;
  return true;
}

template <int EPI>
void launch_linear(specdec_handle *h, LinearArgs a) {
  if (a.R <= 0) return;
  if (try_launch_gemm_w8<EPI>(h, a)) return;
  if (try_launch_gemm<EPI>(h, a)) return;
  const int E = w_int8(h) ? WVec<int8_t>::E : WVec<float>::E;
  const int nc = pick_ncols(a.N, a.R, a.K, E, h->num_sms);
  a.ksplit = pick_ksplit(a.N, a.R, a.K, E, nc, h->num_sms);
  const int cols = nc * (kLinWarps / a.ksplit);
  dim3 grid((a.N + cols - 1) / cols, (a.R + kRowTile - 1) / kRowTile);
  dim3 block(32 * kLinWarps);
  if (a.in_g && act_bf16(h) && static_cast<long long>(grid.x) * a.K > 65536 && ln_rows_ok(a)) {
    // every column block would normalise the same rows again: do it once
    void *dst = a.norm_out ? a.norm_out : h->X1;
    launch_ln_rows(h, a, dst);
    a.x = dst;
    a.ldx = a.K;
    a.in_g = a.in_b = nullptr;
    a.in_rows = nullptr;
    a.norm_out = nullptr;
  }
  if (nc == 4) launch_linear_nc<EPI, 4>(h, a, grid, block);
  else launch_linear_nc<EPI, 2>(h, a, grid, block);
}

// Dynamic shared memory of the input-LayerNorm linear kernels: kLinLnSmemMax
// holds kRowTile rows of up to 4096 fp32 or 8192 bf16 elements.
void set_linear_attrs() {
  const int b = static_cast<int>(kLinLnSmemMax);
  for (int w8 = 0; w8 < 2; ++w8)
    for (int abf = 0; abf < 2; ++abf)
      for (int epi = kEpiStore; epi <= kEpiGelu; ++epi)
        for (int nc : {2, 4})
          CK(cudaFuncSetAttribute(linear_kernel_fn(w8, abf, epi, 1, nc), cudaFuncAttributeMaxDynamicSharedMemorySize, b));
}
// Records in active[ks] how many split-K clusters of ks CTAs (kGemmSmem
// bytes each) the device runs at once (0: none) and returns the largest ks
// it can schedule.
int set_gemm_attrs(int *active) {
  CK(cudaFuncSetAttribute(gemm_kernel<kEpiStore>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmem));
  CK(cudaFuncSetAttribute(gemm_kernel<kEpiResid>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmem));
  CK(cudaFuncSetAttribute(gemm_kernel<kEpiQKV>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmem));
  CK(cudaFuncSetAttribute(gemm_kernel<kEpiSwiGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmem));
  CK(cudaFuncSetAttribute(gemm_kernel<kEpiGelu>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmem));
  int best = 1;
  for (int ks = 2; ks <= kGemmMaxSplit; ks *= 2) {
    cudaLaunchConfig_t lc{};
    lc.gridDim = dim3(1, 1, ks);
    lc.blockDim = dim3(kGemmThreads);
    lc.dynamicSmemBytes = kGemmSmem;
    cudaLaunchAttribute at{};
    at.id = cudaLaunchAttributeClusterDimension;
    at.val.clusterDim.x = 1;
    at.val.clusterDim.y = 1;
    at.val.clusterDim.z = ks;
    lc.attrs = &at;
    lc.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_kernel<kEpiResid>, &lc) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    active[ks] = n;
    if (n > 0) best = ks;
  }
  return best;
}

// Sets the shared-memory size of the cluster samplers for vocabulary V and
// returns the largest cluster (8, 4 or 2 CTAs) the device can schedule.
int set_samp_cluster_attrs(int V) {
  auto one = [&](auto kern, int cs) -> bool {
    const int bytes = static_cast<int>(((V + cs - 1) / cs + 3) & ~3) * static_cast<int>(sizeof(float));
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    cudaLaunchConfig_t lc{};
    lc.gridDim = dim3(cs);
    lc.blockDim = dim3(kSampThreads);
    lc.dynamicSmemBytes = bytes;
    cudaLaunchAttribute at{};
    at.id = cudaLaunchAttributeClusterDimension;
    at.val.clusterDim.x = cs;
    at.val.clusterDim.y = 1;
    at.val.clusterDim.z = 1;
    lc.attrs = &at;
    lc.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &lc) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    return n > 0;
  };
  int best = 1;
  if (one(draft_sample_cluster_kernel<2>, 2)) best = 2;
  if (best == 2 && one(draft_sample_cluster_kernel<4>, 4)) best = 4;
  if (best == 4 && one(draft_sample_cluster_kernel<8>, 8)) best = 8;
  return best;
}

template <typename KT, int D>
void set_attn_attr(int kt) {
  const int bytes = AttnGeom<KT, D>::smem_bytes(2);
  for (int abf = 0; abf < 2; ++abf)
    for (int qt : {1, 2, 4, 8})
      CK(cudaFuncSetAttribute(attention_kernel_fn(abf, kt, D, qt), cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
}
template <typename KT>
void set_attn_attrs(int kt) {
  set_attn_attr<KT, 4>(kt);
  set_attn_attr<KT, 8>(kt);
  set_attn_attr<KT, 16>(kt);
  set_attn_attr<KT, 32>(kt);
  set_attn_attr<KT, 64>(kt);
  set_attn_attr<KT, 128>(kt);
}

// Splits: one tile of positions per split where the cache is long, at most a
// portable cluster (8) of them, and about attn_ctas_per_sm (2) CTAs per SM
// over the grid.
template <typename AT, typename KT, int D>
void launch_attention_d(specdec_handle *h, AttnArgs &a, int ngroups, const void *kc, const void *vc, size_t rows) {
  using G = AttnGeom<KT, D>;
  if (!G::kTma) fail(SPECDEC_ERR_UNSUPPORTED, "a K/V cache row (head_dim x element size) must be a multiple of 16 bytes");
  a.tmk = kv_tensor_map<KT, D>(kc, rows);
  a.tmv = kv_tensor_map<KT, D>(vc, rows);
  const int qt = a.Q <= 1 ? 1 : a.Q <= 2 ? 2 : a.Q <= 4 ? 4 : kAttnQT;
  const int ngt = (a.Q + qt - 1) / qt;
  const int base = ngroups * ngt * a.H;
  int ns = 1;
  if (a.S_cap > G::kTile) {
    const int want = (a.S_cap + G::kTile - 1) / G::kTile;
    const int fit = std::max(1, h->attn_ctas_per_sm * h->num_sms / base);
    ns = std::min(std::min(kAttnMaxSplit, want), fit);
  }
  a.nsplit = ns;
  // whole tiles per split: a tile never straddles a page
  a.chunk = ((a.S_cap + ns - 1) / ns + G::kTile - 1) / G::kTile * G::kTile;
  const size_t smem = static_cast<size_t>(G::smem_bytes(a.chunk > G::kTile ? 2 : 1));
  dim3 grid(ngroups * ngt, a.H, ns);
  dim3 block(kAttnThreads);
  const int kt = std::is_same<KT, int8_t>::value ? 2 : std::is_same<KT, __nv_bfloat16>::value ? 1 : 0;
  const void *fn = attention_kernel_fn(std::is_same<AT, __nv_bfloat16>::value ? 1 : 0, kt, D, qt);
  launch_fn(h, true, fn, grid, block, smem, ns == 1 ? dim3(1, 1, 1) : dim3(1, 1, ns), a);
}

template <typename AT, typename KT>
void launch_attention_t(specdec_handle *h, AttnArgs &a, int D, int ngroups, const void *kc, const void *vc,
                        size_t rows) {
  switch (D) {
    case 4: launch_attention_d<AT, KT, 4>(h, a, ngroups, kc, vc, rows); break;
    case 8: launch_attention_d<AT, KT, 8>(h, a, ngroups, kc, vc, rows); break;
    case 16: launch_attention_d<AT, KT, 16>(h, a, ngroups, kc, vc, rows); break;
    case 32: launch_attention_d<AT, KT, 32>(h, a, ngroups, kc, vc, rows); break;
    case 64: launch_attention_d<AT, KT, 64>(h, a, ngroups, kc, vc, rows); break;
    case 128: launch_attention_d<AT, KT, 128>(h, a, ngroups, kc, vc, rows); break;
    default: fail(SPECDEC_ERR_UNSUPPORTED, "head dimension must be 4, 8, 16, 32, 64 or 128");
  }
}

// Attention over a row batch whose rows form groups of Q consecutive rows of
// one request each.  kc/vc are one layer's page pools of `layer_elems`
// elements ([page][kv head][kKvPage][D]), pg the requests' page tables.
void attention(specdec_handle *h, const Dims &dm, RowsView rows, int R, int Q, const void *kc, const void *vc,
               const float *ks, const float *vs, size_t layer_elems, int S_cap, KvPages pg) {
  if (R <= 0) return;
  AttnArgs a{};
  a.pg = pg;
  a.q = h->Q; a.ldq = dm.dq; a.rows = rows; a.R = R; a.Q = Q;
  a.S_cap = S_cap; a.H = dm.H; a.Hkv = dm.Hkv;
  a.k_scale = ks; a.v_scale = vs;
  a.out = h->ATT; a.ldo = dm.dq; a.err = h->st.err;
  const int ngroups = (R + Q - 1) / Q;
  const size_t nrows = layer_elems / dm.D;
  const bool bf = act_bf16(h);
  const bool kvbf = h->cfg.kv_dtype == SPECDEC_BF16;
  if (h->attn_tc && bf && kvbf && dm.D == kAtcD && Q >= h->attn_tc_min_q && dm.dq % 8 == 0) {
    // groups of many queries (token trees, prefill chunks): tensor cores
    AttnTcArgs t{};
    t.tmq = gemm_operand_map(h->Q, dm.dq, R, dm.dq, 128);
    t.tmk = kv_tensor_map<__nv_bfloat16, kAtcD>(kc, nrows);
    t.tmv = kv_tensor_map<__nv_bfloat16, kAtcD>(vc, nrows);
    t.rows = rows; t.R = R; t.Q = Q; t.S_cap = S_cap; t.H = dm.H; t.Hkv = dm.Hkv; t.pg = pg;
    t.out = static_cast<__nv_bfloat16 *>(h->ATT); t.ldo = dm.dq; t.err = h->st.err;
    launch_pdl(h, attn_tc_kernel, dim3(ngroups * ((Q + 127) / 128), dm.H), dim3(kAtcThreads),
               static_cast<size_t>(kAtcSmem), t);
    return;
  }
  if (h->attn_dec && h->ad_part && bf && kvbf && dm.D == kAdD && dm.H == dm.Hkv && Q <= kAdN && ngroups <= h->ad_groups &&
      dm.dq % 8 == 0) {
    // few queries per request (draft steps, verify blocks): positions on the
    // MMA's M side, persistent CTAs streaming the cache
    AttnDecArgs d{};
    d.tmq = gemm_operand_map(h->Q, dm.dq, R, dm.dq, kAdN);
    d.tmk = kv_tensor_map<__nv_bfloat16, kAdD>(kc, nrows);
    d.tmv = kv_tensor_map<__nv_bfloat16, kAdD>(vc, nrows);
    d.rows = rows; d.R = R; d.Q = Q; d.S_cap = S_cap; d.H = dm.H; d.Hkv = dm.Hkv; d.pg = pg;
    // splits while the (group, head) items would spread unevenly over the SMs
    const int base = ngroups * dm.H;
    const int tiles = (S_cap + kAdTile - 1) / kAdTile;
    int ns = 1;
    const int slots = attn_dec_ctas_per_sm() * h->num_sms;
    auto waste = [&](int n) {
      const double per = static_cast<double>(base) * n / slots;
      return std::ceil(per) / per - 1.0;
    };
    while (ns < kAdMaxSplit && 2 * ns <= tiles && waste(ns) > 0.05) ns *= 2;
    d.nsplit = ns;
    d.n_items = base * ns;
    d.out = static_cast<__nv_bfloat16 *>(h->ATT); d.ldo = dm.dq;
    d.part = h->ad_part; d.ticket = h->ad_ticket; d.err = h->st.err;
    CK(attn_dec_launch(d, std::min(d.n_items, slots), h->stream, h->use_pdl));
    ++h->launches;
    return;
  }
  if (h->cfg.kv_dtype == SPECDEC_INT8) {
    if (bf) launch_attention_t<__nv_bfloat16, int8_t>(h, a, dm.D, ngroups, kc, vc, nrows);
    else launch_attention_t<float, int8_t>(h, a, dm.D, ngroups, kc, vc, nrows);
  } else if (bf && kvbf) launch_attention_t<__nv_bfloat16, __nv_bfloat16>(h, a, dm.D, ngroups, kc, vc, nrows);
  else if (bf) launch_attention_t<__nv_bfloat16, float>(h, a, dm.D, ngroups, kc, vc, nrows);
  else if (kvbf) launch_attention_t<float, __nv_bfloat16>(h, a, dm.D, ngroups, kc, vc, nrows);
  else launch_attention_t<float, float>(h, a, dm.D, ngroups, kc, vc, nrows);
}

// NCCL, looked up at run time (dlopen of libnccl.so.2 returns the copy the
// process already has, e.g. the one torch loaded), so the library itself has
// no link-time NCCL dependency and single-GPU use never touches it.
struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  const char *(*error_string)(ncclResult_t) = nullptr;
};
const NcclApi &nccl() {
  static NcclApi api = [] {
    NcclApi a;
    void *lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!lib) return a;
    a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(lib, "ncclGetUniqueId"));
    a.comm_init_rank = reinterpret_cast<decltype(a.comm_init_rank)>(dlsym(lib, "ncclCommInitRank"));
    a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(dlsym(lib, "ncclAllReduce"));
    a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(dlsym(lib, "ncclCommDestroy"));
    a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(lib, "ncclGetErrorString"));
    return a;
  }();
  if (!api.get_unique_id || !api.comm_init_rank || !api.all_reduce || !api.comm_destroy)
    fail(SPECDEC_ERR_UNSUPPORTED, "libnccl.so.2 is not available");
  return api;
}
void nccl_check(ncclResult_t r, const char *what) {
  if (r != ncclSuccess)
    fail(SPECDEC_ERR_CUDA, std::string(what) + ": " + (nccl().error_string ? nccl().error_string(r) : "NCCL error"));
}

// Sum of the ranks' partial rows [R][d] in place (tensor parallelism: after
// the attention output projection and the FFN down projection).
void tp_all_reduce(specdec_handle *h, void *rows, int R, int d) {
  if (h->tp_world <= 1 || R <= 0) return;
  nccl_check(nccl().all_reduce(rows, rows, static_cast<size_t>(R) * d, act_bf16(h) ? ncclBfloat16 : ncclFloat, ncclSum,
                               h->comm, h->stream),
             "ncclAllReduce");
}

// Where the lm_head reads the last hidden rows, and the LayerNorm it applies
// to them first.
struct HeadInput {
  const void *x;
  const float *g, *b;
};
HeadInput head_input(specdec_handle *h, const ModelW &m) {
  if (m.dm.arch == SPECDEC_ARCH_REF)
    return m.dm.L > 0 ? HeadInput{h->H, m.layers[m.dm.L - 1].g2, m.layers[m.dm.L - 1].b2} : HeadInput{h->X, nullptr, nullptr};
  return HeadInput{h->X, m.gf, m.bfin};
}

// One forward pass of model m over the row batch at pool offset `off`
// (R rows in groups of Q rows per request).  When `logits` is set, the
// lm_head runs over the rows listed in `sel` (n_sel of them; all R rows when
// sel is null) and writes fp32 logits.  Every LayerNorm runs in the prologue
// of the linear kernel that consumes its output.
//
// Reference arch, per layer (src/nn/layer.cpp:1097-1114, post-LN); the
// embedding writes X:
//   QKV    LN2_prev(H) (layer 0: X) -> Q, K/V cache (RoPE, append); stores
//          the normalised rows in X
//   ATT    attention -> ATT
//   OPROJ  ATT.Wo + bo + X -> H
//   GATEUP silu(LN1(H).Wg + bg) * (LN1(H).Wu + bu) -> A; stores LN1(H) in X1
//   DOWN   A.Wd + bd + X1 -> H
//   head   LN2_last(H) -> logits
// cfg arch (pre-LN): QKV reads LN1(X); OPROJ H = X + attn; FC1 GELU over
// LN2(H) -> A; FC2 X = H + ffn; the head reads LN_final(X).
void forward_rows(specdec_handle *h, bool target, int off, int R, int Q, const int *sel, int n_sel, float *logits,
                  bool tree = false) {
  ModelW &m = target ? h->tgt : h->dft;
  const Dims &dm = m.dm;
  const int d = dm.d;
  RowsView rows{h->pool.tok + off, h->pool.pos + off, h->pool.req + off};
  if (tree) {
    rows.slot = h->pool.slot + off;
    rows.tb = h->pool.tb + off;
    rows.mask = h->pool.mask + off;
  }
  void *kc = target ? h->tk : h->dk;
  void *vc = target ? h->tv : h->dv;
  const size_t lstride = target ? h->t_layer_stride : h->d_layer_stride;
  const KvPages pg{h->d_pt, h->ppr};
  const int S_cap = target ? h->t_cap : h->d_cap;
  const bool kv8 = h->cfg.kv_dtype == SPECDEC_INT8;
  const size_t kv_elt = kv8 ? 1 : h->cfg.kv_dtype == SPECDEC_BF16 ? 2 : 4;
  float *ksc = target ? h->tks : h->dks, *vsc = target ? h->tvs : h->dvs;
  const size_t lrows = lstride / dm.D;  // cache rows (and int8 scales) per layer
  const bool ref = dm.arch == SPECDEC_ARCH_REF;

  if (act_bf16(h))
    launch_pdl(h, embed_kernel<__nv_bfloat16>, dim3(R), dim3(128), 0, rows, R, m.emb, m.pos, d, dm.max_seq,
               static_cast<__nv_bfloat16 *>(h->X));
  else
    launch_pdl(h, embed_kernel<float>, dim3(R), dim3(128), 0, rows, R, m.emb, m.pos, d, dm.max_seq,
               static_cast<float *>(h->X));

  for (int l = 0; l < dm.L; ++l) {
    const LayerW &L = m.layers[l];
    void *kcl = static_cast<char *>(kc) + l * lstride * kv_elt;
    void *vcl = static_cast<char *>(vc) + l * lstride * kv_elt;
    LinearArgs a{};
    a.ldx = d; a.R = R; a.W = L.wqkv; a.scale = L.sqkv; a.bias = L.bqkv;
    a.N = dm.dq + 2 * dm.kvd; a.K = d; a.out = h->Q; a.ldo = dm.dq; a.rows = rows;
    if (ref) {
      a.x = l == 0 ? h->X : h->H;
      if (l > 0) { a.in_g = m.layers[l - 1].g2; a.in_b = m.layers[l - 1].b2; a.norm_out = h->X; }
    } else {
      a.x = h->X; a.in_g = L.g1; a.in_b = L.b1;
    }
    a.qkv = QKVArgs{dm.dq, dm.kvd, dm.D, h->rope, h->rope_max, kcl, vcl, pg, S_cap,
                    kv8 ? 2 : h->cfg.kv_dtype == SPECDEC_BF16 ? 1 : 0, h->KVN, h->st.err};
    launch_linear<kEpiQKV>(h, a);
    float *ksl = kv8 ? ksc + l * lrows : nullptr, *vsl = kv8 ? vsc + l * lrows : nullptr;
    if (kv8)
      launch(h, kv_quant_kernel, dim3(R), dim3(256), 0, rows, R, static_cast<const float *>(h->KVN), dm.kvd, dm.D,
             dm.Hkv, S_cap, pg, static_cast<int8_t *>(kcl), static_cast<int8_t *>(vcl), ksl, vsl);
    attention(h, dm, rows, R, Q, kcl, vcl, ksl, vsl, lstride, S_cap, pg);
    // With tensor parallelism each rank multiplies its heads' slice; one rank
    // adds bias and residual, and the all-reduce sums the partial rows.
    const bool lead = h->tp_rank == 0;
    LinearArgs o{};
    o.x = h->ATT; o.ldx = dm.dq; o.R = R; o.W = L.wo; o.scale = L.so; o.bias = L.bo; o.N = d; o.K = dm.dq;
    o.out = h->H; o.ldo = d; o.resid = h->X; o.ldr = d; o.rows = rows;
    if (lead) launch_linear<kEpiResid>(h, o);
    else launch_linear<kEpiStore>(h, o);
    tp_all_reduce(h, h->H, R, d);
    LinearArgs g{};
    g.x = h->H; g.ldx = d; g.R = R; g.W = L.wgu; g.scale = L.sgu; g.bias = L.bgu; g.K = d; g.rows = rows;
    g.out = h->A; g.ldo = dm.F; g.N = ref ? 2 * dm.F : dm.F;
    g.in_g = ref ? L.g1 : L.g2; g.in_b = ref ? L.b1 : L.b2;
    if (ref) {
      g.norm_out = h->X1;
      launch_linear<kEpiSwiGLU>(h, g);
    } else {
      launch_linear<kEpiGelu>(h, g);
    }
    LinearArgs dn{};
    dn.x = h->A; dn.ldx = dm.F; dn.R = R; dn.W = L.wd; dn.scale = L.sd; dn.bias = L.bd; dn.N = d; dn.K = dm.F;
    dn.rows = rows; dn.ldo = d; dn.ldr = d;
    if (ref) { dn.out = h->H; dn.resid = h->X1; }
    else { dn.out = h->X; dn.resid = h->H; }
    if (lead) launch_linear<kEpiResid>(h, dn);
    else launch_linear<kEpiStore>(h, dn);
    tp_all_reduce(h, dn.out, R, d);
  }
  if (!logits) return;
  const HeadInput hi = head_input(h, m);
  LinearArgs hd{};
  hd.x = hi.x; hd.in_g = hi.g; hd.in_b = hi.b; hd.ldx = d; hd.in_rows = sel; hd.R = sel ? n_sel : R;
  hd.W = m.whead; hd.scale = m.shead; hd.bias = m.bhead;
  hd.N = dm.V; hd.K = d; hd.out = logits; hd.ldo = dm.V; hd.out_f32 = 1; hd.rows = rows;
  launch_linear<kEpiStore>(h, hd);
}

}  // namespace

namespace {

void sync_check(specdec_handle *h) { CK(cudaStreamSynchronize(h->stream)); }

// Gives request slots 0 .. B-1 the pages for positions [0, need) (at most
// max_seq_len).  Every generation, session and forward starts with empty
// caches, so the whole pool is free again: slot b's i-th page is the
// (i * B + b)-th page of the pool, so a request's pages are not adjacent.
// Slots past B and pages past need stay -1; a kernel that meets one flags
// SPECDEC_ERR_SEQ_LEN.  The table goes up on the library's stream, ahead of
// the launches that read it.
void assign_pages(specdec_handle *h, int B, int need) {
  const int per = std::min(h->ppr, (std::max(1, need) + kKvPage - 1) / kKvPage);
  if (static_cast<int64_t>(B) * per > h->kv_pages)
    fail(SPECDEC_ERR_OOM, "the KV page pool holds " + std::to_string(h->kv_pages) + " pages of " +
                              std::to_string(kKvPage) + " positions; " + std::to_string(B) + " requests of " +
                              std::to_string(need) + " positions need " + std::to_string(B * per));
  h->h_pt.assign(static_cast<size_t>(h->cfg.max_batch) * h->ppr, -1);
  for (int i = 0; i < per; ++i)
    for (int b = 0; b < B; ++b) h->h_pt[static_cast<size_t>(b) * h->ppr + i] = i * B + b;
  CK(cudaMemcpyAsync(h->d_pt, h->h_pt.data(), h->h_pt.size() * sizeof(int), cudaMemcpyHostToDevice, h->stream));
}

// Cache positions a generation can write: the prompt, the new tokens, and a
// verify block (k + 1 rows, or a tree's nodes) past them.  With the
// reference's catch-up (SPECDEC_CATCHUP_REF) the draft is fed one extra
// position per rejected round (src/nn/layer.cpp:1632-1642, then 1542), so
// its cache can run up to max_new positions ahead of the target's; the page
// table is shared, so the reservation covers that drift.
int positions_needed(const specdec_gen_params *p, int S, const TreeCfg *tree, bool ar) {
  const int n = std::max(0, p->max_new_tokens);
  if (ar) return S + n + 1;
  if (tree) return S + n + tree->N + 1;
  const int drift = p->draft_catchup == SPECDEC_CATCHUP_REF ? n : 0;
  return S + n + drift + std::max(1, p->lookahead) + 1;
}

void validate_gen(specdec_handle *h, const specdec_gen_params *p, int B, int S, const TreeCfg *tree, bool ar) {
  if (!p) fail(SPECDEC_ERR_INVALID, "null params");
  if (ar ? !h->tgt.loaded : (!h->tgt.loaded || !h->dft.loaded))
    fail(SPECDEC_ERR_STATE, ar ? "target weights must be loaded first" : "target and draft weights must be loaded first");
  if (B < 1 || B > h->cfg.max_batch) fail(SPECDEC_ERR_INVALID, "batch out of range");
  if (S < 1 || S > h->cfg.max_prompt_len) fail(SPECDEC_ERR_INVALID, "prompt length out of range");
  if (!tree && !ar && (p->lookahead < 1 || p->lookahead > h->cfg.max_lookahead))
    fail(SPECDEC_ERR_INVALID, "lookahead out of range");
  if (p->max_new_tokens < 0) fail(SPECDEC_ERR_INVALID, "max_new_tokens < 0");
  // The target cache ends at S + max_new positions (every round verifies
  // M = min(k, remaining) drafts); the reference throws when that exceeds
  // max_seq_len (src/nn/layer.cpp:1176-1179).  Autoregressive decoding never
  // feeds its last token: S + max_new - 1 positions.
  const int cache_end = S + (ar ? std::max(0, p->max_new_tokens - 1) : (p->max_new_tokens > 1 ? p->max_new_tokens : 0));
  if (cache_end > h->t_cap)
    fail(SPECDEC_ERR_SEQ_LEN, "Sequence length S plus past cached length exceeds max_seq_len");
  if (!(p->top_p == p->top_p)) fail(SPECDEC_ERR_INVALID, "top_p is NaN");
  if (p->rng_mode == SPECDEC_RNG_HOST_UNIFORM && p->temperature > 0.f) {
    if (!p->uniforms || p->uniform_rounds < 1) fail(SPECDEC_ERR_INVALID, "host-uniform mode needs a uniform table");
  } else if (p->rng_mode != SPECDEC_RNG_MT19937 && p->rng_mode != SPECDEC_RNG_HOST_UNIFORM) {
    fail(SPECDEC_ERR_INVALID, "unknown rng_mode");
  }
  if (!tree && !ar && p->draft_catchup != SPECDEC_CATCHUP_REF && p->draft_catchup != SPECDEC_CATCHUP_CORRECT)
    fail(SPECDEC_ERR_INVALID, "unknown draft_catchup");
}

TreeCfg make_tree(const specdec_handle *h, const specdec_tree *t) {
  if (!t) fail(SPECDEC_ERR_INVALID, "null tree");
  if (h->max_tree == 0) fail(SPECDEC_ERR_STATE, "the handle was created with max_tree_nodes = 0");
  if (t->depth < 1 || t->depth > kTreeMaxDepth) fail(SPECDEC_ERR_INVALID, "tree depth must be 1..8");
  TreeCfg c;
  c.depth = t->depth;
  int level = 1;
  for (int l = 0; l < t->depth; ++l) {
    if (t->branch[l] < 1 || t->branch[l] > h->tgt.dm.V) fail(SPECDEC_ERR_INVALID, "tree branching out of range");
    c.branch[l] = t->branch[l];
    c.bmax = std::max(c.bmax, t->branch[l]);
    level *= t->branch[l];
    if (level > kTreeMaxNodes) fail(SPECDEC_ERR_INVALID, "tree too large");
    c.lev[l + 1] = c.lev[l] + level;
    if (c.lev[l + 1] > h->max_tree) fail(SPECDEC_ERR_INVALID, "tree has more nodes than max_tree_nodes");
  }
  c.N = c.lev[t->depth];
  return c;
}

int samp_threads(const specdec_handle *h) { return h->tgt.dm.V <= 4096 ? 512 : kSampThreads; }
size_t samp_smem(const specdec_handle *h) { return static_cast<size_t>(h->tgt.dm.V) * sizeof(float); }
// Draft sampling after draft step j (one block per request).
// Vocabularies of at least kSampClusterMinV entries without top-k / top-p
// are sampled by clusters of CTAs per request while the grid stays within
// two CTAs per SM.
constexpr int kSampClusterMinV = 8192;
int draft_sample_cluster(const specdec_handle *h, const SpecState &st) {
  if (h->samp_max_cluster < 2 || st.V < kSampClusterMinV || st.tree) return 1;
  if (!st.greedy && ((st.top_k > 0 && st.top_k < st.V) || (st.top_p > 0.f && st.top_p < 1.f))) return 1;
  int cs = h->samp_max_cluster;
  while (cs > 1 && st.B * cs > 2 * h->num_sms) cs /= 2;
  return cs;
}
size_t samp_cluster_smem(int V, int cs) { return static_cast<size_t>(((V + cs - 1) / cs + 3) & ~3) * sizeof(float); }

void launch_draft_sample(specdec_handle *h, const SpecState &st, int j) {
  const int cs = draft_sample_cluster(h, st);
  const float *lg = h->logits;
  if (cs > 1) {
    auto kern = cs >= 8 ? draft_sample_cluster_kernel<8> : cs == 4 ? draft_sample_cluster_kernel<4>
                                                                    : draft_sample_cluster_kernel<2>;
    launch_cluster(h, kern, dim3(st.B * cs), dim3(kSampThreads), samp_cluster_smem(st.V, cs), dim3(cs, 1, 1), st,
                   j, lg);
    return;
  }
  launch_pdl(h, draft_sample_kernel, dim3(st.B), dim3(samp_threads(h)), samp_smem(h), st, j, lg);
}

// Verify rows accept_kernel stages in shared memory at a time (at least one).
constexpr size_t kAcceptStageBytes = 200 * 1024;
int accept_stage_rows(const specdec_handle *h) {
  const size_t row = samp_smem(h);
  return static_cast<int>(std::max<size_t>(1, std::min<size_t>(h->cfg.max_lookahead + 1, kAcceptStageBytes / row)));
}
size_t accept_smem(const specdec_handle *h) { return static_cast<size_t>(accept_stage_rows(h)) * samp_smem(h); }

// Enqueues one full round (everything between two accept kernels).
CacheView cache_view(specdec_handle *h, bool target) {
  const ModelW &m = target ? h->tgt : h->dft;
  CacheView c{};
  c.k = target ? h->tk : h->dk;
  c.v = target ? h->tv : h->dv;
  c.ks = target ? h->tks : h->dks;
  c.vs = target ? h->tvs : h->dvs;
  c.layer_elems = target ? h->t_layer_stride : h->d_layer_stride;
  c.pg = KvPages{h->d_pt, h->ppr};
  c.S_cap = target ? h->t_cap : h->d_cap;
  c.Hkv = m.dm.Hkv;
  c.D = m.dm.D;
  c.L = m.dm.L;
  c.elt = h->cfg.kv_dtype == SPECDEC_INT8 ? 1 : h->cfg.kv_dtype == SPECDEC_BF16 ? 2 : 4;
  return c;
}

// One round of tree speculation (tree.cuh): draft levels 0 .. L-1, verify,
// accept, compaction.
void enqueue_tree_round(specdec_handle *h) {
  SpecState &st = h->st;
  const int B = st.B;
  const dim3 sb(samp_threads(h));
  const float *lg = h->logits;
  forward_rows(h, false, st.rows.off_step0, 2 * B, 2, h->sel_odd, B, h->logits);
  launch(h, tree_topk_kernel, dim3(B, 1), sb, samp_smem(h), st, 0, lg);
  for (int t = 1; t < st.tL; ++t) {
    const int n = st.tlev[t] - st.tlev[t - 1];
    forward_rows(h, false, st.rows.off_tlevel[t], B * n, n, nullptr, B * n, h->logits, true);
    launch(h, tree_topk_kernel, dim3(B, n), sb, samp_smem(h), st, t, lg);
  }
  const int W = st.tN + 1;
  forward_rows(h, true, st.rows.off_tverify, B * W, W, nullptr, B * W, h->logits, true);
  launch(h, tree_accept_kernel, dim3(B), sb, samp_smem(h), st, lg);
  launch(h, tree_compact_kernel, dim3(B, h->tgt.dm.L + h->dft.dm.L), dim3(256), 0, st, cache_view(h, true),
         cache_view(h, false));
}

void enqueue_round(specdec_handle *h) {
  SpecState &st = h->st;
  if (st.tree) {
    enqueue_tree_round(h);
    return;
  }
  if (st.ar) {  // one target row per request: the last token at the next position
    forward_rows(h, true, st.rows.off_verify, st.B, 1, nullptr, st.B, h->logits);
    launch_pdl(h, ar_token_kernel, dim3(st.B), dim3(samp_threads(h)), samp_smem(h), st,
               static_cast<const float *>(h->logits));
    return;
  }
  const int B = st.B, k = st.k;
  forward_rows(h, false, st.rows.off_step0, 2 * B, 2, h->sel_odd, B, h->logits);
  launch_draft_sample(h, st, 0);
  for (int j = 1; j < k; ++j) {
    forward_rows(h, false, st.rows.off_step1 + (j - 1) * B, B, 1, nullptr, B, h->logits);
    launch_draft_sample(h, st, j);
  }
  forward_rows(h, true, st.rows.off_verify, B * (k + 1), k + 1, nullptr, B * (k + 1), h->logits);
  launch_pdl(h, accept_kernel, dim3(B), dim3(kSampThreads), accept_smem(h), st, static_cast<const float *>(h->logits),
             accept_stage_rows(h));
}

void setup_state(specdec_handle *h, const specdec_gen_params *p, int B, int S, const TreeCfg *tree, bool ar) {
  SpecState &st = h->st;
  st.B = B;
  st.k = ar ? 0 : p->lookahead;
  st.ar = ar ? 1 : 0;
  st.kmax = h->cfg.max_lookahead;
  st.V = h->tgt.dm.V;
  st.max_new = p->max_new_tokens;
  st.prompt_len = S;
  st.out_len = S + std::max(1, p->max_new_tokens);
  st.T = p->temperature;
  st.greedy = p->temperature <= 0.f ? 1 : 0;
  st.top_k = p->top_k;
  st.top_p = p->top_p;
  st.rng_mode = p->rng_mode;
  st.catchup = p->draft_catchup;
  st.t_cap = h->t_cap;
  st.d_cap = h->d_cap;
  st.u_slots = ar ? 1 : 2 * p->lookahead + 1;
  st.u_rounds = p->uniform_rounds;
  st.uniforms = h->d_uniforms;
  // row regions: [prefill R_max][step0 2B][steps 1..k-1: B each][verify B(k+1)]
  st.rows = h->pool;
  st.rows.off_step0 = h->R_max;
  st.rows.off_step1 = h->R_max + 2 * B;
  st.rows.off_verify = h->R_max + 2 * B + (st.kmax - 1) * B;
  st.tree = tree ? 1 : 0;
  if (tree) {
    st.k = 1;  // the chain rows are cleared with one draft step; a tree round does not use k
    st.catchup = SPECDEC_CATCHUP_CORRECT;
    st.tL = tree->depth;
    st.tN = tree->N;
    st.tbmax = tree->bmax;
    for (int l = 0; l < kTreeMaxDepth; ++l) st.tbr[l] = tree->branch[l];
    for (int l = 0; l <= kTreeMaxDepth; ++l) st.tlev[l] = tree->lev[l];
    st.u_slots = tree->depth * tree->bmax + 1;
    // tree regions: levels 1 .. L-1 (B * nodes at that depth each), then the
    // verify block (B * (N + 1))
    for (int t = 1; t < tree->depth; ++t) st.rows.off_tlevel[t] = h->tree_base + B * tree->lev[t - 1];
    st.rows.off_tverify = h->tree_base + B * h->max_tree;
  }
}

// Everything up to and including the first token (src/nn/layer.cpp:1396-1512).
void enqueue_prologue(specdec_handle *h, int B, int S, uint32_t seed) {
  SpecState &st = h->st;
  launch(h, init_state_kernel, dim3(B), dim3(128), 0, st, static_cast<const int *>(h->d_prompts), S);
  if (!st.greedy && st.rng_mode == 0) launch(h, mt_seed_kernel, dim3((B + 127) / 128), dim3(128), 0, st.mt, st.mt_idx, seed, B);
  const int chunk = std::max(1, std::min(S, h->R_max / B));
  for (int pass = 0; pass < (st.ar ? 1 : 2); ++pass) {
    const bool target = pass == 0;
    for (int c0 = 0; c0 < S; c0 += chunk) {
      const int clen = std::min(chunk, S - c0);
      const int R = B * clen;
      const bool last = c0 + clen >= S;
      launch(h, plan_prefill_kernel, dim3((R + 255) / 256), dim3(256), 0, static_cast<const int *>(h->d_prompts), B, S,
             c0, clen, h->tgt.dm.V, h->pool.tok, h->pool.pos, h->pool.req, (target && last) ? h->sel_prefill : nullptr);
      // the draft's prefill logits are discarded (src/nn/layer.cpp:1408)
      forward_rows(h, target, 0, R, clen, h->sel_prefill, B, (target && last) ? h->logits : nullptr);
    }
  }
  if (st.ar)
    launch_pdl(h, ar_token_kernel, dim3(B), dim3(samp_threads(h)), samp_smem(h), st, static_cast<const float *>(h->logits));
  else
    launch_pdl(h, first_token_kernel, dim3(B), dim3(samp_threads(h)), samp_smem(h), st,
               static_cast<const float *>(h->logits));
}

void destroy_graphs(specdec_handle *h) {
  for (auto &kv : h->graphs) {
    if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    if (kv.second.graph) cudaGraphDestroy(kv.second.graph);
  }
  h->graphs.clear();
}

// Builds pre -> WHILE(cond) { body } as one executable graph: pre() and
// body() enqueue on the handle's stream (captured); pre ends with the kernel
// that primes the condition, body with the one that re-evaluates it.
template <class Pre, class Body>
GraphEntry build_loop_graph(specdec_handle *h, Pre pre, Body body) {
  GraphEntry ge;
  CK(cudaGraphCreate(&ge.graph, 0));
  cudaGraphConditionalHandle hnd;
  CK(cudaGraphConditionalHandleCreate(&hnd, ge.graph, 0, cudaGraphCondAssignDefault));
  CK(cudaStreamBeginCaptureToGraph(h->stream, ge.graph, nullptr, nullptr, 0, cudaStreamCaptureModeThreadLocal));
  h->launches = 0;
  try {
    pre(hnd);
  } catch (...) {
    cudaGraph_t g;
    cudaStreamEndCapture(h->stream, &g);
    throw;
  }
  ge.fixed_kernels = h->launches;
  CK(cudaStreamEndCapture(h->stream, &ge.graph));
  size_t nn = 0;
  CK(cudaGraphGetNodes(ge.graph, nullptr, &nn));
  std::vector<cudaGraphNode_t> nodes(nn);
  CK(cudaGraphGetNodes(ge.graph, nodes.data(), &nn));
  std::vector<cudaGraphNode_t> sinks;
  for (auto n : nodes) {
    size_t nd = 0;
    CK(cudaGraphNodeGetDependentNodes(n, nullptr, &nd));
    if (nd == 0) sinks.push_back(n);
  }
  cudaGraphNodeParams cp{};
  cp.type = cudaGraphNodeTypeConditional;
  cp.conditional.handle = hnd;
  cp.conditional.type = cudaGraphCondTypeWhile;
  cp.conditional.size = 1;
  cudaGraphNode_t wnode;
  CK(cudaGraphAddNode(&wnode, ge.graph, sinks.data(), sinks.size(), &cp));
  cudaGraph_t bg = cp.conditional.phGraph_out[0];
  CK(cudaStreamBeginCaptureToGraph(h->stream, bg, nullptr, nullptr, 0, cudaStreamCaptureModeThreadLocal));
  h->launches = 0;
  try {
    body(hnd);
  } catch (...) {
    cudaGraph_t g;
    cudaStreamEndCapture(h->stream, &g);
    throw;
  }
  ge.body_kernels = h->launches;
  CK(cudaStreamEndCapture(h->stream, &bg));
  CK(cudaGraphInstantiate(&ge.exec, ge.graph, 0));
  return ge;
}

// Builds prologue -> WHILE(active) { round } as one executable graph.
GraphEntry build_graph(specdec_handle *h, int B, int S, uint32_t seed, int max_iters) {
  return build_loop_graph(
      h,
      [&](cudaGraphConditionalHandle hnd) {
        enqueue_prologue(h, B, S, seed);
        launch(h, prime_cond_kernel, dim3(1), dim3(32), 0, hnd, static_cast<const int *>(h->st.active), B);
      },
      [&](cudaGraphConditionalHandle hnd) {
        enqueue_round(h);
        launch(h, round_cond_kernel, dim3(1), dim3(1), 0, hnd, h->st.active_count, h->d_iters, max_iters, h->st.err);
      });
}

// The step API's rounds: WHILE(active and fewer than *d_step_target rounds) { round }.
GraphEntry build_step_graph(specdec_handle *h) {
  const int B = h->st.B;
  return build_loop_graph(
      h,
      [&](cudaGraphConditionalHandle hnd) {
        launch(h, step_prime_kernel, dim3(1), dim3(32), 0, hnd, static_cast<const int *>(h->st.active), B,
               static_cast<const int *>(h->d_step_target));
      },
      [&](cudaGraphConditionalHandle hnd) {
        enqueue_round(h);
        launch(h, step_cond_kernel, dim3(1), dim3(1), 0, hnd, h->st.active_count, h->d_iters,
               static_cast<const int *>(h->d_step_target));
      });
}

// d_prompts may be any device buffer; it is staged into the handle's prompt
// buffer so captured graphs stay valid across calls.
int generate_impl(specdec_handle *h, const specdec_gen_params *p, const int32_t *d_prompts, int B, int S, int32_t *d_out,
                  int64_t *d_stats_out, const TreeCfg *tree = nullptr, bool ar = false) {
  validate_gen(h, p, B, S, tree, ar);
  SpecState &st = h->st;
  h->step_open = false;  // a generation reuses the speculative state of a step session
  assign_pages(h, B, positions_needed(p, S, tree, ar));
  if (ar && p->max_new_tokens == 0) {  // generate_advanced returns the prompt
    CK(cudaMemcpyAsync(d_out, d_prompts, static_cast<size_t>(B) * S * sizeof(int), cudaMemcpyDeviceToDevice, h->stream));
    if (d_stats_out) CK(cudaMemsetAsync(d_stats_out, 0, static_cast<size_t>(B) * 4 * sizeof(int64_t), h->stream));
    CK(cudaMemsetAsync(st.err, 0, sizeof(int), h->stream));
    h->launches = 0;
    return SPECDEC_OK;
  }
  setup_state(h, p, B, S, tree, ar);
  if (d_prompts != h->d_prompts)
    CK(cudaMemcpyAsync(h->d_prompts, d_prompts, static_cast<size_t>(B) * S * sizeof(int), cudaMemcpyDeviceToDevice,
                       h->stream));
  const bool table = p->rng_mode == SPECDEC_RNG_HOST_UNIFORM && p->temperature > 0.f;
  if (table) {
    const size_t n = static_cast<size_t>(B) * p->uniform_rounds * st.u_slots;
    if (n > h->uniforms_cap) {
      destroy_graphs(h);
      if (h->d_uniforms) cudaFree(h->d_uniforms);
      h->d_uniforms = nullptr;
      h->uniforms_cap = 0;
      CK(cudaMalloc(&h->d_uniforms, n * sizeof(float)));
      h->uniforms_cap = n;
    }
    st.uniforms = h->d_uniforms;
    CK(cudaMemcpyAsync(h->d_uniforms, p->uniforms, n * sizeof(float), cudaMemcpyDefault, h->stream));
  }
  CK(cudaMemsetAsync(st.err, 0, sizeof(int), h->stream));
  CK(cudaMemsetAsync(h->d_iters, 0, sizeof(int), h->stream));
  CK(cudaMemsetAsync(st.active_count, 0, sizeof(int), h->stream));
  const int max_iters = std::max(2, p->max_new_tokens + 2);

  if (h->use_graph) {
    // autoregressive graphs have k = 0 (speculative ones k >= 1)
    GraphKey key{B, S, st.k, st.greedy, table ? 1 : 0, ar ? 0 : p->draft_catchup, p->max_new_tokens,
                 table ? p->uniform_rounds : 0, p->temperature, (!st.greedy && !table) ? p->seed : 0u,
                 st.greedy ? 0 : p->top_k, st.greedy ? 1.f : p->top_p, tree ? tree->sig() : 0ull};
    auto it = h->graphs.find(key);
    if (it == h->graphs.end()) it = h->graphs.emplace(key, build_graph(h, B, S, p->seed, max_iters)).first;
    CK(cudaGraphLaunch(it->second.exec, h->stream));
    h->graph_fixed = it->second.fixed_kernels;
    h->graph_body = it->second.body_kernels;
  } else {
    h->launches = 0;
    enqueue_prologue(h, B, S, p->seed);
    std::vector<int> act(B);
    for (int it = 0; it < max_iters; ++it) {
      CK(cudaMemcpyAsync(act.data(), st.active, B * sizeof(int), cudaMemcpyDeviceToHost, h->stream));
      sync_check(h);
      int n_act = 0;
      for (int v : act) n_act += v;
      if (n_act == 0) break;
      enqueue_round(h);
      launch(h, count_iter_kernel, dim3(1), dim3(1), 0, h->d_iters, st.active_count);
    }
  }
  const int64_t direct = h->launches;
  launch(h, finalize_kernel, dim3(B), dim3(128), 0, st, static_cast<int *>(d_out),
         reinterpret_cast<long long *>(d_stats_out));
  h->extra_launches = 1;
  h->launches = h->use_graph ? -1 : direct + 1;
  return SPECDEC_OK;
}

// Grows the device uniform table to `n` floats (the graphs that hold the old
// table are dropped).
void ensure_uniform_table(specdec_handle *h, size_t n) {
  if (n <= h->uniforms_cap) return;
  destroy_graphs(h);
  if (h->d_uniforms) cudaFree(h->d_uniforms);
  h->d_uniforms = nullptr;
  h->uniforms_cap = 0;
  CK(cudaMalloc(&h->d_uniforms, n * sizeof(float)));
  h->uniforms_cap = n;
}

// specdec_prefill: everything of generate_speculative up to and including the
// first token (src/nn/layer.cpp:1396-1512), then the session stays open for
// specdec_step.  A host uniform table gets room for max_new_tokens + 2 rounds
// at least, so steps can supply the rounds they run.
void prefill_impl(specdec_handle *h, const specdec_gen_params *p, const int32_t *d_prompts, int B, int S) {
  validate_gen(h, p, B, S, nullptr, false);
  h->step_open = false;
  assign_pages(h, B, positions_needed(p, S, nullptr, false));
  SpecState &st = h->st;
  setup_state(h, p, B, S, nullptr, false);
  if (d_prompts != h->d_prompts)
    CK(cudaMemcpyAsync(h->d_prompts, d_prompts, static_cast<size_t>(B) * S * sizeof(int), cudaMemcpyDeviceToDevice,
                       h->stream));
  const bool table = p->rng_mode == SPECDEC_RNG_HOST_UNIFORM && p->temperature > 0.f;
  int cap = 0;
  if (table) {
    cap = std::max(p->uniform_rounds, p->max_new_tokens + 2);
    const size_t row = static_cast<size_t>(st.u_slots) * sizeof(float);
    ensure_uniform_table(h, static_cast<size_t>(B) * cap * st.u_slots);
    st.uniforms = h->d_uniforms;
    st.u_rounds = cap;
    CK(cudaMemsetAsync(h->d_uniforms, 0, static_cast<size_t>(B) * cap * row, h->stream));
    CK(cudaMemcpy2DAsync(h->d_uniforms, cap * row, p->uniforms, static_cast<size_t>(p->uniform_rounds) * row,
                         static_cast<size_t>(p->uniform_rounds) * row, B, cudaMemcpyDefault, h->stream));
  }
  CK(cudaMemsetAsync(st.err, 0, sizeof(int), h->stream));
  CK(cudaMemsetAsync(h->d_iters, 0, sizeof(int), h->stream));
  CK(cudaMemsetAsync(st.active_count, 0, sizeof(int), h->stream));
  h->launches = 0;
  enqueue_prologue(h, B, S, p->seed);
  GraphKey key{B, S, st.k, st.greedy, table ? 1 : 0, p->draft_catchup, p->max_new_tokens, table ? cap : 0,
               p->temperature, 0u, st.greedy ? 0 : p->top_k, st.greedy ? 1.f : p->top_p, 0ull};
  key.mode = 1;
  h->step_key = key;
  h->step_open = true;
  h->step_round = 1;  // round 0 drew the first token
}

// specdec_step: `rounds` rounds of the reference's round loop
// (src/nn/layer.cpp:1514-1656) on the open session, stopping early once no
// request is active.  h_uniforms (optional, host or device) are the rounds'
// draws [B][rounds][2k+1]; they replace the table rows of those rounds.  The
// tokens each request emitted go to d_out [B][cap] and their number to
// d_counts [B] (device buffers).
void step_impl(specdec_handle *h, int rounds, const float *h_uniforms, int32_t *d_out, int32_t *d_counts, int cap) {
  if (!h->step_open) fail(SPECDEC_ERR_STATE, "no open session: call specdec_prefill first");
  if (rounds < 1) fail(SPECDEC_ERR_INVALID, "rounds must be at least 1");
  if (!d_out || !d_counts || cap < 1) fail(SPECDEC_ERR_INVALID, "null output buffer");
  SpecState &st = h->st;
  const int B = st.B;
  const bool table = h->step_key.rng_mode == 1;
  if (h_uniforms) {
    if (!table) fail(SPECDEC_ERR_INVALID, "the session was not opened in host-uniform mode");
    if (h->step_round + rounds > st.u_rounds) fail(SPECDEC_ERR_RNG, "the host uniform table has too few rounds");
    const size_t row = static_cast<size_t>(st.u_slots) * sizeof(float);
    CK(cudaMemcpy2DAsync(h->d_uniforms + static_cast<size_t>(h->step_round) * st.u_slots, st.u_rounds * row,
                         h_uniforms, rounds * row, rounds * row, B, cudaMemcpyDefault, h->stream));
  }
  if (h->use_graph) {
    launch(h, step_begin_kernel, dim3((B + 127) / 128), dim3(128), 0, static_cast<const int *>(st.n_new),
           h->d_step_base, B);
    auto it = h->graphs.find(h->step_key);
    if (it == h->graphs.end()) it = h->graphs.emplace(h->step_key, build_step_graph(h)).first;
    CK(cudaMemsetAsync(h->d_iters, 0, sizeof(int), h->stream));
    CK(cudaMemsetAsync(st.active_count, 0, sizeof(int), h->stream));
    launch(h, set_int_kernel, dim3(1), dim3(1), 0, h->d_step_target, rounds);
    CK(cudaGraphLaunch(it->second.exec, h->stream));
    h->graph_fixed = it->second.fixed_kernels + 3;  // + step_begin, set_int, step_collect
    h->graph_body = it->second.body_kernels;
    h->extra_launches = 0;
  } else {
    h->launches = 0;
    launch(h, step_begin_kernel, dim3((B + 127) / 128), dim3(128), 0, static_cast<const int *>(st.n_new),
           h->d_step_base, B);
    for (int r = 0; r < rounds; ++r) {
      enqueue_round(h);
      launch(h, count_iter_kernel, dim3(1), dim3(1), 0, h->d_iters, st.active_count);
    }
  }
  launch(h, step_collect_kernel, dim3(B), dim3(128), 0, static_cast<const int *>(st.tokens_out), st.out_len,
         st.prompt_len, static_cast<const int *>(st.n_new), static_cast<const int *>(h->d_step_base), B, cap, d_out,
         d_counts);
  if (h->use_graph) h->launches = -1;
  h->step_round += rounds;
}

// Reads the device error word (after a synchronisation) into a status.
void check_device_err(specdec_handle *h) {
  CK(cudaMemcpyAsync(h->h_pinned, h->st.err, sizeof(int), cudaMemcpyDeviceToHost, h->stream));
  sync_check(h);
  const int err = h->h_pinned[0];
  if (err & kErrSeqLen) fail(SPECDEC_ERR_SEQ_LEN, "Sequence length S plus past cached length exceeds max_seq_len");
  if (err & kErrRngTable) fail(SPECDEC_ERR_RNG, "the host uniform table has too few rounds");
  if (err & kErrTimeout) fail(SPECDEC_ERR_CUDA, "an asynchronous copy did not complete within its wait limit");
}

}  // namespace

// ---------------------------------------------------------------------------
extern "C" {

const char *specdec_last_error(const specdec_handle *h) { return h ? h->err.c_str() : g_create_err.c_str(); }

namespace {
int create_impl(const specdec_config *cfg, int device, int rank, int world, const void *uid, specdec_handle **out);
}

int specdec_create(const specdec_config *cfg, int device, specdec_handle **out) {
  return create_impl(cfg, device, 0, 1, nullptr, out);
}

int specdec_tp_unique_id(void *out128) {
  if (!out128) return SPECDEC_ERR_INVALID;
  try {
    ncclUniqueId id;
    nccl_check(nccl().get_unique_id(&id), "ncclGetUniqueId");
    static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id is 128 bytes");
    std::memcpy(out128, &id, sizeof(id));
  } catch (const SpecErr &e) {
    g_create_err = e.msg;
    return e.code;
  }
  return SPECDEC_OK;
}

int specdec_create_tp(const specdec_config *cfg, int device, int rank, int world, const void *unique_id,
                      specdec_handle **out) {
  if (world < 1 || rank < 0 || rank >= world || (world > 1 && !unique_id)) {
    g_create_err = "bad tensor-parallel rank / size / id";
    return SPECDEC_ERR_INVALID;
  }
  return create_impl(cfg, device, rank, world, unique_id, out);
}

}  // extern "C"

namespace {
int create_impl(const specdec_config *cfg, int device, int rank, int world, const void *uid, specdec_handle **out) {
  if (!out) return SPECDEC_ERR_INVALID;
  *out = nullptr;
  auto h = std::make_unique<specdec_handle>();
  try {
    if (!cfg) fail(SPECDEC_ERR_INVALID, "null config");
    h->cfg = *cfg;
    h->device = device;
    h->tp_rank = rank;
    h->tp_world = world;
    CK(cudaSetDevice(device));
    CK(cudaDeviceGetAttribute(&h->num_sms, cudaDevAttrMultiProcessorCount, device));
    Dims td = make_dims(cfg->target);
    check_dims(td, "target");
    shard_dims(td, world, "target");
    specdec_model_config dcfg = cfg->draft;
    if (cfg->draft_shares_target) {
      const int nl = cfg->draft.n_layers;
      dcfg = cfg->target;
      dcfg.n_layers = nl;
      if (nl < 1 || nl > cfg->target.n_layers) fail(SPECDEC_ERR_INVALID, "draft layers must be in [1, target layers]");
    }
    Dims dd = make_dims(dcfg);
    check_dims(dd, "draft");
    shard_dims(dd, world, "draft");
    if (dd.V != td.V) fail(SPECDEC_ERR_INVALID, "target and draft vocab differ");
    if (dd.arch != td.arch) fail(SPECDEC_ERR_INVALID, "target and draft arch differ");
    if (td.L < 1 || dd.L < 1) fail(SPECDEC_ERR_INVALID, "models need at least one layer");
    if (cfg->weight_dtype != SPECDEC_F32 && cfg->weight_dtype != SPECDEC_INT8)
      fail(SPECDEC_ERR_INVALID, "weight_dtype must be F32 or INT8");
    if (cfg->act_dtype != SPECDEC_F32 && cfg->act_dtype != SPECDEC_BF16) fail(SPECDEC_ERR_INVALID, "bad act_dtype");
    if (cfg->kv_dtype != SPECDEC_F32 && cfg->kv_dtype != SPECDEC_BF16 && cfg->kv_dtype != SPECDEC_INT8)
      fail(SPECDEC_ERR_INVALID, "bad kv_dtype");
    if (cfg->max_batch < 1 || cfg->max_lookahead < 1 || cfg->max_lookahead > kMaxLookahead || cfg->max_prompt_len < 1)
      fail(SPECDEC_ERR_INVALID, "max_batch / max_lookahead / max_prompt_len out of range");
    if (td.V > 51200) fail(SPECDEC_ERR_UNSUPPORTED, "vocabularies above 51200 entries are not supported");
    h->tgt.dm = td;
    h->dft.dm = dd;
    CK(cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking));
    h->use_graph = std::getenv("SPECDEC_NO_GRAPH") == nullptr;
    h->use_pdl = std::getenv("SPECDEC_NO_PDL") == nullptr;
    set_attn_attrs<float>(0);
    set_attn_attrs<__nv_bfloat16>(1);
    set_attn_attrs<int8_t>(2);
    set_linear_attrs();
    h->gemm_max_split = set_gemm_attrs(h->gemm_clusters);
    if (const char *e = std::getenv("SPECDEC_GEMM_MAX_SPLIT"))  // a lower cap (1: no split-K), for comparisons
      h->gemm_max_split = std::max(1, std::min(h->gemm_max_split, std::atoi(e)));
    if (const char *e = std::getenv("SPECDEC_ATTN_CTAS_PER_SM")) h->attn_ctas_per_sm = std::max(1, std::atoi(e));
    if (const char *e = std::getenv("SPECDEC_ATTN_TC")) h->attn_tc = std::atoi(e) != 0;  // 0: CUDA-core attention only
    if (const char *e = std::getenv("SPECDEC_ATTN_TC_MIN_Q")) h->attn_tc_min_q = std::max(1, std::atoi(e));
    CK(cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAtcSmem));
    CK(attn_dec_set_attrs());
    CK(gemm_w8_set_attrs(h->w8_clusters));
    CK(gemm_sk_set_attrs());
    if (const char *e = std::getenv("SPECDEC_GEMM_SK")) h->gemm_sk = std::atoi(e) != 0;  // 0: no stream-K GEMM
    if (const char *e = std::getenv("SPECDEC_SK_MIN_TILES")) h->sk_min_tiles = std::max(1, std::atoi(e));
    if (const char *e = std::getenv("SPECDEC_SK_CTAS")) h->sk_max_ctas = std::max(0, std::atoi(e));
    if (const char *e = std::getenv("SPECDEC_GEMM_W8")) h->gemm_w8 = std::atoi(e) != 0;  // 1: the int8-code GEMM
    if (const char *e = std::getenv("SPECDEC_ATTN_DEC")) h->attn_dec = std::atoi(e) != 0;  // 0: not the decode kernel
    // GEMV / GEMM routing thresholds, for tuning measurements
    if (const char *e = std::getenv("SPECDEC_GEMM_MIN_ROWS")) h->gemm_min_rows = std::max(1, std::atoi(e));
    if (const char *e = std::getenv("SPECDEC_GEMM_WIDE_ROWS")) h->gemm_wide_rows = std::max(1, std::atoi(e));
    if (const char *e = std::getenv("SPECDEC_GEMM_WIDE_ELEMS")) h->gemm_wide_elems = std::max(1ll, std::atoll(e));
    {
      const int vs = td.V * static_cast<int>(sizeof(float));
      CK(cudaFuncSetAttribute(first_token_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, vs));
      CK(cudaFuncSetAttribute(draft_sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, vs));
      CK(cudaFuncSetAttribute(accept_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(accept_smem(h.get()))));
      CK(cudaFuncSetAttribute(tree_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, vs));
      CK(cudaFuncSetAttribute(tree_accept_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, vs));
      CK(cudaFuncSetAttribute(ar_token_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, vs));
      h->samp_max_cluster = set_samp_cluster_attrs(td.V);
      if (const char *e = std::getenv("SPECDEC_SAMPLE_MAX_CLUSTER"))  // a lower cap (1: one CTA per request)
        h->samp_max_cluster = std::max(1, std::min(h->samp_max_cluster, std::atoi(e)));
    }

    const int B = cfg->max_batch, k = cfg->max_lookahead;
    const bool kv8 = cfg->kv_dtype == SPECDEC_INT8;
    const size_t kv_elt = kv8 ? 1 : cfg->kv_dtype == SPECDEC_BF16 ? 2 : 4;
    // KV caches: per layer a pool of kv_pages pages, [page][Hkv][kKvPage][D]
    // (by default enough pages for every slot to reach max_seq_len)
    h->t_cap = td.max_seq;
    h->d_cap = dd.max_seq;
    h->ppr = (std::max(h->t_cap, h->d_cap) + kKvPage - 1) / kKvPage;
    if (cfg->kv_pages < 0) fail(SPECDEC_ERR_INVALID, "kv_pages < 0");
    h->kv_pages = cfg->kv_pages > 0 ? cfg->kv_pages : B * h->ppr;
    if (static_cast<int64_t>(h->kv_pages) * std::max(td.Hkv, dd.Hkv) * kKvPage > INT32_MAX)
      fail(SPECDEC_ERR_INVALID, "kv_pages x kv heads x 128 cache rows exceed 2^31");
    h->t_layer_stride = static_cast<size_t>(h->kv_pages) * td.Hkv * kKvPage * td.D;
    h->d_layer_stride = static_cast<size_t>(h->kv_pages) * dd.Hkv * kKvPage * dd.D;
    h->d_pt = static_cast<int *>(h->dalloc(static_cast<size_t>(B) * h->ppr * sizeof(int)));
    CK(cudaMemset(h->d_pt, 0xff, static_cast<size_t>(B) * h->ppr * sizeof(int)));  // -1: no page
    h->tk = h->dalloc(h->t_layer_stride * td.L * kv_elt);
    h->tv = h->dalloc(h->t_layer_stride * td.L * kv_elt);
    h->dk = h->dalloc(h->d_layer_stride * dd.L * kv_elt);
    h->dv = h->dalloc(h->d_layer_stride * dd.L * kv_elt);
    // cache rows past a request's length enter the P.V products with
    // probability 0; zeroed, they are finite from the start
    CK(cudaMemset(h->tk, 0, h->t_layer_stride * td.L * kv_elt));
    CK(cudaMemset(h->tv, 0, h->t_layer_stride * td.L * kv_elt));
    CK(cudaMemset(h->dk, 0, h->d_layer_stride * dd.L * kv_elt));
    CK(cudaMemset(h->dv, 0, h->d_layer_stride * dd.L * kv_elt));
    if (cfg->kv_dtype == SPECDEC_BF16 && cfg->act_dtype == SPECDEC_BF16 && (td.D == kAdD || dd.D == kAdD)) {
      h->ad_groups = B;
      const int Hm = std::max(td.H, dd.H);
      h->ad_part = static_cast<float *>(
          h->dalloc(static_cast<size_t>(B) * Hm * kAdMaxSplit * kAdPartFloats * sizeof(float)));
      h->ad_ticket = static_cast<int *>(h->dalloc(static_cast<size_t>(B) * Hm * sizeof(int)));
      CK(cudaMemset(h->ad_ticket, 0, static_cast<size_t>(B) * Hm * sizeof(int)));
    }
    if (kv8) {
      auto fb = [&](size_t n) { return static_cast<float *>(h->dalloc(n * sizeof(float))); };
      h->tks = fb(h->t_layer_stride / td.D * td.L);
      h->tvs = fb(h->t_layer_stride / td.D * td.L);
      h->dks = fb(h->d_layer_stride / dd.D * dd.L);
      h->dvs = fb(h->d_layer_stride / dd.D * dd.L);
    }
    // RoPE table, computed with the reference's float formula
    // (src/core/tensor.cpp:1147-1152): theta = pow(10000, -2j/D), omega = m*theta.
    h->rope_max = std::max(td.max_seq, dd.max_seq);
    h->rope_D = td.D;
    {
      const int D = td.D;
      std::vector<float2> tab(static_cast<size_t>(h->rope_max) * (D / 2));
      for (int m = 0; m < h->rope_max; ++m)
        for (int j = 0; j < D / 2; ++j) {
          const float theta = std::pow(10000.0f, -2.0f * static_cast<float>(j) / static_cast<float>(D));
          const float omega = static_cast<float>(m) * theta;
          tab[static_cast<size_t>(m) * (D / 2) + j] = make_float2(std::cos(omega), std::sin(omega));
        }
      h->rope = static_cast<float2 *>(h->dalloc(tab.size() * sizeof(float2)));
      CK(cudaMemcpy(h->rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice));
    }
    // activations
    if (cfg->max_tree_nodes < 0 || cfg->max_tree_nodes > kTreeMaxNodes)
      fail(SPECDEC_ERR_INVALID, "max_tree_nodes must be 0..64");
    h->max_tree = cfg->max_tree_nodes;
    const int R_round = std::max(std::max(B * (k + 1), 2 * B), h->max_tree ? B * (h->max_tree + 1) : 0);
    h->R_max = std::max(R_round, std::min(B * cfg->max_prompt_len, std::max(8192, R_round)));
    h->act_elt = act_bf16(h.get()) ? 2 : 4;
    const int dmax = std::max(td.d, dd.d), Fmax = std::max(td.F, dd.F);
    const size_t rowb = static_cast<size_t>(h->R_max) * dmax * h->act_elt;
    h->X = h->dalloc(rowb);
    h->H = h->dalloc(rowb);
    h->X1 = h->dalloc(rowb);
    h->Q = h->dalloc(rowb);
    h->ATT = h->dalloc(rowb);
    h->A = h->dalloc(static_cast<size_t>(h->R_max) * Fmax * h->act_elt);
    if (kv8)
      h->KVN = static_cast<float *>(
          h->dalloc(static_cast<size_t>(h->R_max) * 2 * std::max(td.kvd, dd.kvd) * sizeof(float)));
    h->logits = static_cast<float *>(h->dalloc(static_cast<size_t>(R_round) * td.V * sizeof(float)));
    // split-K partial tiles of the tensor-core GEMM: at most one per SM
    // (tiles x splits <= SMs), fp32 128 x 256 each
    if (cfg->act_dtype == SPECDEC_BF16 && cfg->weight_dtype == SPECDEC_INT8 && h->gemm_max_split > 1)
      h->gemm_ws = static_cast<float *>(h->dalloc(static_cast<size_t>(h->num_sms) * kBM * kBN * sizeof(float)));
    h->logits_rows = R_round;
    if (cfg->act_dtype == SPECDEC_BF16 && cfg->weight_dtype == SPECDEC_INT8) {
      h->w8_ws = static_cast<float *>(
          h->dalloc(static_cast<size_t>(specdec_handle::kW8WsTiles) * kW8MaxRows * kW8Feat * sizeof(float)));
      h->sk_ws = static_cast<float *>(h->dalloc(static_cast<size_t>(h->num_sms) * 2 * 256 * 256 * sizeof(float)));
    }
    h->tree_base =
        h->R_max + 2 * B + (k - 1) * B + B * (k + 1);
    const size_t pool_rows = static_cast<size_t>(h->tree_base) +
                             (h->max_tree ? static_cast<size_t>(B) * h->max_tree + static_cast<size_t>(B) * (h->max_tree + 1) : 0);
    auto ib = [&](size_t n) { return static_cast<int *>(h->dalloc(n * sizeof(int))); };
    h->pool.tok = ib(pool_rows);
    h->pool.pos = ib(pool_rows);
    h->pool.req = ib(pool_rows);
    h->pool.slot = ib(pool_rows);
    h->pool.tb = ib(pool_rows);
    h->pool.mask = static_cast<unsigned long long *>(h->dalloc(pool_rows * sizeof(unsigned long long)));
    CK(cudaMemset(h->pool.tok, 0, pool_rows * sizeof(int)));
    CK(cudaMemset(h->pool.pos, 0, pool_rows * sizeof(int)));
    CK(cudaMemset(h->pool.req, 0xff, pool_rows * sizeof(int)));
    CK(cudaMemset(h->pool.slot, 0, pool_rows * sizeof(int)));
    CK(cudaMemset(h->pool.tb, 0x7f, pool_rows * sizeof(int)));
    CK(cudaMemset(h->pool.mask, 0, pool_rows * sizeof(unsigned long long)));
    h->sel_odd = ib(B);
    h->sel_prefill = ib(B);
    fill_odd_kernel<<<(B + 127) / 128, 128, 0, h->stream>>>(h->sel_odd, B);
    CK(cudaGetLastError());
    // speculative state
    SpecState &st = h->st;
    const int out_len_max = cfg->max_prompt_len + std::max(td.max_seq, 1) + 1;
    st.tokens_out = ib(static_cast<size_t>(B) * out_len_max);
    st.n_new = ib(B); st.t_len = ib(B); st.d_len = ib(B); st.t_start = ib(B); st.d_start = ib(B);
    st.last_tok = ib(B); st.active = ib(B); st.M = ib(B); st.round = ib(B);
    st.cand = ib(static_cast<size_t>(B) * k);
    st.q = static_cast<float *>(h->dalloc(static_cast<size_t>(B) * k * td.V * sizeof(float)));
    st.stats = static_cast<long long *>(h->dalloc(static_cast<size_t>(B) * 4 * sizeof(long long)));
    st.mt = static_cast<uint32_t *>(h->dalloc(static_cast<size_t>(B) * kMtN * sizeof(uint32_t)));
    st.mt_idx = ib(B);
    st.ttok = ib(static_cast<size_t>(B) * kTreeMaxNodes);
    st.d_root = ib(B);
    st.cp_t0 = ib(B); st.cp_d0 = ib(B); st.cp_n = ib(B); st.cp_dn = ib(B);
    st.cp_path = ib(static_cast<size_t>(B) * kTreeMaxDepth);
    st.active_count = ib(1);
    st.err = ib(1);
    CK(cudaMemset(st.err, 0, sizeof(int)));
    CK(cudaMemset(st.active_count, 0, sizeof(int)));
    h->d_iters = ib(1);
    h->d_prompts = ib(static_cast<size_t>(B) * cfg->max_prompt_len);
    h->d_out = ib(static_cast<size_t>(B) * out_len_max);
    h->d_stats = static_cast<long long *>(h->dalloc(static_cast<size_t>(B) * 4 * sizeof(long long)));
    h->d_step_base = ib(B);
    h->d_step_cnt = ib(B);
    h->d_step_target = ib(1);
    h->step_tok_cap = static_cast<size_t>(out_len_max);
    h->d_step_tok = ib(static_cast<size_t>(B) * h->step_tok_cap);
    CK(cudaMallocHost(&h->h_pinned, 64));
    CK(cudaDeviceSynchronize());
    if (world > 1) {
      // NCCL operations cannot sit in the body of a conditional graph node,
      // so tensor-parallel rounds are driven from the host
      h->use_graph = false;
      // collective over the `world` ranks; each calls it with its device current
      ncclUniqueId id;
      std::memcpy(&id, uid, sizeof(id));
      nccl_check(nccl().comm_init_rank(&h->comm, world, id, rank), "ncclCommInitRank");
    }
  } catch (const SpecErr &e) {
    g_create_err = e.msg;
    specdec_destroy(h.release());
    return e.code;
  }
  *out = h.release();
  return SPECDEC_OK;
}
}  // namespace

extern "C" {

int specdec_destroy(specdec_handle *h) {
  if (!h) return SPECDEC_OK;
  cudaSetDevice(h->device);
  if (h->stream) cudaStreamSynchronize(h->stream);
  destroy_graphs(h);  // graphs holding NCCL calls go before the communicator
  if (h->comm) {
    nccl().comm_destroy(h->comm);
    h->comm = nullptr;
  }
  for (int r = 0; r < 2; ++r)
    for (void *p : h->weight_allocs[r]) cudaFree(p);
  for (void *p : h->allocs) cudaFree(p);
  if (h->d_uniforms) cudaFree(h->d_uniforms);
  if (h->h_pinned) cudaFreeHost(h->h_pinned);
  if (h->stream) cudaStreamDestroy(h->stream);
  delete h;
  return SPECDEC_OK;
}

void *specdec_stream(specdec_handle *h) { return h ? static_cast<void *>(h->stream) : nullptr; }

int64_t specdec_last_launch_count(const specdec_handle *h) {
  if (!h) return 0;
  if (h->launches >= 0) return h->launches;
  if (cudaMemcpyAsync(h->h_pinned + 1, h->d_iters, sizeof(int), cudaMemcpyDeviceToHost, h->stream) != cudaSuccess ||
      cudaStreamSynchronize(h->stream) != cudaSuccess)
    return -1;
  return h->graph_fixed + h->graph_body * h->h_pinned[1] + h->extra_launches;
}

int specdec_time_linear(specdec_handle *h, int role, int layer, int which, int rows, int reps, void *flush,
                        size_t flush_bytes, float *avg_us, double *alg_bytes) {
  if (!h || !avg_us || !alg_bytes || reps < 1) return SPECDEC_ERR_INVALID;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  try {
    CK(cudaSetDevice(h->device));
    if (role != SPECDEC_TARGET && role != SPECDEC_DRAFT) fail(SPECDEC_ERR_INVALID, "unknown role");
    ModelW &m = role == SPECDEC_TARGET ? h->tgt : h->dft;
    if (!m.loaded) fail(SPECDEC_ERR_STATE, "weights not loaded");
    const Dims &dm = m.dm;
    if (layer < 0 || layer >= dm.L) fail(SPECDEC_ERR_INVALID, "layer out of range");
    if (rows < 1 || rows > h->R_max) fail(SPECDEC_ERR_INVALID, "rows out of range");
    const LayerW &L = m.layers[layer];
    const bool ref = dm.arch == SPECDEC_ARCH_REF;
    const int d = dm.d;
    // rows of the prefill region marked unused, so a QKV launch appends nothing
    CK(cudaMemsetAsync(h->pool.req, 0xff, static_cast<size_t>(rows) * sizeof(int), h->stream));
    RowsView rv{h->pool.tok, h->pool.pos, h->pool.req};
    const double wb = w_int8(h) ? 1.0 : 4.0, ab = static_cast<double>(h->act_elt);
    LinearArgs a{};
    a.R = rows; a.rows = rv; a.K = d; a.ldx = d;
    int epi = kEpiStore;
    double in_w = d, out_w = d;  // input / output row widths
    switch (which) {
      case SPECDEC_LIN_QKV:
        a.x = h->H; a.W = L.wqkv; a.scale = L.sqkv; a.bias = L.bqkv; a.N = dm.dq + 2 * dm.kvd; a.out = h->Q;
        a.ldo = dm.dq; a.in_g = L.g1; a.in_b = L.b1;
        a.qkv = QKVArgs{dm.dq, dm.kvd, dm.D, h->rope, h->rope_max, h->tk, h->tv, KvPages{h->d_pt, h->ppr}, 1, 0,
                        nullptr, nullptr};
        epi = kEpiQKV; out_w = dm.dq + 2 * dm.kvd;
        break;
      case SPECDEC_LIN_OPROJ:
        a.x = h->ATT; a.ldx = dm.dq; a.K = dm.dq; a.W = L.wo; a.scale = L.so; a.bias = L.bo; a.N = d; a.out = h->H;
        a.ldo = d; a.resid = h->X; a.ldr = d; epi = kEpiResid; in_w = dm.dq; out_w = 2.0 * d;
        break;
      case SPECDEC_LIN_FFN_IN:
        a.x = h->H; a.W = L.wgu; a.scale = L.sgu; a.bias = L.bgu; a.N = ref ? 2 * dm.F : dm.F; a.out = h->A;
        a.ldo = dm.F; a.in_g = ref ? L.g1 : L.g2; a.in_b = ref ? L.b1 : L.b2; a.norm_out = ref ? h->X1 : nullptr;
        epi = ref ? kEpiSwiGLU : kEpiGelu; out_w = dm.F + (ref ? d : 0);
        break;
      case SPECDEC_LIN_FFN_OUT:
        a.x = h->A; a.ldx = dm.F; a.K = dm.F; a.W = L.wd; a.scale = L.sd; a.bias = L.bd; a.N = d; a.out = h->H;
        a.ldo = d; a.resid = h->X1; a.ldr = d; epi = kEpiResid; in_w = dm.F; out_w = 2.0 * d;
        break;
      case SPECDEC_LIN_HEAD:
        a.x = h->H; a.W = m.whead; a.scale = m.shead; a.bias = m.bhead; a.N = dm.V; a.out = h->logits; a.ldo = dm.V;
        a.out_f32 = 1; a.in_g = m.layers[dm.L - 1].g2; a.in_b = m.layers[dm.L - 1].b2; out_w = dm.V;
        if (rows > h->logits_rows) fail(SPECDEC_ERR_INVALID, "rows exceed the logits buffer");
        break;
      default:
        fail(SPECDEC_ERR_INVALID, "unknown linear layer");
    }
    *alg_bytes = static_cast<double>(a.N) * a.K * wb + (w_int8(h) ? 4.0 * a.N : 0.0) + 4.0 * a.N +
                 (a.in_g ? 8.0 * a.K : 0.0) + rows * in_w * ab + rows * out_w * (which == SPECDEC_LIN_HEAD ? 4.0 : ab);
    CK(cudaEventCreate(&e0));
    CK(cudaEventCreate(&e1));
    double tot_ms = 0.0;
    for (int i = 0; i < reps; ++i) {
      if (flush && flush_bytes) CK(cudaMemsetAsync(flush, i & 0xff, flush_bytes, h->stream));
      CK(cudaEventRecord(e0, h->stream));
      switch (epi) {
        case kEpiQKV: launch_linear<kEpiQKV>(h, a); break;
        case kEpiResid: launch_linear<kEpiResid>(h, a); break;
        case kEpiSwiGLU: launch_linear<kEpiSwiGLU>(h, a); break;
        case kEpiGelu: launch_linear<kEpiGelu>(h, a); break;
        default: launch_linear<kEpiStore>(h, a); break;
      }
      CK(cudaEventRecord(e1, h->stream));
      CK(cudaEventSynchronize(e1));
      float ms = 0.f;
      CK(cudaEventElapsedTime(&ms, e0, e1));
      tot_ms += ms;
    }
    *avg_us = static_cast<float>(tot_ms * 1000.0 / reps);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
  } catch (const SpecErr &e) {
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    h->err = e.msg;
    return e.code;
  }
  return SPECDEC_OK;
}

int specdec_time_attention(specdec_handle *h, int role, int layer, int q_per_req, int reps, void *flush,
                           size_t flush_bytes, float *avg_us, double *alg_bytes) {
  if (!h || !avg_us || !alg_bytes || reps < 1) return SPECDEC_ERR_INVALID;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  try {
    CK(cudaSetDevice(h->device));
    if (!h->step_open) fail(SPECDEC_ERR_STATE, "no open session: call specdec_prefill first");
    if (role != SPECDEC_TARGET && role != SPECDEC_DRAFT) fail(SPECDEC_ERR_INVALID, "unknown role");
    const bool target = role == SPECDEC_TARGET;
    const ModelW &m = target ? h->tgt : h->dft;
    const Dims &dm = m.dm;
    if (layer < 0 || layer >= dm.L) fail(SPECDEC_ERR_INVALID, "layer out of range");
    const int B = h->st.B;
    if (q_per_req < 1 || B * q_per_req > h->R_max) fail(SPECDEC_ERR_INVALID, "rows out of range");
    const int R = B * q_per_req;
    const int *len = target ? h->st.t_len : h->st.d_len;
    std::vector<int> hl(B);
    CK(cudaMemcpyAsync(hl.data(), len, B * sizeof(int), cudaMemcpyDeviceToHost, h->stream));
    sync_check(h);
    launch(h, probe_rows_kernel, dim3((R + 127) / 128), dim3(128), 0, len, B, q_per_req, h->pool.tok, h->pool.pos,
           h->pool.req);
    RowsView rows{h->pool.tok, h->pool.pos, h->pool.req};
    const bool kv8 = h->cfg.kv_dtype == SPECDEC_INT8;
    const size_t kv_elt = kv8 ? 1 : h->cfg.kv_dtype == SPECDEC_BF16 ? 2 : 4;
    const size_t lstride = target ? h->t_layer_stride : h->d_layer_stride;
    const size_t lrows = lstride / dm.D;
    void *kcl = static_cast<char *>(target ? h->tk : h->dk) + layer * lstride * kv_elt;
    void *vcl = static_cast<char *>(target ? h->tv : h->dv) + layer * lstride * kv_elt;
    float *ksl = kv8 ? (target ? h->tks : h->dks) + layer * lrows : nullptr;
    float *vsl = kv8 ? (target ? h->tvs : h->dvs) + layer * lrows : nullptr;
    double ctx = 0.0;
    for (int b = 0; b < B; ++b) ctx += std::max(1, hl[b]);
    // every visible K and V row once (plus int8 scales), the query rows in,
    // the output rows out
    *alg_bytes = ctx * 2.0 * dm.kvd * kv_elt + (kv8 ? ctx * 2.0 * dm.Hkv * 4.0 : 0.0) +
                 2.0 * R * dm.dq * static_cast<double>(h->act_elt);
    CK(cudaEventCreate(&e0));
    CK(cudaEventCreate(&e1));
    double tot_ms = 0.0;
    for (int i = 0; i < reps; ++i) {
      if (flush && flush_bytes) CK(cudaMemsetAsync(flush, i & 0xff, flush_bytes, h->stream));
      CK(cudaEventRecord(e0, h->stream));
      attention(h, dm, rows, R, q_per_req, kcl, vcl, ksl, vsl, lstride, target ? h->t_cap : h->d_cap,
                KvPages{h->d_pt, h->ppr});
      CK(cudaEventRecord(e1, h->stream));
      CK(cudaEventSynchronize(e1));
      float ms = 0.f;
      CK(cudaEventElapsedTime(&ms, e0, e1));
      tot_ms += ms;
    }
    *avg_us = static_cast<float>(tot_ms * 1000.0 / reps);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    check_device_err(h);
  } catch (const SpecErr &e) {
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    h->err = e.msg;
    return e.code;
  }
  return SPECDEC_OK;
}

int specdec_load_params(specdec_handle *h, int role, int n_params, const float *const *params, const int64_t *numels) {
  if (!h) return SPECDEC_ERR_INVALID;
  try {
    CK(cudaSetDevice(h->device));
    if (!params || !numels) fail(SPECDEC_ERR_INVALID, "null parameter list");
    if (role == SPECDEC_TARGET) {
      load_model(h, 0, h->tgt, n_params, params, numels);
      if (h->cfg.draft_shares_target) {
        // draft = first n layers + shared embedding / lm_head, same device memory
        ModelW &d = h->dft;
        const ModelW &t = h->tgt;
        d.emb = t.emb; d.pos = t.pos; d.gf = t.gf; d.bfin = t.bfin;
        d.whead = t.whead; d.shead = t.shead; d.bhead = t.bhead;
        d.layers.assign(t.layers.begin(), t.layers.begin() + d.dm.L);
        d.loaded = true;
      }
    } else if (role == SPECDEC_DRAFT) {
      if (h->cfg.draft_shares_target) fail(SPECDEC_ERR_STATE, "the draft shares the target's weights");
      load_model(h, 1, h->dft, n_params, params, numels);
    } else {
      fail(SPECDEC_ERR_INVALID, "unknown role");
    }
    destroy_graphs(h);
    h->step_open = false;
    CK(cudaDeviceSynchronize());
  } catch (const SpecErr &e) {
    h->err = e.msg;
    return e.code;
  }
  return SPECDEC_OK;
}

int specdec_load_params_device(specdec_handle *h, int role, int n_params, const float *const *d_params,
                               const int64_t *numels) {
  if (!h) return SPECDEC_ERR_INVALID;
  h->src_device = true;
  const int rc = specdec_load_params(h, role, n_params, d_params, numels);
  h->src_device = false;
  return rc;
}

int specdec_load_netw(specdec_handle *h, int role, const char *path) {
  if (!h) return SPECDEC_ERR_INVALID;
  try {
    if (!path) fail(SPECDEC_ERR_INVALID, "null path");
    if (role != SPECDEC_TARGET && role != SPECDEC_DRAFT) fail(SPECDEC_ERR_INVALID, "unknown role");
    const auto shapes = param_shapes(role == SPECDEC_TARGET ? h->tgt.dm : h->dft.dm);
    // serialization::load_parameters (src/core/serialization.cpp:49-107):
    // "NETW", u16 version 1, u32 count, then per tensor u32 dims, u64 shape
    // [dims], u64 element count, float32 data; every check throws there.
    std::ifstream in(path, std::ios::binary);
    if (!in) fail(SPECDEC_ERR_INVALID, std::string("Failed to open file for reading: ") + path);
    char magic[4];
    in.read(magic, 4);
    if (in.gcount() != 4 || std::string(magic, 4) != "NETW") fail(SPECDEC_ERR_INVALID, "Invalid file format signature.");
    uint16_t version = 0;
    in.read(reinterpret_cast<char *>(&version), sizeof(version));
    if (!in || version != 1)
      fail(SPECDEC_ERR_INVALID, "Unsupported serialization file version: " + std::to_string(version));
    uint32_t count = 0;
    in.read(reinterpret_cast<char *>(&count), sizeof(count));
    if (!in || count != shapes.size())
      fail(SPECDEC_ERR_INVALID, "Tensor count mismatch (file has " + std::to_string(count) + ", model has " +
                                    std::to_string(shapes.size()) + ").");
    std::vector<std::vector<float>> data(count);
    for (uint32_t t = 0; t < count; ++t) {
      uint32_t dims = 0;
      in.read(reinterpret_cast<char *>(&dims), sizeof(dims));
      if (!in || dims != shapes[t].size()) fail(SPECDEC_ERR_INVALID, "Tensor dimension count mismatch.");
      uint64_t total = 1;
      for (uint32_t i = 0; i < dims; ++i) {
        uint64_t v = 0;
        in.read(reinterpret_cast<char *>(&v), sizeof(v));
        if (!in || v != shapes[t][i])
          fail(SPECDEC_ERR_INVALID, "Tensor shape mismatch at dimension " + std::to_string(i));
        total *= v;
      }
      uint64_t ne = 0;
      in.read(reinterpret_cast<char *>(&ne), sizeof(ne));
      if (!in || ne != total) fail(SPECDEC_ERR_INVALID, "Tensor element count mismatch.");
      data[t].resize(total);
      in.read(reinterpret_cast<char *>(data[t].data()), static_cast<std::streamsize>(total * sizeof(float)));
      if (static_cast<uint64_t>(in.gcount()) != total * sizeof(float))
        fail(SPECDEC_ERR_INVALID, "truncated tensor data in " + std::string(path));
    }
    std::vector<const float *> ptrs(count);
    std::vector<int64_t> numels(count);
    for (uint32_t t = 0; t < count; ++t) {
      ptrs[t] = data[t].data();
      numels[t] = static_cast<int64_t>(data[t].size());
    }
    return specdec_load_params(h, role, static_cast<int>(count), ptrs.data(), numels.data());
  } catch (const SpecErr &e) {
    h->err = e.msg;
    return e.code;
  }
}

int specdec_generate_device(specdec_handle *h, const specdec_gen_params *p, const int32_t *d_prompts, int B, int S,
                            int32_t *d_out_tokens, int64_t *d_out_stats) {
  if (!h) return SPECDEC_ERR_INVALID;
  try {
    CK(cudaSetDevice(h->device));
    if (!d_prompts || !d_out_tokens) fail(SPECDEC_ERR_INVALID, "null buffer");
    return generate_impl(h, p, d_prompts, B, S, d_out_tokens, d_out_stats);
  } catch (const SpecErr &e) {
    h->err = e.msg;
    return e.code;
  }
}

namespace {
int host_generate(specdec_handle *h, const specdec_gen_params *p, const specdec_tree *tr, const int32_t *prompts, int B,
                  int S, int32_t *out_tokens, int64_t *out_stats, bool ar = false);
}

int specdec_generate(specdec_handle *h, const specdec_gen_params *p, const int32_t *prompts, int B, int S,
                     int32_t *out_tokens, int64_t *out_stats) {
  return host_generate(h, p, nullptr, prompts, B, S, out_tokens, out_stats);
}

int specdec_generate_tree_device(specdec_handle *h, const specdec_gen_params *p, const specdec_tree *tree,
                                 const int32_t *d_prompts, int B, int S, int32_t *d_out_tokens,
                                 int64_t *d_out_stats) {
  if (!h) return SPECDEC_ERR_INVALID;
  try {
    CK(cudaSetDevice(h->device));
    if (!d_prompts || !d_out_tokens) fail(SPECDEC_ERR_INVALID, "null buffer");
    const TreeCfg tc = make_tree(h, tree);
    return generate_impl(h, p, d_prompts, B, S, d_out_tokens, d_out_stats, &tc);
  } catch (const SpecErr &e) {
    h->err = e.msg;
    return e.code;
  }
}

int specdec_generate_tree(specdec_handle *h, const specdec_gen_params *p, const specdec_tree *tree,
                          const int32_t *prompts, int B, int S, int32_t *out_tokens, int64_t *out_stats) {
  if (!tree) {
    if (h) h->err = "null tree";
    return SPECDEC_ERR_INVALID;
  }
  return host_generate(h, p, tree, prompts, B, S, out_tokens, out_stats);
}

int specdec_generate_ar(specdec_handle *h, const specdec_gen_params *p, const int32_t *prompts, int B, int S,
                        int32_t *out_tokens, int64_t *out_stats) {
  return host_generate(h, p, nullptr, prompts, B, S, out_tokens, out_stats, true);
}

int specdec_generate_ar_device(specdec_handle *h, const specdec_gen_params *p, const int32_t *d_prompts, int B, int S,
                               int32_t *d_out_tokens, int64_t *d_out_stats) {
  if (!h) return SPECDEC_ERR_INVALID;
  try {
    CK(cudaSetDevice(h->device));
    if (!d_prompts || !d_out_tokens) fail(SPECDEC_ERR_INVALID, "null buffer");
    return generate_impl(h, p, d_prompts, B, S, d_out_tokens, d_out_stats, nullptr, true);
  } catch (const SpecErr &e) {
    h->err = e.msg;
    return e.code;
  }
}

int specdec_prefill(specdec_handle *h, const specdec_gen_params *p, const int32_t *prompts, int B, int S) {
  if (!h) return SPECDEC_ERR_INVALID;
  try {
    CK(cudaSetDevice(h->device));
    if (!prompts) fail(SPECDEC_ERR_INVALID, "null buffer");
    if (B < 1 || B > h->cfg.max_batch || S < 1 || S > h->cfg.max_prompt_len)
      fail(SPECDEC_ERR_INVALID, "batch or prompt length out of range");
    CK(cudaMemcpyAsync(h->d_prompts, prompts, static_cast<size_t>(B) * S * sizeof(int), cudaMemcpyHostToDevice,
                       h->stream));
    prefill_impl(h, p, h->d_prompts, B, S);
    check_device_err(h);
  } catch (const SpecErr &e) {
    h->step_open = false;
    h->err = e.msg;
    return e.code;
  }
  return SPECDEC_OK;
}

int specdec_prefill_device(specdec_handle *h, const specdec_gen_params *p, const int32_t *d_prompts, int B, int S) {
  if (!h) return SPECDEC_ERR_INVALID;
  try {
    CK(cudaSetDevice(h->device));
    if (!d_prompts) fail(SPECDEC_ERR_INVALID, "null buffer");
    prefill_impl(h, p, d_prompts, B, S);
  } catch (const SpecErr &e) {
    h->step_open = false;
    h->err = e.msg;
    return e.code;
  }
  return SPECDEC_OK;
}

int specdec_step(specdec_handle *h, int rounds, const float *uniforms, int32_t *out_tokens, int32_t *out_counts) {
  if (!h) return SPECDEC_ERR_INVALID;
  try {
    CK(cudaSetDevice(h->device));
    if (!out_tokens || !out_counts) fail(SPECDEC_ERR_INVALID, "null buffer");
    if (!h->step_open) fail(SPECDEC_ERR_STATE, "no open session: call specdec_prefill first");
    const int B = h->st.B;
    const long long want = static_cast<long long>(rounds) * (h->st.k + 1);
    const int cap = static_cast<int>(std::max(1LL, std::min<long long>(want, static_cast<long long>(h->step_tok_cap))));
    step_impl(h, rounds, uniforms, h->d_step_tok, h->d_step_cnt, cap);
    // the device rows are cap wide, the caller's rounds * (k + 1)
    CK(cudaMemcpy2DAsync(out_tokens, static_cast<size_t>(want) * sizeof(int), h->d_step_tok, cap * sizeof(int),
                         cap * sizeof(int), B, cudaMemcpyDeviceToHost, h->stream));
    CK(cudaMemcpyAsync(out_counts, h->d_step_cnt, B * sizeof(int), cudaMemcpyDeviceToHost, h->stream));
    check_device_err(h);
  } catch (const SpecErr &e) {
    h->err = e.msg;
    return e.code;
  }
  return SPECDEC_OK;
}

int specdec_step_device(specdec_handle *h, int rounds, const float *uniforms, int32_t *d_out_tokens,
                        int32_t *d_out_counts, int cap) {
  if (!h) return SPECDEC_ERR_INVALID;
  try {
    CK(cudaSetDevice(h->device));
    step_impl(h, rounds, uniforms, d_out_tokens, d_out_counts, cap);
  } catch (const SpecErr &e) {
    h->err = e.msg;
    return e.code;
  }
  return SPECDEC_OK;
}

int specdec_session_tokens(specdec_handle *h, int32_t *out_tokens, int64_t *out_stats) {
  if (!h) return SPECDEC_ERR_INVALID;
  try {
    CK(cudaSetDevice(h->device));
    if (!out_tokens) fail(SPECDEC_ERR_INVALID, "null buffer");
    if (!h->step_open) fail(SPECDEC_ERR_STATE, "no open session: call specdec_prefill first");
    const SpecState &st = h->st;
    launch(h, finalize_kernel, dim3(st.B), dim3(128), 0, st, static_cast<int *>(h->d_out),
           reinterpret_cast<long long *>(h->d_stats));
    const int n = st.prompt_len + std::max(1, st.max_new);
    CK(cudaMemcpyAsync(out_tokens, h->d_out, static_cast<size_t>(st.B) * n * sizeof(int), cudaMemcpyDeviceToHost,
                       h->stream));
    if (out_stats)
      CK(cudaMemcpyAsync(out_stats, h->d_stats, static_cast<size_t>(st.B) * 4 * sizeof(int64_t),
                         cudaMemcpyDeviceToHost, h->stream));
    check_device_err(h);
  } catch (const SpecErr &e) {
    h->err = e.msg;
    return e.code;
  }
  return SPECDEC_OK;
}

}  // extern "C"

namespace {
int host_generate(specdec_handle *h, const specdec_gen_params *p, const specdec_tree *tr, const int32_t *prompts, int B,
                  int S, int32_t *out_tokens, int64_t *out_stats, bool ar) {
  if (!h) return SPECDEC_ERR_INVALID;
  try {
    CK(cudaSetDevice(h->device));
    if (!prompts || !out_tokens) fail(SPECDEC_ERR_INVALID, "null buffer");
    if (!p) fail(SPECDEC_ERR_INVALID, "null params");
    if (B < 1 || B > h->cfg.max_batch || S < 1 || S > h->cfg.max_prompt_len)
      fail(SPECDEC_ERR_INVALID, "batch or prompt length out of range");
    TreeCfg tc;
    if (tr) tc = make_tree(h, tr);
    CK(cudaMemcpyAsync(h->d_prompts, prompts, static_cast<size_t>(B) * S * sizeof(int), cudaMemcpyHostToDevice, h->stream));
    int rc = generate_impl(h, p, h->d_prompts, B, S, h->d_out, reinterpret_cast<int64_t *>(h->d_stats),
                           tr ? &tc : nullptr, ar);
    if (rc != SPECDEC_OK) return rc;
    const int n = S + (ar ? p->max_new_tokens : std::max(1, p->max_new_tokens));
    CK(cudaMemcpyAsync(out_tokens, h->d_out, static_cast<size_t>(B) * n * sizeof(int), cudaMemcpyDeviceToHost, h->stream));
    if (out_stats)
      CK(cudaMemcpyAsync(out_stats, h->d_stats, static_cast<size_t>(B) * 4 * sizeof(int64_t), cudaMemcpyDeviceToHost,
                         h->stream));
    CK(cudaMemcpyAsync(h->h_pinned, h->st.err, sizeof(int), cudaMemcpyDeviceToHost, h->stream));
    sync_check(h);
    const int err = h->h_pinned[0];
    if (err & kErrSeqLen) fail(SPECDEC_ERR_SEQ_LEN, "Sequence length S plus past cached length exceeds max_seq_len");
    if (err & kErrRngTable) fail(SPECDEC_ERR_RNG, "the host uniform table has too few rounds");
    if (err & kErrTimeout) fail(SPECDEC_ERR_CUDA, "an asynchronous copy did not complete within its wait limit");
  } catch (const SpecErr &e) {
    h->err = e.msg;
    return e.code;
  }
  return SPECDEC_OK;
}
}  // namespace

extern "C" {

int specdec_forward_logits(specdec_handle *h, int role, const int32_t *tokens, int S, float *logits) {
  if (!h) return SPECDEC_ERR_INVALID;
  try {
    CK(cudaSetDevice(h->device));
    const bool target = role == SPECDEC_TARGET;
    if (role != SPECDEC_TARGET && role != SPECDEC_DRAFT) fail(SPECDEC_ERR_INVALID, "unknown role");
    ModelW &m = target ? h->tgt : h->dft;
    if (!m.loaded) fail(SPECDEC_ERR_STATE, "weights not loaded");
    if (!tokens || !logits) fail(SPECDEC_ERR_INVALID, "null buffer");
    if (S < 1 || S > (target ? h->t_cap : h->d_cap) || S > h->R_max || S > h->cfg.max_prompt_len * h->cfg.max_batch)
      fail(SPECDEC_ERR_INVALID, "sequence length out of range");
    const Dims &dm = m.dm;
    h->launches = 0;
    // the forward's K/V go to request slot 0's cache: an open session ends
    h->step_open = false;
    assign_pages(h, 1, S);
    CK(cudaMemsetAsync(h->st.err, 0, sizeof(int), h->stream));
    CK(cudaMemcpyAsync(h->d_prompts, tokens, S * sizeof(int), cudaMemcpyHostToDevice, h->stream));
    launch(h, plan_prefill_kernel, dim3((S + 255) / 256), dim3(256), 0, static_cast<const int *>(h->d_prompts), 1, S, 0,
           S, dm.V, h->pool.tok, h->pool.pos, h->pool.req, static_cast<int *>(nullptr));
    forward_rows(h, target, 0, S, S, nullptr, 0, nullptr);
    // the lm_head over row chunks that fit the logits buffer
    const int R_round = std::max(h->cfg.max_batch * (h->cfg.max_lookahead + 1), 2 * h->cfg.max_batch);
    RowsView rows{h->pool.tok, h->pool.pos, h->pool.req};
    const HeadInput hi = head_input(h, m);
    for (int c0 = 0; c0 < S; c0 += R_round) {
      const int n = std::min(R_round, S - c0);
      LinearArgs hd{};
      hd.R = n; hd.W = m.whead; hd.scale = m.shead; hd.bias = m.bhead; hd.N = dm.V; hd.K = dm.d;
      hd.out = h->logits; hd.ldo = dm.V; hd.out_f32 = 1; hd.rows = rows;
      hd.in_g = hi.g; hd.in_b = hi.b;
      hd.x = static_cast<const char *>(hi.x) + static_cast<size_t>(c0) * dm.d * h->act_elt;
      hd.ldx = dm.d;
      launch_linear<kEpiStore>(h, hd);
      CK(cudaMemcpyAsync(logits + static_cast<size_t>(c0) * dm.V, h->logits, static_cast<size_t>(n) * dm.V * sizeof(float),
                         cudaMemcpyDeviceToHost, h->stream));
    }
    CK(cudaMemcpyAsync(h->h_pinned, h->st.err, sizeof(int), cudaMemcpyDeviceToHost, h->stream));
    sync_check(h);
    if (h->h_pinned[0]) fail(SPECDEC_ERR_SEQ_LEN, "cache capacity exceeded");
  } catch (const SpecErr &e) {
    h->err = e.msg;
    return e.code;
  }
  return SPECDEC_OK;
}

int specdec_philox_uniforms(uint64_t seed, int B, int rounds, int slots, float *out) {
  if (!out || B < 0 || rounds < 0 || slots < 0) return SPECDEC_ERR_INVALID;
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
  const int nblk = (slots + 3) / 4;
  for (int b = 0; b < B; ++b)
    for (int r = 0; r < rounds; ++r)
      for (int blk = 0; blk < nblk; ++blk) {
        uint32_t c[4] = {static_cast<uint32_t>(blk), static_cast<uint32_t>(r), static_cast<uint32_t>(b), 0x53504543u};
        uint32_t k0 = static_cast<uint32_t>(seed), k1 = static_cast<uint32_t>(seed >> 32);
        for (int i = 0; i < 10; ++i) {
          const uint64_t p0 = static_cast<uint64_t>(M0) * c[0], p1 = static_cast<uint64_t>(M1) * c[2];
          const uint32_t hi0 = static_cast<uint32_t>(p0 >> 32), lo0 = static_cast<uint32_t>(p0);
          const uint32_t hi1 = static_cast<uint32_t>(p1 >> 32), lo1 = static_cast<uint32_t>(p1);
          const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
          c[0] = n0; c[1] = lo1; c[2] = n2; c[3] = lo0;
          k0 += W0;
          k1 += W1;
        }
        for (int l = 0; l < 4; ++l) {
          const int s = blk * 4 + l;
          if (s < slots) out[(static_cast<size_t>(b) * rounds + r) * slots + s] = static_cast<float>(c[l] >> 8) * (1.0f / 16777216.0f);
        }
      }
  return SPECDEC_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Forward logits without any device allocation.
//
// Some callers cannot call cudaMalloc at the moment they need a forward pass:
// code that runs inside another runtime's memory pool (which owns every
// device byte and forbids allocations behind its back), real-time serving
// loops where an allocation can stall the device, and callers whose CUDA
// context is shared and must not grow.  For them this entry point takes the
// tokens and the logits as device buffers they already own and keeps all of
// its own working memory (activations, the row tables and the per-sequence KV
// cache) in one file-scope device array of
// fixed size, SPECDEC_NOALLOC_SCRATCH_BYTES, which every GPU that loads this
// library holds until the process exits.  It calls no cudaMalloc, cudaFree or
// allocating library routine.
//
// The array is shared by every call on a device and keeps the last call's
// contents; the error word is cleared at the start of each call.  Calls whose
// work overlaps on the GPU (different streams, or different handles on the
// same device) race on the array and must be serialised by the caller.  The
// first call on each device looks up the array's device address
// (cudaGetSymbolAddress) with that device current; make that first call
// before starting any stream capture.
#define SPECDEC_NOALLOC_SCRATCH_BYTES (8u << 20)
static __device__ __align__(256) unsigned char g_noalloc_scratch[SPECDEC_NOALLOC_SCRATCH_BYTES];

namespace {
std::mutex g_noalloc_mu;
std::map<int, unsigned char *> g_noalloc_base;  // device ordinal -> device address of the array

// The device address of the scratch array on the current device (set-up once
// per device).  The host-side name of the array is not a device address.
cudaError_t noalloc_base(int device, unsigned char **out) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  auto it = g_noalloc_base.find(device);
  if (it != g_noalloc_base.end()) {
    *out = it->second;
    return cudaSuccess;
  }
  void *ptr = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
  if (e != cudaSuccess) return e;
  g_noalloc_base[device] = static_cast<unsigned char *>(ptr);
  *out = static_cast<unsigned char *>(ptr);
  return cudaSuccess;
}

// Copies the scratch array's error word to the caller's status word.
// Page table of one request whose pages are 0 .. n-1 of its pool.
__global__ void page_iota_kernel(int *pt, int n) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) pt[i] = i;
}

__global__ void copy_status_kernel(const int *err, int32_t *status) { *status = *err; }

struct ArenaCarver {
  unsigned char *base;
  size_t used = 0;
  void *take(size_t bytes) {
    void *p = base ? base + used : nullptr;
    used += (bytes + 255) & ~size_t(255);
    return p;
  }
};
}  // namespace

extern "C" int specdec_forward_logits_noalloc(specdec_handle *h, int role, const int32_t *d_tokens, int S,
                                              float *d_logits, void *stream, int32_t *d_status) {
  if (!h) return SPECDEC_ERR_INVALID;
  // The handle's working buffers are pointed at the scratch array for the
  // duration of the call and restored on every exit path.
  struct Saved {
    void *X, *H, *X1, *A, *Q, *ATT, *tk, *tv, *dk, *dv;
    float *tks, *tvs, *dks, *dvs, *KVN;
    int *err;
    RowPool pool;
    size_t tls, dls;
    int *pt;
    int ppr, tcap, dcap, R_max;
    cudaStream_t stream;
    float *gemm_ws, *ad_part, *w8_ws, *sk_ws;
  };
  Saved sv{h->X, h->H, h->X1, h->A, h->Q, h->ATT, h->tk, h->tv, h->dk, h->dv, h->tks, h->tvs, h->dks, h->dvs, h->KVN,
           h->st.err, h->pool,
           h->t_layer_stride, h->d_layer_stride, h->d_pt, h->ppr, h->t_cap, h->d_cap, h->R_max,
           h->stream, h->gemm_ws, h->ad_part, h->w8_ws, h->sk_ws};
  auto restore = [&] {
    h->X = sv.X; h->H = sv.H; h->X1 = sv.X1; h->A = sv.A; h->Q = sv.Q; h->ATT = sv.ATT;
    h->tk = sv.tk; h->tv = sv.tv; h->dk = sv.dk; h->dv = sv.dv;
    h->tks = sv.tks; h->tvs = sv.tvs; h->dks = sv.dks; h->dvs = sv.dvs; h->KVN = sv.KVN;
    h->st.err = sv.err; h->pool = sv.pool;
    h->t_layer_stride = sv.tls; h->d_layer_stride = sv.dls; h->d_pt = sv.pt; h->ppr = sv.ppr;
    h->t_cap = sv.tcap; h->d_cap = sv.dcap; h->R_max = sv.R_max; h->stream = sv.stream;
    h->gemm_ws = sv.gemm_ws; h->ad_part = sv.ad_part; h->w8_ws = sv.w8_ws; h->sk_ws = sv.sk_ws;
  };
  try {
    CK(cudaSetDevice(h->device));
    const bool target = role == SPECDEC_TARGET;
    if (role != SPECDEC_TARGET && role != SPECDEC_DRAFT) fail(SPECDEC_ERR_INVALID, "unknown role");
    ModelW &m = target ? h->tgt : h->dft;
    if (!m.loaded) fail(SPECDEC_ERR_STATE, "weights not loaded");
    if (!d_tokens || !d_logits) fail(SPECDEC_ERR_INVALID, "null device buffer");
    const Dims &dm = m.dm;
    // NCCL may allocate on first use and its collectives need every rank in
    // lockstep: tensor-parallel handles have no allocation-free forward
    if (h->tp_world > 1) fail(SPECDEC_ERR_UNSUPPORTED, "the no-allocation forward does not run on tensor-parallel handles");
    // the model's own capacity (the reference throws past max_seq_len,
    // src/nn/layer.cpp:1176-1179); learned position tables end there
    if (S < 1 || S > dm.max_seq) fail(SPECDEC_ERR_SEQ_LEN, "Sequence length S plus past cached length exceeds max_seq_len");
    const size_t act = h->act_elt;
    const bool kv8 = h->cfg.kv_dtype == SPECDEC_INT8;
    const size_t kv_elt = kv8 ? 1 : h->cfg.kv_dtype == SPECDEC_BF16 ? 2 : 4;
    const int np = (S + kKvPage - 1) / kKvPage;
    auto layout = [&](ArenaCarver &c, void **ptrs) {
      const size_t rows_d = static_cast<size_t>(S) * dm.d * act;
      ptrs[0] = c.take(rows_d);                                // X
      ptrs[1] = c.take(rows_d);                                // H
      ptrs[2] = c.take(rows_d);                                // X1
      ptrs[3] = c.take(static_cast<size_t>(S) * dm.F * act);   // A
      ptrs[4] = c.take(rows_d);                                // Q
      ptrs[5] = c.take(rows_d);                                // ATT
      // one request's cache: pages 0 .. np-1 of a scratch pool
      const size_t kv = static_cast<size_t>(std::max(1, dm.L)) * np * dm.Hkv * kKvPage * dm.D * kv_elt;
      ptrs[6] = c.take(kv);                                    // K cache
      ptrs[7] = c.take(kv);                                    // V cache
      ptrs[8] = c.take(S * sizeof(int));                       // row tokens
      ptrs[9] = c.take(S * sizeof(int));                       // row positions
      ptrs[10] = c.take(S * sizeof(int));                      // row requests
      ptrs[11] = c.take(sizeof(int));                          // error word
      const size_t nsc = kv8 ? static_cast<size_t>(std::max(1, dm.L)) * np * dm.Hkv * kKvPage : 0;
      ptrs[12] = c.take(nsc * sizeof(float));                  // int8 cache: K scales
      ptrs[13] = c.take(nsc * sizeof(float));                  // int8 cache: V scales
      ptrs[14] = c.take(kv8 ? static_cast<size_t>(S) * 2 * dm.kvd * sizeof(float) : 0);  // int8 cache: staged rows
      ptrs[15] = c.take(np * sizeof(int));                     // page table of slot 0
    };
    void *ptrs[16];
    ArenaCarver sizing{nullptr};
    layout(sizing, ptrs);
    if (sizing.used > SPECDEC_NOALLOC_SCRATCH_BYTES)
      fail(SPECDEC_ERR_INVALID, "this forward needs " + std::to_string(sizing.used) +
                                    " bytes of scratch; the no-allocation path holds at most " +
                                    std::to_string(static_cast<size_t>(SPECDEC_NOALLOC_SCRATCH_BYTES)));
    unsigned char *base = nullptr;
    CK(noalloc_base(h->device, &base));
    ArenaCarver arena{base};
    layout(arena, ptrs);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : h->stream;
    h->X = ptrs[0]; h->H = ptrs[1]; h->X1 = ptrs[2]; h->A = ptrs[3]; h->Q = ptrs[4]; h->ATT = ptrs[5];
    if (target) { h->tk = ptrs[6]; h->tv = ptrs[7]; } else { h->dk = ptrs[6]; h->dv = ptrs[7]; }
    if (target) { h->tks = static_cast<float *>(ptrs[12]); h->tvs = static_cast<float *>(ptrs[13]); }
    else { h->dks = static_cast<float *>(ptrs[12]); h->dvs = static_cast<float *>(ptrs[13]); }
    h->KVN = static_cast<float *>(ptrs[14]);
    h->pool.tok = static_cast<int *>(ptrs[8]);
    h->pool.pos = static_cast<int *>(ptrs[9]);
    h->pool.req = static_cast<int *>(ptrs[10]);
    h->st.err = static_cast<int *>(ptrs[11]);
    const size_t layer_elems = static_cast<size_t>(np) * dm.Hkv * kKvPage * dm.D;
    if (target) { h->t_layer_stride = layer_elems; h->t_cap = S; }
    else { h->d_layer_stride = layer_elems; h->d_cap = S; }
    h->d_pt = static_cast<int *>(ptrs[15]);
    h->ppr = np;
    h->R_max = S;
    h->stream = st;
    // the handle's split-K workspace and decode-attention partials belong to
    // its own stream: this call uses neither (no split-K, no split attention)
    h->gemm_ws = nullptr;
    h->ad_part = nullptr;
    h->w8_ws = nullptr;
    h->sk_ws = nullptr;
    CK(cudaMemsetAsync(h->st.err, 0, sizeof(int), st));
    // The tensor-core attention multiplies whole 128-position tiles, the
    // rows past S with probability 0: they must hold finite values, and the
    // scratch array holds whatever an earlier call left there.
    {
      const size_t kv = static_cast<size_t>(std::max(1, dm.L)) * np * dm.Hkv * kKvPage * dm.D * kv_elt;
      CK(cudaMemsetAsync(ptrs[6], 0, kv, st));
      CK(cudaMemsetAsync(ptrs[7], 0, kv, st));
    }
    launch(h, page_iota_kernel, dim3(1), dim3(128), 0, h->d_pt, np);
    launch(h, plan_prefill_kernel, dim3((S + 255) / 256), dim3(256), 0, d_tokens, 1, S, 0, S, dm.V, h->pool.tok,
           h->pool.pos, h->pool.req, static_cast<int *>(nullptr));
    forward_rows(h, target, 0, S, S, nullptr, S, d_logits);
    // the device-side status (bounded waits that gave up, cache rows out of
    // range) for callers that cannot synchronise here
    if (d_status) launch(h, copy_status_kernel, dim3(1), dim3(1), 0, static_cast<const int *>(h->st.err), d_status);
    restore();
  } catch (const SpecErr &e) {
    restore();
    h->err = e.msg;
    return e.code;
  }
  return SPECDEC_OK;
}
