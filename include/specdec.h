/*
 * specdec.h — C ABI of the B200 (sm_100a) speculative-decoding backend for
 * islhkafaa/neural-network.
 *
 * The reference runs speculative decoding as one C++ method,
 * TransformerDecoder::generate_speculative (src/nn/layer.cpp:1382-1661,
 * declared include/nn/layer.hpp:318-323), on two TransformerDecoder objects
 * (target and draft) whose weights live behind the ExecutionBackend interface
 * (include/backend/backend.hpp:20-221).  Most of that path bypasses the
 * backend (RoPE, KV append/truncate, attention, sampling are host loops), so
 * this library replaces the whole method rather than individual backend
 * virtuals.  The entry points below are what the reference-side glue binds;
 * the C++ call site is a
 * CudaSpecBackend class beside the reference.
 *
 * Conventions: plain pointers and sizes only; every function returns a
 * specdec_status (0 = success).  On failure specdec_last_error(handle) holds
 * a one-line message.  The reference reports the same conditions as
 * std::runtime_error; the C++ glue rethrows them as such.  A handle is bound
 * to one device and must be used from one host thread at a time (the
 * reference is not thread-safe either: its AMPContext is thread-local and its
 * ThreadPool a process singleton, src/optim/grad_scaler.cpp:4-5,
 * src/backend/thread_pool.cpp:4-7).
 */
#ifndef SPECDEC_H
#define SPECDEC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum specdec_status {
  SPECDEC_OK = 0,
  SPECDEC_ERR_INVALID = 1,     /* bad argument or shape (reference: shape checks throw, src/core/tensor.cpp:393-402) */
  SPECDEC_ERR_CUDA = 2,        /* a CUDA runtime call failed */
  SPECDEC_ERR_OOM = 3,         /* device allocation failed */
  SPECDEC_ERR_SEQ_LEN = 4,     /* a cache would exceed its capacity (reference: src/nn/layer.cpp:1176-1179) */
  SPECDEC_ERR_UNSUPPORTED = 5, /* a mode this build does not implement */
  SPECDEC_ERR_STATE = 6,       /* call order (e.g. generate before both models are loaded) */
  SPECDEC_ERR_RNG = 7          /* the host uniform table has too few rounds */
} specdec_status;

enum { SPECDEC_ARCH_REF = 0,   /* the reference TransformerDecoder: post-LN, SwiGLU, RoPE (src/nn/layer.cpp:1097-1114) */
       SPECDEC_ARCH_CFG = 1 }; /* pre-LN, GELU FFN, learned positions, final LN (no reference counterpart) */

enum { SPECDEC_F32 = 0, SPECDEC_BF16 = 1, SPECDEC_INT8 = 2 };

enum { SPECDEC_TARGET = 0, SPECDEC_DRAFT = 1 };

enum { SPECDEC_RNG_MT19937 = 0,      /* the reference's std::mt19937(seed) stream, per request seed + b */
       SPECDEC_RNG_HOST_UNIFORM = 1 }; /* caller table u[b][round][2k+1] */

enum { SPECDEC_CATCHUP_REF = 0,      /* the reference's draft catch-up (src/nn/layer.cpp:1632-1655) */
       SPECDEC_CATCHUP_CORRECT = 1 };/* consistent draft rollback */

/* Constructor arguments of TransformerDecoder (include/nn/layer.hpp:301-303)
 * plus the number of KV heads of MultiHeadAttention (layer.hpp:238-240). */
typedef struct specdec_model_config {
  int32_t vocab_size;
  int32_t d_model;
  int32_t n_heads;
  int32_t n_kv_heads;  /* 0 -> n_heads */
  int32_t d_ff;
  int32_t n_layers;
  int32_t max_seq_len; /* per-request KV capacity in positions */
  int32_t arch;        /* SPECDEC_ARCH_* */
} specdec_model_config;

typedef struct specdec_config {
  specdec_model_config target;
  specdec_model_config draft;      /* when draft_shares_target, only draft.n_layers is read */
  int32_t draft_shares_target;     /* 1: draft = target's first draft.n_layers layers + its lm_head, same device memory */
  int32_t weight_dtype;            /* SPECDEC_F32 or SPECDEC_INT8 (QuantizedDense, src/nn/quantization.cpp:7-66) */
  int32_t act_dtype;               /* SPECDEC_F32 or SPECDEC_BF16 */
  int32_t kv_dtype;                /* SPECDEC_F32, SPECDEC_BF16 or SPECDEC_INT8 (quantize_kv, src/nn/layer.cpp:635-665) */
  int32_t max_batch;               /* concurrent requests per generate call */
  int32_t max_lookahead;           /* largest k */
  int32_t max_prompt_len;          /* longest prompt */
  int32_t max_tree_nodes;          /* 0: no token trees; else the largest tree (<= 64 nodes) specdec_generate_tree accepts */
  int32_t kv_pages;                /* paged KV cache: pages of 128 positions in each model's pool (the reference's
                                      KVCache, include/nn/layer.hpp:212-230, grows one request's cache by copying);
                                      0 -> max_batch x ceil(max_seq_len / 128).  A call takes the pages its requests
                                      can reach (prompt + new tokens + one verify block, plus max_new
                                      for the draft's drift under SPECDEC_CATCHUP_REF) and returns SPECDEC_ERR_OOM
                                      when the pool is too small */
} specdec_config;

/* The arguments of generate_speculative (include/nn/layer.hpp:318-323) plus
 * the switches the batched B200 path adds. */
typedef struct specdec_gen_params {
  int32_t max_new_tokens;          /* as the reference: at least one token is always emitted */
  int32_t lookahead;               /* k */
  float temperature;               /* <= 0: greedy */
  int32_t top_k;                   /* 0: off */
  float top_p;                     /* >= 1: off */
  int32_t rng_mode;                /* SPECDEC_RNG_* */
  uint32_t seed;                   /* mt19937 mode: request b uses seed + b */
  const float *uniforms;           /* host-uniform mode: [B][uniform_rounds][2k+1] in [0,1) */
  int32_t uniform_rounds;
  int32_t draft_catchup;           /* SPECDEC_CATCHUP_* */
} specdec_gen_params;

typedef struct specdec_handle specdec_handle;

/* Replaces constructing the two TransformerDecoder objects on a backend
 * (include/nn/layer.hpp:301-303). Allocates all device memory up front. */
int specdec_create(const specdec_config *cfg, int device, specdec_handle **out);

int specdec_destroy(specdec_handle *h);

/* Last error message of this handle (or of the last failed create if h is NULL). */
const char *specdec_last_error(const specdec_handle *h);

/* Replaces injecting weights through TransformerDecoder::parameters() +
 * Tensor::copy_from_host (include/nn/layer.hpp:306, tests/nn/gqa_test.cpp:56-62).
 * params[i] is a host fp32 array of numels[i] elements, in parameters() order;
 * Dense weights are [in, out] row-major (src/nn/layer.cpp:153).  With
 * weight_dtype INT8 every Dense weight (attention, FFN, lm_head) is quantised
 * on load exactly as QuantizedDense does.  role = SPECDEC_DRAFT is rejected
 * when draft_shares_target. */
int specdec_load_params(specdec_handle *h, int role, int n_params,
                        const float *const *params, const int64_t *numels);

/* specdec_load_params with DEVICE arrays (params[i] points to device memory
 * on this handle's device; the pointer array itself is on the host): the int8
 * scales, the quantisation and the transpose run on the device, so a model
 * that already lives there (a checkpoint loaded by another runtime, weights
 * drawn on the GPU) never passes through host memory.  The same weights give
 * the same device parameters as specdec_load_params. */
int specdec_load_params_device(specdec_handle *h, int role, int n_params,
                               const float *const *params, const int64_t *numels);

/* Replaces Layer::load_weights (src/nn/layer.cpp:467-469 ->
 * serialization::load_parameters, src/core/serialization.cpp:49-107) on the
 * model of `role`: reads a NETW version-1 file (magic "NETW", u16 version,
 * u32 tensor count, per tensor u32 dims, u64 shape, u64 element count,
 * float32 data) whose tensors are the model's parameters() in order and
 * shape, then loads them as specdec_load_params does.  A wrong signature,
 * version, count, rank, shape or element count fails with
 * SPECDEC_ERR_INVALID and the reference's message. */
int specdec_load_netw(specdec_handle *h, int role, const char *path);

/* Replaces TransformerDecoder::generate_speculative (src/nn/layer.cpp:1382-1661)
 * for B independent requests with equal prompt length S.  prompts [B][S] and
 * out_tokens [B][S + max(1, max_new_tokens)] are HOST buffers (the tokens are
 * the reference's return value: prompt followed by the new tokens).
 * out_stats (optional) [B][4] = rounds, drafted tokens, accepted drafts,
 * rejections. */
int specdec_generate(specdec_handle *h, const specdec_gen_params *p,
                     const int32_t *prompts, int B, int S,
                     int32_t *out_tokens, int64_t *out_stats);

/* The same with DEVICE buffers (no host copies, nothing synchronised): the
 * caller times it on specdec_stream(h).  out_stats is a device int64 [B][4]. */
int specdec_generate_device(specdec_handle *h, const specdec_gen_params *p,
                            const int32_t *d_prompts, int B, int S,
                            int32_t *d_out_tokens, int64_t *d_out_stats);

/* Round-level session: generate_speculative split at its round loop
 * (src/nn/layer.cpp:1514-1656), so a caller (a serving loop, a benchmark)
 * drives rounds itself.  specdec_prefill runs everything up to and including
 * the first token (src/nn/layer.cpp:1396-1512: target and draft prefill, the
 * first sample) for B requests with equal prompt length S (prompts [B][S],
 * HOST) and opens a session on the handle; specdec_generate* and loading
 * weights close it.  Chain speculation only (no trees, no autoregressive
 * mode).  In host-uniform mode the session's table holds
 * max(uniform_rounds, max_new_tokens + 2) rounds: p->uniforms fills its first
 * uniform_rounds rows (row 0 draws the first token), the rest start at 0 and
 * may be supplied by the steps. */
int specdec_prefill(specdec_handle *h, const specdec_gen_params *p,
                    const int32_t *prompts, int B, int S);

/* specdec_prefill with a DEVICE prompt buffer, enqueued on specdec_stream(h)
 * (nothing synchronised, no device-side status). */
int specdec_prefill_device(specdec_handle *h, const specdec_gen_params *p,
                           const int32_t *d_prompts, int B, int S);

/* Up to `rounds` speculative rounds (k draft steps, one verify pass,
 * acceptance and rollback each; src/nn/layer.cpp:1514-1656) of the open
 * session; it stops early once every request has its max_new_tokens.
 * `uniforms` (optional, HOST; host-uniform sessions only) are these rounds'
 * draws [B][rounds][2k+1] and replace the table rows of the rounds about to
 * run.  out_tokens [B][rounds * (k + 1)] and out_counts [B] are HOST
 * buffers: request b emitted out_counts[b] tokens in this call, in
 * out_tokens[b][0 .. out_counts[b]).  Synchronises and reports device-side
 * errors like specdec_generate. */
int specdec_step(specdec_handle *h, int rounds, const float *uniforms,
                 int32_t *out_tokens, int32_t *out_counts);

/* specdec_step on DEVICE output buffers (d_out_tokens [B][cap], at most cap
 * tokens per request are stored; d_out_counts [B] counts them all), enqueued
 * on specdec_stream(h) with nothing synchronised.  `uniforms` may be a host or
 * device pointer. */
int specdec_step_device(specdec_handle *h, int rounds, const float *uniforms,
                        int32_t *d_out_tokens, int32_t *d_out_counts, int cap);

/* The open session's sequences so far (HOST out_tokens [B][S +
 * max(1, max_new_tokens)], prompt then new tokens, unfilled tail
 * unspecified) and statistics (optional HOST out_stats [B][4], as
 * specdec_generate). */
int specdec_session_tokens(specdec_handle *h, int32_t *out_tokens, int64_t *out_stats);

/* Replaces TransformerDecoder::generate_advanced with use_kv_cache = true
 * (src/nn/layer.cpp:1239-1380) for B independent requests: target only (the
 * draft need not be loaded), one token per request and step.  Greedy when
 * temperature <= 0 (first maximum); else get_probs (temperature, top_k,
 * top_p) and one draw per token from request b's mt19937(seed + b) stream,
 * or from u[b][step][0] of a host table with uniform_rounds >= max_new_tokens
 * rows of one slot.  lookahead and draft_catchup are not used.  prompts
 * [B][S] and out_tokens [B][S + max_new_tokens] are HOST buffers;
 * out_stats (optional) [B][4] = steps, 0, 0, 0.  The cache ends at
 * S + max_new_tokens - 1 positions (SPECDEC_ERR_SEQ_LEN beyond the target's
 * max_seq_len, as src/nn/layer.cpp:1176-1179 throws). */
int specdec_generate_ar(specdec_handle *h, const specdec_gen_params *p,
                        const int32_t *prompts, int B, int S,
                        int32_t *out_tokens, int64_t *out_stats);

/* specdec_generate_ar on DEVICE buffers, enqueued on specdec_stream(h)
 * (nothing synchronised).  out_tokens [B][S + max(1, max_new_tokens)]. */
int specdec_generate_ar_device(specdec_handle *h, const specdec_gen_params *p,
                               const int32_t *d_prompts, int B, int S,
                               int32_t *d_out_tokens, int64_t *d_out_stats);

/* The CUDA stream (cudaStream_t) every kernel of this handle runs on. */
void *specdec_stream(specdec_handle *h);

/* TransformerDecoder::forward without a cache (src/nn/layer.cpp:1161-1193) of
 * one model on one host token sequence; logits [S][vocab] fp32, host. */
int specdec_forward_logits(specdec_handle *h, int role, const int32_t *tokens,
                           int S, float *logits);

/* Philox4x32-10 uniform table u[b][round][slot] for SPECDEC_RNG_HOST_UNIFORM:
 * key (seed lo, seed hi), counter (slot/4, round, b, 0x53504543), lane slot%4,
 * value (x >> 8) * 2^-24. */
int specdec_philox_uniforms(uint64_t seed, int B, int rounds, int slots,
                            float *out);

/* No counterpart in the reference.  The forward of specdec_forward_logits for
 * callers that cannot allocate device memory when they need it: code running
 * inside another runtime's memory pool, latency-critical loops where an
 * allocation may stall the device, or a shared context that must not grow.
 * d_tokens [S] int32 and d_logits [S][vocab] fp32 are DEVICE buffers the caller
 * owns; the call is asynchronous on `stream` (a cudaStream_t; NULL selects
 * specdec_stream(h)).  Every byte of working memory (activations, row tables,
 * the sequence's KV cache and its int8 scales) comes from one fixed 8 MiB
 * device array inside the library; work that needs more is rejected with
 * SPECDEC_ERR_INVALID.  No cudaMalloc, cudaFree or other allocating call is
 * made.  The array is shared by all calls on a device and keeps the last
 * call's contents: calls that overlap on the GPU race and must be serialised
 * by the caller, and so must a call that overlaps other work of the same
 * handle on another stream (both read the handle's weights; this call leaves
 * the handle's own workspaces alone).  The first call on each device looks
 * the array's address up (that device current); make it before any stream
 * capture begins.  S is at most the model's max_seq_len
 * (SPECDEC_ERR_SEQ_LEN, as the reference throws, src/nn/layer.cpp:1176-1179).
 * Tensor-parallel handles are rejected (SPECDEC_ERR_UNSUPPORTED): NCCL may
 * allocate and needs every rank.  Device-side failures (a bounded wait that
 * gave up, a cache row out of range) cannot be returned by an asynchronous
 * call: when d_status (a caller-owned DEVICE int32, may be NULL) is given,
 * the call's last kernel writes the error bits there (0 = none; 1 = cache
 * capacity, 4 = a wait gave up) for the caller to read after it synchronises. */
int specdec_forward_logits_noalloc(specdec_handle *h, int role,
                                   const int32_t *d_tokens, int S,
                                   float *d_logits, void *stream, int32_t *d_status);

/* Token tree of specdec_generate_tree: `depth` levels (1..8), every node at
 * depth t < depth has branch[t] children (the draft's most likely next
 * tokens); at most max_tree_nodes nodes in all (config 4: depth 4, branching
 * 4, 3, 2, 1 = 64 nodes). */
typedef struct specdec_tree {
  int32_t depth;
  int32_t branch[8];
} specdec_tree;

/* Tree speculation (no counterpart in the reference, which drafts one chain;
 * this is generate_speculative with a token tree per round): the draft
 * expands `tree` level by level, the target verifies all nodes in one pass
 * with an ancestor mask, and acceptance walks the tree trying each node's
 * children in order as point-mass proposals (greedy: the child equal to the
 * target's argmax; sampled: child c with probability p(c), p renormalised
 * without c after each rejection), which keeps the target's distribution.
 * Same buffers and statuses as specdec_generate; `lookahead` and
 * `draft_catchup` are not used; host-uniform tables have depth * max(branch)
 * + 1 slots per round (slot t * max(branch) + r tests child r at depth t, the
 * last slot draws the emitted token; round 0's last slot the first token).
 * out_stats per request: rounds, tree nodes drafted, accepted, rejections. */
int specdec_generate_tree(specdec_handle *h, const specdec_gen_params *p, const specdec_tree *tree,
                          const int32_t *prompts, int B, int S, int32_t *out_tokens, int64_t *out_stats);

/* specdec_generate_tree on device buffers, enqueued on specdec_stream(h)
 * like specdec_generate_device (no synchronisation, no status from the
 * device side: read the statistics to check). */
int specdec_generate_tree_device(specdec_handle *h, const specdec_gen_params *p, const specdec_tree *tree,
                                 const int32_t *d_prompts, int B, int S, int32_t *d_out_tokens,
                                 int64_t *d_out_stats);

/* Number of kernel launches the last generate call issued on the device. */
int64_t specdec_last_launch_count(const specdec_handle *h);

/* Tensor parallelism (the large configuration's variant; no counterpart in
 * the reference, which runs on one device): `world` handles, one per GPU and
 * process (or thread), each created with its rank and the same 128-byte NCCL
 * unique id, which one rank makes with specdec_tp_unique_id and hands to the
 * others.  Every rank loads the whole model's parameters; each keeps its
 * share of the attention heads (and their KV cache) and of the FFN columns,
 * and the attention output and FFN down projections end in an NCCL
 * all-reduce (sum) over NVLink.  Embedding, LayerNorm, lm_head and sampling
 * are replicated, and every rank returns the same tokens.  All ranks must
 * make the same calls in the same order.  Heads, kv heads and d_ff must
 * divide by `world`.  NCCL (libnccl.so.2) is loaded on first use. */
int specdec_tp_unique_id(void *out128);
int specdec_create_tp(const specdec_config *cfg, int device, int rank, int world, const void *unique_id,
                      specdec_handle **out);

/* Which linear layer specdec_time_linear launches. */
enum specdec_linear {
  SPECDEC_LIN_QKV = 0,     /* fused q/k/v projection (+ RoPE, cache append) */
  SPECDEC_LIN_OPROJ = 1,   /* attention output projection + residual */
  SPECDEC_LIN_FFN_IN = 2,  /* SwiGLU gate/up (arch ref) or fc1 + GELU (arch cfg), with its LayerNorm */
  SPECDEC_LIN_FFN_OUT = 3, /* down / fc2 + residual */
  SPECDEC_LIN_HEAD = 4     /* lm_head over normalised rows */
};

/* Measurement probe (no counterpart in the reference): launches the kernel of
 * one linear layer of `role` exactly as a forward pass over `rows` rows builds
 * it, `reps` times on specdec_stream(h), each launch alone between CUDA
 * events with the L2 cache flushed before it by writing `flush_bytes` of the
 * caller's device buffer `flush`.  Writes the mean launch time in
 * microseconds and the launch's algorithmic bytes (weights, scales, biases,
 * LayerNorm parameters, input and output rows).  Overwrites activation
 * buffers; a QKV launch writes no cache rows (its rows are marked unused). */
int specdec_time_linear(specdec_handle *h, int role, int layer, int which, int rows, int reps,
                        void *flush, size_t flush_bytes, float *avg_us, double *alg_bytes);

/* Measurement probe (no counterpart in the reference): launches the
 * attention of `layer` of `role` as a pass of q_per_req rows per request over
 * the open session's caches builds it (request b's rows are its last
 * q_per_req cached positions), `reps` times on specdec_stream(h), each launch
 * alone between CUDA events after the caller's flush buffer is written.
 * Writes the mean launch time in microseconds and the launch's algorithmic
 * bytes (every visible K and V row once, int8 scales, query rows in, output
 * rows out).  Overwrites the prefill row table and activation buffers only. */
int specdec_time_attention(specdec_handle *h, int role, int layer, int q_per_req, int reps, void *flush,
                           size_t flush_bytes, float *avg_us, double *alg_bytes);

#ifdef __cplusplus
}
#endif

#endif /* SPECDEC_H */
