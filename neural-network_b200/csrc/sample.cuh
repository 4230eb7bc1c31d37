// Sampling, acceptance and bookkeeping kernels of the speculative-decoding
// round (TransformerDecoder::generate_speculative, src/nn/layer.cpp:1382-1661).
//
// Per-request state lives on the device, so a whole round (draft steps,
// verify, accept, rollback) runs without a host round trip and can be
// captured in a CUDA graph.  Row planning kernels turn the state into the row
// batches the forward kernels consume.
#pragma once

#include <cooperative_groups.h>

#include "common.cuh"
#include "forward.cuh"

namespace specdec {

// ---------------------------------------------------------------------------
// MT19937 (Matsumoto & Nishimura, ACM TOMACS 1998), the engine behind the
// reference's std::mt19937 (src/nn/layer.cpp:1394).  Parameters of the
// published generator: n = 624, m = 397, a = 0x9908b0df, tempering
// (11, 7 / 0x9d2c5680, 15 / 0xefc60000, 18).
constexpr int kMtN = 624;
constexpr int kMtM = 397;

__device__ __forceinline__ uint32_t mt_temper(uint32_t y) {
  y ^= y >> 11;
  y ^= (y << 7) & 0x9d2c5680u;
  y ^= (y << 15) & 0xefc60000u;
  y ^= y >> 18;
  return y;
}

__device__ __forceinline__ uint32_t mt_mix(uint32_t cur, uint32_t next, uint32_t far) {
  const uint32_t y = (cur & 0x80000000u) | (next & 0x7fffffffu);
  return far ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
}

// One regeneration of the 624-word state, block-cooperative.  Sequentially,
// word i is rebuilt from old[i], old[i+1] and word (i+397) mod 624, which is
// still old for i < 227 and already rebuilt for i >= 227; word 623 pairs with
// the rebuilt word 0.  That gives four dependency phases.
__device__ void mt_twist_block(const uint32_t *old, uint32_t *nw) {
  for (int i = threadIdx.x; i < kMtN - kMtM; i += blockDim.x) nw[i] = mt_mix(old[i], old[i + 1], old[i + kMtM]);
  __syncthreads();
  for (int i = kMtN - kMtM + threadIdx.x; i < 2 * (kMtN - kMtM); i += blockDim.x)
    nw[i] = mt_mix(old[i], old[i + 1], nw[i - (kMtN - kMtM)]);
  __syncthreads();
  for (int i = 2 * (kMtN - kMtM) + threadIdx.x; i < kMtN - 1; i += blockDim.x)
    nw[i] = mt_mix(old[i], old[i + 1], nw[i - (kMtN - kMtM)]);
  __syncthreads();
  if (threadIdx.x == 0) nw[kMtN - 1] = mt_mix(old[kMtN - 1], nw[0], nw[kMtM - 1]);
  __syncthreads();
}

// std::generate_canonical<double, 53> over a 32-bit engine: two draws,
// (g1 + g2 * 2^32) / 2^64 with one rounding, clamped below 1.
__device__ __forceinline__ double canon_f64(uint32_t g1, uint32_t g2) {
  double s = __dadd_rn(static_cast<double>(g1), static_cast<double>(g2) * 4294967296.0);
  double r = s * 5.421010862427522e-20;  // 2^-64, exact scaling
  return r >= 1.0 ? 0.99999999999999989 : r;  // nextafter(1, 0)
}
// std::generate_canonical<float, 24>: float(g) (round to nearest) / 2^32.
__device__ __forceinline__ float canon_f32(uint32_t g) {
  float r = __uint2float_rn(g) * 2.3283064365386963e-10f;  // 2^-32
  return r >= 1.0f ? 0.99999994f : r;
}

// ---------------------------------------------------------------------------
// Row tables: one pool of (token, position, request) triples with fixed
// regions for the prefill chunk, draft step 0 (two rows per request: the
// catch-up token and the last token), draft steps 1..k-1 (one row per
// request) and the verify block (k+1 rows per request).  The sampling kernels
// write the rows of the next forward pass directly, so no planning kernel
// runs between them.
struct RowPool {
  int *tok, *pos, *req;
  int off_step0, off_step1, off_verify;  // region offsets (the prefill region is at 0)
  // token trees: per-row cache slot, tree base and ancestor mask, and the
  // regions of the tree levels 1 .. depth-1 (draft) and of the tree verify block
  int *slot, *tb;
  unsigned long long *mask;
  int off_tlevel[9], off_tverify;
};

constexpr int kTreeMaxDepth = 8;
constexpr int kTreeMaxNodes = 64;  // one bit per node in a row's ancestor mask

struct SpecState {
  int *tokens_out;     // [B][out_len]
  int out_len;
  int prompt_len;
  int *n_new;          // [B]
  int *t_len, *d_len;  // cache lengths
  int *t_start, *d_start;
  int *last_tok, *active, *M;
  int *cand;           // [B][kmax]
  float *q;            // [B][kmax][V] draft probabilities
  long long *stats;    // [B][4]
  int *round;          // [B]
  uint32_t *mt;        // [B][624]
  int *mt_idx;         // [B]
  int *active_count;
  int *err;
  RowPool rows;
  int B, kmax, V;
  int max_new, k;
  float T;
  int greedy;
  int top_k;           // > 0 and < V: keep the k most probable tokens
  float top_p;         // in (0, 1): keep the smallest descending prefix of mass >= top_p
  int rng_mode;        // 0 mt19937, 1 host table
  const float *uniforms;
  int u_rounds, u_slots;
  int catchup;         // 0 reference, 1 consistent
  int t_cap, d_cap;
  // token trees (tree = 1): depth, branching per level, node count, first node
  // of each depth (tlev[t] = first node at depth t + 1, tlev[depth] = nodes),
  // largest branching; per request the node tokens, the draft cache slot of
  // the round's root and the accepted path handed to the compaction kernel
  int tree, tL, tN, tbmax;
  int tbr[kTreeMaxDepth], tlev[kTreeMaxDepth + 1];
  int *ttok;           // [B][kTreeMaxNodes]
  int *d_root;         // [B]
  int *cp_t0, *cp_d0, *cp_n, *cp_dn;  // [B] root slots and path lengths of the last accept
  int *cp_path;        // [B][kTreeMaxDepth] accepted node indices, root side first
  // autoregressive decoding (ar = 1, k = 0): one target row per request and
  // step at verify_row(b, 0); host-uniform tables have one slot per step
  int ar;
};

// Tree structure (BFS order; the nodes at depth t >= 1 are tlev[t-1] .. tlev[t]-1).
__device__ __forceinline__ int tree_depth_of(const SpecState &st, int j) {
  int t = 1;
  while (t < st.tL && j >= st.tlev[t]) ++t;
  return t;
}
__device__ __forceinline__ int tree_parent(const SpecState &st, int j) {
  const int t = tree_depth_of(st, j);
  return t == 1 ? -1 : st.tlev[t - 2] + (j - st.tlev[t - 1]) / st.tbr[t - 1];
}
__device__ __forceinline__ unsigned long long tree_mask(const SpecState &st, int j) {
  unsigned long long m = 0;
  for (int x = j; x >= 0; x = tree_parent(st, x)) m |= 1ull << x;
  return m;
}
// first child of node j (j < 0: the root) and its depth
__device__ __forceinline__ int tree_first_child(const SpecState &st, int j, int depth) {
  return j < 0 ? 0 : st.tlev[depth] + (j - st.tlev[depth - 1]) * st.tbr[depth];
}

__device__ __forceinline__ void set_row(const SpecState &st, int idx, int tok, int pos, int req) {
  st.rows.tok[idx] = (tok >= 0 && tok < st.V) ? tok : 0;  // an out-of-range id embeds as row 0
  st.rows.pos[idx] = pos;
  st.rows.req[idx] = req;
}
__device__ __forceinline__ void clear_row(const SpecState &st, int idx) { set_row(st, idx, 0, 0, -1); }
__device__ __forceinline__ int step_row(const SpecState &st, int j, int b) {
  return j == 0 ? st.rows.off_step0 + 2 * b + 1 : st.rows.off_step1 + (j - 1) * st.B + b;
}
__device__ __forceinline__ int verify_row(const SpecState &st, int b, int i) {
  return st.rows.off_verify + b * (st.k + 1) + i;
}

// Every row of request b unused (the request finished or failed).
__device__ void clear_request_rows(const SpecState &st, int b) {
  clear_row(st, st.rows.off_step0 + 2 * b);
  clear_row(st, st.rows.off_step0 + 2 * b + 1);
  for (int j = 1; j < st.k; ++j) clear_row(st, step_row(st, j, b));
  for (int i = 0; i <= st.k; ++i) clear_row(st, verify_row(st, b, i));
}

// Draft step 0 rows of the coming round: [catch-up (if any), last token].
// Folding the reference's post-round draft catch-up forward
// (src/nn/layer.cpp:1639-1642, 1649-1653) into the next round's first draft
// step computes the same cache and the same logits for the last row.  Returns
// false (and flags the error) when the round would overflow a cache.
// start_round_at takes the request's n_new, d_len, t_len and last token as
// read by the caller.
__device__ bool start_round_at(const SpecState &st, int b, int catch_tok, int n_new, int d, int t_len, int last_tok) {
  const int M = min(st.k, st.max_new - n_new);
  const int has_c = catch_tok >= 0 ? 1 : 0;
  if (d + has_c + M > st.d_cap || t_len + M + 1 > st.t_cap) {
    atomicOr(st.err, kErrSeqLen);
    st.active[b] = 0;
    clear_request_rows(st, b);
    return false;
  }
  if (has_c) set_row(st, st.rows.off_step0 + 2 * b, catch_tok, d++, b);
  else clear_row(st, st.rows.off_step0 + 2 * b);
  st.d_start[b] = d;
  set_row(st, st.rows.off_step0 + 2 * b + 1, last_tok, d, b);
  st.d_len[b] = d + 1;
  st.M[b] = M;
  return true;
}
__device__ bool start_round(const SpecState &st, int b, int catch_tok) {
  return start_round_at(st, b, catch_tok, st.n_new[b], st.d_len[b], st.t_len[b], st.last_tok[b]);
}

__device__ __forceinline__ void set_tree_row(const SpecState &st, int idx, int tok, int pos, int req, int slot, int tb,
                                             unsigned long long mask) {
  set_row(st, idx, tok, pos, req);
  st.rows.slot[idx] = slot;
  st.rows.tb[idx] = tb;
  st.rows.mask[idx] = mask;
}
__device__ __forceinline__ int tree_verify_row(const SpecState &st, int b, int i) {
  return st.rows.off_tverify + b * (st.tN + 1) + i;  // i = 0: the root, 1 + j: node j
}
__device__ __forceinline__ int tree_level_row(const SpecState &st, int b, int depth, int i) {
  const int n = st.tlev[depth] - st.tlev[depth - 1];
  return st.rows.off_tlevel[depth] + b * n + i;
}
__device__ void tree_clear_rows(const SpecState &st, int b) {
  clear_row(st, st.rows.off_step0 + 2 * b);
  clear_row(st, st.rows.off_step0 + 2 * b + 1);
  for (int t = 1; t < st.tL; ++t)
    for (int i = 0; i < st.tlev[t] - st.tlev[t - 1]; ++i) clear_row(st, tree_level_row(st, b, t, i));
  for (int i = 0; i <= st.tN; ++i) clear_row(st, tree_verify_row(st, b, i));
}

// Rows of a tree round's first draft pass, [catch-up (if any), root], and the
// root row of the verify block; the tree's rows follow as the draft expands.
// Returns false (and flags the error) when the tree would not fit a cache.
__device__ bool tree_start_round(const SpecState &st, int b, int catch_tok) {
  int d = st.d_len[b];
  const int t = st.t_len[b];
  const int has_c = catch_tok >= 0 ? 1 : 0;
  const int draft_nodes = st.tL > 1 ? st.tlev[st.tL - 1] : 0;  // leaves are not fed to the draft
  if (d + has_c + 1 + draft_nodes > st.d_cap || t + 1 + st.tN > st.t_cap) {
    atomicOr(st.err, kErrSeqLen);
    st.active[b] = 0;
    tree_clear_rows(st, b);
    return false;
  }
  if (has_c) set_row(st, st.rows.off_step0 + 2 * b, catch_tok, d++, b);
  else clear_row(st, st.rows.off_step0 + 2 * b);
  set_row(st, st.rows.off_step0 + 2 * b + 1, st.last_tok[b], d, b);
  st.d_root[b] = d;
  st.d_len[b] = d + 1;
  st.t_start[b] = t;
  set_tree_row(st, tree_verify_row(st, b, 0), st.last_tok[b], t, b, t, t + 1, 0ull);
  return true;
}

struct RngCtx {
  uint32_t *old_s, *new_s;  // shared [624] each
  uint32_t *win;            // shared window
  int *used;                // shared counter
  int *twisted;             // shared: new_s holds the regenerated state
};

// Prepares `need` consecutive tempered words of request b's stream in `win`.
// mt_idx = 624 (fresh seed, or every word of the state drawn) regenerates the
// state before the first word, as std::mt19937 does on its next draw.
__device__ void rng_prepare(const SpecState &st, int b, int need, RngCtx &c) {
  if (st.rng_mode != 0) return;
  const int idx = st.mt_idx[b];
  const uint32_t *g = st.mt + static_cast<size_t>(b) * kMtN;
  if (idx + need <= kMtN) {
    for (int t = threadIdx.x; t < need; t += blockDim.x) c.win[t] = mt_temper(g[idx + t]);
  } else {
    for (int t = threadIdx.x; t < kMtN; t += blockDim.x) c.old_s[t] = g[t];
    __syncthreads();
    mt_twist_block(c.old_s, c.new_s);
    const int rem = kMtN - idx;
    for (int t = threadIdx.x; t < need; t += blockDim.x)
      c.win[t] = mt_temper(t < rem ? c.old_s[idx + t] : c.new_s[t - rem]);
  }
  if (threadIdx.x == 0) {
    *c.used = 0;
    *c.twisted = idx + need > kMtN ? 1 : 0;
  }
  __syncthreads();
}

__device__ void rng_commit(const SpecState &st, int b, RngCtx &c) {
  if (st.rng_mode != 0) return;
  __syncthreads();
  const int idx = st.mt_idx[b] + *c.used;
  const bool wrap = idx >= kMtN && *c.twisted;  // the draws reached the regenerated state
  __syncthreads();
  if (wrap) {
    uint32_t *g = st.mt + static_cast<size_t>(b) * kMtN;
    for (int t = threadIdx.x; t < kMtN; t += blockDim.x) g[t] = c.new_s[t];
  }
  // without a regeneration the index stops at 624 at most (state used up)
  if (threadIdx.x == 0) st.mt_idx[b] = wrap ? idx - kMtN : idx;
}

__device__ __forceinline__ double table_u(const SpecState &st, int b, int round, int slot) {
  if (round >= st.u_rounds) {
    atomicOr(st.err, kErrRngTable);
    return 0.5;
  }
  return static_cast<double>(st.uniforms[(static_cast<size_t>(b) * st.u_rounds + round) * st.u_slots + slot]);
}

// Thread 0 only: the uniform for sample_token (discrete_distribution draws a
// 53-bit double) or for the acceptance test (uniform_real_distribution<float>).
__device__ __forceinline__ double draw_sample_u(const SpecState &st, int b, int round, int slot, RngCtx &c) {
  if (st.rng_mode == 0) {
    const int u = *c.used;
    *c.used = u + 2;
    return canon_f64(c.win[u], c.win[u + 1]);
  }
  return table_u(st, b, round, slot);
}
__device__ __forceinline__ float draw_accept_u(const SpecState &st, int b, int round, int slot, RngCtx &c) {
  if (st.rng_mode == 0) {
    const int u = *c.used;
    *c.used = u + 1;
    return canon_f32(c.win[u]);
  }
  return static_cast<float>(table_u(st, b, round, slot));
}

// ---------------------------------------------------------------------------
// The sampling kernels keep the vocabulary row they work on in dynamic shared
// memory (V floats): one coalesced load, then every pass is on-chip.
__device__ void load_row(const float *__restrict__ g, int V, float *srow) {
  if ((V & 3) == 0 && (reinterpret_cast<uintptr_t>(g) & 15) == 0) {
    const float4 *g4 = reinterpret_cast<const float4 *>(g);
    float4 *s4 = reinterpret_cast<float4 *>(srow);
#pragma unroll 4
    for (int v = threadIdx.x; v < V / 4; v += blockDim.x) s4[v] = __ldg(g4 + v);
  } else {
    for (int v = threadIdx.x; v < V; v += blockDim.x) srow[v] = g[v];
  }
  __syncthreads();
}

__device__ void store_row(const float *srow, int V, float *__restrict__ g) {
  if ((V & 3) == 0 && (reinterpret_cast<uintptr_t>(g) & 15) == 0) {
    const float4 *s4 = reinterpret_cast<const float4 *>(srow);
    float4 *g4 = reinterpret_cast<float4 *>(g);
    for (int v = threadIdx.x; v < V / 4; v += blockDim.x) g4[v] = s4[v];
  } else {
    for (int v = threadIdx.x; v < V; v += blockDim.x) g[v] = srow[v];
  }
}

// get_probs for T > 0 without top-k/top-p (src/nn/layer.cpp:1426-1489), in
// place on a shared-memory row: l/T, subtract the max, exp, divide by the
// sum, then divide by the sum of the normalised values (the reference's
// second normalisation, taken there in sorted order).  Max and exp-sum come
// from one pass with a per-thread running maximum.
// Scratch of the top-k / top-p cut.
struct CutShared {
  unsigned int cnt[256];
  unsigned long long mass[256];  // probability mass in units of 2^-40 (exact integer sums)
  unsigned int pfx, above_cnt, eq_cnt;
  unsigned long long above_mass;
  int hit;
};
constexpr double kMassUnit = 1099511627776.0;  // 2^40

__device__ __forceinline__ unsigned long long mass_fixed(float p) {
  return static_cast<unsigned long long>(__double2ull_rn(static_cast<double>(p) * kMassUnit));
}

// Position of the cut in the descending order of the probabilities in srow
// (all >= 0, so their bit patterns order like their values), found by a
// radix descent over the float bits, 8 bits per pass: by count (the target-th
// largest element) or by mass (the element at which the descending running
// sum reaches the target).  On return c.pfx holds the cut value's bits,
// c.above_cnt / c.above_mass the count / mass strictly above it, c.eq_cnt the
// number of elements equal to it; c.hit = 0 when the target is never reached.
__device__ void radix_cut(const float *srow, int V, bool by_mass, unsigned long long target, CutShared &c) {
  if (threadIdx.x == 0) {
    c.pfx = 0;
    c.above_cnt = 0;
    c.above_mass = 0;
    c.hit = 1;
  }
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) {
      c.cnt[i] = 0;
      c.mass[i] = 0;
    }
    __syncthreads();
    const unsigned int pfx = c.pfx;
    const unsigned int hmask = shift == 24 ? 0u : (0xffffffffu << (shift + 8));
    for (int v = threadIdx.x; v < V; v += blockDim.x) {
      const unsigned int bits = __float_as_uint(srow[v]);
      if ((bits & hmask) == pfx) {
        const unsigned int bkt = (bits >> shift) & 255u;
        atomicAdd(&c.cnt[bkt], 1u);
        if (by_mass) atomicAdd(&c.mass[bkt], mass_fixed(srow[v]));
      }
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      // lane l covers buckets 255 - 8l down to 248 - 8l
      const int lane = threadIdx.x;
      unsigned long long lc = 0, lm = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        lc += c.cnt[255 - 8 * lane - j];
        lm += c.mass[255 - 8 * lane - j];
      }
      unsigned long long ic = lc, im = lm;  // inclusive scans in descending bucket order
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long yc = __shfl_up_sync(0xffffffffu, ic, o);
        const unsigned long long ym = __shfl_up_sync(0xffffffffu, im, o);
        if (lane >= o) {
          ic += yc;
          im += ym;
        }
      }
      const unsigned long long bc = c.above_cnt, bm = c.above_mass;
      const bool hit = (by_mass ? bm + im : bc + ic) >= target;
      const unsigned int ballot = __ballot_sync(0xffffffffu, hit);
      const int L = ballot ? __ffs(ballot) - 1 : 31;
      if (lane == L) {
        unsigned long long rc = bc + ic - lc, rm = bm + im - lm;  // above this lane's buckets
        int chosen = 255 - 8 * lane - 7;
        for (int j = 0; j < 8; ++j) {
          const int bkt = 255 - 8 * lane - j;
          if ((by_mass ? rm + c.mass[bkt] : rc + c.cnt[bkt]) >= target) {
            chosen = bkt;
            break;
          }
          rc += c.cnt[bkt];
          rm += c.mass[bkt];
        }
        if (!ballot) c.hit = 0;
        c.pfx = pfx | (static_cast<unsigned int>(chosen) << shift);
        c.above_cnt = static_cast<unsigned int>(rc);
        c.above_mass = rm;
        c.eq_cnt = c.cnt[chosen];
      }
    }
    __syncthreads();
  }
}

// get_probs (src/nn/layer.cpp:1410-1491) for T > 0 on a logits row in
// shared memory: softmax of l / T, then -- when top-k or top-p is active --
// keep the first min(k, m_p) entries of the descending order (m_p = the
// shortest prefix whose running sum reaches top_p) and renormalise by their
// sum; without a filter the second normalisation divides by the total.  Ties
// at the cut keep the lowest token ids (std::sort leaves their order
// unspecified).
__device__ void probs_smem(float *srow, int V, float T, int top_k, float top_p, float *red, CutShared &cut) {
  float mx = -INFINITY, se = 0.f;
  const bool t1 = T == 1.f;
  for (int v = threadIdx.x; v < V; v += blockDim.x) {
    const float x = t1 ? srow[v] : __fdiv_rn(srow[v], T);  // x / 1 is x
    srow[v] = x;
    if (x > mx) {
      se = se * expf(mx - x) + 1.f;
      mx = x;
    } else {
      se += expf(x - mx);
    }
  }
  const float M = block_max(mx, red);
  const float s = block_sum(mx == -INFINITY ? 0.f : se * expf(mx - M), red);
  for (int v = threadIdx.x; v < V; v += blockDim.x) srow[v] = __fdiv_rn(expf(__fsub_rn(srow[v], M)), s);
  __syncthreads();
  const bool use_k = top_k > 0 && top_k < V;
  const bool use_p = top_p > 0.f && top_p < 1.f;
  unsigned int t_bits = 0, keep_eq = 0, eq_cnt = 0;
  bool filter = false;
  if (use_p) {
    radix_cut(srow, V, true, mass_fixed(top_p), cut);
    if (cut.hit) {
      const unsigned long long need = mass_fixed(top_p) - min(mass_fixed(top_p), cut.above_mass);
      const unsigned long long unit = mass_fixed(__uint_as_float(cut.pfx));
      unsigned long long e = unit ? (need + unit - 1) / unit : 1ull;
      e = max(1ull, min(e, static_cast<unsigned long long>(cut.eq_cnt)));
      const unsigned int m_p = cut.above_cnt + static_cast<unsigned int>(e);
      if (!use_k || m_p <= static_cast<unsigned int>(top_k)) {
        filter = true;
        t_bits = cut.pfx;
        keep_eq = static_cast<unsigned int>(e);
        eq_cnt = cut.eq_cnt;
      }
    }
    __syncthreads();
  }
  if (use_k && !filter) {
    radix_cut(srow, V, false, static_cast<unsigned long long>(top_k), cut);
    filter = true;
    t_bits = cut.pfx;
    keep_eq = static_cast<unsigned int>(top_k) - cut.above_cnt;
    eq_cnt = cut.eq_cnt;
    __syncthreads();
  }
  if (filter && keep_eq < eq_cnt && threadIdx.x == 0) {
    // drop the tied entries past the first keep_eq token ids
    unsigned int taken = 0;
    for (int v = 0; v < V; ++v)
      if (__float_as_uint(srow[v]) == t_bits) {
        if (taken < keep_eq) ++taken;
        else srow[v] = 0.f;
      }
  }
  __syncthreads();
  float fs = 0.f;
  for (int v = threadIdx.x; v < V; v += blockDim.x) {
    float p = srow[v];
    if (filter && __float_as_uint(p) < t_bits) {
      p = 0.f;
      srow[v] = 0.f;
    }
    fs += p;
  }
  fs = block_sum(fs, red);
  for (int v = threadIdx.x; v < V; v += blockDim.x) srow[v] = __fdiv_rn(srow[v], fs);
  __syncthreads();
}

__device__ int argmax_smem(const float *srow, int V, float *redv, int *redi) {
  ArgMax a{-INFINITY, 0x7fffffff};
  for (int v = threadIdx.x; v < V; v += blockDim.x) a = argmax_merge(a, ArgMax{srow[v], v});
  a = block_argmax(a, redv, redi);
  return a.i == 0x7fffffff ? 0 : a.i;
}

// sample_token (src/nn/layer.cpp:1493-1498) given the uniform u:
//  mode 0 (mt19937): std::discrete_distribution -- fp64 cumulative of the
//    normalised weights, the last forced to 1, first index with cum >= u;
//  mode 1 (host table): first index whose fp64 running sum exceeds u * total.
// `u` must be the same value in every thread.
__device__ int sample_smem(const float *p, int V, double u, int mode, double *redd, int *redi) {
  const int C = (V + blockDim.x - 1) / blockDim.x;
  const int lo = min(V, static_cast<int>(threadIdx.x) * C), hi = min(V, lo + C);
  double loc = 0.0;
  int last_nz = -1;
  for (int v = lo; v < hi; ++v) {
    loc += static_cast<double>(p[v]);
    if (p[v] > 0.f) last_nz = v;
  }
  double total;
  double cum = block_exscan_d(loc, redd, &total);
  int pick = 0x7fffffff;
  const double thr = u * total;
  for (int v = lo; v < hi; ++v) {
    cum += static_cast<double>(p[v]);
    const bool hit = (mode == 0) ? (v == V - 1 || cum / total >= u) : (cum > thr);
    if (hit) {
      pick = v;
      break;
    }
  }
  __syncthreads();
  int m = pick;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = min(m, __shfl_xor_sync(0xffffffffu, m, o));
  int lz = last_nz;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) lz = max(lz, __shfl_xor_sync(0xffffffffu, lz, o));
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  if (lane == 0) {
    redi[wid] = m;
    redi[32 + wid] = lz;
  }
  __syncthreads();
  m = (lane < nw) ? redi[lane] : 0x7fffffff;
  lz = (lane < nw) ? redi[32 + lane] : -1;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    m = min(m, __shfl_xor_sync(0xffffffffu, m, o));
    lz = max(lz, __shfl_xor_sync(0xffffffffu, lz, o));
  }
  __syncthreads();
  if (m != 0x7fffffff) return m;
  return lz < 0 ? 0 : lz;
}

constexpr int kSampThreads = 1024;
constexpr int kAcceptRows = 32;    // verify rows whose normalisers accept_kernel finds in parallel
constexpr int kMaxLookahead = 32;  // largest draft length k the handle accepts

struct SampShared {
  float red[32];
  float redv[32];
  int redi[64];
  double redd[33];
  uint32_t old_s[kMtN];
  uint32_t new_s[kMtN];
  uint32_t win[40];
  int used, twisted;
  double u;
  int flag;
  CutShared cut;
};

__device__ __forceinline__ RngCtx make_rng(SampShared &s) {
  return RngCtx{s.old_s, s.new_s, s.win, &s.used, &s.twisted};
}

__device__ __forceinline__ void emit(const SpecState &st, int b, int tok) {
  const int n = st.n_new[b];
  if (n < st.out_len - st.prompt_len) st.tokens_out[static_cast<size_t>(b) * st.out_len + st.prompt_len + n] = tok;
  st.n_new[b] = n + 1;
}

// ---------------------------------------------------------------------------
// Request setup: prompt copy, fresh counters, all rows unused.
__global__ void init_state_kernel(SpecState st, const int *__restrict__ prompts, int S) {
  const int b = blockIdx.x;
  if (b >= st.B) return;
  for (int i = threadIdx.x; i < S; i += blockDim.x)
    st.tokens_out[static_cast<size_t>(b) * st.out_len + i] = prompts[static_cast<size_t>(b) * S + i];
  if (threadIdx.x == 0) {
    st.n_new[b] = 0;
    st.t_len[b] = S;
    st.d_len[b] = S;
    st.t_start[b] = S;
    st.d_start[b] = S;
    st.last_tok[b] = 0;
    st.active[b] = 1;
    st.M[b] = 0;
    st.round[b] = 0;
    for (int i = 0; i < 4; ++i) st.stats[4 * b + i] = 0;
    if (S > st.t_cap || S > st.d_cap) atomicOr(st.err, kErrSeqLen);
    clear_request_rows(st, b);
    if (st.tree) tree_clear_rows(st, b);
  }
}

// Prefill rows of one chunk [c0, c0 + clen) of every prompt (row b*clen + i)
// and the head's row selection (the last row of each request).
__global__ void plan_prefill_kernel(const int *__restrict__ prompts, int B, int S, int c0, int clen, int V, int *rtok,
                                    int *rpos, int *rreq, int *sel) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= B * clen) return;
  const int b = r / clen, i = r % clen;
  const int t = prompts[static_cast<size_t>(b) * S + c0 + i];
  rtok[r] = (t >= 0 && t < V) ? t : 0;
  rpos[r] = c0 + i;
  rreq[r] = b;
  if (sel && i == clen - 1) sel[b] = r;
}

// First new token from the target's prefill logits (src/nn/layer.cpp:1500-1510),
// then the rows of the first round's draft step 0.
__global__ void __launch_bounds__(kSampThreads) first_token_kernel(SpecState st, const float *__restrict__ logits) {
  pdl_wait();
  __shared__ SampShared sh;
  extern __shared__ float srow[];  // [V]
  const int b = blockIdx.x;
  RngCtx rc = make_rng(sh);
  load_row(logits + static_cast<size_t>(b) * st.V, st.V, srow);
  int tok;
  if (st.greedy) {
    tok = argmax_smem(srow, st.V, sh.redv, sh.redi);
  } else {
    rng_prepare(st, b, 2, rc);
    probs_smem(srow, st.V, st.T, st.top_k, st.top_p, sh.red, sh.cut);
    if (threadIdx.x == 0) sh.u = draw_sample_u(st, b, 0, st.u_slots - 1, rc);
    __syncthreads();
    tok = sample_smem(srow, st.V, sh.u, st.rng_mode, sh.redd, sh.redi);
    rng_commit(st, b, rc);
  }
  if (threadIdx.x == 0) {
    emit(st, b, tok);
    st.last_tok[b] = tok;
    st.round[b] = 1;
    bool more = st.n_new[b] < st.max_new;
    if (more) more = st.tree ? tree_start_round(st, b, -1) : start_round(st, b, -1);
    st.active[b] = more ? 1 : 0;
  }
}

// Draft sample after draft step j (src/nn/layer.cpp:1541-1558): q_j =
// get_probs(draft logits), candidate j = sample_token(q_j).  Writes the rows
// of draft step j+1, and after the last draft step the verify rows
// [last, c_0 .. c_{M-1}] at t_len + i (src/nn/layer.cpp:1560-1567).
__global__ void __launch_bounds__(kSampThreads) draft_sample_kernel(SpecState st, int j, const float *__restrict__ logits) {
  pdl_wait();
  __shared__ SampShared sh;
  extern __shared__ float srow[];  // [V]
  const int b = blockIdx.x;
  if (!st.active[b]) return;
  const int M = st.M[b];
  if (j >= M) {
    if (threadIdx.x == 0 && j + 1 < st.k) clear_row(st, step_row(st, j + 1, b));
    return;
  }
  // the state the tail of thread 0 writes from, read up front (the earlier
  // candidates only for the last step, which writes the verify rows)
  __shared__ int s_cand[kMaxLookahead];
  __shared__ int s_len[3];  // d_len, t_len, last_tok
  int *cand = st.cand + b * st.kmax;
  if (j == M - 1 && static_cast<int>(threadIdx.x) < j) s_cand[threadIdx.x] = cand[threadIdx.x];
  if (threadIdx.x == 0) {
    s_len[0] = st.d_len[b];
    s_len[1] = st.t_len[b];
    s_len[2] = st.last_tok[b];
  }
  RngCtx rc = make_rng(sh);
  load_row(logits + static_cast<size_t>(b) * st.V, st.V, srow);
  int tok;
  if (st.greedy) {
    tok = argmax_smem(srow, st.V, sh.redv, sh.redi);
  } else {
    rng_prepare(st, b, 2, rc);
    probs_smem(srow, st.V, st.T, st.top_k, st.top_p, sh.red, sh.cut);
    store_row(srow, st.V, st.q + (static_cast<size_t>(b) * st.kmax + j) * st.V);  // q_j, read by accept
    if (threadIdx.x == 0) sh.u = draw_sample_u(st, b, st.round[b], j, rc);
    __syncthreads();
    tok = sample_smem(srow, st.V, sh.u, st.rng_mode, sh.redd, sh.redi);
    rng_commit(st, b, rc);
  }
  pdl_launch();  // the next pass may launch while this block writes its rows
  if (threadIdx.x == 0) {
    cand[j] = tok;
    if (j + 1 < M) {
      const int d = s_len[0];
      set_row(st, step_row(st, j + 1, b), tok, d, b);
      st.d_len[b] = d + 1;
    } else if (j + 1 < st.k) {
      clear_row(st, step_row(st, j + 1, b));
    }
    if (j == M - 1) {
      const int t = s_len[1];
      for (int i = 0; i <= st.k; ++i) {
        if (i <= M) set_row(st, verify_row(st, b, i), i == 0 ? s_len[2] : i - 1 < j ? s_cand[i - 1] : tok, t + i, b);
        else clear_row(st, verify_row(st, b, i));
      }
      st.t_start[b] = t;
      st.t_len[b] = t + M + 1;
    }
  }
}

// draft_sample_kernel for large vocabularies without top-k / top-p: the
// row of request b is split over a thread-block cluster of CS CTAs (rank r
// holds columns [r Vc, (r + 1) Vc)), so the per-element passes (scale, exp,
// the two normalisations, the fp64 inverse-CDF scan) run on CS SMs.  The CTAs
// publish their partials (row max and exp-sum, the filtered sum, the fp64
// slice sum, the first hit) in their own shared memory; after a cluster
// barrier every rank combines all CS partials in rank order, so every rank
// computes the same normalisers.  Rank 0 owns the request's mt19937 state and
// the bookkeeping of draft_sample_kernel.  Same probabilities and token as
// draft_sample_kernel up to the summation order of the normalisers.
constexpr int kSampMaxCluster = 8;

struct SampClusterEx {
  float mx, se, fs;
  float amax;
  int aidx;
  int pick, lastnz;
  double u, tot;
};

template <int CS>
__global__ void __launch_bounds__(kSampThreads) draft_sample_cluster_kernel(SpecState st, int j,
                                                                            const float *__restrict__ logits) {
  namespace cg = cooperative_groups;
  pdl_wait();
  __shared__ SampShared sh;
  __shared__ SampClusterEx ex;
  __shared__ int s_cand[kMaxLookahead];
  __shared__ int s_len[3];
  extern __shared__ float srow[];  // [Vc]: this rank's columns
  cg::cluster_group cl = cg::this_cluster();
  const int rank = static_cast<int>(cl.block_rank());
  const int b = blockIdx.x / CS;
  // exits that depend on the request only: every rank of the cluster takes them
  if (!st.active[b]) return;
  const int M = st.M[b];
  if (j >= M) {
    if (rank == 0 && threadIdx.x == 0 && j + 1 < st.k) clear_row(st, step_row(st, j + 1, b));
    return;
  }
  const int V = st.V;
  const int Vc = ((V + CS - 1) / CS + 3) & ~3;
  const int v0 = min(V, rank * Vc);
  const int n = min(V, v0 + Vc) - v0;
  int *cand = st.cand + b * st.kmax;
  if (rank == 0) {
    if (j == M - 1 && static_cast<int>(threadIdx.x) < j) s_cand[threadIdx.x] = cand[threadIdx.x];
    if (threadIdx.x == 0) {
      s_len[0] = st.d_len[b];
      s_len[1] = st.t_len[b];
      s_len[2] = st.last_tok[b];
    }
  }
  RngCtx rc = make_rng(sh);
  load_row(logits + static_cast<size_t>(b) * V + v0, n, srow);
  int tok;
  if (st.greedy) {
    ArgMax a{-INFINITY, 0x7fffffff};
    for (int v = threadIdx.x; v < n; v += blockDim.x) a = argmax_merge(a, ArgMax{srow[v], v0 + v});
    a = block_argmax(a, sh.redv, sh.redi);
    if (threadIdx.x == 0) { ex.amax = a.v; ex.aidx = a.i; }
    cl.sync();
    ArgMax g{-INFINITY, 0x7fffffff};
    for (int r = 0; r < CS; ++r) {
      const SampClusterEx *e = cl.map_shared_rank(&ex, r);
      g = argmax_merge(g, ArgMax{e->amax, e->aidx});
    }
    tok = g.i == 0x7fffffff ? 0 : g.i;
  } else {
    if (rank == 0) {
      rng_prepare(st, b, 2, rc);
      if (threadIdx.x == 0) ex.u = draw_sample_u(st, b, st.round[b], j, rc);
    }
    // get_probs (src/nn/layer.cpp:1425-1449): x / T, the row max, exp-sum
    const float T = st.T;
    const bool t1 = T == 1.f;
    float mx = -INFINITY, se = 0.f;
    for (int v = threadIdx.x; v < n; v += blockDim.x) {
      const float x = t1 ? srow[v] : __fdiv_rn(srow[v], T);
      srow[v] = x;
      if (x > mx) {
        se = se * expf(mx - x) + 1.f;
        mx = x;
      } else {
        se += expf(x - mx);
      }
    }
    const float bm = block_max(mx, sh.red);
    const float bs = block_sum(mx == -INFINITY ? 0.f : se * expf(mx - bm), sh.red);
    if (threadIdx.x == 0) { ex.mx = bm; ex.se = bs; }
    cl.sync();
    float Mx = -INFINITY;
    for (int r = 0; r < CS; ++r) Mx = fmaxf(Mx, cl.map_shared_rank(&ex, r)->mx);
    float S = 0.f;
    for (int r = 0; r < CS; ++r) {
      const SampClusterEx *e = cl.map_shared_rank(&ex, r);
      if (e->mx != -INFINITY) S += e->se * expf(e->mx - Mx);
    }
    const double u = cl.map_shared_rank(&ex, 0)->u;
    float fs = 0.f;
    for (int v = threadIdx.x; v < n; v += blockDim.x) {
      const float p = __fdiv_rn(expf(__fsub_rn(srow[v], Mx)), S);
      srow[v] = p;
      fs += p;
    }
    fs = block_sum(fs, sh.red);
    __syncthreads();
    if (threadIdx.x == 0) ex.fs = fs;
    cl.sync();
    float FS = 0.f;
    for (int r = 0; r < CS; ++r) FS += cl.map_shared_rank(&ex, r)->fs;
    for (int v = threadIdx.x; v < n; v += blockDim.x) srow[v] = __fdiv_rn(srow[v], FS);
    __syncthreads();
    store_row(srow, n, st.q + (static_cast<size_t>(b) * st.kmax + j) * V + v0);  // q_j, read by accept
    // sample_token (src/nn/layer.cpp:1493-1498) over the whole row: this
    // rank's fp64 slice sum, the ranks below it, then the first hit
    const int C = (n + blockDim.x - 1) / blockDim.x;
    const int lo = min(n, static_cast<int>(threadIdx.x) * C), hi = min(n, lo + C);
    double loc = 0.0;
    int last_nz = -1;
    for (int v = lo; v < hi; ++v) {
      loc += static_cast<double>(srow[v]);
      if (srow[v] > 0.f) last_nz = v0 + v;
    }
    double slice_tot;
    double cum = block_exscan_d(loc, sh.redd, &slice_tot);
    if (threadIdx.x == 0) ex.tot = slice_tot;
    cl.sync();
    double below = 0.0, total = 0.0;
    for (int r = 0; r < CS; ++r) {
      const double t = cl.map_shared_rank(&ex, r)->tot;
      if (r < rank) below += t;
      total += t;
    }
    cum += below;
    int pick = 0x7fffffff;
    const double thr = u * total;
    for (int v = lo; v < hi; ++v) {
      cum += static_cast<double>(srow[v]);
      const bool hit = (st.rng_mode == 0) ? (v0 + v == V - 1 || cum / total >= u) : (cum > thr);
      if (hit) {
        pick = v0 + v;
        break;
      }
    }
    int m = pick, lz = last_nz;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      m = min(m, __shfl_xor_sync(0xffffffffu, m, o));
      lz = max(lz, __shfl_xor_sync(0xffffffffu, lz, o));
    }
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    __syncthreads();
    if (lane == 0) {
      sh.redi[wid] = m;
      sh.redi[32 + wid] = lz;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int bm2 = 0x7fffffff, bl = -1;
      for (int w = 0; w < nw; ++w) {
        bm2 = min(bm2, sh.redi[w]);
        bl = max(bl, sh.redi[32 + w]);
      }
      ex.pick = bm2;
      ex.lastnz = bl;
    }
    cl.sync();
    int gm = 0x7fffffff, gl = -1;
    for (int r = 0; r < CS; ++r) {
      const SampClusterEx *e = cl.map_shared_rank(&ex, r);
      gm = min(gm, e->pick);
      gl = max(gl, e->lastnz);
    }
    tok = gm != 0x7fffffff ? gm : (gl < 0 ? 0 : gl);
    if (rank == 0) rng_commit(st, b, rc);
  }
  cl.sync();  // no rank leaves while another still reads its shared memory
  if (rank != 0) return;
  pdl_launch();
  if (threadIdx.x == 0) {
    cand[j] = tok;
    if (j + 1 < M) {
      const int d = s_len[0];
      set_row(st, step_row(st, j + 1, b), tok, d, b);
      st.d_len[b] = d + 1;
    } else if (j + 1 < st.k) {
      clear_row(st, step_row(st, j + 1, b));
    }
    if (j == M - 1) {
      const int t = s_len[1];
      for (int i = 0; i <= st.k; ++i) {
        if (i <= M) set_row(st, verify_row(st, b, i), i == 0 ? s_len[2] : i - 1 < j ? s_cand[i - 1] : tok, t + i, b);
        else clear_row(st, verify_row(st, b, i));
      }
      st.t_start[b] = t;
      st.t_len[b] = t + M + 1;
    }
  }
}

// Scratch of accept_kernel's unfiltered path: per verify row the get_probs
// normalisers (or the argmax), warp partials, the candidates.
struct AcceptShared {
  float M[kAcceptRows], S[kAcceptRows], F[kAcceptRows];
  int am[kAcceptRows];
  int cand[kAcceptRows];
  float wf[32];
  int wi[32];
  int rj;
  int t_start, t_len, d_len, d_start, last_tok;  // thread 0's bookkeeping state
};

// x = l / T as get_probs forms it (x / 1 is x itself, so T = 1 skips the divide).
__device__ __forceinline__ float scaled_logit(float l, float T, bool t1) { return t1 ? l : __fdiv_rn(l, T); }

// Normalisers of the verify rows [r0, r0 + n) of one request: for sampling
// the max of l/T, the exp-sum and the sum of the normalised values
// (probs_smem's three reductions), for greedy the argmax.  The rows are
// staged in shared memory (row r0 + i at srow + i * V) and a group of warps
// works on each.
__device__ void accept_row_stats(const SpecState &st, const float *lg0, int r0, int n, float *srow, AcceptShared &a) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const bool t1 = st.T == 1.f;
  {
    load_row(lg0 + static_cast<size_t>(r0) * st.V, n * st.V, srow);  // ends with a barrier
    const int G = max(1, nw / n);  // warps past G * n only join the barriers
    const int j = warp / G, gw = warp % G;
    const bool mine = j < n;
    const float *row = srow + static_cast<size_t>(mine ? j : 0) * st.V;
    const int v0 = gw * 32 + lane, dv = G * 32;
    if (st.greedy) {
      ArgMax am{-INFINITY, 0x7fffffff};
      if (mine)
        for (int v = v0; v < st.V; v += dv) am = argmax_merge(am, ArgMax{row[v], v});
      am = warp_argmax(am);
      if (lane == 0) {
        a.wf[warp] = am.v;
        a.wi[warp] = am.i;
      }
      __syncthreads();
      if (mine && gw == 0 && lane == 0) {
        for (int w = 1; w < G; ++w) am = argmax_merge(am, ArgMax{a.wf[warp + w], a.wi[warp + w]});
        a.am[r0 + j] = am.i == 0x7fffffff ? 0 : am.i;
      }
    } else {
      // probs_smem's online max / exp-sum, reduced over the row's warps
      float mx = -INFINITY, se = 0.f;
      if (mine)
        for (int v = v0; v < st.V; v += dv) {
          const float x = scaled_logit(row[v], st.T, t1);
          if (x > mx) {
            se = se * expf(mx - x) + 1.f;
            mx = x;
          } else {
            se += expf(x - mx);
          }
        }
      float r = warp_max(mx);
      if (lane == 0) a.wf[warp] = r;
      __syncthreads();
      float Mx = -INFINITY;
      if (mine)
        for (int w = 0; w < G; ++w) Mx = fmaxf(Mx, a.wf[j * G + w]);
      __syncthreads();
      r = warp_sum(mx == -INFINITY ? 0.f : se * expf(mx - Mx));
      if (lane == 0) a.wf[warp] = r;
      __syncthreads();
      float S = 0.f;
      if (mine)
        for (int w = 0; w < G; ++w) S += a.wf[j * G + w];
      __syncthreads();
      float fs = 0.f;
      if (mine)
        for (int v = v0; v < st.V; v += dv) fs += __fdiv_rn(expf(__fsub_rn(scaled_logit(row[v], st.T, t1), Mx)), S);
      r = warp_sum(fs);
      if (lane == 0) a.wf[warp] = r;
      __syncthreads();
      if (mine && gw == 0 && lane == 0) {
        float F = 0.f;
        for (int w = 0; w < G; ++w) F += a.wf[j * G + w];
        a.M[r0 + j] = Mx;
        a.S[r0 + j] = S;
        a.F[r0 + j] = F;
      }
    }
    __syncthreads();
  }
}

// Acceptance, residual / bonus sample and rollback for one request
// (src/nn/layer.cpp:1581-1655).  Rollback is a length reset: the cache slots
// past the new length are simply overwritten by later rows.  Ends by writing
// the next round's draft step 0 rows.
//
// Without top-k / top-p, get_probs of a row is fixed by its three normalisers.
// The verify rows are staged in shared memory `stage_rows` at a time; the
// normalisers of a staged chunk are found together (accept_row_stats), its
// acceptance tests need p at one token each and run in parallel, one lane
// per test (test j draws the j-th uniform of the round, as the sequential
// walk does when tests 0 .. j-1 accept), and the walk ends at the chunk with
// the first rejection.  Only the row a token is drawn from gets a full pass.
// With a filter the rows are walked one by one through probs_smem.
__global__ void __launch_bounds__(kSampThreads) accept_kernel(SpecState st, const float *__restrict__ logits,
                                                               int stage_rows) {
  pdl_wait();
  __shared__ SampShared sh;
  __shared__ AcceptShared ash;
  extern __shared__ float srow[];  // [V], or stage_rows rows of V on the unfiltered path
  const int b = blockIdx.x;
  if (!st.active[b]) return;
  // thread 0's bookkeeping state, read up front so that its tail does not
  // wait on a chain of loads
  if (threadIdx.x == 0) {
    ash.t_start = st.t_start[b];
    ash.t_len = st.t_len[b];
    ash.d_len = st.d_len[b];
    ash.d_start = st.d_start[b];
    ash.last_tok = st.last_tok[b];
  }
  RngCtx rc = make_rng(sh);
  const int M = st.M[b];
  const int W = st.k + 1;
  const int round = st.round[b];
  const float *lg0 = logits + static_cast<size_t>(b) * W * st.V;
  const int *cand = st.cand + b * st.kmax;
  if (!st.greedy) rng_prepare(st, b, st.k + 2, rc);

  const int n0 = st.n_new[b];
  int rj = -1, am_rj = 0, naccept = 0;
  const bool filtered = (st.top_k > 0 && st.top_k < st.V) || (st.top_p > 0.f && st.top_p < 1.f);
  const bool fast = !filtered && M + 1 <= kAcceptRows;
  if (fast) {
    // chunks of staged rows; the walk stops at the chunk with the first rejection
    int r0 = 0;
    for (;; r0 += stage_rows) {
      const int n = min(stage_rows, M + 1 - r0);
      accept_row_stats(st, lg0, r0, n, srow, ash);
      if (threadIdx.x < 32) {
        const int j = r0 + threadIdx.x;
        bool acc = true;
        if (j < min(M, r0 + n)) {
          const int c = cand[j];
          ash.cand[j] = c;
          if (st.greedy) {
            acc = c == ash.am[j];
          } else {
            const float x = scaled_logit(__ldg(lg0 + static_cast<size_t>(j) * st.V + c), st.T, st.T == 1.f);
            const float pv = __fdiv_rn(__fdiv_rn(expf(__fsub_rn(x, ash.M[j])), ash.S[j]), ash.F[j]);
            const float qv = st.q[(static_cast<size_t>(b) * st.kmax + j) * st.V + c];
            const float r = st.rng_mode == 0 ? canon_f32(rc.win[j]) : static_cast<float>(table_u(st, b, round, st.k + j));
            acc = __fmul_rn(r, qv) < pv;
          }
        }
        const unsigned rej = __ballot_sync(0xffffffffu, !acc);
        if (threadIdx.x == 0) {
          ash.rj = rej ? r0 + __ffs(rej) - 1 : -1;
          if (!st.greedy) *rc.used = rej ? r0 + __ffs(rej) : M;  // uniforms the tests consumed
        }
      }
      __syncthreads();
      rj = ash.rj;
      if (rj >= 0 || r0 + n > M) break;
    }
    naccept = rj >= 0 ? rj : M;
    const int row = rj >= 0 ? rj : M;
    if (st.greedy) {
      am_rj = ash.am[row];
    } else if (rj >= 0 || n0 + naccept < st.max_new) {
      // p of the row the token is drawn from, as probs_smem leaves it (the
      // last chunk staged holds that row)
      const float *src = srow + static_cast<size_t>(row - r0) * st.V;
      const float Mr = ash.M[row], Sr = ash.S[row], Fr = ash.F[row];
      const bool t1 = st.T == 1.f;
      for (int v = threadIdx.x; v < st.V; v += blockDim.x)
        srow[v] = __fdiv_rn(__fdiv_rn(expf(__fsub_rn(scaled_logit(src[v], st.T, t1), Mr)), Sr), Fr);
      __syncthreads();
    }
  } else {
    for (int j = 0; j < M; ++j) {
      const int c = cand[j];
      load_row(lg0 + static_cast<size_t>(j) * st.V, st.V, srow);
      bool acc;
      if (st.greedy) {
        const int am = argmax_smem(srow, st.V, sh.redv, sh.redi);
        acc = (c == am);
        am_rj = am;
      } else {
        probs_smem(srow, st.V, st.T, st.top_k, st.top_p, sh.red, sh.cut);
        if (threadIdx.x == 0) {
          const float qv = st.q[(static_cast<size_t>(b) * st.kmax + j) * st.V + c];
          const float pv = srow[c];
          const float r = draw_accept_u(st, b, round, st.k + j, rc);
          sh.flag = (__fmul_rn(r, qv) < pv) ? 1 : 0;
        }
        __syncthreads();
        acc = sh.flag != 0;
        __syncthreads();
      }
      if (!acc) {
        rj = j;
        break;
      }
      ++naccept;
    }
    if (threadIdx.x == 0)
      for (int j = 0; j < min(M, kAcceptRows); ++j) ash.cand[j] = cand[j];
  }

  int out_tok = -1;
  if (rj >= 0) {
    if (st.greedy) {
      out_tok = am_rj;
    } else {
      // residual max(0, p - q), renormalised; p itself when the residual is
      // empty (srow holds p of row rj)
      const float *q = st.q + (static_cast<size_t>(b) * st.kmax + rj) * st.V;
      float s = 0.f;
      for (int v = threadIdx.x; v < st.V; v += blockDim.x) {
        const float rv = fmaxf(0.0f, __fsub_rn(srow[v], q[v]));
        srow[v] = rv;
        s += rv;
      }
      s = block_sum(s, sh.red);
      if (s <= 0.0f) {
        load_row(lg0 + static_cast<size_t>(rj) * st.V, st.V, srow);
        probs_smem(srow, st.V, st.T, st.top_k, st.top_p, sh.red, sh.cut);
      } else {
        for (int v = threadIdx.x; v < st.V; v += blockDim.x) srow[v] = __fdiv_rn(srow[v], s);
        __syncthreads();
      }
      if (threadIdx.x == 0) sh.u = draw_sample_u(st, b, round, 2 * st.k, rc);
      __syncthreads();
      out_tok = sample_smem(srow, st.V, sh.u, st.rng_mode, sh.redd, sh.redi);
    }
  } else if (n0 + naccept < st.max_new) {
    // bonus token from row M (the unfiltered path has its argmax, or its p in srow)
    if (!fast) load_row(lg0 + static_cast<size_t>(M) * st.V, st.V, srow);
    if (st.greedy) {
      out_tok = fast ? am_rj : argmax_smem(srow, st.V, sh.redv, sh.redi);
    } else {
      if (!fast) probs_smem(srow, st.V, st.T, st.top_k, st.top_p, sh.red, sh.cut);
      if (threadIdx.x == 0) sh.u = draw_sample_u(st, b, round, 2 * st.k, rc);
      __syncthreads();
      out_tok = sample_smem(srow, st.V, sh.u, st.rng_mode, sh.redd, sh.redi);
    }
  }
  if (!st.greedy) rng_commit(st, b, rc);
  pdl_launch();  // the next pass may launch while this block writes its rows
  if (threadIdx.x == 0) {
    int t_len = ash.t_len, d_len = ash.d_len, last_tok = ash.last_tok;
    const int t_start = ash.t_start, d_start = ash.d_start;
    int n = n0;
    const int cap = st.out_len - st.prompt_len;
    int *out = st.tokens_out + static_cast<size_t>(b) * st.out_len + st.prompt_len;
    auto put = [&](int tok) {
      if (n < cap) out[n] = tok;
      ++n;
    };
    for (int j = 0; j < naccept; ++j) put(j < kAcceptRows ? ash.cand[j] : cand[j]);
    int catch_tok = -1;
    const int last_c = M > 0 ? (M - 1 < kAcceptRows ? ash.cand[M - 1] : cand[M - 1]) : -1;
    if (rj >= 0) {
      put(out_tok);
      t_len = t_start + rj + 1;
      d_len = min(d_len, d_start + rj + 1);
      catch_tok = (st.catchup == 0) ? out_tok : -1;
      last_tok = out_tok;
    } else if (out_tok >= 0) {
      put(out_tok);
      catch_tok = last_c;
      last_tok = out_tok;
    } else if (M > 0) {
      last_tok = last_c;
    }
    st.n_new[b] = n;
    st.t_len[b] = t_len;
    st.d_len[b] = d_len;
    st.last_tok[b] = last_tok;
    unsigned long long *sx = reinterpret_cast<unsigned long long *>(st.stats + 4 * b);
    atomicAdd(sx + 0, 1ull);
    atomicAdd(sx + 1, static_cast<unsigned long long>(M));
    atomicAdd(sx + 2, static_cast<unsigned long long>(naccept));
    if (rj >= 0) atomicAdd(sx + 3, 1ull);
    st.round[b] = round + 1;
    bool still = n < st.max_new;
    if (still) still = start_round_at(st, b, catch_tok, n, d_len, t_len, last_tok);
    else clear_request_rows(st, b);
    st.active[b] = still ? 1 : 0;
    if (still) atomicAdd(st.active_count, 1);
  }
}

// Autoregressive decoding, one token per request from the target's logits
// (generate_advanced, src/nn/layer.cpp:1239-1380, with the KV cache): the
// prefill's last row (first call) or the last step's row.  Sampling follows
// generate_advanced: greedy = first maximum; else probabilities as get_probs
// (temperature, top-k, top-p, renormalised) and one discrete_distribution draw
// (request b's mt19937(seed + b) stream, or u[b][step][0] of the host table).
// Writes the row of the next step (the token at the next cache position) or,
// after max_new tokens, retires the request.  stats[b][0] counts the steps.
__global__ void __launch_bounds__(kSampThreads) ar_token_kernel(SpecState st, const float *__restrict__ logits) {
  pdl_wait();
  __shared__ SampShared sh;
  extern __shared__ float srow[];  // [V]
  const int b = blockIdx.x;
  if (!st.active[b]) return;
  __shared__ int s_state[2];  // n_new, t_len
  if (threadIdx.x == 0) {
    s_state[0] = st.n_new[b];
    s_state[1] = st.t_len[b];
  }
  RngCtx rc = make_rng(sh);
  load_row(logits + static_cast<size_t>(b) * st.V, st.V, srow);
  int tok;
  if (st.greedy) {
    tok = argmax_smem(srow, st.V, sh.redv, sh.redi);
  } else {
    rng_prepare(st, b, 2, rc);
    probs_smem(srow, st.V, st.T, st.top_k, st.top_p, sh.red, sh.cut);
    if (threadIdx.x == 0) sh.u = draw_sample_u(st, b, s_state[0], 0, rc);
    __syncthreads();
    tok = sample_smem(srow, st.V, sh.u, st.rng_mode, sh.redd, sh.redi);
    rng_commit(st, b, rc);
  }
  pdl_launch();
  if (threadIdx.x == 0) {
    const int n = s_state[0] + 1;
    st.tokens_out[static_cast<size_t>(b) * st.out_len + st.prompt_len + s_state[0]] = tok;
    st.n_new[b] = n;
    st.stats[4 * b] += 1;
    const int t = s_state[1];
    bool more = n < st.max_new;
    if (more && t + 1 > st.t_cap) {
      atomicOr(st.err, kErrSeqLen);
      more = false;
    }
    if (more) {
      set_row(st, verify_row(st, b, 0), tok, t, b);
      st.t_len[b] = t + 1;
      atomicAdd(st.active_count, 1);
    } else {
      st.active[b] = 0;
      clear_row(st, verify_row(st, b, 0));
    }
  }
}

// Copies the generated sequences and statistics to caller buffers.
__global__ void finalize_kernel(SpecState st, int *__restrict__ out, long long *__restrict__ stats) {
  const int b = blockIdx.x;
  if (b >= st.B) return;
  const int n = st.prompt_len + max(1, st.max_new);
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    out[static_cast<size_t>(b) * n + i] = st.tokens_out[static_cast<size_t>(b) * st.out_len + i];
  if (stats && threadIdx.x < 4) stats[4 * b + threadIdx.x] = st.stats[4 * b + threadIdx.x];
}

}  // namespace specdec
