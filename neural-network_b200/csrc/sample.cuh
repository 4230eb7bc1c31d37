// Sampling, acceptance and bookkeeping kernels of the speculative-decoding
// round (TransformerDecoder::generate_speculative, src/nn/layer.cpp:1382-1661).
//
// Per-request state lives on the device, so a whole round (draft steps,
// verify, accept, rollback) runs without a host round trip and can be
// captured in a CUDA graph.  Row planning kernels turn the state into the row
// batches the forward kernels consume.
#pragma once

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
struct SpecState {
  int *tokens_out;     // [B][out_len]
  int out_len;
  int prompt_len;
  int *n_new;          // [B]
  int *t_len, *d_len;  // cache lengths
  int *t_start, *d_start;
  int *last_tok, *catch_tok, *active, *M;
  int *cand;           // [B][kmax]
  float *q;            // [B][kmax][V]
  float *pbuf;         // [B][V]
  long long *stats;    // [B][4]
  int *round;          // [B]
  uint32_t *mt;        // [B][624]
  int *mt_idx;         // [B]
  int *active_count;
  int *err;
  int B, kmax, V;
  int max_new, k;
  float T;
  int greedy;
  int rng_mode;        // 0 mt19937, 1 host table
  const float *uniforms;
  int u_rounds, u_slots;
  int catchup;         // 0 reference, 1 consistent
  int t_cap, d_cap;
};

struct RngCtx {
  uint32_t *old_s, *new_s;  // shared [624] each
  uint32_t *win;            // shared window
  int *used;                // shared counter
};

// Prepares `need` consecutive tempered words of request b's stream in `win`.
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
  if (threadIdx.x == 0) *c.used = 0;
  __syncthreads();
}

__device__ void rng_commit(const SpecState &st, int b, RngCtx &c) {
  if (st.rng_mode != 0) return;
  __syncthreads();
  const int idx = st.mt_idx[b] + *c.used;
  __syncthreads();
  if (idx >= kMtN) {
    uint32_t *g = st.mt + static_cast<size_t>(b) * kMtN;
    for (int t = threadIdx.x; t < kMtN; t += blockDim.x) g[t] = c.new_s[t];
  }
  if (threadIdx.x == 0) st.mt_idx[b] = idx >= kMtN ? idx - kMtN : idx;
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
// get_probs for T > 0 without top-k/top-p (src/nn/layer.cpp:1426-1489):
// l/T, subtract the max, exp, divide by the sum, then divide by the sum of the
// normalised values (the reference's second normalisation, taken there in
// sorted order).  Writes out[V]; block-cooperative.
__device__ void probs_row(const float *__restrict__ lg, int V, float T, float *__restrict__ out, float *red) {
  float mx = -INFINITY;
  for (int v = threadIdx.x; v < V; v += blockDim.x) mx = fmaxf(mx, __fdiv_rn(lg[v], T));
  mx = block_max(mx, red);
  float s = 0.f;
  for (int v = threadIdx.x; v < V; v += blockDim.x) {
    const float e = expf(__fsub_rn(__fdiv_rn(lg[v], T), mx));
    out[v] = e;
    s += e;
  }
  s = block_sum(s, red);
  float fs = 0.f;
  for (int v = threadIdx.x; v < V; v += blockDim.x) {
    const float p = __fdiv_rn(out[v], s);
    out[v] = p;
    fs += p;
  }
  fs = block_sum(fs, red);
  for (int v = threadIdx.x; v < V; v += blockDim.x) out[v] = __fdiv_rn(out[v], fs);
  __syncthreads();
}

__device__ int argmax_row(const float *__restrict__ lg, int V, float *redv, int *redi) {
  ArgMax a{-INFINITY, 0x7fffffff};
  for (int v = threadIdx.x; v < V; v += blockDim.x) a = argmax_merge(a, ArgMax{lg[v], v});
  a = block_argmax(a, redv, redi);
  return a.i == 0x7fffffff ? 0 : a.i;
}

// sample_token (src/nn/layer.cpp:1493-1498) given the uniform u:
//  mode 0 (mt19937): std::discrete_distribution -- fp64 cumulative of the
//    normalised weights, the last forced to 1, first index with cum >= u;
//  mode 1 (host table): first index whose fp64 running sum exceeds u * total.
// `u` must be the same value in every thread.
__device__ int sample_row(const float *__restrict__ p, int V, double u, int mode, double *redd, int *redi) {
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
    if (hit) { pick = v; break; }
  }
  // block min of pick, block max of last_nz
  __syncthreads();
  int m = pick;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = min(m, __shfl_xor_sync(0xffffffffu, m, o));
  int lz = last_nz;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) lz = max(lz, __shfl_xor_sync(0xffffffffu, lz, o));
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  if (lane == 0) { redi[wid] = m; redi[32 + wid] = lz; }
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

struct SampShared {
  float red[32];
  float redv[32];
  int redi[64];
  double redd[33];
  uint32_t old_s[kMtN];
  uint32_t new_s[kMtN];
  uint32_t win[40];
  int used;
  double u;
  int flag;
  int tok;
};

__device__ __forceinline__ RngCtx make_rng(SampShared &s) { return RngCtx{s.old_s, s.new_s, s.win, &s.used}; }

__device__ __forceinline__ void emit(const SpecState &st, int b, int tok) {
  const int n = st.n_new[b];
  if (n < st.out_len - st.prompt_len) st.tokens_out[static_cast<size_t>(b) * st.out_len + st.prompt_len + n] = tok;
  st.n_new[b] = n + 1;
}

// ---------------------------------------------------------------------------
// Request setup: prompt copy and fresh counters (one thread per request).
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
    st.catch_tok[b] = -1;
    st.active[b] = 1;
    st.M[b] = 0;
    st.round[b] = 0;
    for (int i = 0; i < 4; ++i) st.stats[4 * b + i] = 0;
    if (S > st.t_cap || S > st.d_cap) atomicOr(st.err, kErrSeqLen);
  }
}

// Prefill rows of one chunk [c0, c0 + clen) of every prompt; row b*clen + i.
__global__ void plan_prefill_kernel(const int *__restrict__ prompts, int B, int S, int c0, int clen, int *rtok,
                                    int *rpos, int *rreq, int *sel) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= B * clen) return;
  const int b = r / clen, i = r % clen;
  rtok[r] = prompts[static_cast<size_t>(b) * S + c0 + i];
  rpos[r] = c0 + i;
  rreq[r] = b;
  if (i == clen - 1) sel[b] = r;
}

// First new token from the target's prefill logits (src/nn/layer.cpp:1500-1510).
__global__ void __launch_bounds__(kSampThreads) first_token_kernel(SpecState st, const float *__restrict__ logits) {
  __shared__ SampShared sh;
  const int b = blockIdx.x;
  RngCtx rc = make_rng(sh);
  const float *lg = logits + static_cast<size_t>(b) * st.V;
  int tok;
  if (st.greedy) {
    tok = argmax_row(lg, st.V, sh.redv, sh.redi);
  } else {
    rng_prepare(st, b, 2, rc);
    float *p = st.pbuf + static_cast<size_t>(b) * st.V;
    probs_row(lg, st.V, st.T, p, sh.red);
    if (threadIdx.x == 0) sh.u = draw_sample_u(st, b, 0, 2 * st.k, rc);
    __syncthreads();
    tok = sample_row(p, st.V, sh.u, st.rng_mode, sh.redd, sh.redi);
    rng_commit(st, b, rc);
  }
  if (threadIdx.x == 0) {
    emit(st, b, tok);
    st.last_tok[b] = tok;
    st.active[b] = st.n_new[b] < st.max_new ? 1 : 0;
    st.round[b] = 1;
  }
}

// Draft step 0 rows: [catch-up token (if any), last token] per request at rows
// 2b, 2b+1.  Folding the reference's post-round draft catch-up forward
// (src/nn/layer.cpp:1639-1642, 1649-1653) into the next round's first draft
// step computes the same cache and the same logits for the last row.
__global__ void plan_draft0_kernel(SpecState st, int *rtok, int *rpos, int *rreq, int *sel) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b == 0) *st.active_count = 0;
  if (b >= st.B) return;
  int r0 = 2 * b, r1 = 2 * b + 1;
  sel[b] = r1;
  rreq[r0] = -1; rtok[r0] = 0; rpos[r0] = 0;
  rreq[r1] = -1; rtok[r1] = 0; rpos[r1] = 0;
  if (!st.active[b]) { st.M[b] = 0; return; }
  const int M = min(st.k, st.max_new - st.n_new[b]);
  st.M[b] = M;
  const int c = st.catch_tok[b];
  int d = st.d_len[b];
  if (d + (c >= 0 ? 1 : 0) + M > st.d_cap) {
    atomicOr(st.err, kErrSeqLen);
    st.active[b] = 0;
    st.M[b] = 0;
    return;
  }
  if (c >= 0) { rtok[r0] = c; rpos[r0] = d; rreq[r0] = b; ++d; }
  st.d_start[b] = d;
  rtok[r1] = st.last_tok[b]; rpos[r1] = d; rreq[r1] = b;
  st.d_len[b] = d + 1;
  st.catch_tok[b] = -1;
}

// Draft step j >= 1: row b feeds candidate j-1.
__global__ void plan_draft_kernel(SpecState st, int j, int *rtok, int *rpos, int *rreq, int *sel) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= st.B) return;
  sel[b] = b;
  if (!st.active[b] || j >= st.M[b]) { rreq[b] = -1; rtok[b] = 0; rpos[b] = 0; return; }
  const int d = st.d_len[b];
  rtok[b] = st.cand[b * st.kmax + j - 1];
  rpos[b] = d;
  rreq[b] = b;
  st.d_len[b] = d + 1;
}

// Verify rows b*(k+1) + i: [last, c_0 .. c_{M-1}] at t_len + i
// (src/nn/layer.cpp:1560-1567).  One thread per request.
__global__ void plan_verify_kernel(SpecState st, int *rtok, int *rpos, int *rreq) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= st.B) return;
  const int W = st.k + 1;
  const int M = st.M[b];
  bool on = st.active[b] != 0;
  const int t = st.t_len[b];
  if (on && t + M + 1 > st.t_cap) {
    atomicOr(st.err, kErrSeqLen);
    on = false;
  }
  for (int i = 0; i < W; ++i) {
    const int r = b * W + i;
    const bool ri = on && i <= M;
    rreq[r] = ri ? b : -1;
    rtok[r] = ri ? (i == 0 ? st.last_tok[b] : st.cand[b * st.kmax + i - 1]) : 0;
    rpos[r] = ri ? t + i : 0;
  }
  if (on) {
    st.t_start[b] = t;
    st.t_len[b] = t + M + 1;
  }
}

// Draft sample after draft step j (src/nn/layer.cpp:1541-1558): q_j =
// get_probs(draft logits), candidate j = sample_token(q_j).
__global__ void __launch_bounds__(kSampThreads) draft_sample_kernel(SpecState st, int j, const float *__restrict__ logits) {
  __shared__ SampShared sh;
  const int b = blockIdx.x;
  if (!st.active[b] || j >= st.M[b]) return;
  RngCtx rc = make_rng(sh);
  const float *lg = logits + static_cast<size_t>(b) * st.V;
  int tok;
  if (st.greedy) {
    tok = argmax_row(lg, st.V, sh.redv, sh.redi);
  } else {
    rng_prepare(st, b, 2, rc);
    float *q = st.q + (static_cast<size_t>(b) * st.kmax + j) * st.V;
    probs_row(lg, st.V, st.T, q, sh.red);
    if (threadIdx.x == 0) sh.u = draw_sample_u(st, b, st.round[b], j, rc);
    __syncthreads();
    tok = sample_row(q, st.V, sh.u, st.rng_mode, sh.redd, sh.redi);
    rng_commit(st, b, rc);
  }
  if (threadIdx.x == 0) st.cand[b * st.kmax + j] = tok;
}

// Acceptance, residual / bonus sample and rollback for one request
// (src/nn/layer.cpp:1581-1655).  Rollback is a length reset: the cache slots
// past the new length are simply overwritten by later rows.
__global__ void __launch_bounds__(kSampThreads) accept_kernel(SpecState st, const float *__restrict__ logits) {
  __shared__ SampShared sh;
  const int b = blockIdx.x;
  if (!st.active[b]) return;
  RngCtx rc = make_rng(sh);
  const int M = st.M[b];
  const int W = st.k + 1;
  const int round = st.round[b];
  const float *lg0 = logits + static_cast<size_t>(b) * W * st.V;
  float *p = st.pbuf + static_cast<size_t>(b) * st.V;
  const int *cand = st.cand + b * st.kmax;
  if (!st.greedy) rng_prepare(st, b, st.k + 2, rc);

  const int n0 = st.n_new[b];
  int rj = -1, am_rj = 0, naccept = 0;
  for (int j = 0; j < M; ++j) {
    const int c = cand[j];
    const float *lg = lg0 + static_cast<size_t>(j) * st.V;
    bool acc;
    if (st.greedy) {
      const int am = argmax_row(lg, st.V, sh.redv, sh.redi);
      acc = (c == am);
      am_rj = am;
    } else {
      probs_row(lg, st.V, st.T, p, sh.red);
      if (threadIdx.x == 0) {
        const float qv = st.q[(static_cast<size_t>(b) * st.kmax + j) * st.V + c];
        const float pv = p[c];
        const float r = draw_accept_u(st, b, round, st.k + j, rc);
        sh.flag = (__fmul_rn(r, qv) < pv) ? 1 : 0;
      }
      __syncthreads();
      acc = sh.flag != 0;
      __syncthreads();
    }
    if (!acc) { rj = j; break; }
    ++naccept;
  }

  int out_tok = -1;
  if (rj >= 0) {
    if (st.greedy) {
      out_tok = am_rj;
    } else {
      // residual max(0, p - q), renormalised; p itself when the residual is empty
      const float *q = st.q + (static_cast<size_t>(b) * st.kmax + rj) * st.V;
      float s = 0.f;
      for (int v = threadIdx.x; v < st.V; v += blockDim.x) {
        const float rv = fmaxf(0.0f, __fsub_rn(p[v], q[v]));
        p[v] = rv;
        s += rv;
      }
      s = block_sum(s, sh.red);
      if (s <= 0.0f) {
        probs_row(lg0 + static_cast<size_t>(rj) * st.V, st.V, st.T, p, sh.red);
      } else {
        for (int v = threadIdx.x; v < st.V; v += blockDim.x) p[v] = __fdiv_rn(p[v], s);
        __syncthreads();
      }
      if (threadIdx.x == 0) sh.u = draw_sample_u(st, b, round, 2 * st.k, rc);
      __syncthreads();
      out_tok = sample_row(p, st.V, sh.u, st.rng_mode, sh.redd, sh.redi);
    }
  } else if (n0 + naccept < st.max_new) {
    const float *lg = lg0 + static_cast<size_t>(M) * st.V;
    if (st.greedy) {
      out_tok = argmax_row(lg, st.V, sh.redv, sh.redi);
    } else {
      probs_row(lg, st.V, st.T, p, sh.red);
      if (threadIdx.x == 0) sh.u = draw_sample_u(st, b, round, 2 * st.k, rc);
      __syncthreads();
      out_tok = sample_row(p, st.V, sh.u, st.rng_mode, sh.redd, sh.redi);
    }
  }
  if (!st.greedy) rng_commit(st, b, rc);
  if (threadIdx.x == 0) {
    for (int j = 0; j < naccept; ++j) emit(st, b, cand[j]);
    if (rj >= 0) {
      emit(st, b, out_tok);
      st.t_len[b] = st.t_start[b] + rj + 1;
      st.d_len[b] = min(st.d_len[b], st.d_start[b] + rj + 1);
      st.catch_tok[b] = (st.catchup == 0) ? out_tok : -1;
      st.last_tok[b] = out_tok;
    } else if (out_tok >= 0) {
      emit(st, b, out_tok);
      st.catch_tok[b] = cand[M - 1];
      st.last_tok[b] = out_tok;
    } else {
      st.last_tok[b] = M > 0 ? cand[M - 1] : st.last_tok[b];
    }
    long long *sx = st.stats + 4 * b;
    sx[0] += 1;
    sx[1] += M;
    sx[2] += naccept;
    sx[3] += (rj >= 0) ? 1 : 0;
    st.round[b] = round + 1;
    const int still = st.n_new[b] < st.max_new ? 1 : 0;
    st.active[b] = still;
    if (still) atomicAdd(st.active_count, 1);
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
