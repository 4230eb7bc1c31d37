// Forward-pass kernels of the decoder stack (target and draft share them).
//
// A forward pass runs over a batch of "rows": one row is one token of one
// request at one cache position.  Prefill, a draft step, the (k+1)-token
// verify block and the draft catch-up are all row batches; row r carries
// (token, position, request) and request < 0 marks an unused row.  Every row
// writes its K/V at its own position before attention reads the cache, so
// causal attention over the cache is the reference's masked attention over
// past + new tokens (src/nn/layer.cpp:842-952, mask j > S_past + i).
//
// Device layouts (chosen for coalesced streaming on B200):
//   weights     W^T [N][K] row-major (output-major), fp32 or int8 + fp32
//               per-output scale; the reference keeps W [K][N]
//               (src/nn/layer.cpp:153) and the loader transposes.
//   QKV         one [d + 2*kvd][d] matrix (q rows, k rows, v rows).
//   SwiGLU      gate/up interleaved: row 2c = gate_c, row 2c+1 = up_c.
//   activations [R][d] in the activation dtype (fp32 or bf16).
//   KV cache    [layer][request slot][kv head][position][D].
//
// The small configurations are latency-bound: every kernel here is built to
// issue its global loads together (one or two L2 round trips per kernel)
// rather than in dependent chains.
#pragma once

#include "common.cuh"

namespace specdec {

struct RowsView {
  const int *tok;  // embedding row (clamped to [0, V) by whoever wrote the row)
  const int *pos;
  const int *req;
};

// ---------------------------------------------------------------------------
// Embedding gather (Embedding::forward -> CpuBackend::embedding,
// src/backend/cpu_backend.cpp:998-1033: an out-of-range id reads row 0).  The
// cfg architecture adds the learned position row and also writes LN1(x) for
// the first layer.  One block per row; d <= 32 * blockDim.
template <typename AT>
__global__ void embed_kernel(RowsView rows, int R, const float *__restrict__ emb, const float *__restrict__ pos_emb,
                             int d, int max_pos, AT *__restrict__ x, const float *__restrict__ ln_g,
                             const float *__restrict__ ln_b, AT *__restrict__ x_ln) {
  __shared__ float red[32];
  const int r = blockIdx.x;
  if (r >= R) return;
  const int id = rows.tok[r];
  const int p = min(max(rows.pos[r], 0), max_pos - 1);
  constexpr int kMax = 32;
  float v[kMax];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kMax; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    float t = 0.f;
    if (c < d) {
      t = emb[static_cast<size_t>(id) * d + c];
      if (pos_emb) t += pos_emb[static_cast<size_t>(p) * d + c];
      t = to_f32(from_f32<AT>(t));
      x[static_cast<size_t>(r) * d + c] = from_f32<AT>(t);
    }
    v[i] = t;
    s += t;
  }
  if (!ln_g) return;
  const float mean = __fdiv_rn(block_sum(s, red), static_cast<float>(d));
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < kMax; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < d) {
      const float df = v[i] - mean;
      q = fmaf(df, df, q);
    }
  }
  const float sd = sqrtf(__fdiv_rn(block_sum(q, red), static_cast<float>(d)) + 1e-5f);
#pragma unroll
  for (int i = 0; i < kMax; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < d)
      x_ln[static_cast<size_t>(r) * d + c] =
          from_f32<AT>(__fadd_rn(__fmul_rn(__fdiv_rn(v[i] - mean, sd), ln_g[c]), ln_b[c]));
  }
}

// ---------------------------------------------------------------------------
// Linear layer y = x . W + b on CUDA cores for the small row counts of draft
// steps and verify blocks (a GEMV per tile of kRowTile rows).
//
// A warp owns a PAIR of adjacent output columns (so RoPE pairs and SwiGLU
// gate/up pairs land in one lane); `ksplit` warps of a block share one pair
// and split K, so each lane issues its weight and input vectors in one go.
// Everything the epilogue needs (scale, bias, residual, row position, RoPE
// factors) is loaded before the dot products.  With `ln_out` set, the last
// block to finish a row tile applies the following LayerNorm
// (LayerNorm::forward, src/nn/layer.cpp:242-261) to the complete rows, so no
// separate norm kernel runs.
enum Epi : int {
  kEpiStore = 0,   // out = acc*s + b
  kEpiResid = 1,   // out = acc*s + b + resid
  kEpiQKV = 2,     // RoPE(q), RoPE(k) -> q buffer and K cache; v -> V cache
  kEpiSwiGLU = 3,  // out[c] = silu(gate_c) * up_c
  kEpiGelu = 4,    // out = gelu(acc*s + b), erf form
};

struct QKVArgs {
  int d, kvd, D;             // q width, k/v width, head dim
  const float2 *rope;        // [max_pos][D/2] (cos, sin)
  int rope_max_pos;
  void *kc, *vc;             // this layer's caches
  size_t kv_req_stride;      // elements per request slot
  int S_cap;                 // positions per (request, head)
  int kv_bf16;               // cache element type: 0 fp32, 1 bf16
  int *err;
};

struct LinearArgs {
  const void *x;          // input rows (activation dtype)
  int ldx;
  const int *in_rows;     // optional row map: logical row r reads x row in_rows[r]
  int R;
  const void *W;          // [N][K]
  const float *scale;     // [N] or null
  const float *bias;      // [N] (interleaved like W for SwiGLU)
  int N, K;
  void *out;
  int ldo;
  int out_f32;            // 1: fp32 output (logits); 0: activation dtype
  const void *resid;
  int ldr;
  RowsView rows;          // row metadata (QKV epilogue)
  QKVArgs qkv;
  const float *ln_g, *ln_b;  // optional LayerNorm of the finished output rows ...
  void *ln_out;              // ... written here (activation dtype, leading dim ldo)
  int *tile_counters;        // [row tiles] arrival counters (left at 0)
  int ksplit;                // warps per column pair: 1, 2, 4 or 8
};

constexpr int kLinWarps = 8;
constexpr int kRowTile = 8;
constexpr int kLnMaxPerLane = 32;  // LayerNorm rows held in registers: N <= 1024 per warp

template <typename WT> struct WVec;
template <> struct WVec<float> { static constexpr int E = 4; };
template <> struct WVec<int8_t> { static constexpr int E = 8; };

__device__ __forceinline__ void load_wvec(const float *p, float (&w)[4]) {
  const float4 t = __ldg(reinterpret_cast<const float4 *>(p));
  w[0] = t.x; w[1] = t.y; w[2] = t.z; w[3] = t.w;
}
// int8 -> fp32 without the conversion unit: with u = q + 128 placed in the
// low byte of 0x4B000000 the float is exactly 2^23 + u, so subtracting
// 2^23 + 128 gives q exactly.
__device__ __forceinline__ void i8x4_to_f32(uint32_t word, float *w) {
  const uint32_t u = word ^ 0x80808080u;
  w[0] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7540)) - 8388736.0f;
  w[1] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7541)) - 8388736.0f;
  w[2] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7542)) - 8388736.0f;
  w[3] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7543)) - 8388736.0f;
}
__device__ __forceinline__ void load_wvec(const int8_t *p, float (&w)[8]) {
  const uint2 t = __ldg(reinterpret_cast<const uint2 *>(p));
  i8x4_to_f32(t.x, w);
  i8x4_to_f32(t.y, w + 4);
}

// Reduce-scatter of 2*kRowTile per-lane partial sums over the warp in 16
// shuffles: afterwards lane l holds the full sum of value (column
// (l >> 4) & 1, row ((l >> 1) & 7)); lanes differing only in bit 0 agree.
__device__ __forceinline__ float warp_reduce16(const float (&a0)[kRowTile], const float (&a1)[kRowTile]) {
  const int lane = threadIdx.x & 31;
  float v8[8];
  {
    const bool hi = lane & 16;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float send = hi ? a0[i] : a1[i];
      const float keep = hi ? a1[i] : a0[i];
      v8[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
  }
  float v4[4];
  {
    const bool hi = lane & 8;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float send = hi ? v8[i] : v8[i + 4];
      const float keep = hi ? v8[i + 4] : v8[i];
      v4[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
  }
  float v2[2];
  {
    const bool hi = lane & 4;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float send = hi ? v4[i] : v4[i + 2];
      const float keep = hi ? v4[i + 2] : v4[i];
      v2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
  }
  const bool hi = lane & 2;
  float v = (hi ? v2[1] : v2[0]) + __shfl_xor_sync(0xffffffffu, hi ? v2[0] : v2[1], 2);
  return v + __shfl_xor_sync(0xffffffffu, v, 1);
}

// E consecutive input elements as fp32.
template <typename AT, int E>
__device__ __forceinline__ void load_xvec(const AT *p, float (&xv)[E]) {
  if constexpr (sizeof(AT) == 4) {
#pragma unroll
    for (int i = 0; i < E; i += 4) {
      const float4 t = __ldg(reinterpret_cast<const float4 *>(p + i));
      xv[i] = t.x; xv[i + 1] = t.y; xv[i + 2] = t.z; xv[i + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < E; i += 4) {
      const uint2 t = __ldg(reinterpret_cast<const uint2 *>(p + i));
      const __nv_bfloat162 *hh = reinterpret_cast<const __nv_bfloat162 *>(&t);
      const float2 f0 = __bfloat1622float2(hh[0]), f1 = __bfloat1622float2(hh[1]);
      xv[i] = f0.x; xv[i + 1] = f0.y; xv[i + 2] = f1.x; xv[i + 3] = f1.y;
    }
  }
}

// Operands of one lane's epilogue (row r, columns n and n+1), loaded early.
struct EpiPre {
  float s0, s1, b0, b1;  // scale and bias
  float r0, r1;          // residual
  float c, sn;           // RoPE (cos, sin)
  int req, pos;
};

template <typename AT, int EPI>
__device__ __forceinline__ void epilogue_prefetch(const LinearArgs &a, int r, int n, EpiPre &p) {
  const bool has1 = (n + 1) < a.N;
  p.s0 = a.scale ? __ldg(a.scale + n) : 1.f;
  p.s1 = (a.scale && has1) ? __ldg(a.scale + n + 1) : 1.f;
  p.b0 = __ldg(a.bias + n);
  p.b1 = has1 ? __ldg(a.bias + n + 1) : 0.f;
  p.r0 = p.r1 = 0.f;
  p.c = 1.f;
  p.sn = 0.f;
  p.req = 0;
  p.pos = 0;
  if constexpr (EPI == kEpiResid) {
    const AT *rs = static_cast<const AT *>(a.resid) + static_cast<size_t>(r) * a.ldr;
    p.r0 = to_f32(rs[n]);
    p.r1 = has1 ? to_f32(rs[n + 1]) : 0.f;
  }
  if constexpr (EPI == kEpiQKV) {
    const QKVArgs &q = a.qkv;
    p.req = a.rows.req[r];
    p.pos = a.rows.pos[r];
    if (p.req >= 0 && p.pos >= 0 && p.pos < q.rope_max_pos && n < q.d + q.kvd) {
      const int e = (n < q.d ? n : n - q.d) % q.D;
      const float2 cs = q.rope[static_cast<size_t>(p.pos) * (q.D / 2) + (e >> 1)];
      p.c = cs.x;
      p.sn = cs.y;
    }
  }
}

template <typename AT, int EPI>
__device__ __forceinline__ void linear_epilogue(const LinearArgs &a, int r, int n, float v0, float v1, const EpiPre &p) {
  const bool has1 = (n + 1) < a.N;
  v0 = v0 * p.s0 + p.b0;
  v1 = v1 * p.s1 + p.b1;
  if constexpr (EPI == kEpiStore || EPI == kEpiResid || EPI == kEpiGelu) {
    if constexpr (EPI == kEpiResid) {
      v0 = v0 + p.r0;
      v1 = v1 + p.r1;
    }
    if constexpr (EPI == kEpiGelu) {
      v0 = 0.5f * v0 * (1.0f + erff(v0 * 0.70710678118654752f));
      v1 = 0.5f * v1 * (1.0f + erff(v1 * 0.70710678118654752f));
    }
    if (a.out_f32) {
      float *o = static_cast<float *>(a.out) + static_cast<size_t>(r) * a.ldo;
      o[n] = v0;
      if (has1) o[n + 1] = v1;
    } else {
      AT *o = static_cast<AT *>(a.out) + static_cast<size_t>(r) * a.ldo;
      o[n] = from_f32<AT>(v0);
      if (has1) o[n + 1] = from_f32<AT>(v1);
    }
  } else if constexpr (EPI == kEpiSwiGLU) {
    // SwiGLU::forward (src/nn/layer.cpp:1704-1710): (g * sigmoid(g)) * up,
    // sigmoid = 1 / (1 + exp(-g)) (src/backend/cpu_backend.cpp:487-488).
    const float g = v0, u = v1;
    const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
    AT *o = static_cast<AT *>(a.out) + static_cast<size_t>(r) * a.ldo;
    o[n >> 1] = from_f32<AT>(__fmul_rn(__fmul_rn(g, sg), u));
  } else if constexpr (EPI == kEpiQKV) {
    if (p.req < 0) return;
    const QKVArgs &q = a.qkv;
    const int pos = p.pos;
    if (pos < 0 || pos >= q.S_cap || pos >= q.rope_max_pos) {
      if (q.err) atomicOr(q.err, kErrSeqLen);
      return;
    }
    if (n < q.d + q.kvd) {
      // Tensor::rope (src/core/tensor.cpp:1144-1163): pair (2j, 2j+1) of each
      // head rotated by pos * 10000^(-2j/D); the (cos, sin) table is computed
      // on the host with the reference's float formula.
      const float x0 = __fsub_rn(__fmul_rn(v0, p.c), __fmul_rn(v1, p.sn));
      const float x1 = __fadd_rn(__fmul_rn(v0, p.sn), __fmul_rn(v1, p.c));
      v0 = x0;
      v1 = x1;
    }
    if (n < q.d) {
      AT *o = static_cast<AT *>(a.out) + static_cast<size_t>(r) * a.ldo;
      o[n] = from_f32<AT>(v0);
      o[n + 1] = from_f32<AT>(v1);
    } else {
      const bool is_k = n < q.d + q.kvd;
      const int nn = is_k ? n - q.d : n - q.d - q.kvd;
      const int h = nn / q.D, e = nn % q.D;
      const size_t off = static_cast<size_t>(p.req) * q.kv_req_stride + (static_cast<size_t>(h) * q.S_cap + pos) * q.D + e;
      if (q.kv_bf16) {
        __nv_bfloat16 *c = static_cast<__nv_bfloat16 *>(is_k ? q.kc : q.vc);
        c[off] = __float2bfloat16_rn(v0);
        c[off + 1] = __float2bfloat16_rn(v1);
      } else {
        float *c = static_cast<float *>(is_k ? q.kc : q.vc);
        c[off] = v0;
        c[off + 1] = v1;
      }
    }
  }
}

// LayerNorm of rows [r0, r0 + nrows) of `in` (N columns, fp32 statistics),
// one warp per row with the row in registers; the rows were written by other
// blocks of this grid, so they are read through L2 (ld.global.cg).
template <typename AT>
__device__ void rows_layernorm(const AT *in, int ld, int r0, int nrows, int N, const float *g, const float *b, AT *out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = warp; i < nrows; i += blockDim.x >> 5) {
    const AT *x = in + static_cast<size_t>(r0 + i) * ld;
    float v[kLnMaxPerLane];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < kLnMaxPerLane; ++j) {
      const int c = lane + 32 * j;
      v[j] = (c < N) ? to_f32(__ldcg(x + c)) : 0.f;
      s += v[j];
    }
    const float mean = __fdiv_rn(warp_sum(s), static_cast<float>(N));
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < kLnMaxPerLane; ++j) {
      const int c = lane + 32 * j;
      if (c < N) {
        const float df = v[j] - mean;
        q = fmaf(df, df, q);
      }
    }
    const float sd = sqrtf(__fdiv_rn(warp_sum(q), static_cast<float>(N)) + 1e-5f);
    AT *y = out + static_cast<size_t>(r0 + i) * ld;
#pragma unroll
    for (int j = 0; j < kLnMaxPerLane; ++j) {
      const int c = lane + 32 * j;
      if (c < N) y[c] = from_f32<AT>(__fadd_rn(__fmul_rn(__fdiv_rn(v[j] - mean, sd), __ldg(g + c)), __ldg(b + c)));
    }
  }
}

// grid: (ceil(N / (2 * kLinWarps / ksplit)), ceil(R / kRowTile)); block: 32 * kLinWarps.
template <typename WT, typename AT, int EPI>
__global__ void __launch_bounds__(32 * kLinWarps) linear_kernel(LinearArgs a) {
  constexpr int E = WVec<WT>::E;
  __shared__ float s_red[kLinWarps][2 * kRowTile];
  __shared__ int s_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int ks = a.ksplit;
  const int pairs = kLinWarps / ks;
  const int pair = warp / ks, kidx = warp % ks;
  const int n0 = (blockIdx.x * pairs + pair) * 2;
  const int r0 = blockIdx.y * kRowTile;
  const int nrows = min(kRowTile, a.R - r0);
  const bool col_ok = n0 < a.N;
  const bool has1 = (n0 + 1) < a.N;

  float acc0[kRowTile], acc1[kRowTile];
#pragma unroll
  for (int i = 0; i < kRowTile; ++i) acc0[i] = acc1[i] = 0.f;
  EpiPre pre{};
  if (col_ok) {
    // lane 2i finishes row i: fetch its epilogue operands now
    if (kidx == 0 && lane < 16 && !(lane & 1) && (lane >> 1) < nrows)
      epilogue_prefetch<AT, EPI>(a, r0 + (lane >> 1), n0, pre);
    const WT *w0 = static_cast<const WT *>(a.W) + static_cast<size_t>(n0) * a.K;
    const WT *w1 = has1 ? w0 + a.K : w0;
    const AT *xrow[kRowTile];
#pragma unroll
    for (int i = 0; i < kRowTile; ++i) {
      const int lr = r0 + (i < nrows ? i : 0);
      const int pr = a.in_rows ? a.in_rows[lr] : lr;
      xrow[i] = static_cast<const AT *>(a.x) + static_cast<size_t>(pr) * a.ldx;
    }
    const bool vec_ok = (a.K % E == 0) && (a.ldx % 4 == 0);
    const int kvec = vec_ok ? a.K / E : 0;
#pragma unroll 2
    for (int v = kidx * 32 + lane; v < kvec; v += 32 * ks) {
      float wa[E], wb[E];
      load_wvec(w0 + v * E, wa);
      load_wvec(w1 + v * E, wb);
      float xv[kRowTile][E];
#pragma unroll
      for (int i = 0; i < kRowTile; ++i)
        if (i < nrows) load_xvec<AT, E>(xrow[i] + v * E, xv[i]);
#pragma unroll
      for (int i = 0; i < kRowTile; ++i) {
        if (i < nrows) {
          float t0 = 0.f, t1 = 0.f;
#pragma unroll
          for (int e = 0; e < E; ++e) {
            t0 = fmaf(xv[i][e], wa[e], t0);
            t1 = fmaf(xv[i][e], wb[e], t1);
          }
          acc0[i] += t0;
          acc1[i] += t1;
        }
      }
    }
    for (int k = kvec * E + kidx * 32 + lane; k < a.K; k += 32 * ks) {  // scalar tail / unaligned rows
      const float wa = static_cast<float>(w0[k]), wb = static_cast<float>(w1[k]);
#pragma unroll
      for (int i = 0; i < kRowTile; ++i)
        if (i < nrows) {
          const float xv = to_f32(xrow[i][k]);
          acc0[i] = fmaf(xv, wa, acc0[i]);
          acc1[i] = fmaf(xv, wb, acc1[i]);
        }
    }
  }
  // warp totals: lane l holds (column (l >> 4) & 1, row (l >> 1) & 7)
  float tot = warp_reduce16(acc0, acc1);
  const int vidx = ((lane >> 4) & 1) * kRowTile + ((lane >> 1) & 7);
  if (ks > 1) {
    if (!(lane & 1)) s_red[warp][vidx] = tot;
    __syncthreads();
    if (kidx == 0) {
      float t = 0.f;
      for (int j = 0; j < ks; ++j) t += s_red[warp + j][vidx];
      tot = t;
    }
  }
  const float tot1 = __shfl_xor_sync(0xffffffffu, tot, 16);
  if (col_ok && kidx == 0 && lane < 16 && !(lane & 1) && (lane >> 1) < nrows)
    linear_epilogue<AT, EPI>(a, r0 + (lane >> 1), n0, tot, tot1, pre);
  if (!a.ln_out) return;
  // the last block of this row tile normalises the finished rows
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    int *cnt = a.tile_counters + blockIdx.y;
    const int prev = atomicAdd(cnt, 1);
    s_last = (prev == static_cast<int>(gridDim.x) - 1) ? 1 : 0;
    if (s_last) *cnt = 0;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  rows_layernorm<AT>(static_cast<const AT *>(a.out), a.ldo, r0, nrows, a.N, a.ln_g, a.ln_b, static_cast<AT *>(a.ln_out));
}

// ---------------------------------------------------------------------------
// Causal attention (src/nn/layer.cpp:859-948): score = (q . k) / sqrt(D)
// (layer.cpp:870, 891-897), softmax over positions j <= pos, then P.V.
//
// The rows of one request in one forward pass are consecutive and form a
// "group" of Q queries (the k+1 verify rows, the catch-up + last draft rows,
// a prefill chunk); a block handles up to QT queries of one group for one head
// and one split of the context, so the request's K/V are read once for all of
// them.  K/V arrive in tiles of kAttnTile positions that one thread copies
// into shared memory with TMA bulk copies (cp.async.bulk, completion on an
// mbarrier; a (request, head) tile is contiguous in the cache), double
// buffered so the next tile streams in while the current one is used.  Warp w
// owns tile positions w*32 .. w*32+31 (one per lane) and keeps an online
// softmax per query; P.V is accumulated with lanes owning head dimensions.
// Warps are merged through shared memory.  With several splits each block
// writes (max, sum, acc[D]) partials and the last block of a (query tile,
// head) merges them (log-sum-exp), so no separate combine kernel runs.
constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kAttnQT = 8;  // most queries per block (the group size rounds up to 1, 2, 4 or 8)

// Positions per shared-memory tile: 128 (one per thread), or 64 when a K/V
// row is wider than 256 bytes so two stages of K and V stay within 128 KiB.
template <typename KT, int D>
constexpr int attn_tile() { return (D * sizeof(KT) > 256) ? 64 : 128; }

struct AttnArgs {
  const void *q;
  int ldq;
  RowsView rows;
  int R, Q;                 // rows, queries per group
  const void *kc, *vc;
  size_t kv_req_stride;
  int S_cap, H, Hkv;
  int chunk, nsplit;
  void *out;
  int ldo;
  float *part;              // [R][H][nsplit][D + 2]
  int *counters;            // [R][H] split arrival counters (left at 0)
  int *err;
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Polls an mbarrier phase a bounded number of times; false = gave up.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t phase) {
  const uint32_t addr = smem_u32(bar);
  for (int it = 0; it < (1 << 22); ++it) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(addr), "r"(phase)
        : "memory");
    if (done) return true;
  }
  return false;
}

// One bulk copy global -> this CTA's shared memory (no multicast), completing
// `bytes` (multiple of 16, both addresses 16-byte aligned) on `bar`.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

template <typename KT, int D>
constexpr int attn_smem_bytes() {
  return 2 /*stages*/ * 2 /*K,V*/ * attn_tile<KT, D>() * D * static_cast<int>(sizeof(KT));
}

template <typename AT, typename KT, int D, int QT>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(AttnArgs a) {
  constexpr int DC = (D + 31) / 32;  // dims per lane in P.V
  constexpr bool kBulk = (D * sizeof(KT)) % 16 == 0;
  constexpr int kAttnTile = attn_tile<KT, D>();
  extern __shared__ __align__(128) unsigned char smem_raw[];
  KT *tiles = reinterpret_cast<KT *>(smem_raw);  // [stage][K|V][kAttnTile][D]
  __shared__ float qs[QT][D];
  __shared__ float s_m[kAttnWarps][QT], s_l[kAttnWarps][QT];
  __shared__ float s_acc[kAttnWarps][QT][D];
  __shared__ int s_pos[QT], s_req[QT], s_last;
  __shared__ __align__(8) uint64_t bars[2];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int ngt = (a.Q + QT - 1) / QT;
  const int g = blockIdx.x / ngt, qt = blockIdx.x % ngt;
  const int h = blockIdx.y, split = blockIdx.z;
  const int rq0 = g * a.Q + qt * QT;
  const int nq = max(0, min(QT, min(a.Q - qt * QT, a.R - rq0)));

  // query metadata and vectors, all loads in parallel
  if (threadIdx.x < QT) {
    const int i = threadIdx.x;
    const int rr = (i < nq) ? a.rows.req[rq0 + i] : -1;
    s_req[i] = rr;
    s_pos[i] = (rr >= 0) ? a.rows.pos[rq0 + i] : -1;
  }
  for (int idx = threadIdx.x; idx < QT * D; idx += blockDim.x) {
    const int i = idx / D, e = idx % D;
    qs[i][e] = (i < nq) ? to_f32(static_cast<const AT *>(a.q)[static_cast<size_t>(rq0 + i) * a.ldq + h * D + e]) : 0.f;
  }
  if (kBulk && threadIdx.x == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bars[0])) : "memory");
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bars[1])) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  int req = -1, maxpos = -1;
#pragma unroll
  for (int i = 0; i < QT; ++i)
    if (s_req[i] >= 0) {
      req = s_req[i];
      maxpos = max(maxpos, s_pos[i]);
    }
  if (req < 0 || maxpos >= a.S_cap) return;  // uniform over the block

  const int ctx = maxpos + 1;
  const int j0 = split * a.chunk, j1 = min(ctx, j0 + a.chunk);
  const int hk = h / (a.H / a.Hkv);
  const KT *kb = static_cast<const KT *>(a.kc) + static_cast<size_t>(req) * a.kv_req_stride + static_cast<size_t>(hk) * a.S_cap * D;
  const KT *vb = static_cast<const KT *>(a.vc) + static_cast<size_t>(req) * a.kv_req_stride + static_cast<size_t>(hk) * a.S_cap * D;
  const float scale = sqrtf(static_cast<float>(D));

  float m[QT], l[QT], acc[QT][DC];
  int qpos[QT];
#pragma unroll
  for (int i = 0; i < QT; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
    qpos[i] = s_pos[i];
#pragma unroll
    for (int c = 0; c < DC; ++c) acc[i][c] = 0.f;
  }

  const int ntiles = (j1 > j0) ? (j1 - j0 + kAttnTile - 1) / kAttnTile : 0;
  auto issue = [&](int t) {  // thread 0 only
    const int t0 = j0 + t * kAttnTile;
    const int nt = min(kAttnTile, j1 - t0);
    KT *kt = tiles + (t & 1) * 2 * kAttnTile * D;
    const uint32_t bytes = static_cast<uint32_t>(nt * D * sizeof(KT));
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(&bars[t & 1])), "r"(2 * bytes)
                 : "memory");
    bulk_g2s(kt, kb + static_cast<size_t>(t0) * D, bytes, &bars[t & 1]);
    bulk_g2s(kt + kAttnTile * D, vb + static_cast<size_t>(t0) * D, bytes, &bars[t & 1]);
  };
  if (kBulk && threadIdx.x == 0 && ntiles > 0) issue(0);
  bool ok = true;
  for (int t = 0; t < ntiles; ++t) {
    const int t0 = j0 + t * kAttnTile;
    const int nt = min(kAttnTile, j1 - t0);
    KT *ktile = tiles + (t & 1) * 2 * kAttnTile * D;
    KT *vtile = ktile + kAttnTile * D;
    if constexpr (kBulk) {
      if (threadIdx.x == 0 && t + 1 < ntiles) issue(t + 1);  // the other stage was released at the end of t-1
      ok = __syncthreads_and(mbar_wait(&bars[t & 1], (t >> 1) & 1) ? 1 : 0) != 0;
      if (!ok) break;
    } else {
      for (int idx = threadIdx.x; idx < nt * D; idx += blockDim.x) {
        ktile[idx] = kb[static_cast<size_t>(t0) * D + idx];
        vtile[idx] = vb[static_cast<size_t>(t0) * D + idx];
      }
      __syncthreads();
    }
    // scores: lane = position; the dot product walks the head dimension
    // rotated by the lane so the 32 lanes read 32 different banks
    const int tp = warp * 32 + lane;
    const int pos = t0 + tp;
    float p[QT];
    {
      float kr[D];
      if (tp < nt) {
#pragma unroll
        for (int c = 0; c < D; ++c) kr[c] = to_f32(ktile[tp * D + ((c + lane) % D)]);
      }
      float sc[QT];
#pragma unroll
      for (int i = 0; i < QT; ++i) {
        sc[i] = -INFINITY;
        if (i < nq && tp < nt && pos <= qpos[i]) {
          float dot = 0.f;
#pragma unroll
          for (int c = 0; c < D; ++c) dot = fmaf(qs[i][(c + lane) % D], kr[c], dot);
          sc[i] = __fdiv_rn(dot, scale);
        }
      }
      // tile maxima and sums of all queries, butterflies interleaved
      float tm[QT];
#pragma unroll
      for (int i = 0; i < QT; ++i) tm[i] = sc[i];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int i = 0; i < QT; ++i) tm[i] = fmaxf(tm[i], __shfl_xor_sync(0xffffffffu, tm[i], o));
      float ps[QT], alpha[QT];
#pragma unroll
      for (int i = 0; i < QT; ++i) {
        const float mnew = fmaxf(m[i], tm[i]);
        p[i] = (sc[i] == -INFINITY) ? 0.f : expf(sc[i] - mnew);
        alpha[i] = (m[i] == -INFINITY) ? 0.f : expf(m[i] - mnew);
        m[i] = mnew;
        ps[i] = p[i];
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int i = 0; i < QT; ++i) ps[i] += __shfl_xor_sync(0xffffffffu, ps[i], o);
#pragma unroll
      for (int i = 0; i < QT; ++i) {
        l[i] = l[i] * alpha[i] + ps[i];
#pragma unroll
        for (int c = 0; c < DC; ++c) acc[i][c] *= alpha[i];
      }
    }
    const int nvalid = max(0, min(32, nt - warp * 32));
    for (int pp = 0; pp < nvalid; ++pp) {
      float vv[DC];
#pragma unroll
      for (int c = 0; c < DC; ++c) {
        const int e = lane + 32 * c;
        vv[c] = (e < D) ? to_f32(vtile[(warp * 32 + pp) * D + e]) : 0.f;
      }
#pragma unroll
      for (int i = 0; i < QT; ++i) {
        const float pb = __shfl_sync(0xffffffffu, p[i], pp);
#pragma unroll
        for (int c = 0; c < DC; ++c) acc[i][c] = fmaf(pb, vv[c], acc[i][c]);
      }
    }
    __syncthreads();  // this stage is refilled two tiles later
  }
  if (!ok) {
    if (threadIdx.x == 0 && a.err) atomicOr(a.err, kErrTimeout);
    return;  // uniform: decided by the block vote
  }
  // merge the block's warps
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < QT; ++i) {
      s_m[warp][i] = m[i];
      s_l[warp][i] = l[i];
    }
  }
#pragma unroll
  for (int i = 0; i < QT; ++i)
#pragma unroll
    for (int c = 0; c < DC; ++c) {
      const int e = lane + 32 * c;
      if (e < D) s_acc[warp][i][e] = acc[i][c];
    }
  __syncthreads();
  for (int idx = threadIdx.x; idx < nq * D; idx += blockDim.x) {
    const int i = idx / D, e = idx % D;
    if (s_pos[i] < 0) continue;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, s_m[w][i]);
    float L = 0.f, A = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      if (s_m[w][i] == -INFINITY) continue;
      const float f = expf(s_m[w][i] - M);
      L += s_l[w][i] * f;
      A += s_acc[w][i][e] * f;
    }
    const int r = rq0 + i;
    if (a.nsplit == 1) {
      static_cast<AT *>(a.out)[static_cast<size_t>(r) * a.ldo + h * D + e] = from_f32<AT>(L > 0.f ? A / L : 0.f);
    } else {
      float *pp = a.part + ((static_cast<size_t>(r) * a.H + h) * a.nsplit + split) * (D + 2);
      pp[2 + e] = A;
      if (e == 0) {
        pp[0] = M;
        pp[1] = L;
      }
    }
  }
  if (a.nsplit == 1) return;
  // the last block of this (query tile, head) to arrive merges the splits
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    int *cnt = a.counters + static_cast<size_t>(rq0) * a.H + h;
    const int prev = atomicAdd(cnt, 1);
    s_last = (prev == a.nsplit - 1) ? 1 : 0;
    if (s_last) *cnt = 0;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int idx = threadIdx.x; idx < nq * D; idx += blockDim.x) {
    const int i = idx / D, e = idx % D;
    if (s_pos[i] < 0) continue;
    const int r = rq0 + i;
    const float *pp = a.part + (static_cast<size_t>(r) * a.H + h) * a.nsplit * (D + 2);
    float M = -INFINITY;
    for (int s = 0; s < a.nsplit; ++s)
      if (__ldcg(pp + s * (D + 2) + 1) > 0.f) M = fmaxf(M, __ldcg(pp + s * (D + 2)));
    float L = 0.f, A = 0.f;
    for (int s = 0; s < a.nsplit; ++s) {
      const float *ps = pp + s * (D + 2);
      const float ls = __ldcg(ps + 1);
      if (ls > 0.f) {
        const float w = expf(__ldcg(ps) - M);
        L += ls * w;
        A += __ldcg(ps + 2 + e) * w;
      }
    }
    static_cast<AT *>(a.out)[static_cast<size_t>(r) * a.ldo + h * D + e] = from_f32<AT>(L > 0.f ? A / L : 0.f);
  }
}

}  // namespace specdec
