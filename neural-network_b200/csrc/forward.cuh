// Forward-pass kernels of the decoder stack (target and draft share them).
//
// A forward pass runs over a batch of "rows": one row is one token of one
// request, at one cache position.  Prefill, a draft step, the (k+1)-token
// verify block and the draft catch-up are all row batches; row r carries
// (token, position, request) and request < 0 marks an unused row.  Every row
// writes its K/V at its own position before the attention kernel reads the
// cache, so causal attention over the cache is exactly the reference's
// masked attention over past + new tokens (src/nn/layer.cpp:842-952, mask
// j > S_past + i).
//
// Device layouts (all chosen for coalesced 16-byte streaming on B200):
//   weights     W^T [N][K] row-major (output-major), fp32 or int8 + fp32
//               per-output scale; the reference keeps W [K][N]
//               (src/nn/layer.cpp:153) and the loader transposes.
//   QKV         one [d + 2*kvd][d] matrix (q rows, k rows, v rows).
//   SwiGLU      gate/up interleaved: row 2c = gate_c, row 2c+1 = up_c.
//   activations [R][d] in the activation dtype (fp32 or bf16).
//   KV cache    [layer][request slot][kv head][position][D].
#pragma once

#include "common.cuh"

namespace specdec {

struct RowsView {
  const int *tok;
  const int *pos;
  const int *req;
};

// ---------------------------------------------------------------------------
// Embedding gather (Embedding::forward -> CpuBackend::embedding,
// src/backend/cpu_backend.cpp:998-1033: an out-of-range id reads row 0).  The
// cfg architecture adds the learned position row.
template <typename AT>
__global__ void embed_kernel(RowsView rows, int R, const float *__restrict__ emb,
                             const float *__restrict__ pos_emb, int V, int d, int max_pos,
                             AT *__restrict__ x) {
  const int r = blockIdx.x;
  if (r >= R) return;
  int id = rows.tok[r];
  if (id < 0 || id >= V) id = 0;
  int p = rows.pos[r];
  p = p < 0 ? 0 : (p >= max_pos ? max_pos - 1 : p);
  const float *e = emb + static_cast<size_t>(id) * d;
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    float v = e[i];
    if (pos_emb) v += pos_emb[static_cast<size_t>(p) * d + i];
    x[static_cast<size_t>(r) * d + i] = from_f32<AT>(v);
  }
}

// ---------------------------------------------------------------------------
// Linear layer y = x . W + b on CUDA cores, for the small row counts of
// draft steps and verify blocks.  Each warp owns a PAIR of adjacent output
// columns (so RoPE pairs and SwiGLU gate/up pairs land in one lane) for a tile
// of kRowTile rows; lanes split K in 16-byte weight vectors.
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
  const void *x;       // activations
  int ldx;
  const int *in_rows;  // optional: logical row r reads x row in_rows[r]
  int R;
  const void *W;       // [N][K]
  const float *scale;  // [N] or null
  const float *bias;   // [N] (interleaved like W for SwiGLU)
  int N, K;
  void *out;
  int ldo;
  const void *resid;
  int ldr;
  RowsView rows;       // for kEpiQKV
  QKVArgs qkv;
};

constexpr int kLinWarps = 8;
constexpr int kRowTile = 8;

template <typename WT> struct WVec;
template <> struct WVec<float> { static constexpr int E = 4; };
template <> struct WVec<int8_t> { static constexpr int E = 16; };
template <> struct WVec<__nv_bfloat16> { static constexpr int E = 8; };

__device__ __forceinline__ void unpack_w(const float4 &raw, float (&w)[4]) {
  w[0] = raw.x; w[1] = raw.y; w[2] = raw.z; w[3] = raw.w;
}
__device__ __forceinline__ void unpack_w(const int4 &raw, float (&w)[16]) {
  const int v[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int b = 0; b < 4; ++b) w[4 * i + b] = static_cast<float>(static_cast<int8_t>((v[i] >> (8 * b)) & 0xff));
  }
}

template <typename AT>
__device__ __forceinline__ float load_act(const AT *p) { return to_f32(*p); }

template <typename AT, int E>
__device__ __forceinline__ void load_x(const AT *p, float (&xv)[E]) {
  if constexpr (sizeof(AT) == 4) {
#pragma unroll
    for (int i = 0; i < E; i += 4) {
      float4 t = __ldg(reinterpret_cast<const float4 *>(p + i));
      xv[i] = t.x; xv[i + 1] = t.y; xv[i + 2] = t.z; xv[i + 3] = t.w;
    }
  } else if constexpr (E == 4) {
    uint2 t = __ldg(reinterpret_cast<const uint2 *>(p));
    const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&t);
    float2 f0 = __bfloat1622float2(h[0]), f1 = __bfloat1622float2(h[1]);
    xv[0] = f0.x; xv[1] = f0.y; xv[2] = f1.x; xv[3] = f1.y;
  } else {
#pragma unroll
    for (int i = 0; i < E; i += 8) {
      int4 t = __ldg(reinterpret_cast<const int4 *>(p + i));
      const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&t);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = __bfloat1622float2(h[j]);
        xv[i + 2 * j] = f.x; xv[i + 2 * j + 1] = f.y;
      }
    }
  }
}

template <typename AT, int EPI>
__device__ __forceinline__ void linear_epilogue(const LinearArgs &a, int r, int n, float v0, float v1) {
  const bool has1 = (n + 1) < a.N;
  if (a.scale) {
    v0 *= a.scale[n];
    if (has1) v1 *= a.scale[n + 1];
  }
  v0 += a.bias[n];
  if (has1) v1 += a.bias[n + 1];
  if constexpr (EPI == kEpiStore || EPI == kEpiResid || EPI == kEpiGelu) {
    if constexpr (EPI == kEpiResid) {
      const AT *rs = static_cast<const AT *>(a.resid) + static_cast<size_t>(r) * a.ldr;
      v0 = v0 + to_f32(rs[n]);
      if (has1) v1 = v1 + to_f32(rs[n + 1]);
    }
    if constexpr (EPI == kEpiGelu) {
      v0 = 0.5f * v0 * (1.0f + erff(v0 * 0.70710678118654752f));
      v1 = 0.5f * v1 * (1.0f + erff(v1 * 0.70710678118654752f));
    }
    AT *o = static_cast<AT *>(a.out) + static_cast<size_t>(r) * a.ldo;
    o[n] = from_f32<AT>(v0);
    if (has1) o[n + 1] = from_f32<AT>(v1);
  } else if constexpr (EPI == kEpiSwiGLU) {
    // SwiGLU::forward (src/nn/layer.cpp:1704-1710): (g * sigmoid(g)) * up,
    // sigmoid = 1 / (1 + exp(-g)) (src/backend/cpu_backend.cpp:487-488).
    const float g = v0, u = v1;
    const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
    AT *o = static_cast<AT *>(a.out) + static_cast<size_t>(r) * a.ldo;
    o[n >> 1] = from_f32<AT>(__fmul_rn(__fmul_rn(g, sg), u));
  } else if constexpr (EPI == kEpiQKV) {
    const int req = a.rows.req[r];
    if (req < 0) return;
    const int pos = a.rows.pos[r];
    const QKVArgs &q = a.qkv;
    if (pos < 0 || pos >= q.S_cap || pos >= q.rope_max_pos) {
      if (q.err) atomicOr(q.err, kErrSeqLen);
      return;
    }
    if (n < q.d + q.kvd) {
      // Tensor::rope (src/core/tensor.cpp:1144-1163): pair (2j, 2j+1) of each
      // head rotated by pos * 10000^(-2j/D); the (cos, sin) table is computed
      // on the host with the reference's float formula.
      const int e = (n < q.d ? n : n - q.d) % q.D;
      const float2 cs = q.rope[static_cast<size_t>(pos) * (q.D / 2) + (e >> 1)];
      const float r0 = __fsub_rn(__fmul_rn(v0, cs.x), __fmul_rn(v1, cs.y));
      const float r1 = __fadd_rn(__fmul_rn(v0, cs.y), __fmul_rn(v1, cs.x));
      v0 = r0;
      v1 = r1;
    }
    if (n < q.d) {
      AT *o = static_cast<AT *>(a.out) + static_cast<size_t>(r) * a.ldo;
      o[n] = from_f32<AT>(v0);
      o[n + 1] = from_f32<AT>(v1);
    } else {
      const bool is_k = n < q.d + q.kvd;
      const int nn = is_k ? n - q.d : n - q.d - q.kvd;
      const int h = nn / q.D, e = nn % q.D;
      const size_t off = static_cast<size_t>(req) * q.kv_req_stride +
                         (static_cast<size_t>(h) * q.S_cap + pos) * q.D + e;
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

// grid: (ceil(N / (2*kLinWarps)), ceil(R / kRowTile)); block: 32*kLinWarps.
template <typename WT, typename AT, int EPI>
__global__ void __launch_bounds__(32 * kLinWarps) linear_kernel(LinearArgs a) {
  constexpr int E = WVec<WT>::E;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n0 = (blockIdx.x * kLinWarps + warp) * 2;
  const int r0 = blockIdx.y * kRowTile;
  if (n0 >= a.N) return;
  const bool has1 = (n0 + 1) < a.N;
  const int nrows = min(kRowTile, a.R - r0);

  const WT *w0 = static_cast<const WT *>(a.W) + static_cast<size_t>(n0) * a.K;
  const WT *w1 = has1 ? w0 + a.K : w0;
  const AT *xrow[kRowTile];
#pragma unroll
  for (int i = 0; i < kRowTile; ++i) {
    int lr = r0 + (i < nrows ? i : 0);
    int pr = a.in_rows ? a.in_rows[lr] : lr;
    xrow[i] = static_cast<const AT *>(a.x) + static_cast<size_t>(pr) * a.ldx;
  }

  float acc0[kRowTile], acc1[kRowTile];
#pragma unroll
  for (int i = 0; i < kRowTile; ++i) acc0[i] = acc1[i] = 0.f;

  // 16-byte vector path when rows of W and x are 16-byte aligned.
  const bool vec_ok = ((a.K * static_cast<int>(sizeof(WT))) % 16 == 0) &&
                      ((a.ldx * static_cast<int>(sizeof(AT))) % 16 == 0) &&
                      ((reinterpret_cast<uintptr_t>(a.x) & 15) == 0);
  const int kvec = vec_ok ? a.K / E : 0;
  for (int v = lane; v < kvec; v += 32) {
    float wa[E], wb[E];
    if constexpr (sizeof(WT) == 4) {
      unpack_w(__ldg(reinterpret_cast<const float4 *>(w0) + v), wa);
      unpack_w(__ldg(reinterpret_cast<const float4 *>(w1) + v), wb);
    } else if constexpr (sizeof(WT) == 1) {
      unpack_w(__ldg(reinterpret_cast<const int4 *>(w0) + v), wa);
      unpack_w(__ldg(reinterpret_cast<const int4 *>(w1) + v), wb);
    }
#pragma unroll
    for (int i = 0; i < kRowTile; ++i) {
      if (i < nrows) {
        float xv[E];
        load_x<AT, E>(xrow[i] + v * E, xv);
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) {
          s0 = fmaf(xv[e], wa[e], s0);
          s1 = fmaf(xv[e], wb[e], s1);
        }
        acc0[i] += s0;
        acc1[i] += s1;
      }
    }
  }
  // scalar tail (and the whole K when rows are not 16-byte aligned)
  for (int k = kvec * E + lane; k < a.K; k += 32) {
    const float wa = static_cast<float>(w0[k]);
    const float wb = static_cast<float>(w1[k]);
#pragma unroll
    for (int i = 0; i < kRowTile; ++i) {
      if (i < nrows) {
        const float xv = load_act(xrow[i] + k);
        acc0[i] = fmaf(xv, wa, acc0[i]);
        acc1[i] = fmaf(xv, wb, acc1[i]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kRowTile; ++i) {
    acc0[i] = warp_sum(acc0[i]);
    acc1[i] = warp_sum(acc1[i]);
  }
  // lane i finishes row i
#pragma unroll
  for (int i = 0; i < kRowTile; ++i) {
    if (lane == i && i < nrows) linear_epilogue<AT, EPI>(a, r0 + i, n0, acc0[i], acc1[i]);
  }
}

// ---------------------------------------------------------------------------
// Residual LayerNorm (LayerNorm::forward, src/nn/layer.cpp:242-261):
// mean = sum/N, var = sum((x-mean)^2)/N, y = ((x-mean)/sqrt(var+eps))*g + b.
// One block per row; the row is held in registers (d <= 32 * blockDim).
template <typename AT>
__global__ void layernorm_kernel(const AT *__restrict__ in, int ldi, int R, int d,
                                 const float *__restrict__ g, const float *__restrict__ b,
                                 AT *__restrict__ out, int ldo) {
  __shared__ float red[32];
  const int r = blockIdx.x;
  if (r >= R) return;
  constexpr int kMax = 32;
  float v[kMax];
  const AT *x = in + static_cast<size_t>(r) * ldi;
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kMax; ++i) {
    int c = threadIdx.x + i * blockDim.x;
    v[i] = (c < d) ? to_f32(x[c]) : 0.f;
    s += v[i];
  }
  const float N = static_cast<float>(d);
  const float mean = __fdiv_rn(block_sum(s, red), N);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < kMax; ++i) {
    int c = threadIdx.x + i * blockDim.x;
    if (c < d) {
      float df = v[i] - mean;
      q = fmaf(df, df, q);
    }
  }
  const float var = __fdiv_rn(block_sum(q, red), N);
  const float sd = sqrtf(var + 1e-5f);
  AT *y = out + static_cast<size_t>(r) * ldo;
#pragma unroll
  for (int i = 0; i < kMax; ++i) {
    int c = threadIdx.x + i * blockDim.x;
    if (c < d) y[c] = from_f32<AT>(__fadd_rn(__fmul_rn(__fdiv_rn(v[i] - mean, sd), g[c]), b[c]));
  }
}

// ---------------------------------------------------------------------------
// Causal attention of each row over its request's cache, positions
// [0, pos] (split into chunks of `chunk` positions across blockIdx.z).
// score = (q . k) / sqrt(D) (src/nn/layer.cpp:870, 891-897), softmax, P.V.
// With one split the block writes the normalised output; otherwise it writes
// (max, sum, unnormalised acc[D]) to `part` and attn_combine_kernel merges.
constexpr int kAttnThreads = 128;

template <typename AT, typename KT>
__global__ void __launch_bounds__(kAttnThreads)
attention_kernel(const AT *__restrict__ q, int ldq, RowsView rows, int R, const KT *__restrict__ kc,
                 const KT *__restrict__ vc, size_t kv_req_stride, int S_cap, int H, int Hkv, int D,
                 int chunk, AT *__restrict__ out, int ldo, float *__restrict__ part) {
  extern __shared__ float sm[];
  float *qs = sm;                    // [D]
  float *sc = qs + D;                // [kAttnThreads]
  float *accs = sc + kAttnThreads;   // [kAttnThreads] partial accumulators
  __shared__ float red[32];

  const int r = blockIdx.x, h = blockIdx.y, split = blockIdx.z, nsplit = gridDim.z;
  const int req = rows.req[r];
  const int pos = rows.pos[r];
  const int tid = threadIdx.x;
  const bool valid = req >= 0 && pos >= 0 && pos < S_cap;
  const int ctx = valid ? pos + 1 : 0;
  const int j0 = split * chunk;
  const int j1 = min(ctx, j0 + chunk);

  const int hk = h / (H / Hkv);
  const KT *kbase = kc + (valid ? static_cast<size_t>(req) * kv_req_stride : 0) + static_cast<size_t>(hk) * S_cap * D;
  const KT *vbase = vc + (valid ? static_cast<size_t>(req) * kv_req_stride : 0) + static_cast<size_t>(hk) * S_cap * D;

  for (int e = tid; e < D; e += blockDim.x) qs[e] = valid ? to_f32(q[static_cast<size_t>(r) * ldq + h * D + e]) : 0.f;
  __syncthreads();

  const float scale = sqrtf(static_cast<float>(D));
  float m = -INFINITY, l = 0.f;
  // PV layout: G = blockDim / D groups of D threads; thread (grp, e).
  const int G = blockDim.x / D;
  const int grp = tid / D, e = tid % D;
  float acc = 0.f;

  for (int t0 = j0; t0 < j1; t0 += blockDim.x) {
    const int j = t0 + tid;
    float s = -INFINITY;
    if (j < j1) {
      const KT *kr = kbase + static_cast<size_t>(j) * D;
      float dot = 0.f;
      for (int c = 0; c < D; ++c) dot = fmaf(qs[c], to_f32(kr[c]), dot);
      s = __fdiv_rn(dot, scale);
    }
    const float tmax = block_max(s, red);
    const float mnew = fmaxf(m, tmax);
    const float p = (j < j1) ? expf(s - mnew) : 0.f;
    sc[tid] = p;
    const float psum = block_sum(p, red);  // includes a __syncthreads after sc writes
    const float alpha = (m == -INFINITY) ? 0.f : expf(m - mnew);
    l = l * alpha + psum;
    m = mnew;
    acc *= alpha;
    const int nt = min(static_cast<int>(blockDim.x), j1 - t0);
    if (grp < G) {
      for (int t = grp; t < nt; t += G) acc = fmaf(sc[t], to_f32(vbase[static_cast<size_t>(t0 + t) * D + e]), acc);
    }
    __syncthreads();
  }
  // merge the G groups
  accs[tid] = acc;
  __syncthreads();
  if (tid < D) {
    float a = 0.f;
    for (int g2 = 0; g2 < G; ++g2) a += accs[g2 * D + tid];
    if (nsplit == 1) {
      if (valid) out[static_cast<size_t>(r) * ldo + h * D + tid] = from_f32<AT>(l > 0.f ? a / l : 0.f);
    } else {
      float *pp = part + ((static_cast<size_t>(r) * H + h) * nsplit + split) * (D + 2);
      pp[2 + tid] = a;
      if (tid == 0) { pp[0] = m; pp[1] = l; }
    }
  }
}

template <typename AT>
__global__ void attn_combine_kernel(const float *__restrict__ part, RowsView rows, int R, int H, int D,
                                    int nsplit, AT *__restrict__ out, int ldo) {
  const int r = blockIdx.x, h = blockIdx.y;
  if (rows.req[r] < 0) return;
  const float *pp = part + (static_cast<size_t>(r) * H + h) * nsplit * (D + 2);
  float M = -INFINITY;
  for (int s = 0; s < nsplit; ++s)
    if (pp[s * (D + 2) + 1] > 0.f) M = fmaxf(M, pp[s * (D + 2)]);
  for (int e = threadIdx.x; e < D; e += blockDim.x) {
    float L = 0.f, A = 0.f;
    for (int s = 0; s < nsplit; ++s) {
      const float *ps = pp + s * (D + 2);
      if (ps[1] > 0.f) {
        const float w = expf(ps[0] - M);
        L += ps[1] * w;
        A += ps[2 + e] * w;
      }
    }
    out[static_cast<size_t>(r) * ldo + h * D + e] = from_f32<AT>(L > 0.f ? A / L : 0.f);
  }
}

}  // namespace specdec
