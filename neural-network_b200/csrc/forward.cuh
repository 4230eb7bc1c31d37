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

#include <cooperative_groups.h>
#include <cuda.h>

#include <type_traits>

#include "common.cuh"

namespace specdec {

struct RowsView {
  const int *tok;  // embedding row (clamped to [0, V) by whoever wrote the row)
  const int *pos;  // RoPE position
  const int *req;
  // Token trees (all null otherwise): the cache row the row's K/V go to, and
  // its visibility: cache rows <= slot that are below tb, or whose bit
  // (row - tb) is set in mask (the row's ancestors and itself).
  const int *slot;
  const int *tb;
  const unsigned long long *mask;
};
__device__ __forceinline__ int row_slot(const RowsView &rv, int r) { return rv.slot ? rv.slot[r] : rv.pos[r]; }

// Paged KV cache.  A layer's K (or V) cache is a pool of pages; a page holds
// kKvPage consecutive positions of one request for all its kv heads,
// [Hkv][kKvPage][D].  Request q's position p lives in page
// pt[q * ppr + p / kKvPage] (-1: no page), at cache row
// (page * Hkv + head) * kKvPage + p % kKvPage -- the y coordinate of the
// attention kernels' TMA views and the index of the int8 scale planes.  The
// attention tiles (64 or 128 positions, starting at multiples of their size)
// never straddle a page, so a tile is one TMA box of one page.
constexpr int kKvPage = 128;
struct KvPages {
  const int *pt;  // [slot][ppr] page ids
  int ppr;        // pages per slot
};
__device__ __forceinline__ int kv_page(const KvPages &pg, int req, int pos) {
  return __ldg(pg.pt + static_cast<size_t>(req) * pg.ppr + pos / kKvPage);
}
// Cache row of (request, kv head, position); -1 when the position has no page.
__device__ __forceinline__ int kv_row(const KvPages &pg, int Hkv, int req, int h, int pos) {
  const int page = kv_page(pg, req, pos);
  return page < 0 ? -1 : (page * Hkv + h) * kKvPage + pos % kKvPage;
}

// ---------------------------------------------------------------------------
// Embedding gather (Embedding::forward -> CpuBackend::embedding,
// src/backend/cpu_backend.cpp:998-1033: an out-of-range id reads row 0).  The
// cfg architecture adds the learned position row.  One block per row.
template <typename AT>
__global__ void embed_kernel(RowsView rows, int R, const float *__restrict__ emb, const float *__restrict__ pos_emb,
                             int d, int max_pos, AT *__restrict__ x) {
  pdl_launch();
  pdl_wait();
  const int r = blockIdx.x;
  if (r >= R) return;
  const int id = rows.tok[r];
  const int p = min(max(rows.pos[r], 0), max_pos - 1);
  for (int c = threadIdx.x; c < d; c += blockDim.x) {
    float t = emb[static_cast<size_t>(id) * d + c];
    if (pos_emb) t += pos_emb[static_cast<size_t>(p) * d + c];
    x[static_cast<size_t>(r) * d + c] = from_f32<AT>(t);
  }
}

// ---------------------------------------------------------------------------
// Linear layer y = x . W + b on CUDA cores for the small row counts of draft
// steps and verify blocks (a GEMV per tile of kRowTile rows).
//
// A warp owns four adjacent output columns, i.e. two whole pairs (RoPE pairs
// and SwiGLU gate/up pairs each land in one lane), for kRowTile rows, so each
// input vector it loads feeds four weight columns; `ksplit` warps of a block
// share the four columns and split K, so each lane issues its weight and input
// vectors in one go.  A 32-value warp reduce-scatter leaves every lane one
// finished (row, column).  Everything the epilogue needs (scale, bias,
// residual, row position, RoPE factors) is loaded before the dot products.
//
// LayerNorm is applied by the consumer: with `in_g` set, each block first
// normalises its kRowTile input rows into shared memory (every block holds
// the full rows it multiplies, so a row's statistics never cross blocks),
// and the blocks of column 0 store the normalised rows for the residual
// that follows.  No kernel waits on another block's output and no separate
// norm kernel runs.
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
  void *kc, *vc;             // this layer's page pools
  KvPages pg;                // the requests' page tables
  int S_cap;                 // positions per request
  int kv_mode;               // cache element type: 0 fp32, 1 bf16, 2 int8 (rows staged for kv_quant_kernel)
  float *stage;              // kv_mode 2: [R][2 * kvd] fp32 K and V of this pass's rows
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
  const float *in_g, *in_b;  // optional LayerNorm of the input rows (over K) before the product ...
  void *norm_out;            // ... whose normalised rows the blocks of column 0 also store here (leading dim K)
  int ksplit;                // warps per column pair: 1, 2, 4 or 8
};

constexpr int kLinWarps = 8;
constexpr int kRowTile = 8;
constexpr int kLinColsMax = 4;  // output columns per warp: one pair, or two adjacent pairs

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

// Reduce-scatter of NV (16 or 32) per-lane partial sums over the warp: at
// each halving, lanes with the offset bit set keep the upper half and send the
// lower one.  Afterwards lane l holds the full sum of value l / (32 / NV)
// (with NV = 16 the two lanes of a value agree after a final butterfly).
template <int NV>
__device__ __forceinline__ float warp_reduce_scatter(const float (&v)[NV]) {
  static_assert(NV == 16 || NV == 32, "16 or 32 values");
  const int lane = threadIdx.x & 31;
  float a16[16];
  if constexpr (NV == 32) {
    const bool hi = lane & 16;
#pragma unroll
    for (int i = 0; i < 16; ++i)
      a16[i] = (hi ? v[i + 16] : v[i]) + __shfl_xor_sync(0xffffffffu, hi ? v[i] : v[i + 16], 16);
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) a16[i] = v[i];
  }
  constexpr int o8 = NV == 32 ? 8 : 16, o4 = o8 / 2, o2 = o4 / 2, o1 = o2 / 2;
  float a8[8];
  {
    const bool hi = lane & o8;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      a8[i] = (hi ? a16[i + 8] : a16[i]) + __shfl_xor_sync(0xffffffffu, hi ? a16[i] : a16[i + 8], o8);
  }
  float a4[4];
  {
    const bool hi = lane & o4;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      a4[i] = (hi ? a8[i + 4] : a8[i]) + __shfl_xor_sync(0xffffffffu, hi ? a8[i] : a8[i + 4], o4);
  }
  float a2[2];
  {
    const bool hi = lane & o2;
#pragma unroll
    for (int i = 0; i < 2; ++i)
      a2[i] = (hi ? a4[i + 2] : a4[i]) + __shfl_xor_sync(0xffffffffu, hi ? a4[i] : a4[i + 2], o2);
  }
  const bool hi = lane & o1;
  float r = (hi ? a2[1] : a2[0]) + __shfl_xor_sync(0xffffffffu, hi ? a2[0] : a2[1], o1);
  if constexpr (NV == 16) r += __shfl_xor_sync(0xffffffffu, r, 1);
  return r;
}

// E consecutive input elements as fp32 (kShared: p points into shared memory).
template <typename AT, int E, bool kShared>
__device__ __forceinline__ void load_xvec(const AT *p, float (&xv)[E]) {
  if constexpr (sizeof(AT) == 4) {
#pragma unroll
    for (int i = 0; i < E; i += 4) {
      const float4 t = kShared ? *reinterpret_cast<const float4 *>(p + i) : __ldg(reinterpret_cast<const float4 *>(p + i));
      xv[i] = t.x; xv[i + 1] = t.y; xv[i + 2] = t.z; xv[i + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < E; i += 4) {
      const uint2 t = kShared ? *reinterpret_cast<const uint2 *>(p + i) : __ldg(reinterpret_cast<const uint2 *>(p + i));
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
  int req, pos, slot;
};

// Per-column operands (weights' scale and bias): no kernel writes them.
__device__ __forceinline__ void epilogue_prefetch_cols(const LinearArgs &a, int n, EpiPre &p) {
  const bool has1 = (n + 1) < a.N;
  p.s0 = a.scale ? __ldg(a.scale + n) : 1.f;
  p.s1 = (a.scale && has1) ? __ldg(a.scale + n + 1) : 1.f;
  p.b0 = __ldg(a.bias + n);
  p.b1 = has1 ? __ldg(a.bias + n + 1) : 0.f;
}

// Per-row operands (residual, row position, RoPE factors): written by earlier
// kernels of the pass.
template <typename AT, int EPI>
__device__ __forceinline__ void epilogue_prefetch_rows(const LinearArgs &a, int r, int n, EpiPre &p) {
  const bool has1 = (n + 1) < a.N;
  p.r0 = p.r1 = 0.f;
  p.c = 1.f;
  p.sn = 0.f;
  p.req = 0;
  p.pos = 0;
  p.slot = 0;
  if constexpr (EPI == kEpiResid) {
    const AT *rs = static_cast<const AT *>(a.resid) + static_cast<size_t>(r) * a.ldr;
    p.r0 = to_f32(rs[n]);
    p.r1 = has1 ? to_f32(rs[n + 1]) : 0.f;
  }
  if constexpr (EPI == kEpiQKV) {
    const QKVArgs &q = a.qkv;
    p.req = a.rows.req[r];
    p.pos = a.rows.pos[r];
    p.slot = row_slot(a.rows, r);
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
    const int pos = p.pos, slot = p.slot;
    if (pos < 0 || pos >= q.rope_max_pos || slot < 0 || slot >= q.S_cap) {
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
      const int row = kv_row(q.pg, q.kvd / q.D, p.req, h, slot);
      if (row < 0) {
        if (q.err) atomicOr(q.err, kErrSeqLen);
        return;
      }
      const size_t off = static_cast<size_t>(row) * q.D + e;
      if (q.kv_mode == 2) {
        float *st = q.stage + static_cast<size_t>(r) * 2 * q.kvd + (is_k ? 0 : q.kvd) + nn;
        st[0] = v0;
        st[1] = v1;
      } else if (q.kv_mode == 1) {
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

// grid: (ceil(N / (NC * kLinWarps / ksplit)), ceil(R / kRowTile)); block: 32 * kLinWarps.
// NC: output columns per warp (2 or 4).  IN_LN: dynamic shared memory of
// kRowTile * K activation elements holds the block's normalised input rows.
template <typename WT, typename AT, int EPI, bool IN_LN, int NC>
__global__ void __launch_bounds__(32 * kLinWarps, 2) linear_kernel(LinearArgs a) {
  constexpr int E = WVec<WT>::E;
  constexpr int NV = kRowTile * NC;  // partial sums per lane
  constexpr int LPV = 32 / NV;       // lanes holding each finished value
  static_assert(NC == 2 || NC == 4, "one or two column pairs per warp");
  __shared__ float s_red[kLinWarps][32];
  extern __shared__ __align__(16) unsigned char lin_smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int ks = a.ksplit;
  const int quads = kLinWarps / ks;
  const int quad = warp / ks, kidx = warp % ks;
  const int n0 = (blockIdx.x * quads + quad) * NC;
  const int r0 = blockIdx.y * kRowTile;
  const int nrows = min(kRowTile, a.R - r0);
  const bool col_ok = n0 < a.N;

  // After the reduction lane l holds value l / LPV = (row, column n0 + c) with
  // value = row * NC + c; one lane of each even column finishes the pair
  // (n, n + 1) of its row.
  const int vi = lane / LPV;
  const int er = vi / NC, en = n0 + vi % NC;
  const bool epi_lane = col_ok && kidx == 0 && !((vi % NC) & 1) && (lane % LPV) == 0 && en < a.N && er < nrows;
  EpiPre pre{};
  if (epi_lane) epilogue_prefetch_cols(a, en, pre);

  const WT *wc[NC];
#pragma unroll
  for (int c = 0; c < NC; ++c) wc[c] = static_cast<const WT *>(a.W) + static_cast<size_t>(min(n0 + c, a.N - 1)) * a.K;
  const int ldx = IN_LN ? a.K : a.ldx;
  const bool vec_ok = (a.K % E == 0) && (ldx % 4 == 0);
  const int kvec = vec_ok ? a.K / E : 0;
  const int vstart = kidx * 32 + lane;
  // the first K step's weights are requested before anything else, so their
  // latency overlaps the input rows (and their LayerNorm)
  float wf[NC][E];
  const bool first = col_ok && vstart < kvec;
  if (first) {
#pragma unroll
    for (int c = 0; c < NC; ++c) load_wvec(wc[c] + vstart * E, wf[c]);
  }
  // everything above reads weights only; the rows come from earlier kernels
  pdl_wait();
  if (epi_lane) epilogue_prefetch_rows<AT, EPI>(a, r0 + er, en, pre);

  const AT *xrow[kRowTile];
  if constexpr (IN_LN) {
    // LayerNorm::forward (src/nn/layer.cpp:242-261; eps 1e-5, biased
    // variance) of the input rows, warp i normalising row i with fp32
    // statistics; the normalised row is rounded to the activation type.
    // Columns c = lane + 32 j; the first kLnChunk of them per lane (all of a
    // 256-wide row) keep x, gamma and beta in registers, loaded together.
    constexpr int kLnChunk = 8;
    AT *s_x = reinterpret_cast<AT *>(lin_smem);
    if (warp < nrows) {
      const int lr = r0 + warp;
      const int pr = a.in_rows ? a.in_rows[lr] : lr;
      const AT *x = static_cast<const AT *>(a.x) + static_cast<size_t>(pr) * a.ldx;
      AT *y = s_x + warp * a.K;
      float xv[kLnChunk], gv[kLnChunk], bv[kLnChunk];
#pragma unroll
      for (int j = 0; j < kLnChunk; ++j) {
        const int c = lane + 32 * j;
        const bool in = c < a.K;
        xv[j] = in ? to_f32(x[c]) : 0.f;
        gv[j] = in ? __ldg(a.in_g + c) : 0.f;
        bv[j] = in ? __ldg(a.in_b + c) : 0.f;
      }
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < kLnChunk; ++j) s += xv[j];
      for (int c = lane + 32 * kLnChunk; c < a.K; c += 32) {
        const AT v = x[c];
        y[c] = v;
        s += to_f32(v);
      }
      const float mean = __fdiv_rn(warp_sum(s), static_cast<float>(a.K));
      float q = 0.f;
#pragma unroll
      for (int j = 0; j < kLnChunk; ++j) {
        if (lane + 32 * j < a.K) {
          const float df = xv[j] - mean;
          q = fmaf(df, df, q);
        }
      }
      for (int c = lane + 32 * kLnChunk; c < a.K; c += 32) {
        const float df = to_f32(y[c]) - mean;
        q = fmaf(df, df, q);
      }
      const float sd = sqrtf(__fdiv_rn(warp_sum(q), static_cast<float>(a.K)) + 1e-5f);
      AT *no = (a.norm_out && blockIdx.x == 0) ? static_cast<AT *>(a.norm_out) + static_cast<size_t>(lr) * a.K : nullptr;
#pragma unroll
      for (int j = 0; j < kLnChunk; ++j) {
        const int c = lane + 32 * j;
        if (c < a.K) {
          const AT v = from_f32<AT>(__fadd_rn(__fmul_rn(__fdiv_rn(xv[j] - mean, sd), gv[j]), bv[j]));
          y[c] = v;
          if (no) no[c] = v;
        }
      }
      for (int c = lane + 32 * kLnChunk; c < a.K; c += 32) {
        const AT v = from_f32<AT>(
            __fadd_rn(__fmul_rn(__fdiv_rn(to_f32(y[c]) - mean, sd), __ldg(a.in_g + c)), __ldg(a.in_b + c)));
        y[c] = v;
        if (no) no[c] = v;
      }
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kRowTile; ++i) xrow[i] = s_x + (i < nrows ? i : 0) * a.K;
  } else {
#pragma unroll
    for (int i = 0; i < kRowTile; ++i) {
      const int lr = r0 + (i < nrows ? i : 0);
      const int pr = a.in_rows ? a.in_rows[lr] : lr;
      xrow[i] = static_cast<const AT *>(a.x) + static_cast<size_t>(pr) * a.ldx;
    }
  }

  float acc[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) acc[i] = 0.f;
  // The input vectors of RB rows are requested together before their FMAs
  // (one memory round trip per group): all rows with one column pair, half of
  // them with two pairs to stay within the register budget.
  constexpr int RB = NC == 2 ? kRowTile : kRowTile / 2;
  auto step = [&](int v, const float (&w)[NC][E]) {
#pragma unroll
    for (int h0 = 0; h0 < kRowTile; h0 += RB) {
      float xv[RB][E];
#pragma unroll
      for (int i = 0; i < RB; ++i)
        if (h0 + i < nrows) load_xvec<AT, E, IN_LN>(xrow[h0 + i] + v * E, xv[i]);
#pragma unroll
      for (int i = 0; i < RB; ++i) {
        if (h0 + i < nrows) {
#pragma unroll
          for (int c = 0; c < NC; ++c) {
            float t = 0.f;
#pragma unroll
            for (int e = 0; e < E; ++e) t = fmaf(xv[i][e], w[c][e], t);
            acc[(h0 + i) * NC + c] += t;
          }
        }
      }
    }
  };
  if (col_ok) {
    if (first) step(vstart, wf);
#pragma unroll 2
    for (int v = vstart + 32 * ks; v < kvec; v += 32 * ks) {
      float w[NC][E];
#pragma unroll
      for (int c = 0; c < NC; ++c) load_wvec(wc[c] + v * E, w[c]);
      step(v, w);
    }
    for (int k = kvec * E + kidx * 32 + lane; k < a.K; k += 32 * ks) {  // scalar tail / unaligned rows
      float wk[NC];
#pragma unroll
      for (int c = 0; c < NC; ++c) wk[c] = static_cast<float>(wc[c][k]);
#pragma unroll
      for (int i = 0; i < kRowTile; ++i)
        if (i < nrows) {
          const float xv = to_f32(xrow[i][k]);
#pragma unroll
          for (int c = 0; c < NC; ++c) acc[i * NC + c] = fmaf(xv, wk[c], acc[i * NC + c]);
        }
    }
  }
  pdl_launch();  // the successor may start fetching its weights during the reduction
  float tot = warp_reduce_scatter<NV>(acc);
  if (ks > 1) {
    s_red[warp][lane] = tot;
    __syncthreads();
    if (kidx == 0) {
      float t = 0.f;
      for (int j = 0; j < ks; ++j) t += s_red[warp + j][lane];
      tot = t;
    }
  }
  const float tot1 = __shfl_xor_sync(0xffffffffu, tot, LPV);  // column n + 1 of the same row
  if (epi_lane) linear_epilogue<AT, EPI>(a, r0 + er, en, tot, tot1, pre);
}

// ---------------------------------------------------------------------------
// int8 KV append: quantize_kv (src/nn/layer.cpp:635-665) of the K and V rows a
// QKV pass staged, per (row, kv head): s = absmax / 127 (0 -> 1), q =
// round(x * (1 / s)) clamped to +-127.  One warp per (row, head, K|V).
static __global__ void kv_quant_kernel(RowsView rows, int R, const float *__restrict__ stage, int kvd, int D, int Hkv,
                                int S_cap, KvPages pg, int8_t *__restrict__ kc, int8_t *__restrict__ vc,
                                float *__restrict__ ks, float *__restrict__ vs) {
  const int r = blockIdx.x;
  if (r >= R) return;
  const int req = rows.req[r], pos = row_slot(rows, r);
  if (req < 0 || pos < 0 || pos >= S_cap) return;  // the QKV pass flagged an out-of-range cache row
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int t = warp; t < 2 * Hkv; t += nw) {
    const bool is_v = t >= Hkv;
    const int h = is_v ? t - Hkv : t;
    const float *src = stage + static_cast<size_t>(r) * 2 * kvd + (is_v ? kvd : 0) + h * D;
    float mx = 0.f;
    for (int e = lane; e < D; e += 32) mx = fmaxf(mx, fabsf(src[e]));
    mx = warp_max(mx);
    float sc = __fdiv_rn(mx, 127.0f);
    if (sc == 0.0f) sc = 1.0f;
    const float inv = __fdiv_rn(1.0f, sc);
    const int prow = kv_row(pg, Hkv, req, h, pos);
    if (prow < 0) continue;  // the QKV pass flagged the missing page
    const size_t row = static_cast<size_t>(prow);
    int8_t *dst = (is_v ? vc : kc) + row * D;
    for (int e = lane; e < D; e += 32) {
      const float qv = fminf(127.0f, fmaxf(-127.0f, roundf(__fmul_rn(src[e], inv))));
      dst[e] = static_cast<int8_t>(qv);
    }
    if (lane == 0) (is_v ? vs : ks)[row] = sc;
  }
}

// ---------------------------------------------------------------------------
// Causal attention (src/nn/layer.cpp:859-948): score = (q . k) / sqrt(D)
// (layer.cpp:870, 891-897), softmax over positions j <= pos, then P.V.
//
// Work split.  The rows of one request in one forward pass are consecutive
// and form a "group" of Q queries (the k+1 verify rows, the catch-up + last
// draft rows, a prefill chunk).  A CTA handles up to QT queries of one group
// for one head and one split (a contiguous chunk of positions) of the
// context, so the request's K/V are read once for all of its queries.  The
// splits of one (query tile, head) are one thread-block cluster along z:
// each CTA leaves its (max, sum, unnormalised P.V) in its own shared memory
// and, after a cluster barrier, every CTA merges a share of the outputs
// (log-sum-exp) by reading its peers' shared memory, so the split merge costs
// no global-memory round trip.
//
// Staging.  Thread 0 issues TMA tensor copies (cp.async.bulk.tensor.2d into
// this CTA's own shared memory, completion on an mbarrier) of kTile cache
// rows of K and of V;
// with several tiles per chunk the two stages alternate.  Rows that are a
// multiple of 128 bytes wide arrive with the 128-byte swizzle (16-byte unit
// j of row r lands in unit j ^ (r & 7) of its 128-byte line), so the score
// loop -- thread = position, walking the head dimension -- reads K without
// bank conflicts while all threads read the same q words (broadcast).  P.V
// has lanes over head dimensions and reads the warp's probabilities from
// shared memory as broadcasts.
constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kAttnQT = 8;        // most queries per CTA (a group rounds up to 1, 2, 4 or 8)
constexpr int kAttnMaxSplit = 8;  // portable cluster size

template <typename KT, int D>
struct AttnGeom {
  static constexpr int kRowBytes = D * static_cast<int>(sizeof(KT));
  static constexpr bool kTma = kRowBytes % 16 == 0;  // else the host rejects the shape
  // TMA swizzle span: the widest of 128, 64 or 32 bytes that divides a row
  // (0: rows of 16 bytes, which are conflict-free as they are)
  static constexpr int kSw = kRowBytes % 128 == 0 ? 128 : kRowBytes % 64 == 0 ? 64 : kRowBytes % 32 == 0 ? 32 : 0;
  static constexpr int kTile = kRowBytes > 256 ? 64 : 128;  // rows per stage
  static constexpr int kE = 16 / static_cast<int>(sizeof(KT));  // elements per 16-byte unit
  static constexpr int kNC = kRowBytes / 16;                      // 16-byte units per row
  static constexpr int kStageBytes = 2 * kTile * kRowBytes;       // K tile + V tile
  static constexpr int kEPL = D >= 32 ? D / 32 : 1;               // P.V: head dims per lane
  static constexpr int kLanesPV = D / kEPL;
  static constexpr int kBoxBytes = kSw ? kSw : kRowBytes;         // TMA box width
  static constexpr int kBoxCols = kBoxBytes / static_cast<int>(sizeof(KT));
  static constexpr int smem_bytes(int stages) { return stages * kStageBytes + 1024; }
  // Byte offset of 16-byte unit c of tile row r within a K or V tile.  A box
  // of kSw-byte rows lands with its 16-byte unit j of row r at unit
  // j ^ ((r * kSw / 128) & (kSw / 16 - 1)) (the TMA swizzle XORs address bits
  // [4, 4 + log2(kSw / 16)) with bits [7, ...)), so 8 consecutive rows read
  // at one logical unit hit 8 different bank groups.
  __device__ static __forceinline__ int unit(int r, int c) {
    if constexpr (kSw != 0) {
      constexpr int per = kSw / 16;
      return (c / per) * (kTile * kSw) + r * kSw + (((c % per) ^ ((r * kSw / 128) & (per - 1))) << 4);
    } else {
      return r * kRowBytes + c * 16;
    }
  }
};

struct alignas(64) AttnArgs {
  CUtensorMap tmk, tmv;  // 2-D views [cache row][D] of this layer's K and V page pools
  KvPages pg;
  const void *q;
  int ldq;
  RowsView rows;
  int R, Q;      // rows, queries per group
  int S_cap, H, Hkv;
  int chunk, nsplit;
  const float *k_scale, *v_scale;  // int8 cache: per-row dequantisation scales (same row index as the maps)
  void *out;
  int ldo;
  int *err;
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Waits for an mbarrier phase for at most about a second; false = gave up.
// A failed try sleeps for a few tens of nanoseconds before the next one, so
// waiting warps leave the issue slots to the working ones (a warp that spins
// on try_wait takes them from the producer and MMA threads of its SM).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t phase) {
  const uint32_t addr = smem_u32(bar);
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(addr), "r"(phase)
        : "memory");
    if (done) return true;
    __nanosleep(32);
    if ((it & 63) == 0) {
      const uint64_t now = global_ns();
      if (it == 0) t0 = now;
      else if (now - t0 > 1000000000ull) return false;
    }
  }
}

// One tiled TMA load of box (x, y) of `map` into this CTA's shared memory,
// completing on `bar`.  x * sizeof(element) is a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// 16 bytes of cache elements -> fp32
__device__ __forceinline__ void unpack16(uint4 u, float *f, int8_t) {
  i8x4_to_f32(u.x, f);
  i8x4_to_f32(u.y, f + 4);
  i8x4_to_f32(u.z, f + 8);
  i8x4_to_f32(u.w, f + 12);
}
__device__ __forceinline__ void unpack16(uint4 u, float *f, float) {
  f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y);
  f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
}
__device__ __forceinline__ void unpack16(uint4 u, float *f, __nv_bfloat16) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// N consecutive cache elements at shared address p -> fp32
template <typename KT, int N>
__device__ __forceinline__ void lds_elems(const unsigned char *p, float *f) {
  constexpr int bytes = N * static_cast<int>(sizeof(KT));
  if constexpr (std::is_same<KT, int8_t>::value) {
    if constexpr (bytes == 4) {
      i8x4_to_f32(*reinterpret_cast<const uint32_t *>(p), f);
    } else if constexpr (bytes == 2) {
      const int16_t v = *reinterpret_cast<const int16_t *>(p);
      f[0] = static_cast<float>(static_cast<int8_t>(v & 0xff));
      f[1] = static_cast<float>(static_cast<int8_t>(v >> 8));
    } else {
      f[0] = static_cast<float>(*reinterpret_cast<const int8_t *>(p));
    }
  } else if constexpr (std::is_same<KT, float>::value) {
    if constexpr (bytes == 16) {
      const float4 v = *reinterpret_cast<const float4 *>(p);
      f[0] = v.x; f[1] = v.y; f[2] = v.z; f[3] = v.w;
    } else if constexpr (bytes == 8) {
      const float2 v = *reinterpret_cast<const float2 *>(p);
      f[0] = v.x; f[1] = v.y;
    } else {
      f[0] = *reinterpret_cast<const float *>(p);
    }
  } else {
    if constexpr (bytes == 8) {
      const uint2 v = *reinterpret_cast<const uint2 *>(p);
      f[0] = __uint_as_float(v.x << 16); f[1] = __uint_as_float(v.x & 0xffff0000u);
      f[2] = __uint_as_float(v.y << 16); f[3] = __uint_as_float(v.y & 0xffff0000u);
    } else if constexpr (bytes == 4) {
      const uint32_t v = *reinterpret_cast<const uint32_t *>(p);
      f[0] = __uint_as_float(v << 16); f[1] = __uint_as_float(v & 0xffff0000u);
    } else {
      f[0] = __uint_as_float(static_cast<uint32_t>(*reinterpret_cast<const unsigned short *>(p)) << 16);
    }
  }
}

template <typename AT, typename KT, int D, int QT>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const __grid_constant__ AttnArgs a) {
  using G = AttnGeom<KT, D>;
  pdl_wait();
  if constexpr (!G::kTma) {
    return;  // unreachable: the host rejects rows that are not a multiple of 16 bytes
  } else {
  constexpr int kTile = G::kTile;
  constexpr int EPL = G::kEPL;
  constexpr int NACC = QT == 1 ? 4 : (QT == 2 ? 2 : 1);  // independent partial dots per query
  constexpr bool kI8 = std::is_same<KT, int8_t>::value;
  constexpr bool kSqrtPow2 = D == 4 || D == 16 || D == 64;
  constexpr float kInvSqrt = D == 4 ? 0.5f : D == 16 ? 0.25f : 0.125f;
  extern __shared__ unsigned char attn_smem_raw[];
  unsigned char *tiles =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(attn_smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(16) float qs[QT][D];
  __shared__ __align__(16) float s_p[kAttnWarps][QT][32];
  __shared__ __align__(16) float s_acc[kAttnWarps][QT][D];  // [0] holds the CTA's merged P.V
  __shared__ float s_m[kAttnWarps][QT], s_l[kAttnWarps][QT];
  __shared__ float c_m[QT], c_l[QT];  // the CTA's merged max and sum
  __shared__ int s_pos[QT], s_req[QT], s_tb[QT];  // s_pos: the query's cache row (visibility limit)
  __shared__ unsigned long long s_mask[QT];
  __shared__ __align__(8) uint64_t bars[2];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int ngt = (a.Q + QT - 1) / QT;
  const int g = blockIdx.x / ngt, qt = blockIdx.x % ngt;
  const int h = blockIdx.y, split = blockIdx.z;
  const int rq0 = g * a.Q + qt * QT;
  const int nq = max(0, min(QT, min(a.Q - qt * QT, a.R - rq0)));

  const int hk = h / (a.H / a.Hkv);
  const float scale = sqrtf(static_cast<float>(D));
  __shared__ int s_meta[2];
  // The splits share the positions the group's queries see (0 .. maxpos), so
  // every split has work while the cache is shorter than its capacity; a
  // split never exceeds a.chunk positions (the staging the host sized).
  // Splits start at multiples of the tile, so no tile straddles a page.
  auto span = [&](int maxpos, int &j0, int &j1) {
    const int ch = min(a.chunk, ((maxpos + a.nsplit) / a.nsplit + kTile - 1) / kTile * kTile);
    j0 = split * ch;
    j1 = min(maxpos + 1, j0 + ch);
    return (j1 > j0) ? (j1 - j0 + kTile - 1) / kTile : 0;
  };
  auto issue = [&](int t, int req, int j0) {  // thread 0 only
    const int s = t & 1;
    unsigned char *kdst = tiles + s * G::kStageBytes;
    unsigned char *vdst = kdst + kTile * G::kRowBytes;
    int y = kv_row(a.pg, a.Hkv, req, hk, j0 + t * kTile);
    if (y < 0) {  // a position without a page: flagged, and a valid row is read instead
      if (a.err) atomicOr(a.err, kErrSeqLen);
      y = 0;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(&bars[s])),
                 "r"(G::kStageBytes)
                 : "memory");
#pragma unroll
    for (int cb = 0; cb < D / G::kBoxCols; ++cb) {
      tma_load_2d(kdst + cb * kTile * G::kBoxBytes, &a.tmk, cb * G::kBoxCols, y, &bars[s]);
      tma_load_2d(vdst + cb * kTile * G::kBoxBytes, &a.tmv, cb * G::kBoxCols, y, &bars[s]);
    }
  };
  // Thread 0 reads the queries' rows, then issues the first tile while the
  // other threads fetch the query vectors.
  if (threadIdx.x == 0) {
    int rr[QT], pr[QT];
#pragma unroll
    for (int i = 0; i < QT; ++i) {
      rr[i] = (i < nq) ? a.rows.req[rq0 + i] : -1;
      pr[i] = (i < nq) ? row_slot(a.rows, rq0 + i) : -1;
      s_tb[i] = (i < nq && a.rows.tb) ? a.rows.tb[rq0 + i] : 0x7fffffff;
      s_mask[i] = (i < nq && a.rows.mask) ? a.rows.mask[rq0 + i] : 0ull;
    }
    int req = -1, maxpos = -1;
#pragma unroll
    for (int i = 0; i < QT; ++i) {
      s_req[i] = rr[i];
      s_pos[i] = (rr[i] >= 0) ? pr[i] : -1;
      if (rr[i] >= 0) {
        req = rr[i];
        maxpos = max(maxpos, pr[i]);
      }
    }
    s_meta[0] = req;
    s_meta[1] = maxpos;
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bars[0])) : "memory");
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bars[1])) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    if (req >= 0 && maxpos < a.S_cap) {
      int j0, j1;
      if (span(maxpos, j0, j1) > 0) issue(0, req, j0);
    }
  }
  constexpr int kQIter = (QT * D + kAttnThreads - 1) / kAttnThreads;
#pragma unroll
  for (int k = 0; k < kQIter; ++k) {
    const int idx = threadIdx.x + k * kAttnThreads;
    if (idx < QT * D) {
      const int i = idx / D, e = idx % D;
      qs[i][e] =
          (i < nq) ? to_f32(static_cast<const AT *>(a.q)[static_cast<size_t>(rq0 + i) * a.ldq + h * D + e]) : 0.f;
    }
  }
  __syncthreads();
  const int req = s_meta[0], maxpos = s_meta[1];
  // uniform over the cluster: all its CTAs share (query tile, head)
  if (req < 0 || maxpos >= a.S_cap) return;
  int j0, j1;
  const int ntiles = span(maxpos, j0, j1);

  float m[QT], l[QT], acc[QT][EPL];
  int qpos[QT], qtb[QT];
  unsigned long long qmask[QT];
#pragma unroll
  for (int i = 0; i < QT; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
    qpos[i] = s_pos[i];
    qtb[i] = s_tb[i];
    qmask[i] = s_mask[i];
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc[i][e] = 0.f;
  }
  // P.V: this lane's head dimensions [lane*EPL, lane*EPL + EPL) in unit pv_c at byte pv_b
  const int pv_c = (lane * EPL) / G::kE;
  const int pv_b = ((lane * EPL) % G::kE) * static_cast<int>(sizeof(KT));

  bool ok = true;
  int t = 0;
  for (; t < ntiles; ++t) {
    const int t0 = j0 + t * kTile;
    const int nt = min(kTile, j1 - t0);
    if (threadIdx.x == 0 && t + 1 < ntiles) issue(t + 1, req, j0);  // the other stage was released at the end of t-1
    ok = __syncthreads_and(mbar_wait(&bars[t & 1], (t >> 1) & 1) ? 1 : 0) != 0;
    if (!ok) break;
    const unsigned char *kt = tiles + (t & 1) * G::kStageBytes;
    const unsigned char *vt = kt + kTile * G::kRowBytes;

    // scores: thread = tile row
    const int r = threadIdx.x;
    const int pos = t0 + r;
    float ksc = 1.f, vsc = 1.f;
    if constexpr (kI8) {
      const int yb = kv_row(a.pg, a.Hkv, req, hk, t0);  // the tile's first cache row (one page)
      if (r < nt && yb >= 0) {
        ksc = __ldg(a.k_scale + yb + r);
        vsc = __ldg(a.v_scale + yb + r);
      }
    }
    float sc[QT];
    {
      float dot[QT][NACC];
#pragma unroll
      for (int i = 0; i < QT; ++i)
#pragma unroll
        for (int u = 0; u < NACC; ++u) dot[i][u] = 0.f;
      // Branch-free: all QT queries (rows past nq hold zeros) and all
      // threads (with 64-row tiles the upper threads read in-bounds rows of
      // the stage and are masked below).
#pragma unroll
      for (int c = 0; c < G::kNC; ++c) {
        float kf[G::kE];
        unpack16(*reinterpret_cast<const uint4 *>(kt + G::unit(r, c)), kf, KT{});
#pragma unroll
        for (int i = 0; i < QT; ++i) {
#pragma unroll
          for (int e = 0; e < G::kE; e += 4) {
            const float4 q4 = *reinterpret_cast<const float4 *>(&qs[i][c * G::kE + e]);
            const int u = ((c * G::kE + e) / 4) % NACC;
            dot[i][u] = fmaf(q4.x, kf[e], dot[i][u]);
            dot[i][u] = fmaf(q4.y, kf[e + 1], dot[i][u]);
            dot[i][u] = fmaf(q4.z, kf[e + 2], dot[i][u]);
            dot[i][u] = fmaf(q4.w, kf[e + 3], dot[i][u]);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < QT; ++i) {
        float dd = dot[i][0];
#pragma unroll
        for (int u = 1; u < NACC; ++u) dd += dot[i][u];
        if constexpr (kI8) dd *= ksc;  // q . (k_q * s) = s * (q . k_q)
        // sqrt(D) is a power of two for D = 4, 16, 64: the product by its
        // reciprocal is then the correctly rounded quotient
        const float sv = kSqrtPow2 ? dd * kInvSqrt : __fdiv_rn(dd, scale);
        // causal, and inside a token tree only the prefix, the ancestors and itself
        const bool vis = pos <= qpos[i] &&
                         (pos < qtb[i] || (pos - qtb[i] < 64 && ((qmask[i] >> (pos - qtb[i])) & 1ull)));
        sc[i] = (i < nq && r < nt && vis) ? sv : -INFINITY;
      }
    }
    // online softmax per warp: the warp's running max is shared by its lanes
    float tm[QT];
#pragma unroll
    for (int i = 0; i < QT; ++i) tm[i] = sc[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int i = 0; i < QT; ++i) tm[i] = fmaxf(tm[i], __shfl_xor_sync(0xffffffffu, tm[i], o));
#pragma unroll
    for (int i = 0; i < QT; ++i) {
      const float mnew = fmaxf(m[i], tm[i]);
      const float p = (sc[i] == -INFINITY) ? 0.f : expf(sc[i] - mnew);
      const float alpha = (m[i] == -INFINITY) ? 0.f : expf(m[i] - mnew);
      m[i] = mnew;
      l[i] = l[i] * alpha + p;  // per-lane partial sum, reduced after the loop
#pragma unroll
      for (int e = 0; e < EPL; ++e) acc[i][e] *= alpha;
      s_p[warp][i][lane] = kI8 ? p * vsc : p;  // p * (v_q * s) = (p * s) * v_q
    }
    __syncwarp();
    // P.V over the warp's 32 rows; rows past the tile's end re-read its last
    // row (finite) with probability 0
    const int nvalid = min(32, nt - warp * 32);
    if (lane < G::kLanesPV && nvalid > 0) {
#pragma unroll
      for (int pp = 0; pp < 32; pp += 4) {
        float v[4][EPL];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          lds_elems<KT, EPL>(vt + G::unit(warp * 32 + min(pp + u, nvalid - 1), pv_c) + pv_b, v[u]);
#pragma unroll
        for (int i = 0; i < QT; ++i) {
          const float4 p4 = *reinterpret_cast<const float4 *>(&s_p[warp][i][pp]);
#pragma unroll
          for (int e = 0; e < EPL; ++e) {
            acc[i][e] = fmaf(p4.x, v[0][e], acc[i][e]);
            acc[i][e] = fmaf(p4.y, v[1][e], acc[i][e]);
            acc[i][e] = fmaf(p4.z, v[2][e], acc[i][e]);
            acc[i][e] = fmaf(p4.w, v[3][e], acc[i][e]);
          }
        }
      }
    }
    __syncthreads();  // this stage is refilled two tiles later; s_p is rewritten next tile
  }
  if (!ok) {
    // give the copies in flight a bounded time to land before the CTA moves on
    if (threadIdx.x == 0) {
      mbar_wait(&bars[t & 1], (t >> 1) & 1);
      if (t + 1 < ntiles) mbar_wait(&bars[(t + 1) & 1], ((t + 1) >> 1) & 1);
      if (a.err) atomicOr(a.err, kErrTimeout);
    }
#pragma unroll
    for (int i = 0; i < QT; ++i) {
      m[i] = -INFINITY;
      l[i] = 0.f;
#pragma unroll
      for (int e = 0; e < EPL; ++e) acc[i][e] = 0.f;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int i = 0; i < QT; ++i) l[i] += __shfl_xor_sync(0xffffffffu, l[i], o);

  pdl_launch();
  // merge the CTA's warps
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < QT; ++i) {
      s_m[warp][i] = m[i];
      s_l[warp][i] = l[i];
    }
  }
  if (lane < G::kLanesPV) {
#pragma unroll
    for (int i = 0; i < QT; ++i)
#pragma unroll
      for (int e = 0; e < EPL; ++e) s_acc[warp][i][lane * EPL + e] = acc[i][e];
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < kQIter; ++k) {
    const int idx = threadIdx.x + k * kAttnThreads;
    if (idx >= QT * D) break;
    const int i = idx / D, e = idx % D;
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
    if (a.nsplit == 1) {
      if (i < nq && s_pos[i] >= 0)
        static_cast<AT *>(a.out)[static_cast<size_t>(rq0 + i) * a.ldo + h * D + e] = from_f32<AT>(L > 0.f ? A / L : 0.f);
    } else {
      s_acc[0][i][e] = A;  // only this thread reads or writes (i, e) here
      if (e == 0) {
        c_m[i] = M;
        c_l[i] = L;
      }
    }
  }
  if (a.nsplit == 1) return;

  // merge the splits through distributed shared memory
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  cl.sync();
  const int rank = static_cast<int>(cl.block_rank());
  for (int idx = rank * blockDim.x + threadIdx.x; idx < nq * D; idx += a.nsplit * blockDim.x) {
    const int i = idx / D, e = idx % D;
    if (s_pos[i] < 0) continue;
    float Ms[kAttnMaxSplit], Ls[kAttnMaxSplit], As[kAttnMaxSplit];
#pragma unroll
    for (int s = 0; s < kAttnMaxSplit; ++s) {
      Ls[s] = 0.f;
      if (s < a.nsplit) {
        Ms[s] = *cl.map_shared_rank(&c_m[i], s);
        Ls[s] = *cl.map_shared_rank(&c_l[i], s);
        As[s] = *cl.map_shared_rank(&s_acc[0][i][e], s);
      }
    }
    float M = -INFINITY;
#pragma unroll
    for (int s = 0; s < kAttnMaxSplit; ++s)
      if (Ls[s] > 0.f) M = fmaxf(M, Ms[s]);
    float L = 0.f, A = 0.f;
#pragma unroll
    for (int s = 0; s < kAttnMaxSplit; ++s) {
      if (Ls[s] > 0.f) {
        const float w = expf(Ms[s] - M);
        L += Ls[s] * w;
        A += As[s] * w;
      }
    }
    static_cast<AT *>(a.out)[static_cast<size_t>(rq0 + i) * a.ldo + h * D + e] = from_f32<AT>(L > 0.f ? A / L : 0.f);
  }
  cl.sync();  // every CTA's shared memory stays in place until its peers have read it
  }
}

}  // namespace specdec
