// Linear layer y = x . W + b on tcgen05 for the row batches of a speculative
// round -- draft steps (32 or 64 rows on the large configuration) and verify
// blocks (k + 1 rows per request: 160) -- as a persistent stream-K GEMM
// (Dense / QuantizedDense forward, src/nn/layer.cpp:162-171,
// src/nn/quantization.cpp:7-147: y = x . (q * s) + b, the scale applied per
// output column in the epilogue, as the GEMV does).
//
// Why.  With 128 x 256 tiles a 32-row draft launch of the SwiGLU gate/up
// projection (22016 x 4096) is 86 tiles: 62 of the 148 SMs idle while the
// others stream 2 MB of weights each.  A 160-row verify launch is 172 tiles
// (two row tiles per weight tile), 1.16 waves, and reads every weight tile
// twice.  Here:
//   * one CTA per SM (g.ctas of them) walks an equal share of the units
//     (256-column tile, 64-wide k-block): CTA c takes units
//     [c U / ctas, (c + 1) U / ctas), U = tiles x k-blocks, so every SM
//     streams the same number of weight bytes;
//   * a unit covers all the launch's rows: up to two 128-row accumulators
//     (TMEM columns 0-255 and 256-511) take their MMAs from the same weight
//     tile, so each weight byte crosses HBM once per launch;
//   * a tile that one CTA covers whole gets its epilogue straight from
//     TMEM; the pieces of a tile shared by several CTAs are stored as fp32
//     partial tiles in an L2-resident workspace, and a second, wide launch
//     (gemm_sk_fixup_kernel: one block per tile, row tile and 64 columns)
//     adds them in CTA order -- the same sum on every run -- and runs the
//     epilogue.  No CTA ever waits for another.
//   * With one row tile the two TMEM halves are a double buffer: the
//     epilogue of one segment overlaps the MMAs of the next.
//
// Roles: warp 0 streams (A row tiles, B weight tile) stages with TMA
// (128-byte swizzle, no multicast), warp 1 issues tcgen05.mma (M = 128,
// N = 256, K = 16, both operands K-major from shared memory) and commits the
// stages and accumulators, warps 2-5 read their 32 TMEM lanes (rows) with
// tcgen05.ld and run the epilogue (the chunk functions of gemm.cuh: scale
// and bias, residual, RoPE + paged cache append, SwiGLU, GELU, logits).
// Every mbarrier wait is bounded; a wait that gives up raises kErrTimeout and
// the CTA winds down (the host reports the error).
#include <algorithm>

#include "gemm.cuh"
#include "gemm_sk.cuh"

namespace specdec {

namespace {

constexpr int kSkThreads = 192;         // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int kSkRing = 192 * 1024;     // 4 stages of 48 KB (one row tile) or 3 of 64 KB (two)
constexpr int kSkSmemBytes = kSkRing + 1024;
constexpr int kSkTmemCols = 512;        // two 256-column fp32 accumulators
constexpr int kSkMaxStages = 4;
constexpr int kSkPiece = 256 * 256;     // floats of one partial tile: [256 columns][256 rows]

__device__ __forceinline__ int sk_start(int c, int U, int P) {
  return static_cast<int>(static_cast<long long>(c) * U / P);
}
// The CTA whose units include unit u: the largest c with sk_start(c) <= u.
__device__ __forceinline__ int sk_owner(int u, int U, int P) {
  return static_cast<int>((static_cast<long long>(u + 1) * P + U - 1) / U) - 1;
}

__device__ __forceinline__ bool bar_and_epi(bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, 1, 128, p;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v))
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void bar_epi() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Row metadata of the QKV epilogue (request, RoPE position, cache position).
template <int EPI>
__device__ __forceinline__ void sk_rowmeta(const LinearArgs &a, int row, bool ok, int &req, int &pos, int &slot) {
  req = 0; pos = 0; slot = 0;
  if constexpr (EPI == kEpiQKV) {
    req = ok ? a.rows.req[row] : -1;
    pos = ok ? a.rows.pos[row] : 0;
    slot = ok ? row_slot(a.rows, row) : 0;
  }
}

// The epilogue of one row of a tile this CTA covers whole, from its TMEM
// accumulators at tb, 64 columns at a time (the row operands of the group in
// flight before the TMEM load).  tcgen05.ld is warp-collective: every lane
// runs the loads, rows past R skip the arithmetic and the stores.
template <int EPI>
__device__ __forceinline__ void sk_rows_epilogue(const LinearArgs &a, int row, uint32_t tb, int n0, int ncols,
                                                 const float *s_scale, const float *s_bias) {
  const bool row_ok = row < a.R;
  int req, pos, slot;
  sk_rowmeta<EPI>(a, row, row_ok, req, pos, slot);
  for (int g0 = 0; g0 < ncols; g0 += 64) {
    ChunkOps op[4];
    if (row_ok)
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (g0 + 16 * q < ncols) chunk_load<EPI>(a, row, n0 + g0 + 16 * q, req, pos, op[q]);
    float v[64];
    tmem_ld64(tb + g0, v);
    if (!row_ok) continue;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int cc = g0 + 16 * q;
      if (cc >= ncols) break;
      float w16[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) w16[e] = v[16 * q + e];
      chunk_store<EPI>(a, row, n0 + cc, w16, op[q], s_scale + cc, s_bias + cc, req, pos, slot);
    }
  }
}

template <int EPI>
__global__ void __launch_bounds__(kSkThreads, 1) gemm_sk_kernel(const __grid_constant__ GemmSkArgs g) {
  extern __shared__ unsigned char sk_smem_raw[];
  unsigned char *ring =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(sk_smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[kSkMaxStages], empty[kSkMaxStages], acc_full[2], acc_empty[2], fin;
  __shared__ uint32_t s_tmem;
  __shared__ int s_fail;
  __shared__ __align__(16) float s_scale[kBN], s_bias[kBN];

  const LinearArgs &a = g.lin;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = g.mt, nk = g.nk, P = g.ctas, c = blockIdx.x;
  const int U = g.nt * nk;
  const int u_begin = sk_start(c, U, P), u_end = sk_start(c + 1, U, P);
  const int a_bytes = kBM * kBK * 2, b_bytes = kBN * kBK * 2;
  const int stage_bytes = mt * a_bytes + b_bytes;
  const int S = kSkRing / stage_bytes;  // 4 (one row tile) or 3 (two)
  const int nbuf = mt == 1 ? 2 : 1;     // accumulator buffers

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(kSkTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x == 32) {
    for (int s = 0; s < kSkMaxStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(&fin, 1);
    s_fail = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  // the fix-up launch may begin now: its blocks wait for this grid to finish
  if (threadIdx.x == 0) pdl_launch();
  // launched as a programmatic dependent itself: the predecessors' outputs
  // (input rows, residual, row tables) are read and every write made after
  pdl_wait();

  if (warp == 0) {
    // ---- producer: the CTA's units in order, through the stage ring -------
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int u = u_begin; u < u_end && ok; ++u) {
        const int t = u / nk, kb = u - t * nk;
        const int s = it % S;
        if (it >= S && !mbar_wait(&empty[s], ((it / S) - 1) & 1)) {
          ok = false;
          break;
        }
        unsigned char *st = ring + s * stage_bytes;
        mbar_expect_tx(&full[s], static_cast<uint32_t>(stage_bytes));
        for (int i = 0; i < mt; ++i) tma_load_2d(st + i * a_bytes, &g.tma_a, kb * kBK, i * kBM, &full[s]);
        tma_load_2d(st + mt * a_bytes, &g.tma_b, 0, u * kBN, &full[s]);  // block (t, kb) of the tile-order image
        ++it;
      }
      if (!ok) {
        s_fail = 1;
        // the copies already issued land before the CTA can leave
        for (int j = max(0, it - S); j < it; ++j) mbar_wait(&full[j % S], (j / S) & 1);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer: one segment (a run of units in one tile) at a time ---
    if (lane == 0) {
      int it = 0, seg = 0;
      bool ok = true;
      for (int u = u_begin; u < u_end && ok; ++seg) {
        const int t = u / nk, kb0 = u - t * nk;
        const int kb1 = min(nk, kb0 + (u_end - u));
        const int buf = seg % nbuf;
        // the epilogue has drained this accumulator buffer
        if (seg >= nbuf && !mbar_wait(&acc_empty[buf], ((seg / nbuf) - 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % S;
          if (!mbar_wait(&full[s], (it / S) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(ring + s * stage_bytes);
          const uint32_t sb = sa + mt * a_bytes;
          for (int i = 0; i < mt; ++i) {
            const uint32_t d = tmem + static_cast<uint32_t>((buf + i) * kBN);
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k)
              tc_mma(d, umma_desc_k128(sa + i * a_bytes + 32 * k), umma_desc_k128(sb + 32 * k), kGemmIdesc,
                     (kb > kb0 || k > 0) ? 1u : 0u);
          }
          tc_commit(&empty[s]);  // the stage is free once these MMAs have read it
        }
        if (!ok) break;
        tc_commit(&acc_full[buf]);  // the segment's accumulators are complete
        u += kb1 - kb0;
      }
      if (!ok) s_fail = 1;
      tc_commit(&fin);
      mbar_wait(&fin, 0);  // no MMA in flight when TMEM is released
    }
  } else {
    // ---- epilogue: warps 2-5, TMEM lane group warp % 4 --------------------
    const int lg = warp & 3;
    const int lr = lg * 32 + lane;  // this thread's row within a row tile
    const uint32_t tl = tmem + (static_cast<uint32_t>(lg * 32) << 16);
    int seg = 0;
    for (int u = u_begin; u < u_end; ++seg) {
      const int t = u / nk, kb0 = u - t * nk;
      const int kb1 = min(nk, kb0 + (u_end - u));
      const bool first = u == u_begin;
      u += kb1 - kb0;
      const int buf = seg % nbuf;
      const int n0 = t * kBN;
      const int ncols = min(kBN, a.N - n0);
      if (!bar_and_epi(mbar_wait(&acc_full[buf], (seg / nbuf) & 1))) {
        s_fail = 1;
        break;
      }
      tc_fence_after();
      const bool whole = kb0 == 0 && kb1 == nk;
      if (whole) {
        // the tile's per-column scale and bias (s_scale / s_bias are free:
        // the previous epilogue ended before the barrier in bar_and_epi)
        for (int j = threadIdx.x - 64; j < kBN; j += 128) {
          const int n = n0 + j;
          s_scale[j] = (n < a.N && a.scale) ? __ldg(a.scale + n) : 1.f;
          s_bias[j] = n < a.N ? __ldg(a.bias + n) : 0.f;
        }
        bar_epi();
        for (int i = 0; i < mt; ++i) {
          const uint32_t tb = tl + static_cast<uint32_t>((buf + i) * kBN);
          sk_rows_epilogue<EPI>(a, i * kBM + lr, tb, n0, ncols, s_scale, s_bias);
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[buf]);
        continue;
      }
      // a piece of a shared tile: column-major [256 columns][256 rows] fp32
      // (a warp's 32 rows of one column are one 128-byte line) in this CTA's
      // first or last slot; gemm_sk_fixup_kernel adds the pieces
      float *piece = g.ws + (static_cast<size_t>(c) * 2 + (first ? 0 : 1)) * kSkPiece;
      for (int i = 0; i < mt; ++i) {
        const int row = i * kBM + lr;
        const uint32_t tb = tl + static_cast<uint32_t>((buf + i) * kBN);
        for (int g0 = 0; g0 < ncols; g0 += 64) {
          float v[64];
          tmem_ld64(tb + g0, v);  // warp-collective
          if (row < a.R)
#pragma unroll
            for (int e = 0; e < 64; ++e) __stcg(piece + static_cast<size_t>(g0 + e) * 256 + row, v[e]);
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);  // the MMAs may refill this buffer
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && s_fail && g.err) atomicOr(g.err, kErrTimeout);
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kSkTmemCols) : "memory");
}

// The fix-up of the shared tiles: block (t, i, gq) = tile t, row tile i,
// columns 32 gq .. 32 gq + 31, thread = row.  It adds the pieces of the
// tile's CTAs cf .. cl in CTA order -- the same sum on every run -- and runs
// the epilogue; blocks of whole tiles (one CTA, epilogue already done) return
// at once.  It is launched as a programmatic dependent of the main kernel,
// which allows it to launch at its start: the blocks are resident and wait in
// griddepcontrol.wait (which returns once the main kernel has completed and
// its stores are visible) instead of paying a launch after it.  The pieces
// are loaded four at a time, all in flight together; the tile's scale and
// bias go through shared memory.
template <int EPI>
__global__ void __launch_bounds__(128) gemm_sk_fixup_kernel(const __grid_constant__ GemmSkArgs g) {
  // first of all, in every thread: the main kernel's pieces and every earlier
  // kernel's outputs are complete and visible past this point, and this grid
  // cannot complete before the main kernel (whatever its blocks skip), which
  // the launches after it rely on
  pdl_wait();
  const LinearArgs &a = g.lin;
  const int t = blockIdx.x, i = blockIdx.y, g0 = blockIdx.z * 32;
  const int nk = g.nk, P = g.ctas, U = g.nt * nk;
  const int u0 = t * nk;
  const int cf = sk_owner(u0, U, P), cl = sk_owner(u0 + nk - 1, U, P);
  const int n0 = t * kBN;
  const int ncols = min(kBN, a.N - n0);
  if (cf == cl || g0 >= ncols) return;  // uniform over the block
  __shared__ __align__(16) float ssc[32], sbi[32];
  if (threadIdx.x < 32) {
    const int n = n0 + g0 + threadIdx.x;
    ssc[threadIdx.x] = (n < a.N && a.scale) ? __ldg(a.scale + n) : 1.f;
    sbi[threadIdx.x] = n < a.N ? __ldg(a.bias + n) : 0.f;
  }
  __syncthreads();
  const int row = i * kBM + threadIdx.x;
  if (row >= a.R) return;
  int req, pos, slot;
  sk_rowmeta<EPI>(a, row, true, req, pos, slot);
  ChunkOps op[2];
#pragma unroll
  for (int q = 0; q < 2; ++q)
    if (g0 + 16 * q < ncols) chunk_load<EPI>(a, row, n0 + g0 + 16 * q, req, pos, op[q]);
  float v[32];
#pragma unroll
  for (int e = 0; e < 32; ++e) v[e] = 0.f;
  for (int q0 = cf; q0 <= cl; q0 += 4) {
    float x[4][32];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int q = q0 + j;
      if (q > cl) break;
      // CTA q's piece of this tile is its first segment when q starts inside
      // the tile, else its last
      const int w = sk_start(q, U, P) >= u0 ? 0 : 1;
      const float *src = g.ws + (static_cast<size_t>(q) * 2 + w) * kSkPiece + static_cast<size_t>(g0) * 256 + row;
#pragma unroll
      for (int e = 0; e < 32; ++e) x[j][e] = __ldcg(src + static_cast<size_t>(e) * 256);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (q0 + j > cl) break;
#pragma unroll
      for (int e = 0; e < 32; ++e) v[e] += x[j][e];
    }
  }
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int cc = g0 + 16 * q;
    if (cc >= ncols) break;
    float w16[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) w16[e] = v[16 * q + e];
    chunk_store<EPI>(a, row, n0 + cc, w16, op[q], ssc + 16 * q, sbi + 16 * q, req, pos, slot);
  }
}

template <int EPI>
cudaError_t set_attr_epi() {
  return cudaFuncSetAttribute(gemm_sk_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSkSmemBytes);
}

template <int EPI>
cudaError_t launch_epi(const GemmSkArgs &g, cudaStream_t stream, bool pdl) {
  cudaLaunchAttribute at{};
  at.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at.val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t mc{};
  mc.gridDim = dim3(g.ctas);
  mc.blockDim = dim3(kSkThreads);
  mc.dynamicSmemBytes = kSkSmemBytes;
  mc.stream = stream;
  mc.attrs = &at;
  mc.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&mc, gemm_sk_kernel<EPI>, g);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t lc{};
  lc.gridDim = dim3(g.nt, g.mt, kBN / 32);
  lc.blockDim = dim3(128);
  lc.stream = stream;
  lc.attrs = &at;
  lc.numAttrs = 1;
  return cudaLaunchKernelEx(&lc, gemm_sk_fixup_kernel<EPI>, g);
}

}  // namespace

int gemm_sk_smem() { return kSkSmemBytes; }

cudaError_t gemm_sk_set_attrs() {
  cudaError_t e = set_attr_epi<kEpiStore>();
  if (e == cudaSuccess) e = set_attr_epi<kEpiResid>();
  if (e == cudaSuccess) e = set_attr_epi<kEpiQKV>();
  if (e == cudaSuccess) e = set_attr_epi<kEpiSwiGLU>();
  if (e == cudaSuccess) e = set_attr_epi<kEpiGelu>();
  return e;
}

cudaError_t gemm_sk_launch(int epi, const GemmSkArgs &g, cudaStream_t stream, bool pdl) {
  switch (epi) {
    case kEpiStore: return launch_epi<kEpiStore>(g, stream, pdl);
    case kEpiResid: return launch_epi<kEpiResid>(g, stream, pdl);
    case kEpiQKV: return launch_epi<kEpiQKV>(g, stream, pdl);
    case kEpiSwiGLU: return launch_epi<kEpiSwiGLU>(g, stream, pdl);
    case kEpiGelu: return launch_epi<kEpiGelu>(g, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace specdec
