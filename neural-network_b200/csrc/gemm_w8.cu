// Linear layer y = x . W + b on tcgen05 for the row batches of a speculative
// round -- draft steps (32 rows on the large configuration) and verify blocks
// (k + 1 rows per request: 160) -- reading the int8 weight codes themselves
// (QuantizedDense, src/nn/quantization.cpp:7-147: y = x . (q * s) + b).
//
// These batches are far below the 128 rows of an MMA's M side, so the
// product is taken transposed: D^T = W x^T with the output features on M
// (128 per CTA) and the rows on N (the batch rounded up to 16, at most 256):
//   A = 128 weight rows x 64 K as bf16: the int8 tile arrives by TMA (8 KB)
//       and four converter warps write its exact bf16 values (|q| <= 127)
//       into a 128-byte-swizzled K-major tile
//   B = the input rows [np][64 K] by TMA, 128-byte swizzle, K-major
//   D = fp32 in TMEM, lane = feature, column = row
// so every weight byte crosses HBM once per pass, whatever the row count (a
// tile of rows on M would re-read the weights for every 128 rows, and the
// bf16 image of the codes doubles the bytes).  The per-column scale is
// applied in the epilogue: sum(x * q) * s, the reassociation the GEMV uses.
//
// Warp 0 streams (weights, rows) stage pairs through the ring, warp 1 issues
// the MMAs (4 per 64-wide k-block), warps 2-5 convert and then run the
// epilogue with thread = feature: for each row the 128 threads of a CTA
// write 128 consecutive outputs (coalesced), and the pair operations (RoPE
// pairs, SwiGLU gate/up pairs, interleaved by the loader) meet through a
// lane shuffle.  Few feature tiles (the 4096-wide residual layers) split K
// over a cluster along y: partials meet in an L2-resident workspace, and
// after the cluster barrier rank z sums its slice of the rows in rank order
// (the same sum on every run).  Every mbarrier wait is bounded; a timeout
// raises kErrTimeout and the CTA still joins its cluster barriers.
#include <algorithm>

#include "gemm.cuh"
#include "gemm_w8.cuh"

namespace specdec {

namespace {

constexpr int kW8Threads = 352;  // warp 0 weight TMA, warp 1 MMA, warp 2 row TMA, warps 3-10 convert + epilogue
constexpr int kW8Conv = 8;       // converter warps
constexpr int kW8RingA = 3;      // bf16 tiles between the converters and the MMAs
constexpr int kW8MaxW = 16;      // int8 weight tiles in flight (the HBM stream)
constexpr int kW8MaxX = 4;       // input-row tiles (L2-resident)
constexpr int kW8WBytes = kW8Feat * 64;       // int8 tile: 128 rows x 64 K
constexpr int kW8ABytes = kW8Feat * 64 * 2;   // its bf16 image: 128 rows x 128 bytes
constexpr int kW8SmemBudget = 200 * 1024;


__device__ __forceinline__ void mbar_arrive_w8(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// 4 int8 codes -> 4 bf16 values (exact) in two words: the 2^23 bias trick of
// the GEMV (i8x4_to_f32) gives fp32 values whose low 16 mantissa bits are zero
// (|q| <= 127 has at most 7 significant bits), so each bf16 is the upper half
// of its fp32 word and a byte permute packs a pair -- no conversion unit.
__device__ __forceinline__ uint2 i8x4_to_bf16x4(uint32_t word) {
  float f[4];
  i8x4_to_f32(word, f);
  return make_uint2(__byte_perm(__float_as_uint(f[0]), __float_as_uint(f[1]), 0x7632),
                    __byte_perm(__float_as_uint(f[2]), __float_as_uint(f[3]), 0x7632));
}

// The epilogue of one (row, feature) value, thread = feature f (lane pairs
// are feature pairs); v is acc * s + b.  Arithmetic as linear_epilogue.
template <int EPI>
__device__ __forceinline__ void w8_epilogue(const LinearArgs &a, int r, int f, bool fok, float v, int req, int pos,
                                            int slot, int lane) {
  using AT = __nv_bfloat16;
  if constexpr (EPI == kEpiStore || EPI == kEpiResid || EPI == kEpiGelu) {
    if (!fok) return;
    if constexpr (EPI == kEpiResid) v = v + __bfloat162float(static_cast<const AT *>(a.resid)[static_cast<size_t>(r) * a.ldr + f]);
    if constexpr (EPI == kEpiGelu) v = 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
    if (a.out_f32) static_cast<float *>(a.out)[static_cast<size_t>(r) * a.ldo + f] = v;
    else static_cast<AT *>(a.out)[static_cast<size_t>(r) * a.ldo + f] = __float2bfloat16_rn(v);
  } else if constexpr (EPI == kEpiSwiGLU) {
    // SwiGLU::forward (src/nn/layer.cpp:1704-1710) on the interleaved pair
    // (gate = feature 2c, up = 2c + 1)
    const float u = __shfl_xor_sync(0xffffffffu, v, 1);
    if (fok && (lane & 1) == 0) {
      const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v)));
      static_cast<AT *>(a.out)[static_cast<size_t>(r) * a.ldo + (f >> 1)] = __float2bfloat16_rn(__fmul_rn(__fmul_rn(v, sg), u));
    }
  } else if constexpr (EPI == kEpiQKV) {
    const QKVArgs &q = a.qkv;
    const float other = __shfl_xor_sync(0xffffffffu, v, 1);
    if (req < 0 || !fok) return;  // req is the row's: uniform over the CTA
    if (pos < 0 || pos >= q.rope_max_pos || slot < 0 || slot >= q.S_cap) {
      if (q.err && f == 0) atomicOr(q.err, kErrSeqLen);
      return;
    }
    if (f < q.d + q.kvd) {
      // Tensor::rope (src/core/tensor.cpp:1144-1163) on pairs (2j, 2j+1)
      const int e = (f < q.d ? f : f - q.d) % q.D;
      const float2 cs = __ldg(q.rope + static_cast<size_t>(pos) * (q.D / 2) + (e >> 1));
      const float v0 = (lane & 1) ? other : v, v1 = (lane & 1) ? v : other;
      v = (lane & 1) ? __fadd_rn(__fmul_rn(v0, cs.y), __fmul_rn(v1, cs.x))
                     : __fsub_rn(__fmul_rn(v0, cs.x), __fmul_rn(v1, cs.y));
    }
    if (f < q.d) {
      static_cast<AT *>(a.out)[static_cast<size_t>(r) * a.ldo + f] = __float2bfloat16_rn(v);
    } else {
      const bool is_k = f < q.d + q.kvd;
      const int nn = is_k ? f - q.d : f - q.d - q.kvd;
      const int h = nn / q.D, e = nn % q.D;
      const int crow = kv_row(q.pg, q.kvd / q.D, req, h, slot);
      if (crow < 0) {
        if (q.err) atomicOr(q.err, kErrSeqLen);
        return;
      }
      const size_t off = static_cast<size_t>(crow) * q.D + e;
      if (q.kv_mode == 2) q.stage[static_cast<size_t>(r) * 2 * q.kvd + (is_k ? 0 : q.kvd) + nn] = v;
      else if (q.kv_mode == 1) static_cast<AT *>(is_k ? q.kc : q.vc)[off] = __float2bfloat16_rn(v);
      else static_cast<float *>(is_k ? q.kc : q.vc)[off] = v;
    }
  }
}

template <int EPI>
__global__ void __launch_bounds__(kW8Threads, 1) gemm_w8_kernel(const __grid_constant__ GemmW8Args g) {
  extern __shared__ unsigned char w8_smem_raw[];
  unsigned char *base =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(w8_smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t wfull[kW8MaxW], wempty[kW8MaxW], afull[kW8RingA], aempty[kW8RingA],
      xfull[kW8MaxX], xempty[kW8MaxX], done;
  __shared__ uint32_t s_tmem;
  __shared__ int s_fail;
  __shared__ int s_req[kW8MaxRows], s_pos[kW8MaxRows], s_slot[kW8MaxRows];

  const LinearArgs &a = g.lin;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int np = g.np, SW = g.stages_w, SX = g.stages_x;
  const bool wb = g.w_bf16 != 0;                        // weights as bf16 tiles, straight to the MMAs
  const int wslot = wb ? kW8ABytes : kW8WBytes;
  unsigned char *wring = base;                          // SW weight tiles (8 KB int8 or 16 KB bf16)
  unsigned char *aring = wring + SW * wslot;            // kW8RingA x 16 KB bf16 tiles (int8 weights)
  unsigned char *xring = aring + (wb ? 0 : kW8RingA * kW8ABytes);  // SX x np rows of 128 bytes
  const int n0 = blockIdx.x * kW8Feat;
  const int nk_all = (a.K + 63) / 64;
  const int ks = g.ksplit, z = blockIdx.y;
  const int kb0 = z * nk_all / ks;
  const int nk = (z + 1) * nk_all / ks - kb0;
  // TMEM: np fp32 columns, allocated as a power of two of at least 32
  const uint32_t tcols = np <= 32 ? 32u : np <= 64 ? 64u : np <= 128 ? 128u : 256u;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(tcols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x == 32) {
    for (int s = 0; s < SW; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], wb ? 1 : kW8Conv);  // bf16 tiles are freed by the MMAs' commit
    }
    for (int s = 0; s < kW8RingA; ++s) {
      mbar_init(&afull[s], kW8Conv);
      mbar_init(&aempty[s], 1);
    }
    for (int s = 0; s < SX; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&xempty[s], 1);
    }
    mbar_init(&done, 1);
    s_fail = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  // kind::f16, D fp32, A and B bf16, both K-major, M = 128, N = np
  const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(np >> 3) << 17) |
                         (static_cast<uint32_t>(kW8Feat >> 4) << 24);

  if (warp == 0) {
    if (lane == 0) {
      // weight producer: SW tiles ahead; the weights do not depend on the
      // preceding kernel, so they stream before it has finished
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % SW;
        if (kb >= SW && !mbar_wait(&wempty[s], ((kb / SW) - 1) & 1)) {
          s_fail = 1;
          break;
        }
        mbar_expect_tx(&wfull[s], wslot);
        tma_load_2d(wring + s * wslot, &g.tma_w, (kb0 + kb) * 64, n0, &wfull[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // MMA issuer: four K = 16 products per k-block
      bool ok = true;
      for (int kb = 0; kb < nk; ++kb) {
        const int sa = kb % kW8RingA, sx = kb % SX, sw = kb % SW;
        const bool got = wb ? mbar_wait(&wfull[sw], (kb / SW) & 1) : mbar_wait(&afull[sa], (kb / kW8RingA) & 1);
        if (!got || !mbar_wait(&xfull[sx], (kb / SX) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t ua = wb ? smem_u32(wring + sw * kW8ABytes) : smem_u32(aring + sa * kW8ABytes);
        const uint32_t ux = smem_u32(xring + sx * np * 128);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc_mma(tmem, umma_desc_k128(ua + 32 * k), umma_desc_k128(ux + 32 * k), idesc, (kb | k) ? 1u : 0u);
        // the slots are free once these products have read them
        tc_commit(wb ? &wempty[sw] : &aempty[sa]);
        tc_commit(&xempty[sx]);
      }
      if (!ok) s_fail = 1;
      tc_commit(&done);
    }
  } else if (warp == 2) {
    if (lane == 0) {
      // row producer: the input rows are the preceding kernel's output
      pdl_wait();
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % SX;
        if (kb >= SX && !mbar_wait(&xempty[s], ((kb / SX) - 1) & 1)) {
          s_fail = 1;
          break;
        }
        mbar_expect_tx(&xfull[s], np * 128);
        tma_load_2d(xring + s * np * 128, &g.tma_x, (kb0 + kb) * 64, 0, &xfull[s]);
      }
    }
  } else {
    // converters: int8 tile -> bf16 tile in the 128-byte-swizzled K-major
    // layout (row r's 16-byte unit c at unit c ^ (r & 7)); a thread takes
    // 8-byte pieces (8 codes -> one 16-byte bf16 unit)
    const int t = threadIdx.x - 96;
    bool ok = true;
    for (int kb = 0; kb < (wb ? 0 : nk); ++kb) {
      const int sw = kb % SW, sa = kb % kW8RingA;
      ok = ok && mbar_wait(&wfull[sw], (kb / SW) & 1);
      if (kb >= kW8RingA) ok = ok && mbar_wait(&aempty[sa], ((kb / kW8RingA) - 1) & 1);
      const unsigned char *w8 = wring + sw * kW8WBytes;
      unsigned char *a16 = aring + sa * kW8ABytes;
      uint2 w[kW8WBytes / 8 / (32 * kW8Conv)];
#pragma unroll
      for (int j = 0; j < kW8WBytes / 8 / (32 * kW8Conv); ++j)
        w[j] = *reinterpret_cast<const uint2 *>(w8 + (t + 32 * kW8Conv * j) * 8);
      // the int8 slot is read: the producer may refill it
      __syncwarp();
      if (lane == 0) mbar_arrive_w8(&wempty[sw]);
#pragma unroll
      for (int j = 0; j < kW8WBytes / 8 / (32 * kW8Conv); ++j) {
        const int u = t + 32 * kW8Conv * j;   // 8-byte piece of the int8 tile
        const int r = u >> 3, c = u & 7;      // row, bf16 unit
        const uint2 lo = i8x4_to_bf16x4(w[j].x), hi = i8x4_to_bf16x4(w[j].y);
        *reinterpret_cast<uint4 *>(a16 + r * 128 + ((c ^ (r & 7)) << 4)) = make_uint4(lo.x, lo.y, hi.x, hi.y);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive_w8(&afull[sa]);
    }
    if (!ok) s_fail = 1;
    // row metadata of the QKV epilogue, while the products finish
    pdl_wait();
    if constexpr (EPI == kEpiQKV) {
      for (int r = t; r < a.R; r += 32 * kW8Conv) {
        s_req[r] = a.rows.req[r];
        s_pos[r] = a.rows.pos[r];
        s_slot[r] = row_slot(a.rows, r);
      }
    }
  }
  __syncthreads();
  pdl_launch();

  // epilogue: the 8 converter warps, thread = feature (its TMEM lane); the
  // two warpgroups take alternate 16-row chunks
  const bool epi_warp = warp >= 3;
  const int qd = warp & 3;
  const int grp = (warp - 3) >> 2;
  const int f = n0 + 32 * qd + lane;
  const bool fok = f < a.N;
  const uint32_t tl = tmem + (static_cast<uint32_t>(32 * qd) << 16);
  bool ok = true;
  if (epi_warp) {
    ok = __all_sync(0xffffffffu, mbar_wait(&done, 0) ? 1 : 0) != 0;  // tcgen05.ld is warp-collective
    tc_fence_after();
  }
  const bool good = ok && !s_fail;
  const float sc = (epi_warp && fok && a.scale) ? __ldg(a.scale + f) : 1.f;
  const float bi = (epi_warp && fok) ? __ldg(a.bias + f) : 0.f;
  if (ks == 1) {
    if (epi_warp && good) {
      for (int r0 = 16 * grp; r0 < a.R; r0 += 32) {
        float v[16];
        tmem_ld16(tl + r0, v);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int r = r0 + i;
          if (r >= a.R) break;  // uniform
          const int req = EPI == kEpiQKV ? s_req[r] : 0, pos = EPI == kEpiQKV ? s_pos[r] : 0;
          const int slot = EPI == kEpiQKV ? s_slot[r] : 0;
          w8_epilogue<EPI>(a, r, f, fok, v[i] * sc + bi, req, pos, slot, lane);
        }
      }
    }
  } else {
    // split-K: every rank stores its partial [row][feature] (128 threads
    // write 512 contiguous bytes per row), the cluster barrier, then rank z
    // sums rows [z R / ks, (z + 1) R / ks) over the ranks in order (the same
    // sum on every run), 8 rows per thread at a time
    const size_t tile = blockIdx.x;
    const float *ws = g.ws + tile * ks * static_cast<size_t>(np) * kW8Feat + 32 * qd + lane;
    if (epi_warp) {
      float *mine = const_cast<float *>(ws) + static_cast<size_t>(z) * np * kW8Feat;
      for (int r0 = 16 * grp; r0 < a.R; r0 += 32) {
        float v[16];
        tmem_ld16(tl + r0, v);
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (r0 + i < a.R) mine[static_cast<size_t>(r0 + i) * kW8Feat] = good ? v[i] : 0.f;
      }
      __threadfence();
    }
    cluster_sync_all();
    if (epi_warp && good) {
      const int r_lo = z * a.R / ks, r_hi = (z + 1) * a.R / ks;
      for (int rb = r_lo + 8 * grp; rb < r_hi; rb += 16) {
        float acc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = 0.f;
        for (int zz = 0; zz < ks; ++zz)
#pragma unroll
          for (int i = 0; i < 8; ++i)
            if (rb + i < r_hi) acc[i] += __ldcg(ws + (static_cast<size_t>(zz) * np + rb + i) * kW8Feat);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = rb + i;
          if (r >= r_hi) break;  // uniform
          const int req = EPI == kEpiQKV ? s_req[r] : 0, pos = EPI == kEpiQKV ? s_pos[r] : 0;
          const int slot = EPI == kEpiQKV ? s_slot[r] : 0;
          w8_epilogue<EPI>(a, r, f, fok, acc[i] * sc + bi, req, pos, slot, lane);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && (s_fail || !ok) && g.err) atomicOr(g.err, kErrTimeout);
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tcols) : "memory");
}

template <int EPI>
cudaError_t set_attr_epi() {
  return cudaFuncSetAttribute(gemm_w8_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, kW8SmemBudget + 1024);
}

template <int EPI>
cudaError_t launch_epi(const GemmW8Args &g, int tiles, cudaStream_t stream, bool pdl) {
  cudaLaunchConfig_t lc{};
  lc.gridDim = dim3(tiles, g.ksplit, 1);
  lc.blockDim = dim3(kW8Threads);
  lc.dynamicSmemBytes = gemm_w8_smem(g.np, g.w_bf16);
  lc.stream = stream;
  cudaLaunchAttribute at[2];
  int na = 0;
  if (g.ksplit > 1) {
    at[na].id = cudaLaunchAttributeClusterDimension;
    at[na].val.clusterDim.x = 1;
    at[na].val.clusterDim.y = g.ksplit;
    at[na].val.clusterDim.z = 1;
    ++na;
  }
  if (pdl) {
    at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  lc.attrs = at;
  lc.numAttrs = na;
  return cudaLaunchKernelEx(&lc, gemm_w8_kernel<EPI>, g);
}

}  // namespace

// Ring depths for np rows: the row ring (L2-resident tiles) 3-4 deep, the
// weight ring as deep as the rest of the budget allows (up to 16 tiles).
void gemm_w8_rings(int np, int w_bf16, int *sw, int *sx) {
  const int xb = np * 128;
  *sx = np <= 64 ? 4 : 3;
  const int left = kW8SmemBudget - (w_bf16 ? 0 : kW8RingA * kW8ABytes) - *sx * xb;
  *sw = std::max(2, std::min(kW8MaxW, left / (w_bf16 ? kW8ABytes : kW8WBytes)));
}

int gemm_w8_smem(int np, int w_bf16) {
  int sw, sx;
  gemm_w8_rings(np, w_bf16, &sw, &sx);
  return sw * (w_bf16 ? kW8ABytes : kW8WBytes) + (w_bf16 ? 0 : kW8RingA * kW8ABytes) + sx * np * 128 + 1024;
}

cudaError_t gemm_w8_set_attrs(int *active) {
  cudaError_t e = set_attr_epi<kEpiStore>();
  if (e == cudaSuccess) e = set_attr_epi<kEpiResid>();
  if (e == cudaSuccess) e = set_attr_epi<kEpiQKV>();
  if (e == cudaSuccess) e = set_attr_epi<kEpiSwiGLU>();
  if (e == cudaSuccess) e = set_attr_epi<kEpiGelu>();
  if (e != cudaSuccess) return e;
  for (int ks = 2; ks <= kW8MaxSplit; ks *= 2) {
    cudaLaunchConfig_t lc{};
    lc.gridDim = dim3(1, ks, 1);
    lc.blockDim = dim3(kW8Threads);
    lc.dynamicSmemBytes = kW8SmemBudget + 1024;
    cudaLaunchAttribute at{};
    at.id = cudaLaunchAttributeClusterDimension;
    at.val.clusterDim.x = 1;
    at.val.clusterDim.y = ks;
    at.val.clusterDim.z = 1;
    lc.attrs = &at;
    lc.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_w8_kernel<kEpiResid>, &lc) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    active[ks] = n;
  }
  return cudaSuccess;
}

cudaError_t gemm_w8_launch(int epi, const GemmW8Args &g, int tiles, cudaStream_t stream, bool pdl) {
  switch (epi) {
    case kEpiStore: return launch_epi<kEpiStore>(g, tiles, stream, pdl);
    case kEpiResid: return launch_epi<kEpiResid>(g, tiles, stream, pdl);
    case kEpiQKV: return launch_epi<kEpiQKV>(g, tiles, stream, pdl);
    case kEpiSwiGLU: return launch_epi<kEpiSwiGLU>(g, tiles, stream, pdl);
    case kEpiGelu: return launch_epi<kEpiGelu>(g, tiles, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace specdec
