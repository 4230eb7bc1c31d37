// Tensor-core linear layer for large row batches (prefill, wide verify and
// tree blocks) with bf16 activations: y = x . W^T on tcgen05, fp32
// accumulators in tensor memory, the same epilogues as the GEMV
// (scale and bias, residual, RoPE + cache append, SwiGLU, GELU, logits).
//
// CTA tile kBM x kBN = 128 x 256, K in steps of kBK = 64 bf16 (one 128-byte
// swizzle span).  Thread 0 streams A (activation rows, [R][K]) and B
// (weight rows, [N][K]) tiles with TMA (128-byte swizzle, no multicast) into
// a kStages-deep ring; thread 32 issues tcgen05.mma (M = 128, N = 256,
// K = 16 per instruction, both operands K-major from shared memory) and
// releases each stage with tcgen05.commit; after the last commit all four
// warps read their 32 accumulator lanes (= rows) with tcgen05.ld and run the
// epilogue on column pairs.  int8 weights are multiplied as their exact bf16
// images (|q| <= 127) and scaled per output column in the epilogue, the
// reassociation sum(x * q) * s that the GEMV uses too.
//
// Split-K for grids of few tiles (verify blocks of a few hundred rows through
// narrow layers): the ksplit CTAs of one tile form a thread-block cluster
// along z, rank z multiplying k-blocks [z nk / ks, (z + 1) nk / ks).  Their
// partial tiles meet in an L2-resident workspace (column-major, so a warp's
// stores and loads are contiguous; distributed shared memory measured several
// times slower for 128 KB per CTA), the cluster barrier orders them, and rank
// j adds the ks partials of its column slice in rank order (the same sum on
// every run) and runs the epilogue on its 256 / ks columns.
//
// Epilogue.  The residual operand is staged in the freed ring with
// coalesced row loads (one memory round trip instead of one per chunk), and
// store / residual / GELU / SwiGLU outputs are staged there too and written
// by whole rows with coalesced 16-byte stores.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "forward.cuh"

namespace specdec {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;
constexpr int kStages = 4;
constexpr int kGemmThreads = 128;
constexpr int kGemmMinRows = 64;                        // below this the GEMV is used
constexpr int kGemmABytes = kBM * kBK * 2;              // 16 KB
constexpr int kGemmBBytes = kBN * kBK * 2;              // 32 KB
constexpr int kGemmStageBytes = kGemmABytes + kGemmBBytes;
constexpr int kGemmSmem = kStages * kGemmStageBytes + 1024;
constexpr int kTmemCols = 256;                          // fp32 accumulator columns (one per output column)
constexpr int kGemmMaxSplit = 8;                        // portable cluster size

struct alignas(64) GemmArgs {
  CUtensorMap tma_a;  // [R][K] bf16 rows, box kBK x kBM, 128-byte swizzle
  CUtensorMap tma_b;  // bf16 weight image in tile order ([tile][k-block][256][64]), box kBK x kBN, 128-byte swizzle
  LinearArgs lin;     // epilogue operands (out, scale, bias, resid, rows, qkv), R, N, K
  int *err;
  int ksplit;         // CTAs per tile along z (a cluster), 1, 2, 4 or 8
  float *ws;          // split-K partial tiles: [tile * ksplit + rank][kBN columns][kBM rows] fp32
};

// The freed ring holds the epilogue's residual slice and output staging,
// rows padded by 16 bytes.
static_assert(kBM * (kBN * 2 + 16) * 2 <= kStages * kGemmStageBytes && kBM * (kBN * 4 + 16) <= kStages * kGemmStageBytes,
              "epilogue staging must fit the TMA ring");

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n barrier.cluster.wait.acquire.aligned;" ::: "memory");
}


// Shared-memory matrix descriptor of a K-major operand tile whose rows are
// 128 bytes with the 128-byte swizzle: 8-row core groups 1024 bytes apart
// (stride byte offset), version 1, layout type 2 (128-byte swizzle).
__device__ __forceinline__ uint64_t umma_desc_k128(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
         (2ull << 61);
}

// Instruction descriptor of kind::f16: D fp32, A and B bf16, both K-major,
// N = kBN, M = kBM.
constexpr uint32_t kGemmIdesc = (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(kBN >> 3) << 17) |
                                (static_cast<uint32_t>(kBM >> 4) << 24);

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
// Arrives on `bar` once every tcgen05.mma this thread issued so far has completed.
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Loads without waiting: 16 accumulator columns of the warp's 32 lanes; the
// values are valid after tmem_wait_ld().  Several loads share one wait, so
// their latencies overlap.
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// 64 consecutive accumulator columns (four loads, one wait).
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
  uint32_t r[4][16];
#pragma unroll
  for (int q = 0; q < 4; ++q) tmem_ld16_nowait(taddr + 16 * q, r[q]);
  tmem_wait_ld();
#pragma unroll
  for (int q = 0; q < 4; ++q)
#pragma unroll
    for (int i = 0; i < 16; ++i) v[16 * q + i] = __uint_as_float(r[q][i]);
}

// Row operands of one 16-column chunk (columns n .. n + 15 of row `row`),
// fetched one chunk ahead of use: the residual values (Resid) or the RoPE
// (cos, sin) pairs (QKV).  kBN and the q / k / v section widths are multiples
// of 16 and head_dim is a multiple of 16 on this path, so a chunk never
// straddles a head or a section.
struct ChunkOps {
  float v[16];
};

__device__ __forceinline__ void bf16x8_to_f32(uint4 u, float *f) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
__device__ __forceinline__ uint4 f32x8_to_bf16(const float *f) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 t = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t *>(&t);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

template <int EPI>
__device__ __forceinline__ void chunk_load(const LinearArgs &a, int row, int n, int req, int pos, ChunkOps &op) {
  if constexpr (EPI == kEpiResid) {
    const __nv_bfloat16 *rs = static_cast<const __nv_bfloat16 *>(a.resid) + static_cast<size_t>(row) * a.ldr + n;
    if (n + 16 <= a.N) {
      bf16x8_to_f32(__ldg(reinterpret_cast<const uint4 *>(rs)), op.v);
      bf16x8_to_f32(__ldg(reinterpret_cast<const uint4 *>(rs + 8)), op.v + 8);
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) op.v[j] = (n + j < a.N) ? __bfloat162float(rs[j]) : 0.f;
    }
  } else if constexpr (EPI == kEpiQKV) {
    const QKVArgs &q = a.qkv;
    if (req >= 0 && pos >= 0 && pos < q.rope_max_pos && n < q.d + q.kvd) {
      const int e = (n < q.d ? n : n - q.d) % q.D;
      const float4 *t = reinterpret_cast<const float4 *>(q.rope + static_cast<size_t>(pos) * (q.D / 2) + (e >> 1));
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 c = __ldg(t + i);
        op.v[4 * i] = c.x; op.v[4 * i + 1] = c.y; op.v[4 * i + 2] = c.z; op.v[4 * i + 3] = c.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; j += 2) {
        op.v[j] = 1.f;
        op.v[j + 1] = 0.f;
      }
    }
  }
}

// Arithmetic of the staged epilogues (store, residual, GELU, SwiGLU) on one
// 16-column chunk in place; SwiGLU leaves its 8 outputs in v[0 .. 7].  The
// same operations, in the same order, as chunk_store.
template <int EPI>
__device__ __forceinline__ void chunk_apply(float (&v)[16], const ChunkOps &op, const float *ssc, const float *sbi) {
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = v[j] * ssc[j] + sbi[j];
  if constexpr (EPI == kEpiResid) {
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = v[j] + op.v[j];
  } else if constexpr (EPI == kEpiGelu) {
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = 0.5f * v[j] * (1.0f + erff(v[j] * 0.70710678118654752f));
  } else if constexpr (EPI == kEpiSwiGLU) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float g = v[2 * i], u = v[2 * i + 1];
      const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
      v[i] = __fmul_rn(__fmul_rn(g, sg), u);
    }
  }
}

// Epilogue of one chunk: the arithmetic of linear_epilogue, with the
// chunk's outputs stored as 16-byte vectors.
template <int EPI>
__device__ __forceinline__ void chunk_store(const LinearArgs &a, int row, int n, float (&v)[16], const ChunkOps &op,
                                            const float *ssc, const float *sbi, int req, int pos, int slot) {
  using AT = __nv_bfloat16;
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = v[j] * ssc[j] + sbi[j];
  const bool full = n + 16 <= a.N;
  if constexpr (EPI == kEpiStore || EPI == kEpiResid || EPI == kEpiGelu) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if constexpr (EPI == kEpiResid) v[j] = v[j] + op.v[j];
      if constexpr (EPI == kEpiGelu) v[j] = 0.5f * v[j] * (1.0f + erff(v[j] * 0.70710678118654752f));
    }
    if (a.out_f32) {
      float *o = static_cast<float *>(a.out) + static_cast<size_t>(row) * a.ldo + n;
      if (full) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          reinterpret_cast<float4 *>(o)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
      } else {
        for (int j = 0; j < 16 && n + j < a.N; ++j) o[j] = v[j];
      }
    } else {
      AT *o = static_cast<AT *>(a.out) + static_cast<size_t>(row) * a.ldo + n;
      if (full) {
        reinterpret_cast<uint4 *>(o)[0] = f32x8_to_bf16(v);
        reinterpret_cast<uint4 *>(o)[1] = f32x8_to_bf16(v + 8);
      } else {
        for (int j = 0; j < 16 && n + j < a.N; ++j) o[j] = __float2bfloat16_rn(v[j]);
      }
    }
  } else if constexpr (EPI == kEpiSwiGLU) {
    // SwiGLU::forward (src/nn/layer.cpp:1704-1710) on the interleaved pairs
    float y[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float g = v[2 * i], u = v[2 * i + 1];
      const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
      y[i] = __fmul_rn(__fmul_rn(g, sg), u);
    }
    AT *o = static_cast<AT *>(a.out) + static_cast<size_t>(row) * a.ldo + (n >> 1);
    if (full) *reinterpret_cast<uint4 *>(o) = f32x8_to_bf16(y);
    else
      for (int i = 0; i < 8 && n + 2 * i + 1 < a.N; ++i) o[i] = __float2bfloat16_rn(y[i]);
  } else if constexpr (EPI == kEpiQKV) {
    if (req < 0) return;
    const QKVArgs &q = a.qkv;
    if (pos < 0 || pos >= q.rope_max_pos || slot < 0 || slot >= q.S_cap) {
      if (q.err) atomicOr(q.err, kErrSeqLen);
      return;
    }
    if (n < q.d + q.kvd) {
      // Tensor::rope (src/core/tensor.cpp:1144-1163) on pairs (2j, 2j+1)
#pragma unroll
      for (int j = 0; j < 16; j += 2) {
        const float c = op.v[j], sn = op.v[j + 1];
        const float x0 = __fsub_rn(__fmul_rn(v[j], c), __fmul_rn(v[j + 1], sn));
        const float x1 = __fadd_rn(__fmul_rn(v[j], sn), __fmul_rn(v[j + 1], c));
        v[j] = x0;
        v[j + 1] = x1;
      }
    }
    if (n < q.d) {
      uint4 *o = reinterpret_cast<uint4 *>(static_cast<AT *>(a.out) + static_cast<size_t>(row) * a.ldo + n);
      o[0] = f32x8_to_bf16(v);
      o[1] = f32x8_to_bf16(v + 8);
    } else {
      const bool is_k = n < q.d + q.kvd;
      const int nn = is_k ? n - q.d : n - q.d - q.kvd;
      const int h = nn / q.D, e = nn % q.D;
      const int crow = kv_row(q.pg, q.kvd / q.D, req, h, slot);
      if (crow < 0) {
        if (q.err) atomicOr(q.err, kErrSeqLen);
        return;
      }
      const size_t off = static_cast<size_t>(crow) * q.D + e;
      if (q.kv_mode == 2) {
        float4 *st = reinterpret_cast<float4 *>(q.stage + static_cast<size_t>(row) * 2 * q.kvd + (is_k ? 0 : q.kvd) + nn);
#pragma unroll
        for (int i = 0; i < 4; ++i) st[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
      } else if (q.kv_mode == 1) {
        uint4 *c = reinterpret_cast<uint4 *>(static_cast<AT *>(is_k ? q.kc : q.vc) + off);
        c[0] = f32x8_to_bf16(v);
        c[1] = f32x8_to_bf16(v + 8);
      } else {
        float4 *c = reinterpret_cast<float4 *>(static_cast<float *>(is_k ? q.kc : q.vc) + off);
#pragma unroll
        for (int i = 0; i < 4; ++i) c[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
      }
    }
  }
}

template <int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_kernel(const __grid_constant__ GemmArgs g) {
  extern __shared__ unsigned char gemm_smem_raw[];
  unsigned char *tiles =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(gemm_smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[kStages], empty[kStages], done;
  __shared__ uint32_t s_tmem;
  __shared__ int s_fail;
  __shared__ __align__(16) float s_scale[kBN], s_bias[kBN];

  const LinearArgs &a = g.lin;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kBN, m0 = blockIdx.y * kBM;
  const int nk_all = (a.K + kBK - 1) / kBK;
  const int ks = g.ksplit, z = blockIdx.z;  // the cluster spans z only: rank = z
  const int kb0 = z * nk_all / ks;
  const int nk = (z + 1) * nk_all / ks - kb0;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x == 32) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&done, 1);
    s_fail = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  // programmatic dependent launch: the successor may launch now and waits in
  // griddepcontrol.wait for this grid; this grid's reads of its predecessors'
  // outputs (input rows, residual, row tables) and all its writes come after
  // its own wait, so the set-up above overlaps the predecessor's tail
  pdl_launch();
  pdl_wait();

  if (warp >= 2) {
    // the epilogue's per-column operands, while the main loop runs
    for (int j = threadIdx.x - 64; j < kBN; j += 64) {
      const int n = n0 + j;
      s_scale[j] = (n < a.N && a.scale) ? __ldg(a.scale + n) : 1.f;
      s_bias[j] = n < a.N ? __ldg(a.bias + n) : 0.f;
    }
  }
  if (threadIdx.x == 0) {
    // producer: TMA tiles into the ring
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % kStages;
      if (kb >= kStages && !mbar_wait(&empty[s], ((kb / kStages) - 1) & 1)) {
        s_fail = 1;
        break;
      }
      unsigned char *sa = tiles + s * kGemmStageBytes;
      unsigned char *sb = sa + kGemmABytes;
      mbar_expect_tx(&full[s], kGemmStageBytes);
      tma_load_2d(sa, &g.tma_a, (kb0 + kb) * kBK, m0, &full[s]);
      tma_load_2d(sb, &g.tma_b, 0, (blockIdx.x * nk_all + kb0 + kb) * kBN, &full[s]);
    }
  } else if (threadIdx.x == 32) {
    // MMA issuer
    bool ok = true;
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % kStages;
      if (!mbar_wait(&full[s], (kb / kStages) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t sa = smem_u32(tiles + s * kGemmStageBytes);
      const uint32_t sb = sa + kGemmABytes;
#pragma unroll
      for (int k = 0; k < kBK / 16; ++k)
        tc_mma(tmem, umma_desc_k128(sa + 32 * k), umma_desc_k128(sb + 32 * k), kGemmIdesc, (kb | k) ? 1u : 0u);
      tc_commit(&empty[s]);  // the stage is free once these MMAs have read it
    }
    if (!ok) s_fail = 1;
    tc_commit(&done);
  }
  __syncwarp();

  // epilogue: warp w owns accumulator lanes (rows) 32w .. 32w + 31
  const bool ok = __all_sync(0xffffffffu, mbar_wait(&done, 0) ? 1 : 0) != 0;  // tcgen05.ld is warp-collective
  if (!ok) s_fail = 1;
  tc_fence_after();
  __syncthreads();  // the per-column scale and bias are in shared memory
  const int row = m0 + warp * 32 + lane;
  const bool row_ok = row < a.R;
  int req = 0, pos = 0, slot = 0;
  if constexpr (EPI == kEpiQKV) {
    req = row_ok ? a.rows.req[row] : -1;
    pos = row_ok ? a.rows.pos[row] : 0;
    slot = row_ok ? row_slot(a.rows, row) : 0;
  }
  const int ncols = min(kBN, a.N - n0);
  const int lr = warp * 32 + lane;  // this thread's tile row (accumulator lane)
  const uint32_t tbase = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  // this CTA's output columns within the tile: all 256, or its split-K slice
  const int ew = kBN / ks, ec0 = z * ew;
  const int ecols = max(0, min(ew, ncols - ec0));
  const int wrows = max(0, min(32, a.R - m0 - warp * 32));  // valid rows of this warp (uniform)
  // The ring is free once every MMA is done: [split-K exchange][residual
  // slice][output staging], each row padded by 16 bytes (a warp's row-strided
  // 16-byte accesses then hit distinct bank groups).
  unsigned char *rstage = tiles;
  const int rs_ld = ew * 2 + 16;
  if constexpr (EPI == kEpiResid) {
    // the residual slice, row by row with coalesced 16-byte asynchronous
    // copies, all in flight at once (one memory round trip)
    const int nu = (ecols + 7) / 8;
    if (ok && lane < nu) {
      for (int rr = 0; rr < wrows; ++rr) {
        const __nv_bfloat16 *src =
            static_cast<const __nv_bfloat16 *>(a.resid) + static_cast<size_t>(m0 + warp * 32 + rr) * a.ldr + n0 + ec0;
        unsigned char *dst = rstage + (warp * 32 + rr) * rs_ld + lane * 16;
        if (lane * 8 + 8 <= ecols) {
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)),
                       "l"(reinterpret_cast<const uint4 *>(src) + lane)
                       : "memory");
        } else {
          uint32_t w[4] = {0u, 0u, 0u, 0u};
          const unsigned short *sp = reinterpret_cast<const unsigned short *>(src);
          for (int e = 0; e < 8 && lane * 8 + e < ecols; ++e)
            w[e >> 1] |= static_cast<uint32_t>(sp[lane * 8 + e]) << ((e & 1) * 16);
          *reinterpret_cast<uint4 *>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncwarp();
  }
  auto resid_chunk = [&](int c, ChunkOps &op) {  // c: column within this CTA's slice
    const uint4 *sp = reinterpret_cast<const uint4 *>(rstage + lr * rs_ld + c * 2);
    bf16x8_to_f32(sp[0], op.v);
    bf16x8_to_f32(sp[1], op.v + 8);
  };

  if (ks > 1) {
    // split-K: every rank stores its partial tile column by column (a warp
    // covers 128 contiguous bytes) into the L2-resident workspace; after the
    // cluster barrier rank z sums column slice z of the ks partials in rank
    // order (the same sum on every run) and runs the epilogue on it.
    const size_t tile = static_cast<size_t>(blockIdx.x) + static_cast<size_t>(gridDim.x) * blockIdx.y;
    float *mine = g.ws + (tile * ks + z) * (kBN * kBM) + lr;
    // (rows past R -- 96 of the 128 in a 32-row draft step -- are neither
    // stored nor read: the exchange moves only the launch's real rows)
    for (int c0 = 0; c0 < ncols; c0 += 64) {
      float v[64];
      tmem_ld64(tbase + c0, v);  // warp-collective
      if (row_ok)
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (c0 + i < ncols) mine[(c0 + i) * kBM] = ok ? v[i] : 0.f;
    }
    __threadfence();
    cluster_sync_all();
    const float *part = g.ws + tile * ks * (kBN * kBM) + static_cast<size_t>(ec0) * kBM + lr;
    for (int c = 0; c < ecols; c += 16) {
      if (!(row_ok && ok)) break;
      float v[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = 0.f;
      for (int zz = 0; zz < ks; ++zz)
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] += __ldcg(part + static_cast<size_t>(zz) * (kBN * kBM) + (c + i) * kBM);
      {
        const int n = n0 + ec0 + c;
        ChunkOps op;
        if constexpr (EPI == kEpiResid) resid_chunk(c, op);
        else chunk_load<EPI>(a, row, n, req, pos, op);
        chunk_store<EPI>(a, row, n, v, op, s_scale + ec0 + c, s_bias + ec0 + c, req, pos, slot);
      }
    }
  } else if (ok) {
    if constexpr (EPI == kEpiQKV) {
      // chunks of 16 columns, the next chunk's RoPE operands in flight
      ChunkOps op0, op1;
      if (row_ok) chunk_load<EPI>(a, row, n0, req, pos, op0);
      for (int c = 0; c < ncols; c += 32) {
        float v[16];
        if (row_ok && c + 16 < ncols) chunk_load<EPI>(a, row, n0 + c + 16, req, pos, op1);
        tmem_ld16(tbase + c, v);
        if (row_ok) chunk_store<EPI>(a, row, n0 + c, v, op0, s_scale + c, s_bias + c, req, pos, slot);
        if (c + 16 >= ncols) break;  // warp-uniform
        if (row_ok && c + 32 < ncols) chunk_load<EPI>(a, row, n0 + c + 32, req, pos, op0);
        tmem_ld16(tbase + c + 16, v);
        if (row_ok) chunk_store<EPI>(a, row, n0 + c + 16, v, op1, s_scale + c + 16, s_bias + c + 16, req, pos, slot);
      }
    } else {
      // outputs staged in shared memory by row, then stored by the warp with
      // coalesced 16-byte stores
      const bool f32 = a.out_f32 != 0 && EPI != kEpiSwiGLU;
      const int oelt = f32 ? 4 : 2;
      const int ow = EPI == kEpiSwiGLU ? ew / 2 : ew;
      const int os_ld = ow * oelt + 16;
      unsigned char *ostage = rstage + (EPI == kEpiResid ? kBM * rs_ld : 0);
      unsigned char *orow = ostage + lr * os_ld;
      for (int c0 = 0; c0 < ncols; c0 += 64) {
        float vv[64];
        tmem_ld64(tbase + c0, vv);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int c = c0 + 16 * q;
          if (c >= ncols) break;  // warp-uniform
          float v[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = vv[16 * q + i];
          ChunkOps op;
          if constexpr (EPI == kEpiResid) resid_chunk(c, op);
          chunk_apply<EPI>(v, op, s_scale + c, s_bias + c);
          if constexpr (EPI == kEpiSwiGLU) {
            *reinterpret_cast<uint4 *>(orow + (c / 2) * 2) = f32x8_to_bf16(v);
          } else if (f32) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
              reinterpret_cast<float4 *>(orow + c * 4)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          } else {
            reinterpret_cast<uint4 *>(orow + c * 2)[0] = f32x8_to_bf16(v);
            reinterpret_cast<uint4 *>(orow + c * 2)[1] = f32x8_to_bf16(v + 8);
          }
        }
      }
      __syncwarp();
      const int ocols = EPI == kEpiSwiGLU ? ncols / 2 : ncols;  // valid output columns (N even for SwiGLU)
      const int obytes = ocols * oelt;
      const size_t ocol0 = EPI == kEpiSwiGLU ? static_cast<size_t>(n0 / 2) : static_cast<size_t>(n0);
      for (int rr = 0; rr < wrows; ++rr) {
        unsigned char *gdst = static_cast<unsigned char *>(a.out) +
                              (static_cast<size_t>(m0 + warp * 32 + rr) * a.ldo + ocol0) * oelt;
        const unsigned char *ssrc = ostage + (warp * 32 + rr) * os_ld;
        for (int u = lane; u * 16 < obytes; u += 32) {
          if (u * 16 + 16 <= obytes) {
            *reinterpret_cast<uint4 *>(gdst + u * 16) = *reinterpret_cast<const uint4 *>(ssrc + u * 16);
          } else if (f32) {
            for (int e = u * 4; e < ocols; ++e)
              reinterpret_cast<float *>(gdst)[e] = reinterpret_cast<const float *>(ssrc)[e];
          } else {
            for (int e = u * 8; e < ocols; ++e)
              reinterpret_cast<unsigned short *>(gdst)[e] = reinterpret_cast<const unsigned short *>(ssrc)[e];
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && s_fail && g.err) atomicOr(g.err, kErrTimeout);
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

// LayerNorm of R input rows (optionally gathered through in_rows), one warp
// per row, written as contiguous rows [R][K] of the activation type (the A
// operand of the GEMM, or the input of a GEMV) and, when norm_out is set,
// also there.  Lane l holds elements 8 (l + 32 j) .. + 7 from 16-byte loads,
// NV of them per lane (rows up to 256 NV wide).  Requires K % 8 == 0 and
// 16-byte aligned rows.
template <int NV>
__global__ void ln_rows_kernel(const __nv_bfloat16 *__restrict__ x, int ldx, const int *__restrict__ in_rows, int R,
                               int K, const float *__restrict__ g, const float *__restrict__ b,
                               __nv_bfloat16 *__restrict__ out, __nv_bfloat16 *__restrict__ norm_out) {
  pdl_launch();
  pdl_wait();  // the rows come from the predecessor
  const int lane = threadIdx.x & 31;
  const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= R) return;
  const int pr = in_rows ? in_rows[r] : r;
  const uint4 *xr = reinterpret_cast<const uint4 *>(x + static_cast<size_t>(pr) * ldx);
  const int nv = K / 8;
  float v[NV][8];
  // eight independent partial sums per lane (no 8 NV-long dependent chain)
  float s8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = lane + 32 * j;
    if (c < nv) {
      bf16x8_to_f32(__ldg(xr + c), v[j]);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[j][e] = 0.f;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) s8[e] += v[j][e];
  }
  const float s = ((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7]));
  const float mean = __fdiv_rn(warp_sum(s), static_cast<float>(K));
  float q8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < NV; ++j)
    if (lane + 32 * j < nv)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float df = v[j][e] - mean;
        q8[e] = fmaf(df, df, q8[e]);
      }
  const float q = ((q8[0] + q8[1]) + (q8[2] + q8[3])) + ((q8[4] + q8[5]) + (q8[6] + q8[7]));
  const float sd = sqrtf(__fdiv_rn(warp_sum(q), static_cast<float>(K)) + 1e-5f);
  // bf16 outputs: the product by the reciprocal of sd differs from the
  // quotient by at most one fp32 rounding, far below the output's bf16 rounding
  const float rsd = __fdiv_rn(1.0f, sd);
  uint4 *y = reinterpret_cast<uint4 *>(out + static_cast<size_t>(r) * K);
  uint4 *no = norm_out ? reinterpret_cast<uint4 *>(norm_out + static_cast<size_t>(r) * K) : nullptr;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = lane + 32 * j;
    if (c < nv) {
      const float4 g0 = __ldg(reinterpret_cast<const float4 *>(g) + 2 * c), g1 = __ldg(reinterpret_cast<const float4 *>(g) + 2 * c + 1);
      const float4 b0 = __ldg(reinterpret_cast<const float4 *>(b) + 2 * c), b1 = __ldg(reinterpret_cast<const float4 *>(b) + 2 * c + 1);
      const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
      const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = __fadd_rn(__fmul_rn(__fmul_rn(v[j][e] - mean, rsd), gg[e]), bb[e]);
      const uint4 w = f32x8_to_bf16(o);
      y[c] = w;
      if (no) no[c] = w;
    }
  }
}

// int8 weight codes -> their exact bf16 values.
// The exact bf16 image of int8 codes [N][K] in the tensor-core GEMM's tile
// order: block (t, kb) = weight rows 256 t .. 256 t + 255, columns
// 64 kb .. 64 kb + 63, stored as 32 contiguous KB ([256][64], zeros past N
// and K) at block index t * nkb + kb.  One TMA box of the GEMM is then one
// contiguous read; in the row-major [N][K] layout it was 256 segments of
// 128 bytes, K * 2 bytes apart.
static __global__ void i8_to_bf16_tiles_kernel(const int8_t *__restrict__ q, __nv_bfloat16 *__restrict__ out, int N,
                                               int K, int nkb, size_t total) {
  for (size_t o = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; o < total;
       o += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t blk = o / (kBN * kBK);
    const int within = static_cast<int>(o % (kBN * kBK));
    const int r = within / kBK, c = within % kBK;
    const int t = static_cast<int>(blk / nkb), kb = static_cast<int>(blk % nkb);
    const int n = t * kBN + r, k = kb * kBK + c;
    out[o] = __float2bfloat16_rn((n < N && k < K) ? static_cast<float>(q[static_cast<size_t>(n) * K + k]) : 0.f);
  }
}

}  // namespace specdec
