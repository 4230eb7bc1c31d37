// Attention on the tensor cores for bf16 queries and a bf16 K/V cache with
// head_dim 64, for groups of many queries (token-tree verify blocks, prefill
// chunks): the same arithmetic as attention_kernel (src/nn/layer.cpp:859-948,
// score = q . k / sqrt(D), softmax over the visible positions, then P.V) with
// the two products as tcgen05 MMAs.
//
// A CTA takes up to 128 queries of one group (one request) and one head and
// walks the request's cache in tiles of 128 positions:
//   S = Q K^T      M = 128 queries, N = 128 positions, K = 64: A = the query
//                  tile (TMA, 128-byte swizzle, K-major), B = the K tile as
//                  the cache stores it (positions x dims: K-major);
//                  fp32 accumulators in TMEM columns [0, 128)
//   softmax        thread = query row = TMEM lane: the row's 128 scores are
//                  read with tcgen05.ld, masked (causal, tree ancestors),
//                  scaled by 1/8 and folded into the row's running max / sum
//   O_t = P V      M = 128, N = 64 dims, K = 128 positions: A = P as bf16 in
//                  shared memory (written by the threads in the 128-byte
//                  swizzled K-major layout), B = the V tile as the cache
//                  stores it (positions x dims: MN-major, 1024-byte groups of
//                  8 positions); TMEM columns [128, 192)
//   o = o * alpha + O_t in registers (the running rescale of the online softmax).
// K tiles stream through a two-stage TMA ring (tile t + 1 loads while tile t
// is multiplied); V has one buffer, refilled as soon as O_t is done, which
// leaves S_{t+1} and the softmax to cover its load and keeps the CTA at 97 KB
// of shared memory (two CTAs per SM).  P is rounded to bf16 for the second product (an
// error of at most 2^-9 relative per probability; bf16 activations already
// round every layer output to 8 bits).  Every mbarrier wait is bounded; on
// a timeout the CTA flags kErrTimeout and writes nothing.
#pragma once

#include "gemm.cuh"

namespace specdec {

constexpr int kAtcThreads = 256;  // two threads per query row (warps w and w + 4 share TMEM lanes)
constexpr int kAtcTile = 128;            // positions per tile
constexpr int kAtcD = 64;                // head dimension of this path
constexpr int kAtcMinQ = 16;             // groups with fewer queries keep attention_kernel
constexpr int kAtcQBytes = 128 * 128;    // Q tile: 128 rows x 64 bf16
constexpr int kAtcKVBytes = 128 * 128;   // K or V tile: 128 positions x 64 bf16
constexpr int kAtcPBytes = 2 * 128 * 128;  // P: 128 queries x 128 positions bf16, two 64-position blocks
// Q, two K stages, one V buffer, P: 96 KB (+ alignment), two CTAs per SM
constexpr int kAtcSmem = kAtcQBytes + 3 * kAtcKVBytes + kAtcPBytes + 1024;
constexpr int kAtcTmemCols = 256;        // S: 128 columns, O_t: 64 columns

// kind::f16, D fp32, A and B bf16; S: both K-major, N = 128; O: B MN-major, N = 64.
constexpr uint32_t kAtcIdescS = (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(128 >> 3) << 17) |
                                (static_cast<uint32_t>(128 >> 4) << 24);
constexpr uint32_t kAtcIdescO = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) |
                                (static_cast<uint32_t>(64 >> 3) << 17) | (static_cast<uint32_t>(128 >> 4) << 24);

// MN-major operand with the 128-byte swizzle whose MN extent is one 128-byte
// atom (64 bf16): rows along K 128 bytes apart, groups of 8 rows 1024 bytes
// apart (stride byte offset); the leading byte offset (between atoms along
// MN) is not used.
__device__ __forceinline__ uint64_t umma_desc_mn128(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

// Visibility of positions base .. base + 63 for a query at cache row qpos
// whose tree (if any) starts at qtb with ancestor mask qmask: bit j is set iff
// base + j <= qpos and (base + j < qtb, or bit base + j - qtb of qmask).
__device__ __forceinline__ uint64_t low_bits(long long n) {
  return n <= 0 ? 0ull : n >= 64 ? ~0ull : ((1ull << n) - 1ull);
}
__device__ __forceinline__ uint64_t vis_word(int base, int qpos, int qtb, unsigned long long qmask) {
  const uint64_t causal = low_bits(static_cast<long long>(qpos) + 1 - base);
  const uint64_t prefix = low_bits(static_cast<long long>(qtb) - base);
  const long long d = static_cast<long long>(base) - qtb;  // bit j <-> bit d + j of qmask
  const uint64_t tree = (d >= 64 || d <= -64) ? 0ull : d >= 0 ? (qmask >> d) : (qmask << (-d));
  return causal & (prefix | tree);
}

struct alignas(64) AttnTcArgs {
  CUtensorMap tmq;       // [R][dq] bf16 query rows, box 64 x 128
  CUtensorMap tmk, tmv;  // [cache row][64] bf16 page pools, box 64 x 128 (the attention_kernel maps)
  KvPages pg;
  RowsView rows;
  int R, Q;              // rows, queries per group
  int S_cap, H, Hkv;
  __nv_bfloat16 *out;    // [R][ldo]
  int ldo;
  int *err;
};

__global__ void __launch_bounds__(kAtcThreads, 2) attn_tc_kernel(const __grid_constant__ AttnTcArgs a) {
  pdl_wait();
  extern __shared__ unsigned char atc_smem_raw[];
  unsigned char *sm =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(atc_smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char *sq = sm;                       // Q tile
  unsigned char *sk = sq + kAtcQBytes;          // K stage s at sk + s * kAtcKVBytes
  unsigned char *sv = sk + 2 * kAtcKVBytes;     // V (one buffer: V_{t+1} loads once O_t is done)
  unsigned char *sp = sv + kAtcKVBytes;         // P, two blocks of 64 positions
  __shared__ __align__(8) uint64_t bar_q, bar_kv[2], bar_v, bar_s, bar_o;
  __shared__ uint32_t s_tmem;
  __shared__ int s_req, s_maxpos, s_fail;
  __shared__ float s_rmax[2][128], s_rsum[2][128];  // per column half: the rows' tile max / P sum

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ngt = (a.Q + 127) / 128;
  const int g = blockIdx.x / ngt, qt = blockIdx.x % ngt;
  const int h = blockIdx.y;
  const int rq0 = g * a.Q + qt * 128;
  const int nq = max(0, min(128, min(a.Q - qt * 128, a.R - rq0)));
  const int hk = h / (a.H / a.Hkv);

  // this thread's query row (its warp's TMEM lane quadrant) and column half
  const int r = 32 * (warp & 3) + lane, half = warp >> 2;
  const bool qv = r < nq;
  const int qreq = qv ? a.rows.req[rq0 + r] : -1;
  const int qpos = (qv && qreq >= 0) ? row_slot(a.rows, rq0 + r) : -1;
  const int qtb = (qv && a.rows.tb) ? a.rows.tb[rq0 + r] : 0x7fffffff;
  const unsigned long long qmask = (qv && a.rows.mask) ? a.rows.mask[rq0 + r] : 0ull;

  if (threadIdx.x == 0) {
    s_req = -1;
    s_maxpos = -1;
    s_fail = 0;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(kAtcTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x == 32) {
    mbar_init(&bar_q, 1);
    mbar_init(&bar_kv[0], 1);
    mbar_init(&bar_kv[1], 1);
    mbar_init(&bar_v, 1);
    mbar_init(&bar_s, 1);
    mbar_init(&bar_o, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (qreq >= 0) {
    atomicMax(&s_maxpos, qpos);
    s_req = qreq;  // every valid row of a group belongs to the same request
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  const int req = s_req, maxpos = s_maxpos;
  const bool work = req >= 0 && maxpos >= 0 && maxpos < a.S_cap;
  const int ntiles = work ? maxpos / kAtcTile + 1 : 0;
  // tile t = positions [128 t, 128 t + 128): one page
  auto tile_row = [&](int t) {
    const int y = kv_row(a.pg, a.Hkv, req, hk, t * kAtcTile);
    if (y >= 0) return y;
    if (a.err) atomicOr(a.err, kErrSeqLen);  // no page: flagged, a valid row is read instead
    return 0;
  };
  auto issue_k = [&](int t) {  // thread 0
    const int s = t & 1;
    mbar_expect_tx(&bar_kv[s], kAtcKVBytes);
    tma_load_2d(sk + s * kAtcKVBytes, &a.tmk, 0, tile_row(t), &bar_kv[s]);
  };
  auto issue_v = [&](int t) {  // thread 0
    mbar_expect_tx(&bar_v, kAtcKVBytes);
    tma_load_2d(sv, &a.tmv, 0, tile_row(t), &bar_v);
  };
  if (threadIdx.x == 0 && ntiles > 0) {
    mbar_expect_tx(&bar_q, kAtcQBytes);
    tma_load_2d(sq, &a.tmq, h * kAtcD, rq0, &bar_q);
    issue_k(0);
    issue_v(0);
  }

  float m = -INFINITY, l = 0.f;
  float o[kAtcD / 2];  // this thread's half of the row's output dims
#pragma unroll
  for (int e = 0; e < kAtcD / 2; ++e) o[e] = 0.f;
  const uint32_t trow = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);  // this warp's lanes
  bool ok = true;
  if (ntiles > 0 && threadIdx.x == 32) ok = mbar_wait(&bar_q, 0);
  int t = 0, failed_at = 0;  // 1: waiting for S, 2: waiting for O_t
  for (; t < ntiles; ++t) {
    const int s = t & 1;
    // S = Q K^T (thread 32 issues; the whole CTA waits for the product)
    if (threadIdx.x == 0 && t + 1 < ntiles) issue_k(t + 1);  // its stage was released after S_{t-1}
    if (threadIdx.x == 32) {
      if (ok) ok = mbar_wait(&bar_kv[s], (t >> 1) & 1);
      if (ok) {
        tc_fence_after();
        const uint32_t qa = smem_u32(sq), ka = smem_u32(sk + s * kAtcKVBytes);
#pragma unroll
        for (int k = 0; k < kAtcD / 16; ++k)
          tc_mma(tmem, umma_desc_k128(qa + 32 * k), umma_desc_k128(ka + 32 * k), kAtcIdescS, k ? 1u : 0u);
      }
      tc_commit(&bar_s);
    }
    __syncwarp();
    ok = __syncthreads_and((threadIdx.x == 32 ? ok : true) && mbar_wait(&bar_s, t & 1)) != 0;
    if (!ok) {
      failed_at = 1;
      break;
    }
    tc_fence_after();

    // softmax of this row's 128 scores: this thread takes the 64 positions of
    // its half (read from TMEM twice: max, then P); the row's visible
    // positions of that half as a 64-bit word
    const int t0 = t * kAtcTile;
    const uint64_t vw = vis_word(t0 + 64 * half, qpos, qtb, qmask);
    float tmax = -INFINITY;
    {
      float sc[64];
      tmem_ld64(trow + 64 * half, sc);
#pragma unroll
      for (int j = 0; j < 64; ++j) tmax = fmaxf(tmax, ((vw >> j) & 1ull) ? sc[j] * 0.125f : -INFINITY);
    }
    s_rmax[half][r] = tmax;
    __syncthreads();
    tmax = fmaxf(s_rmax[0][r], s_rmax[1][r]);
    const float mnew = fmaxf(m, tmax);  // / sqrt(64) above: a power of two, so exact
    const float alpha = (m == -INFINITY) ? 0.f : expf(m - mnew);
    float psum = 0.f;
    // P (bf16) into the swizzled K-major tile: row r, 16-byte unit uu of
    // block `half` (positions 64 half ..) lands at unit uu ^ (r & 7) of the row
    {
      float sc[64];
      tmem_ld64(trow + 64 * half, sc);
#pragma unroll
      for (int uu = 0; uu < 8; ++uu) {
        float p[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          p[e] = ((vw >> (8 * uu + e)) & 1ull) ? expf(sc[8 * uu + e] * 0.125f - mnew) : 0.f;
          psum += p[e];
        }
        *reinterpret_cast<uint4 *>(sp + half * (128 * 128) + r * 128 + ((uu ^ (r & 7)) << 4)) = f32x8_to_bf16(p);
      }
    }
    s_rsum[half][r] = psum;
    m = mnew;
    // the P stores must reach the tensor core's (async) view of shared memory
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    l = l * alpha + (s_rsum[0][r] + s_rsum[1][r]);  // both threads of the row add the halves in the same order
    // O_t = P V
    if (threadIdx.x == 32) {
      ok = mbar_wait(&bar_v, t & 1);
      tc_fence_after();
      const uint32_t pa = smem_u32(sp), va = smem_u32(sv);
      if (ok)
#pragma unroll
        for (int k = 0; k < kAtcTile / 16; ++k)
          tc_mma(tmem + 128, umma_desc_k128(pa + (k >> 2) * (128 * 128) + 32 * (k & 3)),
                 umma_desc_mn128(va + 2048 * k), kAtcIdescO, k ? 1u : 0u);
      tc_commit(&bar_o);
    }
    __syncwarp();
    ok = __syncthreads_and((threadIdx.x == 32 ? ok : true) && mbar_wait(&bar_o, t & 1)) != 0;
    if (!ok) {
      failed_at = 2;
      break;
    }
    tc_fence_after();
    if (threadIdx.x == 0 && t + 1 < ntiles) issue_v(t + 1);  // V is free once O_t is done
    {
      uint32_t u0[16], u1[16];
      tmem_ld16_nowait(trow + 128 + 32 * half, u0);
      tmem_ld16_nowait(trow + 128 + 32 * half + 16, u1);
      tmem_wait_ld();
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        o[e] = o[e] * alpha + __uint_as_float(u0[e]);
        o[16 + e] = o[16 + e] * alpha + __uint_as_float(u1[e]);
      }
    }
    tc_fence_before();
    __syncthreads();  // S, O_t and P are free for the next tile
  }

  if (!ok) {
    // bounded waits for this CTA's copies and products still in flight,
    // then the error flag
    if (threadIdx.x == 0) {
      s_fail = 1;
      mbar_wait(&bar_q, 0);
      mbar_wait(&bar_kv[t & 1], (t >> 1) & 1);  // tile t's K
      if (t + 1 < ntiles) mbar_wait(&bar_kv[(t + 1) & 1], ((t + 1) >> 1) & 1);  // the prefetched K
      mbar_wait(&bar_v, t & 1);  // tile t's V
      mbar_wait(failed_at == 1 ? &bar_s : &bar_o, t & 1);  // the product being waited for
      if (a.err) atomicOr(a.err, kErrTimeout);
    }
  } else if (qv && qreq >= 0 && ntiles > 0) {
    uint4 *dst = reinterpret_cast<uint4 *>(a.out + static_cast<size_t>(rq0 + r) * a.ldo + h * kAtcD + 32 * half);
#pragma unroll
    for (int u = 0; u < kAtcD / 16; ++u) {
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = __fdiv_rn(o[8 * u + e], l);
      dst[u] = f32x8_to_bf16(v);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kAtcTmemCols) : "memory");
}

}  // namespace specdec
