// Decode / verify attention on the tensor cores for head_dim 128: the
// arithmetic of attention_kernel (src/nn/layer.cpp:859-948: score = q . k /
// sqrt(D), softmax over the visible positions, then P.V) for groups of at
// most 16 query rows of one request -- draft steps (1 or 2 rows) and the
// (k+1)-row verify block -- over a bf16 cache, with both products on tcgen05.
//
// The cache is what these passes stream (2 x 128 x 2 bytes per position and
// head, about 1.2 MB per request and head on the large configuration), so the
// kernel is built to keep HBM busy: with few queries per group the positions
// go on the MMA's M side, one 128-position tile per product:
//   S^T = K Q^T    M = 128 positions, N = 16 query columns, K = 128 dims:
//                  A = the K tile as the cache stores it (K-major, 128-byte
//                  swizzle, two 64-dim atoms), B = the group's query rows
//                  (TMA, K-major); fp32 accumulators in TMEM, lane = position
//   softmax        thread = position: its 16 scores from one tcgen05.ld,
//                  masked (causal limit, tree ancestors) and divided by
//                  sqrt(128); per query the tile maximum over the 128 threads
//                  (warp shuffles + one named barrier), p = exp(s - m), P^T
//                  written as bf16 into a K-major swizzled tile
//   O^T = V^T P^T  M = 128 dims, N = 16, K = 128 positions: A = the V tile
//                  as the cache stores it (positions x dims: MN-major, two
//                  64-dim atoms 16 KB apart), B = P^T; TMEM lane = dim
//   o = o * alpha + O_t in registers (thread = dim), one tile behind, so the
//   fold overlaps the next tile's products.
// Warp 0 streams K and V tiles through a three-slot TMA ring per CTA (32 KB
// per slot; two CTAs per SM, 192 KB in flight per SM), K one tile ahead of V
// (K_0 K_1 V_0 K_2 V_1 ...: the ring releases slots in the order the MMAs
// read them, so no slot sits loaded while a V tile waits for its softmax
// and the next K queues behind it), warp 1 issues the
// MMAs, and one or two warpgroups do the softmax and the output: for a single
// query one warpgroup, for the 2-, 8- and 16-column variants (draft step 0,
// verify blocks) two warpgroups split the columns, which halves the
// per-thread softmax chain of a tile.  CTAs are persistent and walk work items
// (group, head, split) in a fixed order, so the ring never drains between
// items.  A (group, head) whose cache is split writes unnormalised partials;
// the last of its splits to finish (an arrival counter) merges them with the
// log-sum-exp rule.  Every mbarrier wait is bounded; a timeout raises
// kErrTimeout, the roles stop together and wait (bounded) for the copies and
// products still in flight before the CTA frees its tensor memory.
#include "attn_dec.cuh"
#include "gemm.cuh"

namespace specdec {

namespace {

constexpr int kAdSlots = 3;                      // ring slots of half a tile (K or V)
constexpr int kAdHalf = kAdTile * kAdD * 2;      // 32 KB: 128 positions x 128 bf16
constexpr int kAdBox = kAdTile * 64 * 2;         // 16 KB: one 64-dim atom of a half tile
constexpr int kAdQBytes = kAdN * kAdD * 2;       // 4 KB: 16 query rows, two 2 KB atoms
constexpr int kAdPBytes = kAdN * kAdTile * 2;    // 4 KB: 16 query rows x 128 positions, two atoms
// warp 0 TMA, warp 1 MMA, then the softmax warpgroups: one for a single query
// column, two (one, four or eight columns each) for the 2-, 8- and 16-column
// groups
constexpr int ad_qgroups(int nq) { return nq >= 2 ? 2 : 1; }
constexpr int ad_threads(int nq) { return 64 + 128 * ad_qgroups(nq); }
// three ring slots, two query buffers, one P buffer: 111 KB, two CTAs per SM
constexpr int kAdSmem = kAdSlots * kAdHalf + 2 * kAdQBytes + kAdPBytes + 1024;
constexpr int kAdTmemCols = 64;                  // S0 S1 O0 O1, 16 columns each
// 1 / sqrt(128) in fp32: the scores are scaled by a product (the reference
// divides by sqrt(D); the two differ by at most one rounding, far inside the
// bf16 tolerance of this path)
constexpr float kAdScale = 0.0883883476483184f;

// kind::f16, D fp32, A and B bf16, M = 128, N = 16.  S: A and B K-major.
// O: A (V^T) MN-major, B (P^T) K-major.
constexpr uint32_t kAdIdescS = (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(kAdN >> 3) << 17) |
                               (static_cast<uint32_t>(128 >> 4) << 24);
constexpr uint32_t kAdIdescO = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 15) |
                               (static_cast<uint32_t>(kAdN >> 3) << 17) | (static_cast<uint32_t>(128 >> 4) << 24);

// MN-major operand, 128-byte swizzle, MN extent of two 64-element atoms
// kAdBox bytes apart (leading byte offset); along K, rows 128 bytes apart and
// groups of 8 rows 1024 bytes apart (stride byte offset).
__device__ __forceinline__ uint64_t umma_desc_mn128_2atoms(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(kAdBox >> 4) << 16) |
         (64ull << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Named barrier of the N softmax threads that also ANDs a predicate over
// them, so a decision to stop is taken by all of them at the same point.
template <int N>
__device__ __forceinline__ bool bar_and_softmax(bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, 1, %2, p;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "n"(N)
      : "memory");
  return r != 0;
}
template <int N>
__device__ __forceinline__ void bar_softmax() {
  asm volatile("bar.sync 1, %0;" ::"n"(N) : "memory");
}

// NC accumulator columns of the warp's 32 TMEM lanes (NC = 4, 8 or 16), waited for.
template <int NC>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, float (&v)[NC]) {
  if constexpr (NC == 16) {
    tmem_ld16(taddr, v);
  } else if constexpr (NC == 4) {
    uint32_t r[4];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
  } else {
    static_assert(NC == 8, "4, 8 or 16 columns");
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
  }
}

// Warp reduction of NQ values per lane that leaves lane l with the result for
// query (l / (32 / NQ)): each halving step trades half of the values with
// the partner lane, so NQ queries cost NQ - 1 + log2(32) shuffles, not
// NQ * log2(32).  MAX: maximum, else sum.
template <int NQ, bool MAX>
__device__ __forceinline__ float warp_reduce_scatter(const float (&v)[NQ], int lane) {
  float w[NQ];
#pragma unroll
  for (int i = 0; i < NQ; ++i) w[i] = v[i];
  auto op = [](float a, float b) { return MAX ? fmaxf(a, b) : a + b; };
  int off = 16;
#pragma unroll
  for (int n = NQ; n > 1; n >>= 1, off >>= 1) {
    const bool hi = (lane & off) != 0;
#pragma unroll
    for (int j = 0; j < n / 2; ++j) {
      const float keep = hi ? w[j + n / 2] : w[j];
      const float send = hi ? w[j] : w[j + n / 2];
      w[j] = op(keep, __shfl_xor_sync(0xffffffffu, send, off));
    }
  }
#pragma unroll
  for (; off > 0; off >>= 1) w[0] = op(w[0], __shfl_xor_sync(0xffffffffu, w[0], off));
  return w[0];
}

// One work item: (group g, head h, split) and the range of cache tiles it
// covers.  The splits of a (group, head) share the tiles up to the group's
// last visible position, so every split has work while the cache is shorter
// than its capacity.
struct AdItem {
  int g, h, split, req, t0, nt, nq, rq0;
};
__device__ __forceinline__ AdItem ad_item(const AttnDecArgs &a, int item) {
  AdItem it;
  it.split = item % a.nsplit;
  const int gh = item / a.nsplit;
  it.h = gh % a.H;
  it.g = gh / a.H;
  it.rq0 = it.g * a.Q;
  it.nq = max(0, min(a.Q, a.R - it.rq0));
  it.req = -1;
  int maxpos = -1;
  for (int i = 0; i < it.nq; ++i) {
    const int r = a.rows.req[it.rq0 + i];
    if (r >= 0) {
      it.req = r;
      maxpos = max(maxpos, row_slot(a.rows, it.rq0 + i));
    }
  }
  it.t0 = 0;
  it.nt = 0;
  if (it.req >= 0 && maxpos >= 0 && maxpos < a.S_cap) {
    const int ntot = maxpos / kAdTile + 1;
    const int tps = (ntot + a.nsplit - 1) / a.nsplit;
    it.t0 = it.split * tps;
    it.nt = max(0, min(ntot, it.t0 + tps) - it.t0);
  }
  return it;
}

// Column j QH + h of a thread's NC loaded accumulator columns (h < QH, not a
// compile-time constant: a select, not an indexed register array).
template <int QH, int NC>
__device__ __forceinline__ float pick(const float (&v)[NC], int j, int h) {
  if constexpr (QH == 1) {
    return v[j];
  } else {
    static_assert(QH == 2, "one or two softmax warpgroups");
    return h ? v[2 * j + 1] : v[2 * j];
  }
}

// NQ: the group's queries rounded up to 1, 2, 8 or 16 (the columns the
// softmax threads carry; the MMAs always have 16).
template <int NQ>
__global__ void __launch_bounds__(ad_threads(NQ), 2) attn_dec_kernel(const __grid_constant__ AttnDecArgs a) {
  constexpr int QH = ad_qgroups(NQ);      // softmax warpgroups, each carrying NL query columns
  constexpr int NL = NQ / QH;
  constexpr int kSm = 128 * QH;           // softmax threads
  constexpr int NC = NQ <= 8 ? 8 : 16;  // TMEM columns read per product
  pdl_wait();
  extern __shared__ unsigned char ad_smem_raw[];
  unsigned char *ring =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(ad_smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char *sq = ring + kAdSlots * kAdHalf;  // two query buffers
  unsigned char *sp = sq + 2 * kAdQBytes;         // the P buffer
  __shared__ __align__(8) uint64_t full[kAdSlots], empty[kAdSlots], q_full[2], q_empty[2], s_full[2], s_free[2],
      p_full[2], o_full[2], o_free[2], mma_done;
  __shared__ uint32_t s_tmem;
  __shared__ volatile int s_abort;
  __shared__ int s_issued, s_consumed, s_q_issued, s_q_consumed, s_last;
  __shared__ __align__(16) float red[2][NQ][4];   // per query and softmax warp: the tile maximum
  __shared__ __align__(16) float lred[2][NQ][4];  // per query and softmax warp: the row sum

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(kAdTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x == 32) {
    for (int i = 0; i < kAdSlots; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4 * QH);
      mbar_init(&p_full[i], 4 * QH);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_free[i], 4 * QH);
    }
    mbar_init(&mma_done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_abort = 0;
    s_issued = s_consumed = s_q_issued = s_q_consumed = 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  auto give_up = [&]() {
    if (!s_abort) {
      s_abort = 1;
      if (a.err) atomicOr(a.err, kErrTimeout);
    }
  };

  if (warp == 0) {
    // ---- producer: query rows per item, then K and V half tiles ----------
    // Load order K_0 K_1 V_0 K_2 V_1 ... K_last V_last-1 V_last over the
    // CTA's tiles (T counts them across items): a K slot frees as soon as its
    // scores are on the tensor cores, so K of T + 1 is in flight while V of T
    // waits for its softmax.  Ring index of K_T: 2T - 1 (0 for T = 0); of V_T:
    // 2T + 2 (2T + 1 for the CTA's last tile).
    if (lane == 0) {
      int idx = 0, qi = 0;
      auto load = [&](const CUtensorMap *m, int y) -> bool {
        const int s = idx % kAdSlots;
        if (!mbar_wait(&empty[s], ((idx / kAdSlots) & 1) ^ 1) || s_abort) {
          give_up();
          return false;
        }
        mbar_expect_tx(&full[s], kAdHalf);
        tma_load_2d(ring + s * kAdHalf, m, 0, y, &full[s]);
        tma_load_2d(ring + s * kAdHalf + kAdBox, m, 64, y, &full[s]);
        s_issued = ++idx;
        return true;
      };
      bool stop = false, pend = false;
      int pend_y = 0;  // the cache row of the tile whose V is still to load
      for (int item = blockIdx.x; item < a.n_items && !s_abort && !stop; item += gridDim.x) {
        const AdItem it = ad_item(a, item);
        if (it.nt == 0) continue;
        const int qb = qi & 1;
        if (!mbar_wait(&q_empty[qb], ((qi >> 1) & 1) ^ 1)) {
          give_up();
          break;
        }
        mbar_expect_tx(&q_full[qb], kAdQBytes);
        tma_load_2d(sq + qb * kAdQBytes, &a.tmq, it.h * kAdD, it.rq0, &q_full[qb]);
        tma_load_2d(sq + qb * kAdQBytes + kAdQBytes / 2, &a.tmq, it.h * kAdD + 64, it.rq0, &q_full[qb]);
        s_q_issued = ++qi;
        for (int t = 0; t < it.nt; ++t) {
          int y = kv_row(a.pg, a.Hkv, it.req, it.h, (it.t0 + t) * kAdTile);
          if (y < 0) {  // no page: flagged, a valid row is read instead
            if (a.err) atomicOr(a.err, kErrSeqLen);
            y = 0;
          }
          if (!load(&a.tmk, y) || (pend && !load(&a.tmv, pend_y))) {
            stop = true;
            break;
          }
          pend = true;
          pend_y = y;
        }
      }
      if (!stop && !s_abort && pend) load(&a.tmv, pend_y);
    }
  } else if (warp == 1) {
    // ---- MMA issuer --------------------------------------------------------
    // Order S_0, S_1, O_0, S_2, O_1, ...: the scores of tile T + 1 are on the
    // tensor cores while the softmax of tile T runs.  K of tile T has ring
    // index 2T - 1 (0 for T = 0), V has 2T + 2, or 2T + 1 on the last tile
    // (the producer's order).
    if (lane == 0) {
      struct Cur {
        int item, t, qb;
        AdItem it;
      };
      auto seek = [&](int item, AdItem &it) {  // the next item with tiles, at or after `item`
        for (; item < a.n_items; item += gridDim.x) {
          it = ad_item(a, item);
          if (it.nt > 0) return item;
        }
        return a.n_items;
      };
      auto issue_s = [&](int T, const Cur &c) -> bool {
        const int idx = T ? 2 * T - 1 : 0, sk = idx % kAdSlots, sb = T & 1;
        if (!mbar_wait(&full[sk], (idx / kAdSlots) & 1) || !mbar_wait(&s_free[sb], ((T >> 1) & 1) ^ 1) || s_abort)
          return false;
        tc_fence_after();
        const uint32_t ka = smem_u32(ring + sk * kAdHalf), qa = smem_u32(sq + c.qb * kAdQBytes);
#pragma unroll
        for (int kk = 0; kk < kAdD / 16; ++kk)
          tc_mma(tmem + 16 * sb, umma_desc_k128(ka + (kk >> 2) * kAdBox + 32 * (kk & 3)),
                 umma_desc_k128(qa + (kk >> 2) * (kAdQBytes / 2) + 32 * (kk & 3)), kAdIdescS, kk ? 1u : 0u);
        tc_commit(&empty[sk]);
        tc_commit(&s_full[sb]);
        return true;
      };
      auto issue_o = [&](int T, bool last) -> bool {
        const int idx = last ? 2 * T + 1 : 2 * T + 2, sv = idx % kAdSlots, sb = T & 1;
        const uint32_t ph = (T >> 1) & 1;
        if (!mbar_wait(&full[sv], (idx / kAdSlots) & 1) || !mbar_wait(&p_full[sb], ph) ||
            !mbar_wait(&o_free[sb], ph ^ 1) || s_abort)
          return false;
        tc_fence_after();
        const uint32_t va = smem_u32(ring + sv * kAdHalf), pa = smem_u32(sp);
#pragma unroll
        for (int kk = 0; kk < kAdTile / 16; ++kk)
          tc_mma(tmem + 32 + 16 * sb, umma_desc_mn128_2atoms(va + 2048 * kk),
                 umma_desc_k128(pa + (kk >> 2) * (kAdPBytes / 2) + 32 * (kk & 3)), kAdIdescO, kk ? 1u : 0u);
        tc_commit(&empty[sv]);
        tc_commit(&o_full[sb]);
        return true;
      };
      int qcount = 0;  // items whose queries were waited for
      Cur c;
      c.item = seek(blockIdx.x, c.it);
      c.t = 0;
      c.qb = 0;
      const bool work = c.item < a.n_items;  // this CTA may have only empty splits
      bool ok = true;
      if (work) {
        ok = mbar_wait(&q_full[0], 0);
        s_q_consumed = qcount = 1;
        if (ok) ok = issue_s(0, c);
        if (ok) s_consumed = 1;  // the lowest ring index not yet taken
      }
      for (int T = 0; work && ok; ++T) {
        Cur n = c;
        bool more = true;
        if (c.t + 1 < c.it.nt) {
          n.t = c.t + 1;
        } else {
          n.item = seek(c.item + gridDim.x, n.it);
          n.t = 0;
          more = n.item < a.n_items;
          if (more) {
            n.qb = qcount & 1;
            ok = mbar_wait(&q_full[n.qb], (qcount >> 1) & 1);
            s_q_consumed = ++qcount;
          }
        }
        if (ok && more) ok = issue_s(T + 1, n);
        if (ok) {
          ok = issue_o(T, !more);
          if (ok) s_consumed = more ? 2 * T + 3 : 2 * T + 2;
        }
        if (ok && c.t + 1 == c.it.nt) tc_commit(&q_empty[c.qb]);
        if (!more) break;
        c = n;
      }
      if (!ok) give_up();
      // every product this thread issued has completed before the CTA moves on
      tc_commit(&mma_done);
      if (!mbar_wait(&mma_done, 0)) give_up();
    }
  } else {
    // ---- softmax and output: thread = position of a tile, and = dim of O ---
    // QH warpgroups of four warps: warpgroup h carries query columns
    // h, h + QH, h + 2 QH, ... of every position (its warps cover the four
    // TMEM lane quadrants), so a thread's softmax chain per tile is NL columns
    // long, and the real columns of a group (5 of 8 for k = 4) spread 3 + 2
    const int qd = warp & 3;  // TMEM lane quadrant of this warp
    const int h = (warp - 2) >> 2;
    const int p = 32 * qd + lane;
    const int own = lane / (32 / NL);  // the query (own QH + h) this lane holds after a reduce-scatter
    const bool owner = (lane % (32 / NL)) == 0;
    const uint32_t tl = tmem + (static_cast<uint32_t>(32 * qd) << 16);
    int T = 0, ni = 0;
    // ok: the last barrier's verdict (the same in every softmax thread); lok:
    // this thread's own waits so far, folded into ok at the next barrier, so
    // the softmax warps always stop at the same point
    bool ok = true, lok = true;
    for (int item = blockIdx.x; item < a.n_items; item += gridDim.x, ++ni) {
      const AdItem it = ad_item(a, item);
      int qpos[NL], qtb[NL];
      unsigned long long qmask[NL];
#pragma unroll
      for (int j = 0; j < NL; ++j) {
        const int q = j * QH + h;
        const int r = it.rq0 + q;
        const bool v = q < it.nq && a.rows.req[r] >= 0;
        qpos[j] = v ? row_slot(a.rows, r) : -1;
        qtb[j] = (v && a.rows.tb) ? a.rows.tb[r] : 0x7fffffff;
        qmask[j] = (v && a.rows.mask) ? a.rows.mask[r] : 0ull;
      }
      float m[NL], l[NL], o[NL], al_prev[NL];
#pragma unroll
      for (int j = 0; j < NL; ++j) {
        m[j] = -INFINITY;
        l[j] = 0.f;
        o[j] = 0.f;
        al_prev[j] = 0.f;
      }
      auto fold = [&](int Tp) -> bool {  // o = o * alpha + O_{Tp}
        const int ob = Tp & 1;
        const bool w = mbar_wait(&o_full[ob], (Tp >> 1) & 1);
        tc_fence_after();
        float ov[NC];
        tmem_ld_cols<NC>(tl + 32 + 16 * ob, ov);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&o_free[ob]);
#pragma unroll
        for (int j = 0; j < NL; ++j) o[j] = o[j] * al_prev[j] + pick<QH>(ov, j, h);
        return w;
      };
      for (int t = 0; t < it.nt; ++t, ++T) {
        const int sb = T & 1;
        lok = mbar_wait(&s_full[sb], (T >> 1) & 1) && lok;
        tc_fence_after();
        float sc[NC];
        tmem_ld_cols<NC>(tl + 16 * sb, sc);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[sb]);
        const int pos = (it.t0 + t) * kAdTile + p;
        float s[NL];
#pragma unroll
        for (int j = 0; j < NL; ++j) {
          // causal, and inside a token tree only the prefix, the ancestors and itself
          const bool vis = pos <= qpos[j] &&
                           (pos < qtb[j] || (pos - qtb[j] < 64 && ((qmask[j] >> (pos - qtb[j])) & 1ull)));
          s[j] = vis ? pick<QH>(sc, j, h) * kAdScale : -INFINITY;
        }
        {
          const float wm = warp_reduce_scatter<NL, true>(s, lane);
          if (owner) red[sb][own * QH + h][qd] = wm;
        }
        ok = bar_and_softmax<kSm>(lok && !s_abort);
        if (!ok) break;
        float al[NL], pr[NL];
#pragma unroll
        for (int j = 0; j < NL; ++j) {
          const int q = j * QH + h;
          al[j] = 1.f;
          pr[j] = 0.f;
          if (q < it.nq) {  // uniform over the CTA: columns past the group's queries do no work
            const float4 r4 = *reinterpret_cast<const float4 *>(&red[sb][q][0]);
            const float mn = fmaxf(m[j], fmaxf(fmaxf(r4.x, r4.y), fmaxf(r4.z, r4.w)));
            // the running maximum is the same in every thread: when the tile
            // leaves it unchanged the rescale is 1 without an exponential
            if (mn != m[j]) al[j] = (m[j] == -INFINITY) ? 0.f : __expf(m[j] - mn);
            // P is rounded to bf16 for the product: the fast exponential's
            // error (a few ulp of fp32) is far below that rounding
            pr[j] = (s[j] == -INFINITY) ? 0.f : __expf(s[j] - mn);
            l[j] = l[j] * al[j] + pr[j];
            m[j] = mn;
          }
        }
        // O_{T-1} into the registers: then its product has read P, which
        // tile T overwrites
        if (t > 0) lok = fold(T - 1) && lok;
        // P^T as bf16: row q, position p of the K-major swizzled tile.  Rows
        // of the columns past the group's queries keep whatever they hold:
        // column q of O^T depends on row q of P^T alone, and those columns are
        // never read.
        {
          unsigned char *pt = sp + (p >> 6) * (kAdPBytes / 2);
          const int chunk = (p & 63) >> 3, byte = (p & 7) * 2;
#pragma unroll
          for (int j = 0; j < NL; ++j) {
            const int q = j * QH + h;
            if (q < it.nq)
              *reinterpret_cast<__nv_bfloat16 *>(pt + q * 128 + ((chunk ^ (q & 7)) << 4) + byte) =
                  __float2bfloat16_rn(pr[j]);
          }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[sb]);
#pragma unroll
        for (int j = 0; j < NL; ++j) al_prev[j] = al[j];
      }
      if (ok && it.nt > 0) lok = fold(T - 1) && lok;
      // the row sums over the 128 positions
      const int lb = ni & 1;
      {
        const float ws = warp_reduce_scatter<NL, false>(l, lane);
        if (owner) lred[lb][own * QH + h][qd] = ws;
      }
      ok = bar_and_softmax<kSm>(ok && lok && !s_abort);
      if (!ok) break;
      float L[NL];
#pragma unroll
      for (int j = 0; j < NL; ++j) {
        const float4 r4 = *reinterpret_cast<const float4 *>(&lred[lb][j * QH + h][0]);
        L[j] = (r4.x + r4.y) + (r4.z + r4.w);
      }
      if (a.nsplit == 1) {
#pragma unroll
        for (int j = 0; j < NL; ++j)
          if (qpos[j] >= 0 && qpos[j] < a.S_cap)
            a.out[static_cast<size_t>(it.rq0 + j * QH + h) * a.ldo + it.h * kAdD + p] =
                __float2bfloat16_rn(L[j] > 0.f ? __fdiv_rn(o[j], L[j]) : 0.f);
        continue;
      }
      // split: this item's partial, then the last split of (group, head) merges
      // (whether any query of the group is valid is the same for every split,
      // and for both warpgroups: they read the same rows)
      bool any = false;
      for (int q = 0; q < it.nq; ++q) any |= a.rows.req[it.rq0 + q] >= 0;
      if (!any) continue;
      float *pp = a.part + static_cast<size_t>(item) * kAdPartFloats;
#pragma unroll
      for (int j = 0; j < NL; ++j) pp[(j * QH + h) * kAdD + p] = o[j];
#pragma unroll
      for (int j = 0; j < NL; ++j)
        if (p == j * QH + h) {
          pp[kAdN * kAdD + p] = m[j];
          pp[kAdN * kAdD + kAdN + p] = L[j];
        }
      __threadfence();
      bar_softmax<kSm>();
      const int gh = item / a.nsplit;
      if (p == 0 && h == 0) s_last = (atomicAdd(a.ticket + gh, 1) == a.nsplit - 1) ? 1 : 0;
      bar_softmax<kSm>();
      if (s_last) {
        __threadfence();
        const float *p0 = a.part + static_cast<size_t>(gh) * a.nsplit * kAdPartFloats;
#pragma unroll 1
        for (int j = 0; j < NL; ++j) {
          const int q = j * QH + h;
          if (qpos[j] < 0 || qpos[j] >= a.S_cap) continue;
          float M = -INFINITY;
          for (int s2 = 0; s2 < a.nsplit; ++s2) {
            const float *ps = p0 + static_cast<size_t>(s2) * kAdPartFloats;
            if (__ldcg(ps + kAdN * kAdD + kAdN + q) > 0.f) M = fmaxf(M, __ldcg(ps + kAdN * kAdD + q));
          }
          float num = 0.f, den = 0.f;
          for (int s2 = 0; s2 < a.nsplit; ++s2) {
            const float *ps = p0 + static_cast<size_t>(s2) * kAdPartFloats;
            const float Ls = __ldcg(ps + kAdN * kAdD + kAdN + q);
            if (Ls > 0.f) {
              const float wgt = expf(__ldcg(ps + kAdN * kAdD + q) - M);
              num += wgt * __ldcg(ps + q * kAdD + p);
              den += wgt * Ls;
            }
          }
          a.out[static_cast<size_t>(it.rq0 + q) * a.ldo + it.h * kAdD + p] =
              __float2bfloat16_rn(den > 0.f ? __fdiv_rn(num, den) : 0.f);
        }
        if (p == 0 && h == 0) a.ticket[gh] = 0;
      }
      bar_softmax<kSm>();  // s_last is rewritten by the next item
    }
    if (!ok) give_up();
  }

  pdl_launch();
  __syncthreads();
  // after a timeout: bounded waits for the copies still in flight
  if (s_abort && threadIdx.x == 0) {
    for (int idx = s_consumed; idx < s_issued; ++idx) mbar_wait(&full[idx % kAdSlots], (idx / kAdSlots) & 1);
    for (int qi = s_q_consumed; qi < s_q_issued; ++qi) mbar_wait(&q_full[qi & 1], (qi >> 1) & 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kAdTmemCols) : "memory");
}

}  // namespace

int attn_dec_smem_bytes() { return kAdSmem; }

namespace {
template <int NQ>
cudaError_t set_one() {
  return cudaFuncSetAttribute(attn_dec_kernel<NQ>, cudaFuncAttributeMaxDynamicSharedMemorySize, kAdSmem);
}
template <int NQ>
cudaError_t launch_one(const AttnDecArgs &a, int grid, cudaStream_t stream, bool pdl) {
  cudaLaunchConfig_t lc{};
  lc.gridDim = dim3(grid);
  lc.blockDim = dim3(ad_threads(NQ));
  lc.dynamicSmemBytes = kAdSmem;
  lc.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = at;
  lc.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&lc, attn_dec_kernel<NQ>, a);
}
}  // namespace

cudaError_t attn_dec_set_attrs() {
  cudaError_t e = set_one<1>();
  if (e == cudaSuccess) e = set_one<2>();
  if (e == cudaSuccess) e = set_one<8>();
  if (e == cudaSuccess) e = set_one<16>();
  return e;
}

cudaError_t attn_dec_launch(const AttnDecArgs &a, int grid, cudaStream_t stream, bool pdl) {
  if (a.Q <= 1) return launch_one<1>(a, grid, stream, pdl);
  if (a.Q <= 2) return launch_one<2>(a, grid, stream, pdl);
  if (a.Q <= 8) return launch_one<8>(a, grid, stream, pdl);
  return launch_one<16>(a, grid, stream, pdl);
}

int attn_dec_ctas_per_sm() { return 2; }

}  // namespace specdec
