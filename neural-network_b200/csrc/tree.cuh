// Token-tree speculation (no counterpart in the reference; the tree
// extension of TransformerDecoder::generate_speculative, src/nn/layer.cpp:
// 1382-1661).  Per round and request:
//
//   draft expansion  level 0 is the chain's first draft pass over [catch-up,
//                    root]; every node at depth t < L then gets the branch[t]
//                    largest draft logits as children (ties to the lower id),
//                    and the nodes at depths 1 .. L-1 are fed to the draft
//                    level by level with an ancestor mask;
//   verify           one target pass over [root, all nodes] with the mask;
//   accept           from the root, a node's children are tried in rank order
//                    as point-mass proposals: greedy takes the child equal to
//                    the target argmax; sampled takes child c when u < p(c),
//                    else p(c) = 0 and p is renormalised (this samples exactly
//                    from p); with no child taken the token is drawn from what
//                    is left of p, and after an accepted leaf a bonus token is
//                    drawn from the leaf's p;
//   compaction       the accepted nodes' K/V rows move to the positions after
//                    the root in both caches (no other copy: the tree slots
//                    past them are overwritten by the next round).
//
// A node at depth t sits at RoPE position root + t and in cache slot
// root + 1 + (its BFS index); its ancestor mask holds its own bit and its
// ancestors' bits (at most 64 nodes).
#pragma once

#include "sample.cuh"

namespace specdec {

// Children of every node at depth `depth` (0: the root) from the draft logits
// of the pass that fed those nodes; one block per (request, node).  Writes the
// children's tokens, their rows in the next draft level (when depth + 1 < L)
// and their rows in the verify block.
__global__ void __launch_bounds__(kSampThreads) tree_topk_kernel(SpecState st, int depth, const float *__restrict__ logits) {
  __shared__ SampShared sh;
  __shared__ int s_kid[kTreeMaxNodes];
  extern __shared__ float srow[];  // [V]
  const int b = blockIdx.x, i = blockIdx.y;
  if (!st.active[b]) return;
  const int nl = depth == 0 ? 1 : st.tlev[depth] - st.tlev[depth - 1];
  if (i >= nl) return;
  const int node = depth == 0 ? -1 : st.tlev[depth - 1] + i;
  // level 0 reads the root's row of the first draft pass (one selected row per
  // request); deeper levels read their own pass's rows
  const size_t row = depth == 0 ? static_cast<size_t>(b) : static_cast<size_t>(b) * nl + i;
  load_row(logits + row * st.V, st.V, srow);
  const int nb = st.tbr[depth];
  for (int r = 0; r < nb; ++r) {
    const int am = argmax_smem(srow, st.V, sh.redv, sh.redi);
    if (threadIdx.x == 0) {
      s_kid[r] = am;
      srow[am] = -INFINITY;
    }
    __syncthreads();
  }
  if (threadIdx.x < nb) {
    const int r = threadIdx.x;
    const int c = tree_first_child(st, node, depth) + r;
    const int tok = s_kid[r];
    st.ttok[b * kTreeMaxNodes + c] = tok;
    const unsigned long long m = tree_mask(st, c);
    const int t = st.t_start[b], dr = st.d_root[b];
    if (depth + 1 < st.tL)
      set_tree_row(st, tree_level_row(st, b, depth + 1, i * nb + r), tok, dr + depth + 1, b, dr + 1 + c, dr + 1, m);
    set_tree_row(st, tree_verify_row(st, b, 1 + c), tok, t + depth + 1, b, t + 1 + c, t + 1, m);
  }
}

// Acceptance walk over the verify block's logits (rows [root, node 0 .. N-1]
// per request); one block per request.
__global__ void __launch_bounds__(kSampThreads) tree_accept_kernel(SpecState st, const float *__restrict__ logits) {
  __shared__ SampShared sh;
  __shared__ int s_acc;
  extern __shared__ float srow[];  // [V]
  const int b = blockIdx.x;
  if (!st.active[b]) {
    if (threadIdx.x == 0) st.cp_n[b] = 0;  // nothing for the compaction kernel
    return;
  }
  RngCtx rc = make_rng(sh);
  const int round = st.round[b];
  const float *lg0 = logits + static_cast<size_t>(b) * (st.tN + 1) * st.V;
  const int *tok = st.ttok + b * kTreeMaxNodes;
  if (!st.greedy) rng_prepare(st, b, st.tL * st.tbmax + 2, rc);
  const int n0 = st.n_new[b];
  const int Leff = min(st.tL, st.max_new - n0);

  int node = -1, d = 0, npath = 0, out_tok = -1;
  int path[kTreeMaxDepth];
  bool rejected = false;
  while (d < Leff) {
    load_row(lg0 + static_cast<size_t>(node + 1) * st.V, st.V, srow);
    const int c0 = tree_first_child(st, node, d), nb = st.tbr[d];
    int acc = -1;
    if (st.greedy) {
      const int am = argmax_smem(srow, st.V, sh.redv, sh.redi);
      for (int r = 0; r < nb; ++r)
        if (tok[c0 + r] == am) {
          acc = c0 + r;
          break;
        }
      if (acc < 0) out_tok = am;
    } else {
      probs_smem(srow, st.V, st.T, st.top_k, st.top_p, sh.red, sh.cut);
      for (int r = 0; r < nb && acc < 0; ++r) {
        const int c = tok[c0 + r];
        if (threadIdx.x == 0) {
          const float u = draw_accept_u(st, b, round, d * st.tbmax + r, rc);
          s_acc = u < srow[c] ? 1 : 0;
        }
        __syncthreads();
        if (s_acc) {
          acc = c0 + r;
        } else {
          // p(c) = 0, renormalised
          if (threadIdx.x == 0) srow[c] = 0.f;
          __syncthreads();
          float sum = 0.f;
          for (int v = threadIdx.x; v < st.V; v += blockDim.x) sum += srow[v];
          sum = block_sum(sum, sh.red);
          if (sum > 0.f)
            for (int v = threadIdx.x; v < st.V; v += blockDim.x) srow[v] = __fdiv_rn(srow[v], sum);
        }
        __syncthreads();
      }
      if (acc < 0) {
        if (threadIdx.x == 0) sh.u = draw_sample_u(st, b, round, st.tL * st.tbmax, rc);
        __syncthreads();
        out_tok = sample_smem(srow, st.V, sh.u, st.rng_mode, sh.redd, sh.redi);
      }
    }
    if (acc < 0) {
      rejected = true;
      break;
    }
    path[npath++] = acc;
    node = acc;
    ++d;
  }
  if (!rejected && n0 + npath < st.max_new) {
    // bonus token from the last accepted node (the root when Leff = 0)
    load_row(lg0 + static_cast<size_t>(node + 1) * st.V, st.V, srow);
    if (st.greedy) {
      out_tok = argmax_smem(srow, st.V, sh.redv, sh.redi);
    } else {
      probs_smem(srow, st.V, st.T, st.top_k, st.top_p, sh.red, sh.cut);
      if (threadIdx.x == 0) sh.u = draw_sample_u(st, b, round, st.tL * st.tbmax, rc);
      __syncthreads();
      out_tok = sample_smem(srow, st.V, sh.u, st.rng_mode, sh.redd, sh.redi);
    }
  }
  if (!st.greedy) rng_commit(st, b, rc);
  if (threadIdx.x == 0) {
    for (int j = 0; j < npath; ++j) emit(st, b, tok[path[j]]);
    if (out_tok >= 0) emit(st, b, out_tok);
    // compaction of the accepted nodes (the next kernel)
    const int t = st.t_start[b], dr = st.d_root[b];
    const int ndraft = min(npath, st.tL - 1);  // nodes the draft has seen
    st.cp_t0[b] = t;
    st.cp_d0[b] = dr;
    st.cp_n[b] = npath;
    st.cp_dn[b] = ndraft;
    for (int j = 0; j < npath; ++j) st.cp_path[b * kTreeMaxDepth + j] = path[j];
    st.t_len[b] = t + 1 + npath;
    st.d_len[b] = dr + 1 + ndraft;
    // an accepted leaf has not been fed to the draft: next round's catch-up
    const int catch_tok = (npath > ndraft) ? tok[path[npath - 1]] : -1;
    if (out_tok >= 0) st.last_tok[b] = out_tok;
    else if (npath > 0) st.last_tok[b] = tok[path[npath - 1]];
    long long *sx = st.stats + 4 * b;
    sx[0] += 1;
    sx[1] += st.tN;
    sx[2] += npath;
    sx[3] += rejected ? 1 : 0;
    st.round[b] = round + 1;
    bool still = st.n_new[b] < st.max_new;
    if (still) still = tree_start_round(st, b, out_tok >= 0 ? catch_tok : -1);
    else tree_clear_rows(st, b);
    st.active[b] = still ? 1 : 0;
    if (still) atomicAdd(st.active_count, 1);
  }
}

// One model's KV cache as the compaction kernel sees it.
struct CacheView {
  void *k, *v;        // [layer][cache row][D] page pools
  float *ks, *vs;     // int8 cache: [layer][cache row] scales, else null
  size_t layer_elems;
  KvPages pg;         // the requests' page tables
  int S_cap, Hkv, D, L, elt;
};

// Moves the accepted path's K/V rows to the positions right after the root,
// in both caches (grid: requests x (target layers + draft layers)).  Each
// thread owns fixed (head, element) columns and walks the path from the root
// side, so a row is read before any later copy can overwrite it (every
// source slot is at or above its destination).
__global__ void tree_compact_kernel(SpecState st, CacheView tc, CacheView dc) {
  const int b = blockIdx.x;
  const int n = st.cp_n[b];
  if (n == 0) return;
  const bool tgt = static_cast<int>(blockIdx.y) < tc.L;
  const CacheView &c = tgt ? tc : dc;
  const int layer = tgt ? blockIdx.y : blockIdx.y - tc.L;
  const int cnt = tgt ? n : st.cp_dn[b];
  const int root = tgt ? st.cp_t0[b] : st.cp_d0[b];
  const int *path = st.cp_path + b * kTreeMaxDepth;
  const size_t base = layer * c.layer_elems;
  const int per = c.Hkv * c.D;
  for (int x = threadIdx.x; x < per; x += blockDim.x) {
    const int h = x / c.D, e = x % c.D;
    for (int j = 0; j < cnt; ++j) {
      const int src = root + 1 + path[j], dst = root + 1 + j;
      if (src == dst) continue;
      const int rs = kv_row(c.pg, c.Hkv, b, h, src), rd = kv_row(c.pg, c.Hkv, b, h, dst);
      if (rs < 0 || rd < 0) continue;  // the verify pass flagged positions without pages
      const size_t so = base + static_cast<size_t>(rs) * c.D + e;
      const size_t dof = base + static_cast<size_t>(rd) * c.D + e;
      if (c.elt == 4) {
        static_cast<float *>(c.k)[dof] = static_cast<const float *>(c.k)[so];
        static_cast<float *>(c.v)[dof] = static_cast<const float *>(c.v)[so];
      } else if (c.elt == 2) {
        static_cast<__nv_bfloat16 *>(c.k)[dof] = static_cast<const __nv_bfloat16 *>(c.k)[so];
        static_cast<__nv_bfloat16 *>(c.v)[dof] = static_cast<const __nv_bfloat16 *>(c.v)[so];
      } else {
        static_cast<int8_t *>(c.k)[dof] = static_cast<const int8_t *>(c.k)[so];
        static_cast<int8_t *>(c.v)[dof] = static_cast<const int8_t *>(c.v)[so];
        if (e == 0) {
          const size_t sb = base / c.D;
          c.ks[sb + rd] = c.ks[sb + rs];
          c.vs[sb + rd] = c.vs[sb + rs];
        }
      }
    }
  }
}

}  // namespace specdec
