// Decode / verify attention on the tensor cores for head_dim 128 (the large
// configuration: 32 heads x 128, bf16 queries and KV cache): arguments and
// the host launch wrapper of attn_dec.cu.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include "forward.cuh"

namespace specdec {

constexpr int kAdD = 128;      // head dimension of this path
constexpr int kAdTile = 128;   // cache positions per tile
constexpr int kAdN = 16;       // query columns per item (a group of at most 16 rows of one request)
constexpr int kAdMaxSplit = 8;  // splits of one (group, head) over its cache

struct alignas(64) AttnDecArgs {
  CUtensorMap tmq;       // [R][dq] bf16 query rows, box 64 x 16, 128-byte swizzle
  CUtensorMap tmk, tmv;  // [cache row][128] bf16 page pools, box 64 x 128, 128-byte swizzle
  KvPages pg;            // tile T of a request = positions [128 T, 128 T + 128) = one page
  RowsView rows;
  int R, Q;              // rows of the pass, rows per group (one request each)
  int S_cap, H, Hkv;     // positions per request; heads (H == Hkv)
  int n_items;           // groups * H * nsplit
  int nsplit;            // splits of one (group, head)
  __nv_bfloat16 *out;    // [R][ldo]
  int ldo;
  float *part;           // nsplit > 1: per item the unnormalised output [16][128] then max [16] and sum [16]
  int *ticket;           // nsplit > 1: per (group, head) the splits done so far (0 between launches)
  int *err;
};

// Floats of one item's partial result (nsplit > 1).
constexpr int kAdPartFloats = kAdN * kAdD + 2 * kAdN;

// Dynamic shared memory of attn_dec_kernel.
int attn_dec_smem_bytes();
// Sets the kernel's shared-memory attribute (once per device).
cudaError_t attn_dec_set_attrs();
// Launches attn_dec_kernel with `grid` persistent CTAs on `stream`
// (programmatic stream serialization when pdl is set).  Its variant carries
// the group's queries rounded up to 1, 2, 8 or 16.
cudaError_t attn_dec_launch(const AttnDecArgs &a, int grid, cudaStream_t stream, bool pdl);
// CTAs of the kernel resident per SM (its shared memory fits two).
int attn_dec_ctas_per_sm();

}  // namespace specdec
