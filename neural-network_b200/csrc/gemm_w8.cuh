// Tensor-core linear layer for row batches of at most 256 rows (draft steps,
// verify blocks) over int8 weights: arguments and host wrappers of gemm_w8.cu.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include "forward.cuh"

namespace specdec {

constexpr int kW8MaxRows = 256;  // rows of a pass this kernel takes (the MMA's N)
constexpr int kW8Feat = 128;     // output features per CTA (the MMA's M)
constexpr int kW8MaxSplit = 8;   // splits of K per feature tile (a cluster along y)

struct alignas(64) GemmW8Args {
  CUtensorMap tma_w;  // int8 weight codes [N][K], box 64 x 128, no swizzle
  CUtensorMap tma_x;  // bf16 input rows [R][K], box 64 x np, 128-byte swizzle
  LinearArgs lin;     // epilogue operands (out, scale, bias, resid, rows, qkv), R, N, K
  int np;             // R rounded up to 16 (the MMA's N)
  int stages_w;       // int8 weight tiles in flight
  int stages_x;       // input-row tiles in flight
  int ksplit;         // CTAs per feature tile along y (a cluster), each a contiguous range of K
  int w_bf16;         // 1: tma_w is the codes' bf16 image [N][K] (box 64 x 128, 128-byte swizzle), no conversion
  float *ws;          // ksplit > 1: partials [tile][split][np rows][128 features] fp32
  int *err;
};

// Ring depths for np rows and the dynamic shared memory they take.
void gemm_w8_rings(int np, int w_bf16, int *stages_w, int *stages_x);
int gemm_w8_smem(int np, int w_bf16);
// Sets the kernels' shared-memory attribute; writes to active[ks] how many
// split-K clusters of ks CTAs the device runs at once.
cudaError_t gemm_w8_set_attrs(int *active);
// Launches the kernel of epilogue `epi` (an Epi) over `tiles` feature tiles
// with g.ksplit CTAs each (a cluster along y when > 1) on `stream`.
cudaError_t gemm_w8_launch(int epi, const GemmW8Args &g, int tiles, cudaStream_t stream, bool pdl);

}  // namespace specdec
