// Persistent stream-K tensor-core linear layer for the row batches of a
// speculative round (draft steps, verify blocks: at most 256 rows): arguments
// and host wrappers of gemm_sk.cu.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include "forward.cuh"

namespace specdec {

constexpr int kSkMaxRows = 256;    // two 128-row accumulators share every weight tile
constexpr int kSkMaxTiles = 4096;  // 256-column tiles of one launch (the fix-up grid's x)

struct alignas(64) GemmSkArgs {
  CUtensorMap tma_a;  // [R][K] bf16 input rows, box 64 x 128, 128-byte swizzle
  CUtensorMap tma_b;  // bf16 image of the int8 codes in tile order ([tile][k-block][256][64]), box 64 x 256
  LinearArgs lin;     // epilogue operands (out, scale, bias, resid, rows, qkv), R, N, K
  int mt;             // 128-row tiles (1 or 2)
  int nt;             // 256-column tiles
  int nk;             // 64-wide k-blocks
  int ctas;           // persistent CTAs (the grid): CTA c takes units [c U / ctas, (c + 1) U / ctas), U = nt nk
  float *ws;          // partial tiles: [cta][first | last][256 columns][256 rows] fp32
  int *err;
};

// Dynamic shared memory of the kernel.
int gemm_sk_smem();
// Sets the kernels' shared-memory attribute (once per device).
cudaError_t gemm_sk_set_attrs();
// Launches the kernel of epilogue `epi` (an Epi) with g.ctas CTAs on `stream`
// (a programmatic dependent of the previous launch when `pdl`), then the
// fix-up of its shared tiles (two launches).
cudaError_t gemm_sk_launch(int epi, const GemmSkArgs &g, cudaStream_t stream, bool pdl);

}  // namespace specdec
