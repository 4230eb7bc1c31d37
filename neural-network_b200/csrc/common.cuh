// Shared device helpers for the sm_100a speculative-decoding kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace specdec {

constexpr int kWarp = 32;

// Error flags raised by kernels (bitwise OR into a device word, read by the
// host after a generate call).
enum : int {
  kErrSeqLen = 1,     // a cache position reached its capacity
  kErrRngTable = 2,   // the host uniform table ran out of rounds
  kErrTimeout = 4,    // a bounded wait on an asynchronous copy gave up
};

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// Programmatic dependent launch (griddepcontrol, sm_90+).  A kernel launched
// with programmatic stream serialization may start before its predecessor
// has finished: it calls pdl_launch() to let its own successor start early,
// does only work that reads no predecessor's output (weights), and calls
// pdl_wait() -- which returns once the predecessor grid has completed and
// its memory is visible -- before anything else and before any early exit.
// Both are no-ops for kernels launched without the attribute.
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide reductions for blocks of up to 1024 threads.  `red` must hold 32
// entries; every thread gets the result.
__device__ __forceinline__ float block_sum(float v, float *red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = (lane < nw) ? red[lane] : 0.f;
  return warp_sum(t);
}
__device__ __forceinline__ float block_max(float v, float *red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = (lane < nw) ? red[lane] : -INFINITY;
  return warp_max(t);
}

// Argmax with the reference's tie rule: the FIRST index holding the maximum
// (strict `>` scan, src/nn/layer.cpp:1413-1420).
struct ArgMax {
  float v;
  int i;
};
__device__ __forceinline__ ArgMax argmax_merge(ArgMax a, ArgMax b) {
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}
__device__ __forceinline__ ArgMax warp_argmax(ArgMax a) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ArgMax b;
    b.v = __shfl_xor_sync(0xffffffffu, a.v, o);
    b.i = __shfl_xor_sync(0xffffffffu, a.i, o);
    a = argmax_merge(a, b);
  }
  return a;
}
__device__ __forceinline__ ArgMax block_argmax(ArgMax a, float *redv, int *redi) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  a = warp_argmax(a);
  __syncthreads();
  if (lane == 0) { redv[wid] = a.v; redi[wid] = a.i; }
  __syncthreads();
  ArgMax t{-INFINITY, 0x7fffffff};
  if (lane < nw) { t.v = redv[lane]; t.i = redi[lane]; }
  return warp_argmax(t);
}

// Exclusive block scan of one double per thread; returns the exclusive prefix
// and writes the block total to *total.
__device__ __forceinline__ double block_exscan_d(double v, double *red, double *total) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  double inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    double n = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += n;
  }
  __syncthreads();
  if (lane == 31) red[wid] = inc;
  __syncthreads();
  if (wid == 0) {
    double w = (lane < nw) ? red[lane] : 0.0;
    double wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      double n = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += n;
    }
    if (lane < nw) red[lane] = wi - w;  // exclusive warp offsets
    if (lane == nw - 1) red[32] = wi;
  }
  __syncthreads();
  double ex = red[wid] + (inc - v);
  *total = red[32];
  return ex;
}

}  // namespace specdec
