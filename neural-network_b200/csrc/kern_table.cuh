// Kernel tables of the translation units that instantiate the many variants
// of the GEMV and attention kernels (kern_linear.cu, kern_attn.cu), so the
// host engine launches them by pointer (cudaLaunchKernelExC) and each unit
// compiles on its own.
#pragma once

namespace specdec {

// linear_kernel<W, A, EPI, LN, NC>: w8 = int8 weights (else fp32), abf = bf16
// activations (else fp32), epi = Epi, ln = input LayerNorm, nc = 2 or 4.
const void *linear_kernel_fn(int w8, int abf, int epi, int ln, int nc);

// attention_kernel<A, KT, D, QT>: abf = bf16 queries/outputs (else fp32),
// kt = cache element type (0 fp32, 1 bf16, 2 int8), D in {4, 8, 16, 32, 64,
// 128}, qt in {1, 2, 4, 8}; null for other values.
const void *attention_kernel_fn(int abf, int kt, int D, int qt);

}  // namespace specdec
