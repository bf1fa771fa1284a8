// f32 GEMMs of f32 plans on the tcgen05 tensor cores by the 3xTF32 split (gemm_tf32.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "runtime.h"

namespace kh {

// Whether the 3xTF32 path takes C[M, N] = A[M, K] W[N, K]^T: rows of 16-byte multiples (K % 4)
// and at least one 16-column MMA of outputs (N >= 16; narrower heads stay on the CUDA cores).
bool gemm_tf32_supported(int N, int K);

// The split x = hi + lo of an f32 tensor for the tensor cores: hi keeps the sign, the exponent and
// the 10 leading mantissa bits (exactly a TF32 value), lo = x - hi (exact in f32). Derived once
// per weight (the activations are split inside the GEMM).
void launch_tf32_split(const float* x, float* hi, float* lo, int64_t n, cudaStream_t st);
// The split of weight `name` [N, K] (f32): hi in the first N K floats of ptr, lo in the next.
const DevTensor& gemm_tf32_weight(Ctx* ctx, const std::string& name);

// C = act(A W^T + bias), f32: A = A_hi + A_lo, W = W_hi + W_lo, and the product as
// A_hi W_hi + A_hi W_lo + A_lo W_hi with f32 accumulation in TMEM (the A_lo W_lo term is below
// f32 precision). A [M, K] is split inside the kernel, stage by stage; W_hi / W_lo are the
// weight's split. act: 0 none, 1 relu, 2 GELU, 3 tanh, 4 silu, as the CUDA-core kernels.
void launch_gemm_tf32x3(const float* a, const float* w_hi, const float* w_lo, const float* bias, float* C, int M,
                        int N, int K, int act, cudaStream_t st);

// Code of the first pipeline wait of this GEMM that gave up on the current device (0: none), read
// after a sync and cleared.
int tf32_error_code();

}  // namespace kh
