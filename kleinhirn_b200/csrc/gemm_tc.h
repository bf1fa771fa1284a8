// GEMM dispatch: the tcgen05 tensor-core GEMM for f16 plans (gemm_tc.cu) with the epilogues
// the plan's following ops fold into, the CUDA-core GEMM for f32 plans and odd shapes.
#pragma once

#include <string>

#include "runtime.h"

namespace kh {

// What the epilogue of C = act(A W^T + bias) also does (values are rounded to the storage type
// where the reference stores an intermediate, so the fused result equals the unfused ops):
// - Residual: C is the residual stream, C = round(C + round(act(acc + bias)))   (add.wgsl)
// - GeGLU:    W rows interleaved per 32-column block; C[r, j] = round(gelu(round(a)) * round(b))
//             with a, b the two halves of the projection (geglu.wgsl)
// - Rope:     rotate-half RoPE on the q and k column blocks of the qkv output, table row = the
//             local position of the row (rope.wgsl)
struct GemmEpilogue {
  enum Kind { None, Residual, GeGLU, Rope } kind = None;
  int H = 0, D = 0;
  std::string table_id;
  const float* table = nullptr;
  const int32_t* row_pos = nullptr;
};

bool gemm_tc_supported(int N, int K);
bool gemm_tc_supported_geglu(int N, int K);
bool gemm_tc_supported_rope(int D);
// Interleaved copies of a GeGLU input projection [2I, K] and its bias for the fused epilogue.
DevTensor gemm_geglu_weight(Ctx* ctx, const std::string& name, int N, int K);
DevTensor gemm_geglu_bias(Ctx* ctx, const std::string& name, int N);

void launch_gemm(Ctx* ctx, bool f16, const void* A, const void* W, const void* bias, void* C, int M, int N, int K,
                 int act, const GemmEpilogue& e, cudaStream_t st);

// O = LayerNorm(R + round(A W^T + bias)) * ln_w + ln_b (a matmul followed by a mode-2 layernorm
// over its output, f16), for N in {256, 384}. ln_b may be null.
bool gemm_tc_supported_addln(int N, int K);
void launch_gemm_addln(const void* A, const void* W, const void* bias, const void* R, const void* ln_w,
                       const void* ln_b, float eps, void* O, int M, int N, int K, cudaStream_t st);

}  // namespace kh

namespace kh {
// Code of the first tensor-core pipeline wait of the GEMM kernels that gave up on the current
// device (0: none), read after a sync and cleared, so the next call starts clean.
int tc_error_code();
}  // namespace kh
