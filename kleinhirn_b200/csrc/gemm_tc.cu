// GEMM dispatch (first version: CUDA-core GEMM for every plan; the tcgen05 path follows).
#include "gemm_tc.h"

namespace kh {

bool gemm_tc_supported(int, int) { return false; }
bool gemm_tc_supported_geglu(int, int) { return false; }
bool gemm_tc_supported_rope(int) { return false; }
DevTensor gemm_geglu_weight(Ctx*, const std::string&, int, int) { throw PlanError("geglu fusion unavailable"); }
DevTensor gemm_geglu_bias(Ctx*, const std::string&, int) { throw PlanError("geglu fusion unavailable"); }

void launch_gemm(Ctx*, bool f16, const void* A, const void* W, const void* bias, void* C, int M, int N, int K, int act,
                 const GemmEpilogue& e, cudaStream_t st) {
  if (e.kind != GemmEpilogue::None) throw PlanError("gemm epilogue without the tensor-core path");
  launch_gemm_simt(f16, A, W, bias, C, M, N, K, act, st);
}

}  // namespace kh
