// Activations of f32 plans (the matmul ACT codes of src/plan/layers.ts:36-49), shared by the
// CUDA-core kernels and the 3xTF32 tensor-core GEMM so both apply the same arithmetic.
#pragma once

#include <cuda_runtime.h>

namespace kh {
namespace f32act {

// GELU with the Abramowitz-Stegun 7.1.26 erf (src/kernels/mmtile.wgsl:22-31, the constants the
// reference prints); exp through CUDA's expf.
__device__ __forceinline__ float gelu_as(float v) {
  const float u = v * 0.7071067811865476f;
  const float t = 1.0f / (1.0f + 0.3275911f * fabsf(u));
  const float p = (((((1.061405429f * t - 1.453152027f) * t) + 1.421413741f) * t - 0.284496736f) * t +
                   0.254829592f) * t;
  const float e = 1.0f - p * expf(-u * u);
  return 0.5f * v * (1.0f + (v >= 0.0f ? e : -e));
}

// 0 none, 1 relu, 2 GELU, 3 tanh, 4 silu
__device__ __forceinline__ float activate(float v, int act) {
  if (act == 1) return fmaxf(v, 0.0f);
  if (act == 2) return gelu_as(v);
  if (act == 3) return tanhf(v);
  if (act == 4) return v / (1.0f + expf(-v));
  return v;
}

}  // namespace f32act
}  // namespace kh
