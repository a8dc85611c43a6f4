// Scalar arithmetic shared by every kernel: BF16 rounding points and the
// activation functions the reference applies (ggml's CUDA op definitions,
// restated from their published formulas).
#pragma once

#include <cuda_bf16.h>

namespace wamb {

__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

__device__ __forceinline__ float bf16_to_f(__nv_bfloat16 x) { return __bfloat162float(x); }

// GELU, tanh approximation: 0.5 x (1 + tanh(sqrt(2/pi) x (1 + 0.044715 x^2))).
// Reference: ggml_gelu / bias_gelu_bf16_kernel
// (patches/llama-b9866-native-bf16.patch:507-514).
__device__ __forceinline__ float gelu_tanh(float x) {
  const float k0 = 0.79788456080286535588f;  // sqrt(2/pi)
  const float k1 = 0.044715f;
  return 0.5f * x * (1.0f + tanhf(k0 * x * (1.0f + k1 * x * x)));
}

// GELU, exact erf form: 0.5 x (1 + erf(x / sqrt(2))). Reference: ggml_gelu_erf
// in the action encoder/decoder (src/models/gwp05/engine/mot.cpp:28).
__device__ __forceinline__ float gelu_erf(float x) {
  return 0.5f * x * (1.0f + erff(x * 0.70710678118654752440f));
}

// SiLU: x / (1 + exp(-x)). Reference: ggml_silu in build_condition (mot.cpp:76).
__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }

}  // namespace wamb
