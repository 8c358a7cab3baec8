// Element-wise epilogue math shared by the tensor-core GEMM, the CUDA-core
// GEMV and the reference-shaped element-wise kernels. Each function reproduces
// the rounding points of the reference kernel it names.
#pragma once

#include "common.cuh"

namespace w8a8 {

// dequant_int32_to_bf16_kernel, cuda/activation_quant.cu:129-130:
//   bf16(((float)acc * scale_W[col]) * scale_X[row])
__device__ __forceinline__ float dequant_bf(int32_t acc, float sw, float sx) {
  return round_bf(__fmul_rn(__fmul_rn((float)acc, sw), sx));
}

// add_bias_kernel / add_2d_kernel, cuda/add_bias.cu:14, cuda/add_2d.cu:14:
//   bf16(float(a) + float(b))
__device__ __forceinline__ float add_bf(float a, float b) { return round_bf(__fadd_rn(a, b)); }

// tanh-approximation GELU of cuda/gelu.cu:10-15. The expression is written in
// the same order as the reference so nvcc forms the same fused multiply-adds
// (fmad contraction is on by default for both builds); the result is then
// rounded to bf16 by the caller.
__device__ __forceinline__ float gelu_tanh(float val) {
  const float term = 0.79788456f;
  return 0.5f * val * (1.0f + tanhf(term * (val + 0.044715f * val * val * val)));
}

}  // namespace w8a8
