// Row operations shared by the LayerNorm / quantization kernels and the
// fused tails of the decode GEMMs: one warp holds one row in registers.
//
// Lane l owns the 16-byte vectors v = l + 32k, i.e. elements 8l + e + 256k.
// The reference's LayerNorm block has 1024 threads; slot s (thread s) sums
// elements s, s + 1024, ... in order, then the slots are folded pairwise
// (h = 512 .. 1: slot i += slot i + h) (cuda/layernorm.cu:25-66). Element
// 8l + e + 256k lands in slot 8l + e + 256(k mod 4), so lane l owns slots
// 8l + e + 256m (m < 4): folds h = 512 and 256 are register adds, h = 128 .. 8
// shuffle-down steps between lanes (slot 8l + e + h sits in lane l + h/8),
// h = 4, 2, 1 register adds in lane 0. Every addition is the reference's, in
// the reference's order. Quantization follows cuda/activation_quant.cu:75-91.
#pragma once

#include "common.cuh"

namespace w8a8 {

__device__ __forceinline__ void unpack8(const uint4 &v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

constexpr int kWarpRows = 4;       // rows (warps) per block of the warp-per-row kernels
constexpr int kWarpVec = 8;        // LayerNorm rows up to 8 * 256 = 2048 elements
constexpr int kWarpQuantVec = 24;  // quantized rows up to 6144 elements
// Kernels are instantiated for NV = 4, 5, 8 (LayerNorm) and 5, 8, 16, 20, 24 (quant)
// vectors per lane; a row of n elements uses the smallest NV >= n / 256.

__device__ __forceinline__ float warp_fold1024(float (&s)[4][8]) {
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    s[0][e] += s[2][e];  // h = 512
    s[1][e] += s[3][e];
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) s[0][e] += s[1][e];  // h = 256
#pragma unroll
  for (int h = 16; h >= 1; h >>= 1) {  // h = 128 .. 8 (lane distance h)
#pragma unroll
    for (int e = 0; e < 8; ++e) s[0][e] += __shfl_down_sync(0xffffffffu, s[0][e], h);
  }
#pragma unroll
  for (int e = 0; e < 4; ++e) s[0][e] += s[0][e + 4];  // h = 4
#pragma unroll
  for (int e = 0; e < 2; ++e) s[0][e] += s[0][e + 2];  // h = 2
  const float total = s[0][0] + s[0][1];                // h = 1
  return __shfl_sync(0xffffffffu, total, 0);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Quantize the row values a lane holds (vectors l + 32k, k < NV) with the
// scale of the row's absolute maximum amax (activation_quant.cu:75-91): q[k]
// holds the 8 int8 values of vector k, the return value is the scale.
template <int NV>
__device__ __forceinline__ float warp_quant_pack(const uint4 (&y)[NV], int nv, int lane,
                                                 float amax, uint2 (&q)[NV]) {
  const float scale = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
  const float inv = __fdiv_rn(1.0f, scale);
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    uint32_t w[2] = {0u, 0u};
    if (lane + 32 * k < nv) {
      float f[8];
      unpack8(y[k], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        int qv = __float2int_rn(__fmul_rn(f[e], inv));
        qv = qv > 127 ? 127 : (qv < -127 ? -127 : qv);
        w[e >> 2] |= ((uint32_t)(qv & 0xff)) << (8 * (e & 3));
      }
    }
    q[k] = make_uint2(w[0], w[1]);
  }
  return scale;
}

template <int NV>
__device__ __forceinline__ void warp_quant_put(const uint2 (&q)[NV], float scale, int nv, int lane,
                                               int8_t *xq_row, float *sx_out) {
  if (lane == 0) *sx_out = scale;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int v = lane + 32 * k;
    if (v < nv) *reinterpret_cast<uint2 *>(xq_row + 8 * v) = q[k];
  }
}

template <int NV>
__device__ __forceinline__ void warp_quant_store(const uint4 (&y)[NV], int nv, int lane,
                                                 float amax, int8_t *xq_row, float *sx_out) {
  uint2 q[NV];
  const float scale = warp_quant_pack(y, nv, lane, amax, q);
  warp_quant_put(q, scale, nv, lane, xq_row, sx_out);
}

template <int NV>
__device__ __forceinline__ float warp_row_amax(const uint4 (&y)[NV], int nv, int lane) {
  float amax = 0.0f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    if (lane + 32 * k < nv) {
      float f[8];
      unpack8(y[k], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(f[e]));
    }
  }
  return warp_max(amax);
}

template <int NV>
__device__ __forceinline__ void warp_load_row(const uint16_t *row, int nv, int lane,
                                              uint4 (&x)[NV]) {
  const uint4 *src = reinterpret_cast<const uint4 *>(row);
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int v = lane + 32 * k;
    x[k] = v < nv ? __ldg(src + v) : make_uint4(0, 0, 0, 0);
  }
}

// The same row loaded with L1 bypassed (__ldcg): rows written by other CTAs
// of the running kernel.
template <int NV>
__device__ __forceinline__ void warp_load_row_cg(const uint16_t *row, int nv, int lane,
                                                 uint4 (&x)[NV]) {
  const uint4 *src = reinterpret_cast<const uint4 *>(row);
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int v = lane + 32 * k;
    x[k] = v < nv ? __ldcg(src + v) : make_uint4(0, 0, 0, 0);
  }
}

// LayerNorm of a row of d elements held as x (cuda/layernorm.cu:23-77): fp32
// two-pass statistics over the 1024 slots, rsqrtf, normalise + affine, bf16.
// y receives the bf16 result (zero beyond the row); y_row (optional) too.
template <int NV>
__device__ __forceinline__ void warp_layernorm_row(const uint4 (&x)[NV], int nv, int lane, int d,
                                                   const uint16_t *gamma, const uint16_t *beta,
                                                   float eps, uint4 (&y)[NV], uint16_t *y_row) {
  // mean (layernorm.cu:25-41)
  float s[4][8];
#pragma unroll
  for (int m = 0; m < 4; ++m)
#pragma unroll
    for (int e = 0; e < 8; ++e) s[m][e] = 0.0f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    if (lane + 32 * k < nv) {
      float f[8];
      unpack8(x[k], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) s[k & 3][e] += f[e];
    }
  }
  const float mean = warp_fold1024(s) / (float)d;
  // variance (layernorm.cu:45-66): diff*diff contracted into the running sum
#pragma unroll
  for (int m = 0; m < 4; ++m)
#pragma unroll
    for (int e = 0; e < 8; ++e) s[m][e] = 0.0f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    if (lane + 32 * k < nv) {
      float f[8];
      unpack8(x[k], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float diff = f[e] - mean;
        s[k & 3][e] += diff * diff;
      }
    }
  }
  const float variance = warp_fold1024(s) / (float)d;
  const float inv_std_dev = rsqrtf(variance + eps);
  // normalise + affine, bf16 (layernorm.cu:73-77)
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int v = lane + 32 * k;
    y[k] = make_uint4(0, 0, 0, 0);
    if (v < nv) {
      float f[8], gf[8], bf[8];
      unpack8(x[k], f);
      unpack8(__ldg(reinterpret_cast<const uint4 *>(gamma) + v), gf);
      unpack8(__ldg(reinterpret_cast<const uint4 *>(beta) + v), bf);
      uint32_t w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float n0 = (f[2 * i] - mean) * inv_std_dev;
        float n1 = (f[2 * i + 1] - mean) * inv_std_dev;
        w[i] = (uint32_t)f2bf(n0 * gf[2 * i] + bf[2 * i]) |
               ((uint32_t)f2bf(n1 * gf[2 * i + 1] + bf[2 * i + 1]) << 16);
      }
      y[k] = make_uint4(w[0], w[1], w[2], w[3]);
      if (y_row) reinterpret_cast<uint4 *>(y_row)[v] = y[k];
    }
  }
}

}  // namespace w8a8
