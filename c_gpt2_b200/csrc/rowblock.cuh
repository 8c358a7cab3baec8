// Block-per-row operations (128 threads a row) shared by the LayerNorm /
// quantization kernels and the batch-1 GEMV that forms its own LayerNorm:
// the reference's 1024-slot LayerNorm sums and fold, the row absolute
// maximum and the per-token quantization (cuda/layernorm.cu:25-77,
// cuda/activation_quant.cu:75-91). The functions take the row as NV 16-byte
// vectors a thread (vector v = t + 128k); the arithmetic does not depend on NV.
#pragma once

#include "common.cuh"
#include "rowops.cuh"

namespace w8a8 {

// ---------------------------------------------------------------------------
// Block-per-row kernels (128 threads, d % 8 == 0, d <= 8192): the hot path.
// Thread t owns the 16-byte vectors v = t + 128k, i.e. elements
// 8t + e + 1024k, so its eight running sums are exactly the reference's
// slots 8t..8t+7 (thread s of the reference's 1024-thread block adds
// elements s, s+1024, ... in order). The 1024 slots are then folded in
// shared memory level by level (s = 512 .. 1) as the reference does. Few
// instructions per thread and one memory round trip per row.
// ---------------------------------------------------------------------------
constexpr int kRowThreads = 128;
constexpr int kMaxVec = 8;  // 8 x 1024 = 8192 elements per row

struct RowShared {
  float slots[1024];
  float red[kRowThreads / 32];
};

// The reference's 1024-slot fold (h = 512 .. 1: slot i += slot i + h) over
// the 8 slots each of the 128 threads holds (thread t: slots 8t .. 8t+7):
// h = 512 and 256 through shared memory, h = 128 .. 8 as shuffle-downs inside
// warp 0 (slot 8t + e + h sits in thread t + h/8), h = 4, 2, 1 in thread 0's
// registers. The same additions in the same order, with three block
// barriers instead of ten. `s` is consumed.
__device__ __forceinline__ float fold_slots(RowShared &sh, float (&s)[8], int t) {
  static_assert(kRowThreads == 128, "fold_slots: 128 threads x 8 slots");
  if (t >= 64) {
#pragma unroll
    for (int e = 0; e < 8; ++e) sh.slots[8 * (t - 64) + e] = s[e];
  }
  __syncthreads();
  if (t < 64) {
#pragma unroll
    for (int e = 0; e < 8; ++e) s[e] += sh.slots[8 * t + e];  // h = 512
  }
  __syncthreads();
  if (t >= 32 && t < 64) {
#pragma unroll
    for (int e = 0; e < 8; ++e) sh.slots[8 * (t - 32) + e] = s[e];
  }
  __syncthreads();
  if (t < 32) {
#pragma unroll
    for (int e = 0; e < 8; ++e) s[e] += sh.slots[8 * t + e];  // h = 256
#pragma unroll
    for (int h = 16; h >= 1; h >>= 1) {  // h = 128 .. 8
#pragma unroll
      for (int e = 0; e < 8; ++e) s[e] += __shfl_down_sync(0xffffffffu, s[e], h);
    }
    if (t == 0) {
#pragma unroll
      for (int e = 0; e < 4; ++e) s[e] += s[e + 4];  // h = 4
      s[0] += s[2];                                   // h = 2
      s[1] += s[3];
      sh.red[0] = s[0] + s[1];                        // h = 1
    }
  }
  __syncthreads();
  const float v = sh.red[0];
  __syncthreads();
  return v;
}

__device__ __forceinline__ float block_max(RowShared &sh, float v, int t) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((t & 31) == 0) sh.red[t >> 5] = v;
  __syncthreads();
  float m = sh.red[0];
#pragma unroll
  for (int w = 1; w < kRowThreads / 32; ++w) m = fmaxf(m, sh.red[w]);
  __syncthreads();
  return m;
}

// Largest |value| of the row values a thread holds (bf16 bit patterns in
// y[k]), reduced over the block.
template <int NV>
__device__ __forceinline__ float block_row_amax(RowShared &sh, const uint4 (&y)[NV], int nv,
                                                int t) {
  float amax = 0.0f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    if (t + kRowThreads * k < nv) {
      float f[8];
      unpack8(y[k], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(f[e]));
    }
  }
  return block_max(sh, amax, t);
}

// Quantize the row values a thread holds with the scale of the row's absolute
// maximum amax (activation_quant.cu:75-91) and store them.
template <int NV>
__device__ __forceinline__ void quant_store_amax(const uint4 (&y)[NV], int nv, int t,
                                                 float amax, int8_t *xq_row, float *sx_out) {
  const float scale = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
  const float inv = __fdiv_rn(1.0f, scale);
  if (t == 0) *sx_out = scale;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int v = t + kRowThreads * k;
    if (v < nv) {
      float f[8];
      unpack8(y[k], f);
      uint32_t w[2] = {0u, 0u};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        int q = __float2int_rn(__fmul_rn(f[e], inv));
        q = q > 127 ? 127 : (q < -127 ? -127 : q);
        w[e >> 2] |= ((uint32_t)(q & 0xff)) << (8 * (e & 3));
      }
      *reinterpret_cast<uint2 *>(xq_row + 8 * v) = make_uint2(w[0], w[1]);
    }
  }
}

template <int NV>
__device__ __forceinline__ void quant_store(RowShared &sh, const uint4 (&y)[NV], int nv,
                                            int t, int8_t *xq_row, float *sx_out) {
  quant_store_amax(y, nv, t, block_row_amax(sh, y, nv, t), xq_row, sx_out);
}

template <int NV>
__device__ __forceinline__ void load_row_vec(const uint16_t *row, int nv, int t,
                                             uint4 (&x)[NV]) {
  const uint4 *src = reinterpret_cast<const uint4 *>(row);
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int v = t + kRowThreads * k;
    x[k] = v < nv ? __ldg(src + v) : make_uint4(0, 0, 0, 0);
  }
}

// LayerNorm of one row held as bf16 vectors x[k] (thread t owns vectors
// t + 128k), then the optional bf16 output and the per-token quantization.
template <int NV>
__device__ __forceinline__ void ln_quant_tail(RowShared &sh, const uint4 (&x)[NV],
                                              const uint4 (&g)[NV],
                                              const uint4 (&bt)[NV], int nv, int t, int d,
                                              float eps, uint16_t *y_row, int8_t *xq_row,
                                              float *sx_out) {
  // mean: slot 8t+e accumulates elements 8t+e+1024k in order (layernorm.cu:25-41)
  float s[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) s[e] = 0.0f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    if (t + kRowThreads * k < nv) {
      float f[8];
      unpack8(x[k], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) s[e] += f[e];
    }
  }
  const float mean = fold_slots(sh, s, t) / (float)d;
  // variance (layernorm.cu:45-66): diff*diff contracted into the running sum
#pragma unroll
  for (int e = 0; e < 8; ++e) s[e] = 0.0f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    if (t + kRowThreads * k < nv) {
      float f[8];
      unpack8(x[k], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float diff = f[e] - mean;
        s[e] += diff * diff;
      }
    }
  }
  const float variance = fold_slots(sh, s, t) / (float)d;
  const float inv_std_dev = rsqrtf(variance + eps);
  // normalise + affine, bf16 (layernorm.cu:73-77)
  uint4 y[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int v = t + kRowThreads * k;
    if (v < nv) {
      float f[8], gf[8], bf[8];
      unpack8(x[k], f);
      unpack8(g[k], gf);
      unpack8(bt[k], bf);
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
    } else {
      y[k] = make_uint4(0, 0, 0, 0);
    }
  }
  if (xq_row) quant_store(sh, y, nv, t, xq_row, sx_out);
}

}  // namespace w8a8
