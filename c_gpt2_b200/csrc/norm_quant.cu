// Per-token INT8 activation quantization, LayerNorm, and their fusions
// (LayerNorm -> quant, embedding -> LayerNorm -> quant). One warp per token
// row, 128-bit loads, the row kept on chip between the statistics, the
// normalisation and the quantization, so each row is read from HBM once.
//
// Semantics follow the reference kernels operation for operation:
//   quantization  cuda/activation_quant.cu:54-91
//   LayerNorm     cuda/layernorm.cu:23-77 (two-pass fp32 statistics whose
//                 partial sums are combined in the same 1024-slot binary tree
//                 the reference's 1024-thread block uses, then rsqrtf)
//   embedding     cuda/embeddings.cu:18-23
#include "common.cuh"
#include "runtime.cuh"

namespace w8a8 {

constexpr int kRowWarps = 8;  // rows (warps) per block

// ---------------------------------------------------------------------------
// quantization of one row held in shared memory (bf16 values)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void quantize_row_smem(const uint16_t *row, int K, int8_t *xq_row,
                                                  float *sx_out, int lane) {
  float amax = 0.0f;
  if ((K & 7) == 0) {
    for (int j = lane * 8; j < K; j += 256) {
      const uint4 v = *reinterpret_cast<const uint4 *>(row + j);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        amax = fmaxf(amax, fabsf(__uint_as_float(w[e] << 16)));
        amax = fmaxf(amax, fabsf(__uint_as_float(w[e] & 0xffff0000u)));
      }
    }
  } else {
    for (int j = lane; j < K; j += 32) amax = fmaxf(amax, fabsf(bf2f(row[j])));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  // scale = amax/127 (1.0 for an all-zero row); q = rn(x * (1/scale)), ±127.
  const float scale = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
  const float inv = __fdiv_rn(1.0f, scale);
  if (lane == 0) *sx_out = scale;
  if ((K & 7) == 0 && aligned16(xq_row)) {
    for (int j = lane * 8; j < K; j += 256) {
      uint32_t w[2] = {0u, 0u};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        int q = __float2int_rn(__fmul_rn(bf2f(row[j + e]), inv));
        q = q > 127 ? 127 : (q < -127 ? -127 : q);
        w[e >> 2] |= ((uint32_t)(q & 0xff)) << (8 * (e & 3));
      }
      *reinterpret_cast<uint2 *>(xq_row + j) = make_uint2(w[0], w[1]);
    }
  } else {
    for (int j = lane; j < K; j += 32) {
      int q = __float2int_rn(__fmul_rn(bf2f(row[j]), inv));
      q = q > 127 ? 127 : (q < -127 ? -127 : q);
      xq_row[j] = (int8_t)q;
    }
  }
}

// Copy `n` bf16 from global to shared (vectorised when both allow it).
__device__ __forceinline__ void load_row(uint16_t *dst, const uint16_t *src, int n, int lane) {
  if ((n & 7) == 0 && aligned16(src)) {
    for (int j = lane * 8; j < n; j += 256)
      *reinterpret_cast<uint4 *>(dst + j) = __ldg(reinterpret_cast<const uint4 *>(src + j));
  } else {
    for (int j = lane; j < n; j += 32) dst[j] = src[j];
  }
}

__global__ void __launch_bounds__(kRowWarps * 32)
    quant_rows_kernel(const uint16_t *__restrict__ X, int64_t ldx, int M, int K,
                      int8_t *__restrict__ Xq, float *__restrict__ sX) {
  extern __shared__ uint16_t srow_all[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kRowWarps + warp;
  if (row >= M) return;
  uint16_t *srow = srow_all + (size_t)warp * K;
  load_row(srow, X + (int64_t)row * ldx, K, lane);
  __syncwarp();
  quantize_row_smem(srow, K, Xq + (int64_t)row * K, sX + row, lane);
}

// ---------------------------------------------------------------------------
// LayerNorm of one row in shared memory with the reference's reduction tree.
//
// The reference block has 1024 threads; thread t accumulates elements
// t, t+1024, ... in order, then the 1024 partials are folded pairwise
// (s = 512, 256, ..., 1: slot t += slot t+s). Here lane l owns slots
// l + 32*i (i < 32); the first five folds are register adds, the last five
// are the shuffle-down steps of the same tree.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float tree1024(float (&v)[32]) {
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] += v[i + 16];
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] += v[i + 8];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] += v[i + 4];
#pragma unroll
  for (int i = 0; i < 2; ++i) v[i] += v[i + 2];
  float x = v[0] + v[1];
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) x += __shfl_down_sync(0xffffffffu, x, s);
  return __shfl_sync(0xffffffffu, x, 0);
}

__device__ __forceinline__ void layernorm_row_smem(uint16_t *row, int d, const uint16_t *gamma,
                                                   const uint16_t *beta, float eps, int lane) {
  float v[32];
  // phase 1: mean (layernorm.cu:25-41)
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    float sum = 0.0f;
    for (int j = lane + 32 * i; j < d; j += 1024) sum += bf2f(row[j]);
    v[i] = sum;
  }
  const float mean = tree1024(v) / (float)d;
  // phase 2: variance (layernorm.cu:45-66)
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    float diff_sq_sum = 0.0f;
    for (int j = lane + 32 * i; j < d; j += 1024) {
      float diff = bf2f(row[j]) - mean;
      diff_sq_sum += diff * diff;
    }
    v[i] = diff_sq_sum;
  }
  const float variance = tree1024(v) / (float)d;
  const float inv_std_dev = rsqrtf(variance + eps);
  __syncwarp();
  // phase 3: normalise, affine, round to bf16 (layernorm.cu:73-77). 16-byte
  // vectors of γ/β, all loads of a lane issued before the arithmetic.
  if ((d & 7) == 0 && aligned16(gamma) && aligned16(beta)) {
    constexpr int kMaxVec = 8;  // 8 x 256 elements per lane pass
    for (int base = lane * 8; base < d; base += 256 * kMaxVec) {
      uint4 gv[kMaxVec], bv[kMaxVec];
#pragma unroll
      for (int u = 0; u < kMaxVec; ++u) {
        const int j = base + 256 * u;
        if (j < d) {
          gv[u] = __ldg(reinterpret_cast<const uint4 *>(gamma + j));
          bv[u] = __ldg(reinterpret_cast<const uint4 *>(beta + j));
        }
      }
#pragma unroll
      for (int u = 0; u < kMaxVec; ++u) {
        const int j = base + 256 * u;
        if (j < d) {
          const uint16_t *g = reinterpret_cast<const uint16_t *>(&gv[u]);
          const uint16_t *bb = reinterpret_cast<const uint16_t *>(&bv[u]);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            float val = bf2f(row[j + e]);
            float normalized = (val - mean) * inv_std_dev;
            row[j + e] = f2bf(normalized * bf2f(g[e]) + bf2f(bb[e]));
          }
        }
      }
    }
  } else {
    for (int j = lane; j < d; j += 32) {
      float val = bf2f(row[j]);
      float normalized = (val - mean) * inv_std_dev;
      row[j] = f2bf(normalized * bf2f(gamma[j]) + bf2f(beta[j]));
    }
  }
  __syncwarp();
}

__device__ __forceinline__ void store_row(uint16_t *dst, const uint16_t *src, int n, int lane) {
  if ((n & 7) == 0 && aligned16(dst)) {
    for (int j = lane * 8; j < n; j += 256)
      *reinterpret_cast<uint4 *>(dst + j) = *reinterpret_cast<const uint4 *>(src + j);
  } else {
    for (int j = lane; j < n; j += 32) dst[j] = src[j];
  }
}

__global__ void __launch_bounds__(kRowWarps * 32)
    layernorm_quant_kernel(const uint16_t *__restrict__ X, int64_t ldx, int M, int d,
                           const uint16_t *__restrict__ gamma, const uint16_t *__restrict__ beta,
                           float eps, uint16_t *__restrict__ Y, int64_t ldy,
                           int8_t *__restrict__ Xq, float *__restrict__ sX) {
  extern __shared__ uint16_t srow_all[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kRowWarps + warp;
  if (row >= M) return;
  uint16_t *srow = srow_all + (size_t)warp * d;
  load_row(srow, X + (int64_t)row * ldx, d, lane);
  __syncwarp();
  layernorm_row_smem(srow, d, gamma, beta, eps, lane);
  if (Y) store_row(Y + (int64_t)row * ldy, srow, d, lane);
  if (Xq) quantize_row_smem(srow, d, Xq + (int64_t)row * d, sX + row, lane);
}

// Embedding gather + LayerNorm + quantization of the first block's input.
__global__ void __launch_bounds__(kRowWarps * 32)
    embed_layernorm_quant_kernel(const uint16_t *__restrict__ wte,
                                 const uint16_t *__restrict__ wpe,
                                 const int32_t *__restrict__ tokens, int M, int T,
                                 const int32_t *__restrict__ pos0, int d,
                                 uint16_t *__restrict__ H, const uint16_t *__restrict__ gamma,
                                 const uint16_t *__restrict__ beta, float eps,
                                 uint16_t *__restrict__ Y, int8_t *__restrict__ Xq,
                                 float *__restrict__ sX) {
  extern __shared__ uint16_t srow_all[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kRowWarps + warp;
  if (row >= M) return;
  uint16_t *srow = srow_all + (size_t)warp * d;
  const int b = row / T, t = row - (row / T) * T;
  const int p = (pos0 ? pos0[b] : 0) + t;
  const uint16_t *e = wte + (int64_t)tokens[row] * d;
  const uint16_t *q = wpe + (int64_t)p * d;
  for (int j = lane; j < d; j += 32) srow[j] = f2bf(__fadd_rn(bf2f(e[j]), bf2f(q[j])));
  __syncwarp();
  if (H) store_row(H + (int64_t)row * d, srow, d, lane);
  layernorm_row_smem(srow, d, gamma, beta, eps, lane);
  if (Y) store_row(Y + (int64_t)row * d, srow, d, lane);
  if (Xq) quantize_row_smem(srow, d, Xq + (int64_t)row * d, sX + row, lane);
}

static int row_grid(int M) { return (M + kRowWarps - 1) / kRowWarps; }

int launch_quant_rows(const uint16_t *X, int64_t ldx, int M, int K, int8_t *Xq, float *sX,
                      cudaStream_t s) {
  size_t smem = (size_t)kRowWarps * K * sizeof(uint16_t);
  if (smem > 200 * 1024) return W8A8_ERR_UNSUPPORTED;
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    cudaFuncSetAttribute(quant_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    attr[dev & 63] = true;
  }
  quant_rows_kernel<<<row_grid(M), kRowWarps * 32, smem, s>>>(X, ldx, M, K, Xq, sX);
  return check_launch("quant_rows");
}

int launch_layernorm_quant(const uint16_t *X, int64_t ldx, int M, int d, const uint16_t *gamma,
                           const uint16_t *beta, float eps, uint16_t *Y, int64_t ldy, int8_t *Xq,
                           float *sX, cudaStream_t s) {
  size_t smem = (size_t)kRowWarps * d * sizeof(uint16_t);
  if (smem > 200 * 1024) return W8A8_ERR_UNSUPPORTED;
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    cudaFuncSetAttribute(layernorm_quant_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         200 * 1024);
    attr[dev & 63] = true;
  }
  layernorm_quant_kernel<<<row_grid(M), kRowWarps * 32, smem, s>>>(X, ldx, M, d, gamma, beta,
                                                                     eps, Y, ldy, Xq, sX);
  return check_launch("layernorm_quant");
}

int launch_embed_layernorm_quant(const uint16_t *wte, const uint16_t *wpe, const int32_t *tokens,
                                 int M, int T, const int32_t *pos0, int d, uint16_t *H,
                                 const uint16_t *gamma, const uint16_t *beta, float eps,
                                 uint16_t *Y, int8_t *Xq, float *sX, cudaStream_t s) {
  size_t smem = (size_t)kRowWarps * d * sizeof(uint16_t);
  if (smem > 200 * 1024) return W8A8_ERR_UNSUPPORTED;
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    cudaFuncSetAttribute(embed_layernorm_quant_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         200 * 1024);
    attr[dev & 63] = true;
  }
  embed_layernorm_quant_kernel<<<row_grid(M), kRowWarps * 32, smem, s>>>(
      wte, wpe, tokens, M, T, pos0, d, H, gamma, beta, eps, Y, Xq, sX);
  return check_launch("embed_layernorm_quant");
}

}  // namespace w8a8
