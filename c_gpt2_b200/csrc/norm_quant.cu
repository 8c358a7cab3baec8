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
#include "epilogue.cuh"
#include "kernels.cuh"
#include "rowblock.cuh"
#include "rowops.cuh"
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
  pdl_wait();
  pdl_launch_dependents();
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
  pdl_wait();
  pdl_launch_dependents();
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
  pdl_wait();
  pdl_launch_dependents();
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

__global__ void __launch_bounds__(kRowThreads)
    quant_rows_block_kernel(const uint16_t *__restrict__ X, int64_t ldx, int K,
                            int8_t *__restrict__ Xq, float *__restrict__ sX) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ RowShared sh;
  const int row = blockIdx.x, t = threadIdx.x, nv = K >> 3;
  uint4 x[kMaxVec];
  load_row_vec(X + (int64_t)row * ldx, nv, t, x);
  quant_store(sh, x, nv, t, Xq + (int64_t)row * K, sX + row);
}

// Row absolute maxima of a column block of the rows, for rows whose columns
// are spread over several GPUs (tensor-parallel attention heads, d_ff slices):
// the per-token scale of the whole row comes from the maximum of the parts.
__global__ void __launch_bounds__(kRowThreads)
    row_amax_block_kernel(const uint16_t *__restrict__ X, int64_t ldx, int K,
                          float *__restrict__ amax) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ RowShared sh;
  const int row = blockIdx.x, t = threadIdx.x, nv = K >> 3;
  uint4 x[kMaxVec];
  load_row_vec(X + (int64_t)row * ldx, nv, t, x);
  const float m = block_row_amax(sh, x, nv, t);
  if (t == 0) amax[row] = m;
}

// Per-token quantization of a column block with the scale of the whole row,
// whose absolute maximum is given (the maximum over n_amax partial maxima
// amax[j * amax_stride + row]). Identical to quant_rows on the whole row.
__global__ void __launch_bounds__(kRowThreads)
    quant_rows_amax_block_kernel(const uint16_t *__restrict__ X, int64_t ldx, int K,
                                 const float *__restrict__ amax, int n_amax,
                                 int64_t amax_stride, int8_t *__restrict__ Xq, int64_t ldq,
                                 float *__restrict__ sX) {
  pdl_wait();
  pdl_launch_dependents();
  const int row = blockIdx.x, t = threadIdx.x, nv = K >> 3;
  uint4 x[kMaxVec];
  load_row_vec(X + (int64_t)row * ldx, nv, t, x);
  float m = 0.0f;
  for (int j = 0; j < n_amax; ++j) m = fmaxf(m, __ldcg(amax + j * amax_stride + row));
  quant_store_amax(x, nv, t, m, Xq + (int64_t)row * ldq, sX + row);
}

// MODE 0: rows of X. MODE 1: embedding gather wte[token] + wpe[position]
// (embeddings.cu:18-23), written to H as the residual stream.
template <int MODE>
__global__ void __launch_bounds__(kRowThreads)
    layernorm_block_kernel(const uint16_t *__restrict__ X, int64_t ldx,
                           const uint16_t *__restrict__ wte, const uint16_t *__restrict__ wpe,
                           const int32_t *__restrict__ tokens, int T,
                           const int32_t *__restrict__ pos0, uint16_t *__restrict__ H, int d,
                           const uint16_t *__restrict__ gamma, const uint16_t *__restrict__ beta,
                           float eps, uint16_t *__restrict__ Y, int64_t ldy,
                           int8_t *__restrict__ Xq, float *__restrict__ sX) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ RowShared sh;
  const int row = blockIdx.x, t = threadIdx.x, nv = d >> 3;
  uint4 x[kMaxVec], g[kMaxVec], bt[kMaxVec];
  if (MODE == 0) {
    const uint4 *src = reinterpret_cast<const uint4 *>(X + (int64_t)row * ldx);
#pragma unroll
    for (int k = 0; k < kMaxVec; ++k) {
      const int v = t + kRowThreads * k;
      x[k] = v < nv ? __ldg(src + v) : make_uint4(0, 0, 0, 0);
    }
  } else {
    const int b = row / T, tt = row - (row / T) * T;
    const int p = (pos0 ? pos0[b] : 0) + tt;
    const uint4 *e = reinterpret_cast<const uint4 *>(wte + (int64_t)tokens[row] * d);
    const uint4 *q = reinterpret_cast<const uint4 *>(wpe + (int64_t)p * d);
#pragma unroll
    for (int k = 0; k < kMaxVec; ++k) {
      const int v = t + kRowThreads * k;
      if (v < nv) {
        float fe[8], fq[8];
        unpack8(__ldg(e + v), fe);
        unpack8(__ldg(q + v), fq);
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          w[i] = (uint32_t)f2bf(__fadd_rn(fe[2 * i], fq[2 * i])) |
                 ((uint32_t)f2bf(__fadd_rn(fe[2 * i + 1], fq[2 * i + 1])) << 16);
        x[k] = make_uint4(w[0], w[1], w[2], w[3]);
        if (H) reinterpret_cast<uint4 *>(H + (int64_t)row * d)[v] = x[k];
      } else {
        x[k] = make_uint4(0, 0, 0, 0);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < kMaxVec; ++k) {
    const int v = t + kRowThreads * k;
    if (v < nv) {
      g[k] = __ldg(reinterpret_cast<const uint4 *>(gamma) + v);
      bt[k] = __ldg(reinterpret_cast<const uint4 *>(beta) + v);
    }
  }
  ln_quant_tail(sh, x, g, bt, nv, t, d, eps, Y ? Y + (int64_t)row * ldy : nullptr,
                Xq ? Xq + (int64_t)row * d : nullptr, sX + row);
}

// Residual stream after a GEMM whose reduction was split over GPUs
// (tensor-parallel attn_proj / W2): acc = the sum of n_slots int32 partial rows,
// H = bf16(R + bf16(bf16(acc*sW*sX) + b)) with the rounding points of the
// single-GPU epilogue (activation_quant.cu:129-130, add_bias.cu:14,
// add_2d.cu:14), then optionally LayerNorm and per-token quantization of H.
// Integer sums are exact in any order, so the result equals the single-GPU
// layer bit for bit.
__global__ void __launch_bounds__(kRowThreads) reduce_layernorm_quant_kernel(ReduceArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ RowShared sh;
  const int row = blockIdx.x, t = threadIdx.x, nv = a.d >> 3;
  const float sx = a.sX[row];
  uint4 x[kMaxVec], g[kMaxVec], bt[kMaxVec];
#pragma unroll
  for (int k = 0; k < kMaxVec; ++k) {
    const int v = t + kRowThreads * k;
    x[k] = make_uint4(0, 0, 0, 0);
    if (v < nv) {
      int32_t acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int j = 0; j < a.n_slots; ++j) {
        const int4 *src = reinterpret_cast<const int4 *>(a.acc + j * a.slot_stride +
                                                         (int64_t)row * a.lda) + 2 * v;
        const int4 lo = __ldcg(src), hi = __ldcg(src + 1);
        acc[0] += lo.x; acc[1] += lo.y; acc[2] += lo.z; acc[3] += lo.w;
        acc[4] += hi.x; acc[5] += hi.y; acc[6] += hi.z; acc[7] += hi.w;
      }
      const float4 w0 = __ldg(reinterpret_cast<const float4 *>(a.sW) + 2 * v);
      const float4 w1 = __ldg(reinterpret_cast<const float4 *>(a.sW) + 2 * v + 1);
      const float sw[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      float bf[8], rf[8];
      unpack8(__ldg(reinterpret_cast<const uint4 *>(a.bias) + v), bf);
      unpack8(__ldg(reinterpret_cast<const uint4 *>(a.R + (int64_t)row * a.ldr) + v), rf);
      uint32_t w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float y0 = add_bf(dequant_bf(acc[2 * i], sw[2 * i], sx), bf[2 * i]);
        const float y1 = add_bf(dequant_bf(acc[2 * i + 1], sw[2 * i + 1], sx), bf[2 * i + 1]);
        w[i] = (uint32_t)f2bf(__fadd_rn(rf[2 * i], y0)) |
               ((uint32_t)f2bf(__fadd_rn(rf[2 * i + 1], y1)) << 16);
      }
      x[k] = make_uint4(w[0], w[1], w[2], w[3]);
      reinterpret_cast<uint4 *>(a.H + (int64_t)row * a.ldh)[v] = x[k];
    }
  }
  if (!a.gamma) return;
#pragma unroll
  for (int k = 0; k < kMaxVec; ++k) {
    const int v = t + kRowThreads * k;
    if (v < nv) {
      g[k] = __ldg(reinterpret_cast<const uint4 *>(a.gamma) + v);
      bt[k] = __ldg(reinterpret_cast<const uint4 *>(a.beta) + v);
    }
  }
  ln_quant_tail(sh, x, g, bt, nv, t, a.d, a.eps, nullptr, a.Xq + (int64_t)row * a.ldq,
                a.sXq + row);
}

// ---------------------------------------------------------------------------
// Warp-per-row kernels with the row held in registers (rowops.cuh): no shared
// memory and no block barriers, so thousands of rows stream at HBM speed
// (prefill) and a few rows finish in a short dependency chain (decode).
// ---------------------------------------------------------------------------
// modes of quant_warp_kernel
enum { QW_ROW = 0, QW_AMAX_ONLY = 1, QW_GIVEN_AMAX = 2 };

// Row-maximum outputs of QW_AMAX_ONLY: the same [M] values into n arrays
// (this GPU's and its peers' exchange slots).
struct AmaxOut {
  float *p[8];
  int n;
};

template <int MODE, int NV>
__global__ void __launch_bounds__(kWarpRows * 32)
    quant_warp_kernel(const uint16_t *__restrict__ X, int64_t ldx, int M, int K,
                      const float *__restrict__ amax_in, int n_amax, int64_t amax_stride,
                      int8_t *__restrict__ Xq, int64_t ldq, float *__restrict__ sX,
                      AmaxOut amax_out) {
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * kWarpRows + (threadIdx.x >> 5);
  if (row >= M) return;
  const int nv = K >> 3;
  uint4 x[NV];
  warp_load_row(X + (int64_t)row * ldx, nv, lane, x);
  float amax;
  if (MODE == QW_GIVEN_AMAX) {
    amax = 0.0f;
    for (int j = 0; j < n_amax; ++j) amax = fmaxf(amax, __ldcg(amax_in + j * amax_stride + row));
  } else {
    amax = warp_row_amax(x, nv, lane);
  }
  if (MODE == QW_AMAX_ONLY) {
    if (lane < amax_out.n) amax_out.p[lane][row] = amax;
    return;
  }
  warp_quant_store(x, nv, lane, amax, Xq + (int64_t)row * ldq, sX + row);
}

// Arguments of the warp-per-row LayerNorm (+ quant) kernels.
struct LnWarpArgs {
  int M, d;
  const uint16_t *X;  // LN_ROWS: input rows
  int64_t ldx;
  const uint16_t *wte, *wpe;  // LN_EMBED: token + position embedding gather
  const int32_t *tokens;
  int T;
  const int32_t *pos0;
  ReduceArgs red;  // LN_REDUCE: residual from split-K int32 partial sums
  uint16_t *H;     // residual stream out (LN_EMBED, LN_REDUCE), row stride ldh
  int64_t ldh;
  const uint16_t *gamma, *beta;  // NULL: no LayerNorm (LN_REDUCE only)
  float eps;
  uint16_t *Y;  // LayerNorm output (optional)
  int64_t ldy;
  int8_t *Xq;  // quantized LayerNorm output (optional)
  int64_t ldq;
  float *sX;
};

enum { LN_ROWS = 0, LN_EMBED = 1, LN_REDUCE = 2 };

template <int MODE, int NV>
__global__ void __launch_bounds__(kWarpRows * 32) layernorm_warp_kernel(LnWarpArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * kWarpRows + (threadIdx.x >> 5);
  if (row >= a.M) return;
  const int d = a.d, nv = d >> 3;
  uint4 x[NV];
  if (MODE == LN_ROWS) {
    warp_load_row(a.X + (int64_t)row * a.ldx, nv, lane, x);
  } else if (MODE == LN_EMBED) {
    // embeddings.cu:18-23: bf16(wte[token] + wpe[position])
    const int b = row / a.T, tt = row - (row / a.T) * a.T;
    const int p = (a.pos0 ? a.pos0[b] : 0) + tt;
    const uint4 *e = reinterpret_cast<const uint4 *>(a.wte + (int64_t)a.tokens[row] * d);
    const uint4 *q = reinterpret_cast<const uint4 *>(a.wpe + (int64_t)p * d);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int v = lane + 32 * k;
      x[k] = make_uint4(0, 0, 0, 0);
      if (v < nv) {
        float fe[8], fq[8];
        unpack8(__ldg(e + v), fe);
        unpack8(__ldg(q + v), fq);
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          w[i] = (uint32_t)f2bf(__fadd_rn(fe[2 * i], fq[2 * i])) |
                 ((uint32_t)f2bf(__fadd_rn(fe[2 * i + 1], fq[2 * i + 1])) << 16);
        x[k] = make_uint4(w[0], w[1], w[2], w[3]);
        if (a.H) reinterpret_cast<uint4 *>(a.H + (int64_t)row * a.ldh)[v] = x[k];
      }
    }
  } else {
    // H = bf16(R + bf16(bf16(acc*sW*sX) + b)), acc = sum of the int32 partials
    const ReduceArgs &r = a.red;
    const float sx = r.sX[row];
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int v = lane + 32 * k;
      x[k] = make_uint4(0, 0, 0, 0);
      if (v < nv) {
        int32_t acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int j = 0; j < r.n_slots; ++j) {
          const int4 *src = reinterpret_cast<const int4 *>(r.acc + j * r.slot_stride +
                                                           (int64_t)row * r.lda) + 2 * v;
          const int4 lo = __ldcg(src), hi = __ldcg(src + 1);
          acc[0] += lo.x; acc[1] += lo.y; acc[2] += lo.z; acc[3] += lo.w;
          acc[4] += hi.x; acc[5] += hi.y; acc[6] += hi.z; acc[7] += hi.w;
        }
        const float4 w0 = __ldg(reinterpret_cast<const float4 *>(r.sW) + 2 * v);
        const float4 w1 = __ldg(reinterpret_cast<const float4 *>(r.sW) + 2 * v + 1);
        const float sw[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        float bf[8], rf[8];
        unpack8(__ldg(reinterpret_cast<const uint4 *>(r.bias) + v), bf);
        unpack8(__ldg(reinterpret_cast<const uint4 *>(r.R + (int64_t)row * r.ldr) + v), rf);
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float y0 = add_bf(dequant_bf(acc[2 * i], sw[2 * i], sx), bf[2 * i]);
          const float y1 = add_bf(dequant_bf(acc[2 * i + 1], sw[2 * i + 1], sx), bf[2 * i + 1]);
          w[i] = (uint32_t)f2bf(__fadd_rn(rf[2 * i], y0)) |
                 ((uint32_t)f2bf(__fadd_rn(rf[2 * i + 1], y1)) << 16);
        }
        x[k] = make_uint4(w[0], w[1], w[2], w[3]);
        reinterpret_cast<uint4 *>(a.H + (int64_t)row * a.ldh)[v] = x[k];
      }
    }
    if (!a.gamma) return;
  }
  uint4 y[NV];
  warp_layernorm_row(x, nv, lane, d, a.gamma, a.beta, a.eps, y,
                     a.Y ? a.Y + (int64_t)row * a.ldy : nullptr);
  if (a.Xq) {
    uint2 q[NV];
    const float scale = warp_quant_pack(y, nv, lane, warp_row_amax(y, nv, lane), q);
    warp_quant_put(q, scale, nv, lane, a.Xq + (int64_t)row * a.ldq, a.sX + row);
    if (MODE == LN_REDUCE) {  // copies into the peers' all-gather buffers
      const int64_t r = a.red.bcast_row0 + row;
      for (int j = 0; j < a.red.n_bcast; ++j)
        warp_quant_put(q, scale, nv, lane, a.red.xq_bcast[j] + r * a.ldq, a.red.sx_bcast[j] + r);
    }
  }
}

static int warp_grid(int M) { return (M + kWarpRows - 1) / kWarpRows; }

// Below this many rows the block-per-row kernels finish sooner: a decode step
// has too few rows for one warp per row to spread over the SMs.
constexpr int kWarpMinRows = 1024;

static bool warp_rows_ok(int n, int max_vec, const void *p, int64_t ld) {
  return (n & 7) == 0 && n <= 256 * max_vec && aligned16(p) && (ld & 7) == 0;
}

static bool block_path_ok(int d, const void *a, int64_t lda, const void *b, int64_t ldb) {
  return (d & 7) == 0 && d <= 1024 * kMaxVec && aligned16(a) && (lda & 7) == 0 &&
         (b == nullptr || (aligned16(b) && (ldb & 7) == 0));
}

static int row_grid(int M) { return (M + kRowWarps - 1) / kRowWarps; }

template <int MODE>
static int launch_quant_warp(const uint16_t *X, int64_t ldx, int M, int K, const float *amax_in,
                             int n_amax, int64_t amax_stride, int8_t *Xq, int64_t ldq, float *sX,
                             AmaxOut amax_out, cudaStream_t s) {
  const int need = ((K >> 3) + 31) / 32;
  const dim3 g(warp_grid(M)), b(kWarpRows * 32);
  // the fewest 16-byte vectors a lane needs (fewer registers, more rows in
  // flight): 32768 rows of 5120 99.9 -> 87.7 us with 20 instead of 24, of
  // 1280 32.8 -> 31.2 us with 5 instead of 8
  if (need <= 5)
    launch_pdl(quant_warp_kernel<MODE, 5>, g, b, 0, s, X, ldx, M, K, amax_in, n_amax, amax_stride,
               Xq, ldq, sX, amax_out);
  else if (need <= 8)
    launch_pdl(quant_warp_kernel<MODE, 8>, g, b, 0, s, X, ldx, M, K, amax_in, n_amax, amax_stride,
               Xq, ldq, sX, amax_out);
  else if (need <= 16)
    launch_pdl(quant_warp_kernel<MODE, 16>, g, b, 0, s, X, ldx, M, K, amax_in, n_amax,
               amax_stride, Xq, ldq, sX, amax_out);
  else if (need <= 20)
    launch_pdl(quant_warp_kernel<MODE, 20>, g, b, 0, s, X, ldx, M, K, amax_in, n_amax,
               amax_stride, Xq, ldq, sX, amax_out);
  else
    launch_pdl(quant_warp_kernel<MODE, 24>, g, b, 0, s, X, ldx, M, K, amax_in, n_amax,
               amax_stride, Xq, ldq, sX, amax_out);
  return check_launch("quant_warp");
}

template <int MODE>
static int launch_ln_warp(const LnWarpArgs &a, cudaStream_t s) {
  const dim3 g(warp_grid(a.M)), b(kWarpRows * 32);
  // the fewest 16-byte vectors a lane needs: 5 for GPT-2 large's 1280 (71
  // instead of 80 registers; 32768 rows 65.5 -> 59.2 us)
  if (a.d <= 256 * 4)
    launch_pdl(layernorm_warp_kernel<MODE, 4>, g, b, 0, s, a);
  else if (a.d <= 256 * 5)
    launch_pdl(layernorm_warp_kernel<MODE, 5>, g, b, 0, s, a);
  else
    launch_pdl(layernorm_warp_kernel<MODE, 8>, g, b, 0, s, a);
  return check_launch("layernorm_warp");
}

static bool ln_warp_ok(const LnWarpArgs &a) {
  return (a.d & 7) == 0 && a.d <= 256 * kWarpVec && aligned16(a.gamma) && aligned16(a.beta) &&
         (a.Y == nullptr || (aligned16(a.Y) && (a.ldy & 7) == 0)) &&
         (a.Xq == nullptr || (aligned16(a.Xq) && (a.ldq & 7) == 0)) &&
         (a.H == nullptr || (aligned16(a.H) && (a.ldh & 7) == 0));
}

int launch_quant_rows(const uint16_t *X, int64_t ldx, int M, int K, int8_t *Xq, float *sX,
                      cudaStream_t s) {
  if (M >= kWarpMinRows && warp_rows_ok(K, kWarpQuantVec, X, ldx) && aligned16(Xq))
    return launch_quant_warp<QW_ROW>(X, ldx, M, K, nullptr, 0, 0, Xq, K, sX, AmaxOut{}, s);
  if (block_path_ok(K, X, ldx, Xq, K) && M <= 0x7fffffff) {
    launch_pdl(quant_rows_block_kernel, dim3(M), dim3(kRowThreads), 0, s, X, ldx, K, Xq, sX);
    return check_launch("quant_rows_block");
  }
  size_t smem = (size_t)kRowWarps * K * sizeof(uint16_t);
  if (smem > 200 * 1024) return W8A8_ERR_UNSUPPORTED;
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    cudaFuncSetAttribute(quant_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    attr[dev & 63] = true;
  }
  launch_pdl(quant_rows_kernel, dim3(row_grid(M)), dim3(kRowWarps * 32), smem, s, X, ldx, M, K, Xq, sX);
  return check_launch("quant_rows");
}

int launch_layernorm_quant(const uint16_t *X, int64_t ldx, int M, int d, const uint16_t *gamma,
                           const uint16_t *beta, float eps, uint16_t *Y, int64_t ldy, int8_t *Xq,
                           float *sX, cudaStream_t s) {
  {
    LnWarpArgs a = {};
    a.M = M;
    a.d = d;
    a.X = X;
    a.ldx = ldx;
    a.gamma = gamma;
    a.beta = beta;
    a.eps = eps;
    a.Y = Y;
    a.ldy = ldy;
    a.Xq = Xq;
    a.ldq = d;
    a.sX = sX;
    if (M >= kWarpMinRows && ln_warp_ok(a) && aligned16(X) && (ldx & 7) == 0)
      return launch_ln_warp<LN_ROWS>(a, s);
  }
  if (block_path_ok(d, X, ldx, Y, Y ? ldy : 0) && aligned16(gamma) && aligned16(beta) &&
      (Xq == nullptr || aligned16(Xq))) {
    launch_pdl(layernorm_block_kernel<0>, dim3(M), dim3(kRowThreads), 0, s, X, ldx, nullptr, nullptr, nullptr, 1,
                                                        nullptr, nullptr, d, gamma, beta, eps, Y,
                                                        ldy, Xq, sX);
    return check_launch("layernorm_block");
  }
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
  launch_pdl(layernorm_quant_kernel, dim3(row_grid(M)), dim3(kRowWarps * 32), smem, s, X, ldx, M, d, gamma, beta,
                                                                     eps, Y, ldy, Xq, sX);
  return check_launch("layernorm_quant");
}

int launch_embed_layernorm_quant(const uint16_t *wte, const uint16_t *wpe, const int32_t *tokens,
                                 int M, int T, const int32_t *pos0, int d, uint16_t *H,
                                 const uint16_t *gamma, const uint16_t *beta, float eps,
                                 uint16_t *Y, int8_t *Xq, float *sX, cudaStream_t s) {
  {
    LnWarpArgs a = {};
    a.M = M;
    a.d = d;
    a.wte = wte;
    a.wpe = wpe;
    a.tokens = tokens;
    a.T = T;
    a.pos0 = pos0;
    a.H = H;
    a.ldh = d;
    a.gamma = gamma;
    a.beta = beta;
    a.eps = eps;
    a.Y = Y;
    a.ldy = d;
    a.Xq = Xq;
    a.ldq = d;
    a.sX = sX;
    if (M >= kWarpMinRows && ln_warp_ok(a) && aligned16(wte) && aligned16(wpe))
      return launch_ln_warp<LN_EMBED>(a, s);
  }
  if (block_path_ok(d, wte, d, wpe, d) && aligned16(gamma) && aligned16(beta) &&
      (H == nullptr || aligned16(H)) && (Y == nullptr || aligned16(Y)) &&
      (Xq == nullptr || aligned16(Xq))) {
    launch_pdl(layernorm_block_kernel<1>, dim3(M), dim3(kRowThreads), 0, s, nullptr, 0, wte, wpe, tokens, T, pos0, H,
                                                        d, gamma, beta, eps, Y, d, Xq, sX);
    return check_launch("embed_layernorm_block");
  }
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
  launch_pdl(embed_layernorm_quant_kernel, dim3(row_grid(M)), dim3(kRowWarps * 32), smem, s, 
      wte, wpe, tokens, M, T, pos0, d, H, gamma, beta, eps, Y, Xq, sX);
  return check_launch("embed_layernorm_quant");
}

int launch_row_amax(const uint16_t *X, int64_t ldx, int M, int K, float *const *amax, int n_out,
                    cudaStream_t s) {
  if (n_out < 1 || n_out > 8) return W8A8_ERR_INVALID;
  // several outputs (peer exchange slots) always take the warp kernel
  if ((M >= kWarpMinRows || n_out > 1) && warp_rows_ok(K, kWarpQuantVec, X, ldx)) {
    AmaxOut o = {};
    for (int j = 0; j < n_out; ++j) o.p[j] = amax[j];
    o.n = n_out;
    return launch_quant_warp<QW_AMAX_ONLY>(X, ldx, M, K, nullptr, 0, 0, nullptr, 0, nullptr, o, s);
  }
  if (n_out > 1 || !block_path_ok(K, X, ldx, nullptr, 0)) return W8A8_ERR_UNSUPPORTED;
  launch_pdl(row_amax_block_kernel, dim3(M), dim3(kRowThreads), 0, s, X, ldx, K, amax[0]);
  return check_launch("row_amax_block");
}

int launch_quant_rows_amax(const uint16_t *X, int64_t ldx, int M, int K, const float *amax,
                           int n_amax, int64_t amax_stride, int8_t *Xq, int64_t ldq, float *sX,
                           cudaStream_t s) {
  if (M >= kWarpMinRows && warp_rows_ok(K, kWarpQuantVec, X, ldx) && aligned16(Xq) &&
      (ldq & 7) == 0)
    return launch_quant_warp<QW_GIVEN_AMAX>(X, ldx, M, K, amax, n_amax, amax_stride, Xq, ldq, sX,
                                            AmaxOut{}, s);
  if (!block_path_ok(K, X, ldx, Xq, ldq)) return W8A8_ERR_UNSUPPORTED;
  launch_pdl(quant_rows_amax_block_kernel, dim3(M), dim3(kRowThreads), 0, s, X, ldx, K, amax,
             n_amax, amax_stride, Xq, ldq, sX);
  return check_launch("quant_rows_amax_block");
}

int launch_reduce_layernorm_quant(const ReduceArgs &a, int M, cudaStream_t s) {
  const int d = a.d;
  bool ok = (d & 7) == 0 && d <= 1024 * kMaxVec && aligned16(a.acc) && (a.lda & 3) == 0 &&
            (a.slot_stride & 3) == 0 && aligned16(a.sW) && aligned16(a.bias) &&
            aligned16(a.R) && (a.ldr & 7) == 0 && aligned16(a.H) && (a.ldh & 7) == 0;
  if (a.gamma)
    ok = ok && aligned16(a.gamma) && aligned16(a.beta) && aligned16(a.Xq) && (a.ldq & 7) == 0;
  if (a.n_bcast < 0 || a.n_bcast > 8 || (a.n_bcast > 0 && !a.gamma)) return W8A8_ERR_INVALID;
  for (int j = 0; j < a.n_bcast; ++j)
    if (!aligned16(a.xq_bcast[j]) || !a.sx_bcast[j]) return W8A8_ERR_INVALID;
  if (!ok) return W8A8_ERR_UNSUPPORTED;
  if ((M >= kWarpMinRows || a.n_bcast > 0) && d <= 256 * kWarpVec) {
    LnWarpArgs w = {};
    w.M = M;
    w.d = d;
    w.red = a;
    w.H = a.H;
    w.ldh = a.ldh;
    w.gamma = a.gamma;
    w.beta = a.beta;
    w.eps = a.eps;
    w.Xq = a.Xq;
    w.ldq = a.ldq;
    w.sX = a.sXq;
    return launch_ln_warp<LN_REDUCE>(w, s);
  }
  if (a.n_bcast > 0) return W8A8_ERR_UNSUPPORTED;
  launch_pdl(reduce_layernorm_quant_kernel, dim3(M), dim3(kRowThreads), 0, s, a);
  return check_launch("reduce_layernorm_quant");
}

}  // namespace w8a8
