// Reference-shaped element-wise kernels: the operations of the reference's
// cuda/*.cu files with their exact per-element semantics, behind
// runtime-dimension launchers. The drop-in symbols of include/cuda_kernels.h
// call these. The fused path (gemm_tc.cu, norm_quant.cu, attention.cu) does
// not use them; they exist so an unmodified gpt2.c call site keeps working.
#include "common.cuh"
#include "epilogue.cuh"
#include "runtime.cuh"

namespace w8a8 {

// grid-stride over rows x cols, 2-D index -> (row, col)
#define W8A8_GRID_LOOP(i, total) \
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (total); \
       i += (int64_t)gridDim.x * blockDim.x)

static int grid_for(int64_t total) {
  int64_t g = (total + 255) / 256;
  if (g > 148 * 16) g = 148 * 16;
  return g < 1 ? 1 : (int)g;
}

// embeddings.cu:18-23: emb[row][col] = bf16(wte[tok[row]][col] + wpe[row][col])
__global__ void ref_embeddings_kernel(const uint16_t *wte, const uint16_t *wpe, const int *tok,
                                      uint16_t *emb, int d, int start_row, int n_rows) {
  pdl_wait();
  pdl_launch_dependents();
  W8A8_GRID_LOOP(i, (int64_t)n_rows * d) {
    int row = start_row + (int)(i / d), col = (int)(i % d);
    emb[(int64_t)row * d + col] =
        f2bf(__fadd_rn(bf2f(wte[(int64_t)tok[row] * d + col]), bf2f(wpe[(int64_t)row * d + col])));
  }
}

// add_bias.cu:14 (in place)
__global__ void ref_add_bias_kernel(uint16_t *a, const uint16_t *b, int rows, int cols) {
  pdl_wait();
  pdl_launch_dependents();
  W8A8_GRID_LOOP(i, (int64_t)rows * cols) {
    a[i] = f2bf(__fadd_rn(bf2f(a[i]), bf2f(b[i % cols])));
  }
}

// add_2d.cu:14
__global__ void ref_add_2d_kernel(const uint16_t *a, const uint16_t *b, uint16_t *out, int rows,
                                  int cols) {
  pdl_wait();
  pdl_launch_dependents();
  W8A8_GRID_LOOP(i, (int64_t)rows * cols) { out[i] = f2bf(__fadd_rn(bf2f(a[i]), bf2f(b[i]))); }
}

// gelu.cu:12-16 (in place)
__global__ void ref_gelu_kernel(uint16_t *x, int rows, int cols) {
  pdl_wait();
  pdl_launch_dependents();
  W8A8_GRID_LOOP(i, (int64_t)rows * cols) { x[i] = f2bf(gelu_tanh(bf2f(x[i]))); }
}

// activation_quant.cu:124-130
__global__ void ref_dequant_kernel(const int32_t *Y, const float *sW, const float *sX,
                                   uint16_t *out, int M, int N) {
  pdl_wait();
  pdl_launch_dependents();
  W8A8_GRID_LOOP(i, (int64_t)M * N) {
    int row = (int)(i / N), col = (int)(i % N);
    out[i] = f2bf(dequant_bf(Y[i], sW[col], sX[row]));
  }
}

// casual_masking.cu:7-14: for rows i < tokens, columns i < j < tokens := -inf
__global__ void ref_causal_mask_kernel(uint16_t *x, int stride, int tokens) {
  pdl_wait();
  pdl_launch_dependents();
  W8A8_GRID_LOOP(k, (int64_t)tokens * tokens) {
    int i = (int)(k / tokens), j = (int)(k % tokens);
    if (j > i) x[(int64_t)i * stride + j] = 0xFF80u;  // bf16 -inf
  }
}

// concat_heads.cu:14-23: dest[tok][h*hd + c] = src[h][tok][c]
__global__ void ref_concat_heads_kernel(const uint16_t *src, uint16_t *dest, int token_index,
                                        int H, int hd, int ctx) {
  pdl_wait();
  pdl_launch_dependents();
  W8A8_GRID_LOOP(i, (int64_t)H * hd) {
    int h = (int)(i / hd), c = (int)(i % hd);
    dest[(int64_t)token_index * (H * hd) + h * hd + c] =
        src[(int64_t)h * ctx * hd + (int64_t)token_index * hd + c];
  }
}

// softmax.cu:24-92, one 256-thread block per row with the reference's
// strided partials and pairwise fold; the exponent expression keeps the
// reference's form so the same fused multiply-add is formed.
__global__ void __launch_bounds__(256)
    ref_softmax_kernel(const uint16_t *in, uint16_t *out, int rows, int cols, int stride,
                       float temperature, int causal_mask) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float s_data[256];
  const int tid = threadIdx.x, row_idx = blockIdx.x;
  if (row_idx >= rows) return;
  const float inv_temp = 1.0f / temperature;
  const uint16_t *row_ptr = in + (int64_t)row_idx * stride;
  uint16_t *out_ptr = out + (int64_t)row_idx * stride;
  const int last_col = causal_mask ? row_idx : (cols - 1);
  float local_max = -INFINITY;
  for (int j = tid; j < cols; j += 256) {
    if (j > last_col) continue;
    float val = bf2f(row_ptr[j]) * inv_temp;
    if (val > local_max) local_max = val;
  }
  s_data[tid] = local_max;
  __syncthreads();
  for (int s = 128; s > 0; s >>= 1) {
    if (tid < s && s_data[tid + s] > s_data[tid]) s_data[tid] = s_data[tid + s];
    __syncthreads();
  }
  const float row_max = s_data[0];
  __syncthreads();
  float local_sum = 0.0f;
  for (int j = tid; j < cols; j += 256) {
    if (j > last_col) {
      out_ptr[j] = 0;
      continue;
    }
    float e = expf(bf2f(row_ptr[j]) * inv_temp - row_max);
    out_ptr[j] = f2bf(e);
    local_sum += e;
  }
  s_data[tid] = local_sum;
  __syncthreads();
  for (int s = 128; s > 0; s >>= 1) {
    if (tid < s) s_data[tid] += s_data[tid + s];
    __syncthreads();
  }
  const float inv_sum = 1.0f / s_data[0];
  for (int j = tid; j < cols; j += 256) {
    if (j > last_col) continue;
    out_ptr[j] = f2bf(bf2f(out_ptr[j]) * inv_sum);
  }
}

}  // namespace w8a8

using namespace w8a8;

#define W8A8_CHECK_PTR(p) \
  if (!(p)) return W8A8_ERR_INVALID

extern "C" int w8a8_ref_embeddings(const gpt2_bf16_t *wte, const gpt2_bf16_t *wpe,
                                   const int32_t *tokens, gpt2_bf16_t *emb, int d, int start_row,
                                   int n_rows, void *stream) {
  if (n_rows <= 0) return W8A8_OK;
  W8A8_CHECK_PTR(wte);
  W8A8_CHECK_PTR(wpe);
  W8A8_CHECK_PTR(tokens);
  W8A8_CHECK_PTR(emb);
  if (d <= 0 || start_row < 0) return W8A8_ERR_INVALID;
  launch_pdl(ref_embeddings_kernel, dim3(grid_for((int64_t)n_rows * d)), dim3(256), 0, (cudaStream_t)stream, 
      wte, wpe, tokens, emb, d, start_row, n_rows);
  return check_launch("ref_embeddings");
}

extern "C" int w8a8_ref_add_bias(gpt2_bf16_t *a, int rows, int cols, const gpt2_bf16_t *b,
                                 void *stream) {
  if (rows <= 0 || cols <= 0) return W8A8_OK;
  W8A8_CHECK_PTR(a);
  W8A8_CHECK_PTR(b);
  launch_pdl(ref_add_bias_kernel, dim3(grid_for((int64_t)rows * cols)), dim3(256), 0, (cudaStream_t)stream, a, b, rows,
                                                                                       cols);
  return check_launch("ref_add_bias");
}

extern "C" int w8a8_ref_add_2d(const gpt2_bf16_t *a, int rows, int cols, const gpt2_bf16_t *b,
                               gpt2_bf16_t *out, void *stream) {
  if (rows <= 0 || cols <= 0) return W8A8_OK;
  W8A8_CHECK_PTR(a);
  W8A8_CHECK_PTR(b);
  W8A8_CHECK_PTR(out);
  launch_pdl(ref_add_2d_kernel, dim3(grid_for((int64_t)rows * cols)), dim3(256), 0, (cudaStream_t)stream, a, b, out,
                                                                                     rows, cols);
  return check_launch("ref_add_2d");
}

extern "C" int w8a8_ref_gelu(gpt2_bf16_t *x, int cols, int rows, void *stream) {
  if (rows <= 0 || cols <= 0) return W8A8_OK;
  W8A8_CHECK_PTR(x);
  launch_pdl(ref_gelu_kernel, dim3(grid_for((int64_t)rows * cols)), dim3(256), 0, (cudaStream_t)stream, x, rows, cols);
  return check_launch("ref_gelu");
}

extern "C" int w8a8_ref_dequant(const int32_t *Y, const float *sW, const float *sX,
                                gpt2_bf16_t *out, int M, int N, void *stream) {
  if (M <= 0 || N <= 0) return W8A8_OK;
  W8A8_CHECK_PTR(Y);
  W8A8_CHECK_PTR(sW);
  W8A8_CHECK_PTR(sX);
  W8A8_CHECK_PTR(out);
  launch_pdl(ref_dequant_kernel, dim3(grid_for((int64_t)M * N)), dim3(256), 0, (cudaStream_t)stream, Y, sW, sX, out, M,
                                                                                N);
  return check_launch("ref_dequant");
}

extern "C" int w8a8_ref_causal_mask(gpt2_bf16_t *x, int stride, int tokens, void *stream) {
  if (tokens <= 0) return W8A8_OK;
  W8A8_CHECK_PTR(x);
  if (stride < tokens) return W8A8_ERR_INVALID;
  launch_pdl(ref_causal_mask_kernel, dim3(grid_for((int64_t)tokens * tokens)), dim3(256), 0, (cudaStream_t)stream, 
      x, stride, tokens);
  return check_launch("ref_causal_mask");
}

extern "C" int w8a8_ref_concat_heads(const gpt2_bf16_t *src, gpt2_bf16_t *dest, int token_index,
                                     int n_head, int head_dim, int ctx, void *stream) {
  W8A8_CHECK_PTR(src);
  W8A8_CHECK_PTR(dest);
  if (n_head <= 0 || head_dim <= 0 || token_index < 0 || token_index >= ctx)
    return W8A8_ERR_INVALID;
  launch_pdl(ref_concat_heads_kernel, dim3(grid_for((int64_t)n_head * head_dim)), dim3(256), 0, (cudaStream_t)stream, 
      src, dest, token_index, n_head, head_dim, ctx);
  return check_launch("ref_concat_heads");
}

extern "C" int w8a8_ref_softmax(const gpt2_bf16_t *a, int rows, int cols, int stride,
                                gpt2_bf16_t *out, float temperature, int causal_mask,
                                void *stream) {
  if (rows <= 0 || cols <= 0) return W8A8_OK;
  W8A8_CHECK_PTR(a);
  W8A8_CHECK_PTR(out);
  if (stride < cols) return W8A8_ERR_INVALID;
  launch_pdl(ref_softmax_kernel, dim3(rows), dim3(256), 0, (cudaStream_t)stream, a, out, rows, cols, stride,
                                                             temperature, causal_mask);
  return check_launch("ref_softmax");
}
