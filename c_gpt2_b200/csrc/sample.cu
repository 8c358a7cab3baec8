// On-device greedy sampling and per-sequence bookkeeping.
//
// The reference copies 50257 bf16 probabilities to the host every token and
// picks the first index of the largest probability (gpt2.c:2180-2222), where
// the probabilities come from softmax_cuda (cuda/softmax.cu:24-92) at the
// effective temperature 1. This kernel forms the same bf16 probabilities on
// the GPU (same rounding points, same 256-slot sum tree) and returns only the
// token id, so the step needs no 100 KB device-to-host copy.
#include "common.cuh"
#include "runtime.cuh"

namespace w8a8 {

__global__ void __launch_bounds__(256)
    greedy_sample_kernel(const uint16_t *__restrict__ logits, int64_t ldl, int V,
                         int32_t *__restrict__ out, int32_t *__restrict__ append_to,
                         int64_t append_stride, int32_t *__restrict__ append_pos) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float s_red[256];
  __shared__ int s_idx[256];
  const int row = blockIdx.x, tid = threadIdx.x;
  const uint16_t *x = logits + (int64_t)row * ldl;
  // phase 1: row max (temperature 1: x * (1/1) == x exactly)
  float mx = -INFINITY;
  for (int j = tid; j < V; j += 256) mx = fmaxf(mx, bf2f(x[j]));
  s_red[tid] = mx;
  __syncthreads();
  for (int s = 128; s > 0; s >>= 1) {
    if (tid < s) s_red[tid] = fmaxf(s_red[tid], s_red[tid + s]);
    __syncthreads();
  }
  mx = s_red[0];
  __syncthreads();
  // phase 2: sum of exp in the reference's 256-slot tree
  float local_sum = 0.0f;
  for (int j = tid; j < V; j += 256) local_sum += expf(bf2f(x[j]) - mx);
  s_red[tid] = local_sum;
  __syncthreads();
  for (int s = 128; s > 0; s >>= 1) {
    if (tid < s) s_red[tid] += s_red[tid + s];
    __syncthreads();
  }
  const float inv_sum = 1.0f / s_red[0];
  __syncthreads();
  // phase 3: bf16 probabilities, first index of the maximum
  float best = -1.0f;
  int best_j = 0x7fffffff;
  for (int j = tid; j < V; j += 256) {
    float p = bf2f(f2bf(bf2f(f2bf(expf(bf2f(x[j]) - mx))) * inv_sum));
    if (p > best) {  // j increases within a thread: keeps the first index
      best = p;
      best_j = j;
    }
  }
  s_red[tid] = best;
  s_idx[tid] = best_j;
  __syncthreads();
  for (int s = 128; s > 0; s >>= 1) {
    if (tid < s) {
      float o = s_red[tid + s];
      int oj = s_idx[tid + s];
      if (o > s_red[tid] || (o == s_red[tid] && oj < s_idx[tid])) {
        s_red[tid] = o;
        s_idx[tid] = oj;
      }
    }
    __syncthreads();
  }
  if (tid == 0) {
    // A row with no ordered maximum (all NaN) keeps index 0, as a host argmax
    // that starts from the first entry does; never an id outside the vocabulary.
    const int tok = s_idx[0] < V ? s_idx[0] : 0;
    out[row] = tok;
    if (append_to) {
      const int p = append_pos[row];
      append_to[(int64_t)row * append_stride + p] = tok;
      append_pos[row] = p + 1;
    }
  }
}

__global__ void advance_kernel(int32_t *dst, const int32_t *src, int n, int delta) {
  pdl_wait();
  pdl_launch_dependents();
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = src[i] + delta;
}

int launch_greedy_sample(const uint16_t *logits, int64_t ldl, int M, int V, int32_t *out,
                         int32_t *append_to, int64_t append_stride, int32_t *append_pos,
                         cudaStream_t s) {
  launch_pdl(greedy_sample_kernel, dim3(M), dim3(256), 0, s, logits, ldl, V, out, append_to, append_stride,
                                         append_pos);
  return check_launch("greedy_sample");
}

int launch_advance(int32_t *dst, const int32_t *src, int n, int delta, cudaStream_t s) {
  launch_pdl(advance_kernel, dim3((n + 255) / 256), dim3(256), 0, s, dst, src, n, delta);
  return check_launch("advance");
}

}  // namespace w8a8
