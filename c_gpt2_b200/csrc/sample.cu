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

// The same sampling with one row spread over a cluster of kSampleCluster CTAs
// (a decode step's rows are few: at 1-64 rows one CTA per row leaves most
// SMs idle while each thread evaluates ~200 expf twice). CTA r of the
// cluster owns entries [r*C, (r+1)*C) of the row, C = ceil(V / kSampleCluster):
//   1. the row max: each CTA's max, then every CTA the maximum of all eight
//      (order-independent);
//   2. e_j = expf(x_j - max) for its entries, kept in its shared memory;
//   3. the sum in the reference's order: slot t (0..255) adds e_j for
//      j = t, t + 256, ... in order, reading each e_j from the CTA that holds
//      it (warp 0 of CTA r runs slots 32r .. 32r+31); the 256 slot sums are
//      stored in CTA 0, and every CTA folds them with the same tree
//      (s = 128 .. 1), so every CTA holds the same sum;
//   4. bf16 probabilities of its entries and the first index of their
//      maximum; CTA 0 picks the first index of the largest over the eight.
constexpr int kSampleCluster = 8;
constexpr int kSampleThreads = 256;

__global__ void __launch_bounds__(kSampleThreads)
    greedy_sample_cluster_kernel(const uint16_t *__restrict__ logits, int64_t ldl, int V, int C,
                                 int32_t *__restrict__ out, int32_t *__restrict__ append_to,
                                 int64_t append_stride, int32_t *__restrict__ append_pos) {
  extern __shared__ float s_e[];  // [C] exponentials of this CTA's entries
  __shared__ float s_red[kSampleThreads];
  __shared__ float s_slots[256];   // CTA 0: the 256 slot sums
  __shared__ float s_cmax;         // this CTA's row-part maximum
  __shared__ float s_best;         // this CTA's best probability ...
  __shared__ int s_best_j;         // ... and its first index
  pdl_wait();
  pdl_launch_dependents();
  const uint32_t r = cluster_ctarank();
  const int row = blockIdx.x / kSampleCluster, tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const uint16_t *x = logits + (int64_t)row * ldl;
  const int j0 = (int)r * C, j1 = min(V, j0 + C);
  // 1. maximum of this CTA's entries, then of the row
  float mx = -INFINITY;
  for (int j = j0 + tid; j < j1; j += kSampleThreads) mx = fmaxf(mx, bf2f(x[j]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) s_red[warp] = mx;
  __syncthreads();
  if (tid == 0) {
    float m = s_red[0];
    for (int w = 1; w < kSampleThreads / 32; ++w) m = fmaxf(m, s_red[w]);
    s_cmax = m;
  }
  cluster_sync_all();
  if (tid == 0) {
    float m = ld_dsmem_f32(dsmem_addr(&s_cmax, 0));
    for (int q = 1; q < kSampleCluster; ++q) m = fmaxf(m, ld_dsmem_f32(dsmem_addr(&s_cmax, q)));
    s_red[0] = m;
  }
  __syncthreads();
  mx = s_red[0];
  // 2. exponentials of this CTA's entries
  for (int j = j0 + tid; j < j1; j += kSampleThreads) s_e[j - j0] = expf(bf2f(x[j]) - mx);
  cluster_sync_all();
  // 3. slot sums, in order, over the cluster's shared memory
  if (warp == 0) {
    const int t = 32 * (int)r + lane;
    float acc = 0.0f;
    constexpr int kBatch = 8;  // loads in flight before their additions
    int q = 0, off = t;        // e_j lives in CTA q at offset off (C >= 256: q steps by <= 1)
    for (int jb = t; jb < V; jb += 256 * kBatch) {
      float e[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        e[u] = 0.0f;
        if (jb + 256 * u < V) {
          e[u] = ld_dsmem_f32(dsmem_addr(&s_e[off], (uint32_t)q));
          off += 256;
          if (off >= C) {
            off -= C;
            ++q;
          }
        }
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u)
        if (jb + 256 * u < V) acc += e[u];
    }
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(dsmem_addr(&s_slots[t], 0)), "f"(acc)
                 : "memory");
  }
  cluster_sync_all();
  s_red[tid] = ld_dsmem_f32(dsmem_addr(&s_slots[tid], 0));
  __syncthreads();
  for (int s = 128; s > 0; s >>= 1) {
    if (tid < s) s_red[tid] += s_red[tid + s];
    __syncthreads();
  }
  const float inv_sum = 1.0f / s_red[0];
  // 4. probabilities and the first index of the maximum
  float best = -1.0f;
  int best_j = 0x7fffffff;
  for (int j = j0 + tid; j < j1; j += kSampleThreads) {
    const float p = bf2f(f2bf(bf2f(f2bf(s_e[j - j0])) * inv_sum));
    if (p > best) {  // j increases within a thread: keeps the first index
      best = p;
      best_j = j;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oj = __shfl_xor_sync(0xffffffffu, best_j, o);
    if (ob > best || (ob == best && oj < best_j)) {
      best = ob;
      best_j = oj;
    }
  }
  __syncthreads();  // s_red is reused
  __shared__ int s_wj[kSampleThreads / 32];
  if (lane == 0) {
    s_red[warp] = best;
    s_wj[warp] = best_j;
  }
  __syncthreads();
  if (tid == 0) {
    float b = s_red[0];
    int bj = s_wj[0];
    for (int w = 1; w < kSampleThreads / 32; ++w) {
      if (s_red[w] > b || (s_red[w] == b && s_wj[w] < bj)) {
        b = s_red[w];
        bj = s_wj[w];
      }
    }
    s_best = b;
    s_best_j = bj;
  }
  cluster_sync_all();
  if (r == 0 && tid == 0) {
    float b = s_best;
    int bj = s_best_j;
    for (int q = 1; q < kSampleCluster; ++q) {
      const float ob = ld_dsmem_f32(dsmem_addr(&s_best, (uint32_t)q));
      const int oj = ld_dsmem_s32(dsmem_addr(&s_best_j, (uint32_t)q));
      if (ob > b || (ob == b && oj < bj)) {
        b = ob;
        bj = oj;
      }
    }
    // A row with no ordered maximum (all NaN) keeps index 0, as a host argmax
    // that starts from the first entry does; never an id outside the vocabulary.
    const int tok = bj < V ? bj : 0;
    out[row] = tok;
    if (append_to) {
      const int p = append_pos[row];
      append_to[(int64_t)row * append_stride + p] = tok;
      append_pos[row] = p + 1;
    }
  }
  cluster_sync_all();  // no CTA leaves while CTA 0 still reads its candidate
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
  const int C = (V + kSampleCluster - 1) / kSampleCluster;
  const size_t smem = (size_t)C * sizeof(float);
  if (M > 0 && V >= 256 * kSampleCluster && smem <= 200 * 1024) {
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
      if (cudaFuncSetAttribute(greedy_sample_cluster_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) !=
          cudaSuccess)
        return W8A8_ERR_CUDA;
      attr_set[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(M * kSampleCluster);
    cfg.blockDim = dim3(kSampleThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kSampleCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    if (cudaLaunchKernelEx(&cfg, greedy_sample_cluster_kernel, logits, ldl, V, C, out, append_to,
                           append_stride, append_pos) != cudaSuccess) {
      cudaGetLastError();
      return W8A8_ERR_CUDA;
    }
    return check_launch("greedy_sample_cluster");
  }
  launch_pdl(greedy_sample_kernel, dim3(M), dim3(256), 0, s, logits, ldl, V, out, append_to, append_stride,
                                         append_pos);
  return check_launch("greedy_sample");
}

int launch_advance(int32_t *dst, const int32_t *src, int n, int delta, cudaStream_t s) {
  launch_pdl(advance_kernel, dim3((n + 255) / 256), dim3(256), 0, s, dst, src, n, delta);
  return check_launch("advance");
}

}  // namespace w8a8
