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

// The same pick with one row spread over a cluster of kSampleCluster CTAs
// (at 1-64 rows one CTA per row leaves most SMs idle while each thread
// evaluates ~200 expf). CTA r owns entries [r*C, (r+1)*C) of the row, C a
// multiple of 256, so that slot t of the sum (entries t, t + 256, ...) meets
// its entries in CTA order:
//   1. its logits into shared memory (16-byte loads, all in flight), then
//      the row maximum (each CTA's, then the largest of all: order-free);
//   2. fp32 e_j = expf(x_j - max) for its entries, in every CTA at once;
//   3. the slot sums in the reference's order, passed along the cluster:
//      CTA r adds its entries of every slot to the running sums CTA r-1 left
//      in its shared memory (thread t: slot t) and hands them to CTA r+1; the
//      last CTA folds the 256 slots (s = 128 .. 1) and sends 1 / sum to all;
//   4. bf16 probabilities of its entries and the first index of their
//      maximum; CTA 0 picks the first index of the largest over the cluster.
constexpr int kSampleCluster = 4;
constexpr int kSampleThreads = 256;

__global__ void __launch_bounds__(kSampleThreads)
    greedy_sample_cluster_kernel(const uint16_t *__restrict__ logits, int64_t ldl, int V, int C,
                                 int32_t *__restrict__ out, int32_t *__restrict__ append_to,
                                 int64_t append_stride, int32_t *__restrict__ append_pos) {
  // shared memory: fp32 exponentials [C] | the CTA's logits
  extern __shared__ __align__(16) uint8_t gs_smem[];
  float *s_e = reinterpret_cast<float *>(gs_smem);
  __shared__ float s_red[kSampleThreads];
  __shared__ float s_slots[kSampleThreads];  // running slot sums from the previous CTA
  __shared__ float s_cmax, s_inv;
  __shared__ float s_best;  // this CTA's best probability ...
  __shared__ int s_best_j;  // ... and its first index
  __shared__ int s_wj[kSampleThreads / 32];
  pdl_wait();
  pdl_launch_dependents();
  const uint32_t r = cluster_ctarank();
  const int row = blockIdx.x / kSampleCluster, tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int j0 = (int)r * C, j1 = min(V, j0 + C), n = max(0, j1 - j0);
  const uint16_t *x = logits + (int64_t)row * ldl + j0;  // this CTA's entries
  // at the same position modulo 16 bytes as in global memory
  const int shift = (int)(((uintptr_t)x & 15) >> 1);
  uint16_t *x16 = reinterpret_cast<uint16_t *>(gs_smem + (size_t)C * 4) + shift;
  {
    const int head = min(n, (8 - shift) & 7);  // entries before the first 16-byte boundary
    const int nvec = (n - head) >> 3;
    for (int i = tid; i < head; i += kSampleThreads) x16[i] = x[i];
    const uint4 *xv = reinterpret_cast<const uint4 *>(x + head);
    uint4 *sv = reinterpret_cast<uint4 *>(x16 + head);
#pragma unroll 8
    for (int i = tid; i < nvec; i += kSampleThreads) sv[i] = __ldg(xv + i);
    for (int i = head + nvec * 8 + tid; i < n; i += kSampleThreads) x16[i] = x[i];
  }
  __syncthreads();
  // 1. maximum of this CTA's entries, then of the row
  float mx = -INFINITY;
#pragma unroll 4
  for (int i = tid; i < n; i += kSampleThreads) mx = fmaxf(mx, bf2f(x16[i]));
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
  if (tid < kSampleCluster) s_red[tid] = ld_dsmem_f32(dsmem_addr(&s_cmax, (uint32_t)tid));
  __syncthreads();
  mx = fmaxf(fmaxf(s_red[0], s_red[1]), fmaxf(s_red[2], s_red[3]));
  // 2. exponentials of this CTA's entries
#pragma unroll 4
  for (int i = tid; i < n; i += kSampleThreads) s_e[i] = expf(bf2f(x16[i]) - mx);
  __syncthreads();
  // 3. slot t adds entries t, t + 256, ... in order, CTA by CTA
  for (int q = 0; q < kSampleCluster; ++q) {
    if ((int)r == q) {
      float acc = q == 0 ? 0.0f : s_slots[tid];
#pragma unroll 8
      for (int i = tid; i < n; i += kSampleThreads) acc += s_e[i];
      if (q + 1 < kSampleCluster) {
        asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(dsmem_addr(&s_slots[tid], r + 1)),
                     "f"(acc)
                     : "memory");
      } else {
        s_red[tid] = acc;
      }
    }
    cluster_sync_all();
  }
  if ((int)r == kSampleCluster - 1) {
    for (int h = kSampleThreads / 2; h > 0; h >>= 1) {
      if (tid < h) s_red[tid] += s_red[tid + h];
      __syncthreads();
    }
    if (tid < kSampleCluster) {
      const float inv = 1.0f / s_red[0];
      asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(dsmem_addr(&s_inv, (uint32_t)tid)),
                   "f"(inv)
                   : "memory");
    }
  }
  cluster_sync_all();
  const float inv_sum = s_inv;
  // 4. probabilities and the first index of the maximum
  float best = -1.0f;
  int best_j = 0x7fffffff;
  for (int i = tid; i < n; i += kSampleThreads) {
    const float p = bf2f(f2bf(bf2f(f2bf(s_e[i])) * inv_sum));
    if (p > best) {  // i increases within a thread: keeps the first index
      best = p;
      best_j = j0 + i;
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
  // each CTA a multiple of 256 entries: exponentials (fp32) + logits in shared memory
  const int C = 256 * ((V + 256 * kSampleCluster - 1) / (256 * kSampleCluster));
  const size_t smem = (size_t)C * 4 + ((size_t)(C + 8) * 2 + 15) / 16 * 16;
  if (M > 0 && V >= 2048 && smem <= 200 * 1024) {
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
    attr[1].val.programmaticStreamSerializationAllowed = 1;
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

// ---- top-k sampling at a temperature (gpt2.c:130-180, gpt2.c:2223-2245) ----
//
// The reference, per generated token: probs = softmax_cuda(logits, T) in bf16
// (cuda/softmax.cu:24-92); copies them to the host; sorts (probability, index)
// pairs by descending probability with qsort; sums the first k probabilities
// in that order in fp32; divides each of them by the sum into bf16 (or sets
// every one to bf16(1/k) if the sum is 0); draws r = rand()/RAND_MAX; adds
// the renormalised probabilities in order in fp32 and takes the first token
// whose running sum exceeds r, else the k-th.
//
// One CTA per row does all of it on the GPU. The probabilities are non-negative
// bf16 values at most 1.0, so their bit patterns 0 .. 0x3F80 order them: a
// histogram over those 16257 keys replaces the sort. Every sum depends only on
// the sequence of probability VALUES in sorted order, which ties do not change,
// so the fp32 sums are the reference's to the bit; warp 0 walks the non-empty
// keys from the top and adds each key's value once per token that has it.
// Which of several equal-probability tokens comes first is what qsort leaves
// unspecified; here it is the lowest index (also at the k-th place).
constexpr int kTopkThreads = 256;
constexpr int kTopkBins = 0x3F81;  // keys of +0.0 .. 1.0
constexpr size_t kTopkHistBytes = ((size_t)kTopkBins * 4 + 15) / 16 * 16;
constexpr int kTopkMaxVocab = 81920;

// (A row whose logits hold NaN or infinities gives probabilities outside
// [0, 1]; they count as 1.0, so every index stays in range and the token is
// some id in [0, V).)
__device__ __forceinline__ int topk_key(uint16_t p) { return p <= 0x3F80 ? (int)p : 0x3F80; }

__global__ void __launch_bounds__(kTopkThreads)
    topk_sample_kernel(const uint16_t *__restrict__ logits, int64_t ldl, int V, float inv_temp,
                       int k, const float *__restrict__ rnd, int64_t rnd_stride,
                       const int32_t *__restrict__ rnd_pos, int32_t *__restrict__ out,
                       int32_t *__restrict__ append_to, int64_t append_stride,
                       int32_t *__restrict__ append_pos, uint16_t *__restrict__ probs_out,
                       int64_t ldp) {
  extern __shared__ __align__(16) uint8_t tk_smem[];
  uint32_t *hist = reinterpret_cast<uint32_t *>(tk_smem);  // [kTopkBins]
  __shared__ float s_red[kTopkThreads];
  __shared__ uint32_t s_scan[kTopkThreads];
  __shared__ int s_thr_key, s_take, s_top_key, s_sel_key, s_sel_rank, s_tok, s_first;
  pdl_wait();
  pdl_launch_dependents();
  const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint16_t *x = logits + (int64_t)row * ldl;
  // The row (logits, then exponentials, then probabilities) in shared memory
  // at the same position modulo 16 bytes as in global memory (rows start on
  // 2-byte boundaries), so that the copy moves aligned 16-byte vectors.
  const int shift = (int)(((uintptr_t)x & 15) >> 1);
  uint16_t *p16 = reinterpret_cast<uint16_t *>(tk_smem + kTopkHistBytes) + shift;  // [V]
  for (int b = tid; b < kTopkBins; b += kTopkThreads) hist[b] = 0;
  if (tid == 0) {
    s_tok = 0;
    s_thr_key = 0;
    s_take = 1;
    s_top_key = 0;
    s_first = 0x7fffffff;
  }
  {
    const int head = min(V, (8 - shift) & 7);  // elements before the first 16-byte boundary
    const int nvec = (V - head) >> 3;
    for (int j = tid; j < head; j += kTopkThreads) p16[j] = x[j];
    const uint4 *xv = reinterpret_cast<const uint4 *>(x + head);
    uint4 *sv = reinterpret_cast<uint4 *>(p16 + head);
#pragma unroll 4
    for (int i = tid; i < nvec; i += kTopkThreads) sv[i] = __ldg(xv + i);
    for (int j = head + nvec * 8 + tid; j < V; j += kTopkThreads) p16[j] = x[j];
  }
  __syncthreads();

  // 1. row maximum of x * (1/T)
  float mx = -INFINITY;
#pragma unroll 4
  for (int j = tid; j < V; j += kTopkThreads) mx = fmaxf(mx, bf2f(p16[j]) * inv_temp);
  s_red[tid] = mx;
  __syncthreads();
  for (int s = kTopkThreads / 2; s > 0; s >>= 1) {
    if (tid < s) s_red[tid] = fmaxf(s_red[tid], s_red[tid + s]);
    __syncthreads();
  }
  mx = s_red[0];
  __syncthreads();
  // 2. exponentials (kept as bf16, as the reference stores them) and the
  //    256-slot sum tree of softmax.cu:62-82 (slot t adds j = t, t+256, ...)
  float acc = 0.0f;
#pragma unroll 4
  for (int j = tid; j < V; j += kTopkThreads) {
    const float e = expf(__fmaf_rn(bf2f(p16[j]), inv_temp, -mx));
    p16[j] = f2bf(e);
    acc += e;
  }
  s_red[tid] = acc;
  __syncthreads();
  for (int s = kTopkThreads / 2; s > 0; s >>= 1) {
    if (tid < s) s_red[tid] += s_red[tid + s];
    __syncthreads();
  }
  const float inv_sum = 1.0f / s_red[0];
  // 3. bf16 probabilities and the histogram of their keys (each thread
  //    rewrites only the entries it wrote in step 2; lanes of a warp mostly
  //    hold different keys, and those that share one are serialised by the
  //    shared-memory atomic); s_top_key: the largest key present
  int top_key = 0;
#pragma unroll 4
  for (int j = tid; j < V; j += kTopkThreads) {
    const uint16_t p = f2bf(bf2f(p16[j]) * inv_sum);
    p16[j] = p;
    if (probs_out) probs_out[(int64_t)row * ldp + j] = p;
    const int key = topk_key(p);
    atomicAdd(&hist[key], 1u);
    top_key = max(top_key, key);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) top_key = max(top_key, __shfl_xor_sync(0xffffffffu, top_key, o));
  if (lane == 0) atomicMax(&s_top_key, top_key);
  __syncthreads();

  // 4. the k-th key from the top: thread t sums keys [64t, 64t+64); a scan
  //    over the threads in descending key order gives the count above each
  //    chunk, and the one chunk where the count reaches k is walked key by key
  constexpr int kChunk = (kTopkBins + kTopkThreads - 1) / kTopkThreads;
  const int c_lo = tid * kChunk, c_hi = min(kTopkBins, c_lo + kChunk);
  // (each lane starts at its own offset in its chunk: chunks are 64 words
  // apart, so lanes reading the same offset would all hit one bank)
  uint32_t mine = 0;
  const int c_n = max(0, c_hi - c_lo);
  if (c_n > 0) {
    const int o = lane % c_n;
    for (int i = 0; i < c_n; ++i) {
      const int b = i + o < c_n ? i + o : i + o - c_n;
      mine += hist[c_lo + b];
    }
  }
  s_scan[kTopkThreads - 1 - tid] = mine;
  __syncthreads();
  for (int off = 1; off < kTopkThreads; off <<= 1) {
    const uint32_t v = s_scan[tid] + (tid >= off ? s_scan[tid - off] : 0u);
    __syncthreads();
    s_scan[tid] = v;
    __syncthreads();
  }
  const uint32_t above = s_scan[kTopkThreads - 1 - tid] - mine;  // tokens in higher chunks
  if (above < (uint32_t)k && above + mine >= (uint32_t)k) {
    uint32_t cnt = above;
    for (int b = c_hi - 1; b >= c_lo; --b) {
      if (cnt + hist[b] >= (uint32_t)k) {
        s_thr_key = b;
        s_take = k - (int)cnt;
        break;
      }
      cnt += hist[b];
    }
  }
  __syncthreads();

  // 5. warp 0: fp32 sum of the k probabilities in descending order, their
  //    renormalised bf16 values, and the draw. Lanes hold 32 keys at a time
  //    (lane l: key b0 - l), from the largest present key down, and run the
  //    additions in lock step with the same values.
  if (warp == 0) {
    const int thr = s_thr_key, take = s_take, top = max(s_top_key, thr);
    float sum = 0.0f;
    for (int b0 = top; b0 >= thr; b0 -= 32) {
      const int b = b0 - lane;
      const uint32_t h = b > thr ? hist[b] : (b == thr ? (uint32_t)take : 0u);
      uint32_t nz = __ballot_sync(0xffffffffu, h != 0);
      while (nz) {
        const int l = __ffs(nz) - 1;  // lowest lane = highest key
        nz &= nz - 1;
        const uint32_t n = __shfl_sync(0xffffffffu, h, l);
        const float pv = bf2f((uint16_t)(b0 - l));
        // sum += pv, n times, in order; once an addition leaves the sum
        // unchanged every later one of pv does too
        uint32_t i = 0;
        for (; i + 4 <= n; i += 4) {
          const float a1 = sum + pv, a2 = a1 + pv, a3 = a2 + pv, a4 = a3 + pv;
          sum = a4;
          if (a4 == a3) {
            i = n;
            break;
          }
        }
        for (; i < n; ++i) {
          const float ns = sum + pv;
          if (ns == sum) break;
          sum = ns;
        }
      }
    }
    const bool uniform = !(sum > 0.0f);
    const float q_uniform = bf2f(f2bf(__fdiv_rn(1.0f, (float)k)));
    const float r = rnd[(int64_t)row * rnd_stride + (rnd_pos ? rnd_pos[row] : 0)];
    int sel_key = thr, sel_rank = take - 1;  // no running sum above r: the k-th token
    float cum = 0.0f;
    bool done = false;
    for (int b0 = top; b0 >= thr && !done; b0 -= 32) {
      const int b = b0 - lane;
      const uint32_t h = b > thr ? hist[b] : (b == thr ? (uint32_t)take : 0u);
      // each lane's renormalised value, bf16(p / sum), for its own key
      const float q_l =
          uniform ? q_uniform : bf2f(f2bf(__fdiv_rn(bf2f((uint16_t)max(b, 0)), sum)));
      uint32_t nz = __ballot_sync(0xffffffffu, h != 0);
      while (nz && !done) {
        const int l = __ffs(nz) - 1;
        nz &= nz - 1;
        const uint32_t n = __shfl_sync(0xffffffffu, h, l);
        const float q = __shfl_sync(0xffffffffu, q_l, l);
        // cum += q, n times; the first running sum above r picks the token.
        // Later terms are no larger than q, so a running sum that q no
        // longer moves stays at or below r: the k-th token is taken.
        uint32_t i = 0;
        for (; i + 4 <= n; i += 4) {
          const float c1 = cum + q, c2 = c1 + q, c3 = c2 + q, c4 = c3 + q;
          if (r < c4) {
            sel_key = b0 - l;
            sel_rank = (int)i + (r < c1 ? 0 : r < c2 ? 1 : r < c3 ? 2 : 3);
            done = true;
            break;
          }
          if (c4 == c3) {
            done = true;
            break;
          }
          cum = c4;
        }
        for (; i < n && !done; ++i) {
          const float nc = cum + q;
          if (r < nc) {
            sel_key = b0 - l;
            sel_rank = (int)i;
            done = true;
            break;
          }
          if (nc == cum) {
            done = true;
            break;
          }
          cum = nc;
        }
      }
    }
    if (lane == 0) {
      s_sel_key = sel_key;
      s_sel_rank = sel_rank;
    }
  }
  __syncthreads();

  // 6. the token: the sel_rank-th (from 0) index, in ascending order, whose
  //    key is sel_key. Rank 0 (every drawn probability that no other token
  //    shares): the first such index, each thread stopping at its own first
  //    one. Otherwise thread t counts over its contiguous share of the row, a
  //    scan over the threads finds the share holding the wanted one, and that
  //    thread walks its share.
  const int sel_key = s_sel_key, sel_rank = s_sel_rank;
  if (sel_rank == 0) {
    // (eight entries per round, so that the loads are in flight together; the
    // thread holding the match is usually the only one that stops early)
    int first = 0x7fffffff;
    for (int j0 = tid; j0 < V && first == 0x7fffffff; j0 += 8 * kTopkThreads) {
      int key[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int j = j0 + u * kTopkThreads;
        key[u] = j < V ? topk_key(p16[j]) : -1;
      }
#pragma unroll
      for (int u = 7; u >= 0; --u)
        if (key[u] == sel_key) first = j0 + u * kTopkThreads;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) first = min(first, __shfl_xor_sync(0xffffffffu, first, o));
    if (lane == 0) atomicMin(&s_first, first);
    __syncthreads();
    if (tid == 0 && s_first < V) s_tok = s_first;
  } else {
    const int per = (V + kTopkThreads - 1) / kTopkThreads;
    const int j_lo = min(V, tid * per), j_hi = min(V, j_lo + per);
    uint32_t cnt = 0;
    for (int j = j_lo; j < j_hi; ++j) cnt += topk_key(p16[j]) == sel_key;
    s_scan[tid] = cnt;
    __syncthreads();
    for (int off = 1; off < kTopkThreads; off <<= 1) {
      const uint32_t v = s_scan[tid] + (tid >= off ? s_scan[tid - off] : 0u);
      __syncthreads();
      s_scan[tid] = v;
      __syncthreads();
    }
    const uint32_t before = s_scan[tid] - cnt;
    if (before <= (uint32_t)sel_rank && (uint32_t)sel_rank < before + cnt) {
      uint32_t c = before;
      for (int j = j_lo; j < j_hi; ++j) {
        if (topk_key(p16[j]) == sel_key) {
          if (c == (uint32_t)sel_rank) {
            s_tok = j;
            break;
          }
          ++c;
        }
      }
    }
  }
  __syncthreads();
  if (tid == 0) {
    const int tok = s_tok;
    out[row] = tok;
    if (append_to) {
      const int p = append_pos[row];
      append_to[(int64_t)row * append_stride + p] = tok;
      append_pos[row] = p + 1;
    }
  }
}

// The same top-k sampling with one row spread over a cluster of kTkCluster
// CTAs (one CTA per row leaves most SMs idle while its 8 warps evaluate ~200
// exponentials a thread). CTA r owns entries [r*C, (r+1)*C) of the row, C a
// multiple of 256, so that slot t of the sum (entries t, t + 256, ...) meets
// its entries in CTA order:
//   1. its logits into shared memory (16-byte loads, all in flight), then
//      the row maximum (each CTA's, then the largest of all: order-free);
//   2. the slot sums in the reference's order, passed along the cluster:
//      CTA r adds the exponentials of its entries of every slot to the
//      running sums CTA r-1 left in its shared memory (thread t: slot t) and
//      hands them to CTA r+1; the last CTA folds the 256 slots (s = 128 .. 1)
//      and sends 1 / sum to all;
//   4. bf16 probabilities (the same exponentials again), in place of the
//      logits, and a histogram of their keys (16-bit counts, two to a word:
//      at most 65535 entries a row);
//   5. CTA 0: the threshold key and the draw from the cluster's counts (the
//      per-CTA counts of 64-key chunks, then of the keys of one chunk, then of
//      every key from the threshold up, merged into its own histogram);
//   6. the sel_rank-th entry with the drawn key, counted over the CTAs in
//      index order; the CTA that holds it writes the token.
// Same values, sums and tie rule as topk_sample_kernel.
constexpr int kTkCluster = 4;
constexpr int kTkThreads = 256;
constexpr int kTkHistWords = (kTopkBins + 1) / 2;
constexpr size_t kTkHistBytes = ((size_t)kTkHistWords * 4 + 15) / 16 * 16;  // keeps what follows 16-byte aligned
constexpr int kTkMaxVocab = 65535;

__device__ __forceinline__ uint32_t tk_count(uint32_t w, int b) { return (w >> ((b & 1) * 16)) & 0xffffu; }

// Count of key b over the cluster's histograms.
__device__ __forceinline__ uint32_t tk_cluster_count(const uint32_t *hist, int b) {
  uint32_t c = 0;
#pragma unroll
  for (int q = 0; q < kTkCluster; ++q)
    c += tk_count((uint32_t)ld_dsmem_s32(dsmem_addr(&hist[b >> 1], (uint32_t)q)), b);
  return c;
}

__global__ void __launch_bounds__(kTkThreads)
    topk_sample_cluster_kernel(const uint16_t *__restrict__ logits, int64_t ldl, int V, int C,
                               int ebytes, float inv_temp, int k, const float *__restrict__ rnd,
                               int64_t rnd_stride, const int32_t *__restrict__ rnd_pos,
                               int32_t *__restrict__ out, int32_t *__restrict__ append_to,
                               int64_t append_stride, int32_t *__restrict__ append_pos,
                               uint16_t *__restrict__ probs_out, int64_t ldp) {
  // shared memory: histogram | ebytes: fp32 exponentials [C], then the list
  // of keys in step 4 (at most min(V, kTopkBins) + 1) | the CTA's logits,
  // then its probabilities
  extern __shared__ __align__(16) uint8_t tkc_smem[];
  uint32_t *hist = reinterpret_cast<uint32_t *>(tkc_smem);  // [kTkHistWords]
  float *e32 = reinterpret_cast<float *>(tkc_smem + kTkHistBytes);  // [C]
  __shared__ float s_red[kTkThreads];
  __shared__ float s_slots[kTkThreads];   // running slot sums from the previous CTA
  __shared__ uint32_t s_chunk[kTkThreads];
  __shared__ uint32_t s_scan[kTkThreads];
  __shared__ float s_cmax, s_inv;
  __shared__ int s_top_key, s_thr_key, s_take, s_sel_key, s_sel_rank, s_tok_cnt, s_chunk_sel,
      s_nlist;
  pdl_wait();
  pdl_launch_dependents();
  const uint32_t r = cluster_ctarank();
  const int row = blockIdx.x / kTkCluster, tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int j0 = (int)r * C, j1 = min(V, j0 + C), n = max(0, j1 - j0);
  const uint16_t *x = logits + (int64_t)row * ldl + j0;  // this CTA's entries
  // its logits (then probabilities) at the same position modulo 16 bytes as
  // in global memory, so that the copy moves aligned 16-byte vectors
  const int shift = (int)(((uintptr_t)x & 15) >> 1);
  uint16_t *p16 = reinterpret_cast<uint16_t *>(tkc_smem + kTkHistBytes + ebytes) + shift;
  for (int w = tid; w < kTkHistWords; w += kTkThreads) hist[w] = 0u;
  if (tid == 0) {
    s_top_key = 0;
    s_thr_key = 0;
    s_take = 1;
    s_chunk_sel = -1;
  }
  {
    const int head = min(n, (8 - shift) & 7);  // entries before the first 16-byte boundary
    const int nvec = (n - head) >> 3;
    for (int i = tid; i < head; i += kTkThreads) p16[i] = x[i];
    const uint4 *xv = reinterpret_cast<const uint4 *>(x + head);
    uint4 *sv = reinterpret_cast<uint4 *>(p16 + head);
#pragma unroll 8
    for (int i = tid; i < nvec; i += kTkThreads) sv[i] = __ldg(xv + i);
    for (int i = head + nvec * 8 + tid; i < n; i += kTkThreads) p16[i] = x[i];
  }
  __syncthreads();

  // 1. row maximum of x * (1/T)
  float mx = -INFINITY;
#pragma unroll 4
  for (int i = tid; i < n; i += kTkThreads) mx = fmaxf(mx, bf2f(p16[i]) * inv_temp);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) s_red[warp] = mx;
  __syncthreads();
  if (tid == 0) {
    float m = s_red[0];
    for (int w = 1; w < kTkThreads / 32; ++w) m = fmaxf(m, s_red[w]);
    s_cmax = m;
  }
  cluster_sync_all();
  if (tid < kTkCluster) s_red[tid] = ld_dsmem_f32(dsmem_addr(&s_cmax, (uint32_t)tid));
  __syncthreads();
  mx = fmaxf(fmaxf(s_red[0], s_red[1]), fmaxf(s_red[2], s_red[3]));

  // 2. the exponentials of this CTA's entries (all CTAs at once), then slot t
  //    adds those of entries t, t + 256, ... unrounded, in order: CTA by CTA,
  //    continuing from the running sums of the CTA before
#pragma unroll 4
  for (int i = tid; i < n; i += kTkThreads) e32[i] = expf(__fmaf_rn(bf2f(p16[i]), inv_temp, -mx));
  __syncthreads();
  for (int q = 0; q < kTkCluster; ++q) {
    if ((int)r == q) {
      float acc = q == 0 ? 0.0f : s_slots[tid];
#pragma unroll 8
      for (int i = tid; i < n; i += kTkThreads) acc += e32[i];
      if (q + 1 < kTkCluster) {
        asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(dsmem_addr(&s_slots[tid], r + 1)),
                     "f"(acc)
                     : "memory");
      } else {
        s_red[tid] = acc;
      }
    }
    cluster_sync_all();
  }
  if ((int)r == kTkCluster - 1) {
    for (int h = kTkThreads / 2; h > 0; h >>= 1) {
      if (tid < h) s_red[tid] += s_red[tid + h];
      __syncthreads();
    }
    if (tid < kTkCluster) {
      const float inv = 1.0f / s_red[0];
      asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(dsmem_addr(&s_inv, (uint32_t)tid)),
                   "f"(inv)
                   : "memory");
    }
  }
  cluster_sync_all();
  const float inv_sum = s_inv;

  // 3. bf16 probabilities (in place of the logits), the histogram of their
  //    keys, the largest key
  int top_key = 0;
#pragma unroll 4
  for (int i = tid; i < n; i += kTkThreads) {
    const uint16_t pb = f2bf(bf2f(f2bf(e32[i])) * inv_sum);
    p16[i] = pb;
    if (probs_out) probs_out[(int64_t)row * ldp + j0 + i] = pb;
    const int key = topk_key(pb);
    atomicAdd(&hist[key >> 1], 1u << ((key & 1) * 16));
    top_key = max(top_key, key);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) top_key = max(top_key, __shfl_xor_sync(0xffffffffu, top_key, o));
  if (lane == 0) atomicMax(&s_top_key, top_key);
  __syncthreads();
  // this CTA's count of each 64-key chunk (thread t: keys [64t, 64t + 64);
  // each lane starts at its own offset: chunks are 32 words apart)
  constexpr int kChunk = 64;
  {
    const int w_lo = tid * (kChunk / 2), w_hi = min(kTkHistWords, w_lo + kChunk / 2);
    const int cw = max(0, w_hi - w_lo);
    uint32_t mine = 0;
    if (cw > 0) {
      const int o = lane % cw;
      for (int i = 0; i < cw; ++i) {
        const int w = i + o < cw ? i + o : i + o - cw;
        const uint32_t v = hist[w_lo + w];
        mine += (v & 0xffffu) + (v >> 16);
      }
    }
    s_chunk[tid] = mine;
  }
  cluster_sync_all();

  // 4. CTA 0: the threshold key and the draw
  if (r == 0) {
    uint32_t g = 0;  // the cluster's count of chunk tid
#pragma unroll
    for (int q = 0; q < kTkCluster; ++q)
      g += (uint32_t)ld_dsmem_s32(dsmem_addr(&s_chunk[tid], (uint32_t)q));
    if (tid < kTkCluster) s_red[tid] = (float)ld_dsmem_s32(dsmem_addr(&s_top_key, (uint32_t)tid));
    s_scan[kTkThreads - 1 - tid] = g;
    __syncthreads();
    for (int off = 1; off < kTkThreads; off <<= 1) {
      const uint32_t v = s_scan[tid] + (tid >= off ? s_scan[tid - off] : 0u);
      __syncthreads();
      s_scan[tid] = v;
      __syncthreads();
    }
    const uint32_t above = s_scan[kTkThreads - 1 - tid] - g;  // entries in higher chunks
    if (above < (uint32_t)k && above + g >= (uint32_t)k) {
      s_chunk_sel = tid;
      s_tok_cnt = (int)above;
    }
    __syncthreads();
    const int top = max(max((int)s_red[0], (int)s_red[1]), max((int)s_red[2], (int)s_red[3]));
    if (warp == 0 && s_chunk_sel >= 0) {
      // the chunk's 64 keys from the top, two per lane (lane l: keys
      // c_hi - 1 - l and c_hi - 33 - l), and their running counts from the
      // top: the threshold is the first key where the count reaches k
      const int c_hi = s_chunk_sel * kChunk + kChunk;
      const int b_a = c_hi - 1 - lane, b_b = c_hi - 33 - lane;
      const uint32_t h_a = b_a < kTopkBins ? tk_cluster_count(hist, b_a) : 0u;
      const uint32_t h_b = b_b < kTopkBins ? tk_cluster_count(hist, b_b) : 0u;
      uint32_t c_a = h_a, c_b = h_b;  // inclusive scans over the lanes
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t ta = __shfl_up_sync(0xffffffffu, c_a, o);
        const uint32_t tb = __shfl_up_sync(0xffffffffu, c_b, o);
        if (lane >= o) {
          c_a += ta;
          c_b += tb;
        }
      }
      const uint32_t base = (uint32_t)s_tok_cnt;
      const uint32_t tot_a = __shfl_sync(0xffffffffu, c_a, 31);
      const unsigned hit_a = __ballot_sync(0xffffffffu, base + c_a >= (uint32_t)k);
      const unsigned hit_b = __ballot_sync(0xffffffffu, base + tot_a + c_b >= (uint32_t)k);
      // the count above the threshold key: the scan value of the lane before it
      const int l_a = hit_a ? __ffs(hit_a) - 1 : -1;
      const int l_b = hit_b ? __ffs(hit_b) - 1 : -1;
      const uint32_t prev_a = __shfl_sync(0xffffffffu, c_a - h_a, l_a >= 0 ? l_a : 0);
      const uint32_t prev_b = __shfl_sync(0xffffffffu, c_b - h_b, l_b >= 0 ? l_b : 0);
      if (lane == 0) {
        if (l_a >= 0) {
          s_thr_key = c_hi - 1 - l_a;
          s_take = k - (int)(base + prev_a);
        } else if (l_b >= 0) {
          s_thr_key = c_hi - 33 - l_b;
          s_take = k - (int)(base + tot_a + prev_b);
        }
      }
    }
    __syncthreads();
    // every key from the threshold up: the cluster's counts into this CTA's
    // histogram (each word read here before it is rewritten)
    const int thr = s_thr_key, take = s_take, top_k = max(top, thr);
    for (int w = (thr >> 1) + tid; w <= (top_k >> 1); w += kTkThreads) {
      uint32_t v = hist[w];
#pragma unroll
      for (int q = 1; q < kTkCluster; ++q) v += (uint32_t)ld_dsmem_s32(dsmem_addr(&hist[w], (uint32_t)q));
      hist[w] = v;  // per-key sums stay below 2^16: V <= 65535
    }
    __syncthreads();
    // the keys of [thr, top_k] that entries hold, in descending order: thread
    // t flags a contiguous run of the range, a scan places them
    uint16_t *list = reinterpret_cast<uint16_t *>(e32);
    const int R = top_k - thr + 1;
    const int per = (R + kTkThreads - 1) / kTkThreads;
    const int i_lo = min(R, tid * per), i_hi = min(R, i_lo + per);
    uint32_t cnt = 0;
    for (int i = i_lo; i < i_hi; ++i) {
      const int b = top_k - i;
      cnt += (b == thr || tk_count(hist[b >> 1], b) != 0u) ? 1u : 0u;
    }
    s_scan[tid] = cnt;
    __syncthreads();
    for (int off = 1; off < kTkThreads; off <<= 1) {
      const uint32_t v = s_scan[tid] + (tid >= off ? s_scan[tid - off] : 0u);
      __syncthreads();
      s_scan[tid] = v;
      __syncthreads();
    }
    {
      uint32_t pos = s_scan[tid] - cnt;
      for (int i = i_lo; i < i_hi; ++i) {
        const int b = top_k - i;
        if (b == thr || tk_count(hist[b >> 1], b) != 0u) list[pos++] = (uint16_t)b;
      }
      if (tid == kTkThreads - 1) s_nlist = (int)s_scan[tid];
    }
    __syncthreads();
    if (warp == 0) {
      // the k probabilities in descending order: entry e of the list holds
      // key list[e], present h times (take times for the threshold key)
      const int nl = s_nlist;
      float sum = 0.0f;
      for (int e0 = 0; e0 < nl; e0 += 32) {
        const int e = e0 + lane;
        const int b = e < nl ? (int)list[e] : 0;
        const uint32_t h = e >= nl ? 0u : (b > thr ? tk_count(hist[b >> 1], b) : (uint32_t)take);
        const int m = min(32, nl - e0);
        for (int l = 0; l < m; ++l) {
          const uint32_t cn = __shfl_sync(0xffffffffu, h, l);
          const float pv = bf2f((uint16_t)__shfl_sync(0xffffffffu, b, l));
          // sum += pv, cn times, in order; once an addition leaves the sum
          // unchanged every later one of pv does too
          uint32_t i = 0;
          for (; i + 4 <= cn; i += 4) {
            const float a1 = sum + pv, a2 = a1 + pv, a3 = a2 + pv, a4 = a3 + pv;
            sum = a4;
            if (a4 == a3) {
              i = cn;
              break;
            }
          }
          for (; i < cn; ++i) {
            const float ns = sum + pv;
            if (ns == sum) break;
            sum = ns;
          }
        }
      }
      const bool uniform = !(sum > 0.0f);
      const float q_uniform = bf2f(f2bf(__fdiv_rn(1.0f, (float)k)));
      const float rv = rnd[(int64_t)row * rnd_stride + (rnd_pos ? rnd_pos[row] : 0)];
      int sel_key = thr, sel_rank = take - 1;  // no running sum above r: the k-th token
      float cum = 0.0f;
      bool done = false;
      for (int e0 = 0; e0 < nl && !done; e0 += 32) {
        const int e = e0 + lane;
        const int b = e < nl ? (int)list[e] : 0;
        const uint32_t h = e >= nl ? 0u : (b > thr ? tk_count(hist[b >> 1], b) : (uint32_t)take);
        // each lane's renormalised value, bf16(p / sum), for its own key
        const float q_l = uniform ? q_uniform : bf2f(f2bf(__fdiv_rn(bf2f((uint16_t)b), sum)));
        const int m = min(32, nl - e0);
        for (int l = 0; l < m && !done; ++l) {
          const uint32_t cn = __shfl_sync(0xffffffffu, h, l);
          const float qv = __shfl_sync(0xffffffffu, q_l, l);
          const int bk = __shfl_sync(0xffffffffu, b, l);
          // cum += q, cn times; the first running sum above r picks the
          // token. Later terms are no larger than q, so a running sum that q
          // no longer moves stays at or below r: the k-th token is taken.
          uint32_t i = 0;
          for (; i + 4 <= cn; i += 4) {
            const float c1 = cum + qv, c2 = c1 + qv, c3 = c2 + qv, c4 = c3 + qv;
            if (rv < c4) {
              sel_key = bk;
              sel_rank = (int)i + (rv < c1 ? 0 : rv < c2 ? 1 : rv < c3 ? 2 : 3);
              done = true;
              break;
            }
            if (c4 == c3) {
              done = true;
              break;
            }
            cum = c4;
          }
          for (; i < cn && !done; ++i) {
            const float nc = cum + qv;
            if (rv < nc) {
              sel_key = bk;
              sel_rank = (int)i;
              done = true;
              break;
            }
            if (nc == cum) {
              done = true;
              break;
            }
            cum = nc;
          }
        }
      }
      if (lane < kTkCluster) {
        asm volatile("st.shared::cluster.s32 [%0], %1;" ::"r"(dsmem_addr(&s_sel_key, (uint32_t)lane)),
                     "r"(sel_key)
                     : "memory");
        asm volatile("st.shared::cluster.s32 [%0], %1;" ::"r"(dsmem_addr(&s_sel_rank, (uint32_t)lane)),
                     "r"(sel_rank)
                     : "memory");
      }
    }
  }
  cluster_sync_all();

  // 5. this CTA's entries with the drawn key: thread t counts its contiguous
  //    share; a scan gives the CTA's total and each share's start
  const int sel_key = s_sel_key, sel_rank = s_sel_rank;
  const int per = (n + kTkThreads - 1) / kTkThreads;
  const int i_lo = min(n, tid * per), i_hi = min(n, i_lo + per);
  uint32_t cnt = 0;
  for (int i = i_lo; i < i_hi; ++i) cnt += topk_key(p16[i]) == sel_key;
  s_scan[tid] = cnt;
  __syncthreads();
  for (int off = 1; off < kTkThreads; off <<= 1) {
    const uint32_t v = s_scan[tid] + (tid >= off ? s_scan[tid - off] : 0u);
    __syncthreads();
    s_scan[tid] = v;
    __syncthreads();
  }
  if (tid == kTkThreads - 1) s_tok_cnt = (int)s_scan[tid];
  cluster_sync_all();
  uint32_t before = 0;  // matches in the CTAs before this one
  for (int q = 0; q < (int)r; ++q) before += (uint32_t)ld_dsmem_s32(dsmem_addr(&s_tok_cnt, (uint32_t)q));
  before += s_scan[tid] - cnt;
  if (before <= (uint32_t)sel_rank && (uint32_t)sel_rank < before + cnt) {
    uint32_t c = before;
    for (int i = i_lo; i < i_hi; ++i) {
      if (topk_key(p16[i]) == sel_key) {
        if (c == (uint32_t)sel_rank) {
          const int tok = j0 + i;
          out[row] = tok;
          if (append_to) {
            const int ap = append_pos[row];
            append_to[(int64_t)row * append_stride + ap] = tok;
            append_pos[row] = ap + 1;
          }
          break;
        }
        ++c;
      }
    }
  }
  cluster_sync_all();  // no CTA leaves while another still reads its shared memory
}

int launch_topk_sample(const uint16_t *logits, int64_t ldl, int M, int V, float temperature,
                       int k, const float *rnd, int64_t rnd_stride, const int32_t *rnd_pos,
                       int32_t *out, int32_t *append_to, int64_t append_stride,
                       int32_t *append_pos, uint16_t *probs_out, int64_t ldp, cudaStream_t s) {
  if (V > kTopkMaxVocab) return W8A8_ERR_UNSUPPORTED;
  const size_t smem = kTopkHistBytes + ((size_t)(V + 8) * 2 + 15) / 16 * 16;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    if (cudaFuncSetAttribute(topk_sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)(kTopkHistBytes + (size_t)(kTopkMaxVocab + 8) * 2)) !=
        cudaSuccess)
      return W8A8_ERR_CUDA;
    attr_set[dev] = true;
  }
  if (k < 1) k = 1;  // gpt2.c:1963-1968 clamps top_k to [1, vocab]
  if (k > V) k = V;
  const float inv_temp = 1.0f / temperature;  // IEEE division, as softmax.cu:32 on the device
  if (V <= kTkMaxVocab) {
    // one row over a cluster of kTkCluster CTAs, each with a multiple of 256 entries
    const int C = 256 * ((V + 256 * kTkCluster - 1) / (256 * kTkCluster));
    // the exponentials' region also holds step 4's list of distinct keys
    const size_t list_bytes = (size_t)(min(V, kTopkBins) + 2) * 2;
    const int ebytes = (int)(((list_bytes > (size_t)C * 4 ? list_bytes : (size_t)C * 4) + 15) / 16 * 16);
    const size_t csmem = kTkHistBytes + (size_t)ebytes + ((size_t)(C + 8) * 2 + 15) / 16 * 16;
    static bool cattr[64] = {};
    if (dev >= 0 && dev < 64 && !cattr[dev]) {
      // the largest request of any vocabulary the kernel takes (V = 65535)
      constexpr int kCMax = 256 * ((kTkMaxVocab + 256 * kTkCluster - 1) / (256 * kTkCluster));
      constexpr size_t kMaxSmem = kTkHistBytes + (size_t)kCMax * 4 + ((size_t)(kCMax + 8) * 2 + 15) / 16 * 16;
      static_assert((size_t)kCMax * 4 >= (size_t)(kTopkBins + 2) * 2, "list fits the exponentials");
      if (cudaFuncSetAttribute(topk_sample_cluster_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxSmem) !=
          cudaSuccess)
        return W8A8_ERR_CUDA;
      cattr[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(M * kTkCluster);
    cfg.blockDim = dim3(kTkThreads);
    cfg.dynamicSmemBytes = csmem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kTkCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    if (cudaLaunchKernelEx(&cfg, topk_sample_cluster_kernel, logits, ldl, V, C, ebytes, inv_temp, k, rnd,
                           rnd_stride, rnd_pos, out, append_to, append_stride, append_pos,
                           probs_out, ldp) != cudaSuccess) {
      cudaGetLastError();
      return W8A8_ERR_CUDA;
    }
    return check_launch("topk_sample_cluster");
  }
  launch_pdl(topk_sample_kernel, dim3(M), dim3(kTopkThreads), smem, s, logits, ldl, V, inv_temp,
             k, rnd, rnd_stride, rnd_pos, out, append_to, append_stride, append_pos, probs_out,
             ldp);
  return check_launch("topk_sample");
}

}  // namespace w8a8
