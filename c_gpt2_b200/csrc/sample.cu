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
  launch_pdl(topk_sample_kernel, dim3(M), dim3(kTopkThreads), smem, s, logits, ldl, V, inv_temp,
             k, rnd, rnd_stride, rnd_pos, out, append_to, append_stride, append_pos, probs_out,
             ldp);
  return check_launch("topk_sample");
}

}  // namespace w8a8
