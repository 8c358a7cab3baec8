// HBM-streaming INT8 GEMV for decode (the engine sends it single tokens; the
// API takes up to 16) and the CUDA-core fallback for shapes the TMA path
// cannot take (K % 16 != 0, unaligned rows).
//
// One warp owns one output channel n: it holds W[n, :] in registers (16-byte
// loads, all in flight at once), multiplies against the token rows with dp4a,
// and reduces across lanes. A block holds 4 warps; the grid covers N/4
// blocks, so even the 768-row projections of GPT-2 small spread over more
// blocks than the B200 has SMs. Single tokens with rows longer than 2048
// bytes take 16-warp CTAs, one per SM (gemv_i8_rows_kernel). Exact integer
// accumulation: results are identical to the tensor-core path, and the same
// fused epilogues apply.
#include "common.cuh"
#include "epilogue.cuh"
#include "kernels.cuh"
#include "rowblock.cuh"
#include "runtime.cuh"

namespace w8a8 {

typedef LinearArgs GemvArgs;

constexpr int kGemvWarps = 4;

// Stores output (m, n); returns the stored bf16 value as a float (0 for
// int32 outputs). sX: the per-token scales (a.sX, or the kernel's own).
__device__ __forceinline__ float gemv_store(const GemvArgs &a, const float *sX, int m, int n,
                                           int32_t acc) {
  float sw = (a.epi != 0) ? a.sW[n] : 0.f;
  float sx = (a.epi != 0) ? sX[m] : 0.f;
  uint16_t *yp = reinterpret_cast<uint16_t *>(a.Y) + (int64_t)m * a.ldy + n;
  switch (a.epi) {
    case 0:
      s32_row(a, m)[n] = acc;
      return 0.0f;
    case 1:
      *yp = f2bf(dequant_bf(acc, sw, sx));
      return bf2f(*yp);
    case 2:
      *yp = f2bf(__fadd_rn(dequant_bf(acc, sw, sx), bf2f(a.bias[n])));
      return bf2f(*yp);
    case 3: {
      float y = add_bf(dequant_bf(acc, sw, sx), bf2f(a.bias[n]));
      float r = bf2f(a.R[(int64_t)m * a.ldr + n]);
      *yp = f2bf(__fadd_rn(r, y));
      return bf2f(*yp);
    }
    case 4: {
      float y = add_bf(dequant_bf(acc, sw, sx), bf2f(a.bias[n]));
      *yp = f2bf(gelu_tanh(y));
      return bf2f(*yp);
    }
    default: {  // QKV scatter
      uint16_t v = f2bf(__fadd_rn(dequant_bf(acc, sw, sx), bf2f(a.bias[n])));
      int seg = n / a.dseg, col = n - (n / a.dseg) * a.dseg;
      if (seg == 0) {
        reinterpret_cast<uint16_t *>(a.Y)[(int64_t)m * a.ldy + col] = v;
      } else {
        int b = m / a.T, t = m - (m / a.T) * a.T;
        int p = (a.pos0 ? a.pos0[b] : 0) + t;
        uint16_t *base = seg == 1 ? a.Kc : a.Vc;
        base[(int64_t)b * a.seq_stride + (int64_t)p * a.dseg + col] = v;
      }
      return bf2f(v);
    }
  }
}

// Vector path: K % 16 == 0 and 16-byte aligned rows. Lane l of the warp
// owning channel n holds the 16-byte weight vectors l + 32u (u < NVL) of
// W[n, :] in registers. The weights do not depend on the previous kernel, so
// they are requested before waiting for it (programmatic dependent launch):
// the weight stream overlaps the previous kernel's tail, and only the small
// activation rows (L2-resident, shared by the block's warps through L1) are
// read after the wait. AMAX: the block also writes its row maxima of |Y|
// (the row absmax record, one part per block).
template <int MT, int NVL, bool AMAX>
__global__ void __launch_bounds__(kGemvWarps * 32)
    gemv_i8_vec_kernel(const int8_t *__restrict__ X, int64_t ldx, const int8_t *__restrict__ W,
                       GemvArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x * kGemvWarps + warp;
  const int kv = a.K >> 4;  // 16-byte vectors per row
  __shared__ unsigned s_amax[AMAX ? MT : 1];
  if (AMAX) {
    if (threadIdx.x < MT) s_amax[threadIdx.x] = 0u;
    __syncthreads();
  }
  int4 w[NVL];
  const int4 *wrow = reinterpret_cast<const int4 *>(W + (int64_t)n * a.K);
#pragma unroll
  for (int u = 0; u < NVL; ++u) {
    const int v = lane + 32 * u;
    w[u] = (n < a.N && v < kv) ? __ldg(wrow + v) : make_int4(0, 0, 0, 0);
  }
  pdl_wait();
  pdl_launch_dependents();
  if (!AMAX && n >= a.N) return;
  int acc[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) acc[m] = 0;
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    if (m < a.M) {
      const int4 *xrow = reinterpret_cast<const int4 *>(X + (int64_t)m * ldx);
#pragma unroll
      for (int u = 0; u < NVL; ++u) {
        const int v = lane + 32 * u;
        if (v < kv) {
          const int4 x = __ldg(xrow + v);
          acc[m] = __dp4a(w[u].x, x.x, acc[m]);
          acc[m] = __dp4a(w[u].y, x.y, acc[m]);
          acc[m] = __dp4a(w[u].z, x.z, acc[m]);
          acc[m] = __dp4a(w[u].w, x.w, acc[m]);
        }
      }
    }
  }
#pragma unroll
  for (int m = 0; m < MT; ++m) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
  }
  // lane m stores token m (spreads the epilogue over the warp)
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    if (lane == m && m < a.M && n < a.N) {
      const float y = gemv_store(a, a.sX, m, n, acc[m]);
      if (AMAX) atomicMax(&s_amax[m], __float_as_uint(fabsf(y)));
    }
  }
  if (AMAX) {
    __syncthreads();
    if ((int)threadIdx.x < a.M)
      a.amax_out[(int64_t)blockIdx.x * a.M + threadIdx.x] = __uint_as_float(s_amax[threadIdx.x]);
  }
}

// Batch-1 decode with the LayerNorm folded in: every 4-warp block (128
// threads, the block-per-row LayerNorm's width) forms the token's LayerNorm
// and per-token quantization itself, from the bf16 row, with the reference's
// 1024-slot sums and fold (rowblock.cuh: the arithmetic of
// layernorm_block_kernel, bit for bit), keeps the int8 row in shared memory
// and runs the GEMV of gemv_i8_vec_kernel on it, two output channels a warp
// (half the blocks, so half the repeated LayerNorms, and one wave of blocks
// for GPT-2 large's W1: 640 blocks of 91 registers a thread, 5 per SM). Block 0 also writes the
// quantized row and its scale out. The weights and the LayerNorm's gain and
// bias do not depend on the previous kernel: they are requested before
// waiting for it. Replaces a LayerNorm launch and the quantized row's round
// trip through memory in every layer of a single-sequence decode step.
constexpr int kLnVec = 2;   // rows up to 128 threads x 2 vectors x 8 = 2048 elements
constexpr int kLnRows = 2;  // output channels a warp

template <int NVL, bool AMAX>
__global__ void __launch_bounds__(kGemvWarps * 32)
    gemv_ln_i8_kernel(const int8_t *__restrict__ W, GemvArgs a, GemvLnArgs ln) {
  static_assert(kGemvWarps * 32 == kRowThreads, "one LayerNorm block per GEMV block");
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int n0 = (blockIdx.x * kGemvWarps + warp) * kLnRows;  // channels n0, n0 + 1
  const int kv = a.K >> 4, nv = a.K >> 3;
  __shared__ RowShared sh;
  __shared__ __align__(16) int8_t xq[kLnVec * kRowThreads * 8];
  __shared__ float sx;
  __shared__ unsigned s_amax;
  if (AMAX && t == 0) s_amax = 0u;  // published by the LayerNorm's barriers
  int4 w[kLnRows][NVL];
#pragma unroll
  for (int j = 0; j < kLnRows; ++j) {
    const int n = n0 + j;
    const int4 *wrow = reinterpret_cast<const int4 *>(W + (int64_t)n * a.K);
#pragma unroll
    for (int u = 0; u < NVL; ++u) {
      const int v = lane + 32 * u;
      w[j][u] = (n < a.N && v < kv) ? __ldg(wrow + v) : make_int4(0, 0, 0, 0);
    }
  }
  uint4 g[kLnVec], bt[kLnVec];
  load_row_vec(ln.gamma, nv, t, g);
  load_row_vec(ln.beta, nv, t, bt);
  pdl_wait();
  pdl_launch_dependents();
  uint4 x[kLnVec];
  load_row_vec(ln.X, nv, t, x);
  ln_quant_tail(sh, x, g, bt, nv, t, a.K, ln.eps, nullptr, xq, &sx);
  __syncthreads();
  if (blockIdx.x == 0) {
    if (t < kv) reinterpret_cast<int4 *>(ln.Xq)[t] = reinterpret_cast<const int4 *>(xq)[t];
    if (t == 0) *ln.sX = sx;
  }
  int acc[kLnRows];
#pragma unroll
  for (int j = 0; j < kLnRows; ++j) acc[j] = 0;
  const int4 *xr = reinterpret_cast<const int4 *>(xq);
#pragma unroll
  for (int u = 0; u < NVL; ++u) {
    const int v = lane + 32 * u;
    if (v < kv) {
      const int4 q = xr[v];
#pragma unroll
      for (int j = 0; j < kLnRows; ++j) {
        acc[j] = __dp4a(w[j][u].x, q.x, acc[j]);
        acc[j] = __dp4a(w[j][u].y, q.y, acc[j]);
        acc[j] = __dp4a(w[j][u].z, q.z, acc[j]);
        acc[j] = __dp4a(w[j][u].w, q.w, acc[j]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < kLnRows; ++j) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
  }
  // lane j stores channel n0 + j
#pragma unroll
  for (int j = 0; j < kLnRows; ++j) {
    if (lane == j && n0 + j < a.N) {
      const float y = gemv_store(a, &sx, 0, n0 + j, acc[j]);
      if (AMAX) atomicMax(&s_amax, __float_as_uint(fabsf(y)));
    }
  }
  if (AMAX) {
    __syncthreads();
    if (t == 0) a.amax_out[blockIdx.x] = __uint_as_float(s_amax);
  }
}

// Single-token path for long rows (M == 1, K > 2048: the W2 projection of a
// batch-1 decode step): one CTA of 16 warps per SM, each CTA owning a
// contiguous run of output channels and each warp RPW of them (rows warp,
// warp + 16, ...). Every warp requests all of its weight rows (16-byte loads
// into registers) before waiting for the previous kernel, so the GEMV's
// weight stream is in flight during that kernel's tail (programmatic
// dependent launch).
//
// FROM_BF16: the token row arrives as bf16 (a.Xb) with the row absmax record
// (a.amax_in, a.n_part parts); the CTA quantizes it once into shared memory
// with the reference's per-token rule (cuda/activation_quant.cu:37-110).
constexpr int kRowsWarps = 16;
constexpr int kRowsMaxK = 16 * 32 * 16;  // NVL <= 16 vectors of 16 bytes a lane

template <int NVL, int RPW, bool FROM_BF16>
__global__ void __launch_bounds__(kRowsWarps * 32)
    gemv_i8_rows_kernel(const int8_t *__restrict__ X, const int8_t *__restrict__ W, GemvArgs a,
                        int rows) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * rows;
  const int n_end = min(n0 + rows, a.N);
  const int kv = a.K >> 4;
  int4 w[RPW][NVL];
#pragma unroll
  for (int i = 0; i < RPW; ++i) {
    const int n = n0 + warp + kRowsWarps * i;
    const int4 *wrow = reinterpret_cast<const int4 *>(W + (int64_t)n * a.K);
#pragma unroll
    for (int u = 0; u < NVL; ++u) {
      const int v = lane + 32 * u;
      w[i][u] = (n < n_end && v < kv) ? __ldg(wrow + v) : make_int4(0, 0, 0, 0);
    }
  }
  pdl_wait();
  pdl_launch_dependents();
  __shared__ __align__(16) int8_t xs[FROM_BF16 ? kRowsMaxK : 16];
  __shared__ float s_red[kRowsWarps];
  __shared__ float s_sx[1];
  if (FROM_BF16) {
    constexpr int kT = kRowsWarps * 32;
    constexpr int kU = kRowsMaxK / 16 / kT;  // 16-element units per thread
    uint4 xb[kU][2];
#pragma unroll
    for (int j = 0; j < kU; ++j) {  // the row's loads first: they overlap the maxima
      const int u = (int)threadIdx.x + j * kT;
      if (u * 16 < a.K) {
        const uint4 *src = reinterpret_cast<const uint4 *>(a.Xb + 16 * u);
        xb[j][0] = src[0];
        xb[j][1] = src[1];
      }
    }
    // the record's parts: the first 4 per thread in flight together
    float pv[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int p = (int)threadIdx.x + j * kT;
      pv[j] = p < a.n_part ? a.amax_in[p] : 0.0f;
    }
    float mx = fmaxf(fmaxf(pv[0], pv[1]), fmaxf(pv[2], pv[3]));
    for (int p = (int)threadIdx.x + 4 * kT; p < a.n_part; p += kT) mx = fmaxf(mx, a.amax_in[p]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) s_red[warp] = mx;
    __syncthreads();
    mx = s_red[0];
#pragma unroll
    for (int i = 1; i < kRowsWarps; ++i) mx = fmaxf(mx, s_red[i]);
    const float sc = quant_scale(mx), inv = __fdiv_rn(1.0f, sc);
    if (threadIdx.x == 0) s_sx[0] = sc;
#pragma unroll
    for (int j = 0; j < kU; ++j) {
      const int u = (int)threadIdx.x + j * kT;
      if (u * 16 < a.K) *reinterpret_cast<uint4 *>(xs + 16 * u) = quant16(xb[j][0], xb[j][1], inv);
    }
    __syncthreads();
  }
  int4 x[NVL];
#pragma unroll
  for (int u = 0; u < NVL; ++u) {
    const int v = lane + 32 * u;
    if (FROM_BF16)
      x[u] = v < kv ? reinterpret_cast<const int4 *>(xs)[v] : make_int4(0, 0, 0, 0);
    else
      x[u] = v < kv ? __ldg(reinterpret_cast<const int4 *>(X) + v) : make_int4(0, 0, 0, 0);
  }
#pragma unroll
  for (int i = 0; i < RPW; ++i) {
    const int n = n0 + warp + kRowsWarps * i;
    int acc = 0;
#pragma unroll
    for (int u = 0; u < NVL; ++u) {
      acc = __dp4a(w[i][u].x, x[u].x, acc);
      acc = __dp4a(w[i][u].y, x[u].y, acc);
      acc = __dp4a(w[i][u].z, x[u].z, acc);
      acc = __dp4a(w[i][u].w, x[u].w, acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0 && n < n_end) gemv_store(a, FROM_BF16 ? s_sx : a.sX, 0, n, acc);
  }
}

// Scalar fallback for any K / alignment (correctness path, not a hot path).
__global__ void gemv_i8_scalar_kernel(const int8_t *__restrict__ X, int64_t ldx,
                                      const int8_t *__restrict__ W, GemvArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x * kGemvWarps + warp;
  const int m = blockIdx.y;
  if (n >= a.N || m >= a.M) return;
  int acc = 0;
  for (int k = lane; k < a.K; k += 32)
    acc += (int)X[(int64_t)m * ldx + k] * (int)W[(int64_t)n * a.K + k];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) gemv_store(a, a.sX, m, n, acc);
}

template <int MT, int NVL, bool AMAX = false>
static int launch_vec(const int8_t *X, int64_t ldx, const int8_t *W, const GemvArgs &a,
                      cudaStream_t s) {
  dim3 grid((a.N + kGemvWarps - 1) / kGemvWarps);
  launch_pdl(gemv_i8_vec_kernel<MT, NVL, AMAX>, dim3(grid), dim3(kGemvWarps * 32), 0, s, X, ldx,
             W, a);
  return check_launch("gemv_i8_vec");
}

template <int MT>
static int launch_vec_k(const int8_t *X, int64_t ldx, const int8_t *W, const GemvArgs &a,
                        cudaStream_t s) {
  const int nvl = ((a.K >> 4) + 31) / 32;  // weight vectors per lane
  if (nvl <= 2) return launch_vec<MT, 2>(X, ldx, W, a, s);
  if (nvl <= 4) return launch_vec<MT, 4>(X, ldx, W, a, s);
  if (nvl <= 8) return launch_vec<MT, 8>(X, ldx, W, a, s);
  if (nvl <= 16) return launch_vec<MT, 16>(X, ldx, W, a, s);
  return W8A8_ERR_UNSUPPORTED;
}

template <int NVL, int RPW, bool FROM_BF16 = false>
static int launch_rows(const int8_t *X, const int8_t *W, const GemvArgs &a, int rows,
                       cudaStream_t s) {
  const int grid = (a.N + rows - 1) / rows;
  launch_pdl(gemv_i8_rows_kernel<NVL, RPW, FROM_BF16>, dim3(grid), dim3(kRowsWarps * 32), 0, s,
             X, W, a, rows);
  return check_launch("gemv_i8_rows");
}

// rows per warp (1..3) x 16-byte weight vectors per lane per row (K / 512,
// rounded up): a lane holds at most 16 weight vectors (128 registers a
// thread with 512 threads a CTA, without spilling)
template <int NVL, bool FROM_BF16 = false>
static int launch_rows_k(const int8_t *X, const int8_t *W, const GemvArgs &a, int rows,
                         cudaStream_t s) {
  const int rpw = (rows + kRowsWarps - 1) / kRowsWarps;
  if (rpw <= 1) return launch_rows<NVL, 1, FROM_BF16>(X, W, a, rows, s);
  if (rpw <= 2 && NVL <= 8)
    return launch_rows<NVL, (NVL <= 8 ? 2 : 1), FROM_BF16>(X, W, a, rows, s);
  return W8A8_ERR_UNSUPPORTED;
}

int launch_gemv_i8(const int8_t *X, int64_t ldx, const int8_t *W, const GemvArgs &a,
                   cudaStream_t s) {
  const bool vec = (a.K % 16 == 0) && (ldx % 16 == 0) && aligned16(X) && aligned16(W);
  if (vec && a.M == 1) {
    int st;
    DeviceCtx *ctx = device_ctx(&st);
    if (!ctx) return st;
    // Long rows (K > 2048) only: measured on GPT-2 large, W2 (1280 x 5120)
    // takes 5.1 us this way against 7.0 us with 4-warp blocks, while the
    // K = 1280 projections are faster with the 4-warp blocks below.
    const int rows = (a.N + ctx->sm_count - 1) / ctx->sm_count;  // one CTA per SM
    const int nvl = ((a.K >> 4) + 31) / 32;
    int r = W8A8_ERR_UNSUPPORTED;
    if (nvl > 4 && nvl <= 8) r = launch_rows_k<8>(X, W, a, rows, s);
    else if (nvl > 8 && nvl <= 16) r = launch_rows_k<16>(X, W, a, rows, s);
    if (r != W8A8_ERR_UNSUPPORTED) return r;
  }
  if (vec && a.M <= 16 && a.K <= 16 * 32 * 16) {
    if (a.M <= 1) return launch_vec_k<1>(X, ldx, W, a, s);
    if (a.M <= 2) return launch_vec_k<2>(X, ldx, W, a, s);
    if (a.M <= 4) return launch_vec_k<4>(X, ldx, W, a, s);
    if (a.M <= 8) return launch_vec_k<8>(X, ldx, W, a, s);
    return launch_vec_k<16>(X, ldx, W, a, s);
  }
  if (a.M > 65535) return W8A8_ERR_UNSUPPORTED;
  dim3 grid((a.N + kGemvWarps - 1) / kGemvWarps, a.M);
  launch_pdl(gemv_i8_scalar_kernel, dim3(grid), dim3(kGemvWarps * 32), 0, s, X, ldx, W, a);
  return check_launch("gemv_i8_scalar");
}

// One token through the 4-warp GEMV with the row absmax record (one part per
// block); W8A8_ERR_UNSUPPORTED where another kernel would run.
int gemv_absmax(const int8_t *X, int64_t ldx, const int8_t *W, const GemvArgs &a, int *n_part,
                cudaStream_t s) {
  const bool vec = (a.K % 16 == 0) && (ldx % 16 == 0) && aligned16(X) && aligned16(W);
  if (!vec || a.M != 1 || !a.amax_out || a.epi == EPI_S32) return W8A8_ERR_UNSUPPORTED;
  int st;
  DeviceCtx *ctx = device_ctx(&st);
  if (!ctx) return st;
  const int nvl = ((a.K >> 4) + 31) / 32;
  if (nvl > 4) return W8A8_ERR_UNSUPPORTED;  // long rows take the 16-warp kernel
  *n_part = (a.N + kGemvWarps - 1) / kGemvWarps;
  if (nvl <= 2) return launch_vec<1, 2, true>(X, ldx, W, a, s);
  return launch_vec<1, 4, true>(X, ldx, W, a, s);
}

// One token whose LayerNorm the GEMV forms itself (gemv_ln_i8_kernel); with
// a.amax_out, also the row absmax record (*n_part parts). K <= 2048, K % 16 == 0.
// W8A8_ERR_UNSUPPORTED where the operands do not allow it.
int gemv_layernorm(const int8_t *W, const GemvArgs &a, const GemvLnArgs &ln, int *n_part,
                   cudaStream_t s) {
  if (a.M != 1 || a.K % 16 || a.K > kLnVec * kRowThreads * 8 || a.epi == EPI_S32 || !ln.X ||
      !ln.gamma || !ln.beta || !ln.Xq || !ln.sX || !aligned16(W) || !aligned16(ln.X) ||
      !aligned16(ln.gamma) || !aligned16(ln.beta) || !aligned16(ln.Xq))
    return W8A8_ERR_UNSUPPORTED;
  const int grid = (a.N + kGemvWarps * kLnRows - 1) / (kGemvWarps * kLnRows);
  const int nvl = ((a.K >> 4) + 31) / 32;  // <= 4
  if (a.amax_out) {
    if (n_part) *n_part = grid;
    if (nvl <= 2) launch_pdl(gemv_ln_i8_kernel<2, true>, dim3(grid), dim3(kGemvWarps * 32), 0, s, W, a, ln);
    else launch_pdl(gemv_ln_i8_kernel<4, true>, dim3(grid), dim3(kGemvWarps * 32), 0, s, W, a, ln);
  } else {
    if (nvl <= 2) launch_pdl(gemv_ln_i8_kernel<2, false>, dim3(grid), dim3(kGemvWarps * 32), 0, s, W, a, ln);
    else launch_pdl(gemv_ln_i8_kernel<4, false>, dim3(grid), dim3(kGemvWarps * 32), 0, s, W, a, ln);
  }
  return check_launch("gemv_ln_i8");
}

// One token with a long bf16 row (K > 2048) through the 16-warp GEMV that
// quantizes the row itself; W8A8_ERR_UNSUPPORTED elsewhere.
int gemv_from_bf16(const int8_t *W, const GemvArgs &a, cudaStream_t s) {
  if (a.M != 1 || !a.Xb || !a.amax_in || a.n_part < 1 || a.K % 16 || a.K > kRowsMaxK ||
      !aligned16(a.Xb) || !aligned16(W) || a.epi == EPI_S32)
    return W8A8_ERR_UNSUPPORTED;
  int st;
  DeviceCtx *ctx = device_ctx(&st);
  if (!ctx) return st;
  const int rows = (a.N + ctx->sm_count - 1) / ctx->sm_count;
  const int nvl = ((a.K >> 4) + 31) / 32;
  if (nvl > 4 && nvl <= 8) return launch_rows_k<8, true>(nullptr, W, a, rows, s);
  if (nvl > 8 && nvl <= 16) return launch_rows_k<16, true>(nullptr, W, a, rows, s);
  return W8A8_ERR_UNSUPPORTED;
}

}  // namespace w8a8
