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
#include "runtime.cuh"

namespace w8a8 {

typedef LinearArgs GemvArgs;

constexpr int kGemvWarps = 4;

__device__ __forceinline__ void gemv_store(const GemvArgs &a, int m, int n, int32_t acc) {
  float sw = (a.epi != 0) ? a.sW[n] : 0.f;
  float sx = (a.epi != 0) ? a.sX[m] : 0.f;
  switch (a.epi) {
    case 0:
      s32_row(a, m)[n] = acc;
      break;
    case 1:
      reinterpret_cast<uint16_t *>(a.Y)[(int64_t)m * a.ldy + n] = f2bf(dequant_bf(acc, sw, sx));
      break;
    case 2:
      reinterpret_cast<uint16_t *>(a.Y)[(int64_t)m * a.ldy + n] =
          f2bf(__fadd_rn(dequant_bf(acc, sw, sx), bf2f(a.bias[n])));
      break;
    case 3: {
      float y = add_bf(dequant_bf(acc, sw, sx), bf2f(a.bias[n]));
      float r = bf2f(a.R[(int64_t)m * a.ldr + n]);
      reinterpret_cast<uint16_t *>(a.Y)[(int64_t)m * a.ldy + n] = f2bf(__fadd_rn(r, y));
      break;
    }
    case 4: {
      float y = add_bf(dequant_bf(acc, sw, sx), bf2f(a.bias[n]));
      reinterpret_cast<uint16_t *>(a.Y)[(int64_t)m * a.ldy + n] = f2bf(gelu_tanh(y));
      break;
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
      break;
    }
  }
}

// Vector path: K % 16 == 0 and 16-byte aligned rows. Lane l of the warp
// owning channel n holds the 16-byte weight vectors l + 32u (u < NVL) of
// W[n, :] in registers. The weights do not depend on the previous kernel, so
// they are requested before waiting for it (programmatic dependent launch):
// the weight stream overlaps the previous kernel's tail, and only the small
// activation rows (L2-resident, shared by the block's warps through L1) are
// read after the wait.
template <int MT, int NVL>
__global__ void __launch_bounds__(kGemvWarps * 32)
    gemv_i8_vec_kernel(const int8_t *__restrict__ X, int64_t ldx, const int8_t *__restrict__ W,
                       GemvArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x * kGemvWarps + warp;
  const int kv = a.K >> 4;  // 16-byte vectors per row
  int4 w[NVL];
  if (n < a.N) {
    const int4 *wrow = reinterpret_cast<const int4 *>(W + (int64_t)n * a.K);
#pragma unroll
    for (int u = 0; u < NVL; ++u) {
      const int v = lane + 32 * u;
      w[u] = v < kv ? __ldg(wrow + v) : make_int4(0, 0, 0, 0);
    }
  }
  pdl_wait();
  pdl_launch_dependents();
  if (n >= a.N) return;
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
  for (int m = 0; m < MT; ++m)
    if (lane == m && m < a.M) gemv_store(a, m, n, acc[m]);
}

// Single-token path for long rows (M == 1, K > 2048: the W2 projection of a
// batch-1 decode step): one CTA of 16 warps per SM, each CTA owning a
// contiguous run of output channels and each warp RPW of them (rows warp,
// warp + 16, ...). Every warp requests all of its weight rows (16-byte loads
// into registers) before waiting for the previous kernel, so the GEMV's
// weight stream is in flight during that kernel's tail (programmatic
// dependent launch).
constexpr int kRowsWarps = 16;

template <int NVL, int RPW>
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
  int4 x[NVL];
  const int4 *xrow = reinterpret_cast<const int4 *>(X);
#pragma unroll
  for (int u = 0; u < NVL; ++u) {
    const int v = lane + 32 * u;
    x[u] = v < kv ? __ldg(xrow + v) : make_int4(0, 0, 0, 0);
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
    if (lane == 0 && n < n_end) gemv_store(a, 0, n, acc);
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
  if (lane == 0) gemv_store(a, m, n, acc);
}

template <int MT, int NVL>
static int launch_vec(const int8_t *X, int64_t ldx, const int8_t *W, const GemvArgs &a,
                      cudaStream_t s) {
  dim3 grid((a.N + kGemvWarps - 1) / kGemvWarps);
  launch_pdl(gemv_i8_vec_kernel<MT, NVL>, dim3(grid), dim3(kGemvWarps * 32), 0, s, X, ldx, W, a);
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

template <int NVL, int RPW>
static int launch_rows(const int8_t *X, const int8_t *W, const GemvArgs &a, int rows,
                       cudaStream_t s) {
  const int grid = (a.N + rows - 1) / rows;
  launch_pdl(gemv_i8_rows_kernel<NVL, RPW>, dim3(grid), dim3(kRowsWarps * 32), 0, s, X, W, a,
             rows);
  return check_launch("gemv_i8_rows");
}

// rows per warp (1..3) x 16-byte weight vectors per lane per row (K / 512,
// rounded up): a lane holds at most 16 weight vectors (128 registers a
// thread with 512 threads a CTA, without spilling)
template <int NVL>
static int launch_rows_k(const int8_t *X, const int8_t *W, const GemvArgs &a, int rows,
                         cudaStream_t s) {
  const int rpw = (rows + kRowsWarps - 1) / kRowsWarps;
  if (rpw <= 1) return launch_rows<NVL, 1>(X, W, a, rows, s);
  if (rpw <= 2 && NVL <= 8) return launch_rows<NVL, (NVL <= 8 ? 2 : 1)>(X, W, a, rows, s);
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

}  // namespace w8a8
