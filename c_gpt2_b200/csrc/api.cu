// extern "C" entry points of include/gpt2_w8a8.h: argument validation and
// dispatch between the tensor-core and CUDA-core kernels.
#include "common.cuh"
#include "kernels.cuh"
#include "runtime.cuh"

namespace w8a8 {

// Smallest token count that takes the tensor-core path. A single token takes
// the weight-streaming GEMV; from two tokens on, the cluster split-K GEMM
// (tokens padded to the MMA's N = 32, zero rows from TMA's out-of-bounds fill)
// is faster than a GEMV that re-reads the token rows per output channel.
constexpr int kTcMinM = 2;

static bool tc_ok_i8(const void *X, int64_t ldx, const void *W, int K) {
  return (K % 16 == 0) && (ldx % 16 == 0) && aligned16(X) && aligned16(W);
}

static int dispatch_linear(const int8_t *Xq, int64_t ldx, const int8_t *W, const LinearArgs &a,
                           cudaStream_t s) {
  if (a.M >= kTcMinM && tc_ok_i8(Xq, ldx, W, a.K)) return gemm_tc_i8(W, Xq, ldx, a, s);
  return launch_gemv_i8(Xq, ldx, W, a, s);
}

static LinearArgs make_args(int epi, int M, int N, int K, const float *sX, const float *sW,
                            const uint16_t *bias, const uint16_t *R, int64_t ldr, void *Y,
                            int64_t ldy) {
  LinearArgs a = {};
  a.M = M;
  a.N = N;
  a.K = K;
  a.epi = epi;
  a.sX = sX;
  a.sW = sW;
  a.bias = bias;
  a.R = R;
  a.ldr = ldr;
  a.Y = Y;
  a.ldy = ldy;
  a.T = 1;
  a.dseg = N;
  return a;
}

}  // namespace w8a8

using namespace w8a8;

static int ready(void) {
  int st;
  return device_ctx(&st) ? W8A8_OK : st;
}

extern "C" int w8a8_quant_rows(const gpt2_bf16_t *X, int64_t ldx, int M, int K, int8_t *Xq,
                               float *sX, void *stream) {
  if (M == 0) return W8A8_OK;
  if (!X || !Xq || !sX || M < 0 || K <= 0 || ldx < K) return W8A8_ERR_INVALID;
  int st = ready();
  if (st) return st;
  return launch_quant_rows(X, ldx, M, K, Xq, sX, (cudaStream_t)stream);
}

extern "C" int w8a8_layernorm_quant(const gpt2_bf16_t *X, int64_t ldx, int M, int d,
                                    const gpt2_bf16_t *gamma, const gpt2_bf16_t *beta, float eps,
                                    gpt2_bf16_t *Y, int64_t ldy, int8_t *Xq, float *sX,
                                    void *stream) {
  if (M == 0) return W8A8_OK;
  if (!X || !gamma || !beta || M < 0 || d <= 0 || d > 8192 || ldx < d) return W8A8_ERR_INVALID;
  if (!Y && !Xq) return W8A8_ERR_INVALID;
  if (Y && ldy < d) return W8A8_ERR_INVALID;
  if ((Xq == nullptr) != (sX == nullptr)) return W8A8_ERR_INVALID;
  int st = ready();
  if (st) return st;
  return launch_layernorm_quant(X, ldx, M, d, gamma, beta, eps, Y, ldy, Xq, sX,
                                (cudaStream_t)stream);
}

extern "C" int w8a8_embed_layernorm_quant(const gpt2_bf16_t *wte, const gpt2_bf16_t *wpe,
                                          const int32_t *tokens, int M, int T,
                                          const int32_t *pos0, int d, gpt2_bf16_t *H,
                                          const gpt2_bf16_t *gamma, const gpt2_bf16_t *beta,
                                          float eps, gpt2_bf16_t *Y, int8_t *Xq, float *sX,
                                          void *stream) {
  if (M == 0) return W8A8_OK;
  if (!wte || !wpe || !tokens || !gamma || !beta || M < 0 || T <= 0 || M % T != 0 || d <= 0 ||
      d > 8192)
    return W8A8_ERR_INVALID;
  if ((Xq == nullptr) != (sX == nullptr)) return W8A8_ERR_INVALID;
  int st = ready();
  if (st) return st;
  return launch_embed_layernorm_quant(wte, wpe, tokens, M, T, pos0, d, H, gamma, beta, eps, Y, Xq,
                                      sX, (cudaStream_t)stream);
}

extern "C" int w8a8_gemm_s32(const int8_t *Xq, int M, int K, const int8_t *W, int N, int32_t *Y,
                             void *stream) {
  if (M == 0 || N == 0) return W8A8_OK;
  if (!Xq || !W || !Y || M < 0 || N < 0 || K <= 0) return W8A8_ERR_INVALID;
  int st = ready();
  if (st) return st;
  LinearArgs a = make_args(EPI_S32, M, N, K, nullptr, nullptr, nullptr, nullptr, 0, Y, N);
  return dispatch_linear(Xq, K, W, a, (cudaStream_t)stream);
}

extern "C" int w8a8_linear(const int8_t *Xq, const float *sX, int M, int K, const int8_t *W,
                           const float *sW, const gpt2_bf16_t *bias, int N, int epilogue,
                           const gpt2_bf16_t *R, int64_t ldr, gpt2_bf16_t *Y, int64_t ldy,
                           void *workspace, size_t workspace_bytes, void *stream) {
  if (M == 0 || N == 0) return W8A8_OK;
  if (!Xq || !sX || !W || !sW || !Y || M < 0 || N < 0 || K <= 0 || ldy < N)
    return W8A8_ERR_INVALID;
  int epi;
  switch (epilogue) {
    case W8A8_EPI_DEQUANT: epi = EPI_DEQUANT; break;
    case W8A8_EPI_BIAS: epi = EPI_BIAS; break;
    case W8A8_EPI_BIAS_RESID: epi = EPI_RESID; break;
    case W8A8_EPI_BIAS_GELU: epi = EPI_GELU; break;
    default: return W8A8_ERR_INVALID;
  }
  if (epi != EPI_DEQUANT && !bias) return W8A8_ERR_INVALID;
  if (epi == EPI_RESID && (!R || ldr < N)) return W8A8_ERR_INVALID;
  int st = ready();
  if (st) return st;
  LinearArgs a = make_args(epi, M, N, K, sX, sW, bias, R, ldr, Y, ldy);
  a.workspace = workspace;
  a.workspace_bytes = workspace_bytes;
  return dispatch_linear(Xq, K, W, a, (cudaStream_t)stream);
}

static int epi_code(int epilogue, int *epi) {
  switch (epilogue) {
    case W8A8_EPI_DEQUANT: *epi = EPI_DEQUANT; return W8A8_OK;
    case W8A8_EPI_BIAS: *epi = EPI_BIAS; return W8A8_OK;
    case W8A8_EPI_BIAS_RESID: *epi = EPI_RESID; return W8A8_OK;
    case W8A8_EPI_BIAS_GELU: *epi = EPI_GELU; return W8A8_OK;
    default: return W8A8_ERR_INVALID;
  }
}

// Parts of a row absmax record: one per CTA of the fused kernels (at most
// one per 4 output channels), or 1 from the separate maxima kernel.
extern "C" size_t w8a8_absmax_record_floats(int M, int N) {
  if (M <= 0 || N <= 0) return 0;
  const size_t parts = (size_t)(N + 3) / 4;
  return (size_t)M * (parts > 1 ? parts : 1);
}

extern "C" int w8a8_linear_absmax(const int8_t *Xq, const float *sX, int M, int K,
                                  const int8_t *W, const float *sW, const gpt2_bf16_t *bias,
                                  int N, int epilogue, const gpt2_bf16_t *R, int64_t ldr,
                                  gpt2_bf16_t *Y, int64_t ldy, float *absmax,
                                  size_t absmax_floats, int *n_part, void *workspace,
                                  size_t workspace_bytes, void *stream) {
  if (!n_part) return W8A8_ERR_INVALID;
  *n_part = 0;
  if (M == 0 || N == 0) return W8A8_OK;
  if (!Xq || !sX || !W || !sW || !Y || !absmax || M < 0 || N < 0 || K <= 0 || ldy < N)
    return W8A8_ERR_INVALID;
  int epi;
  if (epi_code(epilogue, &epi)) return W8A8_ERR_INVALID;
  if (epi != EPI_DEQUANT && !bias) return W8A8_ERR_INVALID;
  if (epi == EPI_RESID && (!R || ldr < N)) return W8A8_ERR_INVALID;
  if (absmax_floats < w8a8_absmax_record_floats(M, N)) return W8A8_ERR_INVALID;
  int st = ready();
  if (st) return st;
  LinearArgs a = make_args(epi, M, N, K, sX, sW, bias, R, ldr, Y, ldy);
  a.workspace = workspace;
  a.workspace_bytes = workspace_bytes;
  a.amax_out = absmax;
  const cudaStream_t s = (cudaStream_t)stream;
  int parts = 0;
  st = M == 1 ? gemv_absmax(Xq, K, W, a, &parts, s) : W8A8_ERR_UNSUPPORTED;
  if (st == W8A8_OK) {
    *n_part = parts;
    return W8A8_OK;
  }
  if (st != W8A8_ERR_UNSUPPORTED) return st;
  // any other shape: the GEMM, then the maxima of its output rows
  a.amax_out = nullptr;
  st = dispatch_linear(Xq, K, W, a, s);
  if (st) return st;
  float *out[1] = {absmax};
  st = launch_row_amax(Y, ldy, M, N, out, 1, s);
  if (st == W8A8_OK) *n_part = 1;
  return st;
}

extern "C" int w8a8_linear_from_bf16(const gpt2_bf16_t *X, int64_t ldx, const float *absmax,
                                     int n_part, int M, int K, const int8_t *W, const float *sW,
                                     const gpt2_bf16_t *bias, int N, int epilogue,
                                     const gpt2_bf16_t *R, int64_t ldr, gpt2_bf16_t *Y,
                                     int64_t ldy, int8_t *Xq, float *sX, void *workspace,
                                     size_t workspace_bytes, void *stream) {
  if (M == 0 || N == 0) return W8A8_OK;
  if (!X || !absmax || n_part < 1 || !W || !sW || !Y || !Xq || !sX || M < 0 || N < 0 || K <= 0 ||
      K % 8 || ldx < K || ldy < N)
    return W8A8_ERR_INVALID;
  int epi;
  if (epi_code(epilogue, &epi)) return W8A8_ERR_INVALID;
  if (epi != EPI_DEQUANT && !bias) return W8A8_ERR_INVALID;
  if (epi == EPI_RESID && (!R || ldr < N)) return W8A8_ERR_INVALID;
  int st = ready();
  if (st) return st;
  LinearArgs a = make_args(epi, M, N, K, sX, sW, bias, R, ldr, Y, ldy);
  a.workspace = workspace;
  a.workspace_bytes = workspace_bytes;
  a.Xb = X;
  a.ldxb = ldx;
  a.amax_in = absmax;
  a.n_part = n_part;
  const cudaStream_t s = (cudaStream_t)stream;
  st = M == 1 ? gemv_from_bf16(W, a, s) : W8A8_ERR_UNSUPPORTED;
  if (st != W8A8_ERR_UNSUPPORTED) return st;
  // any other shape: the quantization kernel, then the GEMM on its rows
  st = launch_quant_rows_amax(X, ldx, M, K, absmax, n_part, M, Xq, K, sX, s);
  if (st) return st;
  a.Xb = nullptr;
  a.amax_in = nullptr;
  return dispatch_linear(Xq, K, W, a, s);
}

namespace w8a8 {

// Workspace bytes w8a8_linear would read for these operands given one: nonzero
// only where its dispatch ends in the channel-major tcgen05 GEMM split over K
// (a few tokens whose operands the cluster kernel cannot take). The GEMV, the
// token-major GEMM and the cluster GEMM read none. 0 for arguments that
// w8a8_linear refuses, which it then reports itself.
size_t linear_workspace_used(const int8_t *Xq, const float *sX, int M, int K, const int8_t *W,
                             const float *sW, const gpt2_bf16_t *bias, int N, int epilogue,
                             const gpt2_bf16_t *R, int64_t ldr, gpt2_bf16_t *Y, int64_t ldy) {
  int epi;
  switch (epilogue) {
    case W8A8_EPI_DEQUANT: epi = EPI_DEQUANT; break;
    case W8A8_EPI_BIAS: epi = EPI_BIAS; break;
    case W8A8_EPI_BIAS_RESID: epi = EPI_RESID; break;
    case W8A8_EPI_BIAS_GELU: epi = EPI_GELU; break;
    default: return 0;
  }
  if (M <= 0 || N <= 0 || K <= 0 || ready() != W8A8_OK) return 0;
  if (!(M >= kTcMinM && tc_ok_i8(Xq, K, W, K))) return 0;  // GEMV
  LinearArgs a = make_args(epi, M, N, K, sX, sW, bias, R, ldr, Y, ldy);
  return gemm_i8_workspace_used(Xq, K, a);
}

}  // namespace w8a8

extern "C" size_t w8a8_linear_workspace_size(int M, int N) {
  if (M <= 0 || N <= 0) return 0;
  return linear_workspace_bytes(M, N);
}

static int linear_qkv_impl(const int8_t *Xq, const float *sX, int M, int K, int dq,
                           const int8_t *Wqkv, const float *sWqkv, const gpt2_bf16_t *bqkv,
                           gpt2_bf16_t *Q, int64_t ldq, gpt2_bf16_t *Kc, gpt2_bf16_t *Vc,
                           int64_t seq_stride, int T, const int32_t *pos0, void *workspace,
                           size_t workspace_bytes, void *stream) {
  if (M == 0) return W8A8_OK;
  if (!Xq || !sX || !Wqkv || !sWqkv || !bqkv || !Q || !Kc || !Vc || M < 0 || K <= 0 ||
      dq <= 0 || T <= 0 || M % T != 0 || ldq < dq)
    return W8A8_ERR_INVALID;
  int st = ready();
  if (st) return st;
  LinearArgs a = make_args(EPI_QKV, M, 3 * dq, K, sX, sWqkv, bqkv, nullptr, 0, Q, ldq);
  a.Kc = Kc;
  a.Vc = Vc;
  a.seq_stride = seq_stride;
  a.T = T;
  a.pos0 = pos0;
  a.dseg = dq;
  a.workspace = workspace;
  a.workspace_bytes = workspace_bytes;
  return dispatch_linear(Xq, K, Wqkv, a, (cudaStream_t)stream);
}

extern "C" int w8a8_linear_qkv(const int8_t *Xq, const float *sX, int M, int d,
                               const int8_t *Wqkv, const float *sWqkv, const gpt2_bf16_t *bqkv,
                               gpt2_bf16_t *Q, int64_t ldq, gpt2_bf16_t *Kc, gpt2_bf16_t *Vc,
                               int64_t seq_stride, int T, const int32_t *pos0,
                               void *workspace, size_t workspace_bytes, void *stream) {
  return linear_qkv_impl(Xq, sX, M, d, d, Wqkv, sWqkv, bqkv, Q, ldq, Kc, Vc, seq_stride, T, pos0,
                         workspace, workspace_bytes, stream);
}

extern "C" int w8a8_linear_qkv_heads(const int8_t *Xq, const float *sX, int M, int K,
                                     int d_heads, const int8_t *Wqkv, const float *sWqkv,
                                     const gpt2_bf16_t *bqkv, gpt2_bf16_t *Q, int64_t ldq,
                                     gpt2_bf16_t *Kc, gpt2_bf16_t *Vc, int64_t seq_stride, int T,
                                     const int32_t *pos0, void *workspace,
                                     size_t workspace_bytes, void *stream) {
  if (d_heads % 32) return W8A8_ERR_INVALID;
  return linear_qkv_impl(Xq, sX, M, K, d_heads, Wqkv, sWqkv, bqkv, Q, ldq, Kc, Vc, seq_stride, T,
                         pos0, workspace, workspace_bytes, stream);
}

// LayerNorm folded into the single-token GEMV (gemv_layernorm), else the
// LayerNorm kernel followed by the linear layer on its quantized rows.
extern "C" int w8a8_layernorm_linear_qkv(const gpt2_bf16_t *X, int64_t ldx,
                                         const gpt2_bf16_t *gamma, const gpt2_bf16_t *beta,
                                         float eps, int8_t *Xq, float *sX, int M, int d,
                                         const int8_t *Wqkv, const float *sWqkv,
                                         const gpt2_bf16_t *bqkv, gpt2_bf16_t *Q, int64_t ldq,
                                         gpt2_bf16_t *Kc, gpt2_bf16_t *Vc, int64_t seq_stride,
                                         int T, const int32_t *pos0, void *workspace,
                                         size_t workspace_bytes, void *stream) {
  if (M == 0) return W8A8_OK;
  if (!X || !gamma || !beta || !Xq || !sX || !Wqkv || !sWqkv || !bqkv || !Q || !Kc || !Vc ||
      M < 0 || d <= 0 || d > 8192 || ldx < d || T <= 0 || M % T != 0 || ldq < d)
    return W8A8_ERR_INVALID;
  int st = ready();
  if (st) return st;
  if (M == 1) {
    LinearArgs a = make_args(EPI_QKV, M, 3 * d, d, sX, sWqkv, bqkv, nullptr, 0, Q, ldq);
    a.Kc = Kc;
    a.Vc = Vc;
    a.seq_stride = seq_stride;
    a.T = T;
    a.pos0 = pos0;
    a.dseg = d;
    const GemvLnArgs ln = {X, gamma, beta, eps, Xq, sX};
    st = gemv_layernorm(Wqkv, a, ln, nullptr, (cudaStream_t)stream);
    if (st != W8A8_ERR_UNSUPPORTED) return st;
  }
  st = w8a8_layernorm_quant(X, ldx, M, d, gamma, beta, eps, nullptr, 0, Xq, sX, stream);
  if (st) return st;
  return w8a8_linear_qkv(Xq, sX, M, d, Wqkv, sWqkv, bqkv, Q, ldq, Kc, Vc, seq_stride, T, pos0,
                         workspace, workspace_bytes, stream);
}

extern "C" int w8a8_layernorm_linear_absmax(const gpt2_bf16_t *X, int64_t ldx,
                                            const gpt2_bf16_t *gamma, const gpt2_bf16_t *beta,
                                            float eps, int8_t *Xq, float *sX, int M, int K,
                                            const int8_t *W, const float *sW,
                                            const gpt2_bf16_t *bias, int N, int epilogue,
                                            const gpt2_bf16_t *R, int64_t ldr, gpt2_bf16_t *Y,
                                            int64_t ldy, float *absmax, size_t absmax_floats,
                                            int *n_part, void *workspace,
                                            size_t workspace_bytes, void *stream) {
  if (!n_part) return W8A8_ERR_INVALID;
  *n_part = 0;
  if (M == 0 || N == 0) return W8A8_OK;
  if (!X || !gamma || !beta || !Xq || !sX || !W || !sW || !Y || !absmax || M < 0 || N < 0 ||
      K <= 0 || K > 8192 || ldx < K || ldy < N)
    return W8A8_ERR_INVALID;
  int epi;
  if (epi_code(epilogue, &epi)) return W8A8_ERR_INVALID;
  if (epi != EPI_DEQUANT && !bias) return W8A8_ERR_INVALID;
  if (epi == EPI_RESID && (!R || ldr < N)) return W8A8_ERR_INVALID;
  if (absmax_floats < w8a8_absmax_record_floats(M, N)) return W8A8_ERR_INVALID;
  int st = ready();
  if (st) return st;
  if (M == 1) {
    LinearArgs a = make_args(epi, M, N, K, sX, sW, bias, R, ldr, Y, ldy);
    a.amax_out = absmax;
    const GemvLnArgs ln = {X, gamma, beta, eps, Xq, sX};
    int parts = 0;
    st = gemv_layernorm(W, a, ln, &parts, (cudaStream_t)stream);
    if (st == W8A8_OK) *n_part = parts;
    if (st != W8A8_ERR_UNSUPPORTED) return st;
  }
  st = w8a8_layernorm_quant(X, ldx, M, K, gamma, beta, eps, nullptr, 0, Xq, sX, stream);
  if (st) return st;
  return w8a8_linear_absmax(Xq, sX, M, K, W, sW, bias, N, epilogue, R, ldr, Y, ldy, absmax,
                            absmax_floats, n_part, workspace, workspace_bytes, stream);
}

extern "C" int w8a8_row_amax(const gpt2_bf16_t *X, int64_t ldx, int M, int K, float *amax,
                             void *stream) {
  if (M == 0) return W8A8_OK;
  if (!X || !amax || M < 0 || K <= 0 || ldx < K) return W8A8_ERR_INVALID;
  int st = ready();
  if (st) return st;
  return launch_row_amax(X, ldx, M, K, &amax, 1, (cudaStream_t)stream);
}

extern "C" int w8a8_row_amax_to(const gpt2_bf16_t *X, int64_t ldx, int M, int K,
                                float *const *amax, int n_out, void *stream) {
  if (M == 0) return W8A8_OK;
  if (!X || !amax || M < 0 || K <= 0 || ldx < K || n_out < 1 || n_out > 8)
    return W8A8_ERR_INVALID;
  for (int j = 0; j < n_out; ++j)
    if (!amax[j]) return W8A8_ERR_INVALID;
  int st = ready();
  if (st) return st;
  return launch_row_amax(X, ldx, M, K, amax, n_out, (cudaStream_t)stream);
}

extern "C" int w8a8_quant_rows_amax(const gpt2_bf16_t *X, int64_t ldx, int M, int K,
                                    const float *amax, int n_amax, int64_t amax_stride,
                                    int8_t *Xq, int64_t ldq, float *sX, void *stream) {
  if (M == 0) return W8A8_OK;
  if (!X || !amax || !Xq || !sX || M < 0 || K <= 0 || ldx < K || ldq < K || n_amax <= 0 ||
      (n_amax > 1 && amax_stride < M))
    return W8A8_ERR_INVALID;
  int st = ready();
  if (st) return st;
  return launch_quant_rows_amax(X, ldx, M, K, amax, n_amax, amax_stride, Xq, ldq, sX,
                                (cudaStream_t)stream);
}

extern "C" int w8a8_reduce_residual_layernorm_quant_bcast(
    const int32_t *acc, int64_t lda, int n_slots, int64_t slot_stride, int M, int d,
    const float *sX, const float *sW, const gpt2_bf16_t *bias, const gpt2_bf16_t *R, int64_t ldr,
    gpt2_bf16_t *H, int64_t ldh, const gpt2_bf16_t *gamma, const gpt2_bf16_t *beta, float eps,
    int8_t *Xq, int64_t ldq, float *sXq, int8_t *const *xq_bcast, float *const *sx_bcast,
    int n_bcast, int64_t bcast_row0, void *stream) {
  if (M == 0) return W8A8_OK;
  if (!acc || !sX || !sW || !bias || !R || !H || M < 0 || d <= 0 || lda < d || ldr < d ||
      ldh < d || n_slots <= 0 || (n_slots > 1 && slot_stride < (int64_t)M * lda))
    return W8A8_ERR_INVALID;
  if (gamma && (!beta || !Xq || !sXq || ldq < d)) return W8A8_ERR_INVALID;
  if (n_bcast < 0 || n_bcast > 8 || (n_bcast > 0 && (!xq_bcast || !sx_bcast || bcast_row0 < 0)))
    return W8A8_ERR_INVALID;
  int st = ready();
  if (st) return st;
  ReduceArgs a = {};
  a.acc = acc;
  a.lda = lda;
  a.slot_stride = slot_stride;
  a.n_slots = n_slots;
  a.sX = sX;
  a.sW = sW;
  a.bias = bias;
  a.R = R;
  a.ldr = ldr;
  a.H = H;
  a.ldh = ldh;
  a.gamma = gamma;
  a.beta = beta;
  a.eps = eps;
  a.Xq = Xq;
  a.ldq = ldq;
  a.sXq = sXq;
  a.d = d;
  for (int j = 0; j < n_bcast; ++j) {
    a.xq_bcast[j] = xq_bcast[j];
    a.sx_bcast[j] = sx_bcast[j];
  }
  a.n_bcast = n_bcast;
  a.bcast_row0 = bcast_row0;
  return launch_reduce_layernorm_quant(a, M, (cudaStream_t)stream);
}

extern "C" int w8a8_reduce_residual_layernorm_quant(
    const int32_t *acc, int64_t lda, int n_slots, int64_t slot_stride, int M, int d,
    const float *sX, const float *sW, const gpt2_bf16_t *bias, const gpt2_bf16_t *R, int64_t ldr,
    gpt2_bf16_t *H, int64_t ldh, const gpt2_bf16_t *gamma, const gpt2_bf16_t *beta, float eps,
    int8_t *Xq, int64_t ldq, float *sXq, void *stream) {
  return w8a8_reduce_residual_layernorm_quant_bcast(acc, lda, n_slots, slot_stride, M, d, sX, sW,
                                                    bias, R, ldr, H, ldh, gamma, beta, eps, Xq,
                                                    ldq, sXq, nullptr, nullptr, 0, 0, stream);
}

extern "C" int w8a8_gemm_s32_scatter(const int8_t *Xq, int M, int K, const int8_t *W, int N,
                                     int32_t *const *dst, int n_dst, int rows_per_dst,
                                     void *stream) {
  if (M == 0 || N == 0) return W8A8_OK;
  if (!Xq || !W || !dst || M < 0 || N < 0 || K <= 0 || n_dst < 1 || n_dst > 8 ||
      rows_per_dst <= 0 || (int64_t)rows_per_dst * n_dst < M)
    return W8A8_ERR_INVALID;
  for (int j = 0; j < n_dst; ++j)
    if (!dst[j] || !aligned16(dst[j])) return W8A8_ERR_INVALID;
  int st = ready();
  if (st) return st;
  LinearArgs a = make_args(EPI_S32, M, N, K, nullptr, nullptr, nullptr, nullptr, 0, dst[0], N);
  for (int j = 0; j < n_dst; ++j) a.dst[j] = dst[j];
  a.rows_per_dst = rows_per_dst;
  return dispatch_linear(Xq, K, W, a, (cudaStream_t)stream);
}

extern "C" int w8a8_attention_prefill(const gpt2_bf16_t *Q, int64_t ldq, const gpt2_bf16_t *Kc,
                                      const gpt2_bf16_t *Vc, int64_t seq_stride, int n_seq, int T,
                                      int n_head, int head_dim, gpt2_bf16_t *O, int64_t ldo,
                                      void *stream) {
  if (n_seq == 0 || T == 0) return W8A8_OK;
  if (!Q || !Kc || !Vc || !O || n_seq < 0 || T < 0 || n_head <= 0) return W8A8_ERR_INVALID;
  if (head_dim != 64 || T > 1024) return W8A8_ERR_UNSUPPORTED;
  if (ldq % 8 || ldo % 2 || seq_stride % 8 || !aligned16(Q) || !aligned16(Kc) || !aligned16(Vc) ||
      ((uintptr_t)O & 3))
    return W8A8_ERR_INVALID;
  int st = ready();
  if (st) return st;
  return launch_attention_prefill(Q, ldq, Kc, Vc, seq_stride, n_seq, T, n_head, O, ldo,
                                  (cudaStream_t)stream);
}

extern "C" size_t w8a8_attention_decode_workspace_size(int n_seq, int n_head, int max_ctx) {
  // sized for the largest split count the launcher may pick
  int splits = 1;
  while (splits * 2 * 128 <= max_ctx) splits *= 2;
  return decode_workspace_bytes(n_seq, n_head, max_ctx, splits);
}

extern "C" int w8a8_attention_decode_workspace_reset(void *workspace, size_t workspace_bytes,
                                                    void *stream) {
  return decode_workspace_reset(workspace, workspace_bytes, (cudaStream_t)stream);
}

extern "C" int w8a8_attention_decode_launches(int n_seq, int n_head, int max_ctx) {
  int st;
  DeviceCtx *c = device_ctx(&st);
  if (!c || n_seq <= 0 || n_head <= 0 || max_ctx <= 0) return 0;
  return decode_launches(n_seq, n_head, max_ctx, c->sm_count);
}

static int attention_decode_impl(const gpt2_bf16_t *Q, int64_t ldq, const gpt2_bf16_t *Kc,
                                 const gpt2_bf16_t *Vc, int64_t seq_stride, int n_seq,
                                 const int32_t *n_ctx, int max_ctx, int n_head, int head_dim,
                                 gpt2_bf16_t *O, int64_t ldo, int8_t *Xq, float *sXq,
                                 void *workspace, size_t workspace_bytes, void *stream) {
  if (n_seq == 0) return W8A8_OK;
  if (!Q || !Kc || !Vc || !O || !workspace || n_seq < 0 || n_head <= 0 || max_ctx <= 0)
    return W8A8_ERR_INVALID;
  if (head_dim != 64 || max_ctx > 1024) return W8A8_ERR_UNSUPPORTED;
  if (ldq % 8 || seq_stride % 8 || !aligned16(Q) || !aligned16(Kc) || !aligned16(Vc))
    return W8A8_ERR_INVALID;
  if (Xq && (!sXq || ldo % 8 || !aligned16(O) || ((uintptr_t)Xq & 7))) return W8A8_ERR_INVALID;
  int st;
  DeviceCtx *c = device_ctx(&st);
  if (!c) return st;
  return launch_attention_decode(Q, ldq, Kc, Vc, seq_stride, n_seq, n_ctx, max_ctx, n_head, O, ldo,
                                 Xq, sXq, workspace, workspace_bytes, c->sm_count,
                                 (cudaStream_t)stream);
}

extern "C" int w8a8_attention_decode(const gpt2_bf16_t *Q, int64_t ldq, const gpt2_bf16_t *Kc,
                                     const gpt2_bf16_t *Vc, int64_t seq_stride, int n_seq,
                                     const int32_t *n_ctx, int max_ctx, int n_head, int head_dim,
                                     gpt2_bf16_t *O, int64_t ldo, void *workspace,
                                     size_t workspace_bytes, void *stream) {
  return attention_decode_impl(Q, ldq, Kc, Vc, seq_stride, n_seq, n_ctx, max_ctx, n_head,
                               head_dim, O, ldo, nullptr, nullptr, workspace, workspace_bytes,
                               stream);
}

extern "C" int w8a8_attention_decode_quant(const gpt2_bf16_t *Q, int64_t ldq,
                                           const gpt2_bf16_t *Kc, const gpt2_bf16_t *Vc,
                                           int64_t seq_stride, int n_seq, const int32_t *n_ctx,
                                           int max_ctx, int n_head, int head_dim, gpt2_bf16_t *O,
                                           int64_t ldo, int8_t *Xq, float *sX, void *workspace,
                                           size_t workspace_bytes, void *stream) {
  if (!Xq || !sX) return W8A8_ERR_INVALID;
  return attention_decode_impl(Q, ldq, Kc, Vc, seq_stride, n_seq, n_ctx, max_ctx, n_head,
                               head_dim, O, ldo, Xq, sX, workspace, workspace_bytes, stream);
}

extern "C" int w8a8_lm_head(const gpt2_bf16_t *Xf, int64_t ldx, int M, int d,
                            const gpt2_bf16_t *wte, int V, gpt2_bf16_t *logits, int64_t ldl,
                            void *stream) {
  if (M == 0) return W8A8_OK;
  if (!Xf || !wte || !logits || M < 0 || d <= 0 || V <= 0 || ldl < V || ldx < d)
    return W8A8_ERR_INVALID;
  if (d % 8 || ldx % 8 || !aligned16(Xf) || !aligned16(wte)) return W8A8_ERR_UNSUPPORTED;
  int st = ready();
  if (st) return st;
  LinearArgs a = make_args(EPI_F32_BF16, M, V, d, nullptr, nullptr, nullptr, nullptr, 0, logits, ldl);
  return gemm_tc_bf16(wte, Xf, ldx, a, (cudaStream_t)stream);
}

extern "C" int w8a8_sample_greedy(const gpt2_bf16_t *logits, int64_t ldl, int M, int V,
                                  int32_t *out_tokens, int32_t *append_to, int64_t append_stride,
                                  int32_t *append_pos, void *stream) {
  if (M == 0) return W8A8_OK;
  if (!logits || !out_tokens || M < 0 || V <= 0 || ldl < V) return W8A8_ERR_INVALID;
  if (append_to && !append_pos) return W8A8_ERR_INVALID;
  int st = ready();
  if (st) return st;
  return launch_greedy_sample(logits, ldl, M, V, out_tokens, append_to, append_stride, append_pos,
                              (cudaStream_t)stream);
}

extern "C" int w8a8_sample_topk(const gpt2_bf16_t *logits, int64_t ldl, int M, int V,
                                float temperature, int top_k, const float *rnd,
                                int64_t rnd_stride, const int32_t *rnd_pos, int32_t *out_tokens,
                                int32_t *append_to, int64_t append_stride, int32_t *append_pos,
                                gpt2_bf16_t *probs_out, int64_t ldp, void *stream) {
  if (M == 0) return W8A8_OK;
  if (!logits || !out_tokens || M < 0 || V <= 0 || ldl < V) return W8A8_ERR_INVALID;
  if (append_to && !append_pos) return W8A8_ERR_INVALID;
  if (!(temperature > 0.0f))  // gpt2.c:2212: greedy when the temperature is not positive
    return w8a8_sample_greedy(logits, ldl, M, V, out_tokens, append_to, append_stride, append_pos,
                              stream);
  if (!rnd || rnd_stride < 0 || (probs_out && ldp < V) || ((uintptr_t)logits & 1))
    return W8A8_ERR_INVALID;
  int st = ready();
  if (st) return st;
  return launch_topk_sample(logits, ldl, M, V, temperature, top_k, rnd, rnd_stride, rnd_pos,
                            out_tokens, append_to, append_stride, append_pos, probs_out, ldp,
                            (cudaStream_t)stream);
}

extern "C" int w8a8_advance_positions(int32_t *dst, const int32_t *src, int n, int delta,
                                      void *stream) {
  if (n == 0) return W8A8_OK;
  if (!dst || !src || n < 0) return W8A8_ERR_INVALID;
  return launch_advance(dst, src, n, delta, (cudaStream_t)stream);
}
