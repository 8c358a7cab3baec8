// Launcher interfaces shared between the kernel files and the C-ABI layer.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace w8a8 {

// Epilogue of the INT8 GEMM / GEMV (see epilogue.cuh for the arithmetic).
enum EpiKind {
  EPI_S32 = 0,       // raw int32 accumulators
  EPI_DEQUANT = 1,   // bf16(acc*sW*sX)
  EPI_BIAS = 2,      // + bias
  EPI_RESID = 3,     // + bias, + residual
  EPI_GELU = 4,      // + bias, gelu
  EPI_QKV = 5,       // + bias, scatter into Q / K cache / V cache
  EPI_F32_BF16 = 6,  // bf16(acc) for the bf16 LM head
};

// Arguments of the INT8 linear layer shared by the tensor-core GEMM and the
// CUDA-core GEMV. M tokens, N output channels, K reduction length.
struct LinearArgs {
  int M, N, K;
  int epi;
  const float *sX;
  const float *sW;
  const uint16_t *bias;
  const uint16_t *R;
  int64_t ldr;
  void *Y;
  int64_t ldy;
  // QKV scatter: column n -> segment n / dseg (0 = Q in Y, 1 = K cache,
  // 2 = V cache); token m = b*T + t lands at cache row pos0[b] + t.
  uint16_t *Kc, *Vc;
  int64_t seq_stride;
  int T;
  const int32_t *pos0;
  int dseg;
  // split-K workspace (nullable): int32 [M][N] partial sums + tile tickets,
  // zero-filled before first use; the kernels leave it zeroed.
  void *workspace;
  size_t workspace_bytes;
  // EPI_S32 scatter (rows_per_dst > 0): output row m goes to
  // dst[m / rows_per_dst] + (m % rows_per_dst) * ldy, e.g. into the partial-
  // sum slot that this GPU owns in the buffer of the GPU owning row m.
  int32_t *dst[8];
  int rows_per_dst;
  // Row absmax record of the batch-1 MLP pair (W1 -> W2): a kernel given
  // amax_out also writes, for each of its CTAs, the largest |Y| of every row
  // among the outputs that CTA stored: amax_out[cta * M + m] (0 for rows it
  // did not touch). A kernel given Xb quantizes its bf16 input rows itself
  // (Xb row stride ldxb, the reference's per-token rule) with the row maxima
  // of the n_part partials amax_in[part * M + m].
  float *amax_out;
  const uint16_t *Xb;
  int64_t ldxb;
  const float *amax_in;
  int n_part;
};

// The reference's per-token scale of a row whose largest |x| is amax
// (cuda/activation_quant.cu:75-91), and its quantization of one value.
__device__ __forceinline__ float quant_scale(float amax) {
  return amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
}
__device__ __forceinline__ int quant_value(float x, float inv) {
  const int q = __float2int_rn(__fmul_rn(x, inv));
  return q > 127 ? 127 : (q < -127 ? -127 : q);
}
// 16 bf16 (two 16-byte vectors) -> 16 int8 with the row's 1 / scale.
__device__ __forceinline__ uint4 quant16(const uint4 &lo, const uint4 &hi, float inv) {
  const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int a0 = quant_value(__uint_as_float(w[2 * j] << 16), inv);
    const int a1 = quant_value(__uint_as_float(w[2 * j] & 0xffff0000u), inv);
    const int a2 = quant_value(__uint_as_float(w[2 * j + 1] << 16), inv);
    const int a3 = quant_value(__uint_as_float(w[2 * j + 1] & 0xffff0000u), inv);
    o[j] = (uint32_t)(a0 & 0xff) | ((uint32_t)(a1 & 0xff) << 8) | ((uint32_t)(a2 & 0xff) << 16) |
           ((uint32_t)(a3 & 0xff) << 24);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// Row address of the int32 output of row m (plain or scattered).
__host__ __device__ inline int32_t *s32_row(const LinearArgs &a, int m) {
  if (a.rows_per_dst > 0) {
    const int o = m / a.rows_per_dst;
    return a.dst[o] + (int64_t)(m - o * a.rows_per_dst) * a.ldy;
  }
  return reinterpret_cast<int32_t *>(a.Y) + (int64_t)m * a.ldy;
}

size_t linear_workspace_bytes(int M, int N);

// Residual-stream epilogue of a GEMM whose reduction over K was split across
// GPUs: H = R + (sum of n_slots int32 partials, dequantized, + bias), then
// optionally (gamma != NULL) LayerNorm + per-token quantization into Xq/sXq.
struct ReduceArgs {
  const int32_t *acc;   // partial sums, slot j row m at acc + j*slot_stride + m*lda
  int64_t lda, slot_stride;
  int n_slots;
  const float *sX;      // per-token scale of the GEMM input [M]
  const float *sW;      // per-channel weight scale [d]
  const uint16_t *bias; // [d]
  const uint16_t *R;    // residual input, row stride ldr
  int64_t ldr;
  uint16_t *H;          // residual output, row stride ldh (may equal R)
  int64_t ldh;
  const uint16_t *gamma, *beta;
  float eps;
  int8_t *Xq;           // quantized LayerNorm output, row stride ldq
  int64_t ldq;
  float *sXq;
  int d;
  // optional extra copies of the quantized rows (n_bcast <= 8): row m also
  // goes to xq_bcast[j] + (bcast_row0 + m) * ldq and sx_bcast[j][bcast_row0 + m]
  int8_t *xq_bcast[8];
  float *sx_bcast[8];
  int n_bcast;
  int64_t bcast_row0;
};

// gemm_tc.cu
int gemm_tc_i8(const int8_t *W, const int8_t *X, int64_t ldx, const LinearArgs &a,
               cudaStream_t stream);
// Workspace bytes gemm_tc_i8 reads for these operands (a.workspace set):
// nonzero only where it takes the channel-major kernel split over K.
size_t gemm_i8_workspace_used(const int8_t *X, int64_t ldx, const LinearArgs &a);
int gemm_tc_bf16(const uint16_t *W, const uint16_t *X, int64_t ldx, const LinearArgs &a,
                 cudaStream_t stream);
// gemm_cluster.cu: decode-sized GEMMs (M <= 128) with split-K in a cluster
bool cluster_gemm_ok(const LinearArgs &a, const void *X, int64_t ldx);
int gemm_cluster_i8(const int8_t *W, const int8_t *X, int64_t ldx, const LinearArgs &a,
                    cudaStream_t stream);
// api.cu: workspace bytes w8a8_linear reads for these operands (0 where the
// chosen kernel reads none)
size_t linear_workspace_used(const int8_t *Xq, const float *sX, int M, int K, const int8_t *W,
                             const float *sW, const uint16_t *bias, int N, int epilogue,
                             const uint16_t *R, int64_t ldr, uint16_t *Y, int64_t ldy);
// gemv_i8.cu
int launch_gemv_i8(const int8_t *X, int64_t ldx, const int8_t *W, const LinearArgs &a,
                   cudaStream_t s);
// The batch-1 MLP pair of the row absmax record (LinearArgs::amax_out / Xb):
// W8A8_ERR_UNSUPPORTED where the operands take a kernel without it.
int gemv_absmax(const int8_t *X, int64_t ldx, const int8_t *W, const LinearArgs &a, int *n_part,
                cudaStream_t s);
int gemv_from_bf16(const int8_t *W, const LinearArgs &a, cudaStream_t s);
// The batch-1 GEMV that forms its input row's LayerNorm and quantization
// itself (from the bf16 row X with gain / bias), also writing the quantized
// row to Xq / sX: W8A8_ERR_UNSUPPORTED where the operands do not allow it.
struct GemvLnArgs {
  const uint16_t *X;
  const uint16_t *gamma, *beta;
  float eps;
  int8_t *Xq;
  float *sX;
};
int gemv_layernorm(const int8_t *W, const LinearArgs &a, const GemvLnArgs &ln, int *n_part,
                   cudaStream_t s);
// norm_quant.cu
int launch_quant_rows(const uint16_t *X, int64_t ldx, int M, int K, int8_t *Xq, float *sX,
                      cudaStream_t s);
int launch_layernorm_quant(const uint16_t *X, int64_t ldx, int M, int d, const uint16_t *gamma,
                           const uint16_t *beta, float eps, uint16_t *Y, int64_t ldy, int8_t *Xq,
                           float *sX, cudaStream_t s);
int launch_embed_layernorm_quant(const uint16_t *wte, const uint16_t *wpe, const int32_t *tokens,
                                 int M, int T, const int32_t *pos0, int d, uint16_t *H,
                                 const uint16_t *gamma, const uint16_t *beta, float eps,
                                 uint16_t *Y, int8_t *Xq, float *sX, cudaStream_t s);
int launch_row_amax(const uint16_t *X, int64_t ldx, int M, int K, float *const *amax, int n_out,
                    cudaStream_t s);
int launch_quant_rows_amax(const uint16_t *X, int64_t ldx, int M, int K, const float *amax,
                           int n_amax, int64_t amax_stride, int8_t *Xq, int64_t ldq, float *sX,
                           cudaStream_t s);
int launch_reduce_layernorm_quant(const ReduceArgs &a, int M, cudaStream_t s);
// attention.cu
// attention_tc.cu: tcgen05 prefill attention (head_dim 64, T <= 1024)
bool attention_prefill_tc_ok(const uint16_t *Q, int64_t ldq, const uint16_t *Kc,
                             const uint16_t *Vc, int64_t seq_stride, int T, int n_head);
int launch_attention_prefill_tc(const uint16_t *Q, int64_t ldq, const uint16_t *Kc,
                                const uint16_t *Vc, int64_t seq_stride, int n_seq, int T,
                                int n_head, uint16_t *O, int64_t ldo, cudaStream_t stream);
int launch_attention_prefill(const uint16_t *Q, int64_t ldq, const uint16_t *Kc,
                             const uint16_t *Vc, int64_t seq_stride, int n_seq, int T, int n_head,
                             uint16_t *O, int64_t ldo, cudaStream_t s);
size_t decode_workspace_bytes(int n_seq, int n_head, int max_ctx, int splits);
int decode_launches(int n_seq, int n_head, int max_ctx, int sm_count);
int decode_workspace_reset(void *ws, size_t ws_bytes, cudaStream_t s);
int launch_attention_decode(const uint16_t *Q, int64_t ldq, const uint16_t *Kc,
                            const uint16_t *Vc, int64_t seq_stride, int n_seq,
                            const int32_t *n_ctx, int max_ctx, int n_head, uint16_t *O,
                            int64_t ldo, int8_t *Xq, float *sXq, void *ws, size_t ws_bytes,
                            int sm_count, cudaStream_t s);
// sample.cu
int launch_greedy_sample(const uint16_t *logits, int64_t ldl, int M, int V, int32_t *out,
                         int32_t *append_to, int64_t append_stride, int32_t *append_pos,
                         cudaStream_t s);
int launch_advance(int32_t *dst, const int32_t *src, int n, int delta, cudaStream_t s);
int launch_topk_sample(const uint16_t *logits, int64_t ldl, int M, int V, float temperature,
                       int k, const float *rnd, int64_t rnd_stride, const int32_t *rnd_pos,
                       int32_t *out, int32_t *append_to, int64_t append_stride,
                       int32_t *append_pos, uint16_t *probs_out, int64_t ldp, cudaStream_t s);

}  // namespace w8a8
