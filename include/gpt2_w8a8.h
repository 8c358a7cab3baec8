/*
 * gpt2_w8a8.h — runtime-dimension C ABI of the sm_100a W8A8 GPT-2 kernels.
 *
 * Every pointer argument is device memory owned by the caller; no entry point
 * allocates (the reference's ownership rule: all buffers belong to the host
 * program, gpt2.c:864-942). Streams are passed as `void *` (a cudaStream_t;
 * NULL = legacy default stream, the stream the reference launches on).
 * bf16 tensors are passed as raw 16-bit patterns (gpt2_bf16_t), bit-compatible
 * with __nv_bfloat16 / __bf16.
 *
 * All matrices are row-major. Weights are stored [OUT, IN] exactly as the
 * reference's quant8.bin holds them (tools/offline_quant/src/quantizer.py:3-4),
 * so X[M,K] · W[N,K]^T needs no transpose.
 *
 * Kernels are launched with programmatic dependent launch: a GEMM or GEMV
 * starts reading its weight matrix W before the preceding
 * kernel of the stream has finished, and reads everything else only after.
 * W must therefore not be written by the kernel launched just before the call
 * on the same stream (a copy, an event wait or W8A8_PDL=0 in the environment
 * orders it fully).
 *
 * Every entry point returns W8A8_OK (0) or a negative status; nothing aborts.
 * The reference-shaped drop-in functions (include/cuda_kernels.h) wrap these
 * and keep the reference's abort-on-error convention.
 */
#ifndef GPT2_W8A8_H
#define GPT2_W8A8_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef uint16_t gpt2_bf16_t;

/* ---- status codes ---- */
#define W8A8_OK 0
#define W8A8_ERR_INVALID (-1)     /* bad shape, null pointer, misaligned buffer */
#define W8A8_ERR_UNSUPPORTED (-2) /* shape this build does not handle */
#define W8A8_ERR_CUDA (-3)        /* a CUDA runtime call or launch failed */
#define W8A8_ERR_DEVICE (-4)      /* a kernel recorded an error (see w8a8_device_error) */
#define W8A8_ERR_NOMEM (-5)
#define W8A8_ERR_IO (-6)

/* ---- epilogues of the INT8 linear layer (applied to acc = Xq · W^T) ----
 * t = bf16(((float)acc * sW[n]) * sX[m])          dequant, activation_quant.cu:129-130
 * b-step  y = bf16(float(t) + float(bias[n]))     add_bias.cu:13
 * Each mode stores one bf16 per output element: */
#define W8A8_EPI_DEQUANT 0    /* Y = t                                        */
#define W8A8_EPI_BIAS 1       /* Y = y                                        */
#define W8A8_EPI_BIAS_RESID 2 /* Y = bf16(float(R[m,n]) + float(y))   add_2d.cu:14 */
#define W8A8_EPI_BIAS_GELU 3  /* Y = bf16(gelu_tanh(float(y)))        gelu.cu:10-16 */

/* Per-device set-up: resolves the device error word and the TMA encoder.
 * Call once per device (with that device current) before stream capture. */
int w8a8_init(int device);
const char *w8a8_status_string(int status);
/* The CUDA error behind the calling thread's last W8A8_ERR_CUDA from a launch. */
const char *w8a8_last_cuda_error(void);
/* Returns the first error code a kernel recorded on the current device since
 * the last reset (0 = none); `reset` != 0 clears it. Synchronises the device. */
int w8a8_device_error(int reset);

/* ---- per-token INT8 activation quantization (activation_quant.cu:37-110) ----
 * X [M,K] bf16 (row stride ldx elements) -> Xq [M,K] int8 (row stride K),
 * sX [M] fp32: scale = amax>0 ? amax/127 : 1 ; q = clamp(rn(x*(1/scale)),±127) */
int w8a8_quant_rows(const gpt2_bf16_t *X, int64_t ldx, int M, int K, int8_t *Xq, float *sX,
                    void *stream);

/* ---- LayerNorm (layernorm.cu:7-100) fused with per-token quantization ----
 * Y = bf16(((x-mean)*rsqrt(var+eps))*gamma + beta), with the reference's
 * two-pass fp32 statistics. Y (nullable) receives the bf16 rows; Xq/sX
 * (nullable together) receive the quantized rows of Y. d <= 8192. */
int w8a8_layernorm_quant(const gpt2_bf16_t *X, int64_t ldx, int M, int d,
                         const gpt2_bf16_t *gamma, const gpt2_bf16_t *beta, float eps,
                         gpt2_bf16_t *Y, int64_t ldy, int8_t *Xq, float *sX, void *stream);

/* ---- token + position embedding (embeddings.cu:8-25) fused with LayerNorm
 * and quantization of the first layer's input ----
 * Row m = b*T + t (b < M/T sequences of T new tokens): token id tokens[m],
 * position p = (pos0 ? pos0[b] : 0) + t. H[m] = bf16(wte[id] + wpe[p]) and
 * LayerNorm/quantization of H[m] as in w8a8_layernorm_quant. */
int w8a8_embed_layernorm_quant(const gpt2_bf16_t *wte, const gpt2_bf16_t *wpe,
                               const int32_t *tokens, int M, int T, const int32_t *pos0, int d,
                               gpt2_bf16_t *H, const gpt2_bf16_t *gamma,
                               const gpt2_bf16_t *beta, float eps, gpt2_bf16_t *Y,
                               int8_t *Xq, float *sX, void *stream);

/* ---- INT8 x INT8 -> INT32 GEMM (the reference's cublasGemmEx call,
 * gpt2.c:404-415): Y[M,N] = Xq[M,K] · W[N,K]^T, exact integer arithmetic.
 * K % 16 == 0 and 16-byte aligned operands take the tcgen05 tensor-core path;
 * other shapes take a CUDA-core kernel with the same results. */
int w8a8_gemm_s32(const int8_t *Xq, int M, int K, const int8_t *W, int N, int32_t *Y,
                  void *stream);

/* ---- fused W8A8 linear layer: GEMM + dequant + bias (+ residual / GELU) ----
 * Replaces dot_2d_gpu_int8 + add_bias_cuda (+ add_2d_cuda / gelu_cuda),
 * gpt2.c:384-428, 1145-1325. R is read only for W8A8_EPI_BIAS_RESID and may
 * alias Y (in-place residual add). bias may be NULL only for EPI_DEQUANT. */
int w8a8_linear(const int8_t *Xq, const float *sX, int M, int K, const int8_t *W,
                const float *sW, const gpt2_bf16_t *bias, int N, int epilogue,
                const gpt2_bf16_t *R, int64_t ldr, gpt2_bf16_t *Y, int64_t ldy,
                void *workspace, size_t workspace_bytes, void *stream);

/* ---- the W1 -> W2 pair with the quantization of W1's output fused ----
 * The reference quantizes the GELU output per token as a kernel of its own
 * between the two MLP GEMMs (gpt2.c:1296-1320: gelu_cuda, then
 * dot_2d_gpu_int8 -> per_token_quant_cuda, cuda/activation_quant.cu:37-110).
 * Here the first GEMM's epilogue also records each row's largest |y| as
 * partial maxima (the row absmax record: absmax[part * M + m], one part per
 * CTA of the kernel that wrote the rows), and the second GEMM quantizes its
 * bf16 input rows itself with the reference's rule (scale = amax / 127, or 1
 * for an all-zero row; q = rn(x * (1 / scale)) clamped to +-127): the same
 * int8 rows and scales as w8a8_quant_rows, without its launch and without
 * the int8 copy of the rows. Fused for one token (the batch-1 decode GEMVs,
 * where it saves a launch per layer); other shapes run the separate maxima /
 * quantization kernels, with the same results: there every output tile of
 * the second GEMM would quantize the same input columns again, which costs
 * more than the one quantization launch it saves.
 *
 * w8a8_linear_absmax: w8a8_linear (bf16 epilogues only) that also writes the
 * record into absmax (at least w8a8_absmax_record_floats(M, N) floats) and
 * its part count into *n_part (host). */
size_t w8a8_absmax_record_floats(int M, int N);
int w8a8_linear_absmax(const int8_t *Xq, const float *sX, int M, int K, const int8_t *W,
                       const float *sW, const gpt2_bf16_t *bias, int N, int epilogue,
                       const gpt2_bf16_t *R, int64_t ldr, gpt2_bf16_t *Y, int64_t ldy,
                       float *absmax, size_t absmax_floats, int *n_part, void *workspace,
                       size_t workspace_bytes, void *stream);
/* w8a8_linear on the per-token quantization of the bf16 rows X (row stride
 * ldx, K % 8 == 0), whose row maxima are the n_part partials of absmax.
 * Xq [M][K] / sX [M] receive the quantized rows and scales where the shape
 * takes the separate quantization kernel; the fused kernels leave them as
 * they are. */
int w8a8_linear_from_bf16(const gpt2_bf16_t *X, int64_t ldx, const float *absmax, int n_part,
                          int M, int K, const int8_t *W, const float *sW,
                          const gpt2_bf16_t *bias, int N, int epilogue, const gpt2_bf16_t *R,
                          int64_t ldr, gpt2_bf16_t *Y, int64_t ldy, int8_t *Xq, float *sX,
                          void *workspace, size_t workspace_bytes, void *stream);

/* ---- LayerNorm folded into the GEMV of a single token ----
 * The reference runs LayerNorm (layernorm_cuda, cuda/layernorm.cu) and then
 * quantizes its output per token inside dot_2d_gpu_int8 (gpt2.c:1138-1145,
 * 1293-1296) before the QKV and W1 GEMMs. Each call below is
 * w8a8_layernorm_quant(X, ldx, M, K, gamma, beta, eps, NULL, 0, Xq, sX)
 * followed by w8a8_linear_qkv / w8a8_linear_absmax on Xq, sX, with the same
 * results (Xq and sX are written in both forms). For one token (M == 1,
 * K % 16 == 0, K <= 2048, 16-byte aligned X, gain, bias, Xq and weights)
 * the two run as one kernel: every block of the GEMV forms the row's
 * LayerNorm and quantization itself, so the LayerNorm launch and the
 * quantized row's trip through memory leave the batch-1 decode chain. Other
 * shapes run the two kernels. */
int w8a8_layernorm_linear_qkv(const gpt2_bf16_t *X, int64_t ldx, const gpt2_bf16_t *gamma,
                              const gpt2_bf16_t *beta, float eps, int8_t *Xq, float *sX, int M,
                              int d, const int8_t *Wqkv, const float *sWqkv,
                              const gpt2_bf16_t *bqkv, gpt2_bf16_t *Q, int64_t ldq,
                              gpt2_bf16_t *Kc, gpt2_bf16_t *Vc, int64_t seq_stride, int T,
                              const int32_t *pos0, void *workspace, size_t workspace_bytes,
                              void *stream);
int w8a8_layernorm_linear_absmax(const gpt2_bf16_t *X, int64_t ldx, const gpt2_bf16_t *gamma,
                                 const gpt2_bf16_t *beta, float eps, int8_t *Xq, float *sX,
                                 int M, int K, const int8_t *W, const float *sW,
                                 const gpt2_bf16_t *bias, int N, int epilogue,
                                 const gpt2_bf16_t *R, int64_t ldr, gpt2_bf16_t *Y, int64_t ldy,
                                 float *absmax, size_t absmax_floats, int *n_part,
                                 void *workspace, size_t workspace_bytes, void *stream);

/* ---- w8a8_linear without a caller-provided workspace ----
 * No counterpart in the reference. For callers that cannot allocate device
 * memory (a host that sizes all device memory once at start-up, a plugin whose
 * host owns the allocator, a path that must not pay cudaMalloc's implicit
 * synchronisation). Where w8a8_linear would split a few-token GEMM over K into
 * a caller's workspace (operands the cluster kernel cannot take), this entry
 * point uses a fixed array compiled into this library instead
 * (W8A8_NOALLOC_SCRATCH_BYTES, held by every GPU that loads the library until
 * exit), clearing the part it uses first; such shapes needing more than the
 * array, i.e. M*N*4 bytes plus one 4-byte counter per 128 x 32 output tile,
 * return W8A8_ERR_UNSUPPORTED. Every other shape runs as w8a8_linear with no
 * workspace. Nothing is allocated. The first call on a device looks up the
 * array's device address and must come before any stream capture. All calls
 * share the array: calls whose GPU work overlaps race and must be serialised
 * by the caller. Same arguments and results as w8a8_linear. */
#define W8A8_NOALLOC_SCRATCH_BYTES (4u << 20)
int w8a8_linear_noalloc(const int8_t *Xq, const float *sX, int M, int K, const int8_t *W,
                        const float *sW, const gpt2_bf16_t *bias, int N, int epilogue,
                        const gpt2_bf16_t *R, int64_t ldr, gpt2_bf16_t *Y, int64_t ldy,
                        void *stream);

/* Workspace that lets w8a8_linear / w8a8_linear_qkv split the reduction over
 * K when M is small (decode) and the output tiles alone cannot occupy every
 * SM. Optional (NULL disables splitting). It must be zero-filled once before
 * its first use; every call leaves it zero again. Calls sharing a workspace
 * must not overlap on the GPU. */
size_t w8a8_linear_workspace_size(int M, int N);

/* ---- packed QKV projection straight into Q and the KV cache ----
 * W_qkv [3d, d] stays packed (the reference splits it at load,
 * gpt2.c:1725-1738; splitting changes no output element). Output column n of
 * row m: n < d -> Q[m*ldq + n]; d <= n < 2d -> K cache; 2d <= n -> V cache,
 * each bf16(bf16(acc*sW*sX)+b) as the reference's three calls produce
 * (gpt2.c:1145-1167). Row m = b*T + t belongs to sequence b at cache position
 * p = (pos0 ? pos0[b] : 0) + t; its K row is Kc + b*seq_stride + p*d. */
int w8a8_linear_qkv(const int8_t *Xq, const float *sX, int M, int d, const int8_t *Wqkv,
                    const float *sWqkv, const gpt2_bf16_t *bqkv, gpt2_bf16_t *Q, int64_t ldq,
                    gpt2_bf16_t *Kc, gpt2_bf16_t *Vc, int64_t seq_stride, int T,
                    const int32_t *pos0, void *workspace, size_t workspace_bytes,
                    void *stream);

/* ---- causal attention over the KV cache, prefill (gpt2.c:1205-1217) ----
 * n_seq sequences of T tokens each, cached from position 0. Query row
 * m = b*T + t, head h, reads Q[m*ldq + h*hd ..]; attends keys 0..t of
 * sequence b. S = bf16(q.k / sqrt(hd)); P = bf16(bf16(exp(S-max)) / sum);
 * O[m*ldo + h*hd ..] = bf16(P·V). hd == 64, T <= 1024. */
int w8a8_attention_prefill(const gpt2_bf16_t *Q, int64_t ldq, const gpt2_bf16_t *Kc,
                           const gpt2_bf16_t *Vc, int64_t seq_stride, int n_seq, int T,
                           int n_head, int hd, gpt2_bf16_t *O, int64_t ldo,
                           void *stream);

/* ---- attention of one new token per sequence, decode (gpt2.c:1191-1203) ----
 * Sequence b attends its first n_ctx[b] cache rows (n_ctx includes the new
 * token, device array). max_ctx bounds every n_ctx[b] (<= 1024); with
 * n_ctx == NULL every sequence attends exactly max_ctx rows. The
 * workspace holds scores, split partials and, in its last bytes, ticket
 * counters that must be zero before a call: zero-fill the workspace once
 * (every call leaves the counters zero), or call
 * w8a8_attention_decode_workspace_reset after using the memory for anything
 * else. Size it with w8a8_attention_decode_workspace_size(). */
size_t w8a8_attention_decode_workspace_size(int n_seq, int n_head, int max_ctx);
int w8a8_attention_decode_workspace_reset(void *workspace, size_t workspace_bytes, void *stream);
int w8a8_attention_decode(const gpt2_bf16_t *Q, int64_t ldq, const gpt2_bf16_t *Kc,
                          const gpt2_bf16_t *Vc, int64_t seq_stride, int n_seq,
                          const int32_t *n_ctx, int max_ctx, int n_head, int hd,
                          gpt2_bf16_t *O, int64_t ldo, void *workspace,
                          size_t workspace_bytes, void *stream);

/* Kernels one w8a8_attention_decode(_quant) call launches for this shape:
 * 1 (one CTA per sequence and head) or 2 (keys split over CTAs). */
int w8a8_attention_decode_launches(int n_seq, int n_head, int max_ctx);

/* w8a8_attention_decode fused with the per-token quantization that feeds the
 * attention projection (gpt2.c:1235, per_token_quant_cuda on the concatenated
 * heads): besides O, writes Xq [n_seq][n_head*64] int8 and sX [n_seq] exactly
 * as w8a8_quant_rows(O) would. The CTA that finishes the last head of a
 * sequence quantizes that sequence's row, so no second launch is needed. The
 * workspace must be zero-filled before its first use; every call leaves it
 * so. */
int w8a8_attention_decode_quant(const gpt2_bf16_t *Q, int64_t ldq, const gpt2_bf16_t *Kc,
                                const gpt2_bf16_t *Vc, int64_t seq_stride, int n_seq,
                                const int32_t *n_ctx, int max_ctx, int n_head, int hd,
                                gpt2_bf16_t *O, int64_t ldo, int8_t *Xq, float *sX,
                                void *workspace, size_t workspace_bytes, void *stream);

/* ---- LM head (gpt2.c:2160): logits[M,V] = bf16(Xf[M,d] · wte[V,d]^T), fp32
 * accumulation. wte is used as stored ([vocab, d], K-major); the reference's
 * host transpose wte_T (gpt2.c:1915-1918) is not needed. */
int w8a8_lm_head(const gpt2_bf16_t *Xf, int64_t ldx, int M, int d, const gpt2_bf16_t *wte,
                 int V, gpt2_bf16_t *logits, int64_t ldl, void *stream);

/* ---- greedy next token (gpt2.c:2180-2222) ----
 * Per row: probs = softmax(logits) in the reference's bf16 rounding order
 * (softmax.cu:24-92, temperature 1), token = first index of the largest
 * bf16 probability. Writes out_tokens[m]; if append_to is non-NULL also
 * stores the token at append_to[m*append_stride + append_pos[m]] and
 * increments append_pos[m] (device-side sequence bookkeeping for decode). */
int w8a8_sample_greedy(const gpt2_bf16_t *logits, int64_t ldl, int M, int V,
                       int32_t *out_tokens, int32_t *append_to, int64_t append_stride,
                       int32_t *append_pos, void *stream);

/* ---- top-k sampling at a temperature (gpt2.c:130-180 top_k_sample,
 * gpt2.c:2223-2245 the draw) ----
 * Per row m: probs = softmax(logits / temperature) in the reference's bf16
 * rounding order (softmax.cu:24-92); the top_k largest probabilities (top_k
 * clamped to [1, V] as gpt2.c:1963-1968 clamps it), summed in fp32 in
 * descending order and each divided by that sum into bf16 (all bf16(1/top_k)
 * if the sum is 0); r = rnd[m*rnd_stride + (rnd_pos ? rnd_pos[m] : 0)], the
 * caller's draw in [0, 1] ((float)rand() / RAND_MAX in the reference); the
 * token is the first of the sorted top_k whose fp32 running sum exceeds r,
 * else the top_k-th. Among equal probabilities the lower index sorts first
 * (the reference's qsort leaves that order unspecified). A temperature that
 * is not positive gives the greedy token (w8a8_sample_greedy; rnd unused).
 * probs_out (optional, [M, ldp]) receives the bf16 probabilities. Appends to
 * append_to / append_pos as w8a8_sample_greedy does. V <= 81920, else
 * W8A8_ERR_UNSUPPORTED. */
int w8a8_sample_topk(const gpt2_bf16_t *logits, int64_t ldl, int M, int V, float temperature,
                     int top_k, const float *rnd, int64_t rnd_stride, const int32_t *rnd_pos,
                     int32_t *out_tokens, int32_t *append_to, int64_t append_stride,
                     int32_t *append_pos, gpt2_bf16_t *probs_out, int64_t ldp, void *stream);

/* dst[i] = src[i] + delta for i < n (device arrays; dst may equal src). */
int w8a8_advance_positions(int32_t *dst, const int32_t *src, int n, int delta, void *stream);

/* ---- tensor-parallel building blocks ----
 * No counterpart in the reference, which runs each layer on one GPU
 * (transformer_block_gpu, gpt2.c:1124-1330). These split that layer over G
 * GPUs so that every output equals the single-GPU layer bit for bit:
 * QKV and W1 column-split (whole heads / a d_ff slice per GPU), attn_proj and
 * W2 row-split with int32 partial sums reduced exactly, and the per-token
 * scale of a row whose columns are spread over GPUs taken from the maximum
 * of the per-GPU row maxima. */

/* amax[m] = max_k |X[m, k]| over the K columns given (K % 8 == 0). */
int w8a8_row_amax(const gpt2_bf16_t *X, int64_t ldx, int M, int K, float *amax, void *stream);
/* The same maxima written into n_out <= 8 arrays (host array of device
 * pointers, e.g. this GPU's and its peers' exchange slots). */
int w8a8_row_amax_to(const gpt2_bf16_t *X, int64_t ldx, int M, int K, float *const *amax,
                     int n_out, void *stream);

/* per_token_quant of a column block with the scale of the whole row: the
 * row's absolute maximum is the largest of n_amax partial maxima
 * amax[j * amax_stride + m]. Identical to w8a8_quant_rows on the whole row
 * restricted to these columns. */
int w8a8_quant_rows_amax(const gpt2_bf16_t *X, int64_t ldx, int M, int K, const float *amax,
                         int n_amax, int64_t amax_stride, int8_t *Xq, int64_t ldq, float *sX,
                         void *stream);

/* Residual stream after a row-split GEMM: acc is the sum of n_slots int32
 * partial rows (slot j, row m at acc + j*slot_stride + m*lda), and
 *   H[m, n] = bf16(R[m, n] + bf16(bf16(acc*sW[n]*sX[m]) + bias[n]))
 * as w8a8_linear's W8A8_EPI_BIAS_RESID (activation_quant.cu:129-130,
 * add_bias.cu:14, add_2d.cu:14). With gamma != NULL, then LayerNorm of H
 * (layernorm.cu:7-100) quantized per token into Xq (row stride ldq) / sXq.
 * H may equal R. d % 8 == 0, 16-byte aligned rows. */
int w8a8_reduce_residual_layernorm_quant(const int32_t *acc, int64_t lda, int n_slots,
                                         int64_t slot_stride, int M, int d, const float *sX,
                                         const float *sW, const gpt2_bf16_t *bias,
                                         const gpt2_bf16_t *R, int64_t ldr, gpt2_bf16_t *H,
                                         int64_t ldh, const gpt2_bf16_t *gamma,
                                         const gpt2_bf16_t *beta, float eps, int8_t *Xq,
                                         int64_t ldq, float *sXq, void *stream);

/* As above, and the quantized rows (gamma != NULL) are also stored into
 * n_bcast <= 8 more buffers: row m to xq_bcast[j] + (bcast_row0 + m) * ldq and
 * sx_bcast[j][bcast_row0 + m] (the other GPUs' all-gather buffers). */
int w8a8_reduce_residual_layernorm_quant_bcast(
    const int32_t *acc, int64_t lda, int n_slots, int64_t slot_stride, int M, int d,
    const float *sX, const float *sW, const gpt2_bf16_t *bias, const gpt2_bf16_t *R, int64_t ldr,
    gpt2_bf16_t *H, int64_t ldh, const gpt2_bf16_t *gamma, const gpt2_bf16_t *beta, float eps,
    int8_t *Xq, int64_t ldq, float *sXq, int8_t *const *xq_bcast, float *const *sx_bcast,
    int n_bcast, int64_t bcast_row0, void *stream);

/* w8a8_gemm_s32 whose output row m goes to dst[m / rows_per_dst] +
 * (m % rows_per_dst) * N: the partial sums of the rows other GPUs own are
 * stored straight into their buffers (peer memory, 16-byte stores), the
 * int32 reduce-scatter of a row-split GEMM without a separate collective. */
int w8a8_gemm_s32_scatter(const int8_t *Xq, int M, int K, const int8_t *W, int N,
                          int32_t *const *dst, int n_dst, int rows_per_dst, void *stream);

/* ---- peer memory between the GPUs of one node (no counterpart in the
 * reference) ----
 * w8a8_peer_alloc: zero-filled device buffer + its 64-byte CUDA IPC handle;
 * w8a8_peer_open maps another process's buffer (NVLink peer access).
 * w8a8_peer_signal: after the work before it on the stream, writes `value`
 * into each of the n <= 8 flag words (host array of device pointers, this or
 * other GPUs) with system-scope release; w8a8_peer_wait: the work after it on
 * the stream waits until the n flag words flags[0..n) of this GPU are >= value
 * (system-scope acquire; gives up after ~2 s and records a device error). */
int w8a8_peer_alloc(size_t bytes, void **ptr, void *ipc_handle);
int w8a8_peer_open(const void *ipc_handle, void **ptr);
int w8a8_peer_close(void *ptr);
int w8a8_peer_free(void *ptr);
/* Device-to-device copy on `stream` (either side may be a mapped peer buffer). */
int w8a8_peer_copy(void *dst, const void *src, size_t bytes, void *stream);
int w8a8_peer_signal(uint32_t *const *flags, int n, uint32_t value, void *stream);
int w8a8_peer_wait(const uint32_t *flags, int n, uint32_t value, void *stream);

/* w8a8_linear_qkv for a subset of the heads: Wqkv [3*d_heads, K] holds the
 * Q, K and V rows of those heads (d_heads = 64 * heads, a multiple of 32),
 * and Q, Kc and Vc have rows of d_heads. */
int w8a8_linear_qkv_heads(const int8_t *Xq, const float *sX, int M, int K, int d_heads,
                          const int8_t *Wqkv, const float *sWqkv, const gpt2_bf16_t *bqkv,
                          gpt2_bf16_t *Q, int64_t ldq, gpt2_bf16_t *Kc, gpt2_bf16_t *Vc,
                          int64_t seq_stride, int T, const int32_t *pos0, void *workspace,
                          size_t workspace_bytes, void *stream);

/* ---- reference-shaped element-wise operations ----
 * Runtime-dimension forms of the reference's cuda/ kernels with their
 * exact per-element results; include/cuda_kernels.h maps its drop-in symbols
 * onto these. */
int w8a8_ref_embeddings(const gpt2_bf16_t *wte, const gpt2_bf16_t *wpe, const int32_t *tokens,
                        gpt2_bf16_t *emb, int d, int start_row, int n_rows, void *stream);
int w8a8_ref_add_bias(gpt2_bf16_t *a, int rows, int cols, const gpt2_bf16_t *b, void *stream);
int w8a8_ref_add_2d(const gpt2_bf16_t *a, int rows, int cols, const gpt2_bf16_t *b,
                    gpt2_bf16_t *out, void *stream);
int w8a8_ref_gelu(gpt2_bf16_t *x, int cols, int rows, void *stream);
int w8a8_ref_dequant(const int32_t *Y, const float *sW, const float *sX, gpt2_bf16_t *out, int M,
                     int N, void *stream);
int w8a8_ref_causal_mask(gpt2_bf16_t *x, int stride, int tokens, void *stream);
int w8a8_ref_concat_heads(const gpt2_bf16_t *src, gpt2_bf16_t *dest, int token_index, int n_head,
                          int hd, int ctx, void *stream);
int w8a8_ref_softmax(const gpt2_bf16_t *a, int rows, int cols, int stride, gpt2_bf16_t *out,
                     float temperature, int causal_mask, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* GPT2_W8A8_H */
