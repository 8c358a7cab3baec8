/*
 * cuda_kernels.h — drop-in replacement for the reference's kernel ABI.
 *
 * Declares exactly the extern "C" functions of the reference's
 * include/cuda_kernels.h:1-85 (same names, parameter lists and semantics),
 * implemented by libcuda_kernels_<size>.so on top of the sm_100a kernels of
 * gpt2_w8a8.h, plus the new entry points the W8A8 call sites of gpt2.c use
 * instead of cuBLAS (bottom of this file).
 *
 * As in the reference, `d_model` is a compile-time constant inside the
 * pointer-to-array parameter types, so the ABI is per model size: build with
 * -DGPT2_SMALL_MODEL / -DGPT2_MEDIUM_MODEL / -DGPT2_LARGE_MODEL and link the
 * matching library. All pointers are device memory; launches go to the legacy
 * default stream; a failed launch prints a FATAL line and aborts, as the
 * reference's wrappers do (e.g. cuda/activation_quant.cu:104-109).
 */
#pragma once

#include "gpt2_model_config.h"

#ifdef __cplusplus
extern "C" {
#endif

/* cuda_kernels.h:9-14 */
void embeddings_cuda(weight_t (*wte_d)[d_model], weight_t (*wpe_d)[d_model], int *token_d,
                     act_t (*embeddings_d)[d_model], int start_row, int n_rows);

/* cuda_kernels.h:17-24 (d_model_size is accepted and, as in the reference
 * kernel, the compile-time d_model is used) */
void layernorm_cuda(act_t (*input)[d_model], int n_tokens, int d_model_size, weight_t *gamma,
                    weight_t *beta, act_t (*output)[d_model], float eps);

/* cuda_kernels.h:27-32 (in place; `out` is ignored as in the reference) */
void add_bias_cuda(act_t *a, int a_r, int a_c, weight_t *b, act_t *out);

/* cuda_kernels.h:37-45 */
void softmax_cuda(act_t *a, int a_r, int a_c, int stride, act_t *c_out, float temperature,
                  int causal_mask);

/* cuda_kernels.h:48-50 */
void casual_masking_cuda(act_t *in, int stride, int tokens);

/* cuda_kernels.h:52 (in place; `out` is ignored as in the reference) */
void gelu_cuda(act_t *in, int cols, int rows, act_t *out);

/* cuda_kernels.h:55 */
void concat_heads_cuda(act_t *src, act_t *dest, int token_index, int _nof_heads, int _head_dim,
                       int _ctx_len);

/* cuda_kernels.h:57 (out == NULL -> in place into a) */
void add_2d_cuda(act_t *a, int a_r, int a_c, act_t *b, act_t *out);

/* cuda_kernels.h:65-69 */
void per_token_quant_cuda(const act_t *X, qweight_t *X_q, qscale_t *scale_X, int tokens, int d);

/* cuda_kernels.h:75-79 */
void dequant_int32_to_bf16_cuda(const int32_t *Y_int32, const qscale_t *scale_W,
                                const qscale_t *scale_X, act_t *Y_bf16, int M, int N);

/* ---- new entry points for gpt2.c's W8A8 call sites ----
 * They replace the static dot_2d_gpu_int8 (gpt2.c:384-428, quant + cuBLAS
 * INT8 GEMM + dequant) and the add_bias_cuda / add_2d_cuda / gelu_cuda that
 * follow each call, the per-head cuBLAS attention GEMMs + softmax
 * (gpt2.c:1182-1219) and the LM-head GEMM + vocab softmax + host argmax
 * (gpt2.c:2150-2222). Scratch buffers are the caller's, as in gpt2.c
 * (X_int8_scratch_d / scale_X_scratch_d, gpt2.c:909-911). */

/* y[M,N] = epilogue(quant(x)[M,K] · w[N,K]^T) with
 * epilogue W8A8_EPI_BIAS (bias), W8A8_EPI_BIAS_RESID (bias then + residual,
 * residual may alias y) or W8A8_EPI_BIAS_GELU (bias then GELU). */
void dot_2d_int8_fused_cuda(const act_t *x, int M, int K, const qweight_t *w_int8,
                            const qscale_t *scale_w, const weight_t *bias, int N, act_t *y,
                            int epilogue, const act_t *residual, qweight_t *x_int8_scratch,
                            qscale_t *scale_x_scratch);

/* Causal attention of rows [0, n_tokens) of Q_d against one layer's
 * K_cache_d / V_cache_d ([ctx_len][d_model], heads interleaved by column),
 * written head-concatenated to out ([ctx_len][d_model]): the prefill branch
 * of gpt2.c:1205-1217 followed by concat_heads (gpt2.c:1286-1288). */
void attention_prefill_cuda(act_t *Q_d, act_t *k_cache_layer, act_t *v_cache_layer, int n_tokens,
                            act_t *out);

/* Attention of the single row n_tokens-1 of Q_d over cache rows
 * [0, n_tokens): the decode branch of gpt2.c:1191-1203 plus concat. The
 * workspace may be gpt2.c's scores_h_d buffer ([ctx_len][ctx_len] bf16),
 * which this path otherwise leaves unused. */
void attention_decode_cuda(act_t *Q_d, act_t *k_cache_layer, act_t *v_cache_layer, int n_tokens,
                           act_t *out, void *workspace, size_t workspace_bytes);

/* logits[vocab] = xf[d_model] · wte[vocab][d_model]^T, then the greedy token
 * of gpt2.c:2180-2222 (first index of the largest bf16 probability) into
 * *token_d (device int). wte is the untransposed embedding table. */
void lm_head_greedy_cuda(const act_t *xf, const weight_t *wte, act_t *logits, int *token_d);

/* The same LM head, then the token of gpt2.c:2223-2245 at temperature > 0:
 * top_k_sample (gpt2.c:130-180; top_k clamped to [1, vocab]) and the draw with
 * *r_d, a device float holding the host's (float)rand() / RAND_MAX. Among
 * equal probabilities the lower index comes first (the reference's qsort
 * leaves that order unspecified). temperature <= 0: the greedy token. */
void lm_head_topk_cuda(const act_t *xf, const weight_t *wte, act_t *logits, float temperature,
                       int top_k, const float *r_d, int *token_d);

#ifdef __cplusplus
}
#endif
