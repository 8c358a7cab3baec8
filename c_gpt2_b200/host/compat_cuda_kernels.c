/*
 * Drop-in implementation of include/cuda_kernels.h (the reference's kernel
 * ABI, include/cuda_kernels.h:1-85) on top of the sm_100a kernels. Compiled
 * once per model size (-DGPT2_{SMALL,MEDIUM,LARGE}_MODEL) into
 * libcuda_kernels_<size>.so, exactly as the reference compiles its cuda/ kernels per
 * size (Makefile:87-92).
 *
 * Conventions kept from the reference: void functions, legacy default stream,
 * empty shapes return early, any failure prints "FATAL <name> ..." to stderr
 * and aborts (cuda/activation_quant.cu:104-109).
 */
#include <stdio.h>
#include <stdlib.h>

/* gpt2_w8a8.h first: the size macros of gpt2_model_config.h (d_model, ...)
 * must not reach its declarations */
#include "../../include/gpt2_w8a8.h"
#include "../../include/cuda_kernels.h"

static void check(int st, const char *what, int a, int b) {
  if (st != W8A8_OK) {
    fprintf(stderr, "FATAL %s: %s (%d, %d)\n", what, w8a8_status_string(st), a, b);
    abort();
  }
}

void embeddings_cuda(weight_t (*wte_d)[d_model], weight_t (*wpe_d)[d_model], int *token_d,
                     act_t (*embeddings_d)[d_model], int start_row, int n_rows) {
  if (n_rows <= 0) return;
  check(w8a8_ref_embeddings((const gpt2_bf16_t *)wte_d, (const gpt2_bf16_t *)wpe_d, token_d,
                            (gpt2_bf16_t *)embeddings_d, d_model, start_row, n_rows, NULL),
        "embeddings_cuda", start_row, n_rows);
}

void layernorm_cuda(act_t (*input)[d_model], int n_tokens, int d_model_size, weight_t *gamma,
                    weight_t *beta, act_t (*output)[d_model], float eps) {
  (void)d_model_size;
  if (n_tokens <= 0) return;
  check(w8a8_layernorm_quant((const gpt2_bf16_t *)input, d_model, n_tokens, d_model,
                             (const gpt2_bf16_t *)gamma, (const gpt2_bf16_t *)beta, eps,
                             (gpt2_bf16_t *)output, d_model, NULL, NULL, NULL),
        "layernorm_cuda", n_tokens, d_model);
}

void add_bias_cuda(act_t *a, int a_r, int a_c, weight_t *b, act_t *out) {
  (void)out;
  check(w8a8_ref_add_bias((gpt2_bf16_t *)a, a_r, a_c, (const gpt2_bf16_t *)b, NULL),
        "add_bias_cuda", a_r, a_c);
}

void softmax_cuda(act_t *a, int a_r, int a_c, int stride, act_t *c_out, float temperature,
                  int causal_mask) {
  check(w8a8_ref_softmax((const gpt2_bf16_t *)a, a_r, a_c, stride, (gpt2_bf16_t *)c_out,
                         temperature, causal_mask, NULL),
        "softmax_cuda", a_r, a_c);
}

void casual_masking_cuda(act_t *in, int stride, int tokens) {
  check(w8a8_ref_causal_mask((gpt2_bf16_t *)in, stride, tokens, NULL), "casual_masking_cuda",
        stride, tokens);
}

void gelu_cuda(act_t *in, int cols, int rows, act_t *out) {
  (void)out;
  check(w8a8_ref_gelu((gpt2_bf16_t *)in, cols, rows, NULL), "gelu_cuda", rows, cols);
}

void concat_heads_cuda(act_t *src, act_t *dest, int token_index, int _nof_heads, int _head_dim,
                       int _ctx_len) {
  check(w8a8_ref_concat_heads((const gpt2_bf16_t *)src, (gpt2_bf16_t *)dest, token_index,
                              _nof_heads, _head_dim, _ctx_len, NULL),
        "concat_heads_cuda", token_index, _nof_heads);
}

void add_2d_cuda(act_t *a, int a_r, int a_c, act_t *b, act_t *out) {
  if (out == NULL) out = a;
  check(w8a8_ref_add_2d((const gpt2_bf16_t *)a, a_r, a_c, (const gpt2_bf16_t *)b,
                        (gpt2_bf16_t *)out, NULL),
        "add_2d_cuda", a_r, a_c);
}

void per_token_quant_cuda(const act_t *X, qweight_t *X_q, qscale_t *scale_X, int tokens, int d) {
  if (tokens <= 0) return;
  check(w8a8_quant_rows((const gpt2_bf16_t *)X, d, tokens, d, X_q, scale_X, NULL),
        "per_token_quant_cuda", tokens, d);
}

void dequant_int32_to_bf16_cuda(const int32_t *Y_int32, const qscale_t *scale_W,
                                const qscale_t *scale_X, act_t *Y_bf16, int M, int N) {
  if (M <= 0 || N <= 0) return;
  check(w8a8_ref_dequant(Y_int32, scale_W, scale_X, (gpt2_bf16_t *)Y_bf16, M, N, NULL),
        "dequant_int32_to_bf16_cuda", M, N);
}

void dot_2d_int8_fused_cuda(const act_t *x, int M, int K, const qweight_t *w_int8,
                            const qscale_t *scale_w, const weight_t *bias, int N, act_t *y,
                            int epilogue, const act_t *residual, qweight_t *x_int8_scratch,
                            qscale_t *scale_x_scratch) {
  if (M <= 0 || N <= 0) return;
  check(w8a8_quant_rows((const gpt2_bf16_t *)x, K, M, K, x_int8_scratch, scale_x_scratch, NULL),
        "dot_2d_int8_fused_cuda (quant)", M, K);
  check(w8a8_linear(x_int8_scratch, scale_x_scratch, M, K, w_int8, scale_w,
                    (const gpt2_bf16_t *)bias, N, epilogue, (const gpt2_bf16_t *)residual, N,
                    (gpt2_bf16_t *)y, N, NULL, 0, NULL),
        "dot_2d_int8_fused_cuda", M, N);
}

void attention_prefill_cuda(act_t *Q_d, act_t *k_cache_layer, act_t *v_cache_layer, int n_tokens,
                            act_t *out) {
  if (n_tokens <= 0) return;
  check(w8a8_attention_prefill((const gpt2_bf16_t *)Q_d, d_model,
                               (const gpt2_bf16_t *)k_cache_layer,
                               (const gpt2_bf16_t *)v_cache_layer, 0, 1, n_tokens, nof_heads,
                               head_dim, (gpt2_bf16_t *)out, d_model, NULL),
        "attention_prefill_cuda", n_tokens, d_model);
}

void attention_decode_cuda(act_t *Q_d, act_t *k_cache_layer, act_t *v_cache_layer, int n_tokens,
                           act_t *out, void *workspace, size_t workspace_bytes) {
  if (n_tokens <= 0) return;
  const int row = n_tokens - 1;
  /* the workspace is gpt2.c's score buffer, also used by other kernels:
   * clear the attention's ticket counters before each call */
  check(w8a8_attention_decode_workspace_reset(workspace, workspace_bytes, NULL),
        "attention_decode_cuda (workspace)", n_tokens, d_model);
  check(w8a8_attention_decode((const gpt2_bf16_t *)Q_d + (size_t)row * d_model, d_model,
                              (const gpt2_bf16_t *)k_cache_layer,
                              (const gpt2_bf16_t *)v_cache_layer, 0, 1, NULL, n_tokens, nof_heads,
                              head_dim, (gpt2_bf16_t *)out + (size_t)row * d_model, d_model,
                              workspace, workspace_bytes, NULL),
        "attention_decode_cuda", n_tokens, d_model);
}

void lm_head_greedy_cuda(const act_t *xf, const weight_t *wte, act_t *logits, int *token_d) {
  check(w8a8_lm_head((const gpt2_bf16_t *)xf, d_model, 1, d_model, (const gpt2_bf16_t *)wte,
                     vocab_size, (gpt2_bf16_t *)logits, vocab_size, NULL),
        "lm_head_greedy_cuda (lm head)", 1, vocab_size);
  check(w8a8_sample_greedy((const gpt2_bf16_t *)logits, vocab_size, 1, vocab_size, token_d, NULL,
                           0, NULL, NULL),
        "lm_head_greedy_cuda (sample)", 1, vocab_size);
}

void lm_head_topk_cuda(const act_t *xf, const weight_t *wte, act_t *logits, float temperature,
                       int top_k, const float *r_d, int *token_d) {
  check(w8a8_lm_head((const gpt2_bf16_t *)xf, d_model, 1, d_model, (const gpt2_bf16_t *)wte,
                     vocab_size, (gpt2_bf16_t *)logits, vocab_size, NULL),
        "lm_head_topk_cuda (lm head)", 1, vocab_size);
  check(w8a8_sample_topk((const gpt2_bf16_t *)logits, vocab_size, 1, vocab_size, temperature,
                         top_k, r_d, 0, NULL, token_d, NULL, 0, NULL, NULL, 0, NULL),
        "lm_head_topk_cuda (sample)", 1, vocab_size);
}
