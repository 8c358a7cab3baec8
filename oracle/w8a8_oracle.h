/* CPU oracle of the reference's W8A8 GPT-2 GPU path. Test infrastructure
 * only — see w8a8_oracle.c. bf16 values are raw 16-bit patterns. */
#ifndef W8A8_ORACLE_H
#define W8A8_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#define ORC_EPI_DEQUANT 0
#define ORC_EPI_BIAS 1
#define ORC_EPI_BIAS_RESID 2
#define ORC_EPI_BIAS_GELU 3

float orc_bf2f(uint16_t v);
uint16_t orc_f2bf(float f);
void orc_quant_rows(const uint16_t *x, int M, int K, int8_t *xq, float *sx);
void orc_gemm_s32(const int8_t *xq, int M, int K, const int8_t *W, int N, int32_t *Y);
float orc_gelu(float val);
void orc_linear(const int8_t *xq, const float *sx, int M, int K, const int8_t *W,
                const float *sw, const uint16_t *bias, int N, int epi, const uint16_t *R,
                uint16_t *Y);
void orc_layernorm(const uint16_t *x, int M, int d, const uint16_t *gamma,
                   const uint16_t *beta, float eps, uint16_t *y);
void orc_softmax_row(const uint16_t *in, int n, float temperature, uint16_t *out);
void orc_attention(const uint16_t *Q, const uint16_t *K, const uint16_t *V, int q0, int nq,
                   int n_head, uint16_t *O);
void orc_lm_head(const uint16_t *xf, int d, const uint16_t *wte, int V, uint16_t *logits);
int orc_greedy(const uint16_t *logits, int V);
void orc_top_k(const uint16_t *probs, int V, int k, int *idx, uint16_t *q);
int orc_sample_topk(const uint16_t *probs, int V, int k, float r);
int orc_generate(const uint8_t *image, size_t bytes, int d, int L, int H, int vocab, int ctx,
                 const int32_t *prompt, int T, int n_gen, int32_t *out, uint16_t *last_logits);
void orc_set_sum_order(int order);
int orc_generate_steps(const uint8_t *image, size_t bytes, int d, int L, int H, int vocab,
                       int ctx, const int32_t *prompt, int T, int n_gen, int32_t *out,
                       uint16_t *last_logits, uint16_t *step_logits);

#endif
