/*
 * CPU oracle: a plain-C restatement of the reference's W8A8 GPT-2 GPU path
 * (roeybenhayun/c_gpt2, USE_GPU + USE_BF16 + USE_INT8 build).
 *
 * TEST INFRASTRUCTURE ONLY. The tests, the smoke check and the benchmark's
 * CPU-baseline leg call this as the checker; the product path never links or
 * calls it.
 *
 * Each function follows the reference operation by operation and cites the
 * file:line it restates. fp32 arithmetic is written out explicitly (built
 * with -ffp-contract=off): where nvcc contracts a multiply-add in the
 * reference kernel, fmaf() is used here. Two places cannot be bit-exact on a
 * CPU and are compared within tolerance by the tests: the GPU's
 * approximate rsqrtf in LayerNorm (1/sqrtf here) and the CUDA math library's
 * expf/tanhf (C library versions here). The cuBLAS GEMMs of the reference
 * (INT8 -> exact integers; bf16 attention and LM head -> fp32 sums in an
 * unspecified order) are restated as sequential sums.
 */
#include "w8a8_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* fmaf() is a slow library call on a plain x86-64 build; the hot loops are
 * cloned for CPUs with an FMA unit (same IEEE results either way). */
#if defined(__x86_64__) && defined(__GNUC__)
#define ORC_HOT __attribute__((target_clones("arch=x86-64-v3", "default")))
#else
#define ORC_HOT
#endif

/* ---- bf16 ---- */
float orc_bf2f(uint16_t v) {
  uint32_t u = (uint32_t)v << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}
/* round to nearest, ties to even (the conversion __float2bfloat16 performs) */
uint16_t orc_f2bf(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
static float rbf(float f) { return orc_bf2f(orc_f2bf(f)); }

/* ---- per-token quantization: cuda/activation_quant.cu:54-91 ---- */
void orc_quant_rows(const uint16_t *x, int M, int K, int8_t *xq, float *sx) {
  for (int m = 0; m < M; ++m) {
    const uint16_t *row = x + (size_t)m * K;
    float amax = 0.0f;
    for (int k = 0; k < K; ++k) amax = fmaxf(amax, fabsf(orc_bf2f(row[k])));
    const float scale = amax > 0.0f ? amax / 127.0f : 1.0f;
    const float inv = 1.0f / scale;
    sx[m] = scale;
    for (int k = 0; k < K; ++k) {
      float v = orc_bf2f(row[k]) * inv;
      int q = (int)nearbyintf(v); /* __float2int_rn: round half to even */
      if (q > 127) q = 127;
      if (q < -127) q = -127;
      xq[(size_t)m * K + k] = (int8_t)q;
    }
  }
}

/* ---- INT8 GEMM: the cublasGemmEx call of gpt2.c:404-415 ---- */
ORC_HOT void orc_gemm_s32(const int8_t *xq, int M, int K, const int8_t *W, int N, int32_t *Y) {
  for (int m = 0; m < M; ++m) {
    const int8_t *a = xq + (size_t)m * K;
    for (int n = 0; n < N; ++n) {
      const int8_t *b = W + (size_t)n * K;
      int32_t acc = 0;
      for (int k = 0; k < K; ++k) acc += (int32_t)a[k] * (int32_t)b[k];
      Y[(size_t)m * N + n] = acc;
    }
  }
}

/* dequant_int32_to_bf16_kernel (activation_quant.cu:128-130) */
static float dequant(int32_t acc, float sw, float sx) { return rbf(((float)acc * sw) * sx); }

/* ---- GELU: cuda/gelu.cu:10-15 with nvcc's contraction of
 * val + (0.044715f*val*val)*val into one fused multiply-add ---- */
float orc_gelu(float val) {
  const float term = 0.79788456f;
  const float c = fmaf((0.044715f * val) * val, val, val);
  return (0.5f * val) * (1.0f + tanhf(term * c));
}

/* ---- fused linear epilogues:
 * dequant (activation_quant.cu:129) -> add_bias (add_bias.cu:14)
 * -> add_2d residual (add_2d.cu:14) or gelu (gelu.cu:12-16) ---- */
void orc_linear(const int8_t *xq, const float *sx, int M, int K, const int8_t *W,
                const float *sw, const uint16_t *bias, int N, int epi, const uint16_t *R,
                uint16_t *Y) {
  int32_t *acc = (int32_t *)malloc((size_t)N * sizeof(int32_t));
  for (int m = 0; m < M; ++m) {
    orc_gemm_s32(xq + (size_t)m * K, 1, K, W, N, acc);
    for (int n = 0; n < N; ++n) {
      float t = dequant(acc[n], sw[n], sx[m]);
      float out;
      if (epi == ORC_EPI_DEQUANT) {
        out = t;
      } else {
        float y = rbf(t + orc_bf2f(bias[n]));
        if (epi == ORC_EPI_BIAS)
          out = y;
        else if (epi == ORC_EPI_BIAS_RESID)
          out = rbf(orc_bf2f(R[(size_t)m * N + n]) + y);
        else
          out = rbf(orc_gelu(y));
      }
      Y[(size_t)m * N + n] = orc_f2bf(out);
    }
  }
  free(acc);
}

/* ---- LayerNorm: cuda/layernorm.cu:23-77 ----
 * 1024-thread block: thread t sums elements t, t+1024, ... in order, the
 * 1024 partials fold pairwise (s = 512 .. 1); the variance pass contracts
 * diff*diff into the running sum (fmaf). rsqrtf -> 1/sqrtf (tolerance). */
static float tree1024(float *s) {
  for (int h = 512; h > 0; h >>= 1)
    for (int t = 0; t < h; ++t) s[t] = s[t] + s[t + h];
  return s[0];
}

ORC_HOT void orc_layernorm(const uint16_t *x, int M, int d, const uint16_t *gamma,
                   const uint16_t *beta, float eps, uint16_t *y) {
  float s[1024];
  for (int m = 0; m < M; ++m) {
    const uint16_t *row = x + (size_t)m * d;
    for (int t = 0; t < 1024; ++t) {
      float sum = 0.0f;
      for (int i = t; i < d; i += 1024) sum = sum + orc_bf2f(row[i]);
      s[t] = sum;
    }
    const float mean = tree1024(s) / (float)d;
    for (int t = 0; t < 1024; ++t) {
      float acc = 0.0f;
      for (int i = t; i < d; i += 1024) {
        float diff = orc_bf2f(row[i]) - mean;
        acc = fmaf(diff, diff, acc);
      }
      s[t] = acc;
    }
    const float var = tree1024(s) / (float)d;
    const float inv_std = 1.0f / sqrtf(var + eps);
    for (int i = 0; i < d; ++i) {
      float normalized = (orc_bf2f(row[i]) - mean) * inv_std;
      y[(size_t)m * d + i] = orc_f2bf(fmaf(normalized, orc_bf2f(gamma[i]), orc_bf2f(beta[i])));
    }
  }
}

/* ---- softmax row: cuda/softmax.cu:31-91 (temperature t, 256-thread tree) ----
 * Writes bf16 probabilities for columns [0, n) of `in` to `out`. */
void orc_softmax_row(const uint16_t *in, int n, float temperature, uint16_t *out) {
  const float inv_temp = 1.0f / temperature;
  float mx = -INFINITY;
  for (int j = 0; j < n; ++j) {
    float v = orc_bf2f(in[j]) * inv_temp;
    if (v > mx) mx = v;
  }
  float s[256];
  uint16_t *e16 = (uint16_t *)malloc((size_t)n * 2);
  for (int t = 0; t < 256; ++t) {
    float acc = 0.0f;
    for (int j = t; j < n; j += 256) {
      float e = expf(fmaf(orc_bf2f(in[j]), inv_temp, -mx));
      e16[j] = orc_f2bf(e);
      acc = acc + e;
    }
    s[t] = acc;
  }
  for (int h = 128; h > 0; h >>= 1)
    for (int t = 0; t < h; ++t) s[t] = s[t] + s[t + h];
  const float inv_sum = 1.0f / s[0];
  for (int j = 0; j < n; ++j) out[j] = orc_f2bf(orc_bf2f(e16[j]) * inv_sum);
  free(e16);
}

/* ---- attention of one query row over keys [0, n) of one head:
 * gpt2.c:1191-1203 / 1205-1217 (S = bf16(alpha*q.k), alpha = 1/sqrt(64);
 * softmax_cuda; O = bf16(P.V)); sums in key/dim order with fmaf ---- */
ORC_HOT static void attend_row(const uint16_t *q, const uint16_t *K, const uint16_t *V, int64_t ld, int n,
                       uint16_t *o, uint16_t *srow, uint16_t *prow) {
  for (int j = 0; j < n; ++j) {
    const uint16_t *k = K + (int64_t)j * ld;
    float acc = 0.0f;
    for (int c = 0; c < 64; ++c) acc = fmaf(orc_bf2f(q[c]), orc_bf2f(k[c]), acc);
    srow[j] = orc_f2bf(acc * 0.125f);
  }
  orc_softmax_row(srow, n, 1.0f, prow);
  for (int c = 0; c < 64; ++c) {
    float acc = 0.0f;
    for (int j = 0; j < n; ++j) acc = fmaf(orc_bf2f(prow[j]), orc_bf2f(V[(int64_t)j * ld + c]), acc);
    o[c] = orc_f2bf(acc);
  }
}

/* Causal attention for rows [q0, q0+nq) of one sequence whose K/V cache rows
 * are [0, q0+nq). Q/O rows have stride d; K/V rows stride d. */
void orc_attention(const uint16_t *Q, const uint16_t *K, const uint16_t *V, int q0, int nq,
                   int n_head, uint16_t *O) {
  const int d = n_head * 64;
  const int nmax = q0 + nq;
  uint16_t *srow = (uint16_t *)malloc((size_t)nmax * 2);
  uint16_t *prow = (uint16_t *)malloc((size_t)nmax * 2);
  for (int i = 0; i < nq; ++i)
    for (int h = 0; h < n_head; ++h)
      attend_row(Q + (size_t)i * d + h * 64, K + h * 64, V + h * 64, d, q0 + i + 1,
                 O + (size_t)i * d + h * 64, srow, prow);
  free(srow);
  free(prow);
}

/* ---- LM head: gpt2.c:2160 (bf16 GEMM, fp32 sums) ---- */
ORC_HOT void orc_lm_head(const uint16_t *xf, int d, const uint16_t *wte, int V, uint16_t *logits) {
  /* eight vocabulary rows at a time: independent sums, each still in k order */
  int v = 0;
  for (; v + 8 <= V; v += 8) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int k = 0; k < d; ++k) {
      const float x = orc_bf2f(xf[k]);
      for (int r = 0; r < 8; ++r) acc[r] = fmaf(x, orc_bf2f(wte[(size_t)(v + r) * d + k]), acc[r]);
    }
    for (int r = 0; r < 8; ++r) logits[v + r] = orc_f2bf(acc[r]);
  }
  for (; v < V; ++v) {
    const uint16_t *w = wte + (size_t)v * d;
    float acc = 0.0f;
    for (int k = 0; k < d; ++k) acc = fmaf(orc_bf2f(xf[k]), orc_bf2f(w[k]), acc);
    logits[v] = orc_f2bf(acc);
  }
}

/* ---- greedy pick: softmax_cuda at temperature 1 (gpt2.c:2180-2182) then the
 * host argmax over bf16 probabilities, first index wins (gpt2.c:2214-2222) */
int orc_greedy(const uint16_t *logits, int V) {
  uint16_t *p = (uint16_t *)malloc((size_t)V * 2);
  orc_softmax_row(logits, V, 1.0f, p);
  float best = -1.0f;
  int tok = -1;
  for (int v = 0; v < V; ++v) {
    float pv = orc_bf2f(p[v]);
    if (pv > best) {
      best = pv;
      tok = v;
    }
  }
  free(p);
  return tok;
}

/* ---- top-k sampling: gpt2.c:130-180 (top_k_sample) and the draw of
 * gpt2.c:2223-2245. (probability, index) pairs sorted by descending
 * probability; the reference's qsort (compareTokenProbs, gpt2.c:102-113)
 * leaves the order of equal probabilities unspecified, this sort puts the
 * lower index first. k is clamped to [1, V] as gpt2.c:1963-1968 does. ---- */
typedef struct {
  float prob;
  int index;
} orc_tokprob;

static int cmp_tokprob(const void *a, const void *b) {
  const orc_tokprob *x = (const orc_tokprob *)a, *y = (const orc_tokprob *)b;
  if (x->prob < y->prob) return 1;
  if (x->prob > y->prob) return -1;
  return (x->index > y->index) - (x->index < y->index);
}

/* idx[k], q[k] (bf16): the top k tokens and their renormalised probabilities */
void orc_top_k(const uint16_t *probs, int V, int k, int *idx, uint16_t *q) {
  if (k < 1) k = 1;
  if (k > V) k = V;
  orc_tokprob *t = (orc_tokprob *)malloc((size_t)V * sizeof(orc_tokprob));
  for (int i = 0; i < V; ++i) {
    t[i].prob = orc_bf2f(probs[i]);
    t[i].index = i;
  }
  qsort(t, (size_t)V, sizeof(orc_tokprob), cmp_tokprob);
  float sum = 0.0f;
  for (int i = 0; i < k; ++i) {
    idx[i] = t[i].index;
    q[i] = orc_f2bf(t[i].prob);
    sum += t[i].prob;
  }
  if (sum > 0.0f) {
    for (int i = 0; i < k; ++i) q[i] = orc_f2bf(orc_bf2f(q[i]) / sum);
  } else {
    for (int i = 0; i < k; ++i) q[i] = orc_f2bf(1.0f / (float)k);
  }
  free(t);
}

/* the token drawn with r from the bf16 probabilities of one row */
int orc_sample_topk(const uint16_t *probs, int V, int k, float r) {
  if (k < 1) k = 1;
  if (k > V) k = V;
  int *idx = (int *)malloc((size_t)k * sizeof(int));
  uint16_t *q = (uint16_t *)malloc((size_t)k * 2);
  orc_top_k(probs, V, k, idx, q);
  int tok = idx[k - 1];
  float cum = 0.0f;
  for (int i = 0; i < k; ++i) {
    cum += orc_bf2f(q[i]);
    if (r < cum) {
      tok = idx[i];
      break;
    }
  }
  free(idx);
  free(q);
  return tok;
}

/* ---------------------------------------------------------------------------
 * Whole-model greedy generation from a quant8 image (one sequence), following
 * the INT8 GPU forward of gpt2.c:1124-1330 and the token loop 2094-2247.
 * ------------------------------------------------------------------------- */
typedef struct {
  const float *ln1_g, *ln1_b, *bqkv, *bproj, *ln2_g, *ln2_b, *b1, *b2;
  const int8_t *Wqkv, *Wproj, *W1, *W2;
  const float *sqkv, *sproj, *s1, *s2;
} orc_layer;

static size_t pad16(size_t n) { return (n + 15) & ~(size_t)15; }

static uint16_t *to_bf16(const float *src, size_t n) {
  uint16_t *dst = (uint16_t *)malloc(n * 2);
  for (size_t i = 0; i < n; ++i) dst[i] = orc_f2bf(src[i]);
  return dst;
}

int orc_generate(const uint8_t *image, size_t bytes, int d, int L, int H, int vocab, int ctx,
                 const int32_t *prompt, int T, int n_gen, int32_t *out, uint16_t *last_logits) {
  if (T <= 0 || n_gen <= 0 || T + n_gen - 1 > ctx || d != H * 64) return -1;
  const int f = 4 * d;
  size_t off = 0;
#define TAKE(ptr, type, count)                               \
  do {                                                       \
    size_t nb_ = (size_t)(count) * sizeof(type);             \
    if (off + nb_ > bytes) return -2;                        \
    (ptr) = (const type *)(image + off);                     \
    off += pad16(nb_);                                       \
  } while (0)
  const float *wte32, *wpe32, *lnf_g, *lnf_b;
  orc_layer *ly = (orc_layer *)calloc((size_t)L, sizeof(orc_layer));
  TAKE(wte32, float, (size_t)vocab * d);
  TAKE(wpe32, float, (size_t)ctx * d);
  for (int l = 0; l < L; ++l) {
    orc_layer *w = &ly[l];
    TAKE(w->ln1_g, float, d);
    TAKE(w->ln1_b, float, d);
    TAKE(w->Wqkv, int8_t, (size_t)3 * d * d);
    TAKE(w->sqkv, float, 3 * d);
    TAKE(w->bqkv, float, 3 * d);
    TAKE(w->Wproj, int8_t, (size_t)d * d);
    TAKE(w->sproj, float, d);
    TAKE(w->bproj, float, d);
    TAKE(w->ln2_g, float, d);
    TAKE(w->ln2_b, float, d);
    TAKE(w->W1, int8_t, (size_t)f * d);
    TAKE(w->s1, float, f);
    TAKE(w->b1, float, f);
    TAKE(w->W2, int8_t, (size_t)d * f);
    TAKE(w->s2, float, d);
    TAKE(w->b2, float, d);
  }
  TAKE(lnf_g, float, d);
  TAKE(lnf_b, float, d);
#undef TAKE
  /* FP32 -> bf16 at load (gpt2.c:1613-1628) */
  uint16_t *wte = to_bf16(wte32, (size_t)vocab * d);
  uint16_t *wpe = to_bf16(wpe32, (size_t)ctx * d);
  uint16_t **lb = (uint16_t **)calloc((size_t)L * 8, sizeof(uint16_t *));
  for (int l = 0; l < L; ++l) {
    lb[l * 8 + 0] = to_bf16(ly[l].ln1_g, d);
    lb[l * 8 + 1] = to_bf16(ly[l].ln1_b, d);
    lb[l * 8 + 2] = to_bf16(ly[l].bqkv, 3 * d);
    lb[l * 8 + 3] = to_bf16(ly[l].bproj, d);
    lb[l * 8 + 4] = to_bf16(ly[l].ln2_g, d);
    lb[l * 8 + 5] = to_bf16(ly[l].ln2_b, d);
    lb[l * 8 + 6] = to_bf16(ly[l].b1, f);
    lb[l * 8 + 7] = to_bf16(ly[l].b2, d);
  }
  uint16_t *gf = to_bf16(lnf_g, d), *bf = to_bf16(lnf_b, d);

  const int maxrows = T > 1 ? T : 1;
  uint16_t *Kc = (uint16_t *)calloc((size_t)L * ctx * d, 2);
  uint16_t *Vc = (uint16_t *)calloc((size_t)L * ctx * d, 2);
  uint16_t *h = (uint16_t *)malloc((size_t)maxrows * d * 2);
  uint16_t *xn = (uint16_t *)malloc((size_t)maxrows * d * 2);
  uint16_t *qkv = (uint16_t *)malloc((size_t)maxrows * 3 * d * 2);
  uint16_t *att = (uint16_t *)malloc((size_t)maxrows * d * 2);
  uint16_t *r1 = (uint16_t *)malloc((size_t)maxrows * d * 2);
  uint16_t *x1 = (uint16_t *)malloc((size_t)maxrows * f * 2);
  int8_t *xq = (int8_t *)malloc((size_t)maxrows * f);
  float *sx = (float *)malloc((size_t)maxrows * 4);
  uint16_t *Q = (uint16_t *)malloc((size_t)maxrows * d * 2);
  uint16_t *logits = (uint16_t *)malloc((size_t)vocab * 2);
  uint16_t *xf = (uint16_t *)malloc((size_t)d * 2);
  int32_t *toks = (int32_t *)malloc((size_t)(T + n_gen) * 4);
  memcpy(toks, prompt, (size_t)T * 4);
  int cur = T, start = 0;
  const float eps = 1e-5f;
  for (int g = 0; g < n_gen; ++g) {
    const int nrows = cur - start; /* T in prefill, 1 in decode */
    /* embeddings (embeddings.cu:18-23) */
    for (int i = 0; i < nrows; ++i) {
      const int pos = start + i, tok = toks[pos];
      for (int c = 0; c < d; ++c)
        h[(size_t)i * d + c] =
            orc_f2bf(orc_bf2f(wte[(size_t)tok * d + c]) + orc_bf2f(wpe[(size_t)pos * d + c]));
    }
    for (int l = 0; l < L; ++l) {
      const orc_layer *w = &ly[l];
      uint16_t *Kl = Kc + (size_t)l * ctx * d, *Vl = Vc + (size_t)l * ctx * d;
      orc_layernorm(h, nrows, d, lb[l * 8 + 0], lb[l * 8 + 1], eps, xn);
      orc_quant_rows(xn, nrows, d, xq, sx);
      orc_linear(xq, sx, nrows, d, w->Wqkv, w->sqkv, lb[l * 8 + 2], 3 * d, ORC_EPI_BIAS, NULL, qkv);
      for (int i = 0; i < nrows; ++i) {
        memcpy(Q + (size_t)i * d, qkv + (size_t)i * 3 * d, (size_t)d * 2);
        memcpy(Kl + (size_t)(start + i) * d, qkv + (size_t)i * 3 * d + d, (size_t)d * 2);
        memcpy(Vl + (size_t)(start + i) * d, qkv + (size_t)i * 3 * d + 2 * d, (size_t)d * 2);
      }
      orc_attention(Q, Kl, Vl, start, nrows, H, att);
      orc_quant_rows(att, nrows, d, xq, sx);
      orc_linear(xq, sx, nrows, d, w->Wproj, w->sproj, lb[l * 8 + 3], d, ORC_EPI_BIAS_RESID, h, r1);
      orc_layernorm(r1, nrows, d, lb[l * 8 + 4], lb[l * 8 + 5], eps, xn);
      orc_quant_rows(xn, nrows, d, xq, sx);
      orc_linear(xq, sx, nrows, d, w->W1, w->s1, lb[l * 8 + 6], f, ORC_EPI_BIAS_GELU, NULL, x1);
      orc_quant_rows(x1, nrows, f, xq, sx);
      orc_linear(xq, sx, nrows, f, w->W2, w->s2, lb[l * 8 + 7], d, ORC_EPI_BIAS_RESID, r1, h);
    }
    /* final LN on the last row, LM head, greedy (gpt2.c:2150-2222) */
    orc_layernorm(h + (size_t)(nrows - 1) * d, 1, d, gf, bf, eps, xf);
    orc_lm_head(xf, d, wte, vocab, logits);
    const int tok = orc_greedy(logits, vocab);
    out[g] = tok;
    toks[cur] = tok;
    start = cur;
    cur += 1;
  }
  if (last_logits) memcpy(last_logits, logits, (size_t)vocab * 2);
  free(toks); free(xf); free(logits); free(Q); free(sx); free(xq); free(x1); free(r1);
  free(att); free(qkv); free(xn); free(h); free(Kc); free(Vc);
  for (int i = 0; i < L * 8; ++i) free(lb[i]);
  free(lb); free(gf); free(bf); free(wte); free(wpe); free(ly);
  return 0;
}
