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
 *
 * Loops over independent output elements (rows, channels, heads, vocabulary
 * entries) are spread over a small pthread pool (ORC_THREADS, default: the
 * online CPUs); every element is still computed by the same sequential
 * expression, so results do not depend on the thread count.
 */
#include "w8a8_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* fmaf() is a slow library call on a plain x86-64 build; the hot loops are
 * cloned for CPUs with an FMA unit (same IEEE results either way). */
#if defined(__x86_64__) && defined(__GNUC__)
#define ORC_HOT __attribute__((target_clones("arch=x86-64-v3", "default")))
#else
#define ORC_HOT
#endif

/* ---- parallel for over [0, n): a persistent pthread pool ----
 * fn(ctx, lo, hi) runs on contiguous chunks; the calling thread takes chunk 0.
 * One region at a time (a mutex); a forked child rebuilds the pool. */
typedef void (*orc_range_fn)(void *ctx, long lo, long hi);

#define ORC_MAX_THREADS 64
static struct {
  pthread_mutex_t region, mu;
  pthread_cond_t go, done;
  int nthreads;
  pid_t pid;
  unsigned long gen;
  int pending;
  orc_range_fn fn;
  void *ctx;
  long n, chunk;
} g_pool = {PTHREAD_MUTEX_INITIALIZER, PTHREAD_MUTEX_INITIALIZER, PTHREAD_COND_INITIALIZER,
            PTHREAD_COND_INITIALIZER, 0, 0, 0, 0, NULL, NULL, 0, 0};

static void pool_run_chunk(int i) {
  const long lo = (long)i * g_pool.chunk;
  long hi = lo + g_pool.chunk;
  if (hi > g_pool.n) hi = g_pool.n;
  if (lo < hi) g_pool.fn(g_pool.ctx, lo, hi);
}

static void *pool_worker(void *arg) {
  const int id = (int)(long)arg;
  unsigned long seen = 0;
  pthread_mutex_lock(&g_pool.mu);
  for (;;) {
    while (g_pool.gen == seen) pthread_cond_wait(&g_pool.go, &g_pool.mu);
    seen = g_pool.gen;
    pthread_mutex_unlock(&g_pool.mu);
    pool_run_chunk(id);
    pthread_mutex_lock(&g_pool.mu);
    if (--g_pool.pending == 0) pthread_cond_signal(&g_pool.done);
  }
  return NULL;
}

static void pool_start(void) {
  int t = 0;
  const char *env = getenv("ORC_THREADS");
  if (env) t = atoi(env);
  if (t <= 0) t = (int)sysconf(_SC_NPROCESSORS_ONLN);
  if (t < 1) t = 1;
  if (t > ORC_MAX_THREADS) t = ORC_MAX_THREADS;
  g_pool.nthreads = 1;
  g_pool.gen = 0;
  g_pool.pid = getpid();
  pthread_attr_t attr;
  pthread_attr_init(&attr);
  pthread_attr_setdetachstate(&attr, PTHREAD_CREATE_DETACHED);
  for (int i = 1; i < t; ++i) {
    pthread_t th;
    if (pthread_create(&th, &attr, pool_worker, (void *)(long)i) != 0) break;
    g_pool.nthreads = i + 1;
  }
  pthread_attr_destroy(&attr);
}

/* min_work: elements below which one thread does it all */
static void orc_parallel(long n, long min_work, orc_range_fn fn, void *ctx) {
  if (n <= 0) return;
  pthread_mutex_lock(&g_pool.region);
  if (g_pool.pid != getpid()) pool_start();
  const int workers = g_pool.nthreads;
  if (workers == 1 || n < min_work) {
    pthread_mutex_unlock(&g_pool.region);
    fn(ctx, 0, n);
    return;
  }
  pthread_mutex_lock(&g_pool.mu);
  g_pool.fn = fn;
  g_pool.ctx = ctx;
  g_pool.n = n;
  g_pool.chunk = (n + workers - 1) / workers;
  g_pool.pending = workers - 1;
  g_pool.gen++;
  pthread_cond_broadcast(&g_pool.go);
  pthread_mutex_unlock(&g_pool.mu);
  pool_run_chunk(0);
  pthread_mutex_lock(&g_pool.mu);
  while (g_pool.pending > 0) pthread_cond_wait(&g_pool.done, &g_pool.mu);
  pthread_mutex_unlock(&g_pool.mu);
  pthread_mutex_unlock(&g_pool.region);
}

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
typedef struct {
  const uint16_t *x;
  int K;
  int8_t *xq;
  float *sx;
} quant_job;

static void quant_range(void *ctx, long m0, long m1) {
  const quant_job *j = (const quant_job *)ctx;
  const int K = j->K;
  for (long m = m0; m < m1; ++m) {
    const uint16_t *row = j->x + (size_t)m * K;
    int8_t *xq = j->xq;
    float *sx = j->sx;
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

void orc_quant_rows(const uint16_t *x, int M, int K, int8_t *xq, float *sx) {
  quant_job j = {x, K, xq, sx};
  orc_parallel(M, 2, quant_range, &j);
}

/* ---- INT8 GEMM: the cublasGemmEx call of gpt2.c:404-415 ---- */
ORC_HOT static int32_t dot_i8(const int8_t *a, const int8_t *b, int K) {
  int32_t acc = 0;
  for (int k = 0; k < K; ++k) acc += (int32_t)a[k] * (int32_t)b[k];
  return acc;
}

typedef struct {
  const int8_t *xq, *W;
  int M, K, N;
  int32_t *Y;
} gemm_job;

static void gemm_range(void *ctx, long i0, long i1) {
  const gemm_job *j = (const gemm_job *)ctx;
  for (long i = i0; i < i1; ++i) {
    const long m = i / j->N, n = i % j->N;
    j->Y[i] = dot_i8(j->xq + (size_t)m * j->K, j->W + (size_t)n * j->K, j->K);
  }
}

void orc_gemm_s32(const int8_t *xq, int M, int K, const int8_t *W, int N, int32_t *Y) {
  gemm_job j = {xq, W, M, K, N, Y};
  orc_parallel((long)M * N, 4096, gemm_range, &j);
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
typedef struct {
  const int8_t *xq, *W;
  const float *sx, *sw;
  const uint16_t *bias, *R;
  int K, N, epi;
  uint16_t *Y;
} linear_job;

static void linear_range(void *ctx, long i0, long i1) {
  const linear_job *j = (const linear_job *)ctx;
  const int K = j->K, N = j->N, epi = j->epi;
  const float *sx = j->sx, *sw = j->sw;
  const uint16_t *bias = j->bias, *R = j->R;
  uint16_t *Y = j->Y;
  for (long i = i0; i < i1; ++i) {
    {
      const long m = i / N, n = i % N;
      const int32_t acc = dot_i8(j->xq + (size_t)m * K, j->W + (size_t)n * K, K);
      float t = dequant(acc, sw[n], sx[m]);
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
}

void orc_linear(const int8_t *xq, const float *sx, int M, int K, const int8_t *W,
                const float *sw, const uint16_t *bias, int N, int epi, const uint16_t *R,
                uint16_t *Y) {
  linear_job j = {xq, W, sx, sw, bias, R, K, N, epi, Y};
  orc_parallel((long)M * N, 4096, linear_range, &j);
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

typedef struct {
  const uint16_t *x, *gamma, *beta;
  int d;
  float eps;
  uint16_t *y;
} ln_job;

ORC_HOT static void ln_range(void *ctx, long m0, long m1) {
  const ln_job *j = (const ln_job *)ctx;
  const uint16_t *x = j->x, *gamma = j->gamma, *beta = j->beta;
  const int d = j->d;
  const float eps = j->eps;
  uint16_t *y = j->y;
  for (long m = m0; m < m1; ++m) {
    float s[1024];
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

void orc_layernorm(const uint16_t *x, int M, int d, const uint16_t *gamma, const uint16_t *beta,
                   float eps, uint16_t *y) {
  ln_job j = {x, gamma, beta, d, eps, y};
  orc_parallel(M, 2, ln_range, &j);
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
/* Order of the fp32 sums the reference leaves to cuBLAS (the attention dot
 * products and P.V, the LM head): 0 = ascending index (the oracle), 1 =
 * descending. The second order is just as valid a reading of the reference;
 * the tests use it to measure how far two valid orders drift apart. */
static int g_sum_order = 0;
void orc_set_sum_order(int order) { g_sum_order = order ? 1 : 0; }

ORC_HOT static void attend_row(const uint16_t *q, const uint16_t *K, const uint16_t *V, int64_t ld, int n,
                       uint16_t *o, uint16_t *srow, uint16_t *prow) {
  const int rev = g_sum_order;
  for (int j = 0; j < n; ++j) {
    const uint16_t *k = K + (int64_t)j * ld;
    float acc = 0.0f;
    for (int i = 0; i < 64; ++i) {
      const int c = rev ? 63 - i : i;
      acc = fmaf(orc_bf2f(q[c]), orc_bf2f(k[c]), acc);
    }
    srow[j] = orc_f2bf(acc * 0.125f);
  }
  orc_softmax_row(srow, n, 1.0f, prow);
  for (int c = 0; c < 64; ++c) {
    float acc = 0.0f;
    for (int i = 0; i < n; ++i) {
      const int j = rev ? n - 1 - i : i;
      acc = fmaf(orc_bf2f(prow[j]), orc_bf2f(V[(int64_t)j * ld + c]), acc);
    }
    o[c] = orc_f2bf(acc);
  }
}

typedef struct {
  const uint16_t *Q, *K, *V;
  int q0, nq, n_head;
  uint16_t *O;
} attn_job;

/* work item w: head w % n_head of row r = w / n_head taken in the order
 * 0, nq-1, 1, nq-2, ..., so that every contiguous chunk of items mixes short
 * and long causal rows */
static void attn_range(void *ctx, long w0, long w1) {
  const attn_job *j = (const attn_job *)ctx;
  const int d = j->n_head * 64;
  const int nmax = j->q0 + j->nq;
  uint16_t *srow = (uint16_t *)malloc((size_t)nmax * 2);
  uint16_t *prow = (uint16_t *)malloc((size_t)nmax * 2);
  for (long w = w0; w < w1; ++w) {
    const int h = (int)(w % j->n_head), r = (int)(w / j->n_head);
    const int i = (r & 1) ? j->nq - 1 - r / 2 : r / 2;
    attend_row(j->Q + (size_t)i * d + h * 64, j->K + h * 64, j->V + h * 64, d, j->q0 + i + 1,
               j->O + (size_t)i * d + h * 64, srow, prow);
  }
  free(srow);
  free(prow);
}

/* Causal attention for rows [q0, q0+nq) of one sequence whose K/V cache rows
 * are [0, q0+nq). Q/O rows have stride d; K/V rows stride d. */
void orc_attention(const uint16_t *Q, const uint16_t *K, const uint16_t *V, int q0, int nq,
                   int n_head, uint16_t *O) {
  attn_job j = {Q, K, V, q0, nq, n_head, O};
  orc_parallel((long)nq * n_head, 2, attn_range, &j);
}

/* ---- LM head: gpt2.c:2160 (bf16 GEMM, fp32 sums) ---- */
typedef struct {
  const uint16_t *xf, *wte;
  int d;
  uint16_t *logits;
} lm_job;

/* blocks [b0, b1) of eight vocabulary rows */
ORC_HOT static void lm_range(void *ctx, long b0, long b1) {
  const lm_job *j = (const lm_job *)ctx;
  const uint16_t *xf = j->xf, *wte = j->wte;
  const int d = j->d;
  uint16_t *logits = j->logits;
  const int rev = g_sum_order;
  for (long v = 8 * b0; v < 8 * b1; v += 8) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int i = 0; i < d; ++i) {
      const int k = rev ? d - 1 - i : i;
      const float x = orc_bf2f(xf[k]);
      for (int r = 0; r < 8; ++r) acc[r] = fmaf(x, orc_bf2f(wte[(size_t)(v + r) * d + k]), acc[r]);
    }
    for (int r = 0; r < 8; ++r) logits[v + r] = orc_f2bf(acc[r]);
  }
}

ORC_HOT void orc_lm_head(const uint16_t *xf, int d, const uint16_t *wte, int V, uint16_t *logits) {
  /* eight vocabulary rows at a time: independent sums, each still in k order */
  const int V8 = V & ~7;
  lm_job j = {xf, wte, d, logits};
  orc_parallel(V8 / 8, 64, lm_range, &j);
  for (int v = V8; v < V; ++v) {
    const uint16_t *w = wte + (size_t)v * d;
    float acc = 0.0f;
    for (int i = 0; i < d; ++i) {
      const int k = g_sum_order ? d - 1 - i : i;
      acc = fmaf(orc_bf2f(xf[k]), orc_bf2f(w[k]), acc);
    }
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
  return orc_generate_steps(image, bytes, d, L, H, vocab, ctx, prompt, T, n_gen, out, last_logits,
                            NULL);
}

/* As orc_generate; step_logits (optional, [n_gen][vocab] bf16) receives the
 * logits every generated token was picked from. */
int orc_generate_steps(const uint8_t *image, size_t bytes, int d, int L, int H, int vocab,
                       int ctx, const int32_t *prompt, int T, int n_gen, int32_t *out,
                       uint16_t *last_logits, uint16_t *step_logits) {
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
    if (step_logits) memcpy(step_logits + (size_t)g * vocab, logits, (size_t)vocab * 2);
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
