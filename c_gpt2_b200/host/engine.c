/*
 * Batched W8A8 GPT-2 inference host engine (C). See include/gpt2_engine.h.
 *
 * Per layer, the reference runs 3 quant+GEMM+dequant triplets for Q/K/V, 3
 * bias adds, H x (QK^T, softmax, PV), concat, and 5 more launch groups for
 * the projection / MLP (gpt2.c:1124-1330). Here a prefill layer is 9
 * launches:
 *
 *   LN1+quant -> QKV GEMM (dequant, bias, scatter into Q and the KV cache)
 *   -> attention -> quant -> proj GEMM (dequant, bias, residual)
 *   -> LN2+quant -> W1 GEMM (dequant, bias, GELU) -> quant
 *   -> W2 GEMM (dequant, bias, residual)
 *
 * and a decode layer 8 (the attention kernel quantizes its own output), with
 * the first LN1 fused into the embedding gather. Each intermediate is
 * rounded to bf16 where the reference rounds it, so every output element is
 * the reference's value for the same inputs (see gpt2_w8a8.h).
 */
#include "../../include/gpt2_engine.h"

#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define ALIGN_UP(x, a) (((x) + ((size_t)(a)-1)) & ~((size_t)(a)-1))

typedef struct {
  gpt2_bf16_t *ln1_g, *ln1_b, *bqkv, *bproj, *ln2_g, *ln2_b, *b1, *b2;
  int8_t *Wqkv, *Wproj, *W1, *W2;
  float *sWqkv, *sWproj, *sW1, *sW2;
} layer_w;

struct gpt2_engine {
  gpt2_engine_config cfg;
  int device;
  cudaStream_t stream;
  char err[256];
  /* weights */
  void *wblob;
  size_t wbytes;
  gpt2_bf16_t *wte, *wpe, *lnf_g, *lnf_b;
  layer_w *layers;
  int loaded;
  /* KV cache [max_batch][L][ctx][d] */
  gpt2_bf16_t *Kc, *Vc;
  /* activations */
  void *ablob;
  gpt2_bf16_t *H, *R1, *Q, *ATT, *X1, *Xf, *logits;
  int8_t *Xq;
  float *sX;
  int32_t *len, *nctx, *gen, *next, *tokens_in, *out_default;
  void *attn_ws;
  size_t attn_ws_bytes;
  void *lin_ws; /* split-K workspace of the decode-sized GEMMs (zeroed) */
  size_t lin_ws_bytes;
  /* the second half of a split decode step: its own stream and workspaces */
  cudaStream_t stream2;
  cudaEvent_t ev_fork, ev_join;
  void *attn_ws2, *lin_ws2;
  /* row absmax records of the decode W1 -> W2 pair (one per half) */
  float *amax_rec, *amax_rec2;
  size_t amax_rec_floats;
  int decode_split; /* 1: one chain of B rows; 2: two chains of B/2 rows on two streams */
  /* current batch: B slots (rows) of the decode step */
  int B;
  int32_t *out;
  int out_stride;
  /* host mirror of each slot's device counters (len: cache rows filled,
   * gen: tokens written to its output row); active: the slot holds a
   * sequence whose tokens are wanted (else it is parked and its steps are
   * discarded) */
  int *slot_len, *slot_gen, *slot_active;
  /* sampling: temperature <= 0 greedy, else top-k at that temperature with
   * the draws of slot b in rnd[b*ctx ...], indexed by the slot's output count */
  float temperature;
  int top_k;
  float *rnd;
  /* decode graph */
  int use_graphs;
  cudaGraphExec_t graph;
  int graph_B, graph_stride, graph_split;
  int32_t *graph_out;
};

static int fail(gpt2_engine *e, int st, const char *fmt, ...) {
  if (e) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(e->err, sizeof e->err, fmt, ap);
    va_end(ap);
  }
  return st;
}

#define CUDA_TRY(e, call)                                                           \
  do {                                                                              \
    cudaError_t err__ = (call);                                                     \
    if (err__ != cudaSuccess)                                                       \
      return fail((e), W8A8_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(err__)); \
  } while (0)

#define W8_TRY(e, call)                                                          \
  do {                                                                           \
    int st__ = (call);                                                           \
    if (st__ != W8A8_OK)                                                         \
      return fail((e), st__, "%s: %s", #call, w8a8_status_string(st__));         \
  } while (0)

const char *gpt2_engine_last_error(const gpt2_engine *e) { return e ? e->err : "null engine"; }
void *gpt2_engine_stream(gpt2_engine *e) { return e ? (void *)e->stream : NULL; }

static int cfg_ok(const gpt2_engine_config *c) {
  return c && c->d_model > 0 && c->n_layer > 0 && c->n_head > 0 && c->d_model % c->n_head == 0 &&
         c->d_model / c->n_head == 64 && c->d_model % 16 == 0 && c->vocab > 0 && c->ctx > 0 &&
         c->ctx <= 1024 && c->max_batch > 0 && c->max_tokens >= c->max_batch;
}

/* ---- quant8.bin layout (writer.py: every block padded to 16 bytes) ---- */
static size_t blk(size_t bytes) { return ALIGN_UP(bytes, 16); }

size_t gpt2_engine_quant8_bytes(const gpt2_engine_config *c) {
  if (!c) return 0;
  const size_t d = c->d_model, f = 4 * d;
  size_t n = blk((size_t)c->vocab * d * 4) + blk((size_t)c->ctx * d * 4);
  size_t per = 0;
  per += 2 * blk(d * 4);                          /* ln1 */
  per += blk(3 * d * d) + blk(3 * d * 4);         /* W_qkv + scale */
  per += blk(3 * d * 4);                          /* b_qkv */
  per += blk(d * d) + blk(d * 4) + blk(d * 4);    /* attn_proj + scale + bias */
  per += 2 * blk(d * 4);                          /* ln2 */
  per += blk(f * d) + blk(f * 4) + blk(f * 4);    /* W1 + scale + b1 */
  per += blk(d * f) + blk(d * 4) + blk(d * 4);    /* W2 + scale + b2 */
  n += per * c->n_layer;
  n += 2 * blk(d * 4); /* lnf */
  return n;
}

/* Device weight arena layout: tensors 256-byte aligned. */
static size_t weight_arena_bytes(const gpt2_engine_config *c) {
  const size_t d = c->d_model, f = 4 * d;
  size_t n = 0;
#define ADD(bytes) n += ALIGN_UP((bytes), 256)
  ADD((size_t)c->vocab * d * 2);
  ADD((size_t)c->ctx * d * 2);
  for (int l = 0; l < c->n_layer; ++l) {
    ADD(d * 2); ADD(d * 2);
    ADD(3 * d * d); ADD(3 * d * 4); ADD(3 * d * 2);
    ADD(d * d); ADD(d * 4); ADD(d * 2);
    ADD(d * 2); ADD(d * 2);
    ADD(f * d); ADD(f * 4); ADD(f * 2);
    ADD(d * f); ADD(d * 4); ADD(d * 2);
  }
  ADD(d * 2); ADD(d * 2);
#undef ADD
  return n;
}

static uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
  u += 0x7fffu + ((u >> 16) & 1u); /* round to nearest, ties to even */
  return (uint16_t)(u >> 16);
}

/* Host-side parse of the quant8 image into a host staging copy of the device
 * arena, then one H2D copy. */
typedef struct {
  const uint8_t *p;
  size_t left;
} reader;

static int rd_take(reader *r, size_t bytes, const uint8_t **out) {
  size_t padded = blk(bytes);
  if (r->left < padded) return 0;
  *out = r->p;
  r->p += padded;
  r->left -= padded;
  return 1;
}

int gpt2_engine_create(const gpt2_engine_config *cfg, int device, gpt2_engine **out) {
  if (!out) return W8A8_ERR_INVALID;
  *out = NULL;
  if (!cfg_ok(cfg)) return W8A8_ERR_INVALID;
  gpt2_engine *e = (gpt2_engine *)calloc(1, sizeof *e);
  if (!e) return W8A8_ERR_NOMEM;
  e->cfg = *cfg;
  e->device = device;
  e->use_graphs = 1;
  e->layers = (layer_w *)calloc((size_t)cfg->n_layer, sizeof(layer_w));
  e->slot_len = (int *)calloc((size_t)cfg->max_batch * 3, sizeof(int));
  if (!e->layers || !e->slot_len) {
    free(e->layers);
    free(e->slot_len);
    free(e);
    return W8A8_ERR_NOMEM;
  }
  e->slot_gen = e->slot_len + cfg->max_batch;
  e->slot_active = e->slot_len + 2 * cfg->max_batch;
  int st = w8a8_init(device);
  if (st != W8A8_OK) {
    gpt2_engine_destroy(e);
    return st;
  }
  if (cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaStreamCreateWithFlags(&e->stream2, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&e->ev_fork, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&e->ev_join, cudaEventDisableTiming) != cudaSuccess) {
    gpt2_engine_destroy(e);
    return W8A8_ERR_CUDA;
  }
  const size_t d = cfg->d_model, L = cfg->n_layer, C = cfg->ctx, Bm = cfg->max_batch;
  const size_t Mt = cfg->max_tokens;
  /* KV cache */
  const size_t kv = Bm * L * C * d * 2;
  if (cudaMalloc((void **)&e->Kc, kv) != cudaSuccess ||
      cudaMalloc((void **)&e->Vc, kv) != cudaSuccess) {
    gpt2_engine_destroy(e);
    return W8A8_ERR_NOMEM;
  }
  /* activations */
  e->attn_ws_bytes = w8a8_attention_decode_workspace_size((int)Bm, cfg->n_head, (int)C);
  e->lin_ws_bytes = w8a8_linear_workspace_size((int)Bm, 4 * (int)d);
  e->amax_rec_floats = w8a8_absmax_record_floats((int)Bm, 4 * (int)d);
  size_t off = 0, sizes[19];
  sizes[0] = Mt * d * 2;        /* H */
  sizes[1] = Mt * d * 2;        /* R1 */
  sizes[2] = Mt * d * 2;        /* Q */
  sizes[3] = Mt * d * 2;        /* ATT */
  sizes[4] = Mt * 4 * d * 2;    /* X1 */
  sizes[5] = Bm * d * 2;        /* Xf */
  sizes[6] = Bm * (size_t)cfg->vocab * 2; /* logits */
  sizes[7] = Mt * 4 * d;        /* Xq */
  sizes[8] = Mt * 4;            /* sX */
  sizes[9] = Bm * 4 * 4;        /* len, nctx, gen, next */
  sizes[10] = Mt * 4;           /* tokens_in */
  sizes[11] = Bm * 4 * (size_t)C; /* default output buffer */
  sizes[12] = e->attn_ws_bytes;
  sizes[13] = e->lin_ws_bytes;
  sizes[14] = Bm * C * 4;       /* sampling draws [max_batch][ctx] */
  sizes[15] = e->attn_ws_bytes; /* second decode half */
  sizes[16] = e->lin_ws_bytes;
  sizes[17] = e->amax_rec_floats * 4; /* row absmax records */
  sizes[18] = e->amax_rec_floats * 4;
  size_t offs[19];
  for (int i = 0; i < 19; ++i) {
    offs[i] = off;
    off += ALIGN_UP(sizes[i], 256);
  }
  if (cudaMalloc(&e->ablob, off) != cudaSuccess) {
    gpt2_engine_destroy(e);
    return W8A8_ERR_NOMEM;
  }
  uint8_t *a = (uint8_t *)e->ablob;
  e->H = (gpt2_bf16_t *)(a + offs[0]);
  e->R1 = (gpt2_bf16_t *)(a + offs[1]);
  e->Q = (gpt2_bf16_t *)(a + offs[2]);
  e->ATT = (gpt2_bf16_t *)(a + offs[3]);
  e->X1 = (gpt2_bf16_t *)(a + offs[4]);
  e->Xf = (gpt2_bf16_t *)(a + offs[5]);
  e->logits = (gpt2_bf16_t *)(a + offs[6]);
  e->Xq = (int8_t *)(a + offs[7]);
  e->sX = (float *)(a + offs[8]);
  e->len = (int32_t *)(a + offs[9]);
  e->nctx = e->len + Bm;
  e->gen = e->len + 2 * Bm;
  e->next = e->len + 3 * Bm;
  e->tokens_in = (int32_t *)(a + offs[10]);
  e->out_default = (int32_t *)(a + offs[11]);
  e->attn_ws = a + offs[12];
  e->lin_ws = a + offs[13];
  e->rnd = (float *)(a + offs[14]);
  e->attn_ws2 = a + offs[15];
  e->lin_ws2 = a + offs[16];
  e->amax_rec = (float *)(a + offs[17]);
  e->amax_rec2 = (float *)(a + offs[18]);
  e->top_k = 40;
  e->decode_split = 1;
  if (cudaMemset(e->ablob, 0, off) != cudaSuccess) {
    gpt2_engine_destroy(e);
    return W8A8_ERR_CUDA;
  }
  *out = e;
  return W8A8_OK;
}

void gpt2_engine_destroy(gpt2_engine *e) {
  if (!e) return;
  if (e->graph) cudaGraphExecDestroy(e->graph);
  if (e->wblob) cudaFree(e->wblob);
  if (e->ablob) cudaFree(e->ablob);
  if (e->Kc) cudaFree(e->Kc);
  if (e->Vc) cudaFree(e->Vc);
  if (e->stream) cudaStreamDestroy(e->stream);
  if (e->stream2) cudaStreamDestroy(e->stream2);
  if (e->ev_fork) cudaEventDestroy(e->ev_fork);
  if (e->ev_join) cudaEventDestroy(e->ev_join);
  free(e->slot_len);
  free(e->layers);
  free(e);
}

int gpt2_engine_load_quant8_memory(gpt2_engine *e, const void *data, size_t bytes) {
  if (!e || !data) return W8A8_ERR_INVALID;
  const gpt2_engine_config *c = &e->cfg;
  if (bytes < gpt2_engine_quant8_bytes(c))
    return fail(e, W8A8_ERR_IO, "quant8 image too short: %zu < %zu bytes", bytes,
                gpt2_engine_quant8_bytes(c));
  const size_t d = c->d_model, f = 4 * d;
  const size_t arena = weight_arena_bytes(c);
  uint8_t *host = (uint8_t *)malloc(arena);
  if (!host) return fail(e, W8A8_ERR_NOMEM, "host staging of %zu bytes", arena);
  memset(host, 0, arena);
  if (!e->wblob) {
    if (cudaMalloc(&e->wblob, arena) != cudaSuccess) {
      free(host);
      return fail(e, W8A8_ERR_NOMEM, "weights: cudaMalloc %zu", arena);
    }
    e->wbytes = arena;
  }
  reader r = {(const uint8_t *)data, bytes};
  size_t off = 0;
  uint8_t *dev = (uint8_t *)e->wblob;
  const uint8_t *src;
  int ok = 1;
  /* helpers: place `count` elements at the next arena slot */
#define SLOT(bytes_) (off = ALIGN_UP(off, 256), off += (bytes_), off - (bytes_))
#define PUT_BF16(dst_ptr, count)                                                   \
  do {                                                                             \
    size_t n_ = (count);                                                           \
    size_t o_ = SLOT(n_ * 2);                                                      \
    if (!rd_take(&r, n_ * 4, &src)) { ok = 0; break; }                              \
    uint16_t *h_ = (uint16_t *)(host + o_);                                        \
    for (size_t i_ = 0; i_ < n_; ++i_) {                                           \
      float v_;                                                                    \
      memcpy(&v_, src + 4 * i_, 4);                                                \
      h_[i_] = f32_to_bf16(v_);                                                    \
    }                                                                              \
    (dst_ptr) = (gpt2_bf16_t *)(dev + o_);                                         \
  } while (0)
#define PUT_RAW(dst_ptr, type, bytes_)                                             \
  do {                                                                             \
    size_t b_ = (bytes_);                                                          \
    size_t o_ = SLOT(b_);                                                          \
    if (!rd_take(&r, b_, &src)) { ok = 0; break; }                                  \
    memcpy(host + o_, src, b_);                                                    \
    (dst_ptr) = (type *)(dev + o_);                                                \
  } while (0)

  do {
    PUT_BF16(e->wte, (size_t)c->vocab * d);
    if (!ok) break;
    PUT_BF16(e->wpe, (size_t)c->ctx * d);
    if (!ok) break;
    for (int l = 0; l < c->n_layer && ok; ++l) {
      layer_w *w = &e->layers[l];
      PUT_BF16(w->ln1_g, d);
      if (!ok) break;
      PUT_BF16(w->ln1_b, d);
      if (!ok) break;
      PUT_RAW(w->Wqkv, int8_t, 3 * d * d);
      if (!ok) break;
      PUT_RAW(w->sWqkv, float, 3 * d * 4);
      if (!ok) break;
      PUT_BF16(w->bqkv, 3 * d);
      if (!ok) break;
      PUT_RAW(w->Wproj, int8_t, d * d);
      if (!ok) break;
      PUT_RAW(w->sWproj, float, d * 4);
      if (!ok) break;
      PUT_BF16(w->bproj, d);
      if (!ok) break;
      PUT_BF16(w->ln2_g, d);
      if (!ok) break;
      PUT_BF16(w->ln2_b, d);
      if (!ok) break;
      PUT_RAW(w->W1, int8_t, f * d);
      if (!ok) break;
      PUT_RAW(w->sW1, float, f * 4);
      if (!ok) break;
      PUT_BF16(w->b1, f);
      if (!ok) break;
      PUT_RAW(w->W2, int8_t, d * f);
      if (!ok) break;
      PUT_RAW(w->sW2, float, d * 4);
      if (!ok) break;
      PUT_BF16(w->b2, d);
      if (!ok) break;
    }
    if (!ok) break;
    PUT_BF16(e->lnf_g, d);
    if (!ok) break;
    PUT_BF16(e->lnf_b, d);
  } while (0);
#undef SLOT
#undef PUT_BF16
#undef PUT_RAW
  if (!ok) {
    free(host);
    return fail(e, W8A8_ERR_IO, "quant8 image truncated");
  }
  cudaError_t ce = cudaMemcpy(e->wblob, host, arena, cudaMemcpyHostToDevice);
  free(host);
  if (ce != cudaSuccess) return fail(e, W8A8_ERR_CUDA, "weights H2D: %s", cudaGetErrorString(ce));
  e->loaded = 1;
  return W8A8_OK;
}

/* ---- the quant8.json manifest (tools/offline_quant/src/writer.py:72-124) ----
 * A flat JSON object written by json.dump(indent=2); only the fields below
 * are read, each once, so a key search suffices. */
static const char *mf_skip_ws(const char *p) {
  while (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r') ++p;
  return p;
}

static const char *mf_value(const char *text, const char *key) {
  char pat[64];
  snprintf(pat, sizeof pat, "\"%s\"", key);
  const char *p = strstr(text, pat);
  if (!p) return NULL;
  p = mf_skip_ws(p + strlen(pat));
  return *p == ':' ? mf_skip_ws(p + 1) : NULL;
}

/* the string at p (no escapes) into out; returns the position after it */
static const char *mf_string(const char *p, char *out, size_t cap) {
  if (!p || *p != '"') return NULL;
  size_t n = 0;
  for (++p; *p && *p != '"'; ++p) {
    if (*p == '\\' || n + 1 >= cap) return NULL;
    out[n++] = *p;
  }
  if (*p != '"') return NULL;
  out[n] = 0;
  return p + 1;
}

static int mf_string_is(const char *text, const char *key, const char *want) {
  char buf[128];
  return mf_string(mf_value(text, key), buf, sizeof buf) && strcmp(buf, want) == 0;
}

static int mf_list_is(const char *text, const char *key, const char *const *want, int n) {
  const char *p = mf_value(text, key);
  if (!p || *p != '[') return 0;
  p = mf_skip_ws(p + 1);
  for (int i = 0; i < n; ++i) {
    char buf[64];
    p = mf_string(p, buf, sizeof buf);
    if (!p || strcmp(buf, want[i]) != 0) return 0;
    p = mf_skip_ws(p);
    if (i + 1 < n) {
      if (*p != ',') return 0;
      p = mf_skip_ws(p + 1);
    }
  }
  return *p == ']';
}

/* num / den rounded half to even (Python's round, writer.py:90-96) */
static long long div_round_even(long long num, long long den) {
  long long q = num / den, r = num % den;
  if (2 * r > den || (2 * r == den && (q & 1))) ++q;
  return q;
}

int gpt2_quant8_check_manifest(const gpt2_engine_config *cfg, const char *text, char *err,
                               size_t err_len) {
  char tmp[8];
  if (!err || err_len == 0) {
    err = tmp;
    err_len = sizeof tmp;
  }
  err[0] = 0;
  if (!cfg || !text) {
    snprintf(err, err_len, "no configuration or manifest text");
    return W8A8_ERR_INVALID;
  }
  static const char *const quantized[] = {"W_qkv", "attn_proj", "W1", "W2"};
  static const char *const preserved[] = {"wte", "wpe", "ln1_gamma", "ln1_beta", "b_qkv",
                                          "attn_proj_bias", "ln2_gamma", "ln2_beta", "b1", "b2",
                                          "lnf_gamma", "lnf_beta"};
  if (!mf_string_is(text, "scheme", "int8_per_channel_symmetric") ||
      !mf_string_is(text, "scale_convention", "amax/127") ||
      !mf_string_is(text, "scale_dtype", "fp32")) {
    snprintf(err, err_len, "not per-channel symmetric int8 with fp32 amax/127 scales");
    return W8A8_ERR_INVALID;
  }
  if (!mf_list_is(text, "quantized_tensors", quantized, 4) ||
      !mf_list_is(text, "preserved_tensors", preserved, 12)) {
    snprintf(err, err_len, "tensor lists differ from the quant8.bin layout");
    return W8A8_ERR_INVALID;
  }
  /* model name where the dimensions are a GPT-2 size (reader.py:36-43) */
  static const struct { int d, L, H; const char *name; } sizes[] = {
      {768, 12, 12, "gpt2-small"}, {1024, 24, 16, "gpt2-medium"}, {1280, 36, 20, "gpt2-large"}};
  for (int i = 0; i < 3; ++i)
    if (cfg->d_model == sizes[i].d && cfg->n_layer == sizes[i].L && cfg->n_head == sizes[i].H &&
        !mf_string_is(text, "model", sizes[i].name)) {
      snprintf(err, err_len, "model is not %s", sizes[i].name);
      return W8A8_ERR_INVALID;
    }
  /* memory summary (writer.py:72-96): unpadded tensor bytes */
  const long long d = cfg->d_model, f = 4 * d, L = cfg->n_layer;
  const long long preserved_b =
      4 * ((long long)cfg->vocab * d + (long long)cfg->ctx * d + 2 * d + L * (9 * d + f));
  const long long quant_b = L * (4 * d * d + 2 * f * d);
  const long long scale_b = 4 * L * (5 * d + f);
  const long long mib = 1024 * 1024;
  const struct { const char *key; long long want; } summary[] = {
      {"source_fp32_total_mb", div_round_even(preserved_b + 4 * quant_b, mib)},
      {"quantized_int8_mb", div_round_even(quant_b, mib)},
      {"preserved_fp32_mb", div_round_even(preserved_b, mib)},
      {"scale_overhead_kb", div_round_even(scale_b, 1024)},
      {"artifact_total_mb", div_round_even(preserved_b + quant_b + scale_b, mib)}};
  for (int i = 0; i < 5; ++i) {
    const char *p = mf_value(text, summary[i].key);
    char *end = NULL;
    const long long v = p ? strtoll(p, &end, 10) : -1;
    if (!p || end == p || v != summary[i].want) {
      snprintf(err, err_len, "memory_summary.%s is not %lld", summary[i].key, summary[i].want);
      return W8A8_ERR_INVALID;
    }
  }
  return W8A8_OK;
}

/* The manifest beside a quant8 file (X.bin -> X.json), checked when present. */
static int check_sibling_manifest(gpt2_engine *e, const char *path) {
  const size_t n = strlen(path);
  char *jpath = (char *)malloc(n + 6);
  if (!jpath) return fail(e, W8A8_ERR_NOMEM, "host memory");
  memcpy(jpath, path, n + 1);
  if (n >= 4 && strcmp(jpath + n - 4, ".bin") == 0) jpath[n - 4] = 0;
  strcat(jpath, ".json");
  FILE *fp = fopen(jpath, "rb");
  if (!fp) {
    free(jpath);
    return W8A8_OK;  /* no manifest: the reference's loader needs none either */
  }
  enum { kMax = 1 << 16 };
  char *text = (char *)malloc(kMax + 1);
  size_t got = text ? fread(text, 1, kMax + 1, fp) : 0;
  fclose(fp);
  int st = W8A8_OK;
  if (!text) {
    st = fail(e, W8A8_ERR_NOMEM, "host memory");
  } else if (got > kMax) {
    st = fail(e, W8A8_ERR_INVALID, "%s: larger than %d bytes", jpath, kMax);
  } else {
    text[got] = 0;
    char why[160];
    if (gpt2_quant8_check_manifest(&e->cfg, text, why, sizeof why) != W8A8_OK)
      st = fail(e, W8A8_ERR_INVALID, "%s: %s", jpath, why);
  }
  free(text);
  free(jpath);
  return st;
}

int gpt2_engine_load_quant8(gpt2_engine *e, const char *path) {
  if (!e || !path) return W8A8_ERR_INVALID;
  int mst = check_sibling_manifest(e, path);
  if (mst) return mst;
  FILE *fp = fopen(path, "rb");
  if (!fp) return fail(e, W8A8_ERR_IO, "cannot open %s", path);
  size_t need = gpt2_engine_quant8_bytes(&e->cfg);
  uint8_t *buf = (uint8_t *)malloc(need);
  if (!buf) {
    fclose(fp);
    return fail(e, W8A8_ERR_NOMEM, "host buffer of %zu bytes", need);
  }
  size_t got = fread(buf, 1, need, fp);
  fclose(fp);
  int st = got == need ? gpt2_engine_load_quant8_memory(e, buf, need)
                       : fail(e, W8A8_ERR_IO, "%s: read %zu of %zu bytes", path, got, need);
  free(buf);
  return st;
}

/* ---- forward passes ---- */

/* The activation buffers, workspaces and stream one forward pass uses. A
 * split decode step runs its two halves at the same time on two streams:
 * each half uses the buffer rows of its own slots and its own workspaces. */
typedef struct {
  gpt2_bf16_t *H, *R1, *Q, *ATT, *X1, *Xf, *logits;
  int8_t *Xq;
  float *sX;
  void *attn_ws, *lin_ws;
  float *amax; /* row absmax record */
  void *s;
} act_view;

/* Rows row0.. of every activation buffer; half 1 takes the second workspaces
 * and stream. */
static act_view view_at(gpt2_engine *e, int row0, int half) {
  const int64_t d = e->cfg.d_model, f = 4 * d;
  act_view v;
  v.H = e->H + row0 * d;
  v.R1 = e->R1 + row0 * d;
  v.Q = e->Q + row0 * d;
  v.ATT = e->ATT + row0 * d;
  v.X1 = e->X1 + row0 * f;
  v.Xf = e->Xf + row0 * d;
  v.logits = e->logits + (int64_t)row0 * e->cfg.vocab;
  v.Xq = e->Xq + row0 * f; /* rows of up to 4d int8 */
  v.sX = e->sX + row0;
  v.attn_ws = half ? e->attn_ws2 : e->attn_ws;
  v.lin_ws = half ? e->lin_ws2 : e->lin_ws;
  v.amax = half ? e->amax_rec2 : e->amax_rec;
  v.s = (void *)(half ? e->stream2 : e->stream);
  return v;
}

/* One transformer block over M = B*T rows of H (T tokens per sequence,
 * written at cache rows pos0[b] + t; pos0 == NULL means prefill from 0). */
static int block_forward(gpt2_engine *e, const act_view *v, int l, int slot0, int B, int T,
                         const int32_t *pos0, int first) {
  const gpt2_engine_config *c = &e->cfg;
  const layer_w *w = &e->layers[l];
  const int d = c->d_model, f = 4 * d, M = B * T, Hh = c->n_head;
  const float eps = 1e-5f; /* gpt2.c:627 */
  const int64_t seq_stride = (int64_t)c->n_layer * c->ctx * d;
  /* the caches of slots slot0 .. slot0+B-1 */
  gpt2_bf16_t *Kl = e->Kc + (int64_t)slot0 * seq_stride + (int64_t)l * c->ctx * d;
  gpt2_bf16_t *Vl = e->Vc + (int64_t)slot0 * seq_stride + (int64_t)l * c->ctx * d;
  void *s = v->s;
  const size_t lwb = e->lin_ws_bytes;
  /* one decoding sequence: the LayerNorms run inside the GEMVs that follow them */
  const int one_row = pos0 != NULL && M == 1;
  if (first)
    W8_TRY(e, w8a8_linear_qkv(v->Xq, v->sX, M, d, w->Wqkv, w->sWqkv, w->bqkv, v->Q, d, Kl, Vl,
                              seq_stride, T, pos0, v->lin_ws, lwb, s));
  else if (one_row)
    W8_TRY(e, w8a8_layernorm_linear_qkv(v->H, d, w->ln1_g, w->ln1_b, eps, v->Xq, v->sX, M, d,
                                        w->Wqkv, w->sWqkv, w->bqkv, v->Q, d, Kl, Vl, seq_stride,
                                        T, pos0, v->lin_ws, lwb, s));
  else {
    W8_TRY(e, w8a8_layernorm_quant(v->H, d, M, d, w->ln1_g, w->ln1_b, eps, NULL, 0, v->Xq, v->sX, s));
    W8_TRY(e, w8a8_linear_qkv(v->Xq, v->sX, M, d, w->Wqkv, w->sWqkv, w->bqkv, v->Q, d, Kl, Vl,
                              seq_stride, T, pos0, v->lin_ws, lwb, s));
  }
  if (pos0 == NULL)
    W8_TRY(e, w8a8_attention_prefill(v->Q, d, Kl, Vl, seq_stride, B, T, Hh, 64, v->ATT, d, s));
  else  /* decode: the attention kernel also quantizes its output rows */
    W8_TRY(e, w8a8_attention_decode_quant(v->Q, d, Kl, Vl, seq_stride, B, e->nctx + slot0, c->ctx,
                                          Hh, 64, v->ATT, d, v->Xq, v->sX, v->attn_ws,
                                          e->attn_ws_bytes, s));
  if (pos0 == NULL) W8_TRY(e, w8a8_quant_rows(v->ATT, d, M, d, v->Xq, v->sX, s));
  W8_TRY(e, w8a8_linear(v->Xq, v->sX, M, d, w->Wproj, w->sWproj, w->bproj, d, W8A8_EPI_BIAS_RESID,
                        v->H, d, v->R1, d, v->lin_ws, lwb, s));
  if (one_row) {
    /* batch-1 decode: W1 forms LN2 itself, its epilogue records the row
     * maxima of its GELU output and W2 quantizes the row itself (no
     * LayerNorm or quantization launch) */
    int n_part = 0;
    W8_TRY(e, w8a8_layernorm_linear_absmax(v->R1, d, w->ln2_g, w->ln2_b, eps, v->Xq, v->sX, M,
                                           d, w->W1, w->sW1, w->b1, f, W8A8_EPI_BIAS_GELU, NULL,
                                           0, v->X1, f, v->amax, e->amax_rec_floats, &n_part,
                                           v->lin_ws, lwb, s));
    W8_TRY(e, w8a8_linear_from_bf16(v->X1, f, v->amax, n_part, M, f, w->W2, w->sW2, w->b2, d,
                                    W8A8_EPI_BIAS_RESID, v->R1, d, v->H, d, v->Xq, v->sX,
                                    v->lin_ws, lwb, s));
    return W8A8_OK;
  }
  W8_TRY(e, w8a8_layernorm_quant(v->R1, d, M, d, w->ln2_g, w->ln2_b, eps, NULL, 0, v->Xq, v->sX, s));
  W8_TRY(e, w8a8_linear(v->Xq, v->sX, M, d, w->W1, w->sW1, w->b1, f, W8A8_EPI_BIAS_GELU, NULL, 0,
                        v->X1, f, v->lin_ws, lwb, s));
  W8_TRY(e, w8a8_quant_rows(v->X1, f, M, f, v->Xq, v->sX, s));
  W8_TRY(e, w8a8_linear(v->Xq, v->sX, M, f, w->W2, w->sW2, w->b2, d, W8A8_EPI_BIAS_RESID, v->R1, d,
                        v->H, d, v->lin_ws, lwb, s));
  return W8A8_OK;
}

/* Embedding + all blocks + final LN of the last row of each sequence + LM
 * head + greedy pick appended to the output rows, for the B sequences in
 * slots slot0 .. slot0+B-1. */
static int model_forward(gpt2_engine *e, const act_view *v, const int32_t *tokens_d, int slot0,
                         int B, int T, const int32_t *pos0) {
  const gpt2_engine_config *c = &e->cfg;
  const int d = c->d_model, M = B * T;
  const float eps = 1e-5f;
  void *s = v->s;
  const layer_w *w0 = &e->layers[0];
  W8_TRY(e, w8a8_embed_layernorm_quant(e->wte, e->wpe, tokens_d, M, T, pos0, d, v->H, w0->ln1_g,
                                       w0->ln1_b, eps, NULL, v->Xq, v->sX, s));
  for (int l = 0; l < c->n_layer; ++l) {
    int st = block_forward(e, v, l, slot0, B, T, pos0, l == 0);
    if (st) return st;
  }
  /* final LayerNorm on the last token of every sequence (gpt2.c:2150-2157) */
  W8_TRY(e, w8a8_layernorm_quant(v->H + (int64_t)(T - 1) * d, (int64_t)T * d, B, d, e->lnf_g,
                                 e->lnf_b, eps, v->Xf, d, NULL, NULL, s));
  W8_TRY(e, w8a8_lm_head(v->Xf, d, B, d, e->wte, c->vocab, v->logits, c->vocab, s));
  /* gpt2.c:2176-2245: greedy at temperature <= 0, else top-k sampling; the
   * draw of a slot's i-th token is rnd[slot][i] (i = its output count) */
  if (e->temperature > 0.0f)
    W8_TRY(e, w8a8_sample_topk(v->logits, c->vocab, B, c->vocab, e->temperature, e->top_k,
                               e->rnd + (int64_t)slot0 * c->ctx, c->ctx, e->gen + slot0,
                               e->next + slot0, e->out + (int64_t)slot0 * e->out_stride,
                               e->out_stride, e->gen + slot0, NULL, 0, s));
  else
    W8_TRY(e, w8a8_sample_greedy(v->logits, c->vocab, B, c->vocab, e->next + slot0,
                                 e->out + (int64_t)slot0 * e->out_stride, e->out_stride,
                                 e->gen + slot0, s));
  return W8A8_OK;
}

/* A decode step of B slots runs as one chain, or (decode_split 2, B >= 2) as
 * two chains of ceil(B/2) and floor(B/2) slots on two streams. */
static int decode_halves(const gpt2_engine *e, int B) { return e->decode_split == 2 && B >= 2 ? 2 : 1; }
static int decode_half_rows(const gpt2_engine *e, int B, int h) {
  return decode_halves(e, B) == 1 ? B : (h == 0 ? (B + 1) / 2 : B / 2);
}

int gpt2_engine_launches_per_decode_step(const gpt2_engine *e) {
  /* embed+LN1; per block LN1 (not in the first), QKV, attention (one or two
   * kernels, output quantization fused), attn_proj, LN2, W1, quant, W2; then
   * nctx, final LN, LM head, sample, len advance */
  if (!e) return 0;
  const int B = e->B > 0 ? e->B : e->cfg.max_batch;
  int n = 0;
  for (int h = 0; h < decode_halves(e, B); ++h) {
    const int rows = decode_half_rows(e, B, h);
    const int attn = w8a8_attention_decode_launches(rows, e->cfg.n_head, e->cfg.ctx);
    n += 1 + e->cfg.n_layer * (7 + attn) - 1 + 1 + 3 + 1;
  }
  return n;
}

int gpt2_engine_launches_per_prefill(const gpt2_engine *e) {
  if (!e) return 0;
  return 1 + e->cfg.n_layer * 9 - 1 + 3;
}

int gpt2_engine_prefill(gpt2_engine *e, const int32_t *prompts_d, int B, int T,
                        int32_t *out_tokens_d, int out_stride) {
  if (!e || !prompts_d || !out_tokens_d) return W8A8_ERR_INVALID;
  if (!e->loaded) return fail(e, W8A8_ERR_INVALID, "weights not loaded");
  const gpt2_engine_config *c = &e->cfg;
  if (B <= 0 || T <= 0 || B > c->max_batch || (size_t)B * T > (size_t)c->max_tokens ||
      T > c->ctx)
    return fail(e, W8A8_ERR_INVALID, "batch %d x %d exceeds engine limits", B, T);
  if (out_stride < 1) return fail(e, W8A8_ERR_INVALID, "output stride %d", out_stride);
  e->B = B;
  e->out = out_tokens_d;
  e->out_stride = out_stride;
  /* reset per-sequence state: gen = 0, len = T (after this prefill) */
  CUDA_TRY(e, cudaMemsetAsync(e->gen, 0, (size_t)B * 4, e->stream));
  const act_view v = view_at(e, 0, 0);
  int st = model_forward(e, &v, prompts_d, 0, B, T, NULL);
  if (st) return st;
  CUDA_TRY(e, cudaMemsetAsync(e->len, 0, (size_t)B * 4, e->stream));
  W8_TRY(e, w8a8_advance_positions(e->len, e->len, B, T, (void *)e->stream));
  for (int b = 0; b < B; ++b) {
    e->slot_len[b] = T;
    e->slot_gen[b] = 1;
    e->slot_active[b] = 1;
  }
  return W8A8_OK;
}

/* ---- continuous batching: requests admitted into and released from slots ---- */

/* Put slot b back to position 0 with an empty output row (device and host
 * mirror). A parked slot keeps stepping with the others; its tokens are
 * discarded and its cache rows are scratch. */
static int park_slot(gpt2_engine *e, int b) {
  CUDA_TRY(e, cudaMemsetAsync(e->len + b, 0, 4, e->stream));
  CUDA_TRY(e, cudaMemsetAsync(e->gen + b, 0, 4, e->stream));
  CUDA_TRY(e, cudaMemsetAsync(e->next + b, 0, 4, e->stream));
  e->slot_len[b] = 0;
  e->slot_gen[b] = 0;
  e->slot_active[b] = 0;
  return W8A8_OK;
}

int gpt2_engine_slots_begin(gpt2_engine *e, int B, int32_t *out_tokens_d, int out_stride) {
  if (!e || !out_tokens_d) return W8A8_ERR_INVALID;
  if (!e->loaded) return fail(e, W8A8_ERR_INVALID, "weights not loaded");
  if (B <= 0 || B > e->cfg.max_batch || out_stride < 1)
    return fail(e, W8A8_ERR_INVALID, "%d slots, output stride %d", B, out_stride);
  e->B = B;
  e->out = out_tokens_d;
  e->out_stride = out_stride;
  for (int b = 0; b < B; ++b) {
    int st = park_slot(e, b);
    if (st) return st;
  }
  return W8A8_OK;
}

int gpt2_engine_slot_prefill(gpt2_engine *e, int slot, const int32_t *prompt_d, int T) {
  if (!e || !prompt_d) return W8A8_ERR_INVALID;
  if (!e->loaded) return fail(e, W8A8_ERR_INVALID, "weights not loaded");
  if (e->B <= 0 || slot < 0 || slot >= e->B)
    return fail(e, W8A8_ERR_INVALID, "slot %d outside the %d slots", slot, e->B);
  if (T <= 0 || T > e->cfg.ctx || T > e->cfg.max_tokens)
    return fail(e, W8A8_ERR_INVALID, "prompt of %d tokens", T);
  CUDA_TRY(e, cudaMemsetAsync(e->gen + slot, 0, 4, e->stream));
  const act_view v = view_at(e, 0, 0);
  int st = model_forward(e, &v, prompt_d, slot, 1, T, NULL);
  if (st) return st;
  CUDA_TRY(e, cudaMemsetAsync(e->len + slot, 0, 4, e->stream));
  W8_TRY(e, w8a8_advance_positions(e->len + slot, e->len + slot, 1, T, (void *)e->stream));
  e->slot_len[slot] = T;
  e->slot_gen[slot] = 1;
  e->slot_active[slot] = 1;
  return W8A8_OK;
}

int gpt2_engine_slot_release(gpt2_engine *e, int slot, int32_t *host_tokens) {
  if (!e || e->B <= 0 || slot < 0 || slot >= e->B) return W8A8_ERR_INVALID;
  if (host_tokens && e->slot_active[slot] && e->slot_gen[slot] > 0) {
    CUDA_TRY(e, cudaMemcpyAsync(host_tokens, e->out + (int64_t)slot * e->out_stride,
                                (size_t)e->slot_gen[slot] * 4, cudaMemcpyDeviceToHost,
                                e->stream));
    CUDA_TRY(e, cudaStreamSynchronize(e->stream));
  }
  return park_slot(e, slot);
}

int gpt2_engine_slot_tokens(const gpt2_engine *e, int slot) {
  if (!e || e->B <= 0 || slot < 0 || slot >= e->B || !e->slot_active[slot]) return -1;
  return e->slot_gen[slot];
}

/* One decode step of slots slot0 .. slot0+B-1: token next[b] at position len[b]. */
static int decode_chain(gpt2_engine *e, const act_view *v, int slot0, int B) {
  W8_TRY(e, w8a8_advance_positions(e->nctx + slot0, e->len + slot0, B, 1, v->s));
  int st = model_forward(e, v, e->next + slot0, slot0, B, 1, e->len + slot0);
  if (st) return st;
  W8_TRY(e, w8a8_advance_positions(e->len + slot0, e->len + slot0, B, 1, v->s));
  return W8A8_OK;
}

/* One decode step of all B slots: one chain on the engine stream, or two
 * independent chains (every row of every kernel is computed on its own) on
 * the engine stream and the second stream, forked from and joined back to
 * the engine stream, so that one half's latency-bound GEMMs run while the
 * other half's attention streams its KV cache. */
static int decode_step_launches(gpt2_engine *e) {
  const int B = e->B;
  if (decode_halves(e, B) == 1) {
    const act_view v = view_at(e, 0, 0);
    return decode_chain(e, &v, 0, B);
  }
  const int b0 = decode_half_rows(e, B, 0), b1 = decode_half_rows(e, B, 1);
  CUDA_TRY(e, cudaEventRecord(e->ev_fork, e->stream));
  CUDA_TRY(e, cudaStreamWaitEvent(e->stream2, e->ev_fork, 0));
  const act_view v0 = view_at(e, 0, 0), v1 = view_at(e, b0, 1);
  int st = decode_chain(e, &v0, 0, b0);
  if (!st) st = decode_chain(e, &v1, b0, b1);
  /* join even after an error, so that a capture in progress ends cleanly */
  cudaEventRecord(e->ev_join, e->stream2);
  cudaStreamWaitEvent(e->stream, e->ev_join, 0);
  return st;
}

int gpt2_engine_decode_steps(gpt2_engine *e, int steps) {
  if (!e) return W8A8_ERR_INVALID;
  if (steps <= 0) return W8A8_OK;
  if (e->B <= 0) return fail(e, W8A8_ERR_INVALID, "decode before prefill");
  if (steps > e->cfg.ctx || steps > e->out_stride)
    return fail(e, W8A8_ERR_INVALID, "%d steps at once", steps);
  /* every slot steps: a sequence may not outgrow its cache or output row;
   * a parked slot that would is parked again at position 0 */
  for (int b = 0; b < e->B; ++b) {
    const int over = e->slot_len[b] + steps > e->cfg.ctx || e->slot_gen[b] + steps > e->out_stride;
    if (over && e->slot_active[b])
      return fail(e, W8A8_ERR_INVALID, "slot %d: %d cache rows / %d tokens + %d steps exceed "
                  "ctx %d / %d", b, e->slot_len[b], e->slot_gen[b], steps, e->cfg.ctx,
                  e->out_stride);
    if (over) {
      int st = park_slot(e, b);
      if (st) return st;
    }
  }
  for (int b = 0; b < e->B; ++b) {
    e->slot_len[b] += steps;
    e->slot_gen[b] += steps;
  }
  if (!e->use_graphs) {
    for (int i = 0; i < steps; ++i) {
      int st = decode_step_launches(e);
      if (st) return st;
    }
    return W8A8_OK;
  }
  if (!e->graph || e->graph_B != e->B || e->graph_out != e->out ||
      e->graph_stride != e->out_stride || e->graph_split != e->decode_split) {
    if (e->graph) {
      cudaGraphExecDestroy(e->graph);
      e->graph = NULL;
    }
    cudaGraph_t g;
    CUDA_TRY(e, cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
    int st = decode_step_launches(e);
    cudaGraph_t captured = NULL;
    cudaError_t ce = cudaStreamEndCapture(e->stream, &captured);
    if (st) {
      if (captured) cudaGraphDestroy(captured);
      return st;
    }
    if (ce != cudaSuccess) return fail(e, W8A8_ERR_CUDA, "capture: %s", cudaGetErrorString(ce));
    g = captured;
    ce = cudaGraphInstantiate(&e->graph, g, 0);
    cudaGraphDestroy(g);
    if (ce != cudaSuccess) return fail(e, W8A8_ERR_CUDA, "instantiate: %s", cudaGetErrorString(ce));
    e->graph_B = e->B;
    e->graph_out = e->out;
    e->graph_stride = e->out_stride;
    e->graph_split = e->decode_split;
  }
  for (int i = 0; i < steps; ++i) CUDA_TRY(e, cudaGraphLaunch(e->graph, e->stream));
  return W8A8_OK;
}

int gpt2_engine_generate_device(gpt2_engine *e, const int32_t *prompts_d, int B, int T, int n_gen,
                                int32_t *out_tokens_d, void *stream) {
  if (!e || n_gen <= 0) return W8A8_ERR_INVALID;
  if (T + n_gen - 1 > e->cfg.ctx)
    return fail(e, W8A8_ERR_INVALID, "prompt %d + %d tokens exceeds ctx %d", T, n_gen, e->cfg.ctx);
  cudaStream_t user = (cudaStream_t)stream;
  cudaEvent_t ev = NULL;
  if (user && user != e->stream) {
    /* order the engine stream after the caller's work, and back */
    CUDA_TRY(e, cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    CUDA_TRY(e, cudaEventRecord(ev, user));
    CUDA_TRY(e, cudaStreamWaitEvent(e->stream, ev, 0));
  }
  int st = gpt2_engine_prefill(e, prompts_d, B, T, out_tokens_d, n_gen);
  if (!st) st = gpt2_engine_decode_steps(e, n_gen - 1);
  if (ev) {
    cudaEventRecord(ev, e->stream);
    cudaStreamWaitEvent(user, ev, 0);
    cudaEventDestroy(ev);
  }
  return st;
}

int gpt2_engine_generate(gpt2_engine *e, const int32_t *prompts, int B, int T, int n_gen,
                         int32_t *out_tokens) {
  if (!e || !prompts || !out_tokens || B <= 0 || T <= 0 || n_gen <= 0) return W8A8_ERR_INVALID;
  if ((size_t)B * T > (size_t)e->cfg.max_tokens || B > e->cfg.max_batch)
    return fail(e, W8A8_ERR_INVALID, "batch %d x %d exceeds engine limits", B, T);
  if ((size_t)B * n_gen > (size_t)e->cfg.max_batch * e->cfg.ctx)
    return fail(e, W8A8_ERR_INVALID, "output buffer too small");
  for (size_t i = 0; i < (size_t)B * T; ++i)
    if (prompts[i] < 0 || prompts[i] >= e->cfg.vocab)
      return fail(e, W8A8_ERR_INVALID, "prompt token %d at %zu outside the vocabulary",
                  prompts[i], i);
  CUDA_TRY(e, cudaMemcpyAsync(e->tokens_in, prompts, (size_t)B * T * 4, cudaMemcpyHostToDevice,
                              e->stream));
  int st = gpt2_engine_generate_device(e, e->tokens_in, B, T, n_gen, e->out_default, NULL);
  if (st) return st;
  CUDA_TRY(e, cudaMemcpyAsync(out_tokens, e->out_default, (size_t)B * n_gen * 4,
                              cudaMemcpyDeviceToHost, e->stream));
  CUDA_TRY(e, cudaStreamSynchronize(e->stream));
  int derr = w8a8_device_error(1);
  if (derr) return fail(e, W8A8_ERR_DEVICE, "device error word 0x%x", derr);
  return W8A8_OK;
}

/* Continuous-batching loop over `slots` slots: admit requests in order into
 * free slots (one prefill each), run decode steps until the next request is
 * complete, hand its tokens back and admit the next. */
int gpt2_engine_serve(gpt2_engine *e, gpt2_request *reqs, int n_req, int slots) {
  if (!e || (!reqs && n_req > 0) || n_req < 0) return W8A8_ERR_INVALID;
  if (!e->loaded) return fail(e, W8A8_ERR_INVALID, "weights not loaded");
  const gpt2_engine_config *c = &e->cfg;
  if (slots <= 0 || slots > c->max_batch)
    return fail(e, W8A8_ERR_INVALID, "%d slots (max_batch %d)", slots, c->max_batch);
  for (int i = 0; i < n_req; ++i) {
    const gpt2_request *r = &reqs[i];
    if (!r->prompt || !r->out || r->T <= 0 || r->n_gen <= 0 || r->T > c->max_tokens ||
        r->T + r->n_gen - 1 > c->ctx)
      return fail(e, W8A8_ERR_INVALID, "request %d: %d prompt + %d new tokens", i, r->T,
                  r->n_gen);
    for (int t = 0; t < r->T; ++t)
      if (r->prompt[t] < 0 || r->prompt[t] >= c->vocab)
        return fail(e, W8A8_ERR_INVALID, "request %d: token %d outside the vocabulary", i,
                    r->prompt[t]);
  }
  int st = gpt2_engine_slots_begin(e, slots, e->out_default, c->ctx);
  if (st) return st;
  int *owner = (int *)malloc((size_t)slots * sizeof(int));
  if (!owner) return fail(e, W8A8_ERR_NOMEM, "serve: host memory");
  for (int b = 0; b < slots; ++b) owner[b] = -1;
  int next_req = 0, done = 0;
  while (done < n_req && !st) {
    /* admit into every free slot */
    for (int b = 0; b < slots && next_req < n_req && !st; ++b) {
      if (owner[b] >= 0) continue;
      const gpt2_request *r = &reqs[next_req];
      if (cudaMemcpyAsync(e->tokens_in, r->prompt, (size_t)r->T * 4, cudaMemcpyHostToDevice,
                          e->stream) != cudaSuccess) {
        st = fail(e, W8A8_ERR_CUDA, "serve: prompt copy");
        break;
      }
      /* the request's draws (zeros if it brings none) into the slot's row */
      if (e->temperature > 0.0f) {
        st = r->draws ? gpt2_engine_set_draws(e, b, r->draws, r->n_gen)
                      : (cudaMemsetAsync(e->rnd + (int64_t)b * c->ctx, 0, (size_t)c->ctx * 4,
                                         e->stream) == cudaSuccess ? W8A8_OK
                                                                    : fail(e, W8A8_ERR_CUDA,
                                                                           "serve: draws"));
        if (st) break;
      }
      /* tokens_in is reused by the next admission only after this prefill
       * (one stream) */
      st = gpt2_engine_slot_prefill(e, b, e->tokens_in, r->T);
      owner[b] = next_req++;
    }
    if (st) break;
    /* steps until the first active request is complete */
    int steps = c->ctx;
    for (int b = 0; b < slots; ++b)
      if (owner[b] >= 0) {
        const int left = reqs[owner[b]].n_gen - e->slot_gen[b];
        if (left < steps) steps = left;
      }
    if (steps > 0) st = gpt2_engine_decode_steps(e, steps);
    if (st) break;
    for (int b = 0; b < slots && !st; ++b) {
      if (owner[b] < 0 || e->slot_gen[b] < reqs[owner[b]].n_gen) continue;
      st = gpt2_engine_slot_release(e, b, reqs[owner[b]].out);
      owner[b] = -1;
      ++done;
    }
  }
  free(owner);
  if (!st) {
    CUDA_TRY(e, cudaStreamSynchronize(e->stream));
    const int derr = w8a8_device_error(1);
    if (derr) return fail(e, W8A8_ERR_DEVICE, "device error word 0x%x", derr);
  }
  return st;
}

int gpt2_engine_copy_logits(gpt2_engine *e, gpt2_bf16_t *host, int rows) {
  if (!e || !host || rows <= 0 || rows > e->cfg.max_batch) return W8A8_ERR_INVALID;
  CUDA_TRY(e, cudaMemcpyAsync(host, e->logits, (size_t)rows * e->cfg.vocab * 2,
                              cudaMemcpyDeviceToHost, e->stream));
  CUDA_TRY(e, cudaStreamSynchronize(e->stream));
  return W8A8_OK;
}

int gpt2_engine_set_sampling(gpt2_engine *e, float temperature, int top_k) {
  if (!e) return W8A8_ERR_INVALID;
  if (temperature != temperature) return fail(e, W8A8_ERR_INVALID, "temperature is NaN");
  e->temperature = temperature;
  e->top_k = top_k;
  /* the captured decode step holds the sampler and its arguments */
  if (e->graph) {
    cudaGraphExecDestroy(e->graph);
    e->graph = NULL;
  }
  return W8A8_OK;
}

int gpt2_reference_draws(unsigned seed, float *out, int n) {
  if (n < 0 || (n > 0 && !out)) return W8A8_ERR_INVALID;
  /* glibc's rand() is random() on a 128-byte TYPE_3 state; initstate_r with a
   * 128-byte buffer and the same seed gives the same sequence without
   * touching the process's own generator */
  char state[128];
  struct random_data rd;
  memset(&rd, 0, sizeof rd);
  memset(state, 0, sizeof state);
  if (initstate_r(seed, state, sizeof state, &rd) != 0) return W8A8_ERR_INVALID;
  for (int i = 0; i < n; ++i) {
    int32_t v;
    random_r(&rd, &v);
    out[i] = (float)v / RAND_MAX;  /* gpt2.c:2231 */
  }
  return W8A8_OK;
}

int gpt2_engine_set_draws(gpt2_engine *e, int slot, const float *draws, int n) {
  if (!e || slot < 0 || slot >= e->cfg.max_batch || n < 0 || n > e->cfg.ctx || (n > 0 && !draws))
    return W8A8_ERR_INVALID;
  if (n == 0) return W8A8_OK;
  /* stream-ordered: steps already queued read the slot's previous draws */
  CUDA_TRY(e, cudaMemcpyAsync(e->rnd + (int64_t)slot * e->cfg.ctx, draws, (size_t)n * 4,
                              cudaMemcpyHostToDevice, e->stream));
  return W8A8_OK;
}

int gpt2_engine_set_decode_split(gpt2_engine *e, int halves) {
  if (!e || (halves != 1 && halves != 2)) return W8A8_ERR_INVALID;
  e->decode_split = halves;
  return W8A8_OK;
}

int gpt2_engine_set_graphs(gpt2_engine *e, int enable) {
  if (!e) return W8A8_ERR_INVALID;
  e->use_graphs = enable ? 1 : 0;
  return W8A8_OK;
}
