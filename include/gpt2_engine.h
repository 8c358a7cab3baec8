/*
 * gpt2_engine.h — C host engine for batched W8A8 GPT-2 inference on one GPU.
 *
 * This is the host side of the reference's INT8 GPU build (gpt2.c:1124-1330
 * transformer_block_gpu, gpt2.c:2094-2222 token loop) rebuilt around the
 * kernels of gpt2_w8a8.h: it loads the reference's quant8.bin weight file,
 * keeps W_qkv packed, holds one reference-layout KV cache ([L][ctx][d] bf16)
 * per resident sequence, runs prefill for a batch of equal-length prompts,
 * then greedy (or top-k sampled) decode with one CUDA graph per decode step. Sequences are
 * independent: each sequence's tokens are those it would produce alone.
 *
 * Device memory is allocated once in gpt2_engine_create / load (the
 * reference's allocate_weights_gpu, gpt2.c:864-942); generation allocates
 * nothing.
 */
#ifndef GPT2_ENGINE_H
#define GPT2_ENGINE_H

#include <stddef.h>
#include <stdint.h>

#include "gpt2_w8a8.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct gpt2_engine gpt2_engine;

typedef struct {
  int d_model;     /* 768 / 1024 / 1280 for small / medium / large (model_config.h:10-36) */
  int n_layer;     /* 12 / 24 / 36 */
  int n_head;      /* 12 / 16 / 20; head_dim = d_model / n_head must be 64 */
  int vocab;       /* 50257 */
  int ctx;         /* 1024: KV-cache rows per sequence and wpe rows */
  int max_batch;   /* sequences resident at once */
  int max_tokens;  /* largest prefill: max_batch * prompt length */
} gpt2_engine_config;

int gpt2_engine_create(const gpt2_engine_config *cfg, int device, gpt2_engine **out);
void gpt2_engine_destroy(gpt2_engine *e);

/* Load weights in the reference's quant8.bin layout
 * (tools/offline_quant/src/writer.py:50-69; read by gpt2.c:1703-1800):
 * FP32 wte, wpe, then per layer ln1 γ/β, INT8 W_qkv [3d,d] + FP32 scales,
 * FP32 b_qkv, INT8 attn_proj + scales, bias, ln2 γ/β, INT8 W1 + scales, b1,
 * INT8 W2 + scales, b2; then lnf γ/β. Every block is padded to 16 bytes.
 * FP32 tensors are rounded to bf16 (round-to-nearest-even) as the
 * reference's loader does (gpt2.c:1613-1628). */
int gpt2_engine_load_quant8(gpt2_engine *e, const char *path);
/* The manifest the reference's writer puts beside the file
 * (gpt2_<size>_quant8.json, tools/offline_quant/src/writer.py:72-124):
 * gpt2_engine_load_quant8(path) reads X.json for X.bin when it exists and
 * refuses the load unless it describes per-channel symmetric int8 weights with
 * fp32 amax/127 scales, the quant8.bin tensor lists, the model named by a GPT-2
 * size's dimensions and the memory summary of this configuration.
 * gpt2_quant8_check_manifest runs that check on a manifest's text (host only):
 * W8A8_OK, or W8A8_ERR_INVALID with the reason in err. */
int gpt2_quant8_check_manifest(const gpt2_engine_config *cfg, const char *json_text, char *err,
                               size_t err_len);
int gpt2_engine_load_quant8_memory(gpt2_engine *e, const void *data, size_t bytes);
/* Bytes of a quant8.bin for this configuration. */
size_t gpt2_engine_quant8_bytes(const gpt2_engine_config *cfg);

/* Greedy generation for B prompts of T tokens each: the first new token comes
 * from prefill, the other n_gen-1 from decode steps (the reference counts
 * tokens the same way, gpt2.c:2094-2247). KV caches start empty.
 * Host-buffer form: prompts [B*T] and out_tokens [B*n_gen] are host memory;
 * the call checks every id against the vocabulary, copies prompts in and
 * tokens out (synchronous). */
int gpt2_engine_generate(gpt2_engine *e, const int32_t *prompts, int B, int T, int n_gen,
                         int32_t *out_tokens);
/* Device-buffer form, asynchronous on `stream` (NULL = engine stream). The
 * ids in prompts_d are not checked: each must lie in [0, vocab). */
int gpt2_engine_generate_device(gpt2_engine *e, const int32_t *prompts_d, int B, int T, int n_gen,
                                int32_t *out_tokens_d, void *stream);

/* Step-level interface (device buffers, engine stream):
 * prompt ids must lie in [0, vocab) (not checked);
 * prefill resets the batch, fills the KV caches and writes the first token
 * of each sequence to out_tokens_d[b*out_stride]; decode_steps runs `steps`
 * further steps, appending tokens after those already produced. */
int gpt2_engine_prefill(gpt2_engine *e, const int32_t *prompts_d, int B, int T,
                        int32_t *out_tokens_d, int out_stride);
int gpt2_engine_decode_steps(gpt2_engine *e, int steps);

/* Continuous batching (serving requests of different lengths; the
 * reference serves one sequence per process, gpt2.c:2026-2036).
 * The decode step runs over B slots; each slot holds one sequence or is
 * parked (it steps at position 0 and its tokens are discarded). A slot's
 * sequence produces exactly the tokens it would produce in any other batch
 * of B slots: every row of every kernel is computed on its own.
 *   slots_begin:  B slots (B <= max_batch), all parked; slot b writes its
 *                 tokens to out_tokens_d[b*out_stride ...] (device memory).
 *   slot_prefill: prefill prompt_d[0..T) (device ids in [0, vocab), not
 *                 checked) into slot `slot`, writing its first token; the
 *                 other slots keep their state.
 *   decode_steps: every slot steps (as above); fails when an active slot
 *                 would pass ctx cache rows or out_stride tokens.
 *   slot_release: copy the slot's tokens so far to host_tokens (NULL: drop
 *                 them; synchronous) and park the slot.
 *   slot_tokens:  tokens the slot's sequence has produced, -1 if parked. */
int gpt2_engine_slots_begin(gpt2_engine *e, int B, int32_t *out_tokens_d, int out_stride);
int gpt2_engine_slot_prefill(gpt2_engine *e, int slot, const int32_t *prompt_d, int T);
int gpt2_engine_slot_release(gpt2_engine *e, int slot, int32_t *host_tokens);
int gpt2_engine_slot_tokens(const gpt2_engine *e, int slot);

/* One request of gpt2_engine_serve: T host prompt ids -> n_gen new ids. */
typedef struct {
  const int32_t *prompt;
  int T;
  int n_gen;
  int32_t *out;        /* host, n_gen ids */
  const float *draws;  /* host, n_gen draws for top-k sampling (NULL: all 0) */
} gpt2_request;
/* Serve n_req requests over `slots` slots (continuous batching): requests
 * are admitted in order as slots free up; each gets the tokens it would get
 * alone at this slot count. Checks every id; synchronous. */
int gpt2_engine_serve(gpt2_engine *e, gpt2_request *reqs, int n_req, int slots);

/* Sampling of every following prefill and decode step (gpt2.c:2176-2245).
 * temperature <= 0 (the default): greedy. Otherwise top-k sampling at that
 * temperature (w8a8_sample_topk; top_k clamped to [1, vocab], default 40):
 * slot b's i-th token (i from 0; the prefill writes i = 0) is drawn with the
 * i-th value set by gpt2_engine_set_draws for slot b (0 where none was set).
 * The reference draws (float)rand() / RAND_MAX for each token (gpt2.c:2231). */
int gpt2_engine_set_sampling(gpt2_engine *e, float temperature, int top_k);
/* draws[0..n) (host memory, n <= ctx) become slot `slot`'s draws from its
 * first token on; ordered on the engine stream after the work queued so far. */
int gpt2_engine_set_draws(gpt2_engine *e, int slot, const float *draws, int n);
/* The draws of the reference's sampling loop for one sequence: out[i] =
 * (float)rand() / RAND_MAX at the i-th call of glibc's rand() after
 * srand(seed) (gpt2.c:2231; the reference never seeds, which is seed 1),
 * from a private generator state (the process's rand() is not touched). */
int gpt2_reference_draws(unsigned seed, float *out, int n);

/* Copy the logits of the last step ([B, vocab] bf16) to host memory. */
int gpt2_engine_copy_logits(gpt2_engine *e, gpt2_bf16_t *host, int rows);
/* Decode steps as one chain of kernels over all B slots (1, the default) or
 * as two independent chains over the first ceil(B/2) and the other slots,
 * run at the same time on two streams (2). Tokens are the same either way. */
int gpt2_engine_set_decode_split(gpt2_engine *e, int halves);
/* Enable (default) or disable CUDA-graph replay of decode steps. */
int gpt2_engine_set_graphs(gpt2_engine *e, int enable);
/* Kernel launches per decode step (for launch accounting). */
int gpt2_engine_launches_per_decode_step(const gpt2_engine *e);
int gpt2_engine_launches_per_prefill(const gpt2_engine *e);
void *gpt2_engine_stream(gpt2_engine *e);
const char *gpt2_engine_last_error(const gpt2_engine *e);

#ifdef __cplusplus
}
#endif

#endif /* GPT2_ENGINE_H */
