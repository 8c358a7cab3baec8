/*
 * gpt2_model_config.h — model dimensions and element types of the W8A8 build,
 * in the form the reference's kernel ABI expects (include/model_config.h of
 * the reference: vocab_size, ctx_len, d_model, num_layers, nof_heads,
 * head_dim, d_ff; act_t / weight_t = bf16, qweight_t = int8, qscale_t = fp32
 * under USE_BF16 + USE_INT8, model_config.h:41-80).
 *
 * Select the size with -DGPT2_SMALL_MODEL, -DGPT2_MEDIUM_MODEL or
 * -DGPT2_LARGE_MODEL (default: medium, as in the reference).
 */
#pragma once

#include <stddef.h>
#include <stdint.h>

#define vocab_size (50257)
#define ctx_len (1024)

#if !defined(GPT2_SMALL_MODEL) && !defined(GPT2_MEDIUM_MODEL) && !defined(GPT2_LARGE_MODEL)
#define GPT2_MEDIUM_MODEL
#endif

#if defined(GPT2_SMALL_MODEL)
#define d_model (768)
#define num_layers (12)
#define nof_heads (12)
#elif defined(GPT2_MEDIUM_MODEL)
#define d_model (1024)
#define num_layers (24)
#define nof_heads (16)
#else
#define d_model (1280)
#define num_layers (36)
#define nof_heads (20)
#endif

#define head_dim (d_model / nof_heads)
#define d_ff (d_model * 4)

#if defined(__CUDACC__)
#include <cuda_bf16.h>
typedef __nv_bfloat16 act_t;
typedef __nv_bfloat16 weight_t;
#else
typedef __bf16 act_t;
typedef __bf16 weight_t;
#endif
typedef int8_t qweight_t;
typedef float qscale_t;
