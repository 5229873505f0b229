/*
 * attention.h -- the inference SDK's paged decoder entry points, served by
 * libpkv_b200.so.
 *
 * This is the paged subset of the SDK's include/attention.h (types at
 * include/attention.h:20-72, functions at :128-130) with identical names,
 * field order and types, so a caller compiled against the SDK's header links
 * against this library unchanged.  The include guard is the SDK's, so only
 * one of the two definitions is ever seen.  TensorWeightQuantization is the
 * SDK's enum (include/tensor_quant.h:10-13).
 *
 * tensor_attention_decode_sequence_paged replaces the SDK's transaction
 * (src/common/attention.c:124-176) together with its CUDA backend
 * (src/platform/cuda/attention_cuda.cu:754-1090): greedy decoding of
 * token_count tokens for one sequence, every layer's K/V appended to the
 * cache's pages (RoPE applied to K), the first call importing past_length
 * positions from the host key_cache/value_cache arrays.  Returns 1 on success,
 * 0 on failure (the sequence keeps its previous length).
 */
#ifndef ATTENTION_H
#define ATTENTION_H

#include <stddef.h>
#include <stdint.h>

#include "paged_kv_cache.h"

#ifdef __cplusplus
extern "C" {
#endif

#ifndef TENSOR_QUANT_H
#define TENSOR_QUANT_H
typedef enum {
    TENSOR_WEIGHT_Q8_0 = 1, /* 32 weights: fp16 scale + 32 int8 (34 bytes) */
    TENSOR_WEIGHT_Q4_0 = 2  /* 32 weights: fp16 scale + 16 bytes of nibbles, value q - 8 (18 bytes) */
} TensorWeightQuantization;
#endif

/* Row-major [out][in] matrices; norms are vectors of hidden_size. */
typedef struct {
    const float *input_norm;
    const float *q_weight;
    const float *k_weight;
    const float *v_weight;
    const float *o_weight;
    const float *post_norm;
    const float *gate_weight;
    const float *up_weight;
    const float *down_weight;
} TensorAttentionDecoderLayer;

typedef struct {
    const uint16_t *input_norm, *q_weight, *k_weight, *v_weight, *o_weight;
    const uint16_t *post_norm, *gate_weight, *up_weight, *down_weight;
} TensorAttentionDecoderLayerF16;

typedef struct {
    const uint16_t *input_norm, *post_norm;
    const uint8_t *q_weight, *k_weight, *v_weight, *o_weight;
    const uint8_t *gate_weight, *up_weight, *down_weight;
} TensorAttentionDecoderLayerQuantF16;

typedef enum {
    TENSOR_PAGED_KV_F32 = 0,       /* F32 weights, activations and pages */
    TENSOR_PAGED_KV_F16 = 1,       /* F16 weights, activations and pages */
    TENSOR_PAGED_KV_QUANT_F16 = 2  /* Q8_0/Q4_0 matrices, F16 norms, activations and pages */
} TensorPagedKVStorage;

typedef struct {
    TensorPagedKVCache *cache;
    TensorPagedKVSequence sequence;
    TensorPagedKVStorage storage;
    const void *layers;             /* layer_count layer structs of the storage's kind */
    size_t layer_count;
    const void *embedding;          /* [vocabulary_size][hidden_size] */
    uint32_t initial_token;
    size_t token_count;
    uint32_t *generated_tokens;     /* token_count outputs (host) */
    const void *const *key_cache;   /* per layer, host [>= past_length][kv_width]: prefix import */
    const void *const *value_cache;
    size_t past_length;
    size_t hidden_size;             /* = query_heads * head_dim */
    size_t intermediate_size;
    size_t query_heads;
    size_t kv_heads;
    size_t head_dim;
    float rms_norm_epsilon;
    double rope_theta;
    const void *final_norm;
    const void *lm_head;            /* [vocabulary_size][hidden_size] (quantised for QUANT_F16) */
    size_t vocabulary_size;
    TensorWeightQuantization weight_quantization;
} TensorPagedKVDecodeRequest;

int tensor_attention_decode_sequence_paged(const TensorPagedKVDecodeRequest *request);

/* Frees the device copies of weights this library made (they are keyed by
 * host pointer, as in the SDK's CUDA backend). */
void tensor_attention_decode_cache_clear(void);

#ifdef __cplusplus
}
#endif

#endif
