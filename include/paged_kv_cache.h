/*
 * paged_kv_cache.h -- host-side page allocator for a paged KV cache.
 *
 * This header declares the same C API as the inference SDK's
 * include/paged_kv_cache.h (reference lines 23-65): identical function names,
 * argument order, types and 1-on-success / 0-on-failure results, so that code
 * written against the SDK links against libpkv_b200.so unchanged.  The include
 * guard is the SDK's own so the two headers can never both be active.
 *
 * Semantics (implemented in inference_c_b200/csrc/paged_kv_cache.c):
 *   - a cache owns `block_count` pages of `block_size` token slots each;
 *   - free pages sit on a LIFO stack initialised so a fresh cache hands out
 *     page 0, 1, 2, ... in that order;
 *   - each sequence owns an ordered block table (logical page i -> page id);
 *   - handles are (generation << 32) | (slot + 1); 0 is never a valid handle
 *     and a released slot's old handle stays invalid after the slot is reused;
 *   - reserve is all-or-nothing; set_length frees whole trailing pages;
 *   - begin/end_decode is a per-sequence lock that also blocks release;
 *   - one device backend may attach its payload (the page memory itself) with
 *     a destroy callback (run by cache_free) and a per-sequence release hook
 *     (run by sequence_release after the allocator lock is dropped).
 */
#ifndef PAGED_KV_CACHE_H
#define PAGED_KV_CACHE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct TensorPagedKVCache TensorPagedKVCache;
typedef uint64_t TensorPagedKVSequence;
typedef void (*TensorPagedKVBackendStateDestroy)(void *state);
typedef void (*TensorPagedKVBackendSequenceRelease)(void *state,
                                                     TensorPagedKVSequence sequence);
typedef enum {
    TENSOR_PAGED_KV_BACKEND_CUDA = 1,
    TENSOR_PAGED_KV_BACKEND_METAL = 2
} TensorPagedKVBackendStateKind;

/* Creates a cache of block_count pages of block_size tokens and room for
 * max_sequences live sequences. */
int tensor_paged_kv_cache_create(size_t block_size, size_t block_count,
                                 size_t max_sequences,
                                 TensorPagedKVCache **cache);
/* Runs the attached backend's destroy callback, then frees all metadata. */
void tensor_paged_kv_cache_free(TensorPagedKVCache *cache);
/* Takes the first free sequence slot; the new sequence has length 0. */
int tensor_paged_kv_sequence_create(TensorPagedKVCache *cache,
                                    TensorPagedKVSequence *sequence);
/* Grows the block table to cover token_capacity tokens; the visible length
 * is unchanged.  Fails without side effects when pages run out. */
int tensor_paged_kv_sequence_reserve(TensorPagedKVCache *cache,
                                     TensorPagedKVSequence sequence,
                                     size_t token_capacity);
/* Sets the visible length (at most the reserved capacity) and returns any
 * whole trailing pages that the new length no longer needs. */
int tensor_paged_kv_sequence_set_length(TensorPagedKVCache *cache,
                                        TensorPagedKVSequence sequence,
                                        size_t token_length);
/* Snapshots the block table under the allocator lock.  With block_ids NULL
 * only *block_count is written; a too-small capacity fails. */
int tensor_paged_kv_sequence_copy_block_table(TensorPagedKVCache *cache,
                                              TensorPagedKVSequence sequence,
                                              uint32_t *block_ids,
                                              size_t block_id_capacity,
                                              size_t *block_count);
int tensor_paged_kv_sequence_length(TensorPagedKVCache *cache,
                                    TensorPagedKVSequence sequence,
                                    size_t *token_length);
/* Returns every page of the sequence; fails while a decode is active. */
int tensor_paged_kv_sequence_release(TensorPagedKVCache *cache,
                                     TensorPagedKVSequence sequence);
/* Per-sequence decode lock: a second begin fails until end is called. */
int tensor_paged_kv_sequence_begin_decode(TensorPagedKVCache *cache,
                                          TensorPagedKVSequence sequence);
void tensor_paged_kv_sequence_end_decode(TensorPagedKVCache *cache,
                                         TensorPagedKVSequence sequence);
size_t tensor_paged_kv_cache_free_blocks(TensorPagedKVCache *cache);
size_t tensor_paged_kv_cache_block_size(const TensorPagedKVCache *cache);
size_t tensor_paged_kv_cache_block_count(const TensorPagedKVCache *cache);
/* Backend payload lookup; NULL unless a payload of this kind is attached. */
void *tensor_paged_kv_cache_backend_state(TensorPagedKVCache *cache,
                                          TensorPagedKVBackendStateKind kind);
/* Attaches the single backend payload; a second attach fails. */
int tensor_paged_kv_cache_set_backend_state(
    TensorPagedKVCache *cache, TensorPagedKVBackendStateKind kind, void *state,
    TensorPagedKVBackendStateDestroy destroy_state,
    TensorPagedKVBackendSequenceRelease release_sequence);

#ifdef __cplusplus
}
#endif

#endif
