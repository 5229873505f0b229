/*
 * paged_kv_cache.c -- C11 page allocator behind include/paged_kv_cache.h.
 *
 * Written from the behaviour of the inference SDK's
 * src/common/paged_kv_cache.c (reference lines 7-309).  Everything a caller
 * can observe is kept identical, because block tables produced here are
 * compared bit-for-bit with the SDK's:
 *   - the free stack starts as [n-1, ..., 1, 0] so pages pop as 0, 1, 2, ...
 *     (reference :71-72) and reserve pops from the top (:151-152);
 *   - set_length pushes trailing pages back last-page-first (:170-172);
 *   - release pushes the table first-page-first (:234-235), so the next
 *     reserve receives the released sequence's last page first;
 *   - handles are (generation << 32) | (slot + 1), generation skips 0
 *     (:31-44, :96-97);
 *   - the backend release hook runs after the lock is dropped (:231-241).
 * The data structure is this file's own: a per-sequence growable page vector
 * and one mutex per cache.
 */
#include "paged_kv_cache.h"
#include "pkv_internal.h"

#include <pthread.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    uint32_t *pages;       /* logical page -> page id */
    size_t page_count;
    size_t page_capacity;
    size_t length;         /* visible tokens */
    uint32_t generation;   /* bumped on every create of this slot */
    uint32_t shrink_epoch; /* bumped whenever pages leave the table */
    unsigned char live;
    unsigned char decoding;
} SeqSlot;

struct TensorPagedKVCache {
    pthread_mutex_t lock;
    size_t page_tokens;
    size_t page_total;
    uint32_t *free_stack;  /* free page ids; top is free_stack[free_top-1] */
    size_t free_top;
    SeqSlot *slots;
    size_t slot_total;
    TensorPagedKVBackendStateKind payload_kind;
    void *payload;
    TensorPagedKVBackendStateDestroy payload_destroy;
    TensorPagedKVBackendSequenceRelease payload_release;
};

static TensorPagedKVSequence encode_handle(size_t slot, uint32_t generation) {
    return ((uint64_t)generation << 32) | (uint64_t)(uint32_t)(slot + 1u);
}

/* Caller holds the lock.  NULL for 0, stale or out-of-range handles. */
static SeqSlot *lookup(TensorPagedKVCache *c, TensorPagedKVSequence h) {
    const uint32_t slot_plus_one = (uint32_t)(h & 0xffffffffu);
    const uint32_t generation = (uint32_t)(h >> 32);
    if (slot_plus_one == 0u || generation == 0u) return NULL;
    if ((size_t)(slot_plus_one - 1u) >= c->slot_total) return NULL;
    SeqSlot *s = &c->slots[slot_plus_one - 1u];
    if (!s->live || s->generation != generation) return NULL;
    return s;
}

static size_t pages_for(size_t tokens, size_t page_tokens) {
    return tokens / page_tokens + (tokens % page_tokens != 0);
}

/* What a cache needs from its sizes: at least one token per page, one page
 * and one sequence slot; page ids and slot numbers travel as 32-bit values
 * (block tables, the low half of a handle); the token count of the whole
 * pool and the two host arrays must be representable. */
static int cache_sizes_valid(size_t block_size, size_t block_count, size_t max_sequences) {
    if (block_size == 0 || block_count == 0 || max_sequences == 0) return 0;
    const int ids_fit = block_count <= UINT32_MAX && max_sequences <= UINT32_MAX;
    const int tokens_fit = block_count <= SIZE_MAX / block_size;
    const int arrays_fit = block_count <= SIZE_MAX / sizeof(uint32_t) &&
                           max_sequences <= SIZE_MAX / sizeof(SeqSlot);
    return ids_fit && tokens_fit && arrays_fit;
}

int tensor_paged_kv_cache_create(size_t block_size, size_t block_count,
                                 size_t max_sequences,
                                 TensorPagedKVCache **cache) {
    if (cache == NULL || !cache_sizes_valid(block_size, block_count, max_sequences)) return 0;
    *cache = NULL;
    TensorPagedKVCache *c = (TensorPagedKVCache *)calloc(1, sizeof(*c));
    if (c == NULL) return 0;
    c->free_stack = (uint32_t *)malloc(block_count * sizeof(uint32_t));
    c->slots = (SeqSlot *)calloc(max_sequences, sizeof(SeqSlot));
    if (c->free_stack == NULL || c->slots == NULL ||
        pthread_mutex_init(&c->lock, NULL) != 0) {
        free(c->free_stack);
        free(c->slots);
        free(c);
        return 0;
    }
    c->page_tokens = block_size;
    c->page_total = block_count;
    c->slot_total = max_sequences;
    /* Bottom of the stack holds the highest id, so pops yield 0, 1, 2, ... */
    for (size_t k = 0; k < block_count; ++k)
        c->free_stack[k] = (uint32_t)(block_count - 1u - k);
    c->free_top = block_count;
    *cache = c;
    return 1;
}

void tensor_paged_kv_cache_free(TensorPagedKVCache *cache) {
    if (cache == NULL) return;
    if (cache->payload != NULL && cache->payload_destroy != NULL)
        cache->payload_destroy(cache->payload);
    for (size_t k = 0; k < cache->slot_total; ++k) free(cache->slots[k].pages);
    pthread_mutex_destroy(&cache->lock);
    free(cache->slots);
    free(cache->free_stack);
    free(cache);
}

int tensor_paged_kv_sequence_create(TensorPagedKVCache *cache,
                                    TensorPagedKVSequence *sequence) {
    if (cache == NULL || sequence == NULL) return 0;
    int ok = 0;
    pthread_mutex_lock(&cache->lock);
    for (size_t k = 0; k < cache->slot_total; ++k) {
        SeqSlot *s = &cache->slots[k];
        if (s->live) continue;
        s->generation = s->generation + 1u == 0u ? 1u : s->generation + 1u;
        s->live = 1;
        s->decoding = 0;
        s->length = 0;
        s->page_count = 0;
        *sequence = encode_handle(k, s->generation);
        ok = 1;
        break;
    }
    pthread_mutex_unlock(&cache->lock);
    return ok;
}

/* Caller holds the lock.  Makes room for `need` page ids in the slot.  The
 * vector grows by half its size (to at least `need` and at least 16 ids), so
 * a sequence that gains a page per step reallocates a logarithmic number of
 * times; the capacity is not observable through the API. */
static int grow_pages(SeqSlot *s, size_t need) {
    if (need <= s->page_capacity) return 1;
    if (need > SIZE_MAX / sizeof(uint32_t)) return 0;
    size_t cap = s->page_capacity + s->page_capacity / 2u;
    if (cap < need) cap = need;
    if (cap < 16u) cap = 16u;
    if (cap > SIZE_MAX / sizeof(uint32_t)) cap = need;
    uint32_t *p = (uint32_t *)realloc(s->pages, cap * sizeof(uint32_t));
    if (p == NULL) return 0;
    s->pages = p;
    s->page_capacity = cap;
    return 1;
}

int tensor_paged_kv_sequence_reserve(TensorPagedKVCache *cache,
                                     TensorPagedKVSequence sequence,
                                     size_t token_capacity) {
    if (cache == NULL || token_capacity > SIZE_MAX - (cache->page_tokens - 1u))
        return 0;
    const size_t need = pages_for(token_capacity, cache->page_tokens);
    int ok = 0;
    pthread_mutex_lock(&cache->lock);
    SeqSlot *s = lookup(cache, sequence);
    if (s != NULL) {
        if (need <= s->page_count) {
            ok = 1;
        } else if (need - s->page_count <= cache->free_top && grow_pages(s, need)) {
            while (s->page_count < need)
                s->pages[s->page_count++] = cache->free_stack[--cache->free_top];
            ok = 1;
        }
    }
    pthread_mutex_unlock(&cache->lock);
    return ok;
}

int tensor_paged_kv_sequence_set_length(TensorPagedKVCache *cache,
                                        TensorPagedKVSequence sequence,
                                        size_t token_length) {
    if (cache == NULL) return 0;
    int ok = 0;
    pthread_mutex_lock(&cache->lock);
    SeqSlot *s = lookup(cache, sequence);
    if (s != NULL && token_length <= s->page_count * cache->page_tokens) {
        const size_t keep = pages_for(token_length, cache->page_tokens);
        if (s->page_count > keep) s->shrink_epoch++;
        while (s->page_count > keep)
            cache->free_stack[cache->free_top++] = s->pages[--s->page_count];
        s->length = token_length;
        ok = 1;
    }
    pthread_mutex_unlock(&cache->lock);
    return ok;
}

int tensor_paged_kv_sequence_copy_block_table(TensorPagedKVCache *cache,
                                              TensorPagedKVSequence sequence,
                                              uint32_t *block_ids,
                                              size_t block_id_capacity,
                                              size_t *block_count) {
    if (cache == NULL || block_count == NULL) return 0;
    int ok = 0;
    pthread_mutex_lock(&cache->lock);
    SeqSlot *s = lookup(cache, sequence);
    if (s != NULL) {
        *block_count = s->page_count;
        if (block_ids == NULL) {
            ok = 1;
        } else if (block_id_capacity >= s->page_count) {
            if (s->page_count)
                memcpy(block_ids, s->pages, s->page_count * sizeof(uint32_t));
            ok = 1;
        }
    }
    pthread_mutex_unlock(&cache->lock);
    return ok;
}

int tensor_paged_kv_sequence_length(TensorPagedKVCache *cache,
                                    TensorPagedKVSequence sequence,
                                    size_t *token_length) {
    if (cache == NULL || token_length == NULL) return 0;
    int ok = 0;
    pthread_mutex_lock(&cache->lock);
    SeqSlot *s = lookup(cache, sequence);
    if (s != NULL) {
        *token_length = s->length;
        ok = 1;
    }
    pthread_mutex_unlock(&cache->lock);
    return ok;
}

int tensor_paged_kv_sequence_release(TensorPagedKVCache *cache,
                                     TensorPagedKVSequence sequence) {
    if (cache == NULL) return 0;
    void *payload = NULL;
    TensorPagedKVBackendSequenceRelease hook = NULL;
    pthread_mutex_lock(&cache->lock);
    SeqSlot *s = lookup(cache, sequence);
    if (s == NULL || s->decoding) {
        pthread_mutex_unlock(&cache->lock);
        return 0;
    }
    for (size_t k = 0; k < s->page_count; ++k)
        cache->free_stack[cache->free_top++] = s->pages[k];
    s->page_count = 0;
    s->length = 0;
    s->live = 0;
    s->shrink_epoch++;
    payload = cache->payload;
    hook = cache->payload_release;
    pthread_mutex_unlock(&cache->lock);
    if (hook != NULL && payload != NULL) hook(payload, sequence);
    return 1;
}

int tensor_paged_kv_sequence_begin_decode(TensorPagedKVCache *cache,
                                          TensorPagedKVSequence sequence) {
    if (cache == NULL) return 0;
    int ok = 0;
    pthread_mutex_lock(&cache->lock);
    SeqSlot *s = lookup(cache, sequence);
    if (s != NULL && !s->decoding) {
        s->decoding = 1;
        ok = 1;
    }
    pthread_mutex_unlock(&cache->lock);
    return ok;
}

void tensor_paged_kv_sequence_end_decode(TensorPagedKVCache *cache,
                                         TensorPagedKVSequence sequence) {
    if (cache == NULL) return;
    pthread_mutex_lock(&cache->lock);
    SeqSlot *s = lookup(cache, sequence);
    if (s != NULL) s->decoding = 0;
    pthread_mutex_unlock(&cache->lock);
}

size_t tensor_paged_kv_cache_free_blocks(TensorPagedKVCache *cache) {
    if (cache == NULL) return 0;
    pthread_mutex_lock(&cache->lock);
    const size_t n = cache->free_top;
    pthread_mutex_unlock(&cache->lock);
    return n;
}

size_t tensor_paged_kv_cache_block_size(const TensorPagedKVCache *cache) {
    return cache == NULL ? 0 : cache->page_tokens;
}

size_t tensor_paged_kv_cache_block_count(const TensorPagedKVCache *cache) {
    return cache == NULL ? 0 : cache->page_total;
}

void *tensor_paged_kv_cache_backend_state(TensorPagedKVCache *cache,
                                          TensorPagedKVBackendStateKind kind) {
    if (cache == NULL) return NULL;
    pthread_mutex_lock(&cache->lock);
    void *p = cache->payload_kind == kind ? cache->payload : NULL;
    pthread_mutex_unlock(&cache->lock);
    return p;
}

int tensor_paged_kv_cache_set_backend_state(
    TensorPagedKVCache *cache, TensorPagedKVBackendStateKind kind, void *state,
    TensorPagedKVBackendStateDestroy destroy_state,
    TensorPagedKVBackendSequenceRelease release_sequence) {
    if (cache == NULL || state == NULL || destroy_state == NULL) return 0;
    int ok = 0;
    pthread_mutex_lock(&cache->lock);
    if (cache->payload == NULL) {
        cache->payload_kind = kind;
        cache->payload = state;
        cache->payload_destroy = destroy_state;
        cache->payload_release = release_sequence;
        ok = 1;
    }
    pthread_mutex_unlock(&cache->lock);
    return ok;
}

/* Host-layer helper (pkv_internal.h): the page ids from index `from` on, the
 * page count, the visible length and the shrink epoch, in one lock round
 * trip.  A changed epoch tells the caller that earlier entries may differ. */
int pkv_internal_copy_table_tail(TensorPagedKVCache *cache,
                                 TensorPagedKVSequence sequence, size_t from,
                                 uint32_t *dst, size_t capacity,
                                 size_t *page_count, size_t *length,
                                 uint32_t *shrink_epoch) {
    if (cache == NULL || page_count == NULL) return 0;
    int ok = 0;
    pthread_mutex_lock(&cache->lock);
    SeqSlot *s = lookup(cache, sequence);
    if (s != NULL) {
        *page_count = s->page_count;
        if (length != NULL) *length = s->length;
        if (shrink_epoch != NULL) *shrink_epoch = s->shrink_epoch;
        const size_t n = s->page_count > from ? s->page_count - from : 0;
        if (dst == NULL) {
            ok = 1;
        } else if (n <= capacity) {
            if (n) memcpy(dst, s->pages + from, n * sizeof(uint32_t));
            ok = 1;
        }
    }
    pthread_mutex_unlock(&cache->lock);
    return ok;
}
