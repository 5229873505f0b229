/*
 * alloc_stress.c -- multi-threaded stress of the page allocator
 * (inference_c_b200/csrc/paged_kv_cache.c), built by tests/test_sanitizers.py
 * under AddressSanitizer + UndefinedBehaviorSanitizer and under
 * ThreadSanitizer.  TEST ONLY.
 *
 * Eight threads create sequences, reserve, shrink, copy block tables, take
 * and drop the decode lock and release, while an ownership array checks
 * that no page is ever held by two sequences.  A backend payload is attached
 * whose release hook calls back into the cache (it would deadlock if the
 * hook ran under the cache lock) and counts its calls.  At the end every page
 * is free again.  Prints "stress ok" and exits 0 on success.
 */
#include <pthread.h>
#include <stdatomic.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "paged_kv_cache.h"

enum { kBlock = 16, kPages = 512, kSeqs = 64, kThreads = 8, kIters = 3000 };

static TensorPagedKVCache *g_cache;
static atomic_int g_owner[kPages];
static atomic_int g_errors;
static atomic_int g_hook_calls;
static int g_payload;

static void fail(const char *what) {
    atomic_fetch_add(&g_errors, 1);
    fprintf(stderr, "stress: %s\n", what);
}

static void destroy_payload(void *state) { (void)state; }

static void release_hook(void *state, TensorPagedKVSequence sequence) {
    (void)sequence;
    if (state != &g_payload) fail("release hook got the wrong payload");
    (void)tensor_paged_kv_cache_free_blocks(g_cache); /* takes the cache lock */
    atomic_fetch_add(&g_hook_calls, 1);
}

/* Marks (owner = id) or clears (owner = 0) the pages of a block table. */
static void mark(const uint32_t *pages, size_t n, int id) {
    for (size_t i = 0; i < n; ++i) {
        if (pages[i] >= kPages) { fail("page id out of range"); continue; }
        const int prev = atomic_exchange(&g_owner[pages[i]], id);
        if (id != 0 && prev != 0) fail("page held by two sequences");
        if (id == 0 && prev == 0) fail("page released twice");
    }
}

static void *worker(void *arg) {
    const int id = (int)(intptr_t)arg;
    unsigned seed = 1234u + (unsigned)id * 7919u;
    uint32_t pages[kPages];
    size_t held = 0;
    for (int it = 0; it < kIters; ++it) {
        TensorPagedKVSequence s = 0;
        if (!tensor_paged_kv_sequence_create(g_cache, &s)) continue;
        const size_t want = 1 + (size_t)(rand_r(&seed) % (kBlock * 24));
        if (tensor_paged_kv_sequence_reserve(g_cache, s, want)) {
            size_t count = 0;
            if (!tensor_paged_kv_sequence_copy_block_table(g_cache, s, pages, kPages, &count) ||
                count != (want + kBlock - 1) / kBlock)
                fail("block table of a reserved sequence");
            mark(pages, count, id);
            held = count;
            if (!tensor_paged_kv_sequence_begin_decode(g_cache, s)) fail("begin_decode");
            if (tensor_paged_kv_sequence_begin_decode(g_cache, s)) fail("double begin_decode");
            if (tensor_paged_kv_sequence_release(g_cache, s)) fail("release while decoding");
            tensor_paged_kv_sequence_end_decode(g_cache, s);
            const size_t shorter = (size_t)(rand_r(&seed) % (want + 1));
            const size_t keep = (shorter + kBlock - 1) / kBlock;
            mark(pages + keep, held - keep, 0); /* unmark before the pages go back */
            if (!tensor_paged_kv_sequence_set_length(g_cache, s, shorter)) fail("set_length");
            held = keep;
            size_t len = 0;
            if (!tensor_paged_kv_sequence_length(g_cache, s, &len) || len != shorter)
                fail("length after set_length");
        } else {
            held = 0;
        }
        mark(pages, held, 0);
        if (!tensor_paged_kv_sequence_release(g_cache, s)) fail("release");
        if (tensor_paged_kv_sequence_reserve(g_cache, s, 1)) fail("stale handle accepted");
    }
    return NULL;
}

int main(void) {
    if (!tensor_paged_kv_cache_create(kBlock, kPages, kSeqs, &g_cache)) return 2;
    if (!tensor_paged_kv_cache_set_backend_state(g_cache, TENSOR_PAGED_KV_BACKEND_CUDA,
                                                 &g_payload, destroy_payload, release_hook))
        return 3;
    pthread_t t[kThreads];
    for (int i = 0; i < kThreads; ++i)
        if (pthread_create(&t[i], NULL, worker, (void *)(intptr_t)(i + 1)) != 0) return 4;
    for (int i = 0; i < kThreads; ++i) pthread_join(t[i], NULL);
    if (tensor_paged_kv_cache_free_blocks(g_cache) != kPages) fail("pages leaked");
    for (int p = 0; p < kPages; ++p)
        if (atomic_load(&g_owner[p]) != 0) fail("page still marked");
    if (atomic_load(&g_hook_calls) == 0) fail("release hook never ran");
    tensor_paged_kv_cache_free(g_cache);
    if (atomic_load(&g_errors) != 0) return 1;
    printf("stress ok (%d release hook calls)\n", atomic_load(&g_hook_calls));
    return 0;
}
