/*
 * pkv_pool.c -- C11 host layer: device page pool + batch step transaction.
 *
 * The pool is the CUDA payload of a TensorPagedKVCache, attached with the
 * SDK's own hook tensor_paged_kv_cache_set_backend_state (as
 * get_cuda_paged_kv_state does, attention_cuda.cu:570-612): per layer one K
 * and one V array of [block_count * block_size][kv_heads * head_dim]
 * elements, zero-initialised, freed by the cache's destroy callback.
 *
 * The step functions are the SDK transaction of
 * tensor_attention_decode_sequence_paged (attention.c:124-176) applied to a
 * whole batch: begin_decode, length check (0 or past), reserve(past + new),
 * device work, then set_length(target) on success or set_length(current) on
 * failure, and end_decode.  Unlike the SDK, which re-uploads every block
 * table for every layer on every call (attention_cuda.cu:877-893), the pool
 * keeps one padded device table per batch row and sends only entries that
 * changed, together with the step's lengths, once per step for all layers:
 * the host writes them into a pinned, device-mapped staging slot and one
 * small kernel on the step's stream reads the slot over the bus and applies
 * it (no copy engine round trip; launched with programmatic dependent launch
 * so it chains with the append and decode kernels).  That kernel marks the
 * slot consumed in host memory; the host waits for the mark before it
 * refills the slot two steps later.
 */
#include <cuda_runtime_api.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "pkv_b200.h"
#include "pkv_internal.h"
#include "pkv_trace.h"

enum { kStageSlots = 2 };

typedef struct {
    TensorPagedKVSequence seq;  /* sequence whose pages the row holds (0: none) */
    size_t pages;               /* entries of that sequence already uploaded */
    uint32_t epoch;             /* its shrink epoch when they were uploaded */
} RowState;

struct PkvPool {
    TensorPagedKVCache *cache;
    int device;
    PkvDType dtype;
    size_t layer_count, kv_heads, head_dim, block_size, block_count;
    size_t max_batch, max_pages;
    void **kpools;
    void **vpools;
    uint32_t *d_tables;           /* [max_batch][max_pages] */
    RowState *rows;
    uint32_t *tmp_pages;          /* max_pages */
    /* staging: [seq_lens i32 max_batch][row_offsets i32 max_batch+1][pad][patches];
     * h_stage is pinned and device-mapped (h_stage_dev: its device address),
     * d_stage holds the applied lengths and offsets the kernels read */
    size_t stage_bytes, patch_offset, patch_capacity;
    unsigned char *h_stage[kStageSlots];
    unsigned char *h_stage_dev[kStageSlots];
    unsigned char *d_stage[kStageSlots];
    uint32_t *h_consumed;         /* [kStageSlots], pinned and mapped: last ticket applied */
    uint32_t *h_consumed_dev;
    uint32_t stage_ticket[kStageSlots];  /* ticket of the slot's last use (0: none) */
    uint32_t next_ticket;
    int slot;
    /* open step */
    int open;
    size_t step_batch;
    TensorPagedKVSequence *step_seq;
    size_t *step_current;
    size_t *step_target;
};

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

static void pool_free_device(PkvPool *p) {
    int prev = 0;
    const int have_prev = cudaGetDevice(&prev) == cudaSuccess;
    cudaSetDevice(p->device);
    if (p->kpools)
        for (size_t l = 0; l < p->layer_count; ++l) cudaFree(p->kpools[l]);
    if (p->vpools)
        for (size_t l = 0; l < p->layer_count; ++l) cudaFree(p->vpools[l]);
    cudaFree(p->d_tables);
    for (int s = 0; s < kStageSlots; ++s) {
        cudaFreeHost(p->h_stage[s]);
        cudaFree(p->d_stage[s]);
    }
    cudaFreeHost(p->h_consumed);
    if (have_prev) cudaSetDevice(prev);
}

static void pool_destroy(void *state) {
    PkvPool *p = (PkvPool *)state;
    if (p == NULL) return;
    pool_free_device(p);
    free(p->kpools);
    free(p->vpools);
    free(p->rows);
    free(p->tmp_pages);
    free(p->step_seq);
    free(p->step_current);
    free(p->step_target);
    free(p);
}

/* Release hook: the row that held the sequence must be re-uploaded. */
static void pool_release_sequence(void *state, TensorPagedKVSequence sequence) {
    PkvPool *p = (PkvPool *)state;
    for (size_t r = 0; r < p->max_batch; ++r)
        if (p->rows[r].seq == sequence) p->rows[r].seq = 0;
}

int pkv_pool_create(TensorPagedKVCache *cache, int device, PkvDType dtype,
                    size_t layer_count, size_t kv_heads, size_t head_dim,
                    size_t max_batch, size_t max_pages_per_seq, PkvPool **pool,
                    char *error, size_t cap) {
    if (pool == NULL || cache == NULL) {
        pkv_internal_set_error(error, cap, "pkv_pool_create: null argument");
        return 0;
    }
    *pool = NULL;
    if ((dtype != PKV_DTYPE_F16 && dtype != PKV_DTYPE_BF16 && dtype != PKV_DTYPE_F32) ||
        layer_count == 0 || kv_heads == 0 || head_dim == 0 ||
        max_batch == 0 || max_batch > INT32_MAX || max_pages_per_seq == 0 ||
        max_pages_per_seq > INT32_MAX) {
        pkv_internal_set_error(error, cap, "pkv_pool_create: invalid shape or dtype");
        return 0;
    }
    if (tensor_paged_kv_cache_backend_state(cache, TENSOR_PAGED_KV_BACKEND_CUDA) != NULL) {
        pkv_internal_set_error(error, cap, "pkv_pool_create: cache already has a CUDA pool");
        return 0;
    }
    PkvPool *p = (PkvPool *)calloc(1, sizeof(*p));
    if (p == NULL) return 0;
    p->cache = cache;
    p->device = device;
    p->dtype = dtype;
    p->layer_count = layer_count;
    p->kv_heads = kv_heads;
    p->head_dim = head_dim;
    p->block_size = tensor_paged_kv_cache_block_size(cache);
    p->block_count = tensor_paged_kv_cache_block_count(cache);
    p->max_batch = max_batch;
    p->max_pages = max_pages_per_seq;
    p->kpools = (void **)calloc(layer_count, sizeof(void *));
    p->vpools = (void **)calloc(layer_count, sizeof(void *));
    p->rows = (RowState *)calloc(max_batch, sizeof(RowState));
    p->tmp_pages = (uint32_t *)malloc(max_pages_per_seq * sizeof(uint32_t));
    p->step_seq = (TensorPagedKVSequence *)calloc(max_batch, sizeof(TensorPagedKVSequence));
    p->step_current = (size_t *)calloc(max_batch, sizeof(size_t));
    p->step_target = (size_t *)calloc(max_batch, sizeof(size_t));
    if (!p->kpools || !p->vpools || !p->rows || !p->tmp_pages || !p->step_seq ||
        !p->step_current || !p->step_target) {
        pool_destroy(p);
        pkv_internal_set_error(error, cap, "pkv_pool_create: out of host memory");
        return 0;
    }
    int prev = 0;
    const int have_prev = cudaGetDevice(&prev) == cudaSuccess;
    cudaError_t st = cudaSetDevice(device);
    const size_t kv_width = kv_heads * head_dim;
    const size_t elem = dtype == PKV_DTYPE_F32 ? 4u : 2u;
    const size_t pool_bytes = p->block_count * p->block_size * kv_width * elem;
    for (size_t l = 0; st == cudaSuccess && l < layer_count; ++l) {
        st = cudaMalloc(&p->kpools[l], pool_bytes);
        if (st == cudaSuccess) st = cudaMalloc(&p->vpools[l], pool_bytes);
        if (st == cudaSuccess) st = cudaMemset(p->kpools[l], 0, pool_bytes);
        if (st == cudaSuccess) st = cudaMemset(p->vpools[l], 0, pool_bytes);
    }
    const size_t table_bytes = max_batch * max_pages_per_seq * sizeof(uint32_t);
    if (st == cudaSuccess) st = cudaMalloc((void **)&p->d_tables, table_bytes);
    if (st == cudaSuccess) st = cudaMemset(p->d_tables, 0, table_bytes);
    p->patch_offset = align_up((2u * max_batch + 1u) * sizeof(int32_t), 256);
    p->patch_capacity = max_batch * max_pages_per_seq;
    p->stage_bytes = p->patch_offset + p->patch_capacity * sizeof(PkvTablePatch);
    const unsigned map_flags = cudaHostAllocMapped | cudaHostAllocPortable;
    for (int s = 0; st == cudaSuccess && s < kStageSlots; ++s) {
        st = cudaHostAlloc((void **)&p->h_stage[s], p->stage_bytes, map_flags);
        if (st == cudaSuccess)
            st = cudaHostGetDevicePointer((void **)&p->h_stage_dev[s], p->h_stage[s], 0);
        /* lengths and offsets, then the staging kernel's arrival counter */
        if (st == cudaSuccess)
            st = cudaMalloc((void **)&p->d_stage[s], p->patch_offset + 256);
        if (st == cudaSuccess) st = cudaMemset(p->d_stage[s], 0, p->patch_offset + 256);
    }
    if (st == cudaSuccess)
        st = cudaHostAlloc((void **)&p->h_consumed, kStageSlots * sizeof(uint32_t), map_flags);
    if (st == cudaSuccess) {
        memset(p->h_consumed, 0, kStageSlots * sizeof(uint32_t));
        st = cudaHostGetDevicePointer((void **)&p->h_consumed_dev, p->h_consumed, 0);
    }
    p->next_ticket = 1;
    if (st == cudaSuccess) st = cudaDeviceSynchronize();
    if (have_prev) cudaSetDevice(prev);
    if (st != cudaSuccess) {
        pkv_internal_set_error(error, cap, "pkv_pool_create: %s (pool of %zu bytes per array)",
                               cudaGetErrorString(st), pool_bytes);
        pool_destroy(p);
        return 0;
    }
    if (!tensor_paged_kv_cache_set_backend_state(cache, TENSOR_PAGED_KV_BACKEND_CUDA, p,
                                                 pool_destroy, pool_release_sequence)) {
        pkv_internal_set_error(error, cap, "pkv_pool_create: cache refused the attachment");
        pool_destroy(p);
        return 0;
    }
    *pool = p;
    return 1;
}

PkvPool *pkv_pool_from_cache(TensorPagedKVCache *cache) {
    return (PkvPool *)tensor_paged_kv_cache_backend_state(cache, TENSOR_PAGED_KV_BACKEND_CUDA);
}

int pkv_pool_layer(PkvPool *pool, size_t layer, PkvPagedLayer *out) {
    if (pool == NULL || out == NULL || layer >= pool->layer_count) return 0;
    out->key_pool = pool->kpools[layer];
    out->value_pool = pool->vpools[layer];
    out->block_size = pool->block_size;
    out->block_count = pool->block_count;
    out->kv_heads = pool->kv_heads;
    out->head_dim = pool->head_dim;
    out->dtype = pool->dtype;
    return 1;
}

/* Waits until the kernel that applied the slot's last contents has read
 * them (it writes its ticket to h_consumed).  Bounded: gives up after about
 * a minute, or at once when the device reports a sticky error. */
static int wait_slot_free(PkvPool *p, int slot) {
    const uint32_t want = p->stage_ticket[slot];
    volatile const uint32_t *done = p->h_consumed + slot;
    if (want == 0 || *done == want) return 1;
    struct timespec t0, now, nap = {0, 20000};
    clock_gettime(CLOCK_MONOTONIC, &t0);
    for (unsigned spin = 0;; ++spin) {
        if (*done == want) return 1;
        if (spin < 4096) continue;
        if ((spin & 255u) == 0) {
            const cudaError_t e = cudaPeekAtLastError();
            if (e != cudaSuccess && e != cudaErrorNotReady) return 0;
            clock_gettime(CLOCK_MONOTONIC, &now);
            if (now.tv_sec - t0.tv_sec > 60) return 0;
        }
        nanosleep(&nap, NULL);
    }
}

/* Undo the first `n` sequences of a half-opened step. */
static void rollback(PkvPool *p, size_t n, int reserved) {
    for (size_t b = 0; b < n; ++b) {
        if (reserved)
            (void)tensor_paged_kv_sequence_set_length(p->cache, p->step_seq[b],
                                                      p->step_current[b]);
        tensor_paged_kv_sequence_end_decode(p->cache, p->step_seq[b]);
    }
}

static int step_begin_impl(PkvPool *pool, const TensorPagedKVSequence *sequences,
                           const size_t *past_lengths, const size_t *new_tokens, size_t batch,
                           PkvStream stream, char *error, size_t cap) {
    PkvPool *p = pool;
    if (p == NULL || sequences == NULL || new_tokens == NULL) {
        pkv_internal_set_error(error, cap, "pkv_step_begin: null argument");
        return 0;
    }
    if (p->open) {
        pkv_internal_set_error(error, cap, "pkv_step_begin: a step is already open");
        return 0;
    }
    if (batch == 0 || batch > p->max_batch) {
        pkv_internal_set_error(error, cap, "pkv_step_begin: batch must be 1..%zu", p->max_batch);
        return 0;
    }
    const size_t max_tokens = p->max_pages * p->block_size;
    /* 1. decode locks */
    for (size_t b = 0; b < batch; ++b) {
        p->step_seq[b] = sequences[b];
        if (!tensor_paged_kv_sequence_begin_decode(p->cache, sequences[b])) {
            rollback(p, b, 0);
            pkv_internal_set_error(error, cap,
                                   "pkv_step_begin: sequence %zu is unknown or already decoding", b);
            return 0;
        }
    }
    /* 2. length checks and reservations (SDK order: length, then reserve) */
    for (size_t b = 0; b < batch; ++b) {
        size_t current = 0;
        int bad = !tensor_paged_kv_sequence_length(p->cache, sequences[b], &current);
        const size_t past = past_lengths ? past_lengths[b] : current;
        p->step_current[b] = current;
        bad = bad || (current != 0 && current != past);
        bad = bad || past > max_tokens || new_tokens[b] > max_tokens - past;
        if (bad || !tensor_paged_kv_sequence_reserve(p->cache, sequences[b], past + new_tokens[b])) {
            /* [0, b) hold reservations to undo; every sequence holds a lock */
            rollback(p, b, 1);
            for (size_t k = b; k < batch; ++k)
                tensor_paged_kv_sequence_end_decode(p->cache, sequences[k]);
            pkv_internal_set_error(error, cap,
                                   bad ? "pkv_step_begin: sequence %zu length mismatch or exceeds "
                                         "the table stride"
                                       : "pkv_step_begin: out of pages reserving sequence %zu",
                                   b);
            return 0;
        }
        p->step_target[b] = past + new_tokens[b];
    }
    /* 3. stage lengths, row offsets and table patches */
    const int slot = p->slot;
    if (!wait_slot_free(p, slot)) {
        rollback(p, batch, 1);
        pkv_internal_set_error(error, cap,
                               "pkv_step_begin: staging slot still in use (device stalled or "
                               "failed: %s)",
                               cudaGetErrorString(cudaPeekAtLastError()));
        return 0;
    }
    int32_t *lens = (int32_t *)p->h_stage[slot];
    int32_t *offs = lens + p->max_batch;
    PkvTablePatch *patches = (PkvTablePatch *)(p->h_stage[slot] + p->patch_offset);
    size_t npatch = 0;
    int32_t running = 0;
    for (size_t b = 0; b < batch; ++b) {
        RowState *row = &p->rows[b];
        size_t count = 0, from = row->seq == sequences[b] ? row->pages : 0;
        uint32_t epoch = 0;
        int ok = pkv_internal_copy_table_tail(p->cache, sequences[b], from, p->tmp_pages,
                                              p->max_pages, &count, NULL, &epoch);
        if (ok && from != 0 && (epoch != row->epoch || count < from)) {
            /* pages left the table since the last upload: resend the row */
            from = 0;
            ok = pkv_internal_copy_table_tail(p->cache, sequences[b], 0, p->tmp_pages,
                                              p->max_pages, &count, NULL, &epoch);
        }
        if (!ok) {
            for (size_t k = 0; k <= b; ++k) p->rows[k].seq = 0;
            rollback(p, batch, 1);
            pkv_internal_set_error(error, cap, "pkv_step_begin: table of sequence %zu too long", b);
            return 0;
        }
        for (size_t i = from; i < count; ++i) {
            PkvTablePatch *q = &patches[npatch++];
            q->row = (uint32_t)b;
            q->index = (uint32_t)i;
            q->page = p->tmp_pages[i - from];
            q->pad = 0;
        }
        row->seq = sequences[b];
        row->pages = count;
        row->epoch = epoch;
        lens[b] = (int32_t)p->step_target[b];
        offs[b] = running;
        running += (int32_t)new_tokens[b];
    }
    offs[batch] = running;
    int prev = 0;
    const int have_prev = cudaGetDevice(&prev) == cudaSuccess;
    cudaSetDevice(p->device);
    /* one kernel reads the slot and applies it */
    const uint32_t ticket = p->next_ticket;
    p->next_ticket = p->next_ticket + 1u == 0u ? 1u : p->next_ticket + 1u;
    cudaError_t st = cudaSuccess;
    if (!pkv_internal_stage_apply((const int32_t *)p->h_stage_dev[slot],
                                  (int32_t *)p->d_stage[slot], batch, p->max_batch,
                                  (const PkvTablePatch *)(p->h_stage_dev[slot] + p->patch_offset),
                                  npatch, p->d_tables, p->max_pages, p->max_batch,
                                  (uint32_t *)(p->d_stage[slot] + p->patch_offset),
                                  p->h_consumed_dev + slot, ticket, stream))
        st = cudaErrorLaunchFailure;
    else
        p->stage_ticket[slot] = ticket;
    if (have_prev) cudaSetDevice(prev);
    if (st != cudaSuccess) {
        for (size_t b = 0; b < batch; ++b) p->rows[b].seq = 0;
        rollback(p, batch, 1);
        pkv_internal_set_error(error, cap, "pkv_step_begin: %s", cudaGetErrorString(st));
        return 0;
    }
    p->open = 1;
    p->step_batch = batch;
    return 1;
}

int pkv_step_begin(PkvPool *pool, const TensorPagedKVSequence *sequences,
                   const size_t *past_lengths, const size_t *new_tokens, size_t batch,
                   PkvStream stream, char *error, size_t cap) {
    PKV_RANGE_PUSH("pkv_step_begin");
    const int ok = step_begin_impl(pool, sequences, past_lengths, new_tokens, batch, stream,
                                   error, cap);
    PKV_RANGE_POP();
    return ok;
}

int pkv_step_batch(PkvPool *pool, PkvBatch *out) {
    if (pool == NULL || out == NULL || !pool->open) return 0;
    out->block_tables = pool->d_tables;
    out->table_stride = pool->max_pages;
    out->seq_lens = (const int32_t *)pool->d_stage[pool->slot];
    out->batch = pool->step_batch;
    return 1;
}

const int32_t *pkv_step_row_offsets(PkvPool *pool) {
    if (pool == NULL || !pool->open) return NULL;
    return (const int32_t *)pool->d_stage[pool->slot] + pool->max_batch;
}

static int step_end_impl(PkvPool *pool, int commit, char *error, size_t cap) {
    PkvPool *p = pool;
    if (p == NULL || !p->open) {
        pkv_internal_set_error(error, cap, "pkv_step_end: no open step");
        return 0;
    }
    int ok = 1;
    for (size_t b = 0; b < p->step_batch; ++b) {
        const TensorPagedKVSequence s = p->step_seq[b];
        if (commit && tensor_paged_kv_sequence_set_length(p->cache, s, p->step_target[b]))
            ;
        else {
            if (commit) ok = 0;
            (void)tensor_paged_kv_sequence_set_length(p->cache, s, p->step_current[b]);
        }
        tensor_paged_kv_sequence_end_decode(p->cache, s);
    }
    p->open = 0;
    p->slot = (p->slot + 1) % kStageSlots;
    if (!ok) pkv_internal_set_error(error, cap, "pkv_step_end: commit failed; rolled back");
    return commit ? ok : 1;
}

int pkv_step_end(PkvPool *pool, int commit, char *error, size_t cap) {
    PKV_RANGE_PUSH("pkv_step_end");
    const int ok = step_end_impl(pool, commit, error, cap);
    PKV_RANGE_POP();
    return ok;
}

int pkv_device_fault(int device, uint32_t *code, char *error, size_t cap) {
    if (code == NULL) {
        pkv_internal_set_error(error, cap, "pkv_device_fault: null argument");
        return 0;
    }
    int prev = 0;
    const int have_prev = cudaGetDevice(&prev) == cudaSuccess;
    cudaError_t st = cudaSetDevice(device);
    if (st == cudaSuccess) st = cudaDeviceSynchronize();
    uint32_t a = 0, b = 0, c = 0, d = 0, e = 0;
    int ok = st == cudaSuccess && pkv_internal_take_copy_fault(&a) &&
             pkv_internal_take_decode_fault(&b) && pkv_internal_take_prefill_fault(&c) &&
             pkv_internal_take_sequence_fault(&d) && pkv_internal_take_peer_fault(&e);
    if (have_prev) cudaSetDevice(prev);
    if (!ok) {
        pkv_internal_set_error(error, cap, "pkv_device_fault: %s",
                               cudaGetErrorString(st != cudaSuccess ? st : cudaGetLastError()));
        return 0;
    }
    *code = a ? a : (b ? b : (c ? c : (d ? d : e)));
    return 1;
}
