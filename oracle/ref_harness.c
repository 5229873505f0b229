/*
 * ref_harness.c -- drives the inference SDK's own CPU code as the oracle.
 *
 * TEST INFRASTRUCTURE ONLY (tests/, smoke(), bench.py's reference arm and
 * cpu_baseline).  oracle/Makefile compiles this file together with the SDK's
 * unmodified CPU sources (attention.c, paged_kv_cache.c, tensor_f16.c,
 * tensor_buffer.c, tensor_workspace.c and the backend stubs) into
 * oracle/_ref/libref_oracle.so.  Nothing of the SDK is copied here.
 *
 * The SDK has no CPU paged attention (its CPU build's CUDA/Metal getters
 * return NULL, attention_cuda_stub.c:1-5), so the reference for one paged
 * sequence is: gather K/V through the block table (page addressing of
 * attention_cuda.cu:301-305, restated in pkv_oracle.c), widen to FP32 with
 * the SDK's tensor_f16_to_f32 / tensor_bf16_to_f32 (tensor_f16.c:17-46),
 * then the SDK's tensor_sdpa_f32 (attention.c:212-406) on [1, Hkv, L, d].
 *
 * Work is split into a prepare phase (gather + widen, untimed) and a run
 * phase (only tensor_sdpa_f32 calls, timed), mirroring the prepare/run split
 * of the SDK's benchmark API (include/benchmark.h).  The run phase spreads
 * sequences over pthreads, each with its own TensorWorkspace.
 */
#define _POSIX_C_SOURCE 200112L
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "attention.h"
#include "tensor_buffer.h"
#include "tensor_f16.h"
#include "tensor_workspace.h"

int64_t orc_pool_row(const uint32_t *table_row, size_t table_len, size_t block_size,
                     size_t block_count, int64_t pos);

enum { REF_F16 = 1, REF_BF16 = 2 };

static float widen(uint16_t x, int dtype) {
    return dtype == REF_BF16 ? tensor_bf16_to_f32(x) : tensor_f16_to_f32(x);
}

static TensorBuffer *make_f32(const uint64_t shape[4]) {
    TensorBuffer *t = NULL;
    char err[128];
    if (!tensor_buffer_create(TENSOR_DTYPE_F32, shape, 4, &t, err, sizeof(err))) return NULL;
    return t;
}

/* Plain-pointer wrapper over tensor_sdpa_f32 for [B][H][L][d] arrays. */
int ref_sdpa_f32(const float *q, const float *k, const float *v, const float *mask,
                 float *out, size_t batch, size_t q_heads, size_t kv_heads, size_t q_len,
                 size_t kv_len, size_t head_dim, size_t value_dim, float scale, int causal,
                 char *error, size_t error_capacity) {
    const uint64_t qs[4] = {batch, q_heads, q_len, head_dim};
    const uint64_t ks[4] = {batch, kv_heads, kv_len, head_dim};
    const uint64_t vs[4] = {batch, kv_heads, kv_len, value_dim};
    const uint64_t os[4] = {batch, q_heads, q_len, value_dim};
    const uint64_t ms[2] = {q_len, kv_len};
    TensorBuffer *tq = make_f32(qs), *tk = make_f32(ks), *tv = make_f32(vs), *to = make_f32(os);
    TensorBuffer *tm = NULL;
    TensorWorkspace *ws = NULL;
    int ok = tq && tk && tv && to &&
             tensor_workspace_create(1u << 16, &ws, error, error_capacity);
    if (ok && mask) {
        char err[128];
        ok = tensor_buffer_create(TENSOR_DTYPE_F32, ms, 2, &tm, err, sizeof(err));
        if (ok) memcpy(tensor_buffer_data_mut(tm), mask, q_len * kv_len * sizeof(float));
    }
    if (ok) {
        memcpy(tensor_buffer_data_mut(tq), q, batch * q_heads * q_len * head_dim * 4);
        memcpy(tensor_buffer_data_mut(tk), k, batch * kv_heads * kv_len * head_dim * 4);
        memcpy(tensor_buffer_data_mut(tv), v, batch * kv_heads * kv_len * value_dim * 4);
        TensorAttentionBackend used;
        ok = tensor_sdpa_f32(tq, tk, tv, tm, scale, causal, to, ws, &used, error,
                             error_capacity);
        if (ok) memcpy(out, tensor_buffer_data(to), batch * q_heads * q_len * value_dim * 4);
    }
    tensor_buffer_free(tq); tensor_buffer_free(tk); tensor_buffer_free(tv);
    tensor_buffer_free(to); tensor_buffer_free(tm);
    tensor_workspace_free(ws);
    return ok;
}

typedef struct {
    TensorBuffer *q, *k, *v, *o;
    size_t n_rows;
} RefItem;

typedef struct {
    RefItem *items;
    size_t n_items;
    size_t q_heads, head_dim;
    float scale;
    int causal;
    size_t max_scores;
    /* run phase */
    size_t next;
    pthread_mutex_t lock;
    int failed;
} RefJob;

/* Prepares one tensor_sdpa_f32 call per selected sequence.
 *   q           [rows][q_heads][head_dim] storage of `dtype`
 *   q_offsets   [batch+1] rows per sequence, or NULL for one row each
 *   tail_rows   0: use all of a sequence's rows; n: only its last n rows
 *   kv_head0/n  which KV heads (and their query heads) to include
 *   subset      sequence indices to include (NULL: all)
 * A sequence's query rows are its last positions, so the SDK's causal
 * offset kv_len - q_len places them correctly. */
RefJob *ref_job_prepare(int dtype, const uint16_t *q, const int32_t *q_offsets,
                        const uint16_t *kpool, const uint16_t *vpool, size_t kv_heads,
                        size_t head_dim, size_t block_size, size_t block_count,
                        const uint32_t *tables, size_t table_stride, const int32_t *seq_lens,
                        size_t batch, size_t q_heads, const int32_t *subset, size_t n_subset,
                        size_t kv_head0, size_t kv_head_n, size_t tail_rows, float scale,
                        int causal) {
    if (kv_heads == 0 || q_heads % kv_heads || kv_head0 + kv_head_n > kv_heads || kv_head_n == 0)
        return NULL;
    RefJob *job = (RefJob *)calloc(1, sizeof(RefJob));
    if (!job) return NULL;
    const size_t n = subset ? n_subset : batch;
    job->items = (RefItem *)calloc(n ? n : 1, sizeof(RefItem));
    job->n_items = n;
    const size_t group = q_heads / kv_heads, kv_width = kv_heads * head_dim;
    job->q_heads = kv_head_n * group;
    job->head_dim = head_dim;
    job->scale = scale;
    job->causal = causal;
    pthread_mutex_init(&job->lock, NULL);
    int ok = job->items != NULL;
    for (size_t i = 0; ok && i < n; ++i) {
        const size_t b = subset ? (size_t)subset[i] : i;
        const size_t L = (size_t)seq_lens[b];
        const size_t first = q_offsets ? (size_t)q_offsets[b] : b;
        size_t rows = q_offsets ? (size_t)(q_offsets[b + 1] - q_offsets[b]) : 1;
        size_t skip = 0;
        if (tail_rows && tail_rows < rows) { skip = rows - tail_rows; rows = tail_rows; }
        if (L == 0 || rows == 0) { ok = 0; break; }
        const uint64_t qs[4] = {1, job->q_heads, rows, head_dim};
        const uint64_t ks[4] = {1, kv_head_n, L, head_dim};
        RefItem *it = &job->items[i];
        it->n_rows = rows;
        it->q = make_f32(qs); it->o = make_f32(qs);
        it->k = make_f32(ks); it->v = make_f32(ks);
        if (!it->q || !it->o || !it->k || !it->v) { ok = 0; break; }
        float *kq = (float *)tensor_buffer_data_mut(it->q);
        float *kk = (float *)tensor_buffer_data_mut(it->k);
        float *kv = (float *)tensor_buffer_data_mut(it->v);
        for (size_t j = 0; ok && j < L; ++j) {
            const int64_t row = orc_pool_row(tables + b * table_stride, table_stride, block_size,
                                             block_count, (int64_t)j);
            if (row < 0) { ok = 0; break; }
            for (size_t g = 0; g < kv_head_n; ++g)
                for (size_t d = 0; d < head_dim; ++d) {
                    const size_t src = (size_t)row * kv_width + (kv_head0 + g) * head_dim + d;
                    kk[(g * L + j) * head_dim + d] = widen(kpool[src], dtype);
                    kv[(g * L + j) * head_dim + d] = widen(vpool[src], dtype);
                }
        }
        for (size_t r = 0; r < rows; ++r)
            for (size_t h = 0; h < job->q_heads; ++h)
                for (size_t d = 0; d < head_dim; ++d)
                    kq[(h * rows + r) * head_dim + d] =
                        widen(q[((first + skip + r) * q_heads + kv_head0 * group + h) * head_dim + d],
                              dtype);
        if (rows * L > job->max_scores) job->max_scores = rows * L;
    }
    if (!ok) {
        for (size_t i = 0; i < n; ++i) {
            tensor_buffer_free(job->items[i].q); tensor_buffer_free(job->items[i].k);
            tensor_buffer_free(job->items[i].v); tensor_buffer_free(job->items[i].o);
        }
        free(job->items);
        pthread_mutex_destroy(&job->lock);
        free(job);
        return NULL;
    }
    return job;
}

typedef struct {
    RefJob *job;
    TensorWorkspace *ws;
} Worker;

static void *worker_main(void *arg) {
    Worker *w = (Worker *)arg;
    RefJob *job = w->job;
    char err[256];
    for (;;) {
        pthread_mutex_lock(&job->lock);
        const size_t i = job->next++;
        pthread_mutex_unlock(&job->lock);
        if (i >= job->n_items) break;
        RefItem *it = &job->items[i];
        TensorAttentionBackend used;
        if (!tensor_sdpa_f32(it->q, it->k, it->v, NULL, job->scale, job->causal, it->o, w->ws,
                             &used, err, sizeof(err))) {
            pthread_mutex_lock(&job->lock);
            job->failed = 1;
            pthread_mutex_unlock(&job->lock);
        }
    }
    return NULL;
}

/* Runs every prepared tensor_sdpa_f32 call on `threads` threads; *seconds
 * is the wall time of that phase alone. */
int ref_job_run(RefJob *job, int threads, double *seconds) {
    if (job == NULL || threads < 1) return 0;
    Worker *ws = (Worker *)calloc((size_t)threads, sizeof(Worker));
    pthread_t *tids = (pthread_t *)calloc((size_t)threads, sizeof(pthread_t));
    int ok = ws && tids;
    char err[128];
    for (int t = 0; ok && t < threads; ++t) {
        ws[t].job = job;
        ok = tensor_workspace_create(job->max_scores * sizeof(float) + 4096, &ws[t].ws, err,
                                     sizeof(err));
        if (ok) {  /* grow the arena once so the timed phase does not allocate */
            TensorWorkspaceMark m = tensor_workspace_mark(ws[t].ws);
            ok = tensor_workspace_allocate(ws[t].ws, job->max_scores * sizeof(float), 4, err,
                                           sizeof(err)) != NULL &&
                 tensor_workspace_release(ws[t].ws, m, err, sizeof(err));
        }
    }
    job->next = 0;
    job->failed = 0;
    struct timespec t0, t1;
    clock_gettime(CLOCK_MONOTONIC, &t0);
    int started = 0;
    for (int t = 0; ok && t < threads; ++t, ++started)
        if (pthread_create(&tids[t], NULL, worker_main, &ws[t]) != 0) { ok = 0; break; }
    for (int t = 0; t < started; ++t) pthread_join(tids[t], NULL);
    clock_gettime(CLOCK_MONOTONIC, &t1);
    if (seconds) *seconds = (double)(t1.tv_sec - t0.tv_sec) + 1e-9 * (double)(t1.tv_nsec - t0.tv_nsec);
    for (int t = 0; ws && t < threads; ++t) tensor_workspace_free(ws[t].ws);
    free(ws);
    free(tids);
    return ok && !job->failed;
}

/* Output of prepared item `index` as [rows][q_heads_of_job][head_dim]. */
int ref_job_output(const RefJob *job, size_t index, float *out) {
    if (job == NULL || index >= job->n_items) return 0;
    const RefItem *it = &job->items[index];
    const float *o = (const float *)tensor_buffer_data(it->o);
    for (size_t r = 0; r < it->n_rows; ++r)
        for (size_t h = 0; h < job->q_heads; ++h)
            memcpy(out + (r * job->q_heads + h) * job->head_dim,
                   o + (h * it->n_rows + r) * job->head_dim, job->head_dim * sizeof(float));
    return 1;
}

void ref_job_free(RefJob *job) {
    if (job == NULL) return;
    for (size_t i = 0; i < job->n_items; ++i) {
        tensor_buffer_free(job->items[i].q); tensor_buffer_free(job->items[i].k);
        tensor_buffer_free(job->items[i].v); tensor_buffer_free(job->items[i].o);
    }
    free(job->items);
    pthread_mutex_destroy(&job->lock);
    free(job);
}
