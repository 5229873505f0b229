/*
 * pkv_b200.h -- B200 (sm_100a) paged-KV attention: the C ABI.
 *
 * Two layers, both plain C (no C++ or torch types cross this boundary):
 *
 *  1. Kernel entry points.  Device pointers in, device pointers out, one CUDA
 *     stream per call.  Each replaces one piece of the inference SDK's CUDA
 *     backend (src/platform/cuda/attention_cuda.cu) and batches it over many
 *     sequences per launch instead of one sequence per call.
 *
 *  2. Host transaction layer (C11).  A device page pool attached to a
 *     TensorPagedKVCache through tensor_paged_kv_cache_set_backend_state
 *     (the SDK's own attach point), plus a batch version of the transaction
 *     in tensor_attention_decode_sequence_paged (src/common/attention.c:124-176):
 *     begin_decode -> length check -> reserve -> kernels -> set_length or
 *     rollback -> end_decode, for every sequence of a batch at once.
 *
 * Conventions (same as the SDK): every int-returning call gives 1 on success
 * and 0 on failure; calls that take (error, error_capacity) write a
 * NUL-terminated reason there on failure (either may be NULL/0).
 *
 * Pool layout (SDK attention_cuda.cu:301-305 and :547-612): one K pool and
 * one V pool per layer, each [block_count * block_size][kv_heads * head_dim]
 * elements of 2 bytes.  Token `pos` of a sequence lives in row
 *     table[pos / block_size] * block_size + pos % block_size
 * and KV head h occupies columns [h * head_dim, (h + 1) * head_dim).
 *
 * Block tables are dense and padded: row b (the b-th sequence of a batch)
 * starts at block_tables + b * table_stride and lists that sequence's page ids
 * in logical order.  seq_lens[b] is the sequence length AFTER this step's
 * append: append writes the last n_b positions, attention reads all of them.
 */
#ifndef PKV_B200_H
#define PKV_B200_H

#include <stddef.h>
#include <stdint.h>

#include "paged_kv_cache.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t; NULL selects the legacy default stream. */
typedef struct CUstream_st *PkvStream;

typedef enum {
    PKV_DTYPE_F16 = 1,
    PKV_DTYPE_BF16 = 2,
    PKV_DTYPE_F32 = 3 /* outputs only */
} PkvDType;

/* One layer of a device page pool. */
typedef struct {
    void *key_pool;
    void *value_pool;
    size_t block_size;  /* tokens per page */
    size_t block_count; /* pages in the pool (device bounds checks use it) */
    size_t kv_heads;
    size_t head_dim;    /* kernels: 64 or 128 */
    PkvDType dtype;     /* storage: F16 or BF16 (F32 pools serve only the decoder entry point) */
} PkvPagedLayer;

/* The sequences of one batch, as the kernels see them (device pointers). */
typedef struct {
    const uint32_t *block_tables; /* [batch][table_stride] page ids */
    size_t table_stride;          /* >= pages of the longest sequence */
    const int32_t *seq_lens;      /* [batch] lengths after this step's append */
    size_t batch;
} PkvBatch;

/* ---------------------------------------------------------------------- */
/* 1. Kernel entry points                                                  */
/* ---------------------------------------------------------------------- */

/* KV append: scatters new K/V rows into their pages with 16-byte stores.
 * Rows row_offsets[b] .. row_offsets[b+1]-1 of key_rows/value_rows
 * ([total_rows][kv_heads*head_dim], pool dtype) become positions
 * seq_lens[b]-n_b .. seq_lens[b]-1 of sequence b.  row_offsets == NULL means
 * one row per sequence (row b belongs to sequence b, total_rows == batch).
 * Replaces the K/V stores of decode_rope_cache_kernel
 * (attention_cuda.cu:307-341, launched :996-1000), without RoPE. */
int pkv_kv_append(const PkvPagedLayer *layer, const PkvBatch *batch,
                  const int32_t *row_offsets, const void *key_rows,
                  const void *value_rows, size_t total_rows, PkvStream stream,
                  char *error, size_t error_capacity);

/* Prefix import: copies each sequence's contiguous K/V prefix
 * ([sum seq_lens][kv_width], sequences back to back in batch order) into its
 * pages, all sequences in one launch.  Replaces the per-page-run cudaMemcpy
 * loop of attention_cuda.cu:894-915. */
int pkv_kv_import(const PkvPagedLayer *layer, const PkvBatch *batch,
                  const int32_t *row_offsets, const void *key_rows,
                  const void *value_rows, size_t total_rows, PkvStream stream,
                  char *error, size_t error_capacity);

/* Gather: the inverse of import.  Writes sequence b's first seq_lens[b]
 * tokens to rows row_offsets[b] .. of key_out/value_out.  The SDK never reads
 * pages back (attention_cuda.cu:1084-1086); this exists for checkpointing and
 * for the bit-exact page tests. */
int pkv_kv_gather(const PkvPagedLayer *layer, const PkvBatch *batch,
                  const int32_t *row_offsets, void *key_out, void *value_out,
                  size_t total_rows, PkvStream stream, char *error,
                  size_t error_capacity);

/* Scratch needed by pkv_paged_decode for this shape (bytes). */
size_t pkv_decode_workspace_bytes(size_t batch, size_t q_heads,
                                  size_t head_dim, size_t max_seq_len,
                                  size_t chunk_tokens);
/* Decode scratch must start zeroed once; pkv_paged_decode leaves it zeroed. */
int pkv_decode_workspace_init(void *workspace, size_t workspace_bytes,
                              PkvStream stream, char *error,
                              size_t error_capacity);

/* Paged decode SDPA, one query token per sequence, GQA.
 * query/output: [batch][q_heads][head_dim]; output dtype F16, BF16 or F32.
 * head_dim 128 with pages of 16-128 tokens runs on the tensor cores: one
 * persistent CTA per SM, TMA page loads straight through the block table,
 * S = K.Q^T and O = V^T.P^T on tcgen05 with FP32 accumulators in TMEM, so
 * each page byte is read once for all q_heads/kv_heads query heads of its KV
 * head.  The 128-token tiles of all (sequence, KV head) segments form one
 * stream (stream-K): most of it is cut evenly across the CTAs, and on long
 * launches the last part is cut into smaller work units that CTAs claim as
 * they finish, so SMs that stream faster take more.  A segment split between
 * units is merged from FP32 partials (m, l, O) by the last CTA to finish a
 * piece of it, or, when few segments are cut into many pieces, by a
 * separate merge kernel.
 * head_dim 64 with an even KV-head count runs there too, KV heads 2g and
 * 2g+1 as one 128-column segment.  Other shapes (head_dim 64 with an odd
 * KV-head count, other page sizes) run a CUDA-core kernel: one CTA per
 * (sequence, KV head, chunk of chunk_tokens positions), a cp.async ring and
 * a warp-shuffle online softmax, chunks merged by the last CTA.
 * max_seq_len bounds seq_lens (it sizes the scratch); chunk_tokens 0 picks a
 * split from batch and max_seq_len (the tensor-core kernel ignores it).
 * seq_lens[b] == 0 yields zeros, like the SDK's all-masked softmax.
 * The tensor-core kernel releases programmatic dependents early: a kernel
 * the caller launches after it on the same stream WITH programmatic stream
 * serialization starts while it runs and must execute griddepcontrol.wait
 * (cudaGridDependencySynchronize) before it reads the output or writes the
 * pages or tables.  Ordinary launches, copies and events wait for it as usual.
 * Replaces decode_score_kernel, decode_softmax_kernel and
 * decode_attention_output_kernel (attention_cuda.cu:343-398, launched
 * :1001-1011). */
int pkv_paged_decode(const PkvPagedLayer *layer, const PkvBatch *batch,
                     size_t q_heads, const void *query, float scale,
                     void *output, PkvDType output_dtype, size_t max_seq_len,
                     size_t chunk_tokens, void *workspace,
                     size_t workspace_bytes, PkvStream stream, char *error,
                     size_t error_capacity);

/* A decode step's append and paged decode in one call: the same result as
 * pkv_kv_append(layer, batch, NULL, key_rows, value_rows, batch->batch, ...)
 * followed by pkv_paged_decode(...) on the same stream -- each sequence's new
 * K/V row ([batch][kv_heads * head_dim], 16-byte aligned) is stored at
 * position seq_lens[b] - 1, bit for bit as the append kernel stores it, and
 * the decode attends over it.  On the tensor-core path this is one launch:
 * the producer warp that loads the 128-token tile holding the new row first
 * stores the row into its page (and fences it against the TMA that reads the
 * page), so no separate append kernel sits between the step's staging and
 * its decode.  Other shapes run the two kernels.  A sequence with
 * seq_lens[b] == 0 has no room for its row: nothing is stored, its output is
 * zeros and fault code 3 is recorded, as pkv_kv_append does.  Replaces the
 * SDK backend's per-layer decode call: decode_rope_cache_kernel's K/V store
 * (attention_cuda.cu:307-341; RoPE stays the caller's) and the three decode
 * kernels (:343-398), launched at :996-1011. */
int pkv_paged_decode_append(const PkvPagedLayer *layer, const PkvBatch *batch,
                            const void *key_rows, const void *value_rows,
                            size_t q_heads, const void *query, float scale,
                            void *output, PkvDType output_dtype,
                            size_t max_seq_len, size_t chunk_tokens,
                            void *workspace, size_t workspace_bytes,
                            PkvStream stream, char *error,
                            size_t error_capacity);

/* Paged decode that allocates nothing:pkv_paged_decode with its scratch in
 * a static 8 MiB device array inside this library instead of a workspace.
 * No counterpart in the SDK.  For callers that cannot allocate device memory
 * at call time (a serving loop whose device memory is planned once up front,
 * where cudaMalloc could synchronise the device or fragment the pool; a host
 * behind an FFI that only passes the buffers it was given).  Shapes whose
 * scratch would exceed 8 MiB fail with an error naming the size.  Every GPU
 * that loads the library holds the 8 MiB until exit.  The first call on a
 * device looks up the array's device address (once per device, and again
 * if the device's context changed, e.g. after cudaDeviceReset), so make it
 * before any stream capture.  Arguments are checked before the array is
 * touched: a refused call writes no device memory.  Each call clears the
 * split-K tickets at the start of the array (one small memset on `stream`).
 * All calls share the array: calls that overlap on the GPU (other streams,
 * other threads) race; serialise them. */
int pkv_paged_decode_static_scratch(const PkvPagedLayer *layer, const PkvBatch *batch,
                                    size_t q_heads, const void *query, float scale,
                                    void *output, PkvDType output_dtype,
                                    size_t max_seq_len, PkvStream stream, char *error,
                                    size_t error_capacity);

/* Chunked prefill over the paged cache (tcgen05 tensor cores, FP32
 * accumulation in TMEM; head_dim 64 or 128, pages of 16-128 tokens).
 * Sequence b contributes query rows query_offsets[b] ..
 * query_offsets[b+1]-1 ([total_q][q_heads][head_dim]);
 * they are its LAST n_b positions, so query j sees keys
 * 0 .. seq_lens[b]-n_b+j when causal (the SDK's causal offset
 * kv_len - q_len, attention.c:251,352) and all seq_lens[b] keys otherwise.
 * max_query_len bounds n_b.  Replaces the dense sdpa<T> path
 * (attention_cuda.cu:25-99 via tensor_sdpa_f16, attention.c:408-459). */
int pkv_paged_prefill(const PkvPagedLayer *layer, const PkvBatch *batch,
                      size_t q_heads, const int32_t *query_offsets,
                      const void *query, size_t total_query_rows,
                      size_t max_query_len, float scale, int causal,
                      void *output, PkvDType output_dtype, PkvStream stream,
                      char *error, size_t error_capacity);

/* Reads and clears the device fault word of `device` (synchronises it).
 * Kernels never trap: an out-of-range page id or position skips the access
 * and records a code here.  *code == 0 means no fault was recorded. */
int pkv_device_fault(int device, uint32_t *code, char *error,
                     size_t error_capacity);

/* Self-test of the failure path the kernels rely on (synchronises the
 * current device, takes about half a second): a one-CTA kernel holding TMEM
 * waits on an mbarrier nothing arrives on; the bounded wait gives up, the CTA
 * frees TMEM and exits.  *code receives the recorded fault code -- 4
 * (wait timeout) when the bounded wait works.  The device stays usable. */
int pkv_selftest_wait_timeout(uint32_t *code, char *error, size_t error_capacity);

/* Dense FP16 SDPA on the tcgen05 prefill kernel: query [batch][q_heads]
 * [q_len][head_dim], key/value [batch][kv_heads][kv_len][head_dim], output
 * like query, optional additive mask [q_len][kv_len] (NULL: none; shared by
 * every batch and head), all device pointers (tensors 16-byte aligned, the
 * mask 2-byte).  head_dim 64 or 128 (value_dim = head_dim).  GQA (q_heads a
 * multiple of kv_heads), score = q.k * scale + mask, causal rule
 * key > query + max(kv_len - q_len, 0), FP32 accumulation, FP16 output;
 * a row whose maximum score is not finite (all keys -inf, or a +inf) is
 * zero.  Replaces the CUDA backend's dense sdpa<T> (attention_cuda.cu:25-99)
 * behind tensor_sdpa_f16 (attention.c:408-459).  Each (batch, KV head) is
 * one sequence of the paged prefill kernel with an identity page table. */
size_t pkv_sdpa_workspace_bytes(size_t batch, size_t q_heads, size_t kv_heads,
                                size_t q_len, size_t kv_len, size_t head_dim);
int pkv_sdpa_f16(const void *query, const void *key, const void *value,
                 const void *additive_mask, void *output, size_t batch,
                 size_t q_heads, size_t kv_heads, size_t q_len, size_t kv_len,
                 size_t head_dim, float scale, int causal, void *workspace,
                 size_t workspace_bytes, PkvStream stream, char *error,
                 size_t error_capacity);
/* The same with host tensors, in the argument order of the SDK backend hook
 * run_f16 (src/attention_backend.h:14-18), so it can be installed as that
 * hook: uploads, computes on the current device, downloads, synchronous.
 * Takes head_dim = value_dim = 64 or 128; returns 0 for other shapes (the
 * SDK's sdpa<T> also allows value_dim != head_dim and any head_dim; those
 * calls are refused here, not computed another way).  Returns 0 as well
 * when the kernel recorded a fault (its prefill fault word is read and
 * cleared after the call).  Its first call allocates,
 * and keeps until exit, a device buffer sized for the largest call so far
 * and 32 MiB of pinned host memory (two staging buffers that up to 8 host
 * threads fill while the DMA engine moves the other); calls are serialised
 * internally. */
int pkv_sdpa_f16_host(const uint16_t *query, const uint16_t *key,
                      const uint16_t *value, const uint16_t *additive_mask,
                      uint16_t *output, size_t batch, size_t query_heads,
                      size_t kv_heads, size_t query_length, size_t kv_length,
                      size_t head_dim, size_t value_dim, float scale, int causal);

/* ---------------------------------------------------------------------- */
/* Multi-GPU: NCCL all-gather with a host deadline                         */
/* ---------------------------------------------------------------------- */

/* The SDK has no multi-GPU code (its failure handling is the transaction's
 * return code and rollback, attention.c:159-166).  For the KV-head split of
 * one long sequence across GPUs, each GPU decodes its heads and the outputs
 * are all-gathered with NCCL.  These calls run NCCL in non-blocking mode and
 * poll it against a deadline, so a peer that never joins or stalls makes
 * the call return 0 (after ncclCommAbort) instead of hanging; the caller
 * then ends its step without commit (pkv_step_end(..., 0, ...)), which rolls
 * the step back.  NCCL is loaded at run time (PKV_NCCL_LIBRARY, default
 * libnccl.so.2). */
typedef struct PkvComm PkvComm;
#define PKV_COMM_ID_BYTES 256
/* A new communicator id (rank 0 makes it and sends it to the others; it
 * holds two NCCL ids: the joining and the collectives' communicator). */
int pkv_comm_unique_id(unsigned char *id, size_t id_bytes, char *error, size_t error_capacity);
/* Joins the communicator of `id` as `rank` of `nranks` on `device`; waits at
 * most timeout_s seconds for every rank to join. */
int pkv_comm_init(const unsigned char *id, size_t id_bytes, int nranks, int rank, int device,
                  double timeout_s, PkvComm **comm, char *error, size_t error_capacity);
/* Enqueues on `stream` the all-gather of bytes_per_rank bytes from every
 * rank into recv (rank order); waits at most timeout_s for the enqueue. */
int pkv_comm_all_gather(PkvComm *comm, const void *send, void *recv, size_t bytes_per_rank,
                        PkvStream stream, double timeout_s, char *error,
                        size_t error_capacity);
/* Waits at most timeout_s for `stream`'s work (the collectives enqueued on
 * it) to finish, watching NCCL's asynchronous error state; 0 (and the
 * communicator aborted) on error or timeout. */
int pkv_comm_wait(PkvComm *comm, PkvStream stream, double timeout_s, char *error,
                  size_t error_capacity);
/* 1 when the communicator was aborted (or is NULL): it takes no more work. */
int pkv_comm_aborted(const PkvComm *comm);
void pkv_comm_destroy(PkvComm *comm);

/* All-gather by peer stores over NVLink (an A/B alternative to the NCCL
 * all-gather above for small per-rank outputs; no counterpart in the SDK).
 * Each rank allocates a device area, exports it with CUDA IPC (the handle,
 * PKV_PEER_HANDLE_BYTES), and maps every other rank's.  One single-CTA
 * kernel per call stores this rank's bytes into every rank's area and waits
 * (bounded by timeout_s, on the GPU) until every rank's bytes of this step
 * arrived, then copies the nranks slots (rank order) to recv.  A wait that
 * gives up records fault code 4 (pkv_device_fault) and leaves recv as it
 * was.  All ranks must call it the same number of times, on GPUs of one
 * node with peer access.  Up to 8 ranks and 1 MiB per rank. */
typedef struct PkvPeerGather PkvPeerGather;
#define PKV_PEER_HANDLE_BYTES 64
int pkv_peer_gather_create(int device, int nranks, int rank, size_t bytes_per_rank,
                           PkvPeerGather **gather, void *handle, size_t handle_bytes,
                           char *error, size_t error_capacity);
/* handles: every rank's handle, rank order (nranks * PKV_PEER_HANDLE_BYTES). */
int pkv_peer_gather_connect(PkvPeerGather *gather, const void *handles, size_t handles_bytes,
                            char *error, size_t error_capacity);
int pkv_peer_all_gather(PkvPeerGather *gather, const void *send, void *recv, double timeout_s,
                        PkvStream stream, char *error, size_t error_capacity);
void pkv_peer_gather_destroy(PkvPeerGather *gather);

/* ---------------------------------------------------------------------- */
/* 2. Host transaction layer                                               */
/* ---------------------------------------------------------------------- */

typedef struct PkvPool PkvPool;

/* Allocates layer_count K and V pools on `device` for every page of `cache`,
 * a padded device block table for up to max_batch sequences of up to
 * max_pages_per_seq pages, and attaches the pool to the cache as its CUDA
 * backend state (tensor_paged_kv_cache_free destroys it).  Pools start
 * zeroed.  dtype F16 or BF16 (F32 for the decoder entry point of
 * attention.h).  Replaces get_cuda_paged_kv_state (attention_cuda.cu:570-612). */
int pkv_pool_create(TensorPagedKVCache *cache, int device, PkvDType dtype,
                    size_t layer_count, size_t kv_heads, size_t head_dim,
                    size_t max_batch, size_t max_pages_per_seq,
                    PkvPool **pool, char *error, size_t error_capacity);
/* The pool attached to `cache`, or NULL. */
PkvPool *pkv_pool_from_cache(TensorPagedKVCache *cache);
/* Device view of one layer. */
int pkv_pool_layer(PkvPool *pool, size_t layer, PkvPagedLayer *out);

/* Opens a batch step: for each sequence (in order; row b of the batch) takes
 * the decode lock, checks its length is 0 or past_lengths[b] (NULL: accept
 * the current length), reserves past + new_tokens[b] tokens, and stages the
 * new page-table entries and lengths for the device on `stream`.  All or
 * nothing: any failure rolls every sequence back and releases its lock. */
int pkv_step_begin(PkvPool *pool, const TensorPagedKVSequence *sequences,
                   const size_t *past_lengths, const size_t *new_tokens,
                   size_t batch, PkvStream stream, char *error,
                   size_t error_capacity);
/* Device view of the open step (block tables, post-append lengths). */
int pkv_step_batch(PkvPool *pool, PkvBatch *out);
/* Device row offsets of the open step's new tokens ([batch+1], int32). */
const int32_t *pkv_step_row_offsets(PkvPool *pool);
/* Closes the step: commit sets every length to past + new; otherwise the
 * reservations are rolled back.  Always releases the decode locks. */
int pkv_step_end(PkvPool *pool, int commit, char *error,
                 size_t error_capacity);

#ifdef __cplusplus
}
#endif

#endif
