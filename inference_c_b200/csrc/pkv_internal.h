/*
 * pkv_internal.h -- declarations shared between the C11 host layer
 * (pkv_pool.c, paged_kv_cache.c) and the CUDA translation units.  Not part of
 * the public ABI in include/pkv_b200.h.
 */
#ifndef PKV_INTERNAL_H
#define PKV_INTERNAL_H

#include <stddef.h>
#include <stdint.h>

#include "pkv_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* One new page-table entry: table[row * stride + index] = page. */
typedef struct {
    uint32_t row;
    uint32_t index;
    uint32_t page;
    uint32_t pad;
} PkvTablePatch;

/* Applies one step's staging on `stream` with one kernel that reads the
 * pinned host slot directly (device-visible pointers host_lens, host_patches
 * and host_done): lengths [batch] and row offsets [batch+1] (laid out at
 * host_lens and host_lens + max_batch) go to dev_lens (same layout), `count`
 * patches into the padded device table; then `ticket` is written to
 * *host_done, after which the host may refill the slot.  `arrive` is a
 * device word, zero before the launch (the kernel leaves it zero), that the
 * kernel's CTAs count themselves out on. */
int pkv_internal_stage_apply(const int32_t *host_lens, int32_t *dev_lens, size_t batch,
                             size_t max_batch, const PkvTablePatch *host_patches, size_t count,
                             uint32_t *table, size_t table_stride, size_t table_rows,
                             uint32_t *arrive, uint32_t *host_done, uint32_t ticket,
                             PkvStream stream);

/* Copies page ids [from, page_count) of `sequence` into dst and reports the
 * full page count; 0 for an unknown handle or a too-small capacity.  One
 * lock round trip, so the host layer uploads only the table's new tail;
 * *shrink_epoch changes whenever pages were removed from the table. */
int pkv_internal_copy_table_tail(TensorPagedKVCache *cache,
                                 TensorPagedKVSequence sequence, size_t from,
                                 uint32_t *dst, size_t capacity,
                                 size_t *page_count, size_t *length,
                                 uint32_t *shrink_epoch);

/* Read and clear the fault word of one kernel translation unit. */
int pkv_internal_take_copy_fault(uint32_t *code);
int pkv_internal_take_decode_fault(uint32_t *code);
int pkv_internal_take_prefill_fault(uint32_t *code);
int pkv_internal_take_sequence_fault(uint32_t *code);
int pkv_internal_take_peer_fault(uint32_t *code);

/* Tests on one GPU: makes `area` (a device buffer of
 * pkv_internal_peer_gather_area_bytes bytes on this GPU) stand in for the
 * area of `rank`, so a peer that never stores can be simulated. */
int pkv_internal_peer_gather_set_area(PkvPeerGather *gather, int rank, void *area);
size_t pkv_internal_peer_gather_area_bytes(const PkvPeerGather *gather);

/* Writes `code` into the prefill fault word of the current device: a
 * host-side stand-in for a kernel that recorded a fault, so tests can check
 * that callers report it (no kernel runs, nothing faults).  Exported for the
 * tests only. */
int pkv_internal_plant_prefill_fault(uint32_t code);

/* Replaces the completion check pkv_comm_wait uses (cudaStreamQuery) with
 * `probe` (1 done, 0 pending, -1 failed): tests of the deadline logic on
 * machines without a GPU.  Exported for the tests only. */
void pkv_internal_comm_set_probe(PkvComm *comm, int (*probe)(void *arg, PkvStream stream),
                                 void *arg);

/* pkv_paged_prefill with the general options the dense SDPA needs: an
 * additive FP16 mask [query row of the chunk][key] with a row stride in
 * elements (NULL: none), dense mode (a chunk may be longer than its
 * sequence; the causal offset kv_len - q_len clamps at 0), and the dense
 * layout (query and output are [sequences * q_heads][max_query_len][128],
 * every sequence holding max_query_len rows, read and written in place).
 * Errors name `what`. */
int pkv_internal_paged_prefill_ex(const PkvPagedLayer *layer, const PkvBatch *batch,
                                  size_t q_heads, const int32_t *query_offsets, const void *query,
                                  size_t total_query_rows, size_t max_query_len, float scale,
                                  int causal, void *output, PkvDType output_dtype,
                                  const uint16_t *mask, size_t mask_stride, int dense,
                                  int dense_layout, PkvStream stream, char *error,
                                  size_t error_capacity, const char *what);

/* Writes a message into a caller error buffer (NULL-safe). */
void pkv_internal_set_error(char *error, size_t capacity, const char *fmt, ...);

#ifdef __cplusplus
}
#endif

#endif
