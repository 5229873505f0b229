// pkv_copy.cu -- KV append / prefix import / gather through the block table.
//
// All three are the same bandwidth-bound row copy between a contiguous
// [rows][kv_width] buffer and the paged pool, one warp per token row, 16-byte
// vector loads and stores (a 2 KiB Llama-3-8B row is 4 uint4 per lane for K
// and 4 for V, all issued before the first store).  The page address of a
// position follows the SDK's decode_kv_position (attention_cuda.cu:301-305).
#include <stdarg.h>
#include <stdio.h>

#include "pkv_device.cuh"
#include "pkv_internal.h"
#include "pkv_trace.h"

namespace pkv {
namespace {

__device__ uint32_t g_copy_fault;

constexpr int kCopyWarps = 8;

// Sequence owning contiguous row `row`: largest b with offsets[b] <= row.
__device__ __forceinline__ int find_sequence(const int32_t *offsets, int batch, int32_t row) {
    int lo = 0, hi = batch - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (__ldg(offsets + mid) <= row) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// TO_POOL: rows -> pages (append, import).  Otherwise pages -> rows (gather).
// `tail` selects where a sequence's rows land: its last n_b positions
// (append) or its first n_b positions (import, gather).
template <bool TO_POOL, int VEC>
__global__ void __launch_bounds__(kCopyWarps * 32)
kv_rows_kernel(uint4 *__restrict__ kpool, uint4 *__restrict__ vpool,
               uint4 *__restrict__ krows, uint4 *__restrict__ vrows,
               const uint32_t *__restrict__ tables, int32_t table_stride,
               const int32_t *__restrict__ seq_lens, const int32_t *__restrict__ offsets,
               int batch, int32_t total_rows, int vec_per_row, int block_size,
               int block_shift, uint32_t block_count, bool tail) {
    pdl_launch_dependents();  // a decode launched after this may set itself up now
    pdl_wait();               // the kernel before this one (tables, lengths, rows) is done
    const int lane = threadIdx.x & 31;
    const int32_t row = blockIdx.x * kCopyWarps + (threadIdx.x >> 5);
    if (row >= total_rows) return;
    int b;
    int32_t first, count;
    if (offsets == nullptr) {
        b = row;
        first = row;
        count = 1;
    } else {
        b = find_sequence(offsets, batch, row);
        first = __ldg(offsets + b);
        count = __ldg(offsets + b + 1) - first;
    }
    const int32_t len = __ldg(seq_lens + b);
    if (count > len) {
        if (lane == 0) record_fault(&g_copy_fault, kFaultRowsMismatch);
        return;
    }
    const int32_t pos = (tail ? len - count : 0) + (row - first);
    PageMap map{tables + (int64_t)b * table_stride, block_size, block_shift, block_count,
                table_stride};
    int64_t prow = 0;
    const uint32_t fault = map.row_of(pos, prow);
    if (fault != kFaultNone) {
        if (lane == 0) record_fault(&g_copy_fault, fault);
        return;
    }
    const int64_t src = (int64_t)row * vec_per_row;
    const int64_t dst = prow * vec_per_row;
    if constexpr (VEC > 0) {
        // Fixed row width: load everything first, then store.
        uint4 k[VEC], v[VEC];
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
            const int c = lane + 32 * i;
            k[i] = TO_POOL ? __ldg(krows + src + c) : __ldg(kpool + dst + c);
            v[i] = TO_POOL ? __ldg(vrows + src + c) : __ldg(vpool + dst + c);
        }
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
            const int c = lane + 32 * i;
            if (TO_POOL) { kpool[dst + c] = k[i]; vpool[dst + c] = v[i]; }
            else { krows[src + c] = k[i]; vrows[src + c] = v[i]; }
        }
    } else {
        for (int c = lane; c < vec_per_row; c += 32) {
            if (TO_POOL) {
                kpool[dst + c] = __ldg(krows + src + c);
                vpool[dst + c] = __ldg(vrows + src + c);
            } else {
                krows[src + c] = __ldg(kpool + dst + c);
                vrows[src + c] = __ldg(vpool + dst + c);
            }
        }
    }
}

// One step's staging, read straight from the pinned host slot (no copy on
// the stream): the lengths and row offsets go to the device slot the kernels
// of the step read, the new page-table entries into the padded table.  One
// CTA for a decode step; a large staging (a prefix import: thousands of new
// entries) spreads over several, which count themselves out on `arrive`
// (a device word, zero between launches).  The last CTA to finish writes
// `ticket` to the slot's host word, which tells the host the slot may be
// refilled; a one-CTA staging whose reads all precede its grid-dependency
// wait writes it before that wait.
__global__ void __launch_bounds__(512)
stage_apply_kernel(const int32_t *__restrict__ host_lens, int32_t *__restrict__ dev_lens,
                   int batch, int max_batch, const PkvTablePatch *__restrict__ host_patches,
                   int64_t count, uint32_t *__restrict__ table, int64_t stride, int64_t rows,
                   uint32_t *arrive, volatile uint32_t *host_done, uint32_t ticket) {
    pdl_launch_dependents();
    const int64_t first = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    // Each thread's first items cross the bus while the kernels before this
    // one drain (the decode kernel releases its dependents early): the host
    // slot stays the host's, unchanged, until the ticket below, and no kernel
    // writes it.  Nothing the earlier kernels read is written before the wait.
    int32_t len0 = 0, off0 = 0;
    PkvTablePatch p0 = {};
    if (first < batch) len0 = host_lens[first];
    if (first <= batch) off0 = host_lens[max_batch + first];
    if (first < count) p0 = host_patches[first];
    // A launch whose every slot read is one of those first items (one CTA,
    // batch + 1 lengths and count patches within its threads: every decode
    // step) hands the slot back before the wait.  Its reads have returned
    // once the CTA passes the barrier, and the ticket orders nothing else:
    // the host only refills the slot after seeing it.  The kernel after this
    // one then waits for nothing but the device writes below.
    const bool prefetched = gridDim.x == 1 && batch < (int)blockDim.x && count <= blockDim.x;
    if (prefetched) {
        __syncthreads();
        if (threadIdx.x == 0) *host_done = ticket;
    }
    pdl_wait();  // the previous step's kernels no longer read the table or this slot
    for (int64_t i = first; i <= batch; i += step) {
        if (i < batch) dev_lens[i] = i == first ? len0 : host_lens[i];
        dev_lens[max_batch + i] = i == first ? off0 : host_lens[max_batch + i];
    }
    for (int64_t i = first; i < count; i += step) {
        const PkvTablePatch p = i == first ? p0 : host_patches[i];
        if ((int64_t)p.row >= rows || (int64_t)p.index >= stride) {
            record_fault(&g_copy_fault, kFaultPositionOutOfRange);
            continue;
        }
        table[(int64_t)p.row * stride + p.index] = p.page;
    }
    if (prefetched) return;
    __syncthreads();  // every read of the host slot by this CTA has returned
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(arrive, 1u) == gridDim.x - 1) {  // the last CTA
            *arrive = 0u;
            __threadfence_system();
            *host_done = ticket;
        }
    }
}

// Launch with programmatic dependent launch: the kernel may start while the
// one before it in the stream drains; griddepcontrol.wait inside orders it.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, cudaStream_t s,
                       Args... args) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

int block_shift_of(size_t block_size) {
    if (block_size == 0 || (block_size & (block_size - 1)) != 0) return -1;
    int s = 0;
    while ((size_t(1) << s) < block_size) ++s;
    return s;
}

template <bool TO_POOL>
int launch_rows(const PkvPagedLayer *layer, const PkvBatch *batch, const int32_t *offsets,
                const void *krows, const void *vrows, size_t total_rows, bool tail,
                PkvStream stream, char *error, size_t cap, const char *what) {
    if (layer == nullptr || batch == nullptr || layer->key_pool == nullptr ||
        layer->value_pool == nullptr || krows == nullptr || vrows == nullptr ||
        batch->block_tables == nullptr || batch->seq_lens == nullptr) {
        pkv_internal_set_error(error, cap, "%s: null argument", what);
        return 0;
    }
    if (layer->dtype != PKV_DTYPE_F16 && layer->dtype != PKV_DTYPE_BF16) {
        pkv_internal_set_error(error, cap, "%s: pool dtype must be F16 or BF16", what);
        return 0;
    }
    const size_t kv_width = layer->kv_heads * layer->head_dim;
    if (kv_width == 0 || (kv_width * 2) % 16 != 0 || layer->block_size == 0 ||
        layer->block_count == 0 || batch->batch == 0 || batch->table_stride == 0 ||
        total_rows > INT32_MAX || batch->batch > INT32_MAX ||
        batch->table_stride > INT32_MAX || layer->block_size > INT32_MAX ||
        layer->block_count > UINT32_MAX) {
        pkv_internal_set_error(error, cap,
                               "%s: invalid shape (kv_width*2 must be a multiple of 16 bytes)",
                               what);
        return 0;
    }
    if (offsets == nullptr && total_rows != batch->batch) {
        pkv_internal_set_error(error, cap, "%s: one row per sequence needs total_rows == batch",
                               what);
        return 0;
    }
    if (((uintptr_t)layer->key_pool | (uintptr_t)layer->value_pool | (uintptr_t)krows |
         (uintptr_t)vrows) % 16 != 0) {
        pkv_internal_set_error(error, cap, "%s: buffers must be 16-byte aligned", what);
        return 0;
    }
    if (total_rows == 0) return 1;
    const int vec = (int)(kv_width * 2 / 16);
    const unsigned grid = (unsigned)((total_rows + kCopyWarps - 1) / kCopyWarps);
    auto *kp = static_cast<uint4 *>(layer->key_pool);
    auto *vp = static_cast<uint4 *>(layer->value_pool);
    auto *kr = static_cast<uint4 *>(const_cast<void *>(krows));
    auto *vr = static_cast<uint4 *>(const_cast<void *>(vrows));
    const int shift = block_shift_of(layer->block_size);
#define PKV_ROWS(V)                                                                           \
    launch_pdl(kv_rows_kernel<TO_POOL, V>, dim3(grid), dim3(kCopyWarps * 32),                \
               (cudaStream_t)stream, kp, vp, kr, vr, batch->block_tables,                     \
               (int32_t)batch->table_stride, batch->seq_lens, offsets, (int)batch->batch,     \
               (int32_t)total_rows, vec, (int)layer->block_size, shift,                      \
               (uint32_t)layer->block_count, tail)
    switch (vec) {
        case 32: PKV_ROWS(1); break;    // 512 B rows (e.g. 2 heads x 128)
        case 64: PKV_ROWS(2); break;
        case 128: PKV_ROWS(4); break;   // 2 KiB rows (8 heads x 128)
        case 256: PKV_ROWS(8); break;
        default: PKV_ROWS(0); break;
    }
#undef PKV_ROWS
    const cudaError_t st = cudaGetLastError();
    if (st != cudaSuccess) {
        pkv_internal_set_error(error, cap, "%s: launch failed: %s", what, cudaGetErrorString(st));
        return 0;
    }
    return 1;
}

}  // namespace
}  // namespace pkv

extern "C" {

void pkv_internal_set_error(char *error, size_t capacity, const char *fmt, ...) {
    if (error == nullptr || capacity == 0) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(error, capacity, fmt, ap);
    va_end(ap);
}

int pkv_kv_append(const PkvPagedLayer *layer, const PkvBatch *batch, const int32_t *row_offsets,
                  const void *key_rows, const void *value_rows, size_t total_rows,
                  PkvStream stream, char *error, size_t error_capacity) {
    PKV_RANGE("pkv_kv_append");
    return pkv::launch_rows<true>(layer, batch, row_offsets, key_rows, value_rows, total_rows,
                                  true, stream, error, error_capacity, "pkv_kv_append");
}

int pkv_kv_import(const PkvPagedLayer *layer, const PkvBatch *batch, const int32_t *row_offsets,
                  const void *key_rows, const void *value_rows, size_t total_rows,
                  PkvStream stream, char *error, size_t error_capacity) {
    PKV_RANGE("pkv_kv_import");
    return pkv::launch_rows<true>(layer, batch, row_offsets, key_rows, value_rows, total_rows,
                                  false, stream, error, error_capacity, "pkv_kv_import");
}

int pkv_kv_gather(const PkvPagedLayer *layer, const PkvBatch *batch, const int32_t *row_offsets,
                  void *key_out, void *value_out, size_t total_rows, PkvStream stream,
                  char *error, size_t error_capacity) {
    PKV_RANGE("pkv_kv_gather");
    return pkv::launch_rows<false>(layer, batch, row_offsets, key_out, value_out, total_rows,
                                   false, stream, error, error_capacity, "pkv_kv_gather");
}

int pkv_internal_stage_apply(const int32_t *host_lens, int32_t *dev_lens, size_t batch,
                             size_t max_batch, const PkvTablePatch *host_patches, size_t count,
                             uint32_t *table, size_t table_stride, size_t table_rows,
                             uint32_t *arrive, uint32_t *host_done, uint32_t ticket,
                             PkvStream stream) {
    // batch + 1 lengths and the patches within one CTA's threads let the
    // kernel read the whole slot before its grid-dependency wait
    const unsigned threads = count > 256 || batch >= 256 ? 512u : 256u;
    const size_t work = count > batch ? count : batch;
    const size_t per_cta = 4096;  // bus reads in flight per CTA, roughly
    const unsigned grid = (unsigned)(work <= per_cta ? 1 : (work + per_cta - 1) / per_cta < 64
                                                                ? (work + per_cta - 1) / per_cta
                                                                : 64);
    const cudaError_t st = pkv::launch_pdl(
        pkv::stage_apply_kernel, dim3(grid), dim3(threads), (cudaStream_t)stream, host_lens,
        dev_lens, (int)batch, (int)max_batch, host_patches, (int64_t)count, table,
        (int64_t)table_stride, (int64_t)table_rows, arrive, (volatile uint32_t *)host_done,
        ticket);
    return st == cudaSuccess && cudaGetLastError() == cudaSuccess;
}

// Reads and clears this unit's fault word on the current device.
int pkv_internal_take_copy_fault(uint32_t *code) {
    uint32_t zero = 0;
    if (cudaMemcpyFromSymbol(code, pkv::g_copy_fault, sizeof(uint32_t)) != cudaSuccess) return 0;
    return cudaMemcpyToSymbol(pkv::g_copy_fault, &zero, sizeof(uint32_t)) == cudaSuccess;
}

}  // extern "C"
