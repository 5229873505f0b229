// pkv_dense.cu -- dense FP16 SDPA served by the tcgen05 paged prefill kernel.
//
// The SDK's tensor_sdpa_f16 (src/common/attention.c:408-459) hands its
// backend [batch][heads][length][dim] FP16 tensors (run_f16 of
// src/attention_backend.h; the CUDA backend's sdpa<T>, attention_cuda.cu:
// 25-99, materialises every score row).  Here each (batch, KV head) becomes
// one "sequence" of the paged prefill kernel with an identity page table:
//   * K and V of (b, g) are kv_len contiguous rows of head_dim elements, i.e. a
//     pool with one KV head whose pages are consecutive; when kv_len is a
//     multiple of 16 the tensors themselves are the pool (no copy), otherwise
//     each sequence is copied to a whole number of 16-row pages;
//   * the query and output tensors are read and written in place: the
//     kernel's dense layout addresses head (b, h) row i at ((b*Hq + h)*Lq +
//     i)*head_dim, the group of KV head g being heads g*G .. g*G+G-1;
//   * the causal rule key > query + max(kv_len - q_len, 0) is the prefill
//     kernel's own (in dense mode, which lets q_len exceed kv_len);
//   * an additive FP16 mask [q_len][kv_len] (shared by every batch and head,
//     as the SDK's) is added to the scaled scores inside the kernel's softmax;
//     a row whose maximum is not finite gives zeros (the CUDA backend's rule,
//     softmax_rows_kernel, attention_cuda.cu:45-55).
// head_dim = value_dim, 64 or 128 (the prefill kernel's instantiations).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "pkv_b200.h"
#include "pkv_internal.h"
#include "pkv_trace.h"

namespace pkv {
namespace {

constexpr int kPage = 16;

bool head_dim_ok(size_t d) { return d == 64 || d == 128; }

// K or V of every (b, g) into a whole number of 16-row pages; `chunks` is
// the number of 16-byte chunks in a row (head_dim / 8).
__global__ void pad_rows_kernel(const uint4 *src, uint4 *dst, int64_t S, int Lk, int pages,
                                int chunks) {
    const int64_t n = S * (int64_t)Lk * chunks;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(e % chunks);
        const int64_t r = e / chunks;
        const int64_t s = r / Lk;
        const int i = (int)(r - s * Lk);
        dst[((s * pages * kPage) + i) * chunks + c] = src[e];
    }
}

// Identity page tables, lengths and query row offsets of the S sequences.
__global__ void tables_kernel(uint32_t *tables, int32_t *lens, int32_t *offs, int64_t S,
                              int pages, int Lk, int Lq) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < S * pages;
         e += (int64_t)gridDim.x * blockDim.x)
        tables[e] = (uint32_t)e;  // sequence s, page p -> pool page s * pages + p
    for (int64_t s = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; s <= S;
         s += (int64_t)gridDim.x * blockDim.x) {
        if (s < S) lens[s] = Lk;
        offs[s] = (int32_t)(s * Lq);
    }
}

size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

struct DenseLayout {
    size_t tables, lens, offs, kpad, vpad, total;
};

DenseLayout dense_layout(size_t B, size_t Hq, size_t Hkv, size_t Lq, size_t Lk, size_t d) {
    const size_t S = B * Hkv, pages = (Lk + kPage - 1) / kPage;
    const bool pad = Lk % kPage != 0;
    DenseLayout w;
    w.tables = 0;
    w.lens = w.tables + align256(S * pages * 4);
    w.offs = w.lens + align256(S * 4);
    w.kpad = w.offs + align256((S + 1) * 4);
    w.vpad = w.kpad + (pad ? align256(S * pages * kPage * d * 2) : 0);
    w.total = w.vpad + (pad ? align256(S * pages * kPage * d * 2) : 0);
    return w;
}

int grid_for(int64_t n) {
    int64_t g = (n + 255) / 256;
    return (int)(g < 148 * 16 ? (g < 1 ? 1 : g) : 148 * 16);
}

std::mutex g_host_mutex;
void *g_host_ws[64];
size_t g_host_ws_bytes[64];

// Host staging for the run_f16 hook.  The SDK hands it pageable host arrays;
// a plain cudaMemcpy of those moves ~8 GB/s.  Instead each chunk is copied by
// several host threads into one of two pinned buffers while the DMA engine
// moves the other (events keep a buffer from being refilled before its copy
// ended).  Allocated once per process, used under g_host_mutex.
constexpr size_t kStageChunk = size_t(16) << 20;
struct HostStage {
    unsigned char *buf[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    int device = -1;
};
HostStage g_stage;

bool stage_ready(int dev) {
    if (g_stage.buf[0] != nullptr && g_stage.device == dev) return true;
    for (int i = 0; i < 2; ++i) {
        // An earlier call that failed part-way may have left a copy from
        // this pinned buffer in flight on the old device: wait for it before
        // the buffer is refilled under new events.
        if (g_stage.done[i] != nullptr) {
            cudaEventSynchronize(g_stage.done[i]);
            cudaEventDestroy(g_stage.done[i]);
        }
        g_stage.done[i] = nullptr;
        if (g_stage.buf[i] == nullptr &&
            cudaHostAlloc(reinterpret_cast<void **>(&g_stage.buf[i]), kStageChunk,
                          cudaHostAllocPortable) != cudaSuccess) {
            g_stage.buf[i] = nullptr;
            return false;
        }
        if (cudaEventCreateWithFlags(&g_stage.done[i], cudaEventDisableTiming) != cudaSuccess)
            return false;
    }
    g_stage.device = dev;  // events belong to the device current at creation
    return true;
}

// memcpy split over up to 8 host threads (one when the copy is small)
void par_copy(void *dst, const void *src, size_t n) {
    const unsigned hw = std::thread::hardware_concurrency();
    const size_t nt = n < (size_t(1) << 20) ? 1 : (hw < 2 ? 1 : (hw < 8 ? hw : 8));
    if (nt == 1) {
        std::memcpy(dst, src, n);
        return;
    }
    std::vector<std::thread> ts;
    const size_t part = (n / nt + 63) & ~size_t(63);
    size_t off = 0;
    try {  // no exception may leave the C ABI: a thread that cannot start
        ts.reserve(nt);  // leaves its part to this thread
        for (; off < n && ts.size() + 1 < nt; off += part) {
            const size_t len = off + part < n ? part : n - off;
            ts.emplace_back([=] {
                std::memcpy(static_cast<unsigned char *>(dst) + off,
                            static_cast<const unsigned char *>(src) + off, len);
            });
        }
    } catch (...) {
    }
    if (off < n)
        std::memcpy(static_cast<unsigned char *>(dst) + off,
                    static_cast<const unsigned char *>(src) + off, n - off);
    for (auto &t : ts) t.join();
}

// host (pageable) -> device through the staging buffers; `k` counts the
// chunks staged so far (it picks the buffer), the default stream is used.
bool stage_upload(void *dst, const void *src, size_t n, unsigned &k) {
    for (size_t off = 0; off < n; off += kStageChunk, ++k) {
        const int b = (int)(k & 1u);
        const size_t len = n - off < kStageChunk ? n - off : kStageChunk;
        if (cudaEventSynchronize(g_stage.done[b]) != cudaSuccess) return false;
        par_copy(g_stage.buf[b], static_cast<const unsigned char *>(src) + off, len);
        if (cudaMemcpyAsync(static_cast<unsigned char *>(dst) + off, g_stage.buf[b], len,
                            cudaMemcpyHostToDevice, nullptr) != cudaSuccess ||
            cudaEventRecord(g_stage.done[b], nullptr) != cudaSuccess)
            return false;
    }
    return true;
}

// device -> host (pageable): chunk c lands in a staging buffer while the
// host threads copy chunk c - 1 out of the other.
bool stage_download(void *dst, const void *src, size_t n, unsigned &k) {
    size_t prev_off = 0, prev_len = 0;
    int prev_b = -1;
    for (size_t off = 0;; off += kStageChunk, ++k) {
        int b = -1;
        size_t len = 0;
        if (off < n) {
            b = (int)(k & 1u);
            len = n - off < kStageChunk ? n - off : kStageChunk;
            if (cudaEventSynchronize(g_stage.done[b]) != cudaSuccess ||
                cudaMemcpyAsync(g_stage.buf[b], static_cast<const unsigned char *>(src) + off,
                                len, cudaMemcpyDeviceToHost, nullptr) != cudaSuccess ||
                cudaEventRecord(g_stage.done[b], nullptr) != cudaSuccess)
                return false;
        }
        if (prev_b >= 0) {
            if (cudaEventSynchronize(g_stage.done[prev_b]) != cudaSuccess) return false;
            par_copy(static_cast<unsigned char *>(dst) + prev_off, g_stage.buf[prev_b], prev_len);
        }
        if (b < 0) return true;
        prev_b = b;
        prev_off = off;
        prev_len = len;
    }
}

}  // namespace
}  // namespace pkv

extern "C" {

size_t pkv_sdpa_workspace_bytes(size_t batch, size_t q_heads, size_t kv_heads, size_t q_len,
                                size_t kv_len, size_t head_dim) {
    return pkv::dense_layout(batch, q_heads, kv_heads, q_len, kv_len, head_dim).total;
}

int pkv_sdpa_f16(const void *query, const void *key, const void *value,
                 const void *additive_mask, void *output, size_t batch, size_t q_heads,
                 size_t kv_heads, size_t q_len, size_t kv_len, size_t head_dim, float scale,
                 int causal, void *workspace, size_t workspace_bytes, PkvStream stream,
                 char *error, size_t error_capacity) {
    PKV_RANGE("pkv_sdpa_f16");
    using namespace pkv;
    const char *what = "pkv_sdpa_f16";
    if (query == nullptr || key == nullptr || value == nullptr || output == nullptr ||
        workspace == nullptr) {
        pkv_internal_set_error(error, error_capacity, "%s: null argument", what);
        return 0;
    }
    if (batch == 0 || q_heads == 0 || kv_heads == 0 || q_len == 0 || kv_len == 0 ||
        q_heads % kv_heads != 0 || q_heads / kv_heads > 65535 || q_len > (1u << 30) ||
        kv_len > (1u << 30) || batch * kv_heads > (1u << 24) ||
        batch * q_heads * q_len >= (size_t(1) << 31) || (causal != 0 && causal != 1) ||
        !isfinite(scale) || !head_dim_ok(head_dim)) {
        pkv_internal_set_error(error, error_capacity,
                               "%s: needs head_dim 64 or 128, q_heads a multiple of kv_heads, a "
                               "finite scale and causal 0 or 1",
                               what);
        return 0;
    }
    const DenseLayout w = dense_layout(batch, q_heads, kv_heads, q_len, kv_len, head_dim);
    if (workspace_bytes < w.total || (uintptr_t)workspace % 256 ||
        ((uintptr_t)query | (uintptr_t)key | (uintptr_t)value | (uintptr_t)output) % 16) {
        pkv_internal_set_error(error, error_capacity,
                               "%s: workspace needs %zu bytes (256-aligned), tensors 16-aligned",
                               what, w.total);
        return 0;
    }
    const cudaStream_t s = (cudaStream_t)stream;
    auto *ws = static_cast<unsigned char *>(workspace);
    const int64_t S = (int64_t)(batch * kv_heads);
    const int G = (int)(q_heads / kv_heads);
    const int pages = (int)((kv_len + kPage - 1) / kPage);
    const bool pad = kv_len % kPage != 0;
    auto *tables = reinterpret_cast<uint32_t *>(ws + w.tables);
    auto *lens = reinterpret_cast<int32_t *>(ws + w.lens);
    auto *offs = reinterpret_cast<int32_t *>(ws + w.offs);
    const void *kpool = key, *vpool = value;
    tables_kernel<<<grid_for(S * pages + S + 1), 256, 0, s>>>(tables, lens, offs, S, pages,
                                                              (int)kv_len, (int)q_len);
    if (pad) {
        const int chunks = (int)(head_dim / 8);
        const int64_t kn = S * (int64_t)kv_len * chunks;
        pad_rows_kernel<<<grid_for(kn), 256, 0, s>>>(static_cast<const uint4 *>(key),
                                                      reinterpret_cast<uint4 *>(ws + w.kpad), S,
                                                      (int)kv_len, pages, chunks);
        pad_rows_kernel<<<grid_for(kn), 256, 0, s>>>(static_cast<const uint4 *>(value),
                                                      reinterpret_cast<uint4 *>(ws + w.vpad), S,
                                                      (int)kv_len, pages, chunks);
        kpool = ws + w.kpad;
        vpool = ws + w.vpad;
    }
    if (cudaGetLastError() != cudaSuccess) {
        pkv_internal_set_error(error, error_capacity, "%s: launch failed", what);
        return 0;
    }
    PkvPagedLayer layer;
    layer.key_pool = const_cast<void *>(kpool);
    layer.value_pool = const_cast<void *>(vpool);
    layer.block_size = kPage;
    layer.block_count = (size_t)S * pages;
    layer.kv_heads = 1;
    layer.head_dim = head_dim;
    layer.dtype = PKV_DTYPE_F16;
    PkvBatch b;
    b.block_tables = tables;
    b.table_stride = (size_t)pages;
    b.seq_lens = lens;
    b.batch = (size_t)S;
    return pkv_internal_paged_prefill_ex(&layer, &b, (size_t)G, offs, query,
                                         (size_t)(S * (int64_t)q_len), q_len, scale, causal,
                                         output, PKV_DTYPE_F16,
                                         static_cast<const uint16_t *>(additive_mask), kv_len,
                                         q_len > kv_len, 1, stream, error, error_capacity, what);
}

int pkv_sdpa_f16_host(const uint16_t *query, const uint16_t *key, const uint16_t *value,
                      const uint16_t *additive_mask, uint16_t *output, size_t batch,
                      size_t query_heads, size_t kv_heads, size_t query_length,
                      size_t kv_length, size_t head_dim, size_t value_dim, float scale,
                      int causal) {
    PKV_RANGE("pkv_sdpa_f16_host");
    using namespace pkv;
    if (query == nullptr || key == nullptr || value == nullptr || output == nullptr ||
        !head_dim_ok(head_dim) || value_dim != head_dim || batch == 0 || query_heads == 0 ||
        kv_heads == 0 || query_length == 0 || kv_length == 0 || query_heads % kv_heads != 0)
        return 0;
    std::lock_guard<std::mutex> lock(g_host_mutex);
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    const size_t qb = batch * query_heads * query_length * head_dim * 2;
    const size_t kb = batch * kv_heads * kv_length * head_dim * 2;
    const size_t wsb = pkv_sdpa_workspace_bytes(batch, query_heads, kv_heads, query_length,
                                                kv_length, head_dim);
    const size_t mb = additive_mask != nullptr ? query_length * kv_length * 2 : 0;
    const size_t need = align256(qb) * 2 + align256(kb) * 2 + align256(mb) + wsb;
    if (g_host_ws_bytes[dev] < need) {
        if (g_host_ws[dev] != nullptr) cudaFree(g_host_ws[dev]);
        g_host_ws[dev] = nullptr;
        g_host_ws_bytes[dev] = 0;
        if (cudaMalloc(&g_host_ws[dev], need) != cudaSuccess) return 0;
        g_host_ws_bytes[dev] = need;
    }
    auto *base = static_cast<unsigned char *>(g_host_ws[dev]);
    unsigned char *dq = base, *dout = dq + align256(qb), *dk = dout + align256(qb);
    unsigned char *dv = dk + align256(kb), *dm = dv + align256(kb), *dws = dm + align256(mb);
    // the SDK's backends are synchronous and use the default stream
    if (!stage_ready(dev)) return 0;
    unsigned k = 0;
    if (!stage_upload(dq, query, qb, k) || !stage_upload(dk, key, kb, k) ||
        !stage_upload(dv, value, kb, k) ||
        (mb != 0 && !stage_upload(dm, additive_mask, mb, k)))
        return 0;
    if (!pkv_sdpa_f16(dq, dk, dv, mb != 0 ? dm : nullptr, dout, batch, query_heads, kv_heads,
                      query_length, kv_length, head_dim, scale, causal, dws, wsb, nullptr,
                      nullptr, 0))
        return 0;
    if (!stage_download(output, dout, qb, k) || cudaStreamSynchronize(nullptr) != cudaSuccess)
        return 0;
    // The kernel never traps: a bounded wait that gave up or an addressing
    // fault leaves a code in the prefill fault word and the output partial.
    // Only that word is read (and cleared) here, so fault codes of the other
    // kernels stay for pkv_device_fault.
    uint32_t fault = 0;
    return pkv_internal_take_prefill_fault(&fault) && fault == 0;
}

}  // extern "C"
