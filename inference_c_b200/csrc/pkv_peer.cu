// pkv_peer.cu -- all-gather of small per-rank outputs by plain stores into
// every peer GPU's memory over NVLink (the config-4 head split: each GPU
// decodes its KV heads, then every GPU needs every head's output).
//
// Each rank owns one device area, exported with CUDA IPC and mapped by the
// other ranks' processes:
//     [2 parities][nranks][bytes]   data (step s uses parity s & 1)
//     [kMaxRanks] u32               flags: flags[r] = last step rank r stored
// One single-CTA kernel per call: store this rank's `bytes` into slot `rank`
// of every rank's area (peer areas through their IPC mappings), fence at
// system scope, raise flags[rank] = step in every area (release), then wait
// until every flag of its own area reached `step` (acquire) and copy the
// gathered slots out to `recv`.  The wait is bounded: past its budget the
// kernel records kFaultWaitTimeout (read by pkv_device_fault) and returns
// without copying, so a missing peer never hangs the GPU.
//
// Parity double-buffering makes the slots reusable: a rank can write parity
// p again only at step s + 2, after its own wait at step s + 1 saw every
// rank's step-(s + 1) store, and a rank stores step s + 1 only after its
// kernel of step s (which copied parity p out) finished.  No load or store
// here uses TMA or multicast.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <new>

#include "pkv_b200.h"
#include "pkv_device.cuh"
#include "pkv_internal.h"
#include "pkv_trace.h"

namespace pkv {
namespace {

__device__ uint32_t g_peer_fault;

constexpr int kMaxRanks = 8;
constexpr size_t kMaxPeerBytes = size_t(1) << 20;  // per rank

struct PeerArgs {
    unsigned char *areas[kMaxRanks];  // each rank's area, valid on this device
    const unsigned char *send;
    unsigned char *recv;
    uint64_t bytes;      // per rank, a multiple of 16
    uint64_t flag_off;   // offset of the flags in an area
    int nranks, rank;
    uint32_t step;
    long long wait_cycles;
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__global__ void __launch_bounds__(256) peer_gather_kernel(const PeerArgs a) {
    pdl_wait();  // `send` comes from the kernel before this one
    __shared__ int all_arrived;
    const int tid = threadIdx.x;
    if (tid == 0) all_arrived = 1;
    const uint64_t n16 = a.bytes / 16;
    const uint64_t par = a.step & 1u;
    const uint4 *src = reinterpret_cast<const uint4 *>(a.send);
    for (int r = 0; r < a.nranks; ++r) {
        uint4 *dst = reinterpret_cast<uint4 *>(a.areas[r] + (par * a.nranks + a.rank) * a.bytes);
        for (uint64_t i = tid; i < n16; i += blockDim.x) dst[i] = src[i];
    }
    __syncthreads();  // every data store of the CTA is issued before a flag
    if (tid < a.nranks) {
        __threadfence_system();
        st_release_sys(reinterpret_cast<uint32_t *>(a.areas[tid] + a.flag_off) + a.rank, a.step);
    }
    if (tid < a.nranks) {
        const uint32_t *f =
            reinterpret_cast<const uint32_t *>(a.areas[a.rank] + a.flag_off) + tid;
        const long long start = clock64();
        bool ok = true;
        while ((int32_t)(ld_acquire_sys(f) - a.step) < 0) {
            if (clock64() - start > a.wait_cycles) {
                ok = false;
                break;
            }
            __nanosleep(64);
        }
        if (!ok) {
            record_fault(&g_peer_fault, kFaultWaitTimeout);
            atomicAnd(&all_arrived, 0);
        }
    }
    __syncthreads();
    if (!all_arrived) return;
    // L1 is not coherent with the peers' stores: read through L2
    const uint4 *mine = reinterpret_cast<const uint4 *>(a.areas[a.rank] + par * a.nranks * a.bytes);
    uint4 *out = reinterpret_cast<uint4 *>(a.recv);
    for (uint64_t i = tid; i < n16 * a.nranks; i += blockDim.x) out[i] = __ldcg(mine + i);
}

}  // namespace
}  // namespace pkv

struct PkvPeerGather {
    int device, nranks, rank;
    size_t bytes, flag_off, area_bytes;
    unsigned char *area;                        // this rank's (cudaMalloc)
    unsigned char *areas[pkv::kMaxRanks];       // every rank's, valid on `device`
    int opened[pkv::kMaxRanks];                 // IPC mappings to close
    uint32_t step;
};

extern "C" {

int pkv_peer_gather_create(int device, int nranks, int rank, size_t bytes_per_rank,
                           PkvPeerGather **gather, void *handle, size_t handle_bytes,
                           char *error, size_t cap) {
    const char *what = "pkv_peer_gather_create";
    PKV_RANGE("pkv_peer_gather_create");
    if (gather == nullptr || handle == nullptr || handle_bytes != PKV_PEER_HANDLE_BYTES ||
        nranks < 1 || nranks > pkv::kMaxRanks || rank < 0 || rank >= nranks ||
        bytes_per_rank == 0 || bytes_per_rank % 16 != 0 || bytes_per_rank > pkv::kMaxPeerBytes) {
        pkv_internal_set_error(error, cap,
                               "%s: needs 1..%d ranks, 16..%zu bytes per rank (a multiple of 16) "
                               "and a %d-byte handle buffer",
                               what, pkv::kMaxRanks, pkv::kMaxPeerBytes, PKV_PEER_HANDLE_BYTES);
        return 0;
    }
    *gather = nullptr;
    PkvPeerGather *g = new (std::nothrow) PkvPeerGather();
    if (g == nullptr) {
        pkv_internal_set_error(error, cap, "%s: out of host memory", what);
        return 0;
    }
    g->device = device;
    g->nranks = nranks;
    g->rank = rank;
    g->bytes = bytes_per_rank;
    g->flag_off = 2 * (size_t)nranks * bytes_per_rank;
    g->area_bytes = g->flag_off + 256;
    cudaIpcMemHandle_t h;
    cudaError_t st = cudaSetDevice(device);
    if (st == cudaSuccess) st = cudaMalloc(reinterpret_cast<void **>(&g->area), g->area_bytes);
    if (st == cudaSuccess) st = cudaMemset(g->area, 0, g->area_bytes);
    if (st == cudaSuccess) st = cudaIpcGetMemHandle(&h, g->area);
    if (st == cudaSuccess) st = cudaDeviceSynchronize();
    if (st != cudaSuccess) {
        pkv_internal_set_error(error, cap, "%s: %s", what, cudaGetErrorString(st));
        if (g->area != nullptr) cudaFree(g->area);
        delete g;
        return 0;
    }
    static_assert(sizeof(cudaIpcMemHandle_t) <= PKV_PEER_HANDLE_BYTES, "handle size");
    memset(handle, 0, PKV_PEER_HANDLE_BYTES);
    memcpy(handle, &h, sizeof h);
    g->areas[rank] = g->area;
    *gather = g;
    return 1;
}

int pkv_peer_gather_connect(PkvPeerGather *g, const void *handles, size_t handles_bytes,
                            char *error, size_t cap) {
    const char *what = "pkv_peer_gather_connect";
    PKV_RANGE("pkv_peer_gather_connect");
    if (g == nullptr || handles == nullptr ||
        handles_bytes != (size_t)g->nranks * PKV_PEER_HANDLE_BYTES) {
        pkv_internal_set_error(error, cap, "%s: needs nranks handles of %d bytes", what,
                               PKV_PEER_HANDLE_BYTES);
        return 0;
    }
    if (cudaSetDevice(g->device) != cudaSuccess) {
        pkv_internal_set_error(error, cap, "%s: cannot select device %d", what, g->device);
        return 0;
    }
    for (int r = 0; r < g->nranks; ++r) {
        if (r == g->rank || g->opened[r]) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const unsigned char *>(handles) + (size_t)r * PKV_PEER_HANDLE_BYTES,
               sizeof h);
        void *p = nullptr;
        const cudaError_t st = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (st != cudaSuccess) {
            pkv_internal_set_error(error, cap, "%s: rank %d's area: %s", what, r,
                                   cudaGetErrorString(st));
            return 0;
        }
        g->areas[r] = static_cast<unsigned char *>(p);
        g->opened[r] = 1;
    }
    return 1;
}

int pkv_peer_all_gather(PkvPeerGather *g, const void *send, void *recv, double timeout_s,
                        PkvStream stream, char *error, size_t cap) {
    const char *what = "pkv_peer_all_gather";
    PKV_RANGE("pkv_peer_all_gather");
    if (g == nullptr || send == nullptr || recv == nullptr || !(timeout_s > 0) ||
        timeout_s > 60 || ((uintptr_t)send | (uintptr_t)recv) % 16 != 0) {
        pkv_internal_set_error(error, cap, "%s: invalid arguments (16-byte aligned buffers, "
                               "a timeout in (0, 60] s)", what);
        return 0;
    }
    for (int r = 0; r < g->nranks; ++r)
        if (g->areas[r] == nullptr) {
            pkv_internal_set_error(error, cap, "%s: not connected to rank %d", what, r);
            return 0;
        }
    g->step = g->step + 1u == 0u ? 1u : g->step + 1u;
    pkv::PeerArgs a;
    for (int r = 0; r < pkv::kMaxRanks; ++r) a.areas[r] = r < g->nranks ? g->areas[r] : nullptr;
    a.send = static_cast<const unsigned char *>(send);
    a.recv = static_cast<unsigned char *>(recv);
    a.bytes = g->bytes;
    a.flag_off = g->flag_off;
    a.nranks = g->nranks;
    a.rank = g->rank;
    a.step = g->step;
    a.wait_cycles = (long long)(timeout_s * 2.0e9);  // SM cycles run at <= ~2 GHz
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(256);
    cfg.stream = (cudaStream_t)stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t st = cudaLaunchKernelEx(&cfg, pkv::peer_gather_kernel, a);
    if (st != cudaSuccess) {
        pkv_internal_set_error(error, cap, "%s: launch failed: %s", what, cudaGetErrorString(st));
        return 0;
    }
    return 1;
}

void pkv_peer_gather_destroy(PkvPeerGather *g) {
    if (g == nullptr) return;
    int prev = 0;
    const bool have_prev = cudaGetDevice(&prev) == cudaSuccess;
    cudaSetDevice(g->device);
    for (int r = 0; r < g->nranks; ++r)
        if (g->opened[r]) cudaIpcCloseMemHandle(g->areas[r]);
    cudaFree(g->area);
    if (have_prev) cudaSetDevice(prev);
    delete g;
}

int pkv_internal_take_peer_fault(uint32_t *code) {
    uint32_t zero = 0;
    if (cudaMemcpyFromSymbol(code, pkv::g_peer_fault, sizeof(uint32_t)) != cudaSuccess) return 0;
    return cudaMemcpyToSymbol(pkv::g_peer_fault, &zero, sizeof(uint32_t)) == cudaSuccess;
}

int pkv_internal_peer_gather_set_area(PkvPeerGather *g, int rank, void *area) {
    if (g == nullptr || rank < 0 || rank >= g->nranks || rank == g->rank || g->opened[rank])
        return 0;
    g->areas[rank] = static_cast<unsigned char *>(area);
    return 1;
}

size_t pkv_internal_peer_gather_area_bytes(const PkvPeerGather *g) {
    return g == nullptr ? 0 : g->area_bytes;
}

}  // extern "C"
