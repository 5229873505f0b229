// pkv_device.cuh -- device helpers shared by the sm_100a paged-KV kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace pkv {

// Fault codes written to a translation unit's fault word instead of trapping.
enum : uint32_t {
    kFaultNone = 0,
    kFaultPageOutOfRange = 1,   // block table entry >= block_count
    kFaultPositionOutOfRange = 2,  // position outside [0, table_stride*block_size)
    kFaultRowsMismatch = 3,     // new rows of a sequence exceed its length
    kFaultWaitTimeout = 4,      // a bounded spin-wait gave up
};

__device__ __forceinline__ void record_fault(uint32_t *word, uint32_t code) {
    atomicCAS(word, 0u, code);
}

// 16-byte async global->shared copy that skips L1 (cp.async.cg).
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Eight 2-byte storage elements packed in a uint4 -> eight floats.
template <typename T>
__device__ __forceinline__ void unpack8(const uint4 &raw, float (&f)[8]);

template <>
__device__ __forceinline__ void unpack8<__half>(const uint4 &raw, float (&f)[8]) {
    const __half2 *h = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 v = __half22float2(h[i]);
        f[2 * i] = v.x;
        f[2 * i + 1] = v.y;
    }
}

template <>
__device__ __forceinline__ void unpack8<__nv_bfloat16>(const uint4 &raw, float (&f)[8]) {
    // bf16 -> f32 is exact: the bf16 bits are the high half of the f32.
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        f[2 * i] = __uint_as_float(w[i] << 16);
        f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
}

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
    return __float2bfloat16_rn(v);
}

// Programmatic dependent launch.  launch_dependents lets the next kernel of
// the stream (when launched with programmatic serialization) start its
// prologue while this one runs; wait blocks until every kernel this one
// depends on has finished and its writes are visible.  Both are no-ops for
// kernels launched without the attribute.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

// 2^x on the SFU (PTX ex2.approx.ftz: relative error about 2^-22, results
// below 2^-126 flush to zero -- far beneath any softmax weight that matters).
__device__ __forceinline__ float ex2_fast(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, m));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
    return v;
}

// Page lookup.  Positions address logical token slots of one sequence.
struct PageMap {
    const uint32_t *table;  // this sequence's row of the padded table
    int32_t block_size;
    int32_t block_shift;    // log2(block_size) when a power of two, else -1
    uint32_t block_count;
    int32_t table_stride;

    // Physical pool row of logical position `pos`; returns a fault code
    // (kFaultNone on success) instead of touching memory out of range.
    __device__ __forceinline__ uint32_t row_of(int32_t pos, int64_t &row) const {
        int32_t page_idx, in_page;
        if (block_shift >= 0) {
            page_idx = pos >> block_shift;
            in_page = pos & (block_size - 1);
        } else {
            page_idx = pos / block_size;
            in_page = pos - page_idx * block_size;
        }
        if (pos < 0 || page_idx >= table_stride) return kFaultPositionOutOfRange;
        const uint32_t page = __ldg(table + page_idx);
        if (page >= block_count) return kFaultPageOutOfRange;
        row = (int64_t)page * block_size + in_page;
        return kFaultNone;
    }
};

}  // namespace pkv
