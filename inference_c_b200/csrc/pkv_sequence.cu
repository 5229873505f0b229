// pkv_sequence.cu -- tensor_attention_decode_sequence_paged on the B200 path.
//
// Greedy decoding of one sequence through a dense decoder stack, with every
// layer's K/V kept in the cache's pages.  This replaces the SDK's transaction
// (src/common/attention.c:124-176) and its CUDA backend
// (src/platform/cuda/attention_cuda.cu:754-1090) with the same arithmetic
// contract, step by step:
//
//   x      = embedding[token]                                     (T)
//   per layer:
//     n    = x * rsqrt(mean(x^2) + eps) * input_norm               (T)  :106-124
//     qkv  = [Wq; Wk; Wv] . n                                      (T)  :126-143
//     q, k = RoPE(q), RoPE(k) at `position` (split halves, angle =
//            position / theta^(2f/d)); k and v stored in the page row
//            table[position / P] * P + position % P                (T)  :307-341
//     a    = softmax(q . K^T / sqrt(d)) . V over positions 0..pos  (T)  :343-398
//     r    = Wo . a + x                                            (T)  :145-163
//     n2   = rms(r) * post_norm                                    (T)
//     g    = silu(Wg . n2) * (Wu . n2)                             (T)  :165-195
//     x    = Wd . g + r                                            (T)
//   logits = lm_head . rms(x) * final_norm; token = first argmax        :400-410
//
// T is float for F32 storage and half otherwise; values are rounded to T at
// exactly these points, as in the SDK.  For QUANT_F16 storage the matrices
// are Q8_0/Q4_0 blocks and the residual adds are a separate rounding of the
// half result (attention_cuda.cu:293-299).  Sums run in FP32 in a different
// order than the SDK's 128-lane trees, so results agree to FP32 rounding,
// not bit for bit.
//
// B200 choices: matrices are streamed with one warp per output row and
// 16-byte vector loads (the GEMVs are HBM-bound on weight bytes); RoPE is
// fused into the page store; attention runs on the tcgen05 paged decode
// kernel (F16 pages, head_dim 128) or the CUDA-core one (head_dim 64), and on
// a generic split-K kernel for other shapes; the host transaction, block
// table upload and prefix import go through the batch pool (pkv_pool.c),
// the prefix as one device scatter instead of one copy per page run.
#include <cuda_runtime.h>
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <mutex>
#include <unordered_map>
#include <vector>

#include "attention.h"
#include "pkv_b200.h"
#include "pkv_device.cuh"
#include "pkv_internal.h"
#include "pkv_trace.h"

namespace pkv {
namespace {

__device__ uint32_t g_sequence_fault;

constexpr int kGemvThreads = 256;
constexpr int kAttnThreads = 256;
constexpr int kAttnChunk = 512;   // positions per split of the generic attention
constexpr int kGemvMaxGrid = 148 * 16;
constexpr int kGemvMaxIn = 53248;  // input elements staged in shared memory (208 KiB)

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---------------------------------------------------------------- GEMV ----
enum class WF : int { Dense = 0, Q8 = 1, Q4 = 2 };
enum Epi : int { kPlain = 0, kResidual = 1, kSwiGLU = 2, kArgmax = 3 };

struct GemvArgs {
    const void *m[3];  // matrices; output rows stack m[0], m[1], m[2] (SwiGLU: gate, up)
    int rows[3];
    int in;
    int out;
    const void *x;       // input vector (T)
    const void *norm_w;  // RMSNorm weight applied to x first (nullptr: none)
    float eps;
    const void *res;     // residual (T) for kResidual
    void *y;             // output (T)
    // kArgmax: per-CTA best (value, index), ticket, outputs
    float *part_v;
    int *part_i;
    unsigned *ticket;
    uint32_t *tokens;      // outputs, indexed by *step
    uint32_t *next_token;  // the next step's input token
    int32_t *step;         // tokens generated so far in this call
    int32_t *position;     // position of the next token
};

// One element of a Q*_0 block (scale * q, exact in FP32).
template <WF F>
__device__ __forceinline__ float quant_value(const uint8_t *block, float scale, int k) {
    if (F == WF::Q8) return scale * (float)(int8_t)block[2 + k];
    const uint8_t packed = block[2 + (k & 15)];
    return scale * (float)((int)(k < 16 ? packed & 15 : packed >> 4) - 8);
}

// E input elements starting at element i: from shared memory (FP32) or from
// global memory (T, one 16-byte load when E elements fill it).
template <typename T, int E>
__device__ __forceinline__ void load_x(const float *xs, int i, float (&v)[E]) {
#pragma unroll
    for (int e = 0; e < E; ++e) v[e] = xs[i + e];
}
template <typename T, int E>
__device__ __forceinline__ void load_x(const T *x, int i, float (&v)[E]) {
    const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(x + i));
    const T *t = reinterpret_cast<const T *>(&raw);
#pragma unroll
    for (int e = 0; e < E; ++e) v[e] = to_f(t[e]);
}
__device__ __forceinline__ float load_x1(const float *xs, int i) { return xs[i]; }
template <typename T>
__device__ __forceinline__ float load_x1(const T *x, int i) { return to_f(x[i]); }

// Dot product of one matrix row with the input vector (XT: FP32 staged in
// shared memory, or T read from global memory), summed over the warp.
template <typename T, WF F, typename XT>
__device__ __forceinline__ float row_dot(const void *mat, int row, int in, const XT *x, int lane) {
    float acc = 0.f;
    if (F == WF::Dense) {
        const T *w = static_cast<const T *>(mat) + (size_t)row * in;
        constexpr int E = 16 / sizeof(T);  // elements per 16-byte vector
        const bool vec = ((size_t)in * sizeof(T)) % 16 == 0 &&
                         ((uintptr_t)w | (uintptr_t)x) % 16 == 0;
        if (vec) {
            const int nv = in / E;
            const uint4 *wv = reinterpret_cast<const uint4 *>(w);
            int c = lane;
            for (; c + 96 < nv; c += 128) {  // four 16-byte weight loads in flight per lane
                uint4 a[4];
                float xv[4][E];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    a[u] = __ldg(wv + c + 32 * u);
                    load_x<T, E>(x, (c + 32 * u) * E, xv[u]);
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const T *wa = reinterpret_cast<const T *>(&a[u]);
#pragma unroll
                    for (int e = 0; e < E; ++e) acc = fmaf(xv[u][e], to_f(wa[e]), acc);
                }
            }
            for (; c < nv; c += 32) {
                const uint4 a = __ldg(wv + c);
                float xv[E];
                load_x<T, E>(x, c * E, xv);
                const T *wa = reinterpret_cast<const T *>(&a);
#pragma unroll
                for (int e = 0; e < E; ++e) acc = fmaf(xv[e], to_f(wa[e]), acc);
            }
        } else {
            for (int i = lane; i < in; i += 32) acc = fmaf(load_x1(x, i), to_f(w[i]), acc);
        }
    } else {
        constexpr int BB = F == WF::Q8 ? 34 : 18;
        const int nb = in / 32;
        const uint8_t *w = static_cast<const uint8_t *>(mat) + (size_t)row * nb * BB;
        for (int b = lane; b < nb; b += 32) {
            const uint8_t *blk = w + (size_t)b * BB;
            const uint16_t bits = (uint16_t)blk[0] | ((uint16_t)blk[1] << 8);
            const float scale = __half2float(__ushort_as_half(bits));
#pragma unroll 8
            for (int k = 0; k < 32; ++k)
                acc = fmaf(load_x1(x, b * 32 + k), quant_value<F>(blk, scale, k), acc);
        }
    }
    return warp_sum_f(acc);
}

// First maximum merge: (v, i) replaces (bv, bi) when strictly larger, or
// equal with a smaller index.  NaN never wins.
__device__ __forceinline__ void best_merge(float &bv, int &bi, float v, int i) {
    if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
    }
}

// y[r] = epilogue(M[r] . n), n = x, or RMSNorm(x) rounded to T as the SDK
// stores it, then staged once per CTA in shared memory as FP32.  One warp
// per output row; the CTAs stride over the rows.
template <typename T, WF F, int EPI, bool NORM>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const GemvArgs a) {
    extern __shared__ float xs[];
    __shared__ float red[kGemvThreads / 32];
    __shared__ int redi[kGemvThreads / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int warps = kGemvThreads / 32;
    pdl_launch_dependents();
    // The weights do not depend on earlier kernels: start pulling the first
    // 2 KiB of this warp's first row into L2 while they finish.
    {
        const int r = blockIdx.x * warps + warp;
        if (F == WF::Dense && r < a.out && r < a.rows[0]) {
            const char *w = static_cast<const char *>(a.m[0]) + (size_t)r * a.in * sizeof(T);
            const int bytes = min(a.in * (int)sizeof(T), 2048);
            if (lane * 128 < bytes) asm volatile("prefetch.global.L2 [%0];" ::"l"(w + lane * 128));
        }
    }
    pdl_wait();  // x, the residual and the argmax ticket come from earlier kernels
    const T *x = static_cast<const T *>(a.x);
    if (NORM) {
        // RMSNorm (attention_cuda.cu:106-124): x * rsqrt(mean(x^2) + eps) * w
        float s = 0.f;
        for (int i = threadIdx.x; i < a.in; i += kGemvThreads) {
            const float v = to_f(x[i]);
            s = fmaf(v, v, s);
        }
        s = warp_sum_f(s);
        if (lane == 0) red[warp] = s;
        __syncthreads();
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < warps; ++w) tot += red[w];
        const float scale = rsqrtf(tot / (float)a.in + a.eps);
        const T *nw = static_cast<const T *>(a.norm_w);
        for (int i = threadIdx.x; i < a.in; i += kGemvThreads)
            xs[i] = to_f(from_f32<T>(to_f(x[i]) * scale * to_f(nw[i])));
        __syncthreads();
    }
    T *y = static_cast<T *>(a.y);
    float bv = -INFINITY;
    int bi = INT32_MAX;
    for (int r = blockIdx.x * warps + warp; r < a.out; r += gridDim.x * warps) {
        if (EPI == kSwiGLU) {
            const float g = NORM ? row_dot<T, F>(a.m[0], r, a.in, xs, lane)
                                 : row_dot<T, F>(a.m[0], r, a.in, x, lane);
            const float u = NORM ? row_dot<T, F>(a.m[1], r, a.in, xs, lane)
                                 : row_dot<T, F>(a.m[1], r, a.in, x, lane);
            if (lane == 0) y[r] = from_f32<T>(g / (1.0f + expf(-g)) * u);
            continue;
        }
        int mi = 0, rr = r;
        while (mi < 2 && rr >= a.rows[mi]) rr -= a.rows[mi++];
        const float s = NORM ? row_dot<T, F>(a.m[mi], rr, a.in, xs, lane)
                             : row_dot<T, F>(a.m[mi], rr, a.in, x, lane);
        if (EPI == kResidual) {
            if (lane == 0) {
                const float res = to_f(static_cast<const T *>(a.res)[r]);
                // the quantised path rounds the product before the residual add
                const float v = F == WF::Dense ? s : to_f(from_f32<T>(s));
                y[r] = from_f32<T>(v + res);
            }
        } else {
            const T t = from_f32<T>(s);
            if (lane == 0) y[r] = t;
            if (EPI == kArgmax) {
                const float v = to_f(t);
                if (v == v) best_merge(bv, bi, v, r);
            }
        }
    }
    if (EPI != kArgmax) return;
    // first argmax over all CTAs (attention_cuda.cu:400-410): per-CTA best,
    // then the last CTA to finish reduces them
    __shared__ int last;
    if (lane == 0) {
        red[warp] = bv;
        redi[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < warps; ++w) best_merge(bv, bi, red[w], redi[w]);
        a.part_v[blockIdx.x] = bv;
        a.part_i[blockIdx.x] = bi;
        __threadfence();
        last = atomicAdd(a.ticket, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    bv = -INFINITY;
    bi = INT32_MAX;
    for (int c = threadIdx.x; c < (int)gridDim.x; c += kGemvThreads)
        best_merge(bv, bi, __ldcg(a.part_v + c), __ldcg(a.part_i + c));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        best_merge(bv, bi, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o));
    if (lane == 0) {
        red[warp] = bv;
        redi[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < warps; ++w) best_merge(bv, bi, red[w], redi[w]);
        // logits[0] starts the SDK's scan: a NaN there keeps index 0, and only
        // a strictly larger value replaces it
        const float first = to_f(__ldcg(static_cast<const T *>(a.y)));
        const uint32_t t =
            (first != first || bi == INT32_MAX || !(bv > first)) ? 0u : (uint32_t)bi;
        a.tokens[*a.step] = t;
        *a.next_token = t;
        *a.step += 1;
        *a.position += 1;
        *a.ticket = 0u;
    }
}

// ------------------------------------------------------ elementwise -------
template <typename T>
__global__ void embed_kernel(const T *emb, const uint32_t *token, T *x, int width,
                             uint32_t vocab) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t t = *token;
    if (t >= vocab) {
        if (blockIdx.x == 0 && threadIdx.x == 0) record_fault(&g_sequence_fault, kFaultPositionOutOfRange);
        return;
    }
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < width; i += gridDim.x * blockDim.x)
        x[i] = emb[(size_t)t * width + i];
}

// RoPE of q (into qrot) and of the new k, k and v stored in their page row,
// and the visible length position + 1 for the attention that follows.  The
// position lives on the device (advanced by the argmax), so one token's
// launches are the same every step and replay as a CUDA graph.
template <typename T>
__global__ void rope_store_kernel(const T *qkv, T *qrot, T *kpool, T *vpool,
                                  const uint32_t *table, int table_stride, int block_size,
                                  uint32_t block_count, int hidden, int kv_width, int head_dim,
                                  const int32_t *position_dev, float theta, int32_t *seq_len) {
    pdl_launch_dependents();
    pdl_wait();
    const int index = blockIdx.x * blockDim.x + threadIdx.x;
    const int half_dim = head_dim / 2;
    const int position = *position_dev;
    if (index == 0) *seq_len = position + 1;
    auto rotate = [&](const T *v, int i) -> float {
        const int dim = i % head_dim;
        const int base = i - dim;
        const int paired = base + (dim < half_dim ? dim + half_dim : dim - half_dim);
        const int freq = dim < half_dim ? dim : dim - half_dim;
        const float angle =
            (float)position / powf(theta, 2.0f * (float)freq / (float)head_dim);
        const float sign = dim < half_dim ? -1.0f : 1.0f;
        return to_f(v[i]) * cosf(angle) + sign * to_f(v[paired]) * sinf(angle);
    };
    if (index < hidden) qrot[index] = from_f32<T>(rotate(qkv, index));
    if (index < kv_width) {
        const int page = position / block_size;
        const uint32_t pid = page < table_stride ? table[page] : block_count;
        if (pid >= block_count) {
            record_fault(&g_sequence_fault, kFaultPageOutOfRange);
            return;
        }
        const size_t row = (size_t)pid * block_size + position % block_size;
        kpool[row * kv_width + index] = from_f32<T>(rotate(qkv + hidden, index));
        vpool[row * kv_width + index] = qkv[hidden + kv_width + index];
    }
}

// Prefix import: contiguous host rows [past][kv_width] (staged on the
// device) scattered into their page rows.
template <typename T>
__global__ void scatter_prefix_kernel(const T *krows, const T *vrows, T *kpool, T *vpool,
                                      const uint32_t *table, int table_stride, int block_size,
                                      uint32_t block_count, int kv_width, int64_t count) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < count;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t pos = e / kv_width;
        const int col = (int)(e - pos * kv_width);
        const int64_t page = pos / block_size;
        const uint32_t pid = page < table_stride ? table[page] : block_count;
        if (pid >= block_count) {
            record_fault(&g_sequence_fault, kFaultPageOutOfRange);
            continue;
        }
        const size_t row = (size_t)pid * block_size + (size_t)(pos % block_size);
        kpool[row * kv_width + col] = krows[e];
        vpool[row * kv_width + col] = vrows[e];
    }
}

// -------------------------------------------------- generic attention -----
// Any head_dim (<= 256) and page size.  Grid (query heads, splits of
// kAttnChunk positions); 8 warps per CTA stride over the split's positions
// with a running max; partials (m, l, o[head_dim]) go to `part`, merged by
// attn_merge_kernel.
template <typename T>
__global__ void __launch_bounds__(kAttnThreads) attn_split_kernel(
    const T *q, const T *kpool, const T *vpool, const uint32_t *table, int table_stride,
    int block_size, uint32_t block_count, const int32_t *seq_len, int q_heads, int kv_heads,
    int head_dim, float scale, float *part) {
    constexpr int kMaxJ = 8;  // head_dim / 32 rounded up
    __shared__ float wm[8], wl[8];
    __shared__ float wo[8][256];
    const int h = blockIdx.x, split = blockIdx.y, splits = gridDim.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    pdl_launch_dependents();
    pdl_wait();
    const int L = *seq_len;
    const int kvh = h / (q_heads / kv_heads);
    const int kv_width = kv_heads * head_dim;
    float qv[kMaxJ], acc[kMaxJ];
#pragma unroll
    for (int j = 0; j < kMaxJ; ++j) {
        const int d = lane + 32 * j;
        qv[j] = d < head_dim ? to_f(q[h * head_dim + d]) : 0.f;
        acc[j] = 0.f;
    }
    float m = -INFINITY, l = 0.f;
    const int p0 = split * kAttnChunk, p1 = min(L, p0 + kAttnChunk);
    for (int p = p0 + warp; p < p1; p += 8) {
        const int page = p / block_size;
        const uint32_t pid = page < table_stride ? table[page] : block_count;
        if (pid >= block_count) {
            if (lane == 0) record_fault(&g_sequence_fault, kFaultPageOutOfRange);
            continue;
        }
        const size_t base = ((size_t)pid * block_size + p % block_size) * kv_width +
                            (size_t)kvh * head_dim;
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < kMaxJ; ++j) {
            const int d = lane + 32 * j;
            if (d < head_dim) s = fmaf(qv[j], to_f(kpool[base + d]), s);
        }
        s = warp_sum_f(s) * scale;
        const float m_new = fmaxf(m, s);
        const float c = m == -INFINITY ? 0.f : expf(m - m_new);
        const float e = expf(s - m_new);
        l = l * c + e;
#pragma unroll
        for (int j = 0; j < kMaxJ; ++j) {
            const int d = lane + 32 * j;
            const float v = d < head_dim ? to_f(vpool[base + d]) : 0.f;
            acc[j] = fmaf(e, v, acc[j] * c);
        }
        m = m_new;
    }
    if (lane == 0) {
        wm[warp] = m;
        wl[warp] = l;
    }
#pragma unroll
    for (int j = 0; j < kMaxJ; ++j) {
        const int d = lane + 32 * j;
        if (d < head_dim) wo[warp][d] = acc[j];
    }
    __syncthreads();
    float M = -INFINITY;
    for (int w = 0; w < 8; ++w) M = fmaxf(M, wm[w]);
    float* out = part + ((size_t)h * splits + split) * (head_dim + 2);
    for (int d = threadIdx.x; d < head_dim; d += blockDim.x) {
        float o = 0.f;
        for (int w = 0; w < 8; ++w)
            if (wm[w] != -INFINITY) o += wo[w][d] * expf(wm[w] - M);
        out[2 + d] = o;
    }
    if (threadIdx.x == 0) {
        float lt = 0.f;
        for (int w = 0; w < 8; ++w)
            if (wm[w] != -INFINITY) lt += wl[w] * expf(wm[w] - M);
        out[0] = M;
        out[1] = lt;
    }
}

template <typename T>
__global__ void attn_merge_kernel(const float *part, int splits, int head_dim, T *out) {
    pdl_launch_dependents();
    pdl_wait();
    const int h = blockIdx.x;
    const float *p = part + (size_t)h * splits * (head_dim + 2);
    float M = -INFINITY;
    for (int s = 0; s < splits; ++s) M = fmaxf(M, p[(size_t)s * (head_dim + 2)]);
    float L = 0.f;
    for (int s = 0; s < splits; ++s) {
        const float ms = p[(size_t)s * (head_dim + 2)];
        if (ms != -INFINITY) L += p[(size_t)s * (head_dim + 2) + 1] * expf(ms - M);
    }
    for (int d = threadIdx.x; d < head_dim; d += blockDim.x) {
        float o = 0.f;
        for (int s = 0; s < splits; ++s) {
            const float ms = p[(size_t)s * (head_dim + 2)];
            if (ms != -INFINITY) o += p[(size_t)s * (head_dim + 2) + 2 + d] * expf(ms - M);
        }
        // all scores non-finite: zeros, as the SDK's softmax (attention_cuda.cu:367-370)
        out[h * head_dim + d] = from_f32<T>(M == -INFINITY || !(L > 0.f) ? 0.f : o / L);
    }
}

// ------------------------------------------------------------ host -------
struct DevWeight {
    void *ptr = nullptr;
    size_t bytes = 0;
};

struct Context {
    int device = -1;
    cudaStream_t stream = nullptr;
    void *blk = nullptr;       // activations, carved per call
    void *logits = nullptr;
    uint32_t *tokens = nullptr;  // [count] outputs, then the current token and visible length
    float *apart = nullptr;    // generic attention partials
    void *ws = nullptr;        // paged decode workspace
    void *stage = nullptr;     // prefix rows staged on the device
    size_t cap_blk = 0, cap_logits = 0, cap_tokens = 0, cap_apart = 0, cap_ws = 0, cap_stage = 0;
};

std::mutex g_mutex;
std::unordered_map<const void *, DevWeight> g_weights;  // host pointer -> device copy
std::unordered_map<int, Context> g_contexts;              // per device

void *weight(const void *host, size_t bytes) {
    if (host == nullptr || bytes == 0) return nullptr;
    auto it = g_weights.find(host);
    if (it != g_weights.end()) {
        if (it->second.bytes == bytes) return it->second.ptr;
        cudaFree(it->second.ptr);
        g_weights.erase(it);
    }
    void *d = nullptr;
    if (cudaMalloc(&d, bytes) != cudaSuccess) return nullptr;
    if (cudaMemcpy(d, host, bytes, cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaFree(d);
        return nullptr;
    }
    g_weights.emplace(host, DevWeight{d, bytes});
    return d;
}

bool grow(void **p, size_t *cap, size_t need) {
    if (need <= *cap && *p != nullptr) return true;
    if (*p != nullptr) cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    if (cudaMalloc(p, need) != cudaSuccess) {
        *p = nullptr;
        return false;
    }
    *cap = need;
    return true;
}

Context *context_for_device(int dev) {
    Context &c = g_contexts[dev];
    if (c.stream == nullptr) {
        c.device = dev;
        if (cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking) != cudaSuccess) {
            c.stream = nullptr;
            return nullptr;
        }
    }
    return &c;
}

void free_context(Context &c) {
    void *bufs[] = {c.blk, c.logits, c.tokens, c.apart, c.ws, c.stage};
    for (void *b : bufs)
        if (b != nullptr) cudaFree(b);
    if (c.stream != nullptr) cudaStreamDestroy(c.stream);
    c = Context();
}

struct Dims {
    size_t hidden, inter, qh, kvh, hd, kvw, vocab, layers, past, count, target;
    float eps, theta;
};

// Launches with programmatic dependent launch: the kernel may start while the
// one before it in the stream finishes; every decoder kernel waits
// (griddepcontrol.wait) before it reads what earlier kernels wrote.
template <typename... KArgs, typename... Args>
bool launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                Args... args) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...) == cudaSuccess;
}

template <typename T, WF F, int EPI, bool NORM>
bool launch_gemv_n(const GemvArgs &a, cudaStream_t s) {
    const int warps = kGemvThreads / 32;
    int grid = (a.out + warps - 1) / warps;
    if (grid > kGemvMaxGrid) grid = kGemvMaxGrid;
    const size_t smem = NORM ? (size_t)a.in * sizeof(float) : 0;
    static bool configured[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (smem > 48 * 1024 && dev >= 0 && dev < 64 && !configured[dev]) {
        if (cudaFuncSetAttribute(gemv_kernel<T, F, EPI, NORM>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)(kGemvMaxIn * sizeof(float))) != cudaSuccess)
            return false;
        configured[dev] = true;
    }
    return launch_pdl(gemv_kernel<T, F, EPI, NORM>, dim3(grid), dim3(kGemvThreads), smem, s, a);
}

template <typename T, WF F, int EPI>
bool launch_gemv(const GemvArgs &a, cudaStream_t s) {
    return a.norm_w != nullptr ? launch_gemv_n<T, F, EPI, true>(a, s)
                               : launch_gemv_n<T, F, EPI, false>(a, s);
}

// One matrix-vector product of the decoder.
struct Gemv {
    const void *m0 = nullptr, *m1 = nullptr, *m2 = nullptr;
    int r0 = 0, r1 = 0, r2 = 0, in = 0, out = 0;
    const void *x = nullptr, *norm_w = nullptr, *res = nullptr;
    void *y = nullptr;
    float eps = 0.f;
    int epi = kPlain;
    float *part_v = nullptr;
    int *part_i = nullptr;
    unsigned *ticket = nullptr;
    uint32_t *tokens = nullptr, *next_token = nullptr;
    int32_t *step = nullptr, *position = nullptr;
};

template <typename T, WF F>
bool run_gemv_f(const Gemv &g, cudaStream_t s) {
    GemvArgs a;
    a.m[0] = g.m0;
    a.m[1] = g.m1;
    a.m[2] = g.m2;
    a.rows[0] = g.r0;
    a.rows[1] = g.r1;
    a.rows[2] = g.r2;
    a.in = g.in;
    a.out = g.out;
    a.x = g.x;
    a.norm_w = g.norm_w;
    a.eps = g.eps;
    a.res = g.res;
    a.y = g.y;
    a.part_v = g.part_v;
    a.part_i = g.part_i;
    a.ticket = g.ticket;
    a.tokens = g.tokens;
    a.next_token = g.next_token;
    a.step = g.step;
    a.position = g.position;
    switch (g.epi) {
        case kResidual: return launch_gemv<T, F, kResidual>(a, s);
        case kSwiGLU: return launch_gemv<T, F, kSwiGLU>(a, s);
        case kArgmax: return launch_gemv<T, F, kArgmax>(a, s);
        default: return launch_gemv<T, F, kPlain>(a, s);
    }
}

template <typename T>
bool run_gemv(WF f, const Gemv &g, cudaStream_t s) {
    if (f == WF::Q8) return run_gemv_f<T, WF::Q8>(g, s);
    if (f == WF::Q4) return run_gemv_f<T, WF::Q4>(g, s);
    return run_gemv_f<T, WF::Dense>(g, s);
}

// Bytes of an [out][in] matrix in format f with element type T.
template <typename T>
size_t mat_bytes(WF f, size_t out, size_t in) {
    if (f == WF::Dense) return out * in * sizeof(T);
    return out * (in / 32) * (f == WF::Q8 ? 34u : 18u);
}

// Device pointers of one layer's tensors.
struct DevLayer {
    const void *input_norm, *q, *k, *v, *o, *post_norm, *gate, *up, *down;
};

template <typename T>
bool run_decoder(const TensorPagedKVDecodeRequest *rq, const Dims &D, WF fmt, PkvPool *pool,
                 const PkvBatch &batch, size_t current, Context &c) {
    const cudaStream_t s = c.stream;
    const size_t es = sizeof(T);
    // ---- weights (device copies keyed by host pointer) ----
    std::vector<DevLayer> L(D.layers);
    for (size_t l = 0; l < D.layers; ++l) {
        const void *in_norm, *post_norm, *q, *k, *v, *o, *g, *u, *d;
        if (rq->storage == TENSOR_PAGED_KV_F32) {
            const auto &h = static_cast<const TensorAttentionDecoderLayer *>(rq->layers)[l];
            in_norm = h.input_norm; post_norm = h.post_norm; q = h.q_weight; k = h.k_weight;
            v = h.v_weight; o = h.o_weight; g = h.gate_weight; u = h.up_weight; d = h.down_weight;
        } else if (rq->storage == TENSOR_PAGED_KV_F16) {
            const auto &h = static_cast<const TensorAttentionDecoderLayerF16 *>(rq->layers)[l];
            in_norm = h.input_norm; post_norm = h.post_norm; q = h.q_weight; k = h.k_weight;
            v = h.v_weight; o = h.o_weight; g = h.gate_weight; u = h.up_weight; d = h.down_weight;
        } else {
            const auto &h = static_cast<const TensorAttentionDecoderLayerQuantF16 *>(rq->layers)[l];
            in_norm = h.input_norm; post_norm = h.post_norm; q = h.q_weight; k = h.k_weight;
            v = h.v_weight; o = h.o_weight; g = h.gate_weight; u = h.up_weight; d = h.down_weight;
        }
        if (!in_norm || !post_norm || !q || !k || !v || !o || !g || !u || !d ||
            !rq->key_cache[l] || !rq->value_cache[l])
            return false;
        DevLayer &dl = L[l];
        dl.input_norm = weight(in_norm, D.hidden * es);
        dl.post_norm = weight(post_norm, D.hidden * es);
        dl.q = weight(q, mat_bytes<T>(fmt, D.hidden, D.hidden));
        dl.k = weight(k, mat_bytes<T>(fmt, D.kvw, D.hidden));
        dl.v = weight(v, mat_bytes<T>(fmt, D.kvw, D.hidden));
        dl.o = weight(o, mat_bytes<T>(fmt, D.hidden, D.hidden));
        dl.gate = weight(g, mat_bytes<T>(fmt, D.inter, D.hidden));
        dl.up = weight(u, mat_bytes<T>(fmt, D.inter, D.hidden));
        dl.down = weight(d, mat_bytes<T>(fmt, D.hidden, D.inter));
        if (!dl.input_norm || !dl.post_norm || !dl.q || !dl.k || !dl.v || !dl.o || !dl.gate ||
            !dl.up || !dl.down)
            return false;
    }
    const void *emb = weight(rq->embedding, D.vocab * D.hidden * es);
    const void *fnorm = weight(rq->final_norm, D.hidden * es);
    const void *head = weight(rq->lm_head, mat_bytes<T>(fmt, D.vocab, D.hidden));
    if (!emb || !fnorm || !head) return false;

    // ---- scratch ----
    const size_t qkvw = D.hidden + 2 * D.kvw;
    const size_t sizes[8] = {D.hidden, D.hidden, qkvw, D.hidden, D.hidden, D.hidden, D.hidden,
                             D.inter};  // x (spare) qkv qrot attn r (spare) act
    size_t blk_bytes = 0;
    for (size_t z : sizes) blk_bytes += (z * es + 255) & ~size_t(255);
    // tokens: [count] outputs, current token, visible length, argmax ticket,
    // then the argmax partials of the lm_head CTAs
    const size_t head_words = (D.count + 5 + 63) & ~size_t(63);
    if (!grow(&c.blk, &c.cap_blk, blk_bytes) ||
        !grow(&c.logits, &c.cap_logits, D.vocab * es) ||
        !grow(reinterpret_cast<void **>(&c.tokens), &c.cap_tokens,
              (head_words + 2 * kGemvMaxGrid) * sizeof(uint32_t)))
        return false;
    void *buf[8];
    {
        auto *p = static_cast<unsigned char *>(c.blk);
        for (int i = 0; i < 8; ++i) {
            buf[i] = p;
            p += (sizes[i] * es + 255) & ~size_t(255);
        }
    }
    void *x = buf[0], *qkv = buf[2], *qrot = buf[3], *attn = buf[4], *r = buf[5], *act = buf[7];
    uint32_t *cur = c.tokens + D.count;
    int32_t *seq_len = reinterpret_cast<int32_t *>(c.tokens + D.count + 1);
    unsigned *ticket = c.tokens + D.count + 2;
    int32_t *step = reinterpret_cast<int32_t *>(c.tokens + D.count + 3);
    int32_t *position = reinterpret_cast<int32_t *>(c.tokens + D.count + 4);
    float *part_v = reinterpret_cast<float *>(c.tokens + head_words);
    int *part_i = reinterpret_cast<int *>(c.tokens + head_words + kGemvMaxGrid);
    {
        const int32_t init[3] = {0, 0, (int32_t)D.past};  // ticket, step, position
        if (cudaMemcpyAsync(ticket, init, sizeof(init), cudaMemcpyHostToDevice, s) != cudaSuccess ||
            cudaStreamSynchronize(s) != cudaSuccess)
            return false;
    }

    // ---- layer pools and prefix import ----
    std::vector<PkvPagedLayer> pl(D.layers);
    for (size_t l = 0; l < D.layers; ++l)
        if (!pkv_pool_layer(pool, l, &pl[l])) return false;
    if (current == 0 && D.past > 0) {
        const size_t rows_bytes = D.past * D.kvw * es;
        if (!grow(&c.stage, &c.cap_stage, 2 * rows_bytes)) return false;
        for (size_t l = 0; l < D.layers; ++l) {
            auto *kst = static_cast<unsigned char *>(c.stage);
            if (cudaMemcpyAsync(kst, rq->key_cache[l], rows_bytes, cudaMemcpyHostToDevice, s) !=
                    cudaSuccess ||
                cudaMemcpyAsync(kst + rows_bytes, rq->value_cache[l], rows_bytes,
                                cudaMemcpyHostToDevice, s) != cudaSuccess)
                return false;
            const int64_t count = (int64_t)(D.past * D.kvw);
            int grid = (int)((count + 255) / 256);
            if (grid > 148 * 8) grid = 148 * 8;
            scatter_prefix_kernel<T><<<grid, 256, 0, s>>>(
                reinterpret_cast<const T *>(kst), reinterpret_cast<const T *>(kst + rows_bytes),
                static_cast<T *>(pl[l].key_pool), static_cast<T *>(pl[l].value_pool),
                batch.block_tables, (int)batch.table_stride, (int)pl[l].block_size,
                (uint32_t)pl[l].block_count, (int)D.kvw, count);
        }
    }
    if (cudaMemcpyAsync(cur, &rq->initial_token, sizeof(uint32_t), cudaMemcpyHostToDevice, s) !=
        cudaSuccess)
        return false;

    // ---- attention path ----
    const size_t group = D.qh / D.kvh;
    const bool fast = sizeof(T) == 2 && (D.hd == 64 || D.hd == 128) &&
                      (group == 1 || group == 2 || group == 4 || group == 8 ||
                       (group == 16 && D.hd == 128));
    if (fast) {
        const size_t wsb = pkv_decode_workspace_bytes(1, D.qh, D.hd, D.target, 0);
        if (wsb == 0 || !grow(&c.ws, &c.cap_ws, wsb)) return false;
        if (!pkv_decode_workspace_init(c.ws, c.cap_ws, (PkvStream)s, nullptr, 0)) return false;
    }
    const int splits = (int)((D.target + kAttnChunk - 1) / kAttnChunk);
    if (!grow(reinterpret_cast<void **>(&c.apart), &c.cap_apart,
              D.qh * (size_t)splits * (D.hd + 2) * sizeof(float)))
        return false;

    const float scale = 1.0f / sqrtf((float)D.hd);
    const int hidden = (int)D.hidden, kvw = (int)D.kvw, inter = (int)D.inter;
    // one token: the same launches every step (position and output slot are
    // device-side), so they are captured once and replayed as a CUDA graph
    auto enqueue_token = [&]() -> bool {
        if (!launch_pdl(embed_kernel<T>, dim3((hidden + 255) / 256), dim3(256), 0, s,
                        static_cast<const T *>(emb), (const uint32_t *)cur, static_cast<T *>(x),
                        hidden, (uint32_t)D.vocab))
            return false;
        for (size_t l = 0; l < D.layers; ++l) {
            const DevLayer &w = L[l];
            Gemv g;  // qkv = [Wq; Wk; Wv] . rms(x)
            g.m0 = w.q; g.r0 = hidden; g.m1 = w.k; g.r1 = kvw; g.m2 = w.v; g.r2 = kvw;
            g.in = hidden; g.out = (int)qkvw; g.x = x; g.norm_w = w.input_norm; g.eps = D.eps;
            g.y = qkv;
            if (!run_gemv<T>(fmt, g, s)) return false;
            const int width = hidden > kvw ? hidden : kvw;
            if (!launch_pdl(rope_store_kernel<T>, dim3((width + 255) / 256), dim3(256), 0, s,
                            static_cast<const T *>(qkv), static_cast<T *>(qrot),
                            static_cast<T *>(pl[l].key_pool), static_cast<T *>(pl[l].value_pool),
                            batch.block_tables, (int)batch.table_stride, (int)pl[l].block_size,
                            (uint32_t)pl[l].block_count, hidden, kvw, (int)D.hd,
                            (const int32_t *)position, D.theta, seq_len))
                return false;
            bool done = false;
            if (fast) {
                PkvBatch one = batch;
                one.seq_lens = seq_len;
                one.batch = 1;
                done = pkv_paged_decode(&pl[l], &one, D.qh, qrot, scale, attn, PKV_DTYPE_F16,
                                        D.target, 0, c.ws, c.cap_ws, (PkvStream)s, nullptr,
                                        0) != 0;
            }
            if (!done) {
                if (!launch_pdl(attn_split_kernel<T>, dim3((unsigned)D.qh, (unsigned)splits),
                                dim3(kAttnThreads), 0, s, static_cast<const T *>(qrot),
                                static_cast<const T *>(pl[l].key_pool),
                                static_cast<const T *>(pl[l].value_pool), batch.block_tables,
                                (int)batch.table_stride, (int)pl[l].block_size,
                                (uint32_t)pl[l].block_count, (const int32_t *)seq_len, (int)D.qh,
                                (int)D.kvh, (int)D.hd, scale, c.apart) ||
                    !launch_pdl(attn_merge_kernel<T>, dim3((unsigned)D.qh), dim3(128), 0, s,
                                (const float *)c.apart, splits, (int)D.hd,
                                static_cast<T *>(attn)))
                    return false;
            }
            Gemv o;  // r = Wo . attn + x
            o.m0 = w.o; o.r0 = hidden; o.in = hidden; o.out = hidden; o.x = attn; o.res = x;
            o.y = r; o.epi = kResidual;
            Gemv gu;  // act = silu(Wg . rms(r)) * (Wu . rms(r))
            gu.m0 = w.gate; gu.r0 = inter; gu.m1 = w.up; gu.r1 = inter; gu.in = hidden;
            gu.out = inter; gu.x = r; gu.norm_w = w.post_norm; gu.eps = D.eps; gu.y = act;
            gu.epi = kSwiGLU;
            Gemv dn;  // x = Wd . act + r
            dn.m0 = w.down; dn.r0 = hidden; dn.in = inter; dn.out = hidden; dn.x = act;
            dn.res = r; dn.y = x; dn.epi = kResidual;
            if (!run_gemv<T>(fmt, o, s) || !run_gemv<T>(fmt, gu, s) || !run_gemv<T>(fmt, dn, s))
                return false;
        }
        Gemv hd;  // logits = lm_head . rms(x) * final_norm, then the first argmax
        hd.m0 = head; hd.r0 = (int)D.vocab; hd.in = hidden; hd.out = (int)D.vocab; hd.x = x;
        hd.norm_w = fnorm; hd.eps = D.eps; hd.y = c.logits; hd.epi = kArgmax;
        hd.part_v = part_v; hd.part_i = part_i; hd.ticket = ticket; hd.tokens = c.tokens;
        hd.next_token = cur; hd.step = step; hd.position = position;
        return run_gemv<T>(fmt, hd, s);
    };
    bool graphed = false;
    if (D.count > 1) {
        cudaGraph_t graph = nullptr;
        cudaGraphExec_t exec = nullptr;
        if (cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
            const bool enq = enqueue_token();
            const cudaError_t end = cudaStreamEndCapture(s, &graph);
            if (enq && end == cudaSuccess && graph != nullptr &&
                cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess) {
                graphed = true;
                for (size_t t = 0; graphed && t < D.count; ++t)
                    graphed = cudaGraphLaunch(exec, s) == cudaSuccess;
            }
        }
        if (exec != nullptr) cudaGraphExecDestroy(exec);
        if (graph != nullptr) cudaGraphDestroy(graph);
        cudaGetLastError();  // a failed capture falls back to direct launches
        if (!graphed && cudaStreamSynchronize(s) != cudaSuccess) return false;
    }
    if (!graphed) {
        // direct launches; after a failed replay the step counter tells where to resume
        int32_t done = 0;
        if (D.count > 1 &&
            cudaMemcpy(&done, step, sizeof(done), cudaMemcpyDeviceToHost) != cudaSuccess)
            return false;
        for (size_t t = (size_t)done; t < D.count; ++t)
            if (!enqueue_token()) return false;
    }
    if (cudaGetLastError() != cudaSuccess) return false;
    if (cudaMemcpyAsync(rq->generated_tokens, c.tokens, D.count * sizeof(uint32_t),
                        cudaMemcpyDeviceToHost, s) != cudaSuccess)
        return false;
    return cudaStreamSynchronize(s) == cudaSuccess;
}

bool valid_request(const TensorPagedKVDecodeRequest *r) {
    // attention.c:126-140
    return r != nullptr && r->cache != nullptr && r->sequence != 0 && r->layers != nullptr &&
           r->layer_count != 0 && r->embedding != nullptr && r->generated_tokens != nullptr &&
           r->key_cache != nullptr && r->value_cache != nullptr && r->final_norm != nullptr &&
           r->lm_head != nullptr && r->token_count != 0 && r->hidden_size != 0 &&
           r->intermediate_size != 0 && r->query_heads != 0 && r->kv_heads != 0 &&
           r->head_dim != 0 && r->past_length <= SIZE_MAX - r->token_count &&
           (r->storage == TENSOR_PAGED_KV_F32 || r->storage == TENSOR_PAGED_KV_F16 ||
            r->storage == TENSOR_PAGED_KV_QUANT_F16) &&
           (r->storage != TENSOR_PAGED_KV_QUANT_F16 ||
            r->weight_quantization == TENSOR_WEIGHT_Q4_0 ||
            r->weight_quantization == TENSOR_WEIGHT_Q8_0);
}

// Dimension rules of decode_sequence_impl (attention_cuda.cu:764-790, paged
// checks :801-807), plus the 32-bit index limits of these kernels.
bool valid_dims(const TensorPagedKVDecodeRequest *r, size_t capacity, bool quantized) {
    const size_t h = r->hidden_size, qh = r->query_heads, kvh = r->kv_heads, hd = r->head_dim;
    if (qh > SIZE_MAX / hd || qh * hd != h || qh % kvh != 0 || hd % 2 != 0 || hd > 256 ||
        r->past_length >= capacity || r->token_count > capacity - r->past_length ||
        capacity > INT32_MAX || r->vocabulary_size == 0 || r->vocabulary_size > INT32_MAX ||
        h > INT32_MAX / 4 || r->intermediate_size > INT32_MAX / 4 ||
        r->vocabulary_size > SIZE_MAX / h / 4)
        return false;
    if (kvh > SIZE_MAX / hd) return false;
    const size_t kvw = kvh * hd;
    if (kvw > (size_t)INT32_MAX / 4 || capacity > SIZE_MAX / kvw) return false;
    if (quantized && (h % 32 || r->intermediate_size % 32 || kvw % 32)) return false;
    // GEMV inputs are staged in shared memory
    if (h > (size_t)kGemvMaxIn || r->intermediate_size > (size_t)kGemvMaxIn) return false;
    return true;
}

}  // namespace
}  // namespace pkv

extern "C" {

int pkv_internal_take_sequence_fault(uint32_t *code) {
    uint32_t zero = 0;
    if (cudaMemcpyFromSymbol(code, pkv::g_sequence_fault, sizeof(uint32_t)) != cudaSuccess)
        return 0;
    return cudaMemcpyToSymbol(pkv::g_sequence_fault, &zero, sizeof(uint32_t)) == cudaSuccess;
}

int tensor_attention_decode_sequence_paged(const TensorPagedKVDecodeRequest *request) {
    PKV_RANGE("tensor_attention_decode_sequence_paged");
    using namespace pkv;
    if (!valid_request(request)) return 0;
    TensorPagedKVCache *cache = request->cache;
    const size_t bs = tensor_paged_kv_cache_block_size(cache);
    const size_t bc = tensor_paged_kv_cache_block_count(cache);
    if (bs == 0 || bc == 0 || bc > SIZE_MAX / bs) return 0;
    const size_t capacity = bs * bc;
    const bool quantized = request->storage == TENSOR_PAGED_KV_QUANT_F16;
    std::lock_guard<std::mutex> lock(g_mutex);
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    // The SDK checks dimensions inside its backend, after the reservation,
    // and rolls back; checking first leaves the cache untouched the same way.
    if (!valid_dims(request, capacity, quantized)) return 0;
    Dims D;
    D.hidden = request->hidden_size;
    D.inter = request->intermediate_size;
    D.qh = request->query_heads;
    D.kvh = request->kv_heads;
    D.hd = request->head_dim;
    D.kvw = D.kvh * D.hd;
    D.vocab = request->vocabulary_size;
    D.layers = request->layer_count;
    D.past = request->past_length;
    D.count = request->token_count;
    D.target = D.past + D.count;
    D.eps = request->rms_norm_epsilon;
    D.theta = (float)request->rope_theta;
    const PkvDType dtype = request->storage == TENSOR_PAGED_KV_F32 ? PKV_DTYPE_F32 : PKV_DTYPE_F16;

    // the cache's pool: created on first use, then it must match
    PkvPool *pool = pkv_pool_from_cache(cache);
    if (pool == nullptr) {
        if (!pkv_pool_create(cache, dev, dtype, D.layers, D.kvh, D.hd, 1, bc, &pool, nullptr, 0))
            return 0;
    }
    PkvPagedLayer l0;
    if (!pkv_pool_layer(pool, 0, &l0) || l0.dtype != dtype || l0.kv_heads != D.kvh ||
        l0.head_dim != D.hd || !pkv_pool_layer(pool, D.layers - 1, &l0) ||
        pkv_pool_layer(pool, D.layers, &l0))
        return 0;
    Context *c = nullptr;
    try {  // the first call on a device adds its context (a host allocation)
        c = context_for_device(dev);
    } catch (...) {
        c = nullptr;
    }
    if (c == nullptr) return 0;
    size_t current = 0;
    if (!tensor_paged_kv_sequence_length(cache, request->sequence, &current)) return 0;
    const TensorPagedKVSequence seq = request->sequence;
    // begin_decode, length check (0 or past), reserve(past + count), table upload
    if (!pkv_step_begin(pool, &seq, &D.past, &D.count, 1, (PkvStream)c->stream, nullptr, 0))
        return 0;
    PkvBatch batch;
    bool ok = pkv_step_batch(pool, &batch) != 0;
    const WF fmt = !quantized ? WF::Dense
                              : (request->weight_quantization == TENSOR_WEIGHT_Q8_0 ? WF::Q8
                                                                                    : WF::Q4);
    // no C++ exception (a host allocation failing) may leave this C function
    // or skip the rollback below
    if (ok) {
        try {
            ok = request->storage == TENSOR_PAGED_KV_F32
                     ? run_decoder<float>(request, D, fmt, pool, batch, current, *c)
                     : run_decoder<__half>(request, D, fmt, pool, batch, current, *c);
        } catch (...) {
            ok = false;
        }
    }
    if (ok) {
        uint32_t fault = 0;
        ok = pkv_device_fault(dev, &fault, nullptr, 0) && fault == 0;
    }
    if (!ok) cudaStreamSynchronize(c->stream);
    // set_length(target) and end_decode, or the rollback to the old length
    if (!pkv_step_end(pool, ok ? 1 : 0, nullptr, 0)) ok = false;
    return ok ? 1 : 0;
}

void tensor_attention_decode_cache_clear(void) {
    using namespace pkv;
    std::lock_guard<std::mutex> lock(g_mutex);
    for (auto &kv : g_weights)
        if (kv.second.ptr != nullptr) cudaFree(kv.second.ptr);
    g_weights.clear();
    for (auto &kv : g_contexts) free_context(kv.second);
    g_contexts.clear();
}

}  // extern "C"
