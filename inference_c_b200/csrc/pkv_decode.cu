// pkv_decode.cu -- paged decode SDPA for sm_100a (one query token per sequence).
//
// Work unit = (sequence b, KV head g, chunk c of `chunk` positions).  A
// persistent grid of 256-thread CTAs strides over the units.  Per unit:
//   * the G = q_heads/kv_heads query heads of KV head g are held in registers
//     (pre-scaled by scale*log2(e) so the softmax uses exp2);
//   * 64-token tiles of K and V for head g are staged through a 3-deep
//     cp.async ring straight from the pages named by the block table, so each
//     page byte is read from HBM once for all G heads (GQA sharing);
//   * QK: 16 lanes per token (one 16-byte chunk of the head row each), the G
//     partial dots are reduce-scattered across the 16 lanes with shuffles;
//   * running-max (online) softmax in FP32, one warp per query head;
//   * PV: each thread owns one 16-byte column chunk and accumulates G x 8
//     outputs in FP32 over its token group;
//   * a unit covering a whole sequence writes the output directly; otherwise
//     it writes (m, l, O) partials and the last unit of that (b, g) to finish
//     (atomic ticket after __threadfence) merges all chunks.
// The merge is the split-K combine of the SDK's Metal path
// (attention_kernels.metal:693-875: per-partition max/sum/acc rescaled by
// exp(m_i - m_max)); the result equals softmax(q.K^T * scale) . V as computed
// by tensor_sdpa_f32 (attention.c:212-406) up to FP32 rounding.
#include <math.h>

#include "pkv_device.cuh"
#include "pkv_internal.h"

namespace pkv {
namespace {

__device__ uint32_t g_decode_fault;

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kTile = 64;
constexpr int kStages = 3;
constexpr int kMaxBatch = 8192;
constexpr float kLog2e = 1.4426950408889634f;

struct DecodeArgs {
    const void *kpool;
    const void *vpool;
    const uint32_t *tables;
    const int32_t *seq_lens;
    const void *query;
    void *out;
    uint32_t *counters;  // [batch * kv_heads]
    float *part_ml;      // [batch][kv_heads][max_chunks][G][2]
    float *part_o;       // [batch][kv_heads][max_chunks][G][HD]
    int32_t table_stride;
    int32_t batch;
    int32_t kv_heads;
    int32_t kv_width;
    int32_t block_size;
    int32_t block_shift;
    uint32_t block_count;
    int32_t chunk;
    int32_t max_chunks;
    float scale_log2;
};

template <int HD, int G>
struct Cfg {
    static constexpr int CH = HD / 8;            // 16-byte chunks per head row
    static constexpr int TP = kThreads / CH;     // tokens per QK pass / PV token groups
    static constexpr int PASSES = kTile / TP;
    static constexpr int LOADS = kTile * CH / kThreads;  // cp.async per thread per tile (K, V each)
    static constexpr int GP = G < 4 ? 4 : G;     // padded P row
    static constexpr int STAGE = kTile * HD;     // elements of one K (or V) stage
    static_assert(G <= CH && kThreads % CH == 0 && kTile % TP == 0, "shape");
};

template <int HD, int G>
size_t smem_bytes(int batch) {
    using C = Cfg<HD, G>;
    size_t kv = 2u * kStages * C::STAGE * 2u;
    size_t red = (size_t)kWarps * G * HD * 4u;
    size_t base = kv > red ? kv : red;
    return base + (size_t)kTile * C::GP * 4u + 3u * 8u * 4u + 16u * 4u + ((size_t)batch + 1u) * 4u;
}

template <int HD, int G, typename T, typename OT>
__global__ void __launch_bounds__(kThreads, (G >= 8 ? 1 : 2))
paged_decode_kernel(const DecodeArgs a) {
    using C = Cfg<HD, G>;
    extern __shared__ __align__(128) unsigned char smem[];
    constexpr size_t kKV = 2u * kStages * C::STAGE * sizeof(T);
    constexpr size_t kRed = (size_t)kWarps * G * HD * 4u;
    constexpr size_t kBase = kKV > kRed ? kKV : kRed;
    T *Ks = reinterpret_cast<T *>(smem);
    T *Vs = Ks + kStages * C::STAGE;
    float *red = reinterpret_cast<float *>(smem);  // reused after the tile loop
    float *P = reinterpret_cast<float *>(smem + kBase);
    float *alpha_s = P + kTile * C::GP;
    float *m_s = alpha_s + 8;
    float *l_s = m_s + 8;
    int *misc = reinterpret_cast<int *>(l_s + 8);  // [0]=ticket flag, [8..15]=warp totals
    int *prefix = misc + 16;                       // [batch+1]

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int cq = tid % C::CH;     // this thread's 16-byte chunk of a head row
    const int tq = tid / C::CH;     // this thread's token slot / token group

    // Prefix sums of chunk counts (every sequence has at least one unit so
    // that empty sequences still get their zero output).
    {
        const int per = (a.batch + kThreads - 1) / kThreads;
        int local = 0;
        for (int k = 0; k < per; ++k) {
            const int b = tid * per + k;
            if (b < a.batch) {
                const int L = max(0, __ldg(a.seq_lens + b));
                local += max(1, (L + a.chunk - 1) / a.chunk);
            }
        }
        int incl = local;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        if (lane == 31) misc[8 + warp] = incl;
        __syncthreads();
        int before = 0;
        for (int w = 0; w < warp; ++w) before += misc[8 + w];
        int run = before + incl - local;
        for (int k = 0; k < per; ++k) {
            const int b = tid * per + k;
            if (b < a.batch) {
                prefix[b] = run;
                const int L = max(0, __ldg(a.seq_lens + b));
                run += max(1, (L + a.chunk - 1) / a.chunk);
            }
        }
        if (tid == kThreads - 1) prefix[a.batch] = before + incl;
        __syncthreads();
    }
    const int total_w = prefix[a.batch];
    const int64_t total_units = (int64_t)total_w * a.kv_heads;
    const int q_heads = a.kv_heads * G;

    for (int64_t u = blockIdx.x; u < total_units; u += gridDim.x) {
        const int w = (int)(u / a.kv_heads);
        const int g = (int)(u - (int64_t)w * a.kv_heads);
        int lo = 0, hi = a.batch - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (prefix[mid] <= w) lo = mid; else hi = mid - 1;
        }
        const int b = lo;
        const int c = w - prefix[b];
        const int nchunks = prefix[b + 1] - prefix[b];
        const int L = max(0, __ldg(a.seq_lens + b));
        const int t0 = c * a.chunk;
        const int t1 = min(L, t0 + a.chunk);
        const int ntok = max(0, t1 - t0);
        const int ntiles = (ntok + kTile - 1) / kTile;

        float q[G][8];
        {
            const T *qp = static_cast<const T *>(a.query) +
                          ((int64_t)b * q_heads + (int64_t)g * G) * HD + cq * 8;
#pragma unroll
            for (int h = 0; h < G; ++h) {
                const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(qp + (int64_t)h * HD));
                unpack8<T>(raw, q[h]);
#pragma unroll
                for (int i = 0; i < 8; ++i) q[h][i] *= a.scale_log2;
            }
        }
        float acc[G][8];
#pragma unroll
        for (int h = 0; h < G; ++h)
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[h][i] = 0.f;
        float m_run = -INFINITY, l_run = 0.f;

        PageMap map{a.tables + (int64_t)b * a.table_stride, a.block_size, a.block_shift,
                    a.block_count, a.table_stride};
        const T *kbase = static_cast<const T *>(a.kpool) + (int64_t)g * HD + cq * 8;
        const T *vbase = static_cast<const T *>(a.vpool) + (int64_t)g * HD + cq * 8;

        auto load_tile = [&](int tile, int stage) {
            const int base = t0 + tile * kTile;
#pragma unroll
            for (int r = 0; r < C::LOADS; ++r) {
                const int tok = tq + r * C::TP;
                const int pos = base + tok;
                if (pos < t1) {
                    int64_t row;
                    const uint32_t f = map.row_of(pos, row);
                    if (f != kFaultNone) {
                        record_fault(&g_decode_fault, f);
                    } else {
                        const int64_t off = row * a.kv_width;
                        cp_async16(Ks + stage * C::STAGE + tok * HD + cq * 8, kbase + off);
                        cp_async16(Vs + stage * C::STAGE + tok * HD + cq * 8, vbase + off);
                    }
                }
            }
        };

        __syncthreads();  // previous unit is done with shared memory
#pragma unroll
        for (int s = 0; s < kStages - 1; ++s) {
            if (s < ntiles) load_tile(s, s);
            cp_async_commit();
        }
        for (int tile = 0; tile < ntiles; ++tile) {
            cp_async_wait<kStages - 2>();
            __syncthreads();
            {
                const int nt = tile + kStages - 1;
                if (nt < ntiles) load_tile(nt, nt % kStages);
                cp_async_commit();
            }
            const int stage = tile % kStages;
            const int valid = min(kTile, ntok - tile * kTile);
            const T *Kst = Ks + stage * C::STAGE;
            const T *Vst = Vs + stage * C::STAGE;

            // ---- scores: s[t][h] = sum_d q[h][d] * k[t][d] ----
#pragma unroll
            for (int pass = 0; pass < C::PASSES; ++pass) {
                const int t = pass * C::TP + tq;
                const uint4 raw = *reinterpret_cast<const uint4 *>(Kst + t * HD + cq * 8);
                float k[8];
                unpack8<T>(raw, k);
                float v[G];
#pragma unroll
                for (int h = 0; h < G; ++h) {
                    float s = 0.f;
#pragma unroll
                    for (int i = 0; i < 8; ++i) s = fmaf(q[h][i], k[i], s);
                    v[h] = s;
                }
                // Reduce-scatter the G partial dots over the CH lanes of this
                // token: each level halves the vector, so G values cost
                // G-1 + log2(CH/G) shuffles instead of G*log2(CH).
                int n = G;
#pragma unroll
                for (int m = C::CH / 2; m >= 1; m >>= 1) {
                    if (n > 1) {
                        const int half = n / 2;
                        const bool upper = (cq & m) != 0;
#pragma unroll
                        for (int i = 0; i < half; ++i) {
                            const float keep = upper ? v[i + half] : v[i];
                            const float send = upper ? v[i] : v[i + half];
                            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, m);
                        }
                        n = half;
                    } else {
                        v[0] += __shfl_xor_sync(0xffffffffu, v[0], m);
                    }
                }
                constexpr int DUP = C::CH / G;
                if ((cq & (DUP - 1)) == 0) P[t * C::GP + cq / DUP] = t < valid ? v[0] : -INFINITY;
            }
            __syncthreads();

            // ---- online softmax, one warp per query head ----
            if (warp < G) {
                const float s0 = P[lane * C::GP + warp];
                const float s1 = P[(lane + 32) * C::GP + warp];
                const float m_new = fmaxf(m_run, warp_max(fmaxf(s0, s1)));
                const float alpha = exp2f(m_run - m_new);
                const float p0 = exp2f(s0 - m_new);
                const float p1 = exp2f(s1 - m_new);
                l_run = l_run * alpha + warp_sum(p0 + p1);
                m_run = m_new;
                P[lane * C::GP + warp] = p0;
                P[(lane + 32) * C::GP + warp] = p1;
                if (lane == 0) alpha_s[warp] = alpha;
            }
            __syncthreads();

            // ---- O[h][:] = O[h][:] * alpha[h] + sum_t p[t][h] * v[t][:] ----
#pragma unroll
            for (int h = 0; h < G; ++h) {
                const float al = alpha_s[h];
                if (al != 1.f) {
#pragma unroll
                    for (int i = 0; i < 8; ++i) acc[h][i] *= al;
                }
            }
            for (int t = tq; t < valid; t += C::TP) {
                const uint4 raw = *reinterpret_cast<const uint4 *>(Vst + t * HD + cq * 8);
                float vv[8];
                unpack8<T>(raw, vv);
                float p[C::GP];
                if (C::GP == 4) {
                    const float4 p4 = *reinterpret_cast<const float4 *>(P + t * C::GP);
                    p[0] = p4.x; p[1] = p4.y; p[2] = p4.z; p[3] = p4.w;
                } else {
#pragma unroll
                    for (int h = 0; h < C::GP; h += 4) {
                        const float4 p4 = *reinterpret_cast<const float4 *>(P + t * C::GP + h);
                        p[h] = p4.x; p[h + 1] = p4.y; p[h + 2] = p4.z; p[h + 3] = p4.w;
                    }
                }
#pragma unroll
                for (int h = 0; h < G; ++h)
#pragma unroll
                    for (int i = 0; i < 8; ++i) acc[h][i] = fmaf(p[h], vv[i], acc[h][i]);
            }
        }
        cp_async_wait<0>();
        __syncthreads();  // stages are free; reuse them as the reduction buffer

        // ---- reduce the token groups: lanes first, then warps via smem ----
#pragma unroll
        for (int m = C::CH; m < 32; m <<= 1)
#pragma unroll
            for (int h = 0; h < G; ++h)
#pragma unroll
                for (int i = 0; i < 8; ++i) acc[h][i] += __shfl_xor_sync(0xffffffffu, acc[h][i], m);
        if (lane < C::CH) {
#pragma unroll
            for (int h = 0; h < G; ++h) {
                float4 *dst = reinterpret_cast<float4 *>(red + (warp * G + h) * HD + cq * 8);
                dst[0] = make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
                dst[1] = make_float4(acc[h][4], acc[h][5], acc[h][6], acc[h][7]);
            }
        }
        if (warp < G && lane == 0) {
            m_s[warp] = m_run;
            l_s[warp] = l_run;
        }
        __syncthreads();

        OT *out = static_cast<OT *>(a.out) + ((int64_t)b * q_heads + (int64_t)g * G) * HD;
        const int64_t slot = ((int64_t)b * a.kv_heads + g) * a.max_chunks;
        if (nchunks == 1) {
            for (int idx = tid; idx < G * HD; idx += kThreads) {
                const int h = idx / HD;
                float o = 0.f;
#pragma unroll
                for (int w2 = 0; w2 < kWarps; ++w2) o += red[(w2 * G + h) * HD + (idx - h * HD)];
                const float l = l_s[h];
                out[idx] = from_f32<OT>(l > 0.f ? o / l : 0.f);
            }
            continue;
        }
        if (nchunks > a.max_chunks) {
            if (tid == 0) record_fault(&g_decode_fault, kFaultPositionOutOfRange);
            continue;
        }
        {
            float *po = a.part_o + (slot + c) * G * HD;
            for (int idx = tid; idx < G * HD; idx += kThreads) {
                const int h = idx / HD;
                float o = 0.f;
#pragma unroll
                for (int w2 = 0; w2 < kWarps; ++w2) o += red[(w2 * G + h) * HD + (idx - h * HD)];
                po[idx] = o;
            }
            if (tid < G) {
                float *pm = a.part_ml + ((slot + c) * G + tid) * 2;
                pm[0] = m_s[tid];
                pm[1] = l_s[tid];
            }
        }
        __threadfence();
        __syncthreads();
        if (tid == 0) {
            const uint32_t ticket = atomicAdd(a.counters + (int64_t)b * a.kv_heads + g, 1u);
            misc[0] = ticket == (uint32_t)(nchunks - 1);
        }
        __syncthreads();
        if (misc[0]) {
            __threadfence();
            if (tid < G) {
                float mx = -INFINITY;
                for (int cc = 0; cc < nchunks; ++cc)
                    mx = fmaxf(mx, __ldcg(a.part_ml + ((slot + cc) * G + tid) * 2));
                float l = 0.f;
                for (int cc = 0; cc < nchunks; ++cc) {
                    const float mc = __ldcg(a.part_ml + ((slot + cc) * G + tid) * 2);
                    const float lc = __ldcg(a.part_ml + ((slot + cc) * G + tid) * 2 + 1);
                    if (mc != -INFINITY) l += lc * exp2f(mc - mx);
                }
                m_s[tid] = mx;
                l_s[tid] = l;
            }
            __syncthreads();
            for (int idx = tid; idx < G * HD; idx += kThreads) {
                const int h = idx / HD;
                const float mx = m_s[h];
                float o = 0.f;
                for (int cc = 0; cc < nchunks; ++cc) {
                    const float mc = __ldcg(a.part_ml + ((slot + cc) * G + h) * 2);
                    if (mc != -INFINITY)
                        o += __ldcg(a.part_o + (slot + cc) * G * HD + idx) * exp2f(mc - mx);
                }
                const float l = l_s[h];
                out[idx] = from_f32<OT>(l > 0.f ? o / l : 0.f);
            }
            if (tid == 0) a.counters[(int64_t)b * a.kv_heads + g] = 0u;
        }
    }
}

int g_sm_count[64];

int sm_count() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (g_sm_count[dev] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        g_sm_count[dev] = n > 0 ? n : 148;
    }
    return g_sm_count[dev];
}

size_t round_up(size_t v, size_t m) { return (v + m - 1) / m * m; }

struct WsLayout {
    size_t counters, ml, o, total;
};

WsLayout ws_layout(size_t batch, size_t q_heads, size_t kv_heads, size_t head_dim,
                   size_t max_chunks) {
    WsLayout w;
    w.counters = 0;
    w.ml = round_up(batch * kv_heads * sizeof(uint32_t), 256);
    w.o = w.ml + round_up(batch * q_heads * max_chunks * 2 * sizeof(float), 256);
    w.total = w.o + round_up(batch * q_heads * max_chunks * head_dim * sizeof(float), 256);
    return w;
}

size_t pick_chunk(size_t chunk_tokens) {
    size_t c = chunk_tokens == 0 ? 256 : chunk_tokens;
    return round_up(c, kTile);
}

template <int HD, int G, typename T, typename OT>
int launch_decode(const DecodeArgs &args, cudaStream_t stream) {
    auto kern = paged_decode_kernel<HD, G, T, OT>;
    const size_t smem = smem_bytes<HD, G>(args.batch);
    static int configured[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem_bytes<HD, G>(kMaxBatch)) != cudaSuccess)
            return 0;
        configured[dev] = 1;
    }
    const int per_sm = G >= 8 ? 1 : 2;
    kern<<<sm_count() * per_sm, kThreads, smem, stream>>>(args);
    return cudaGetLastError() == cudaSuccess;
}

template <int HD, int G, typename T>
int dispatch_out(const DecodeArgs &args, PkvDType out, cudaStream_t s) {
    if (out == PKV_DTYPE_F32) return launch_decode<HD, G, T, float>(args, s);
    if (out == PKV_DTYPE_F16) return launch_decode<HD, G, T, __half>(args, s);
    return launch_decode<HD, G, T, __nv_bfloat16>(args, s);
}

template <int HD, typename T>
int dispatch_group(const DecodeArgs &args, int group, PkvDType out, cudaStream_t s) {
    switch (group) {
        case 1: return dispatch_out<HD, 1, T>(args, out, s);
        case 2: return dispatch_out<HD, 2, T>(args, out, s);
        case 4: return dispatch_out<HD, 4, T>(args, out, s);
        case 8: return dispatch_out<HD, 8, T>(args, out, s);
        default: return 0;
    }
}

}  // namespace
}  // namespace pkv

extern "C" {

size_t pkv_decode_workspace_bytes(size_t batch, size_t q_heads, size_t head_dim,
                                  size_t max_seq_len, size_t chunk_tokens) {
    const size_t chunk = pkv::pick_chunk(chunk_tokens);
    const size_t max_chunks = max_seq_len / chunk + 1;
    // kv_heads only sizes the ticket counters; q_heads bounds it.
    return pkv::ws_layout(batch, q_heads, q_heads, head_dim, max_chunks).total;
}

int pkv_decode_workspace_init(void *workspace, size_t workspace_bytes, PkvStream stream,
                              char *error, size_t error_capacity) {
    if (workspace == nullptr && workspace_bytes != 0) {
        pkv_internal_set_error(error, error_capacity, "pkv_decode_workspace_init: null workspace");
        return 0;
    }
    if (workspace_bytes == 0) return 1;
    const cudaError_t st = cudaMemsetAsync(workspace, 0, workspace_bytes, (cudaStream_t)stream);
    if (st != cudaSuccess) {
        pkv_internal_set_error(error, error_capacity, "pkv_decode_workspace_init: %s",
                               cudaGetErrorString(st));
        return 0;
    }
    return 1;
}

int pkv_paged_decode(const PkvPagedLayer *layer, const PkvBatch *batch, size_t q_heads,
                     const void *query, float scale, void *output, PkvDType output_dtype,
                     size_t max_seq_len, size_t chunk_tokens, void *workspace,
                     size_t workspace_bytes, PkvStream stream, char *error,
                     size_t error_capacity) {
    const char *what = "pkv_paged_decode";
    if (layer == nullptr || batch == nullptr || query == nullptr || output == nullptr ||
        layer->key_pool == nullptr || layer->value_pool == nullptr ||
        batch->block_tables == nullptr || batch->seq_lens == nullptr) {
        pkv_internal_set_error(error, error_capacity, "%s: null argument", what);
        return 0;
    }
    if (layer->dtype != PKV_DTYPE_F16 && layer->dtype != PKV_DTYPE_BF16) {
        pkv_internal_set_error(error, error_capacity, "%s: pool dtype must be F16 or BF16", what);
        return 0;
    }
    if (output_dtype != PKV_DTYPE_F32 && output_dtype != layer->dtype) {
        pkv_internal_set_error(error, error_capacity,
                               "%s: output dtype must be F32 or the pool dtype", what);
        return 0;
    }
    const size_t hd = layer->head_dim, kvh = layer->kv_heads;
    if ((hd != 64 && hd != 128) || kvh == 0 || q_heads == 0 || q_heads % kvh != 0) {
        pkv_internal_set_error(error, error_capacity,
                               "%s: head_dim must be 64 or 128 and q_heads a multiple of kv_heads",
                               what);
        return 0;
    }
    const size_t group = q_heads / kvh;
    if (group != 1 && group != 2 && group != 4 && group != 8) {
        pkv_internal_set_error(error, error_capacity,
                               "%s: q_heads/kv_heads must be 1, 2, 4 or 8 (got %zu)", what, group);
        return 0;
    }
    if (batch->batch == 0 || batch->batch > (size_t)pkv::kMaxBatch || batch->table_stride == 0 ||
        batch->table_stride > INT32_MAX || layer->block_size == 0 ||
        layer->block_size > INT32_MAX || layer->block_count == 0 ||
        layer->block_count > UINT32_MAX || !isfinite(scale) || max_seq_len > INT32_MAX / 2) {
        pkv_internal_set_error(error, error_capacity,
                               "%s: invalid batch (1..%d), table, block or scale", what,
                               pkv::kMaxBatch);
        return 0;
    }
    if (((uintptr_t)layer->key_pool | (uintptr_t)layer->value_pool | (uintptr_t)query) % 16 != 0) {
        pkv_internal_set_error(error, error_capacity, "%s: buffers must be 16-byte aligned", what);
        return 0;
    }
    const size_t chunk = pkv::pick_chunk(chunk_tokens);
    const size_t max_chunks = max_seq_len / chunk + 1;
    const pkv::WsLayout ws = pkv::ws_layout(batch->batch, q_heads, kvh, hd, max_chunks);
    if (workspace == nullptr || workspace_bytes < ws.total || ((uintptr_t)workspace % 256) != 0) {
        pkv_internal_set_error(error, error_capacity,
                               "%s: workspace needs %zu bytes, 256-byte aligned (got %zu)", what,
                               ws.total, workspace_bytes);
        return 0;
    }
    pkv::DecodeArgs a;
    a.kpool = layer->key_pool;
    a.vpool = layer->value_pool;
    a.tables = batch->block_tables;
    a.seq_lens = batch->seq_lens;
    a.query = query;
    a.out = output;
    auto *wsb = static_cast<unsigned char *>(workspace);
    a.counters = reinterpret_cast<uint32_t *>(wsb + ws.counters);
    a.part_ml = reinterpret_cast<float *>(wsb + ws.ml);
    a.part_o = reinterpret_cast<float *>(wsb + ws.o);
    a.table_stride = (int32_t)batch->table_stride;
    a.batch = (int32_t)batch->batch;
    a.kv_heads = (int32_t)kvh;
    a.kv_width = (int32_t)(kvh * hd);
    a.block_size = (int32_t)layer->block_size;
    a.block_shift = -1;
    if ((layer->block_size & (layer->block_size - 1)) == 0) {
        int s = 0;
        while ((size_t(1) << s) < layer->block_size) ++s;
        a.block_shift = s;
    }
    a.block_count = (uint32_t)layer->block_count;
    a.chunk = (int32_t)chunk;
    a.max_chunks = (int32_t)max_chunks;
    a.scale_log2 = scale * pkv::kLog2e;
    const cudaStream_t s = (cudaStream_t)stream;
    int ok;
    if (layer->dtype == PKV_DTYPE_F16)
        ok = hd == 128 ? pkv::dispatch_group<128, __half>(a, (int)group, output_dtype, s)
                       : pkv::dispatch_group<64, __half>(a, (int)group, output_dtype, s);
    else
        ok = hd == 128 ? pkv::dispatch_group<128, __nv_bfloat16>(a, (int)group, output_dtype, s)
                       : pkv::dispatch_group<64, __nv_bfloat16>(a, (int)group, output_dtype, s);
    if (!ok) {
        pkv_internal_set_error(error, error_capacity, "%s: launch failed: %s", what,
                               cudaGetErrorString(cudaGetLastError()));
        return 0;
    }
    return 1;
}

int pkv_internal_take_decode_fault(uint32_t *code) {
    uint32_t zero = 0;
    if (cudaMemcpyFromSymbol(code, pkv::g_decode_fault, sizeof(uint32_t)) != cudaSuccess) return 0;
    return cudaMemcpyToSymbol(pkv::g_decode_fault, &zero, sizeof(uint32_t)) == cudaSuccess;
}

}  // extern "C"
