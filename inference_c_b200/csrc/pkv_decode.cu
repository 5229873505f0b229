// pkv_decode.cu -- paged decode SDPA for sm_100a (one query token per sequence).
//
// Two kernels behind pkv_paged_decode:
//
// paged_decode_tc_kernel (head_dim 128, pages of 16-128 tokens): tensor cores.
//   One persistent 224-thread CTA per SM: a K producer warp and a V producer
//   warp (TMA: the query rows of a GQA group and, per 128-token tile, every
//   page of the tile straight from the pool through the block table, 128-byte
//   swizzle), one thread issuing tcgen05.mma and a 4-warp softmax/merge group.
//   Per tile:  S^T[128 tok][16] = K . Q^T  and  O^T[128 d][16] += V^T . P^T,
//   FP32 accumulators in TMEM (M = tokens or dims, N = the query heads of the
//   KV head padded to 16), so each page byte is read from HBM once for all
//   its query heads.  P is written as a 16-bit high half plus the low
//   remainder in the otherwise-zero rows of the N=16 operand (one MMA, ~22
//   bits of P).  Work split is stream-K: the tiles of all (sequence, KV head)
//   segments form one stream, cut evenly across the CTAs up to a dynamic
//   tail (long launches only) of smaller units that CTAs claim with an
//   atomic as they finish; a segment cut between units leaves FP32 partials
//   (m, l, O) that the last CTA to finish a piece merges (atomic ticket), or,
//   with few segments cut into many pieces, the separate pkv_tc_merge_kernel.
//
// paged_decode_simt_kernel (head_dim 64 or 128, any page size): CUDA cores.
//   Work unit = (sequence b, KV head g, chunk c of `chunk` positions); a
//   persistent grid of 256-thread CTAs strides over the units.  The G query
//   heads of KV head g are held in registers (pre-scaled by scale*log2(e));
//   64-token tiles of K and V stream through a 3-deep cp.async ring straight
//   from the pages; 16 lanes per token for QK with shuffle reductions,
//   running-max softmax in FP32, PV accumulated per 16-byte column chunk; a
//   unit covering a whole sequence writes the output, otherwise it writes
//   (m, l, O) partials and the last unit of (b, g) to finish merges them.
//
// The merges are the split-K combine of the SDK's Metal path
// (attention_kernels.metal:693-875: per-partition max/sum/acc rescaled by
// exp(m_i - m_max)); the result equals softmax(q.K^T * scale) . V as computed
// by tensor_sdpa_f32 (attention.c:212-406) up to FP32 rounding.
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <cudaTypedefs.h>

#include <mutex>

#include "pkv_device.cuh"
#include "pkv_internal.h"
#include "pkv_trace.h"
#include "pkv_sm100.cuh"

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
paged_decode_simt_kernel(const DecodeArgs a) {
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
        __syncthreads();
        if (tid == 0) {
            __threadfence();  // publishes the whole block's partials (bar.sync is cumulative)
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

size_t round_up(size_t v, size_t m) { return (v + m - 1) / m * m; }

// ---------------------------------------------------------------------------
// tcgen05 path (head_dim 128, page sizes 16/32/64/128, q_heads/kv_heads <= 16)
//
// One persistent CTA per SM, 224 threads, warp-specialised:
//   warp 0     K producer: TMA-loads the piece's query rows (the B operand)
//              and the K rows of every page of a 128-token tile straight
//              from the pool (one 2-D box per page and 64-column half: no
//              gather copy); warp 6 does the same for V.  3 stage slots of
//              K 32 KiB + V 32 KiB; K and V slots have their own barriers, so
//              a K slot refills as soon as its QK^T ran;
//   warp 1     one thread issues tcgen05.mma, the S of tile j before the PV
//              of tile j-1:
//                S^T[128 tok][16] = K[128 tok][128] . Q^T         (TMEM, f32)
//                O^T[128 d][PN]  = V^T[128 d][128 tok] . P^T       (TMEM, f32)
//              M = 128 tokens / dims, N = the query heads of the GQA group
//              (zero-padded), so each page byte feeds every head once;
//   warps 2-5  softmax / merge group: thread i owns token i of S^T (and dim i
//              of O^T); per tile it takes the block-wide running max per head,
//              writes P = exp2(s - m) to shared memory, zeroes V rows past the
//              length, and folds the previous tile's O into FP32 registers with
//              the running-max correction (one tile late, so the PV round trip
//              overlaps the next tile's softmax).
// P is written as two storage-dtype halves, hi = round(p) in B rows [0, G)
// and lo = round(p - hi) in rows [PN/2, PN/2 + G), so the one PV MMA returns
// O_hi and O_lo side by side and their sum carries ~22 bits of P (a single
// FP16 P costs ~1% relative error on small outputs).
//
// Work split ("stream-K"): the 128-token tiles of every (sequence, KV head)
// segment, sequence-major, form one stream of T tiles, cut into work units of
// consecutive tiles.  Static units: unit i < n (one per CTA) is tiles
// [S*i/n, S*(i+1)/n) of the static region [0, S), so every CTA streams the
// same number of bytes whatever the length mix.  SMs do not stream at the same
// rate (a few percent apart, differently in every launch), so with the
// dynamic tail the last T - S tiles form rounds of n units each, unit sizes
// halving from about an eighth of a CTA's share, and a CTA that finishes its
// static unit claims the next unit with one atomic: the CTAs then finish
// within about one small unit of one another instead of spreading over the
// rate differences.  A segment inside one unit is finished there; a segment
// cut by unit ends leaves one partial (m, l, O) per piece, in slot 0 (the
// unit's first piece) or slot 1 (its last piece).  The last CTA to finish a
// piece of such a segment merges them (atomic ticket), unless one segment can
// span more than kInKernelMergeMax units (few KV heads, one long sequence);
// then there is no dynamic tail and pkv_tc_merge_kernel, one CTA per
// (sequence, query head), merges after the decode kernel.
// ---------------------------------------------------------------------------
constexpr int kTcThreads = 224;
constexpr int kTcTile = 128;
constexpr int kTcStages = 3;
constexpr int kTcMaxBatch = 1024;
constexpr int kTcMaxGrid = 256;
constexpr int kInKernelMergeMax = 32;
constexpr int kMaxRounds = 5;                               // dynamic rounds
constexpr int kTcMaxUnits = kTcMaxGrid * (1 + kMaxRounds);  // work units of one launch
constexpr int kRing = 4;  // unit ids in flight from the K producer to the other roles
constexpr size_t kMinUnitTiles = 8;  // smallest dynamic unit
constexpr uint32_t kTcStageBytes = 65536;
constexpr uint32_t kTcHalf = 16384;       // 128 rows x 128 bytes
constexpr uint32_t kTcQOff = kTcStages * kTcStageBytes;
constexpr uint32_t kTcPOff = kTcQOff + 2 * 4096;
constexpr uint32_t kTcPBuf = 8192;        // one P^T tile of up to 32 rows
constexpr uint32_t kTcBarOff = kTcPOff + 2 * kTcPBuf;
constexpr uint32_t kTcMiscOff = kTcBarOff + 512;  // 34 barriers, the unit ring, the schedule
constexpr uint32_t kTcPrefixOff = kTcMiscOff + 5120;
constexpr uint32_t kTcTmemCols = 128;

size_t tc_smem_bytes(int batch) { return kTcPrefixOff + 4u * ((size_t)batch + 1u) + 1024u; }
static_assert(kTcPrefixOff + 4u * (kTcMaxBatch + 1u) + 1024u <= 232448u, "shared memory budget");
static_assert(64 + 512 + 256 + 2 * 4 * 16 * kInKernelMergeMax + 4 * kInKernelMergeMax <= 5120,
              "misc area");

struct TcArgs {
    const uint32_t *tables;
    const int32_t *seq_lens;
    const void *query;
    void *out;
    uint32_t *counters;     // [kTcMaxUnits] tickets of the in-kernel merge, by first unit
    uint32_t *claim;        // [2]: next dynamic unit, CTAs done claiming (zero between launches)
    float *part_ml;         // [units][2 slots][GV heads][m, l]
    float *part_o;          // [units][2 slots][GV heads][128]
    int32_t *tile_prefix;   // [batch + 1] copy of the tile prefix for the merge kernel
    int32_t table_stride;
    int32_t batch;
    int32_t kv_heads;
    int32_t block_size;
    uint32_t block_count;
    float scale_log2;
    int32_t merge_in_kernel;
    int32_t q_row0;         // query row (sequence * q_heads) of this launch's first sequence
    // head_dim 64: two KV heads (2g, 2g+1) form one 128-column segment g.
    // Query heads h < pair_split of a segment use its dims 0-63, the others
    // dims 64-127; outputs are rows of 64.  0: head_dim 128, rows of 128.
    int32_t pair_split;
    // dynamic tail: smallest unit (tiles; bounds the pieces of one segment),
    // 0 = static units only
    int32_t min_unit;
    // Fused append (pkv_paged_decode_append), else null: this step's new
    // K/V row of every sequence ([batch][row_vecs] uint4), stored at
    // position seq_lens[b] - 1 of the pools (same rows, as uint4) by the
    // producer that loads the tile holding it, before that tile's TMA.
    const uint4 *new_k, *new_v;
    uint4 *kpool, *vpool;
    int32_t row_vecs;  // uint4 per pool row (kv_heads * head_dim / 8)
};

// Tensor maps of one launch: K and V pools (one page x 64 columns per box)
// and the query rows (G heads x 64 columns per box).
struct TcMaps {
    CUtensorMap k, v, q;
};

struct TcWorkspace {
    size_t claim, counters, prefix, ml, o, total;
};

// Scratch of one launch.  The claim words and the merge tickets (zero between
// launches) sit at fixed offsets whatever the batch, so a workspace may serve
// calls of any batch and head count it is large enough for; the partials of
// `units` work units of `heads` query heads follow and need no zeroing.
TcWorkspace tc_workspace(size_t units, size_t heads) {
    TcWorkspace w;
    w.claim = 0;
    w.counters = 256;
    w.prefix = w.counters + round_up((size_t)kTcMaxUnits * sizeof(uint32_t), 256);
    w.ml = w.prefix + round_up(((size_t)kTcMaxBatch + 1) * sizeof(int32_t), 256);
    w.o = w.ml + round_up(units * 2 * heads * 2 * sizeof(float), 256);
    w.total = w.o + round_up(units * 2 * heads * 128 * sizeof(float), 256);
    return w;
}

// Work units of one launch; every CTA (and the merge kernel) derives the same
// schedule from T, the grid and the smallest unit.
struct Sched {
    int64_t T, S;  // tiles; static region [0, S)
    int n;         // working CTAs = static units
    int rounds;    // dynamic rounds of n units each
    int size[kMaxRounds];
};

// Written in place (shared memory in the decode kernel: no local copy).
__host__ __device__ inline void make_sched(Sched &s, int64_t T, int grid, int min_unit) {
    s.T = T;
    s.n = (int)(T < (int64_t)grid ? (T > 1 ? T : 1) : grid);
    s.rounds = 0;
    int64_t dyn = 0;
    // an eighth of a CTA's share first, halving down to min_unit: the
    // dynamic tiles stay under a quarter of T, every unit >= min_unit
    int64_t sz = T / ((int64_t)s.n * 8);
    if (min_unit > 0 && sz >= min_unit) {
        while (s.rounds < kMaxRounds) {
            const int64_t cur = sz > min_unit ? sz : min_unit;
            s.size[s.rounds++] = (int)cur;
            dyn += cur * s.n;
            if (cur == min_unit) break;
            sz >>= 1;
        }
    }
    s.S = T - dyn;
}

__host__ __device__ inline int sched_units(const Sched &s) { return s.n * (1 + s.rounds); }

// First tile of unit u (T for u == sched_units).
__device__ __forceinline__ int64_t unit_start(const Sched &s, int u) {
    if (u < s.n) return s.S * u / s.n;
    int64_t off = s.S;
    int k = u - s.n;
    for (int r = 0; r < s.rounds; ++r) {
        if (k < s.n) return off + (int64_t)k * s.size[r];
        off += (int64_t)s.n * s.size[r];
        k -= s.n;
    }
    return s.T;
}

// The unit that holds tile t.
__device__ __forceinline__ int unit_of_tile(const Sched &s, int64_t t) {
    if (t < s.S) return (int)(((t + 1) * s.n - 1) / s.S);
    int64_t off = t - s.S;
    int u = s.n;
    for (int r = 0; r < s.rounds; ++r) {
        const int64_t span = (int64_t)s.n * s.size[r];
        if (off < span) return u + (int)(off / s.size[r]);
        off -= span;
        u += s.n;
    }
    return u;
}

// Partial slot a unit used for the piece of the segment starting at tile `seg`.
__device__ __forceinline__ int unit_slot(const Sched &s, int u, int64_t seg) {
    return unit_start(s, u) < seg ? 1 : 0;
}

// Exclusive prefix of tiles per sequence times kv_heads (0 for empty ones).
__device__ void build_tile_prefix(const TcArgs &a, int *prefix, int *scratch) {
    const int tid = threadIdx.x, nthr = blockDim.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int per = (a.batch + nthr - 1) / nthr;
    int local = 0;
    for (int k = 0; k < per; ++k) {
        const int b = tid * per + k;
        if (b < a.batch)
            local += (max(0, __ldg(a.seq_lens + b)) + kTcTile - 1) / kTcTile * a.kv_heads;
    }
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) scratch[warp] = incl;
    __syncthreads();
    int before = 0;
    for (int w = 0; w < warp; ++w) before += scratch[w];
    int run = before + incl - local;
    for (int k = 0; k < per; ++k) {
        const int b = tid * per + k;
        if (b < a.batch) {
            prefix[b] = run;
            run += (max(0, __ldg(a.seq_lens + b)) + kTcTile - 1) / kTcTile * a.kv_heads;
        }
    }
    if (tid == nthr - 1) prefix[a.batch] = before + incl;
}

// One contiguous run of tiles of one (sequence, KV head) segment.
struct Piece {
    int b, g, k0, k1, nt;
    int64_t seg;  // stream index of the segment's first tile
};

__device__ __forceinline__ Piece piece_at(int64_t t, int64_t end, const int *prefix,
                                          const TcArgs &a) {
    Piece P;
    int lo = 0, hi = a.batch - 1;  // last sequence whose first tile is <= t
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (prefix[mid] <= t) lo = mid; else hi = mid - 1;
    }
    P.b = lo;
    P.nt = (prefix[lo + 1] - prefix[lo]) / a.kv_heads;
    const int64_t within = t - prefix[lo];
    P.g = (int)(within / P.nt);
    P.k0 = (int)(within - (int64_t)P.g * P.nt);
    P.seg = prefix[lo] + (int64_t)P.g * P.nt;
    P.k1 = (int)min((int64_t)P.nt, (int64_t)P.k0 + (end - t));
    return P;
}

template <typename T>
struct IsBf16 { static constexpr bool value = false; };
template <>
struct IsBf16<__nv_bfloat16> { static constexpr bool value = true; };

// Merges the partials of heads [h0, h0 + nh) of segment (b, g) into `out`
// (nh rows of 128); `heads` is the head stride of a partial slot (the GV of
// the decode kernel).  Every piece's (m, l) per head is staged in shared memory
// (`wst`, `lst`: np * nh floats each); one warp per head, lanes over the
// pieces, turns them into weights exp2(m_c - m) / l; then each output float4
// is the weighted sum of the pieces' partial rows: `ps` threads share one
// float4 (pieces c = lane-in-share mod ps, summed through `red`,
// ps * nh * 32 float4s), each keeping up to 16 loads in flight.  `tid`/`nthr`
// are the participating threads (whole warps); `sync` is their barrier.
template <typename OT, typename Sync>
__device__ __forceinline__ void merge_segment(const TcArgs &a, int h0, int nh, int heads,
                                              int64_t seg, int nt, const Sched &sc, int tid,
                                              int nthr, int ps, float *wst, float *lst, int *slot,
                                              float4 *red, int cap, OT *out, Sync sync) {
    const int first = unit_of_tile(sc, seg);
    const int np = unit_of_tile(sc, seg + nt - 1) - first + 1;
    if (np > cap) {  // cannot happen with the host's choice of merge mode and unit sizes
        if (tid == 0) record_fault(&g_decode_fault, kFaultPositionOutOfRange);
        return;
    }
    for (int c = tid; c < np; c += nthr) slot[c] = unit_slot(sc, first + c, seg);
    sync();
    for (int i = tid; i < np * nh; i += nthr) {
        const int c = i / nh, h = h0 + (i - c * nh);
        const float2 ml = __ldcg(reinterpret_cast<const float2 *>(
            a.part_ml + (((int64_t)(first + c) * 2 + slot[c]) * heads + h) * 2));
        wst[i] = ml.x;
        lst[i] = ml.y;
    }
    sync();
    // weights: one warp per head, lanes over the pieces
    for (int hh = tid >> 5; hh < nh; hh += nthr >> 5) {
        const int lane = tid & 31;
        float mx = -INFINITY;
        for (int c = lane; c < np; c += 32) mx = fmaxf(mx, wst[c * nh + hh]);
        mx = warp_max(mx);
        float lt = 0.f;
        for (int c = lane; c < np; c += 32) {
            const float mc = wst[c * nh + hh];
            const float f = mc == -INFINITY ? 0.f : exp2f(mc - mx);
            lt += lst[c * nh + hh] * f;
            wst[c * nh + hh] = f;
        }
        lt = warp_sum(lt);
        const float inv = lt > 0.f ? 1.f / lt : 0.f;
        for (int c = lane; c < np; c += 32) wst[c * nh + hh] *= inv;
    }
    sync();
    const int nf = nh * 32;  // float4s of output
    for (int base = 0; base < nf * ps; base += nthr) {
        const int w = base + tid;
        const int f4 = w % nf, pl = w / nf;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        if (pl < ps) {
            const int hh = f4 >> 5, d = (f4 & 31) * 4;
            for (int c0 = pl; c0 < np; c0 += 16 * ps) {
                float4 v[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int c = c0 + i * ps;
                    v[i] = c < np ? __ldcg(reinterpret_cast<const float4 *>(
                                        a.part_o + (((int64_t)(first + c) * 2 + slot[c]) * heads +
                                                    h0 + hh) * 128 + d))
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int c = c0 + i * ps;
                    const float f = c < np ? wst[c * nh + hh] : 0.f;
                    acc.x += f * v[i].x;
                    acc.y += f * v[i].y;
                    acc.z += f * v[i].z;
                    acc.w += f * v[i].w;
                }
            }
        }
        if (ps > 1) {
            if (pl < ps) red[w] = acc;
            sync();
            if (pl == 0) {
                for (int k = 1; k < ps; ++k) {
                    const float4 r = red[k * nf + f4];
                    acc.x += r.x;
                    acc.y += r.y;
                    acc.z += r.z;
                    acc.w += r.w;
                }
            }
        }
        const int hh = f4 >> 5, d = (f4 & 31) * 4;
        // paired head_dim 64: each head owns one half of the 128 rows
        const bool owned = a.pair_split == 0 || ((h0 + hh < a.pair_split) == (d < 64));
        if (pl == 0 && owned) {
            OT *o = a.pair_split == 0 ? out + hh * 128 + d : out + hh * 64 + (d & 63);
            o[0] = from_f32<OT>(acc.x);
            o[1] = from_f32<OT>(acc.y);
            o[2] = from_f32<OT>(acc.z);
            o[3] = from_f32<OT>(acc.w);
        }
        if (ps > 1) sync();
    }
    sync();
}

// PAIR (head_dim 64): segment g is KV heads 2g and 2g+1 side by side (128
// pool columns); its GV = 2G query heads sit in S^T columns 0..G-1 (KV head
// 2g, Q rows zero in dims 64-127) and 8..8+G-1 (KV head 2g+1, Q rows zero in
// dims 0-63), so one K . Q^T gives every head its own scores; O^T rows 0-63
// are the dims of KV head 2g, rows 64-127 those of 2g+1.
template <int G, typename T, typename OT, bool PAIR>
__global__ void __launch_bounds__(kTcThreads, 1)
paged_decode_tc_kernel(const TcArgs a, const __grid_constant__ CUtensorMap kmap,
                       const __grid_constant__ CUtensorMap vmap,
                       const __grid_constant__ CUtensorMap qmap) {
    using namespace sm100;
    static_assert(!PAIR || G <= 8, "paired heads need G <= 8");
    constexpr int GV = PAIR ? 2 * G : G;  // query heads of one segment
    constexpr int GN = PAIR ? 16 : (G <= 4 ? 4 : G);  // S^T columns read per thread
    constexpr int PN = GV <= 8 ? 16 : 32;  // P^T rows (= O^T columns): hi and lo halves
    constexpr int OD = PAIR ? 64 : 128;    // output row (head_dim)
    constexpr int LO = PN / 2;
    constexpr uint32_t kPChunk = PN * 128;  // bytes of one 64-token column chunk of P^T
    constexpr uint32_t kIdescQK = idesc_f16(128, 16, IsBf16<T>::value, false, false);
    constexpr uint32_t kIdescPV = idesc_f16(128, PN, IsBf16<T>::value, true, false);
    extern __shared__ unsigned char smem_raw[];
    unsigned char *sm = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + kTcBarOff);
    uint64_t *kfull = bars, *kempty = bars + 3, *s_full = bars + 6, *s_empty = bars + 8;
    uint64_t *p_full = bars + 10, *o_full = bars + 12, *o_empty = bars + 14;
    uint64_t *q_full = bars + 16, *q_empty = bars + 18;
    uint64_t *vfull = bars + 20, *vempty = bars + 23;
    // unit ids from the K producer (which claims them) to the V producer, the
    // MMA thread and the softmax group, in claim order
    uint64_t *ring_full = bars + 26, *ring_empty = bars + 30;
    volatile int *ring = reinterpret_cast<volatile int *>(sm + kTcBarOff + 288);  // kRing ints
    Sched *sched = reinterpret_cast<Sched *>(sm + kTcBarOff + 320);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sm + kTcMiscOff);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(sm + kTcMiscOff + 4);
    int *ticket = reinterpret_cast<int *>(sm + kTcMiscOff + 8);
    volatile int *group_unit = reinterpret_cast<volatile int *>(sm + kTcMiscOff + 12);
    int *scan = reinterpret_cast<int *>(sm + kTcMiscOff + 32);    // 8 ints
    float *red = reinterpret_cast<float *>(sm + kTcMiscOff + 64);  // [2][4][16]
    float *lred = red + 128;                                        // [4][16]
    float *mwst = lred + 64;                                        // kInKernelMergeMax * 16
    float *mlst = mwst + kInKernelMergeMax * 16;                    // kInKernelMergeMax * 16
    int *mslot = reinterpret_cast<int *>(mlst + kInKernelMergeMax * 16);  // kInKernelMergeMax
    int *prefix = reinterpret_cast<int *>(sm + kTcPrefixOff);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < kTcStages; ++s) {
            mbar_init(&kfull[s], 1);
            mbar_init(&kempty[s], 1);
            mbar_init(&vfull[s], 1);
            mbar_init(&vempty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&s_empty[i], 128);
            mbar_init(&p_full[i], 128);
            mbar_init(&o_full[i], 1);
            mbar_init(&o_empty[i], 128);
            mbar_init(&q_full[i], 1);
            mbar_init(&q_empty[i], 1);
        }
        for (int i = 0; i < kRing; ++i) {
            mbar_init(&ring_full[i], 1);
            mbar_init(&ring_empty[i], 3);  // V producer, MMA thread, softmax group
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    // Q and P tiles: rows past the group stay zero for the whole kernel.
    for (int i = tid; i < (int)(2 * 4096 + 2 * kTcPBuf) / 16; i += kTcThreads)
        reinterpret_cast<uint4 *>(sm + kTcQOff)[i] = make_uint4(0, 0, 0, 0);
    if (warp == 1) {
        tmem_alloc(tmem_slot, kTcTmemCols);
        tmem_relinquish();
    }
    if (tid == 0) {
        tma_prefetch_desc(&kmap);
        tma_prefetch_desc(&vmap);
        tma_prefetch_desc(&qmap);
    }
    // The block-table rows of this launch into L2 while the kernel before
    // this one finishes, so the producers' first table reads after the wait
    // hit L2 rather than HBM.  A prefetch leaves no copy in registers or L1:
    // an entry the previous kernel still writes is read later at its new
    // value (L2 holds the one copy every SM sees).
    {
        const size_t bytes = (size_t)a.batch * (size_t)a.table_stride * 4u;
        const char *tb = reinterpret_cast<const char *>(a.tables);
        for (size_t off = ((size_t)blockIdx.x * kTcThreads + tid) * 128u; off < bytes;
             off += (size_t)gridDim.x * kTcThreads * 128u)
            prefetch_l2(tb + off);
    }
    // Everything above touches only this CTA's shared memory and TMEM, so it
    // overlaps the previous kernel under programmatic dependent launch; from
    // here on global memory written by earlier kernels (pages, tables,
    // lengths, queries) is read.
    pdl_wait();
    // Dependents (the next step's staging and append, the merge kernel) may
    // launch now: they start only once every CTA of this grid has run this
    // line, i.e. once all of them are resident, so none can hold an SM a CTA
    // of this grid still needs; each runs griddepcontrol.wait before it
    // touches anything this grid reads or writes, and meanwhile takes the
    // shared memory the CTAs of this grid leave over or free as they finish.
    pdl_launch_dependents();
    build_tile_prefix(a, prefix, scan);
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int64_t total_tiles = prefix[a.batch];
    if (tid == 0) make_sched(*sched, total_tiles, (int)gridDim.x, a.min_unit);
    __syncthreads();
    const Sched &sc = *sched;
    // CTAs past the tile count idle, so every working CTA owns >= 1 tile and
    // the units spanned by a segment are exactly its pieces.
    const bool works = (int)blockIdx.x < sc.n && total_tiles > 0;
    const int n_units = sched_units(sc);
    const int q_heads = a.kv_heads * GV;
    uint32_t *fault = &g_decode_fault;
    if (blockIdx.x == 0 && a.tile_prefix != nullptr)
        for (int b = tid; b <= a.batch; b += kTcThreads) a.tile_prefix[b] = prefix[b];

    // Block-table entries of a piece, 32 pages at a time, one per lane of a
    // producer warp: one load round trip serves the pages of several tiles
    // (four at 16-token pages), and a piece's first window is requested when
    // the piece starts, before its producer waits for a free stage slot.
    // Entries past the table row read as an invalid page id.
    struct TableWindow {
        int first;       // page index held by lane 0
        uint32_t entry;  // page first + lane
    };
    auto window_at = [&](const uint32_t *trow, int first) {
        TableWindow w;
        w.first = first;
        w.entry = first + lane < a.table_stride ? __ldg(trow + first + lane) : 0xffffffffu;
        return w;
    };
    // One tile's pages of one pool (K: warp 0, V: warp 6) into stage slot
    // `dst` (two 64-column halves), completing on `bar`.  Lanes < np each load
    // one page, its id taken from the window `win` (reloaded when the tile's
    // pages leave it).  `pool` non-null (fused append, only for the segment's
    // last tile, whose last page holds position L - 1): lanes 0-15 first
    // store the segment's 256 bytes of the new row, `nrow`, into that page;
    // each fences its store against the async proxy and the warp converges
    // before any lane issues the TMA, so the tile reads the new row.
    auto load_tile = [&](const CUtensorMap *map, uint64_t *bar, unsigned char *dst,
                         const uint32_t *trow, TableWindow &win, int k, int L, int g,
                         uint4 *pool, uint4 nrow) {
        const int ts = k * kTcTile;
        const int te = min(L, ts + kTcTile);
        const int p0 = ts / a.block_size;
        const int np = (te - ts + a.block_size - 1) / a.block_size;  // 1..8
        if (p0 < win.first || p0 + np > win.first + 32) win = window_at(trow, p0);
        const uint32_t e = __shfl_sync(0xffffffffu, win.entry, (p0 - win.first + lane) & 31);
        uint32_t pid = 0;
        bool good = false;
        if (lane < np) {
            if (p0 + lane < a.table_stride) {
                pid = e;
                good = pid < a.block_count;
            }
            if (!good) record_fault(fault, kFaultPageOutOfRange);
        }
        const unsigned mask = __ballot_sync(0xffffffffu, good);
        if (pool != nullptr) {
            const uint32_t lp = __shfl_sync(0xffffffffu, pid, np - 1);
            if (((mask >> (np - 1)) & 1u) != 0 && lane < 16) {
                const int64_t prow = (int64_t)lp * a.block_size + (L - 1) % a.block_size;
                pool[prow * a.row_vecs + g * 16 + lane] = nrow;
                fence_proxy_async_global();
            }
            __syncwarp();
        }
        if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)__popc(mask) * a.block_size * 256u);
        __syncwarp();
        if (good) {
            const uint32_t ro = (uint32_t)lane * a.block_size * 128u;
            const int32_t y = (int32_t)pid * a.block_size;
            tma_load_2d(dst + ro, map, bar, g * 128, y);
            tma_load_2d(dst + kTcHalf + ro, map, bar, g * 128 + 64, y);
        }
    };
    if (warp == 0) {
        // ---------------------------- K producer ----------------------------
        // Also stages each piece's query rows (the B operand of QK^T).
        uint32_t j = 0, qi = 0;
        bool ok = true;
        int u = works ? (int)blockIdx.x : -1;
        for (uint32_t ku = 0;; ++ku) {
            // publish the unit (-1: no more) to the other roles
            const int rs = (int)(ku % kRing);
            if (!mbar_wait(&ring_empty[rs], ((ku / kRing) & 1) ^ 1, abort_flag, fault)) ok = false;
            if (!ok) u = -1;
            if (lane == 0) {
                ring[rs] = u;
                mbar_arrive(&ring_full[rs]);
            }
            __syncwarp();
            if (u < 0) break;
            const int64_t ue = unit_start(sc, u + 1);
        for (int64_t t = unit_start(sc, u); ok && t < ue;) {
            const Piece P = piece_at(t, ue, prefix, a);
            t += P.k1 - P.k0;
            const int L = __ldg(a.seq_lens + P.b);
            // fused append: this piece ends its segment, so it loads the tile
            // holding the new row; fetch the row now, store it at that tile
            const bool app = a.new_k != nullptr && P.k1 == P.nt;
            uint4 nrow = make_uint4(0, 0, 0, 0);
            if (app && lane < 16)
                nrow = __ldg(a.new_k + (int64_t)P.b * a.row_vecs + P.g * 16 + lane);
            const uint32_t *trow = a.tables + (int64_t)P.b * a.table_stride;
            TableWindow win = window_at(trow, P.k0 * kTcTile / a.block_size);
            if (!mbar_wait(&q_empty[qi & 1], ((qi >> 1) & 1) ^ 1, abort_flag, fault)) {
                ok = false;
                break;
            }
            if (lane == 0) {  // G query rows, two 64-column halves, 128-byte swizzle
                unsigned char *qb = sm + kTcQOff + (qi & 1) * 4096;
                const int32_t qrow = a.q_row0 + P.b * q_heads + P.g * GV;
                mbar_arrive_expect_tx(&q_full[qi & 1], (uint32_t)G * 256u);
                if constexpr (PAIR) {
                    // KV head 2g's rows into dims 0-63 at rows 0.., KV head
                    // 2g+1's into dims 64-127 at rows 8.. (a 1024-byte-aligned
                    // atom); the rest of the tile stays zero
                    tma_load_2d(qb, &qmap, &q_full[qi & 1], 0, qrow);
                    tma_load_2d(qb + 2048 + 1024, &qmap, &q_full[qi & 1], 0, qrow + G);
                } else {
                    tma_load_2d(qb, &qmap, &q_full[qi & 1], 0, qrow);
                    tma_load_2d(qb + 2048, &qmap, &q_full[qi & 1], 64, qrow);
                }
            }
            __syncwarp();
            for (int k = P.k0; k < P.k1; ++k, ++j) {
                const int stage = (int)(j % kTcStages);
                if (!mbar_wait(&kempty[stage], ((j / kTcStages) & 1) ^ 1, abort_flag, fault)) {
                    ok = false;
                    break;
                }
                load_tile(&kmap, &kfull[stage], sm + stage * kTcStageBytes, trow, win, k, L, P.g,
                          app && k == P.nt - 1 ? a.kpool : nullptr, nrow);
            }
            ++qi;
        }
            // claim the next dynamic unit (this CTA's loads of the current one
            // are issued, its last tiles still stream)
            int next = -1;
            if (ok && sc.rounds > 0 && lane == 0) {
                const int c = sc.n + (int)atomicAdd(a.claim, 1u);
                next = c < n_units ? c : -1;
            }
            u = __shfl_sync(0xffffffffu, next, 0);
        }
        // The last CTA done claiming zeroes the claim words for the next launch
        // (every CTA's final claim precedes its count here).
        if (sc.rounds > 0 && works && lane == 0) {
            __threadfence();
            if (atomicAdd(a.claim + 1, 1u) == (uint32_t)sc.n - 1) {
                atomicExch(a.claim, 0u);
                atomicExch(a.claim + 1, 0u);
            }
        }
    } else if (warp == 6) {
        // ---------------------------- V producer ----------------------------
        // V slots free later than K slots (after the PV, not the QK^T), so the
        // two rings run on their own barriers and K loads can run ahead.
        uint32_t j = 0;
        bool ok = true;
        for (uint32_t ku = 0; ok; ++ku) {
            const int rs = (int)(ku % kRing);
            int u = -1;
            if (lane == 0) {
                if (mbar_wait(&ring_full[rs], (ku / kRing) & 1, abort_flag, fault)) u = ring[rs];
                mbar_arrive(&ring_empty[rs]);
            }
            u = __shfl_sync(0xffffffffu, u, 0);
            if (u < 0) break;
            const int64_t ue = unit_start(sc, u + 1);
        for (int64_t t = unit_start(sc, u); ok && t < ue;) {
            const Piece P = piece_at(t, ue, prefix, a);
            t += P.k1 - P.k0;
            const int L = __ldg(a.seq_lens + P.b);
            const bool app = a.new_v != nullptr && P.k1 == P.nt;  // as the K producer
            uint4 nrow = make_uint4(0, 0, 0, 0);
            if (app && lane < 16)
                nrow = __ldg(a.new_v + (int64_t)P.b * a.row_vecs + P.g * 16 + lane);
            const uint32_t *trow = a.tables + (int64_t)P.b * a.table_stride;
            TableWindow win = window_at(trow, P.k0 * kTcTile / a.block_size);
            for (int k = P.k0; k < P.k1; ++k, ++j) {
                const int stage = (int)(j % kTcStages);
                if (!mbar_wait(&vempty[stage], ((j / kTcStages) & 1) ^ 1, abort_flag, fault)) {
                    ok = false;
                    break;
                }
                load_tile(&vmap, &vfull[stage], sm + stage * kTcStageBytes + 2 * kTcHalf, trow,
                          win, k, L, P.g, app && k == P.nt - 1 ? a.vpool : nullptr, nrow);
            }
        }
        }
    } else if (warp == 1) {
        // ------------------------------ MMA issuer ------------------------------
        if (lane == 0) {
            uint32_t j = 0, qi = 0;
            bool ok = true;
            for (uint32_t ku = 0; ok; ++ku) {
                const int rs = (int)(ku % kRing);
                int u = -1;
                if (mbar_wait(&ring_full[rs], (ku / kRing) & 1, abort_flag, fault)) u = ring[rs];
                mbar_arrive(&ring_empty[rs]);
                if (u < 0) break;
                const int64_t ue = unit_start(sc, u + 1);
            for (int64_t t = unit_start(sc, u); ok && t < ue;) {
                const Piece P = piece_at(t, ue, prefix, a);
                t += P.k1 - P.k0;
                if (!mbar_wait(&q_full[qi & 1], (qi >> 1) & 1, abort_flag, fault)) {
                    ok = false;
                    break;
                }
                const uint32_t qaddr = smem_u32(sm + kTcQOff + (qi & 1) * 4096);
                // PV of tile jp: O^T[buf] = V^T . P^T once the group wrote P
                // and read the O of tile jp - 2 out of that buffer.
                auto issue_pv = [&](uint32_t jp) -> bool {
                    const int stage = (int)(jp % kTcStages);
                    const uint32_t buf = jp & 1, par = (jp >> 1) & 1;
                    if (!mbar_wait(&vfull[stage], (jp / kTcStages) & 1, abort_flag, fault) ||
                        !mbar_wait(&p_full[buf], par, abort_flag, fault) ||
                        !mbar_wait(&o_empty[buf], par ^ 1, abort_flag, fault))
                        return false;
                    tc_fence_after();
                    const uint32_t vaddr = smem_u32(sm + stage * kTcStageBytes) + 2 * kTcHalf;
                    const uint32_t paddr = smem_u32(sm + kTcPOff + buf * kTcPBuf);
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint64_t ad = sw128_desc(vaddr + kk * 2048, kTcHalf, 1024);
                        const uint64_t bd = sw128_desc(paddr + (kk >> 2) * kPChunk + (kk & 3) * 32, 16, 1024);
                        mma_f16_ss(tmem + 32 + buf * PN, ad, bd, kIdescPV, kk > 0);
                    }
                    mma_commit(&o_full[buf]);
                    mma_commit(&vempty[stage]);
                    return true;
                };
                // S of tile j is issued before the PV of tile j - 1, so the
                // group finds the next scores ready when it finishes a tile.
                for (int k = P.k0; k < P.k1; ++k, ++j) {
                    const int stage = (int)(j % kTcStages);
                    const uint32_t buf = j & 1, par = (j >> 1) & 1;
                    if (!mbar_wait(&kfull[stage], (j / kTcStages) & 1, abort_flag, fault) ||
                        !mbar_wait(&s_empty[buf], par ^ 1, abort_flag, fault)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t kaddr = smem_u32(sm + stage * kTcStageBytes);
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint64_t ad = sw128_desc(kaddr + (kk >> 2) * kTcHalf + (kk & 3) * 32, 16, 1024);
                        const uint64_t bd = sw128_desc(qaddr + (kk >> 2) * 2048 + (kk & 3) * 32, 16, 1024);
                        mma_f16_ss(tmem + buf * 16, ad, bd, kIdescQK, kk > 0);
                    }
                    mma_commit(&s_full[buf]);
                    mma_commit(&kempty[stage]);
                    if (k == P.k1 - 1) mma_commit(&q_empty[qi & 1]);
                    if (k > P.k0 && !issue_pv(j - 1)) {
                        ok = false;
                        break;
                    }
                }
                if (ok && P.k1 > P.k0 && !issue_pv(j - 1)) ok = false;
                ++qi;
            }
            }
        }
        __syncwarp();
    } else if (warp < 6) {
        // --------------------------- softmax / merge ---------------------------
        // On an abort (a wait gave up) the group keeps running the same loops
        // and named barriers -- so no thread can be left waiting at one -- but
        // stops reading TMEM; the fault word already records the failure.
        const int q4 = warp & 3;             // TMEM lane quadrant of this warp
        const int row = q4 * 32 + lane;      // token of S^T, dim of O^T
        const int wt = tid - 64;             // 0..127 within the group
        const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
        auto group_sync = [] { named_barrier(1, 128); };
        uint32_t j = 0;
        bool aborted = false;
        for (uint32_t ku = 0;; ++ku) {
            const int rs = (int)(ku % kRing);
            if (wt == 0) {
                int uu = -1;
                if (mbar_wait(&ring_full[rs], (ku / kRing) & 1, abort_flag, fault)) uu = ring[rs];
                *group_unit = uu;
                mbar_arrive(&ring_empty[rs]);
            }
            group_sync();
            const int u = *group_unit;
            group_sync();  // read by all before thread 0 of the group writes the next one
            if (u < 0) break;
            const int64_t us = unit_start(sc, u), ue = unit_start(sc, u + 1);
        for (int64_t t = us; t < ue;) {
            const Piece P = piece_at(t, ue, prefix, a);
            const bool first_piece = t == us;
            t += P.k1 - P.k0;
            const int L = __ldg(a.seq_lens + P.b);
            float m_run[GV], l_part[GV], acc[GV];
#pragma unroll
            for (int h = 0; h < GV; ++h) {
                m_run[h] = -INFINITY;
                l_part[h] = 0.f;
                acc[h] = 0.f;
            }
            // O of tile jp (its PV used P relative to the max of tile jp) folds
            // into acc after the correction alpha of tile jp.
            float alpha_prev[GV];
            auto fold = [&](uint32_t jp) {
                const uint32_t buf = jp & 1, par = (jp >> 1) & 1;
                aborted = aborted ||
                          !__all_sync(0xffffffffu, mbar_wait(&o_full[buf], par, abort_flag, fault));
                float o[PN];
#pragma unroll
                for (int i = 0; i < PN; ++i) o[i] = 0.f;
                if (!aborted) {
                    tc_fence_after();
                    tmem_ld_32x32b<PN>(tmem + 32 + buf * PN + lane_off, o);
                    tmem_wait_ld();
                    tc_fence_before();
                }
                mbar_arrive(&o_empty[buf]);
#pragma unroll
                for (int h = 0; h < GV; ++h) acc[h] = acc[h] * alpha_prev[h] + (o[h] + o[LO + h]);
            };
            // Tile j's scores and P first, then the O of tile j - 1: the PV
            // round trip of one tile hides behind the softmax of the next.
            for (int k = P.k0; k < P.k1; ++k, ++j) {
                const uint32_t buf = j & 1, par = (j >> 1) & 1;
                aborted = aborted ||
                          !__all_sync(0xffffffffu, mbar_wait(&s_full[buf], par, abort_flag, fault));
                float s[GN];
#pragma unroll
                for (int i = 0; i < GN; ++i) s[i] = 0.f;
                if (!aborted) {
                    tc_fence_after();
                    tmem_ld_32x32b<GN>(tmem + buf * 16 + lane_off, s);
                    tmem_wait_ld();
                    tc_fence_before();
                }
                mbar_arrive(&s_empty[buf]);
                const int valid = min(kTcTile, L - k * kTcTile);
                const bool live = row < valid;
                float x[GV];
#pragma unroll
                for (int h = 0; h < GV; ++h) {
                    const int col = PAIR && h >= G ? 8 + h - G : h;  // S^T column of head h
                    x[h] = live ? s[col] * a.scale_log2 : -INFINITY;
                    const float wm = warp_max(x[h]);
                    if (lane == 0) red[buf * 64 + q4 * 16 + h] = wm;
                }
                group_sync();
                float alpha[GV];
                unsigned char *pbuf = sm + kTcPOff + buf * kTcPBuf;
#pragma unroll
                for (int h = 0; h < GV; ++h) {
                    const float *rr = red + buf * 64 + h;
                    const float tmax = fmaxf(fmaxf(rr[0], rr[16]), fmaxf(rr[32], rr[48]));
                    const float m_new = fmaxf(m_run[h], tmax);
                    alpha[h] = ex2_fast(m_run[h] - m_new);
                    m_run[h] = m_new;
                    const float p = ex2_fast(x[h] - m_new);
                    const T hi = from_f32<T>(p);
                    const T lo = from_f32<T>(p - static_cast<float>(hi));
                    l_part[h] = l_part[h] * alpha[h] + p;
                    *reinterpret_cast<T *>(pbuf + sw128_offset(h, row, kPChunk)) = hi;
                    *reinterpret_cast<T *>(pbuf + sw128_offset(LO + h, row, kPChunk)) = lo;
                }
                // V rows past the length may hold anything: zero them once the
                // tile's V landed (its own barrier: V may arrive after S ran)
                if (!live && !aborted &&
                    mbar_wait(&vfull[j % kTcStages], (j / kTcStages) & 1, abort_flag, fault)) {
                    unsigned char *vrow =
                        sm + (j % kTcStages) * kTcStageBytes + 2 * kTcHalf + row * 128;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        reinterpret_cast<uint4 *>(vrow)[i] = make_uint4(0, 0, 0, 0);
                        reinterpret_cast<uint4 *>(vrow + kTcHalf)[i] = make_uint4(0, 0, 0, 0);
                    }
                }
                fence_proxy_async_smem();
                mbar_arrive(&p_full[buf]);
                if (k > P.k0) fold(j - 1);
#pragma unroll
                for (int h = 0; h < GV; ++h) alpha_prev[h] = alpha[h];
            }
            if (P.k1 > P.k0) fold(j - 1);
            // ---- finish the piece: l over the group, then output or partial ----
            float l[GV];
#pragma unroll
            for (int h = 0; h < GV; ++h) {
                const float ls = warp_sum(l_part[h]);
                if (lane == 0) lred[q4 * 16 + h] = ls;
            }
            group_sync();
#pragma unroll
            for (int h = 0; h < GV; ++h) l[h] = lred[h] + lred[16 + h] + lred[32 + h] + lred[48 + h];
            group_sync();
            OT *out = static_cast<OT *>(a.out) + ((int64_t)P.b * q_heads + (int64_t)P.g * GV) * OD;
            if (P.k0 == 0 && P.k1 == P.nt) {  // the whole segment ran here
#pragma unroll
                for (int h = 0; h < GV; ++h) {
                    const float v = l[h] > 0.f ? acc[h] / l[h] : 0.f;
                    if constexpr (PAIR) {
                        if ((h < G) == (row < 64)) out[h * 64 + (row & 63)] = from_f32<OT>(v);
                    } else {
                        out[h * 128 + row] = from_f32<OT>(v);
                    }
                }
                continue;
            }
            const int kslot = first_piece ? 0 : 1;
            const int64_t slot = ((int64_t)u * 2 + kslot) * GV;
#pragma unroll
            for (int h = 0; h < GV; ++h) {
                a.part_o[(slot + h) * 128 + row] = acc[h];
                if (wt == h) {
                    a.part_ml[(slot + h) * 2] = m_run[h];
                    a.part_ml[(slot + h) * 2 + 1] = l[h];
                }
            }
            if (!a.merge_in_kernel) continue;
            // a unit is the first unit of at most one cut segment (the last
            // segment starting in it), so the first unit names the ticket
            const int u0 = unit_of_tile(sc, P.seg);
            const int np = unit_of_tile(sc, P.seg + P.nt - 1) - u0 + 1;
            group_sync();
            if (wt == 0) {
                __threadfence();  // publishes the group's partials (bar.sync is cumulative)
                const uint32_t tk = atomicAdd(a.counters + u0, 1u);
                *ticket = tk == (uint32_t)(np - 1);
            }
            group_sync();
            if (*ticket) {
                __threadfence();
                merge_segment<OT>(a, 0, GV, GV, P.seg, P.nt, sc, wt, 128, 1, mwst, mlst, mslot,
                                  nullptr, kInKernelMergeMax, out, group_sync);
                if (wt == 0) a.counters[u0] = 0u;
            }
        }
        }
        // empty sequences: no tile, zero output (the SDK's all-masked rule)
        for (int b = blockIdx.x; b < a.batch; b += gridDim.x) {
            if (__ldg(a.seq_lens + b) > 0) continue;
            // a fused append needs room for its row (pkv_kv_append's rule)
            if (a.new_k != nullptr && wt == 0) record_fault(fault, kFaultRowsMismatch);
            OT *ob = static_cast<OT *>(a.out) + (int64_t)b * q_heads * OD;
            if (row < OD)
                for (int h = 0; h < q_heads; ++h) ob[h * OD + row] = from_f32<OT>(0.f);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, kTcTmemCols);
}

// Merges segments that span more than kInKernelMergeMax CTAs.  Grid:
// (kv_heads * G, batch), one query head per CTA; kMergeThreads threads,
// sixteen per output float4 (each summing every sixteenth piece), so the
// ~150 partial rows of a segment cut across every SM load in one round.
constexpr int kMergeThreads = 512;
template <typename OT>
__global__ void __launch_bounds__(kMergeThreads)
pkv_tc_merge_kernel(const TcArgs a, int group, int grid) {
    pdl_wait();
    pdl_launch_dependents();  // e.g. the all-gather of the merged heads
    __shared__ float wst[kTcMaxGrid];
    __shared__ float lst[kTcMaxGrid];
    __shared__ int slot[kTcMaxGrid];
    __shared__ float4 red[kMergeThreads];
    const int b = blockIdx.y;
    const int g = blockIdx.x / group, h = blockIdx.x - g * group;
    const int64_t T = a.tile_prefix[a.batch];
    __shared__ Sched sc;
    if (threadIdx.x == 0) make_sched(sc, T, grid, a.min_unit);  // as the decode kernel
    __syncthreads();
    const int nt = (a.tile_prefix[b + 1] - a.tile_prefix[b]) / a.kv_heads;
    if (nt == 0 || T == 0) return;
    const int64_t seg = a.tile_prefix[b] + (int64_t)g * nt;
    if (unit_of_tile(sc, seg) == unit_of_tile(sc, seg + nt - 1)) return;
    OT *out = static_cast<OT *>(a.out) +
              ((int64_t)b * a.kv_heads * group + (int64_t)g * group + h) *
                  (a.pair_split != 0 ? 64 : 128);
    merge_segment<OT>(a, h, 1, group, seg, nt, sc, threadIdx.x, kMergeThreads, kMergeThreads / 32,
                      wst, lst, slot, red, kTcMaxGrid, out, [] { __syncthreads(); });
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

// Grid of the tensor-core decode kernel and its work units.
int tc_grid() { return sm_count() < kTcMaxGrid ? sm_count() : kTcMaxGrid; }
size_t tc_units(int grid, bool dynamic) { return (size_t)grid * (dynamic ? 1 + kMaxRounds : 1); }


struct WsLayout {
    size_t counters, ml, o, total;
};

// The tickets ([batch][kv_heads], zero between launches) get room for
// kMaxBatch sequences of q_heads heads whatever this call's batch, so the
// partials of an earlier, smaller call never sit where a later call's
// tickets are.
WsLayout ws_layout(size_t batch, size_t q_heads, size_t head_dim, size_t max_chunks) {
    WsLayout w;
    w.counters = 0;
    w.ml = round_up((size_t)kMaxBatch * q_heads * sizeof(uint32_t), 256);
    w.o = w.ml + round_up(batch * q_heads * max_chunks * 2 * sizeof(float), 256);
    w.total = w.o + round_up(batch * q_heads * max_chunks * head_dim * sizeof(float), 256);
    return w;
}

// Positions per work unit: a multiple of the 128-token tcgen05 tile.  0
// picks from the longest sequence (bigger splits for long contexts).
size_t pick_chunk(size_t chunk_tokens, size_t max_seq_len) {
    size_t c = chunk_tokens;
    if (c == 0) c = max_seq_len <= 4096 ? 256 : (max_seq_len <= 32768 ? 512 : 1024);
    return round_up(c, 128);
}

template <int HD, int G, typename T, typename OT>
int launch_decode(const DecodeArgs &args, cudaStream_t stream) {
    auto kern = paged_decode_simt_kernel<HD, G, T, OT>;
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

// ---- tcgen05 path host side ----
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (fn == nullptr) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// 2-D view of [rows][width] two-byte elements (a pool, or the query rows),
// box = box_rows rows (one page, or one GQA group) of one 64-column half,
// 128-byte swizzle (the UMMA canonical layout).
bool encode_pool_map(CUtensorMap *map, const void *pool, uint64_t rows, uint64_t kv_width,
                     uint32_t box_rows, bool bf16) {
    auto enc = tensor_map_encoder();
    if (enc == nullptr) return false;
    cuuint64_t dims[2] = {kv_width, rows};
    cuuint64_t strides[1] = {kv_width * 2};
    cuuint32_t box[2] = {64, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
               const_cast<void *>(pool), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int G, typename T, typename OT, bool PAIR>
int launch_tc(const TcArgs &args, const TcMaps &mp, int ncta,
              cudaStream_t stream) {
    auto kern = paged_decode_tc_kernel<G, T, OT, PAIR>;
    constexpr int GV = PAIR ? 2 * G : G;  // query heads per segment
    static int configured[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)tc_smem_bytes(kTcMaxBatch)) != cudaSuccess)
            return 0;
        configured[dev] = 1;
    }
    // Programmatic dependent launch: the prologue (barriers, TMEM, shared
    // memory) overlaps the tail of the kernel before it in the stream, and
    // the kernel releases its own dependents once all its CTAs are resident
    // (the merge kernel and the next step's staging then launch while it
    // streams and wait on griddepcontrol.wait).
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ncta);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = tc_smem_bytes(args.batch);
    cfg.stream = stream;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, args, mp.k, mp.v, mp.q) != cudaSuccess) return 0;
    if (!args.merge_in_kernel) {
        cudaLaunchConfig_t mc = cfg;
        mc.gridDim = dim3(args.kv_heads * GV, args.batch);
        mc.blockDim = dim3(kMergeThreads);
        mc.dynamicSmemBytes = 0;
        if (cudaLaunchKernelEx(&mc, pkv_tc_merge_kernel<OT>, args, GV, ncta) != cudaSuccess)
            return 0;
    }
    return cudaGetLastError() == cudaSuccess;
}

template <typename T, typename OT>
int dispatch_tc_group(const TcArgs &args, int group, bool pair, const TcMaps &mp, int ncta,
                      cudaStream_t s) {
    if (pair) {
        switch (group) {
            case 1: return launch_tc<1, T, OT, true>(args, mp, ncta, s);
            case 2: return launch_tc<2, T, OT, true>(args, mp, ncta, s);
            case 4: return launch_tc<4, T, OT, true>(args, mp, ncta, s);
            case 8: return launch_tc<8, T, OT, true>(args, mp, ncta, s);
            default: return 0;
        }
    }
    switch (group) {
        case 1: return launch_tc<1, T, OT, false>(args, mp, ncta, s);
        case 2: return launch_tc<2, T, OT, false>(args, mp, ncta, s);
        case 4: return launch_tc<4, T, OT, false>(args, mp, ncta, s);
        case 8: return launch_tc<8, T, OT, false>(args, mp, ncta, s);
        case 16: return launch_tc<16, T, OT, false>(args, mp, ncta, s);
        default: return 0;
    }
}

int dispatch_tc(const TcArgs &args, int group, bool pair, bool bf16, PkvDType out,
                const TcMaps &mp, int ncta, cudaStream_t s) {
    if (!bf16)
        return out == PKV_DTYPE_F32
                   ? dispatch_tc_group<__half, float>(args, group, pair, mp, ncta, s)
                   : dispatch_tc_group<__half, __half>(args, group, pair, mp, ncta, s);
    return out == PKV_DTYPE_F32
               ? dispatch_tc_group<__nv_bfloat16, float>(args, group, pair, mp, ncta, s)
               : dispatch_tc_group<__nv_bfloat16, __nv_bfloat16>(args, group, pair, mp, ncta, s);
}

// The tensor-core kernel takes head_dim 128 (GQA groups up to 16), and
// head_dim 64 when the KV heads pair up (an even count, groups up to 8).
bool tc_eligible(size_t head_dim, size_t kv_heads, size_t block_size, size_t group,
                 size_t rows) {
    const char *force = getenv("PKV_DECODE_KERNEL");
    if (force != nullptr && strcmp(force, "simt") == 0) return false;
    const bool pages = block_size == 16 || block_size == 32 || block_size == 64 ||
                       block_size == 128;
    const bool g128 = group == 1 || group == 2 || group == 4 || group == 8 || group == 16;
    const bool g64 = (group == 1 || group == 2 || group == 4 || group == 8) && kv_heads % 2 == 0;
    return pages && rows < (size_t(1) << 31) &&
           ((head_dim == 128 && g128) || (head_dim == 64 && g64));
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
    const size_t chunk = pkv::pick_chunk(chunk_tokens, max_seq_len);
    const size_t max_chunks = max_seq_len / chunk + 1;
    // The larger of the two kernels' layouts, so either may run; the tensor-
    // core one with room for the dynamic tail's units and 16 heads a segment.
    const size_t simt = pkv::ws_layout(batch, q_heads, head_dim, max_chunks).total;
    const size_t tc = pkv::tc_workspace(pkv::tc_units(pkv::tc_grid(), true), 16).total;
    return simt > tc ? simt : tc;
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

}  // extern "C"

namespace pkv {
namespace {

// pkv_paged_decode, and with key_rows/value_rows non-null
// pkv_paged_decode_append: the tensor-core kernel stores the new rows itself
// (TcArgs::new_k), the CUDA-core path launches the append kernel first.
int paged_decode_impl(const char *what, const PkvPagedLayer *layer, const PkvBatch *batch,
                      const void *key_rows, const void *value_rows, size_t q_heads,
                      const void *query, float scale, void *output, PkvDType output_dtype,
                      size_t max_seq_len, size_t chunk_tokens, void *workspace,
                      size_t workspace_bytes, PkvStream stream, char *error,
                      size_t error_capacity) {
    if (layer == nullptr || batch == nullptr || query == nullptr || output == nullptr ||
        layer->key_pool == nullptr || layer->value_pool == nullptr ||
        batch->block_tables == nullptr || batch->seq_lens == nullptr) {
        pkv_internal_set_error(error, error_capacity, "%s: null argument", what);
        return 0;
    }
    const bool fused = key_rows != nullptr || value_rows != nullptr;
    if (fused && (key_rows == nullptr || value_rows == nullptr ||
                  ((uintptr_t)key_rows | (uintptr_t)value_rows) % 16 != 0)) {
        pkv_internal_set_error(error, error_capacity,
                               "%s: key_rows and value_rows must both be given, 16-byte aligned",
                               what);
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
    const bool use_tc = pkv::tc_eligible(hd, kvh, layer->block_size, group,
                                         layer->block_count * layer->block_size);
    if (group != 1 && group != 2 && group != 4 && group != 8 && !(use_tc && group == 16)) {
        pkv_internal_set_error(error, error_capacity,
                               "%s: q_heads/kv_heads must be 1, 2, 4 or 8 (16 with head_dim 128 "
                               "and pages of 16-128 tokens), got %zu",
                               what, group);
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
    const size_t chunk = pkv::pick_chunk(chunk_tokens, max_seq_len);
    const size_t max_chunks = max_seq_len / chunk + 1;
    const pkv::WsLayout ws = pkv::ws_layout(batch->batch, q_heads, hd, max_chunks);
    // tensor-core path: the static units' layout is the minimum; the dynamic
    // tail also needs the partials of its rounds' units
    const int ncta = pkv::tc_grid();
    const size_t gv = hd == 64 ? 2 * group : group;  // query heads of one segment
    const pkv::TcWorkspace tws_static = pkv::tc_workspace(pkv::tc_units(ncta, false), gv);
    const pkv::TcWorkspace tws_dyn = pkv::tc_workspace(pkv::tc_units(ncta, true), gv);
    const bool dyn_fits = workspace_bytes >= tws_dyn.total;
    const pkv::TcWorkspace tws = dyn_fits ? tws_dyn : tws_static;
    const size_t need = use_tc ? tws_static.total : ws.total;
    if (workspace == nullptr || workspace_bytes < need || ((uintptr_t)workspace % 256) != 0) {
        pkv_internal_set_error(error, error_capacity,
                               "%s: workspace needs %zu bytes, 256-byte aligned (got %zu)", what,
                               need, workspace_bytes);
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
    if (use_tc) {
        pkv::TcMaps mp;
        const bool bf16 = layer->dtype == PKV_DTYPE_BF16;
        const uint64_t rows = (uint64_t)layer->block_count * layer->block_size;
        if (!pkv::encode_pool_map(&mp.k, layer->key_pool, rows, kvh * hd,
                                  (uint32_t)layer->block_size, bf16) ||
            !pkv::encode_pool_map(&mp.v, layer->value_pool, rows, kvh * hd,
                                  (uint32_t)layer->block_size, bf16) ||
            !pkv::encode_pool_map(&mp.q, query, (uint64_t)batch->batch * q_heads, hd,
                                  (uint32_t)group, bf16)) {
            pkv_internal_set_error(error, error_capacity, "%s: tensor map encoding failed", what);
            return 0;
        }
        auto *wsb = static_cast<unsigned char *>(workspace);
        pkv::TcArgs t;
        t.claim = reinterpret_cast<uint32_t *>(wsb + tws.claim);
        t.counters = reinterpret_cast<uint32_t *>(wsb + tws.counters);
        t.part_ml = reinterpret_cast<float *>(wsb + tws.ml);
        t.part_o = reinterpret_cast<float *>(wsb + tws.o);
        t.tile_prefix = reinterpret_cast<int32_t *>(wsb + tws.prefix);
        t.table_stride = (int32_t)batch->table_stride;
        // head_dim 64: KV heads 2g and 2g+1 are one 128-column segment g
        const bool pair = hd == 64;
        const size_t segs = pair ? kvh / 2 : kvh;  // segments per sequence
        t.kv_heads = (int32_t)segs;
        t.pair_split = pair ? (int32_t)group : 0;
        t.block_size = (int32_t)layer->block_size;
        t.block_count = (uint32_t)layer->block_count;
        t.scale_log2 = scale * pkv::kLog2e;
        t.new_k = static_cast<const uint4 *>(key_rows);
        t.new_v = static_cast<const uint4 *>(value_rows);
        t.kpool = static_cast<uint4 *>(layer->key_pool);
        t.vpool = static_cast<uint4 *>(layer->value_pool);
        t.row_vecs = (int32_t)(kvh * hd / 8);
        // In-kernel merges need every segment to span at most
        // kInKernelMergeMax CTAs.  They also sit on the critical path of the
        // CTA that finishes last, so with few segments (each cut into many
        // pieces, e.g. one long sequence) the separate merge kernel, one CTA
        // per query head, finishes sooner.
        const bool fits = ncta / (int)segs + 2 <= pkv::kInKernelMergeMax;
        const bool many_segments = batch->batch * segs * 2 >= (size_t)ncta;
        t.merge_in_kernel = fits && many_segments;
        // Dynamic tail (in-kernel merges only): every unit holds at least
        // min_unit tiles, so a segment of at most max_tiles tiles meets at
        // most max_tiles / min_unit + 2 <= kInKernelMergeMax units.  Each
        // piece costs the CTA a pipeline drain at its end (the last PV, the
        // l reduction, partial stores, a ticket), so units are never below
        // kMinUnitTiles and short launches (a CTA share under ~64 tiles,
        // below 8 * kMinUnitTiles) keep the static split.
        const size_t max_tiles = (max_seq_len + pkv::kTcTile - 1) / pkv::kTcTile;
        const size_t by_pieces = (max_tiles + 23) / 24;
        t.min_unit = t.merge_in_kernel && dyn_fits
                         ? (int32_t)(by_pieces > pkv::kMinUnitTiles ? by_pieces
                                                                    : pkv::kMinUnitTiles)
                         : 0;
        // launches of at most kTcMaxBatch sequences (their prefix lives in smem)
        const size_t osz = output_dtype == PKV_DTYPE_F32 ? 4 : 2;
        ok = 1;
        for (size_t b0 = 0; ok && b0 < batch->batch; b0 += pkv::kTcMaxBatch) {
            const size_t n = batch->batch - b0 < (size_t)pkv::kTcMaxBatch
                                 ? batch->batch - b0
                                 : (size_t)pkv::kTcMaxBatch;
            pkv::TcArgs sl = t;
            sl.batch = (int32_t)n;
            sl.tables = batch->block_tables + b0 * batch->table_stride;
            sl.seq_lens = batch->seq_lens + b0;
            sl.query = static_cast<const char *>(query) + b0 * q_heads * hd * 2;
            sl.q_row0 = (int32_t)(b0 * q_heads);
            sl.out = static_cast<char *>(output) + b0 * q_heads * hd * osz;
            if (fused) {
                sl.new_k += b0 * (size_t)t.row_vecs;
                sl.new_v += b0 * (size_t)t.row_vecs;
            }
            ok = pkv::dispatch_tc(sl, (int)group, pair, bf16, output_dtype, mp, ncta, s);
        }
    } else if (fused && !pkv_kv_append(layer, batch, nullptr, key_rows, value_rows, batch->batch,
                                       stream, error, error_capacity)) {
        return 0;  // pkv_kv_append wrote the message
    } else if (layer->dtype == PKV_DTYPE_F16)
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

}  // namespace
}  // namespace pkv

extern "C" {

int pkv_paged_decode(const PkvPagedLayer *layer, const PkvBatch *batch, size_t q_heads,
                     const void *query, float scale, void *output, PkvDType output_dtype,
                     size_t max_seq_len, size_t chunk_tokens, void *workspace,
                     size_t workspace_bytes, PkvStream stream, char *error,
                     size_t error_capacity) {
    PKV_RANGE("pkv_paged_decode");
    return pkv::paged_decode_impl("pkv_paged_decode", layer, batch, nullptr, nullptr, q_heads,
                                  query, scale, output, output_dtype, max_seq_len, chunk_tokens,
                                  workspace, workspace_bytes, stream, error, error_capacity);
}

int pkv_paged_decode_append(const PkvPagedLayer *layer, const PkvBatch *batch,
                            const void *key_rows, const void *value_rows, size_t q_heads,
                            const void *query, float scale, void *output, PkvDType output_dtype,
                            size_t max_seq_len, size_t chunk_tokens, void *workspace,
                            size_t workspace_bytes, PkvStream stream, char *error,
                            size_t error_capacity) {
    PKV_RANGE("pkv_paged_decode_append");
    const char *what = "pkv_paged_decode_append";
    if (key_rows == nullptr || value_rows == nullptr) {
        pkv_internal_set_error(error, error_capacity, "%s: null key_rows or value_rows", what);
        return 0;
    }
    return pkv::paged_decode_impl(what, layer, batch, key_rows, value_rows, q_heads, query, scale,
                                  output, output_dtype, max_seq_len, chunk_tokens, workspace,
                                  workspace_bytes, stream, error, error_capacity);
}

int pkv_internal_take_decode_fault(uint32_t *code) {
    uint32_t zero = 0;
    if (cudaMemcpyFromSymbol(code, pkv::g_decode_fault, sizeof(uint32_t)) != cudaSuccess) return 0;
    return cudaMemcpyToSymbol(pkv::g_decode_fault, &zero, sizeof(uint32_t)) == cudaSuccess;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Decode without caller-provided scratch.
//
// For callers that cannot allocate device memory when they call decode --
// for instance a serving loop whose device memory is planned once up front
// (cudaMalloc may synchronise the device and fragments a pre-sized pool), or
// a host bound through an FFI that only passes the buffers it was handed and
// has no way to own extra device memory.  The split-K scratch lives in the
// static device array below instead: every GPU that loads this library holds
// kDecodeStaticScratchBytes (8 MiB) of it until the process exits.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kDecodeStaticScratchBytes = size_t(8) << 20;
static __device__ __align__(256) unsigned char g_decode_static_scratch[kDecodeStaticScratchBytes];

std::mutex g_static_scratch_lock;
// Per device: the array's device address and the id of the CUDA context it
// was looked up in.  The address belongs to that context; after a
// cudaDeviceReset (or under another context) the module is loaded again,
// possibly elsewhere, so a changed context id triggers a new lookup.
struct StaticScratchSlot {
    unsigned long long ctx_id;
    void *addr;
};
StaticScratchSlot g_static_scratch[64];

typedef CUresult (*CtxGetCurrentFn)(CUcontext *);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long *);

// Unique id of the context current on this thread (0 when there is none or
// the driver cannot say; 0 never matches a cached slot).
unsigned long long current_context_id() {
    static CtxGetCurrentFn get_current = nullptr;
    static CtxGetIdFn get_id = nullptr;
    static bool resolved = false;
    if (!resolved) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<CtxGetCurrentFn>(p);
        p = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<CtxGetIdFn>(p);
        resolved = true;
    }
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (get_current == nullptr || get_id == nullptr || get_current(&ctx) != CUDA_SUCCESS ||
        ctx == nullptr || get_id(ctx, &id) != CUDA_SUCCESS)
        return 0;
    return id;
}

// The array's device address for the current device, looked up with that
// device current the first time a context of it calls (cudaGetSymbolAddress;
// it allocates nothing).  In host code the symbol itself is only a host-side
// stand-in and must never be handed to a kernel.
void *static_scratch_for_current_device(char *error, size_t cap) {
    int dev = -1;
    cudaError_t st = cudaGetDevice(&dev);
    if (st != cudaSuccess || dev < 0 || dev >= 64) {
        pkv_internal_set_error(error, cap, "pkv_paged_decode_static_scratch: no usable device (%s)",
                               cudaGetErrorString(st));
        return nullptr;
    }
    std::lock_guard<std::mutex> guard(g_static_scratch_lock);
    StaticScratchSlot &slot = g_static_scratch[dev];
    const unsigned long long id = current_context_id();
    if (slot.addr == nullptr || id == 0 || slot.ctx_id != id) {
        void *p = nullptr;
        st = cudaGetSymbolAddress(&p, g_decode_static_scratch);
        if (st != cudaSuccess || p == nullptr) {
            pkv_internal_set_error(error, cap,
                                   "pkv_paged_decode_static_scratch: cudaGetSymbolAddress failed: %s",
                                   cudaGetErrorString(st));
            return nullptr;
        }
        slot.addr = p;
        // the lookup made the device's primary context current if none was
        slot.ctx_id = id != 0 ? id : current_context_id();
    }
    return slot.addr;
}

}  // namespace

extern "C" int pkv_paged_decode_static_scratch(const PkvPagedLayer *layer, const PkvBatch *batch,
                                               size_t q_heads, const void *query, float scale,
                                               void *output, PkvDType output_dtype,
                                               size_t max_seq_len, PkvStream stream, char *error,
                                               size_t error_capacity) {
    PKV_RANGE("pkv_paged_decode_static_scratch");
    const char *what = "pkv_paged_decode_static_scratch";
    // Everything the scratch size depends on is checked before the array is
    // touched, so a refused call writes no device memory.
    if (layer == nullptr || batch == nullptr || query == nullptr || output == nullptr ||
        layer->key_pool == nullptr || layer->value_pool == nullptr ||
        batch->block_tables == nullptr || batch->seq_lens == nullptr) {
        pkv_internal_set_error(error, error_capacity, "%s: null argument", what);
        return 0;
    }
    const size_t kvh = layer->kv_heads, hd = layer->head_dim;
    if (batch->batch == 0 || batch->batch > (size_t)pkv::kMaxBatch || kvh == 0 ||
        q_heads == 0 || q_heads % kvh != 0 || q_heads > 65536 || (hd != 64 && hd != 128) ||
        max_seq_len > INT32_MAX / 2) {
        pkv_internal_set_error(error, error_capacity,
                               "%s: invalid batch (1..%d), heads, head_dim or max_seq_len", what,
                               pkv::kMaxBatch);
        return 0;
    }
    // Scratch of the kernel pkv_paged_decode will pick for this shape;
    // anything above the array is refused.
    const size_t group = q_heads / kvh;
    size_t need, tickets;
    if (pkv::tc_eligible(hd, kvh, layer->block_size, group,
                         layer->block_count * layer->block_size)) {
        // the static units' layout; the dynamic tail runs when its larger
        // layout fits the array as well
        const pkv::TcWorkspace w =
            pkv::tc_workspace(pkv::tc_units(pkv::tc_grid(), false), hd == 64 ? 2 * group : group);
        need = w.total;
        tickets = w.prefix;  // claim words and tickets
    } else {
        const size_t chunk = pkv::pick_chunk(0, max_seq_len);
        need = pkv::ws_layout(batch->batch, q_heads, hd, max_seq_len / chunk + 1).total;
        tickets = pkv::round_up(batch->batch * kvh * sizeof(uint32_t), 256);
    }
    if (need > kDecodeStaticScratchBytes) {
        pkv_internal_set_error(error, error_capacity,
                               "%s: this shape needs %zu bytes of scratch, above the static "
                               "maximum of %zu bytes; use pkv_paged_decode with a workspace",
                               what, need, kDecodeStaticScratchBytes);
        return 0;
    }
    void *scratch = static_scratch_for_current_device(error, error_capacity);
    if (scratch == nullptr) return 0;
    // The split-K tickets (and the dynamic tail's claim words) must be zero
    // when a decode starts; both layouts keep them first.  A decode that
    // completes leaves them at zero, but one that gave up part-way (a bounded
    // wait that expired) may not, and the array outlives every call, so each
    // call clears them (one small memset on the caller's stream).
    const cudaError_t st = cudaMemsetAsync(scratch, 0, tickets, (cudaStream_t)stream);
    if (st != cudaSuccess) {
        pkv_internal_set_error(error, error_capacity, "%s: clearing the tickets failed: %s", what,
                               cudaGetErrorString(st));
        return 0;
    }
    return pkv_paged_decode(layer, batch, q_heads, query, scale, output, output_dtype,
                            max_seq_len, 0, scratch, kDecodeStaticScratchBytes, stream, error,
                            error_capacity);
}

// ---------------------------------------------------------------------------
// Self-test of the bounded waits (the failure path every warp-specialised
// kernel here relies on), run on the GPU without faulting it: one CTA holds
// TMEM, one warp waits on an mbarrier that nothing arrives on, the wait gives
// up after its cycle budget, raises the CTA's abort flag and records
// kFaultWaitTimeout, and the CTA frees TMEM and exits -- the context stays
// usable.
// ---------------------------------------------------------------------------
namespace {

__device__ uint32_t g_selftest_word;

__global__ void __launch_bounds__(64) selftest_wait_kernel() {
    using namespace pkv::sm100;
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    __shared__ uint32_t tmem_slot;
    const int warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(&tmem_slot, 32);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        // phase 0 of a fresh barrier with one expected arrival never completes
        const bool ok = __all_sync(0xffffffffu, mbar_wait(&bar, 0, &abort_flag, &g_selftest_word));
        if (ok && (threadIdx.x & 31) == 0) g_selftest_word = 0xffffffffu;  // cannot happen
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem_slot, 32);
}

}  // namespace

extern "C" int pkv_selftest_wait_timeout(uint32_t *code, char *error, size_t error_capacity) {
    const char *what = "pkv_selftest_wait_timeout";
    if (code == nullptr) {
        pkv_internal_set_error(error, error_capacity, "%s: null argument", what);
        return 0;
    }
    const uint32_t zero = 0;
    cudaError_t st = cudaMemcpyToSymbol(g_selftest_word, &zero, sizeof zero);
    if (st == cudaSuccess) {
        selftest_wait_kernel<<<1, 64>>>();
        st = cudaGetLastError();
    }
    if (st == cudaSuccess) st = cudaDeviceSynchronize();
    if (st == cudaSuccess) st = cudaMemcpyFromSymbol(code, g_selftest_word, sizeof *code);
    if (st != cudaSuccess) {
        pkv_internal_set_error(error, error_capacity, "%s: %s", what, cudaGetErrorString(st));
        return 0;
    }
    return 1;
}
