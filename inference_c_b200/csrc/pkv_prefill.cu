// pkv_prefill.cu -- chunked prefill attention over the paged cache (sm_100a).
//
// Each sequence b brings n_b new query rows that are its last n_b positions
// (the chunk just appended); with `causal` query j attends to keys
// 0 .. L_b - n_b + j, the SDK's causal offset kv_len - q_len
// (attention.c:251, :352-353), otherwise to all L_b keys.
//
// Work item = 128 query rows of two query heads of the same KV head (one head
// when the GQA group is odd).  One persistent 384-thread CTA per SM:
//   warp 0       producer: TMA-loads the item's query rows of both heads
//                (3-D boxes over [rows][heads][head_dim]) and, per 128-key
//                tile, every page of K and V of the KV head straight from the
//                pool (2-D boxes of one page x 64 columns); K and V rings of 2;
//   warp 1       one thread issues tcgen05.mma, interleaving the two heads
//                so each softmax group works while the tensor cores serve
//                the other:  S_A(j), PV_B(j-1), S_B(j), PV_A(j), ...
//                  S[128 q][128 k] = Q[128][d] . K^T          (smem x smem)
//                  O[128 q][d]    += P[128 q][128 k] . V[128][d] (P in TMEM)
//   warps 4-7    softmax of head A, warps 8-11 softmax of head B: thread r
//                owns query row r (TMEM lane r), so row max and sum need no
//                cross-thread traffic; all 128 scores of a row come from one
//                TMEM load.
// Each head's P replaces its S in TMEM as 16-bit pairs, a high half and a
// low half (p - round(p)) per 32-key chunk, and feeds the PV MMA as the
// A operand (two MMAs: high then low, ~22 bits of P).  One 16-bit P alone is
// not enough: with BF16 P the output error (~1e-4 at 2k-10k keys) breaks
// max-rel 1e-2 on outputs near 1e-2, and with FP16 P (V converted to FP16)
// rows over a few keys whose terms cancel reach 1.1e-2 (measured on the
// golden small case), so the split is always on.
// O accumulates in TMEM (FP32); the running max is raised only when a tile's
// max exceeds it by more than 2^8 (lazy rescale of O in TMEM).  A head's S/P
// buffer is reused for its next tile only after its PV completed.  TMEM:
// head A S/P 0-127, O 128-(128+d); head B S/P 256-383, O 384-(384+d).
// head_dim d is 64 or 128 (one or two 64-column halves per row).
#include <cudaTypedefs.h>
#include <math.h>
#include <stdio.h>

#include <utility>

#include "pkv_device.cuh"
#include "pkv_internal.h"
#include "pkv_trace.h"
#include "pkv_sm100.cuh"

namespace pkv {
namespace {

__device__ uint32_t g_prefill_fault;

constexpr int kPfThreads = 384;
constexpr int kPfTile = 128;
constexpr int kStages = 2;                // K ring and V ring depth
constexpr int kPfMaxBatch = 512;
constexpr float kRescaleThreshold = 8.f;  // log2 units
constexpr uint32_t kHalf = 16384;         // 128 rows x 128 bytes
constexpr uint32_t kQOff = 0;             // Q of head A then head B, [2 halves][128][64] each
constexpr uint32_t kKOff = 65536;         // K stages of 32 KiB
constexpr uint32_t kVOff = kKOff + kStages * 32768;
constexpr uint32_t kBarOff = kVOff + kStages * 32768;
constexpr uint32_t kMiscOff = kBarOff + 256;
constexpr uint32_t kPrefixOff = kMiscOff + 256;
constexpr uint32_t kTmemCols = 512;
constexpr int kRegsControl = 64, kRegsSoftmax = 216;
static_assert(128 * kRegsControl + 256 * kRegsSoftmax <= kPfThreads * 168, "register split");
constexpr float kLog2e = 1.4426950408889634f;

size_t pf_smem_bytes(int batch) { return kPrefixOff + 4u * ((size_t)batch + 1u) + 1024u; }

struct PfArgs {
    const uint32_t *tables;
    const int32_t *seq_lens;
    const int32_t *q_offsets;
    void *out;
    int32_t table_stride;
    int32_t batch;
    int32_t q_heads;
    int32_t kv_heads;
    int32_t block_size;
    uint32_t block_count;
    float scale_log2;
    int32_t causal;
    int32_t paired;  // GQA group even: items carry two heads
    // General instantiation only: an additive FP16 mask [query row of the
    // chunk][key] (nullptr: none) with its row stride in elements, whether
    // 16-byte loads may read it, and dense mode (a chunk may be longer than
    // its keys; the causal offset kv_len - q_len clamps at 0).
    const uint16_t *mask;
    int64_t mask_stride;
    int32_t mask_vec;
    int32_t dense;
    // Dense layout (the SDK's [batch][heads][rows][128] tensors): sequence s
    // holds rows [0, dense_rows) of query/output heads s*q_heads .. +q_heads-1,
    // read and written in place instead of token-major rows.
    int32_t dense_layout;
    int32_t dense_rows;
    int32_t seq0;  // dense layout: the launch's first sequence (launches hold <= kPfMaxBatch)
};

struct Item {
    int b, h0, g, q0, qrel, nrows, L, pos0, ntiles;
    bool bad;
};

__device__ __forceinline__ int items_per_qtile(const PfArgs &a) {
    const int group = a.q_heads / a.kv_heads;
    return a.kv_heads * (a.paired ? group / 2 : group);
}

__device__ __forceinline__ Item item_at(int64_t u, const int *prefix, const PfArgs &a) {
    Item I;
    int lo = 0, hi = a.batch - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (prefix[mid] <= u) lo = mid; else hi = mid - 1;
    }
    I.b = lo;
    const int qstart = __ldg(a.q_offsets + lo);
    const int nq = __ldg(a.q_offsets + lo + 1) - qstart;
    const int nqt = (nq + kPfTile - 1) / kPfTile;
    const int per = items_per_qtile(a);
    const int w = (int)(u - prefix[lo]);
    const int qt = nqt - 1 - w / per;  // longest tiles of a sequence first
    const int rest = w - (w / per) * per;
    const int group = a.q_heads / a.kv_heads;
    const int np = a.paired ? group / 2 : group;
    I.g = rest / np;
    I.h0 = I.g * group + (rest - I.g * np) * (a.paired ? 2 : 1);
    I.q0 = qstart + qt * kPfTile;
    I.qrel = qt * kPfTile;
    I.nrows = min(kPfTile, nq - qt * kPfTile);
    I.L = __ldg(a.seq_lens + lo);
    I.bad = nq > I.L && !a.dense;
    I.pos0 = max(I.L - nq, 0) + qt * kPfTile;
    const int kmax = a.causal ? min(I.L, I.pos0 + I.nrows) : I.L;
    I.ntiles = I.bad ? 0 : (kmax + kPfTile - 1) / kPfTile;
    return I;
}

// The k-th item of this CTA: rounds of gridDim.x consecutive items.  Items
// come longest first within a sequence, so a plain stride gives the first
// CTAs the longest item of every round; in the dense layout (one long causal
// sequence per (batch, KV head): item sizes from 1 to q_len/128 key tiles)
// the CTA order is reversed in every other round, pairing long with short
// (config 7: the heaviest CTA 74 -> ~58 key tiles against a mean of 57).
// Paged chunks over a long past have items of similar size and keep the
// plain stride (measured 0.9 % faster there).
__device__ __forceinline__ int64_t item_order(int64_t k, bool serpentine) {
    const int64_t c =
        serpentine && (k & 1) ? (int64_t)gridDim.x - 1 - blockIdx.x : (int64_t)blockIdx.x;
    return k * gridDim.x + c;
}

__device__ void build_item_prefix(const PfArgs &a, int *prefix, int *scratch) {
    const int tid = threadIdx.x, nthr = blockDim.x, lane = tid & 31, warp = tid >> 5;
    const int per = (a.batch + nthr - 1) / nthr;
    const int items = items_per_qtile(a);
    int local = 0;
    for (int k = 0; k < per; ++k) {
        const int b = tid * per + k;
        if (b < a.batch) {
            const int nq = __ldg(a.q_offsets + b + 1) - __ldg(a.q_offsets + b);
            local += (max(nq, 0) + kPfTile - 1) / kPfTile * items;
        }
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
            const int nq = __ldg(a.q_offsets + b + 1) - __ldg(a.q_offsets + b);
            run += (max(nq, 0) + kPfTile - 1) / kPfTile * items;
        }
    }
    if (tid == nthr - 1) prefix[a.batch] = before + incl;
}

// exp2 on the SFU (ex2.approx.ftz): results below 2^-126 flush to zero, far
// beneath anything a softmax weight can contribute.
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Three-input max (sm_100 max.f32 with three sources).
__device__ __forceinline__ float max3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// Packed two-lane FP32 arithmetic (sm_100 .f32x2): one instruction per pair.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    uint64_t d;
    asm("{\n.reg .b64 ra, rb, rc;\nmov.b64 ra, {%1, %2};\nmov.b64 rb, {%3, %4};\n"
        "mov.b64 rc, {%5, %6};\nfma.rn.f32x2 %0, ra, rb, rc;\n}"
        : "=l"(d) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(d));
    return r;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    uint64_t d;
    asm("{\n.reg .b64 ra, rb;\nmov.b64 ra, {%1, %2};\nmov.b64 rb, {%3, %4};\n"
        "add.rn.f32x2 %0, ra, rb;\n}"
        : "=l"(d) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(d));
    return r;
}

// Scores of keys at or past `limit` in the 32-key chunk starting at key kc
// become -inf (their weight is exactly 0).
__device__ __forceinline__ void mask_chunk(uint32_t (&v)[32], int kc, int limit) {
#pragma unroll
    for (int i = 0; i < 32; ++i)
        if (kc + i >= limit) v[i] = 0xff800000u;
}

template <typename T>
struct Bf16Flag { static constexpr bool value = false; };
template <>
struct Bf16Flag<__nv_bfloat16> { static constexpr bool value = true; };

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}
template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t v);
template <>
__device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t v) {
    return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
}
template <>
__device__ __forceinline__ float2 unpack2<__half>(uint32_t v) {
    return __half22float2(*reinterpret_cast<__half2 *>(&v));
}

// 32 FP32 accumulator words of one output row, times `inv`, as 16-byte stores.
template <typename OT>
__device__ __forceinline__ void store_row32(OT *dst, const uint32_t (&v)[32], float inv);
template <>
__device__ __forceinline__ void store_row32<float>(float *dst, const uint32_t (&v)[32], float inv) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
        reinterpret_cast<float4 *>(dst)[i] =
            make_float4(__uint_as_float(v[4 * i]) * inv, __uint_as_float(v[4 * i + 1]) * inv,
                        __uint_as_float(v[4 * i + 2]) * inv, __uint_as_float(v[4 * i + 3]) * inv);
}
template <typename OT>
__device__ __forceinline__ void store_row32(OT *dst, const uint32_t (&v)[32], float inv) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint4 w;
        w.x = pack2<OT>(__uint_as_float(v[8 * i]) * inv, __uint_as_float(v[8 * i + 1]) * inv);
        w.y = pack2<OT>(__uint_as_float(v[8 * i + 2]) * inv, __uint_as_float(v[8 * i + 3]) * inv);
        w.z = pack2<OT>(__uint_as_float(v[8 * i + 4]) * inv, __uint_as_float(v[8 * i + 5]) * inv);
        w.w = pack2<OT>(__uint_as_float(v[8 * i + 6]) * inv, __uint_as_float(v[8 * i + 7]) * inv);
        reinterpret_cast<uint4 *>(dst)[i] = w;
    }
}

// S[128 q][128 k] = Q . K^T: HD/16 K=16 steps over the 64-column halves of Q
// and K (SWIZZLE_128B, K-major: step kk starts 32 bytes further along a
// 128-byte row; steps 4-7 read the second half when HD = 128).
__host__ __device__ constexpr uint32_t s_step(uint32_t kk) { return ((kk >> 2) * kHalf + (kk & 3) * 32) >> 4; }
__host__ __device__ constexpr uint32_t p_col(uint32_t kk) { return (kk >> 1) * 32 + (kk & 1) * 8; }
__host__ __device__ constexpr uint32_t v_step(uint32_t kk) { return kk * (2048 >> 4); }

template <uint32_t... KK>
__device__ __forceinline__ void s_mmas(uint32_t dst, uint64_t qd, uint64_t kd, uint32_t idesc,
                                       std::integer_sequence<uint32_t, KK...>) {
    (sm100::mma_f16_ss_at<s_step(KK), s_step(KK)>(dst, qd, kd, idesc, KK > 0 ? 1u : 0u), ...);
}
// O[128 q][HD] (+)= P . V with P from TMEM: step kk covers keys 16kk..16kk+15,
// whose high halves sit in columns 32(kk/2) + 8(kk%2) .. +7 and low halves 16
// columns further; V (MN-major) advances 16 rows = 2048 bytes per step.  The
// high-half MMAs run first (the first of an item starts the accumulator),
// then the low halves add in.
template <uint32_t... KK>
__device__ __forceinline__ void pv_mmas(uint32_t ocol, uint32_t pcol, uint64_t vd, uint32_t idesc,
                                        uint32_t acc, std::integer_sequence<uint32_t, KK...>) {
    (sm100::mma_f16_ts_at<p_col(KK), v_step(KK)>(ocol, pcol, vd, idesc, (acc | KK) ? 1u : 0u),
     ...);
    (sm100::mma_f16_ts_at<p_col(KK) + 16, v_step(KK)>(ocol, pcol, vd, idesc, 1u), ...);
}

// Adds the mask (times log2 e) to a chunk of 32 scaled scores of keys kc..;
// keys at or past L read nothing (the length mask covers them).
__device__ __forceinline__ void add_mask_chunk(uint32_t (&v)[32], const uint16_t *mrow, int kc,
                                               int L, bool vec) {
    if (vec && kc + 32 <= L) {
        uint4 m[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) m[i] = __ldg(reinterpret_cast<const uint4 *>(mrow + kc) + i);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t w[4] = {m[i].x, m[i].y, m[i].z, m[i].w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[k]));
                v[8 * i + 2 * k] = __float_as_uint(__uint_as_float(v[8 * i + 2 * k]) + f.x * kLog2e);
                v[8 * i + 2 * k + 1] =
                    __float_as_uint(__uint_as_float(v[8 * i + 2 * k + 1]) + f.y * kLog2e);
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
            if (kc + i < L)
                v[i] = __float_as_uint(__uint_as_float(v[i]) +
                                       __half2float(__ushort_as_half(__ldg(mrow + kc + i))) * kLog2e);
    }
}

// GEN = false: the paged prefill path (no mask, scale > 0, so the max can be
// taken over raw scores and scaled once).  GEN = true: scores are scaled (and
// masked) before the max, any finite scale, and rows whose running max
// becomes +inf give zeros (the SDK CUDA backend's rule for a non-finite max).
// HD = head_dim (64 or 128).
template <typename T, typename OT, bool GEN, int HD>
__global__ void __launch_bounds__(kPfThreads, 1)
paged_prefill_tc_kernel(const PfArgs a, const __grid_constant__ CUtensorMap qmap,
                        const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap) {
    using namespace sm100;
    static_assert(HD == 64 || HD == 128, "head_dim");
    constexpr int kHalves = HD / 64;          // 64-column halves of a Q/K/V row
    constexpr uint32_t kIdescS = idesc_f16(128, 128, Bf16Flag<T>::value, false, false);
    constexpr uint32_t kIdescPV = idesc_f16(128, HD, Bf16Flag<T>::value, false, true);
    extern __shared__ unsigned char smem_raw[];
    unsigned char *sm = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + kBarOff);
    uint64_t *kfull = bars, *kempty = bars + 2, *vfull = bars + 4, *vempty = bars + 6;
    uint64_t *s_full = bars + 8, *p_full = bars + 10, *pv_done = bars + 12;  // [head A, head B]
    uint64_t *q_full = bars + 14, *q_empty = bars + 15;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sm + kMiscOff);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(sm + kMiscOff + 4);
    int *scan = reinterpret_cast<int *>(sm + kMiscOff + 32);  // 12 ints
    int *prefix = reinterpret_cast<int *>(sm + kPrefixOff);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool paired = a.paired != 0;
    if (tid == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&kfull[i], 1);
            mbar_init(&kempty[i], 1);
            mbar_init(&vfull[i], 1);
            mbar_init(&vempty[i], 1);
        }
        for (int w = 0; w < 2; ++w) {
            mbar_init(&s_full[w], 1);
            mbar_init(&p_full[w], 128);
            mbar_init(&pv_done[w], 1);
        }
        mbar_init(q_full, 1);
        mbar_init(q_empty, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    if (tid == 0) {
        tma_prefetch_desc(&qmap);
        tma_prefetch_desc(&kmap);
        tma_prefetch_desc(&vmap);
    }
    build_item_prefix(a, prefix, scan);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int64_t total_items = prefix[a.batch];
    const bool serp = a.dense_layout != 0;
    uint32_t *fault = &g_prefill_fault;

    if (warp < 4) {
    // Control warpgroup (producer, MMA issuer, two idle warps) hands registers
    // to the softmax warpgroups: 128 x 64 + 256 x 216 = 384 x 168.
    setmaxnreg_dec<kRegsControl>();
    if (warp == 0) {
        // ------------------------------ producer ------------------------------
        uint32_t jj = 0, qi = 0;
        bool ok = true;
        for (int64_t k = 0, u = item_order(0, serp); ok && u < total_items;
             u = item_order(++k, serp)) {
            const Item I = item_at(u, prefix, a);
            if (I.bad) {
                if (lane == 0) record_fault(fault, kFaultRowsMismatch);
                continue;
            }
            if (I.ntiles == 0) continue;
            if (!mbar_wait(q_empty, (qi & 1) ^ 1, abort_flag, fault)) break;
            if (lane == 0) {
                mbar_arrive_expect_tx(q_full, (paired ? 2u : 1u) * kHalves * kHalf);
                // token-major rows: (column, head, row); dense: (column, row, head)
                const int32_t c1 = a.dense_layout ? I.qrel : I.h0;
                const int32_t c2 = a.dense_layout ? (a.seq0 + I.b) * a.q_heads + I.h0 : I.q0;
                const int32_t d1 = a.dense_layout ? 0 : 1, d2 = a.dense_layout ? 1 : 0;
#pragma unroll
                for (int hf = 0; hf < kHalves; ++hf) {
                    tma_load_3d(sm + kQOff + hf * kHalf, &qmap, q_full, 64 * hf, c1, c2);
                    if (paired)
                        tma_load_3d(sm + kQOff + (2 + hf) * kHalf, &qmap, q_full, 64 * hf,
                                    c1 + d1, c2 + d2);
                }
            }
            __syncwarp();
            const uint32_t *trow = a.tables + (int64_t)I.b * a.table_stride;
            for (int jt = 0; jt < I.ntiles; ++jt, ++jj) {
                const int k0 = jt * kPfTile;
                const int kend = min(I.L, k0 + kPfTile);
                const int p0 = k0 / a.block_size;
                const int np = (kend - k0 + a.block_size - 1) / a.block_size;
                uint32_t pid = 0;
                bool good = false;
                if (lane < np) {
                    const int pi = p0 + lane;
                    if (pi < a.table_stride) {
                        pid = __ldg(trow + pi);
                        good = pid < a.block_count;
                    }
                    if (!good) record_fault(fault, kFaultPageOutOfRange);
                }
                const unsigned mask = __ballot_sync(0xffffffffu, good);
                const uint32_t bytes = (uint32_t)__popc(mask) * a.block_size * (2u * HD);
                const uint32_t ro = (uint32_t)lane * a.block_size * 128u;
                const int32_t y = (int32_t)pid * a.block_size, x = I.g * HD;
                const int st = (int)(jj % kStages);
                const uint32_t par = ((jj / kStages) & 1) ^ 1;
                if (!mbar_wait(&kempty[st], par, abort_flag, fault)) {
                    ok = false;
                    break;
                }
                if (lane == 0) mbar_arrive_expect_tx(&kfull[st], bytes);
                __syncwarp();
                if (good) {
                    unsigned char *kst = sm + kKOff + st * 32768;
#pragma unroll
                    for (int hf = 0; hf < kHalves; ++hf)
                        tma_load_2d(kst + hf * kHalf + ro, &kmap, &kfull[st], x + 64 * hf, y);
                }
                if (!mbar_wait(&vempty[st], par, abort_flag, fault)) {
                    ok = false;
                    break;
                }
                if (lane == 0) mbar_arrive_expect_tx(&vfull[st], bytes);
                __syncwarp();
                if (good) {
                    unsigned char *vst = sm + kVOff + st * 32768;
#pragma unroll
                    for (int hf = 0; hf < kHalves; ++hf)
                        tma_load_2d(vst + hf * kHalf + ro, &vmap, &vfull[st], x + 64 * hf, y);
                }
            }
            ++qi;
        }
    } else if (warp == 1) {
        // ------------------------------ MMA issuer ------------------------------
        if (lane == 0) {
            uint32_t jj = 0, qi = 0;
            bool ok = true;
            // Paired: head w owns S/P buffer w and O buffer w.  Unpaired: the
            // one head alternates S/P buffers by tile and accumulates in O 0.
            auto sbuf = [&](int w, uint32_t t) -> uint32_t {
                return tmem + (paired ? (uint32_t)w : (t & 1u)) * 256u;
            };
            // S of head w for global tile t.  Its S/P buffer was last read by
            // a PV MMA this thread issued earlier; tcgen05.mma operations of
            // one thread execute in issue order, so the new S overwrites the
            // old P only after that PV consumed it (the same ordering the
            // CUTLASS sm100 FMHA mainloop relies on for its S/P aliasing).
            // Shared-memory descriptors of the tiles; a k-step or a stage moves
            // the start-address field (16-byte units, bits 0-13) by a constant.
            const uint64_t qdesc = sw128_desc(smem_u32(sm + kQOff), 16, 1024);
            const uint64_t kdesc = sw128_desc(smem_u32(sm + kKOff), 16, 1024);
            const uint64_t vdesc = sw128_desc(smem_u32(sm + kVOff), kHalf, 1024);
            auto issue_s = [&](int w, uint32_t t) -> bool {
                const uint64_t qd = qdesc + (uint64_t)((uint32_t)w * (2 * kHalf >> 4));
                const uint64_t kd = kdesc + (uint64_t)((t % kStages) * (32768u >> 4));
                s_mmas(sbuf(w, t), qd, kd, kIdescS,
                       std::make_integer_sequence<uint32_t, HD / 16>{});
                mma_commit(&s_full[w]);
                return true;
            };
            // PV of head w for global tile t (jt: its index within the item),
            // then release the tile's V stage when no other head still reads it.
            auto issue_pv = [&](int w, uint32_t t, int jt, bool last_reader) -> bool {
                const int st = (int)(t % kStages);
                if (!mbar_wait(&vfull[st], (t / kStages) & 1, abort_flag, fault) ||
                    !mbar_wait(&p_full[w], t & 1, abort_flag, fault))
                    return false;
                tc_fence_after();
                const uint64_t vd = vdesc + (uint64_t)((uint32_t)st * (32768u >> 4));
                const uint32_t ocol = tmem + (paired ? (uint32_t)w * 256u : 0u) + 128u;
                pv_mmas(ocol, sbuf(w, t), vd, kIdescPV, jt > 0 ? 1u : 0u,
                        std::make_integer_sequence<uint32_t, 8>{});
                mma_commit(&pv_done[w]);
                if (last_reader) mma_commit(&vempty[st]);
                return true;
            };
            // Issue order per tile j: paired  S_A(j) PV_B(j-1) S_B(j) PV_A(j);
            //                         unpaired S(j) PV(j-1).
            // Each softmax group works while the tensor pipe serves the other.
            for (int64_t k = 0, u = item_order(0, serp); ok && u < total_items;
                 u = item_order(++k, serp)) {
                const Item I = item_at(u, prefix, a);
                if (I.bad || I.ntiles == 0) continue;
                if (!mbar_wait(q_full, qi & 1, abort_flag, fault)) break;
                for (int jt = 0; jt < I.ntiles && ok; ++jt, ++jj) {
                    const int st = (int)(jj % kStages);
                    ok = mbar_wait(&kfull[st], (jj / kStages) & 1, abort_flag, fault) &&
                         issue_s(0, jj);
                    if (ok && jt > 0) ok = issue_pv(paired ? 1 : 0, jj - 1, jt - 1, true);
                    if (ok && paired) ok = issue_s(1, jj);
                    if (!ok) break;
                    mma_commit(&kempty[st]);
                    if (jt == I.ntiles - 1) mma_commit(q_empty);
                    if (paired) ok = issue_pv(0, jj, jt, false);
                }
                if (ok) ok = issue_pv(paired ? 1 : 0, jj - 1, I.ntiles - 1, true);
                ++qi;
            }
        }
        __syncwarp();
    }
    } else if (warp < 8 || paired) {
        setmaxnreg_inc<kRegsSoftmax>();
        // ------------------------------- softmax -------------------------------
        // A wait that gives up (abort or timeout) ends the warp's work; the
        // vote keeps the .sync.aligned TMEM instructions warp-uniform.
        auto wait = [&](uint64_t *bar, uint32_t par) -> bool {
            return __all_sync(0xffffffffu, mbar_wait(bar, par, abort_flag, fault));
        };
        const int w = warp < 8 ? 0 : 1;         // head A or head B
        const int q4 = warp & 3;
        const int r = q4 * 32 + lane;            // query row = TMEM lane
        const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
        const uint32_t ocol = tmem + w * 256 + 128 + lane_off;
        uint32_t jj = 0;
        bool ok = true;
        for (int64_t k = 0, u = item_order(0, serp); ok && u < total_items;
             u = item_order(++k, serp)) {
            const Item I = item_at(u, prefix, a);
            if (I.bad || I.ntiles == 0) continue;
            const bool row_ok = r < I.nrows;
            const int pos = I.pos0 + (row_ok ? r : I.nrows - 1);
            const int limit = a.causal ? min(pos + 1, I.L) : I.L;  // keys < limit attend
            float m_run = -INFINITY, l = 0.f;
            bool dead = false;  // GEN: the row's max reached +inf
            const uint16_t *mrow =
                GEN && a.mask != nullptr
                    ? a.mask + (int64_t)(I.qrel + (row_ok ? r : I.nrows - 1)) * a.mask_stride
                    : nullptr;
            for (int jt = 0; jt < I.ntiles; ++jt, ++jj) {
                const int k0 = jt * kPfTile;
                const bool masked = k0 + kPfTile > limit;
                const uint32_t scol = tmem + (paired ? (uint32_t)w : (jj & 1u)) * 256u + lane_off;
                if (!wait(&s_full[w], jj & 1)) { ok = false; break; }
                tc_fence_after();
                // the row's 128 scores in registers with one TMEM round trip
                uint32_t v[4][32];
#pragma unroll
                for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(scol + c * 32, v[c]);
                tmem_wait_ld();
                if constexpr (GEN) {
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            v[c][i] = __float_as_uint(__uint_as_float(v[c][i]) * a.scale_log2);
                        if (mrow != nullptr) add_mask_chunk(v[c], mrow, k0 + c * 32, I.L, a.mask_vec);
                    }
                }
                if (masked) {
#pragma unroll
                    for (int c = 0; c < 4; ++c) mask_chunk(v[c], k0 + c * 32, limit);
                }
                float mc[4];  // one running max per chunk: four short chains
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    mc[c] = max3(__uint_as_float(v[c][0]), __uint_as_float(v[c][1]),
                                 __uint_as_float(v[c][2]));
#pragma unroll
                    for (int i = 3; i < 31; i += 2)
                        mc[c] = max3(mc[c], __uint_as_float(v[c][i]), __uint_as_float(v[c][i + 1]));
                    mc[c] = fmaxf(mc[c], __uint_as_float(v[c][31]));
                }
                float mx = max3(mc[0], mc[1], fmaxf(mc[2], mc[3]));
                if constexpr (!GEN) mx *= a.scale_log2;  // scale > 0 commutes with max
                float alpha = 1.f;
                bool rescale = false;
                if (mx > m_run + kRescaleThreshold) {  // first tile: m_run = -inf
                    alpha = ex2_approx(m_run - mx);
                    m_run = mx;
                    rescale = jt > 0;
                    l *= alpha;
                }
                // V rows of keys past the sequence may hold anything: head A
                // zeroes them (once their TMA landed) before either PV reads.
                if (w == 0 && k0 + kPfTile > I.L) {
                    const int st = (int)(jj % kStages);
                    if (!wait(&vfull[st], (jj / kStages) & 1)) { ok = false; break; }
                    if (k0 + r >= I.L) {
                        unsigned char *vrow = sm + kVOff + st * 32768 + r * 128;
#pragma unroll
                        for (int hf = 0; hf < kHalves; ++hf)
#pragma unroll
                            for (int i = 0; i < 8; ++i)
                                reinterpret_cast<uint4 *>(vrow + hf * kHalf)[i] =
                                    make_uint4(0, 0, 0, 0);
                    }
                    fence_proxy_async_smem();
                }
                // rescaling O needs this head's previous PV to be done
                if (__any_sync(0xffffffffu, rescale)) {
                    if (!wait(&pv_done[w], (jj - 1) & 1)) { ok = false; break; }
                    tc_fence_after();
#pragma unroll
                    for (int c = 0; c < HD / 32; ++c) {
                        uint32_t o[32];
                        tmem_ld_32x32b_x32(ocol + c * 32, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                        tmem_st_32x32b_x32(ocol + c * 32, o);
                    }
                }
                // P = exp2(s * scale - m) chunk by chunk into the chunk's own
                // columns, as a 16-bit high half and the low remainder
                const float sc = GEN ? 1.f : a.scale_log2;
                const float2 sc2 = make_float2(sc, sc);
                // GEN: a row that has seen only -inf keeps m = -inf (use 0: its
                // P is 0); one whose max is +inf is dead (P = 0, output 0)
                // a row that has seen only masked keys so far keeps m = -inf:
                // use 0 (its P is 0) rather than produce NaN from -inf + inf
                float nm = m_run == -INFINITY ? 0.f : -m_run;
                if constexpr (GEN) {
                    dead = dead || m_run == INFINITY;
                    if (dead) {
#pragma unroll
                        for (int c = 0; c < 4; ++c)
#pragma unroll
                            for (int i = 0; i < 32; ++i) v[c][i] = 0xff800000u;
                        nm = 0.f;
                    }
                }
                const float2 nm2 = make_float2(nm, nm);
                const float2 neg1 = make_float2(-1.f, -1.f);
                float2 lsum2 = make_float2(0.f, 0.f);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint32_t hi[16], lo[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float2 x = ffma2(make_float2(__uint_as_float(v[c][2 * i]),
                                                           __uint_as_float(v[c][2 * i + 1])),
                                               sc2, nm2);
                        const float2 e = make_float2(ex2_approx(x.x), ex2_approx(x.y));
                        hi[i] = pack2<T>(e.x, e.y);
                        const float2 rem = ffma2(unpack2<T>(hi[i]), neg1, e);  // exact
                        lo[i] = pack2<T>(rem.x, rem.y);
                        lsum2 = fadd2(lsum2, e);
                    }
                    tmem_st_32x32b_x16(scol + c * 32, hi);
                    tmem_st_32x32b_x16(scol + c * 32 + 16, lo);
                }
                l += lsum2.x + lsum2.y;
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(&p_full[w]);
            }
            // ---- O / l for this head's rows ----
            if (!ok || !wait(&pv_done[w], (jj - 1) & 1)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const float inv = l > 0.f && !dead ? 1.f / l : 0.f;
            OT *orow = static_cast<OT *>(a.out) +
                       (a.dense_layout
                            ? (((int64_t)(a.seq0 + I.b) * a.q_heads + I.h0 + w) * a.dense_rows +
                               I.qrel + r) * HD
                            : ((int64_t)(I.q0 + r) * a.q_heads + I.h0 + w) * HD);
#pragma unroll
            for (int c = 0; c < HD / 32; ++c) {
                uint32_t o[32];
                tmem_ld_32x32b_x32(ocol + c * 32, o);
                tmem_wait_ld();
                if (row_ok) store_row32<OT>(orow + c * 32, o, inv);
            }
            tc_fence_before();
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
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

int g_sms[64];
int sms() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (g_sms[dev] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        g_sms[dev] = n > 0 ? n : 148;
    }
    return g_sms[dev];
}

template <typename T, typename OT, bool GEN, int HD>
int launch(const PfArgs &args, const CUtensorMap &qm, const CUtensorMap &km,
           const CUtensorMap &vm, cudaStream_t s) {
    auto kern = paged_prefill_tc_kernel<T, OT, GEN, HD>;
    static int configured[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)pf_smem_bytes(kPfMaxBatch)) != cudaSuccess)
            return 0;
        configured[dev] = 1;
    }
    kern<<<sms(), kPfThreads, pf_smem_bytes(args.batch), s>>>(args, qm, km, vm);
    return cudaGetLastError() == cudaSuccess;
}

template <typename T, typename OT, int HD>
int launch_gen(bool gen, const PfArgs &args, const CUtensorMap &qm, const CUtensorMap &km,
               const CUtensorMap &vm, cudaStream_t s) {
    return gen ? launch<T, OT, true, HD>(args, qm, km, vm, s)
               : launch<T, OT, false, HD>(args, qm, km, vm, s);
}

template <int HD>
int launch_typed(bool bf16, PkvDType out, bool gen, const PfArgs &args, const CUtensorMap &qm,
                 const CUtensorMap &km, const CUtensorMap &vm, cudaStream_t s) {
    if (!bf16)
        return out == PKV_DTYPE_F32 ? launch_gen<__half, float, HD>(gen, args, qm, km, vm, s)
                                    : launch_gen<__half, __half, HD>(gen, args, qm, km, vm, s);
    return out == PKV_DTYPE_F32
               ? launch_gen<__nv_bfloat16, float, HD>(gen, args, qm, km, vm, s)
               : launch_gen<__nv_bfloat16, __nv_bfloat16, HD>(gen, args, qm, km, vm, s);
}

}  // namespace
}  // namespace pkv

extern "C" {

int pkv_paged_prefill(const PkvPagedLayer *layer, const PkvBatch *batch, size_t q_heads,
                      const int32_t *query_offsets, const void *query, size_t total_query_rows,
                      size_t max_query_len, float scale, int causal, void *output,
                      PkvDType output_dtype, PkvStream stream, char *error,
                      size_t error_capacity) {
    PKV_RANGE("pkv_paged_prefill");
    return pkv_internal_paged_prefill_ex(layer, batch, q_heads, query_offsets, query,
                                         total_query_rows, max_query_len, scale, causal, output,
                                         output_dtype, nullptr, 0, 0, 0, stream, error,
                                         error_capacity, "pkv_paged_prefill");
}

int pkv_internal_paged_prefill_ex(const PkvPagedLayer *layer, const PkvBatch *batch,
                                  size_t q_heads, const int32_t *query_offsets, const void *query,
                                  size_t total_query_rows, size_t max_query_len, float scale,
                                  int causal, void *output, PkvDType output_dtype,
                                  const uint16_t *mask, size_t mask_stride, int dense,
                                  int dense_layout, PkvStream stream, char *error,
                                  size_t error_capacity, const char *what) {
    if (layer == nullptr || batch == nullptr || query_offsets == nullptr || query == nullptr ||
        output == nullptr || layer->key_pool == nullptr || layer->value_pool == nullptr ||
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
    const size_t kvh = layer->kv_heads;
    const size_t bs = layer->block_size;
    const size_t hd = layer->head_dim;
    if ((hd != 64 && hd != 128) || kvh == 0 || q_heads == 0 || q_heads % kvh != 0 ||
        q_heads > 65535 || (bs != 16 && bs != 32 && bs != 64 && bs != 128)) {
        pkv_internal_set_error(error, error_capacity,
                               "%s: needs head_dim 64 or 128, q_heads a multiple of kv_heads and "
                               "pages of 16, 32, 64 or 128 tokens",
                               what);
        return 0;
    }
    const uint64_t rows = (uint64_t)layer->block_count * bs;
    if (batch->batch == 0 || batch->table_stride == 0 || batch->table_stride > INT32_MAX ||
        rows >= (uint64_t(1) << 31) || total_query_rows >= (size_t(1) << 31) ||
        !isfinite(scale) || (causal != 0 && causal != 1) || max_query_len > INT32_MAX) {
        pkv_internal_set_error(error, error_capacity, "%s: invalid batch, table, sizes or scale",
                               what);
        return 0;
    }
    if (((uintptr_t)layer->key_pool | (uintptr_t)layer->value_pool | (uintptr_t)query) % 16) {
        pkv_internal_set_error(error, error_capacity, "%s: buffers must be 16-byte aligned", what);
        return 0;
    }
    if (total_query_rows == 0) return 1;
    auto enc = pkv::encoder();
    if (enc == nullptr) {
        pkv_internal_set_error(error, error_capacity, "%s: no tensor-map encoder", what);
        return 0;
    }
    const bool bf16 = layer->dtype == PKV_DTYPE_BF16;
    const CUtensorMapDataType dt =
        bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUtensorMap qm, km, vm;
    {
        // token-major [rows][q_heads][128], or dense [sequences * q_heads]
        // [max_query_len][128] with every sequence holding max_query_len rows
        const uint64_t nseq_heads = dense_layout ? total_query_rows / max_query_len * q_heads : 0;
        cuuint64_t dims[3] = {hd, q_heads, total_query_rows};
        cuuint64_t strides[2] = {hd * 2, q_heads * hd * 2};
        cuuint32_t box[3] = {64, 1, 128};
        if (dense_layout) {
            dims[1] = max_query_len;
            dims[2] = nseq_heads;
            strides[0] = hd * 2;
            strides[1] = max_query_len * hd * 2;
            box[1] = 128;
            box[2] = 1;
        }
        cuuint32_t es[3] = {1, 1, 1};
        if (enc(&qm, dt, 3, const_cast<void *>(query), dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
            pkv_internal_set_error(error, error_capacity, "%s: query tensor map failed", what);
            return 0;
        }
    }
    for (int i = 0; i < 2; ++i) {
        cuuint64_t dims[2] = {kvh * hd, rows};
        cuuint64_t strides[1] = {kvh * hd * 2};
        cuuint32_t box[2] = {64, (cuuint32_t)bs};
        cuuint32_t es[2] = {1, 1};
        if (enc(i == 0 ? &km : &vm, dt, 2, i == 0 ? layer->key_pool : layer->value_pool, dims,
                strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
            pkv_internal_set_error(error, error_capacity, "%s: pool tensor map failed", what);
            return 0;
        }
    }
    pkv::PfArgs args;
    args.table_stride = (int32_t)batch->table_stride;
    args.q_heads = (int32_t)q_heads;
    args.kv_heads = (int32_t)kvh;
    args.block_size = (int32_t)bs;
    args.block_count = (uint32_t)layer->block_count;
    args.scale_log2 = scale * pkv::kLog2e;
    args.causal = causal;
    args.paired = ((q_heads / kvh) % 2) == 0;
    args.mask = mask;
    args.mask_stride = (int64_t)mask_stride;
    args.mask_vec = mask != nullptr && (uintptr_t)mask % 16 == 0 && mask_stride % 8 == 0;
    args.dense = dense != 0;
    args.dense_layout = dense_layout != 0;
    args.dense_rows = (int32_t)max_query_len;
    args.seq0 = 0;
    // the general instantiation: a mask, or a scale <= 0 (the max is then
    // taken after scaling); dense mode works in both
    const bool gen = mask != nullptr || !(scale > 0.f);
    const cudaStream_t s = (cudaStream_t)stream;
    int ok = 1;
    for (size_t b0 = 0; ok && b0 < batch->batch; b0 += pkv::kPfMaxBatch) {
        const size_t n = batch->batch - b0 < (size_t)pkv::kPfMaxBatch ? batch->batch - b0
                                                                      : (size_t)pkv::kPfMaxBatch;
        pkv::PfArgs sl = args;
        sl.batch = (int32_t)n;
        sl.seq0 = (int32_t)b0;
        sl.tables = batch->block_tables + b0 * batch->table_stride;
        sl.seq_lens = batch->seq_lens + b0;
        sl.q_offsets = query_offsets + b0;  // absolute row offsets: query/out stay global
        sl.out = output;
        ok = hd == 128 ? pkv::launch_typed<128>(bf16, output_dtype, gen, sl, qm, km, vm, s)
                       : pkv::launch_typed<64>(bf16, output_dtype, gen, sl, qm, km, vm, s);
    }
    if (!ok) {
        pkv_internal_set_error(error, error_capacity, "%s: launch failed: %s", what,
                               cudaGetErrorString(cudaGetLastError()));
        return 0;
    }
    return 1;
}

int pkv_internal_take_prefill_fault(uint32_t *code) {
    uint32_t zero = 0;
    if (cudaMemcpyFromSymbol(code, pkv::g_prefill_fault, sizeof(uint32_t)) != cudaSuccess) return 0;
    return cudaMemcpyToSymbol(pkv::g_prefill_fault, &zero, sizeof(uint32_t)) == cudaSuccess;
}

int pkv_internal_plant_prefill_fault(uint32_t code) {
    return cudaMemcpyToSymbol(pkv::g_prefill_fault, &code, sizeof(uint32_t)) == cudaSuccess;
}

}  // extern "C"
