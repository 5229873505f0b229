/*
 * pkv_oracle.c -- CPU restatement of the paged-KV attention path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (inference_c_b200/)
 * links, loads or calls this file; tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py use it as the checker.
 *
 * Each function restates one piece of the inference SDK in plain C:
 *   orc_f16_to_f32 / orc_f32_to_f16 / orc_bf16_to_f32
 *       IEEE half <-> single conversion with round-to-nearest-even and
 *       subnormals, as tensor_f16.c:17-85 does.
 *   orc_f32_to_bf16
 *       round-to-nearest-even to bfloat16.  The SDK has no such function;
 *       the seeded-input generator needs one (NaN stays NaN).
 *   orc_pool_row
 *       page addressing of decode_kv_position (attention_cuda.cu:301-305).
 *   orc_kv_rows
 *       the K/V stores of decode_rope_cache_kernel (attention_cuda.cu:
 *       334-338, without RoPE) for appends, the prefix-import page-run copy
 *       (:894-915) for imports, and the reverse copy for gathers.
 *   orc_sdpa_f32
 *       the CPU branch of tensor_sdpa_f32 (attention.c:212-406): GQA head
 *       mapping kv = h / (Hq/Hkv) (:317-321), sequential dot products times
 *       scale (:343-348), optional additive mask (:350-351), causal -inf for
 *       key > query + (Lk - Lq) (:251, :352-353), the all -inf / NaN / +inf
 *       rules (:355-377), expf and division (:369-379) and the key-ordered
 *       P.V sum (:389-401).  Same loop order, so with the same compiler flags
 *       its results match the SDK's bit for bit.
 *   orc_paged_attention
 *       gather a sequence's K/V through its block table, widen to FP32 with
 *       the conversions above, and run orc_sdpa_f32 on [1, Hkv, L, d] -- the
 *       oracle the SDK's own paged path is judged against (the SDK has no
 *       CPU paged attention: its CPU build's backend getter returns NULL,
 *       attention_cuda_stub.c:1-5).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

enum { ORC_F16 = 1, ORC_BF16 = 2 };

static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

float orc_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    const uint32_t e = (h >> 10) & 31u;
    uint32_t m = h & 1023u;
    if (e == 31u) return u2f(sign | 0x7f800000u | (m << 13));
    if (e != 0u) return u2f(sign | ((e + 112u) << 23) | (m << 13));
    if (m == 0u) return u2f(sign);
    /* subnormal: shift the leading one into the hidden-bit position */
    int exp = 113;
    while ((m & 1024u) == 0u) { m <<= 1; --exp; }
    return u2f(sign | ((uint32_t)exp << 23) | ((m & 1023u) << 13));
}

uint16_t orc_f32_to_f16(float f) {
    const uint32_t u = f2u(f);
    const uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    const int e = (int)((u >> 23) & 255u);
    const uint32_t m = u & 0x7fffffu;
    if (e == 255) {                       /* inf or NaN (keep a payload bit) */
        uint16_t pay = (uint16_t)(m >> 13);
        if (m != 0u && pay == 0u) pay = 1u;
        return (uint16_t)(sign | 0x7c00u | pay);
    }
    const int he = e - 112;               /* rebias 127 -> 15 */
    if (he >= 31) return (uint16_t)(sign | 0x7c00u);
    if (he <= 0) {                        /* half subnormal or zero */
        if (he < -10) return sign;
        const uint32_t sig = m | 0x800000u;
        const unsigned shift = (unsigned)(14 - he);
        uint32_t q = sig >> shift;
        const uint32_t rem = sig & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        return (uint16_t)(sign | q);
    }
    uint32_t q = (uint32_t)he << 10 | (m >> 13);
    const uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) ++q;  /* carry may reach inf */
    return (uint16_t)(sign | q);
}

float orc_bf16_to_f32(uint16_t b) { return u2f((uint32_t)b << 16); }

uint16_t orc_f32_to_bf16(float f) {
    const uint32_t u = f2u(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    const uint32_t lsb = (u >> 16) & 1u;
    return (uint16_t)((u + 0x7fffu + lsb) >> 16);
}

static float widen(uint16_t x, int dtype) {
    return dtype == ORC_BF16 ? orc_bf16_to_f32(x) : orc_f16_to_f32(x);
}

void orc_convert_to_f32(const uint16_t *src, float *dst, size_t n, int dtype) {
    for (size_t i = 0; i < n; ++i) dst[i] = widen(src[i], dtype);
}

void orc_convert_from_f32(const float *src, uint16_t *dst, size_t n, int dtype) {
    for (size_t i = 0; i < n; ++i)
        dst[i] = dtype == ORC_BF16 ? orc_f32_to_bf16(src[i]) : orc_f32_to_f16(src[i]);
}

/* Pool row of logical position `pos` of a sequence, or -1 when the position
 * or its page id is out of range. */
int64_t orc_pool_row(const uint32_t *table_row, size_t table_len, size_t block_size,
                     size_t block_count, int64_t pos) {
    if (pos < 0) return -1;
    const size_t page_idx = (size_t)pos / block_size;
    if (page_idx >= table_len) return -1;
    const uint32_t page = table_row[page_idx];
    if ((size_t)page >= block_count) return -1;
    return (int64_t)page * (int64_t)block_size + (int64_t)((size_t)pos % block_size);
}

/* Row copy between contiguous rows and pages (elements are 2-byte bit
 * patterns, copied untouched).  to_pool: rows -> pages.  tail: a sequence's
 * rows are its last n_b positions (append) instead of its first (import,
 * gather).  row_offsets NULL: one row per sequence.  Returns 0 on any
 * out-of-range position or page id. */
int orc_kv_rows(uint16_t *kpool, uint16_t *vpool, size_t kv_width, size_t block_size,
                size_t block_count, const uint32_t *tables, size_t table_stride,
                const int32_t *seq_lens, const int32_t *row_offsets, size_t batch,
                uint16_t *krows, uint16_t *vrows, int to_pool, int tail) {
    for (size_t b = 0; b < batch; ++b) {
        const int64_t first = row_offsets ? row_offsets[b] : (int64_t)b;
        const int64_t count = row_offsets ? row_offsets[b + 1] - row_offsets[b] : 1;
        const int64_t len = seq_lens[b];
        if (count > len) return 0;
        for (int64_t j = 0; j < count; ++j) {
            const int64_t pos = (tail ? len - count : 0) + j;
            const int64_t row = orc_pool_row(tables + b * table_stride, table_stride,
                                             block_size, block_count, pos);
            if (row < 0) return 0;
            uint16_t *kp = kpool + row * (int64_t)kv_width;
            uint16_t *vp = vpool + row * (int64_t)kv_width;
            uint16_t *kr = krows + (first + j) * (int64_t)kv_width;
            uint16_t *vr = vrows + (first + j) * (int64_t)kv_width;
            if (to_pool) {
                memcpy(kp, kr, kv_width * 2);
                memcpy(vp, vr, kv_width * 2);
            } else {
                memcpy(kr, kp, kv_width * 2);
                memcpy(vr, vp, kv_width * 2);
            }
        }
    }
    return 1;
}

/* Restatement of tensor_sdpa_f32's CPU branch on [B][H][L][d] arrays.
 * `scores` must hold Lq * Lk floats.  Returns 0 on shape errors. */
int orc_sdpa_f32(const float *q, const float *k, const float *v, const float *mask,
                 float *out, size_t batch, size_t q_heads, size_t kv_heads, size_t q_len,
                 size_t kv_len, size_t head_dim, size_t value_dim, float scale, int causal,
                 float *scores) {
    if (batch == 0 || q_heads == 0 || kv_heads == 0 || q_len == 0 || kv_len == 0 ||
        head_dim == 0 || value_dim == 0 || q_heads % kv_heads != 0 || !isfinite(scale))
        return 0;
    const size_t offset = kv_len > q_len ? kv_len - q_len : 0;
    const size_t group = q_heads / kv_heads;
    for (size_t bi = 0; bi < batch; ++bi) {
        for (size_t h = 0; h < q_heads; ++h) {
            const size_t g = h / group;
            const float *qh = q + (bi * q_heads + h) * q_len * head_dim;
            const float *kh = k + (bi * kv_heads + g) * kv_len * head_dim;
            const float *vh = v + (bi * kv_heads + g) * kv_len * value_dim;
            float *oh = out + (bi * q_heads + h) * q_len * value_dim;
            for (size_t i = 0; i < q_len; ++i) {
                float *row = scores + i * kv_len;
                float mx = -INFINITY;
                size_t n_inf = 0;
                for (size_t j = 0; j < kv_len; ++j) {
                    float s = 0.0f;
                    for (size_t d = 0; d < head_dim; ++d)
                        s += qh[i * head_dim + d] * kh[j * head_dim + d];
                    s *= scale;
                    if (mask) s += mask[i * kv_len + j];
                    if (causal && j > i + offset) s = -INFINITY;
                    row[j] = s;
                    if (s == INFINITY) ++n_inf;
                    if (s > mx) mx = s;
                }
                if (mx == -INFINITY || isnan(mx)) {
                    for (size_t d = 0; d < value_dim; ++d)
                        oh[i * value_dim + d] = mx == -INFINITY ? 0.0f : NAN;
                    if (mx == -INFINITY) memset(row, 0, kv_len * sizeof(float));
                    continue;
                }
                float den = 0.0f;
                if (n_inf == 0) {
                    for (size_t j = 0; j < kv_len; ++j) {
                        row[j] = expf(row[j] - mx);
                        den += row[j];
                    }
                } else {
                    den = (float)n_inf;
                    for (size_t j = 0; j < kv_len; ++j) row[j] = row[j] == INFINITY ? 1.0f : 0.0f;
                }
                for (size_t j = 0; j < kv_len; ++j) row[j] /= den;
            }
            /* Like the SDK, P.V runs for every row after all score rows are
             * done and overwrites what the early exit wrote: an all -inf row
             * (scores zeroed above) comes out as sum 0 * v. */
            for (size_t i = 0; i < q_len; ++i) {
                const float *row = scores + i * kv_len;
                for (size_t d = 0; d < value_dim; ++d) {
                    float acc = 0.0f;
                    for (size_t j = 0; j < kv_len; ++j) acc += row[j] * vh[j * value_dim + d];
                    oh[i * value_dim + d] = acc;
                }
            }
        }
    }
    return 1;
}

/* Paged attention for a list of query rows of ONE sequence.
 *   q_rows   [n_rows][q_heads][head_dim] 2-byte storage
 *   q_pos    absolute position of each row (causal: keys <= q_pos attend);
 *            the SDK's chunk rule is q_pos = seq_len - n_rows + i
 *   out      [n_rows][q_heads][head_dim] float
 * Each (row, head) runs through orc_sdpa_f32 with Lq = 1 and the key range
 * cut at q_pos + 1 when causal, which equals the SDK's masked row because
 * masked keys get weight exactly 0 (finite V rows assumed, as in the SDK's
 * own data).  Returns 0 on addressing errors or allocation failure. */
int orc_paged_attention_rows(const uint16_t *q_rows, const int64_t *q_pos, size_t n_rows,
                             int causal, int dtype, const uint16_t *kpool,
                             const uint16_t *vpool, size_t kv_heads, size_t head_dim,
                             size_t block_size, size_t block_count, const uint32_t *table_row,
                             size_t table_len, int64_t seq_len, size_t q_heads, float scale,
                             float *out) {
    if (kv_heads == 0 || q_heads % kv_heads != 0 || seq_len < 0) return 0;
    const size_t kv_width = kv_heads * head_dim, group = q_heads / kv_heads;
    const size_t L = (size_t)seq_len;
    float *kf = (float *)malloc((L ? L : 1) * head_dim * sizeof(float));
    float *vf = (float *)malloc((L ? L : 1) * head_dim * sizeof(float));
    float *qf = (float *)malloc(head_dim * sizeof(float));
    float *sc = (float *)malloc((L ? L : 1) * sizeof(float));
    float *of = (float *)malloc(head_dim * sizeof(float));
    int ok = kf && vf && qf && sc && of;
    for (size_t g = 0; ok && g < kv_heads; ++g) {
        for (size_t j = 0; ok && j < L; ++j) {
            const int64_t row = orc_pool_row(table_row, table_len, block_size, block_count,
                                             (int64_t)j);
            if (row < 0) { ok = 0; break; }
            for (size_t d = 0; d < head_dim; ++d) {
                kf[j * head_dim + d] = widen(kpool[row * (int64_t)kv_width + g * head_dim + d], dtype);
                vf[j * head_dim + d] = widen(vpool[row * (int64_t)kv_width + g * head_dim + d], dtype);
            }
        }
        for (size_t r = 0; ok && r < n_rows; ++r) {
            size_t lk = L;
            if (causal) {
                const int64_t lim = q_pos[r] + 1;
                lk = lim < 0 ? 0 : ((size_t)lim < L ? (size_t)lim : L);
            }
            for (size_t hh = 0; hh < group; ++hh) {
                const size_t h = g * group + hh;
                float *o = out + (r * q_heads + h) * head_dim;
                if (lk == 0) {  /* every key masked: the SDK writes zeros */
                    memset(o, 0, head_dim * sizeof(float));
                    continue;
                }
                for (size_t d = 0; d < head_dim; ++d)
                    qf[d] = widen(q_rows[(r * q_heads + h) * head_dim + d], dtype);
                if (!orc_sdpa_f32(qf, kf, vf, NULL, of, 1, 1, 1, 1, lk, head_dim, head_dim,
                                  scale, 0, sc)) { ok = 0; break; }
                memcpy(o, of, head_dim * sizeof(float));
            }
        }
    }
    free(kf); free(vf); free(qf); free(sc); free(of);
    return ok;
}
