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
 *   orc_decode_sequence
 *       the SDK's greedy paged decoder loop (attention_cuda.cu:754-1090:
 *       RMSNorm, GEMVs, RoPE on q and the stored k, softmax attention,
 *       SwiGLU, argmax), rounding to the storage type where the SDK does.
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

/* ------------------------------------------------------------------------
 * orc_decode_sequence -- greedy decoding of one sequence through the SDK's
 * dense decoder stack, restating decode_sequence_impl
 * (attention_cuda.cu:754-1090) and its kernels on the CPU:
 *   embedding row (:100-104); RMSNorm x * (1/sqrt(mean(x^2) + eps)) * w
 *   (:106-124); GEMV with FP32 sums (:126-163; quantised Q8_0/Q4_0 blocks
 *   :197-213, scale * q exactly); RoPE over split halves with angle
 *   position / theta^(2f/d) applied to q and to the stored k, v stored as
 *   is (:307-341); scores q.k * (1/sqrt(d)), softmax with the all-non-finite
 *   rule and expf (:343-379), P.V (:381-398); o-projection + residual, the
 *   quantised path rounding the product first (:293-299, :1040-1046);
 *   SwiGLU g / (1 + expf(-g)) * u (:165-195); final norm, lm_head, first
 *   strict argmax (:400-410).  Every value the SDK stores in T (float for
 *   F32 storage, half otherwise) is rounded to T here at the same point.
 *   Sums are sequential; the GPU's are tree-shaped, so the two agree to
 *   FP32 rounding.
 * storage 0 = F32, 1 = F16, 2 = quantised F16 (fmt 1 = Q8_0, 2 = Q4_0).
 * layers: per layer 9 pointers (input_norm, q, k, v, o, post_norm, gate, up,
 * down).  kcache/vcache: per layer [capacity][kv_width] in T, positions
 * [0, past) hold the prefix; positions [past, past + count) are written.
 * all_logits (optional, token_count * vocab floats): every step's logits.
 * ------------------------------------------------------------------------ */
static int dec_storage;
static float dec_ld(const void *p, size_t i) {
    return dec_storage == 0 ? ((const float *)p)[i] : orc_f16_to_f32(((const uint16_t *)p)[i]);
}
static float dec_rt(float v) { return dec_storage == 0 ? v : orc_f16_to_f32(orc_f32_to_f16(v)); }
static void dec_st(void *p, size_t i, float v) {
    if (dec_storage == 0) ((float *)p)[i] = v;
    else ((uint16_t *)p)[i] = orc_f32_to_f16(v);
}

static void dec_rms(const float *x, const void *w, float *y, size_t n, float eps) {
    float sum = 0.0f;
    for (size_t i = 0; i < n; ++i) sum = fmaf(x[i], x[i], sum);
    const float scale = 1.0f / sqrtf(sum / (float)n + eps);
    for (size_t i = 0; i < n; ++i) y[i] = dec_rt(x[i] * scale * dec_ld(w, i));
}

/* one row's FP32 sum */
static float dec_dot(const void *m, int fmt, size_t row, const float *x, size_t in) {
    float sum = 0.0f;
    if (fmt == 0) {
        for (size_t i = 0; i < in; ++i) sum = fmaf(x[i], dec_ld(m, row * in + i), sum);
        return sum;
    }
    const size_t bb = fmt == 1 ? 34 : 18, nb = in / 32;
    const uint8_t *w = (const uint8_t *)m + row * nb * bb;
    for (size_t b = 0; b < nb; ++b) {
        const uint8_t *blk = w + b * bb;
        const float scale = orc_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
        for (size_t k = 0; k < 32; ++k) {
            int q;
            if (fmt == 1) q = (int)(int8_t)blk[2 + k];
            else {
                const uint8_t packed = blk[2 + (k & 15)];
                q = (int)(k < 16 ? packed & 15 : packed >> 4) - 8;
            }
            sum = fmaf(x[b * 32 + k], scale * (float)q, sum);
        }
    }
    return sum;
}

int orc_decode_sequence(int storage, int fmt, const void *const *layers, size_t layer_count,
                        const void *embedding, uint32_t initial_token, size_t token_count,
                        uint32_t *generated, void *const *kcache, void *const *vcache,
                        size_t past, size_t capacity, size_t hidden, size_t inter, size_t qh,
                        size_t kvh, size_t hd, float eps, double theta, const void *final_norm,
                        const void *lm_head, size_t vocab, float *all_logits) {
    if (storage < 0 || storage > 2 || qh * hd != hidden || qh % kvh || hd % 2 ||
        past + token_count > capacity || (storage == 2 && fmt != 1 && fmt != 2))
        return 0;
    dec_storage = storage;
    const int wf = storage == 2 ? fmt : 0;
    const size_t kvw = kvh * hd, qkvw = hidden + 2 * kvw, group = qh / kvh;
    float *x = malloc(hidden * 4), *n = malloc(hidden * 4), *qkv = malloc(qkvw * 4);
    float *q = malloc(hidden * 4), *att = malloc(hidden * 4), *r = malloc(hidden * 4);
    float *act = malloc(inter * 4), *logits = malloc(vocab * 4);
    float *scores = malloc((past + token_count) * 4);
    if (!x || !n || !qkv || !q || !att || !r || !act || !logits || !scores) return 0;
    const float ftheta = (float)theta, scale = 1.0f / sqrtf((float)hd);
    uint32_t token = initial_token;
    for (size_t t = 0; t < token_count; ++t) {
        const size_t pos = past + t, len = pos + 1;
        for (size_t i = 0; i < hidden; ++i) x[i] = dec_ld(embedding, (size_t)token * hidden + i);
        for (size_t l = 0; l < layer_count; ++l) {
            const void *const *w = layers + 9 * l;
            dec_rms(x, w[0], n, hidden, eps);
            for (size_t o = 0; o < qkvw; ++o) {
                const void *m = o < hidden ? w[1] : (o < hidden + kvw ? w[2] : w[3]);
                const size_t row = o < hidden ? o : (o < hidden + kvw ? o - hidden : o - hidden - kvw);
                qkv[o] = dec_rt(dec_dot(m, wf, row, n, hidden));
            }
            const size_t half = hd / 2;
            for (size_t i = 0; i < (hidden > kvw ? hidden : kvw); ++i) {
                const size_t dim = i % hd, base = i - dim;
                const size_t paired = base + (dim < half ? dim + half : dim - half);
                const size_t freq = dim < half ? dim : dim - half;
                const float angle = (float)pos / powf(ftheta, 2.0f * (float)freq / (float)hd);
                const float sign = dim < half ? -1.0f : 1.0f;
                if (i < hidden) q[i] = dec_rt(qkv[i] * cosf(angle) + sign * qkv[paired] * sinf(angle));
                if (i < kvw) {
                    const float *k = qkv + hidden;
                    dec_st(kcache[l], pos * kvw + i, k[i] * cosf(angle) + sign * k[paired] * sinf(angle));
                    dec_st(vcache[l], pos * kvw + i, qkv[hidden + kvw + i]);
                }
            }
            for (size_t h = 0; h < qh; ++h) {
                const size_t g = h / group;
                float mx = -INFINITY;
                for (size_t p = 0; p < len; ++p) {
                    float s = 0.0f;
                    for (size_t d = 0; d < hd; ++d)
                        s = fmaf(q[h * hd + d], dec_ld(kcache[l], p * kvw + g * hd + d), s);
                    scores[p] = s * scale;
                    mx = fmaxf(mx, scores[p]);
                }
                if (!isfinite(mx)) {
                    for (size_t p = 0; p < len; ++p) scores[p] = 0.0f;
                } else {
                    float sum = 0.0f;
                    for (size_t p = 0; p < len; ++p) {
                        scores[p] = expf(scores[p] - mx);
                        sum += scores[p];
                    }
                    const float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
                    for (size_t p = 0; p < len; ++p) scores[p] *= inv;
                }
                for (size_t d = 0; d < hd; ++d) {
                    float s = 0.0f;
                    for (size_t p = 0; p < len; ++p)
                        s = fmaf(scores[p], dec_ld(vcache[l], p * kvw + g * hd + d), s);
                    att[h * hd + d] = dec_rt(s);
                }
            }
            for (size_t o = 0; o < hidden; ++o) {
                float v = dec_dot(w[4], wf, o, att, hidden);
                if (wf) v = dec_rt(v);
                r[o] = dec_rt(v + x[o]);
            }
            dec_rms(r, w[5], n, hidden, eps);
            for (size_t o = 0; o < inter; ++o) {
                const float g = dec_dot(w[6], wf, o, n, hidden);
                const float u = dec_dot(w[7], wf, o, n, hidden);
                act[o] = dec_rt(g / (1.0f + expf(-g)) * u);
            }
            for (size_t o = 0; o < hidden; ++o) {
                float v = dec_dot(w[8], wf, o, act, inter);
                if (wf) v = dec_rt(v);
                x[o] = dec_rt(v + r[o]);
            }
        }
        dec_rms(x, final_norm, n, hidden, eps);
        for (size_t o = 0; o < vocab; ++o) logits[o] = dec_rt(dec_dot(lm_head, wf, o, n, hidden));
        size_t best = 0;
        float maximum = logits[0];
        for (size_t i = 1; i < vocab; ++i)
            if (logits[i] > maximum) {
                maximum = logits[i];
                best = i;
            }
        token = (uint32_t)best;
        generated[t] = token;
        if (all_logits) memcpy(all_logits + t * vocab, logits, vocab * 4);
    }
    free(x); free(n); free(qkv); free(q); free(att); free(r); free(act); free(logits); free(scores);
    return 1;
}
