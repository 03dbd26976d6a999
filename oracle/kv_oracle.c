/*
 * kv_oracle.c -- CPU oracle for the paged KV-cache path (TEST INFRASTRUCTURE).
 *
 * Checker only: the product never links or calls this file.  Built with
 *   gcc -O3 -march=x86-64-v3 -ffp-contract=off -fno-fast-math -pthread
 * (-march follows the reference's .cargo/config.toml:3-4; -ffp-contract=off
 * because Rust does not contract a*b+c).  Every restated function cites the
 * reference lines it follows; the comments give the Rust expression each C
 * line stands for.
 */
#include "kv_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

uint16_t orc_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u); /* quiet NaN */
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

float orc_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* IEEE binary16 <-> binary32, round to nearest even (the `half` crate's
 * f16::from_f32 / to_f32, which llm-quant uses for block scales). */
uint16_t orc_f32_to_f16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    const uint32_t sign = (u >> 16) & 0x8000u;
    const uint32_t ex = (u >> 23) & 0xffu;
    uint32_t man = u & 0x7fffffu;
    if (ex == 0xffu) return (uint16_t)(sign | 0x7c00u | (man ? 0x200u | (man >> 13) : 0u)); /* inf / nan */
    const int e = (int)ex - 127 + 15;                                                    /* rebiased */
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);                                       /* overflow: inf */
    if (e <= 0) {                                                                         /* subnormal or zero */
        if (e < -10) return (uint16_t)sign;
        man |= 0x800000u;                       /* implicit bit */
        const int shift = 14 - e;               /* 24-bit significand -> 10 - (1 - e) bits */
        uint32_t h = man >> shift;
        const uint32_t rem = man & ((1u << shift) - 1u), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1u))) ++h;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((uint32_t)e << 10) | (man >> 13);
    const uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h; /* may carry into the exponent: still right */
    return (uint16_t)(sign | h);
}

float orc_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t ex = (h >> 10) & 0x1fu, man = h & 0x3ffu;
    uint32_t u;
    if (ex == 0x1fu)
        u = sign | 0x7f800000u | (man << 13);
    else if (ex != 0)
        u = sign | ((ex - 15 + 127) << 23) | (man << 13);
    else if (man == 0)
        u = sign;
    else { /* subnormal: normalise */
        int e = -1;
        uint32_t m = man;
        do {
            ++e;
            m <<= 1;
        } while (!(m & 0x400u));
        u = sign | ((uint32_t)(127 - 15 - e) << 23) | ((m & 0x3ffu) << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* crates/llm-quant/src/lib.rs:26-36 (BlockQ8_0::quantize)
 *   amax = fold(0.0, |acc, v| acc.max(v.abs())); scale = f16::from_f32(amax / 127.0);
 *   inv = if scale_f == 0.0 { 0.0 } else { 1.0 / scale_f };
 *   q = (src * inv).round().clamp(-127.0, 127.0) as i8 */
void orc_quantize_q8_0(const float *src, uint16_t *scale, int8_t *qs) {
    float amax = 0.0f;
    for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(src[i]));
    const uint16_t sc = orc_f32_to_f16(amax / 127.0f);
    const float sf = orc_f16_to_f32(sc);
    const float inv = sf == 0.0f ? 0.0f : 1.0f / sf;
    for (int i = 0; i < 32; i++) {
        float q = roundf(src[i] * inv);
        q = q < -127.0f ? -127.0f : (q > 127.0f ? 127.0f : q);
        qs[i] = (int8_t)q;
    }
    *scale = sc;
}

/* crates/llm-quant/src/lib.rs:63-78 (BlockQ4::quantize): scale amax / 8,
 * q clamped to -8..7, element 2i in the low nibble of byte i, 2i + 1 high. */
void orc_quantize_q4(const float *src, uint16_t *scale, uint8_t *qs) {
    float amax = 0.0f;
    for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(src[i]));
    const uint16_t sc = orc_f32_to_f16(amax / 8.0f);
    const float sf = orc_f16_to_f32(sc);
    const float inv = sf == 0.0f ? 0.0f : 1.0f / sf;
    for (int i = 0; i < 16; i++) qs[i] = 0;
    for (int i = 0; i < 32; i++) {
        float q = roundf(src[i] * inv);
        q = q < -8.0f ? -8.0f : (q > 7.0f ? 7.0f : q);
        const uint8_t nib = (uint8_t)((int8_t)q) & 0x0fu;
        qs[i / 2] |= (i & 1) ? (uint8_t)(nib << 4) : nib;
    }
    *scale = sc;
}

/* BlockQ8_0::dequantize / BlockQ4::dequantize (lib.rs:40-45, 83-100):
 * f32::from(q) * scale. */
static inline float deq_q8(int8_t q, float scale) { return (float)q * scale; }
static inline float deq_q4(uint8_t packed, int hi, float scale) {
    const uint8_t nib = hi ? (uint8_t)(packed >> 4) : (uint8_t)(packed & 0x0fu);
    const int8_t v = (int8_t)(nib << 4) >> 4;
    return (float)v * scale;
}

/* rope.rs:6-14
 *   let dim_f = dim as f32;
 *   for i in (0..dim).step_by(2) { let expo = i as f32 / dim_f;
 *                                  out.push(1.0 / theta.powf(expo)); } */
void orc_inv_freq(size_t dim, float theta, float *out) {
    float dim_f = (float)dim;
    for (size_t i = 0; i < dim; i += 2) {
        float expo = (float)i / dim_f;
        out[i / 2] = 1.0f / powf(theta, expo);
    }
}

/* rope.rs:18-43
 *   let pos = (start + t) as f32; let freq = pos * inv_freq[i];
 *   cos[t*dim+i] = cos[t*dim+half+i] = freq.cos(); same for sin. */
void orc_cos_sin(const float *inv_freq, size_t start, size_t tokens, size_t dim,
                 float *cos_out, float *sin_out) {
    size_t half = dim / 2;
    for (size_t t = 0; t < tokens; t++) {
        float pos = (float)(start + t);
        for (size_t i = 0; i < half; i++) {
            float freq = pos * inv_freq[i];
            float c = cosf(freq);
            float s = sinf(freq);
            cos_out[t * dim + i] = c;
            cos_out[t * dim + half + i] = c;
            sin_out[t * dim + i] = s;
            sin_out[t * dim + half + i] = s;
        }
    }
}

/* rope.rs:46-81
 *   rotated = cat(-x[half:], x[:half]);  rotated[d] = q[d] * c[d] + rotated[d] * s[d]
 * Two roundings (product, product) and one for the sum: no FMA. */
void orc_apply_rope_in_place(float *states, const float *cos_t, const float *sin_t,
                             size_t heads, size_t tokens, size_t dim) {
    size_t half = dim / 2;
    float *rot = (float *)malloc(dim * sizeof(float));
    for (size_t h = 0; h < heads; h++) {
        for (size_t t = 0; t < tokens; t++) {
            float *q = states + (h * tokens + t) * dim;
            for (size_t i = 0; i < half; i++) {
                rot[i] = -q[half + i];
                rot[half + i] = q[i];
            }
            const float *c = cos_t + t * dim;
            const float *s = sin_t + t * dim;
            for (size_t d = 0; d < dim; d++) {
                float a = q[d] * c[d];
                float b = rot[d] * s[d];
                rot[d] = a + b;
            }
            memcpy(q, rot, dim * sizeof(float));
        }
    }
    free(rot);
}

/* ops.rs:64-79
 *   max = fold(NEG_INFINITY, f32::max); v = (v - max).exp(); sum += v;
 *   inv = if sum == 0.0 { 0.0 } else { 1.0 / sum }; v *= inv */
void orc_softmax_last_axis(float *logits, size_t len, size_t n) {
    if (n == 0) return; /* Rust's chunks_exact_mut(0) panics; callers never pass 0 */
    for (size_t r = 0; r + n <= len; r += n) {
        float *row = logits + r;
        float max = -INFINITY;
        for (size_t i = 0; i < n; i++) max = fmaxf(max, row[i]);
        float sum = 0.0f;
        for (size_t i = 0; i < n; i++) {
            row[i] = expf(row[i] - max);
            sum += row[i];
        }
        float inv = (sum == 0.0f) ? 0.0f : 1.0f / sum;
        for (size_t i = 0; i < n; i++) row[i] *= inv;
    }
}

/* lfm2.rs:1006-1056 (attention_decode_cached) */
void orc_attention_decode_cached(const float *q, const float *k_cache, const float *v_cache,
                                 size_t n_q, size_t n_kv, size_t kv_len, size_t kv_cap,
                                 size_t dim, const uint8_t *key_valid, size_t key_valid_len,
                                 float *scores, float *out) {
    /* let scale = (dim as f32).sqrt().recip(); */
    float scale = 1.0f / sqrtf((float)dim);
    size_t n_rep = n_q / n_kv;
    memset(out, 0, n_q * dim * sizeof(float));
    for (size_t qh = 0; qh < n_q; qh++) {
        size_t kv_h = qh / n_rep;
        const float *qv = q + qh * dim;
        float *row = scores + qh * kv_len;
        for (size_t s = 0; s < kv_len; s++) {
            /* if key_valid.get(s) == Some(&false) */
            if (key_valid && s < key_valid_len && !key_valid[s]) {
                row[s] = -INFINITY;
                continue;
            }
            const float *kv = k_cache + (kv_h * kv_cap + s) * dim;
            float acc = 0.0f;
            for (size_t d = 0; d < dim; d++) acc = fmaf(qv[d], kv[d], acc); /* mul_add */
            row[s] = acc * scale;
        }
        orc_softmax_last_axis(row, kv_len, kv_len);
        float *dst = out + qh * dim;
        for (size_t s = 0; s < kv_len; s++) {
            float w = row[s];
            if (w == 0.0f) continue;
            const float *vv = v_cache + (kv_h * kv_cap + s) * dim;
            for (size_t d = 0; d < dim; d++) dst[d] = fmaf(w, vv[d], dst[d]);
        }
    }
}

/* Which (query t, key s) pairs are masked.  EXPLICIT: !mask[t*kv_len+s];
 * FORWARD: lfm2.rs:1083 `(causal && s > t) || !key_valid[s]`; PREFIX: the
 * build's chunk after `prefix` cached keys (every cached key visible; chunk
 * key j = s - prefix visible when j <= t, or when bit j of bits[t] is set). */
enum { MASK_EXPLICIT, MASK_FORWARD, MASK_PREFIX };
typedef struct {
    int kind;
    const uint8_t *mask;      /* EXPLICIT */
    int causal;               /* FORWARD */
    const uint8_t *key_valid; /* FORWARD, may be NULL */
    size_t prefix;            /* PREFIX */
    const uint64_t *bits;     /* PREFIX: NULL = causal chunk */
} mask_desc;

static inline int is_masked(const mask_desc *m, size_t kv_len, size_t t, size_t s) {
    switch (m->kind) {
    case MASK_EXPLICIT:
        return !m->mask[t * kv_len + s];
    case MASK_FORWARD:
        return (m->causal && s > t) || (m->key_valid && !m->key_valid[s]);
    default:
        if (s < m->prefix) return 0;
        return m->bits ? !((m->bits[t] >> (s - m->prefix)) & 1u) : (s - m->prefix > t);
    }
}

/* One query head of attention_forward (lfm2.rs:1058-1111): q rows [q_len][dim],
 * the head's K and V [kv_len][dim], scores [q_len * kv_len] scratch; output row
 * t goes to out + t * out_stride.  Heads are independent in the reference's
 * loop, so running them one at a time gives the same bits. */
static void attention_one_head(const float *q, const float *k, const float *v, size_t q_len,
                               size_t kv_len, size_t dim, const mask_desc *m, float *scores,
                               float *out, size_t out_stride) {
    float scale = 1.0f / sqrtf((float)dim);
    for (size_t t = 0; t < q_len; t++) {
        const float *qv = q + t * dim;
        for (size_t s = 0; s < kv_len; s++) {
            if (is_masked(m, kv_len, t, s)) {
                scores[t * kv_len + s] = -INFINITY;
                continue;
            }
            const float *kv = k + s * dim;
            float acc = 0.0f;
            for (size_t d = 0; d < dim; d++) acc = fmaf(qv[d], kv[d], acc);
            scores[t * kv_len + s] = acc * scale;
        }
    }
    orc_softmax_last_axis(scores, q_len * kv_len, kv_len);
    for (size_t t = 0; t < q_len; t++) {
        float *dst = out + t * out_stride;
        memset(dst, 0, dim * sizeof(float));
        for (size_t s = 0; s < kv_len; s++) {
            float w = scores[t * kv_len + s];
            if (w == 0.0f) continue;
            const float *vv = v + s * dim;
            for (size_t d = 0; d < dim; d++) dst[d] = fmaf(w, vv[d], dst[d]);
        }
    }
}

/* Shared body of attention_forward (lfm2.rs:1058-1111) and attention_masked:
 * q [n_q, q_len, dim], k/v [n_kv, kv_len, dim], out [n_q, q_len, dim]. */
static void attention_rows(const float *q, const float *k, const float *v, size_t n_q,
                           size_t n_kv, size_t q_len, size_t kv_len, size_t dim, const mask_desc *m,
                           float *out) {
    size_t n_rep = n_q / n_kv;
    float *scores = (float *)malloc((q_len * kv_len + 1) * sizeof(float));
    for (size_t qh = 0; qh < n_q; qh++) {
        size_t kv_h = qh / n_rep;
        attention_one_head(q + qh * q_len * dim, k + kv_h * kv_len * dim, v + kv_h * kv_len * dim, q_len,
                           kv_len, dim, m, scores, out + qh * q_len * dim, dim);
    }
    free(scores);
}

/* lfm2.rs:1058-1111 (attention_forward) */
void orc_attention_forward(const float *q, const float *k, const float *v, size_t n_q,
                           size_t n_kv, size_t q_len, size_t kv_len, size_t dim, int causal,
                           const uint8_t *key_valid, float *out) {
    mask_desc m = {MASK_FORWARD, NULL, causal, key_valid, 0, NULL};
    attention_rows(q, k, v, n_q, n_kv, q_len, kv_len, dim, &m, out);
}

void orc_attention_masked(const float *q, const float *k, const float *v, size_t n_q,
                          size_t n_kv, size_t q_len, size_t kv_len, size_t dim,
                          const uint8_t *mask, float *out) {
    mask_desc m = {MASK_EXPLICIT, mask, 0, NULL, 0, NULL};
    attention_rows(q, k, v, n_q, n_kv, q_len, kv_len, dim, &m, out);
}

/* ---- paged layout (build-defined) ---------------------------------------- */

static inline float load_elem(const void *base, int dtype, size_t i) {
    if (dtype == ORC_BF16) return orc_bf16_to_f32(((const uint16_t *)base)[i]);
    if (dtype == ORC_F16) return orc_f16_to_f32(((const uint16_t *)base)[i]);
    return ((const float *)base)[i];
}

static inline void store_elem(void *base, int dtype, size_t i, float x) {
    if (dtype == ORC_BF16)
        ((uint16_t *)base)[i] = orc_f32_to_bf16(x);
    else if (dtype == ORC_F16)
        ((uint16_t *)base)[i] = orc_f32_to_f16(x);
    else
        ((float *)base)[i] = x;
}

/* ops.rs:8-23
 *   let inv_dim = 1.0 / dim as f64;
 *   for row: let mut sumsq = 0.0f64; for &v in row { sumsq += f64::from(v) * f64::from(v); }
 *            let scale = ((sumsq * inv_dim + f64::from(eps)).sqrt().recip()) as f32;
 *            *d = w * (v * scale); */
void orc_rms_norm(const float *x, const float *weight, float eps, size_t dim, size_t rows, float *out) {
    double inv_dim = 1.0 / (double)dim;
    for (size_t r = 0; r < rows; r++) {
        const float *row = x + r * dim;
        double sumsq = 0.0;
        for (size_t i = 0; i < dim; i++) sumsq += (double)row[i] * (double)row[i];
        float scale = (float)(1.0 / sqrt(sumsq * inv_dim + (double)eps));
        for (size_t i = 0; i < dim; i++) {
            float t = row[i] * scale;
            out[r * dim + i] = weight[i] * t;
        }
    }
}

/* Quantised pages (ORC_Q8: K and V as Q8_0 blocks; ORC_K8V4: K as Q8_0, V as
 * Q4), head_dim 64 = two 32-element blocks per (head, token).  A page is
 * n_kv head blocks, each holding in order: K codes [P][64] int8, V codes
 * [P][64] int8 (Q8) or [P][32] packed nibbles (K8V4), scales [P][2 blocks]
 * [K, V] f16.  Queries, outputs and the appended k/v stay bf16. */
static inline int is_quant(int dtype) { return dtype == ORC_Q8 || dtype == ORC_K8V4; }
/* Element type of the appended k / v, q and out: bf16 for quantised and half pages. */
static inline int io_dtype(int dtype) { return (is_quant(dtype) || dtype == ORC_F16) ? ORC_BF16 : dtype; }
static inline size_t q_vrow(int dtype) { return dtype == ORC_Q8 ? 64 : 32; }
size_t orc_page_bytes(int dtype, size_t n_kv, size_t P, size_t d) {
    if (is_quant(dtype)) return n_kv * P * (d + q_vrow(dtype) + 8);
    return 2 * n_kv * P * d * ((dtype == ORC_BF16 || dtype == ORC_F16) ? 2 : 4);
}
static inline size_t q_head(size_t P, int dtype, size_t h) { return h * P * (64 + q_vrow(dtype) + 8); }
static inline size_t q_koff(size_t n_kv, size_t P, int dtype, size_t h, size_t j) {
    (void)n_kv;
    return q_head(P, dtype, h) + j * 64;
}
static inline size_t q_voff(size_t n_kv, size_t P, int dtype, size_t h, size_t j) {
    (void)n_kv;
    return q_head(P, dtype, h) + P * 64 + j * q_vrow(dtype);
}
/* K scale of block 0 of token j; block b is 4 bytes on, V scale 2 on. */
static inline size_t q_ksoff(size_t n_kv, size_t P, int dtype, size_t h, size_t j) {
    (void)n_kv;
    return q_head(P, dtype, h) + P * (64 + q_vrow(dtype)) + j * 8;
}
static inline size_t q_vsoff(size_t n_kv, size_t P, int dtype, size_t h, size_t j) {
    return q_ksoff(n_kv, P, dtype, h, j) + 2;
}

/* One token's rotated K (fp32 [n_kv][64]) and V (bf16 bits) into a quantised page. */
static void q_store_token(uint8_t *page, int dtype, size_t n_kv, size_t P, size_t j, const float *kr,
                          const void *v_raw) {
    for (size_t h = 0; h < n_kv; h++) {
        float vv[64];
        for (int e = 0; e < 64; e++) vv[e] = orc_bf16_to_f32(((const uint16_t *)v_raw)[h * 64 + e]);
        for (int b = 0; b < 2; b++) {
            uint16_t sc;
            orc_quantize_q8_0(kr + h * 64 + 32 * b, &sc, (int8_t *)(page + q_koff(n_kv, P, dtype, h, j) + 32 * b));
            memcpy(page + q_ksoff(n_kv, P, dtype, h, j) + 4 * b, &sc, 2);
            if (dtype == ORC_Q8)
                orc_quantize_q8_0(vv + 32 * b, &sc, (int8_t *)(page + q_voff(n_kv, P, dtype, h, j) + 32 * b));
            else
                orc_quantize_q4(vv + 32 * b, &sc, page + q_voff(n_kv, P, dtype, h, j) + 16 * b);
            memcpy(page + q_vsoff(n_kv, P, dtype, h, j) + 4 * b, &sc, 2);
        }
    }
}

/* Dequantised K and V of (head h, slot j) of a quantised page into fp32 rows. */
static void q_load_token(const uint8_t *page, int dtype, size_t n_kv, size_t P, size_t h, size_t j, float *kd,
                         float *vd) {
    for (int b = 0; b < 2; b++) {
        uint16_t ks, vs;
        memcpy(&ks, page + q_ksoff(n_kv, P, dtype, h, j) + 4 * b, 2);
        memcpy(&vs, page + q_vsoff(n_kv, P, dtype, h, j) + 4 * b, 2);
        const float kf = orc_f16_to_f32(ks), vf = orc_f16_to_f32(vs);
        const int8_t *kq = (const int8_t *)(page + q_koff(n_kv, P, dtype, h, j)) + 32 * b;
        for (int e = 0; e < 32; e++) kd[32 * b + e] = deq_q8(kq[e], kf);
        if (dtype == ORC_Q8) {
            const int8_t *vq = (const int8_t *)(page + q_voff(n_kv, P, dtype, h, j)) + 32 * b;
            for (int e = 0; e < 32; e++) vd[32 * b + e] = deq_q8(vq[e], vf);
        } else {
            const uint8_t *vq = page + q_voff(n_kv, P, dtype, h, j) + 16 * b;
            for (int e = 0; e < 32; e++) vd[32 * b + e] = deq_q4(vq[e / 2], e & 1, vf);
        }
    }
}

/* k_norm non-NULL: lfm2.rs:805-812 rms_norm_heads on k (heads = n_kv) first. */
static void append_token_impl(void *pages, int dtype, size_t n_kv, size_t P, size_t d, const uint32_t *bt,
                              size_t slot, const void *k_raw, const void *v, const float *cos_row,
                              const float *sin_row, const float *k_norm, float eps) {
    size_t page_elems = 2 * n_kv * P * d;
    uint32_t page = bt[slot / P];
    size_t j = slot % P;
    float *kr = (float *)malloc(n_kv * d * sizeof(float));
    for (size_t i = 0; i < n_kv * d; i++) kr[i] = load_elem(k_raw, io_dtype(dtype), i);
    if (k_norm) orc_rms_norm(kr, k_norm, eps, d, n_kv, kr);
    /* lfm2.rs:816-825: RoPE on k (heads = n_kv, tokens = 1) before the store
     * at lfm2.rs:828-832. */
    orc_apply_rope_in_place(kr, cos_row, sin_row, n_kv, 1, d);
    if (is_quant(dtype)) {
        q_store_token((uint8_t *)pages + (size_t)page * orc_page_bytes(dtype, n_kv, P, d), dtype, n_kv, P, j, kr,
                      v);
        free(kr);
        return;
    }
    for (size_t h = 0; h < n_kv; h++) {
        size_t kofs = (size_t)page * page_elems + (h * P + j) * d;
        size_t vofs = (size_t)page * page_elems + ((n_kv + h) * P + j) * d;
        for (size_t e = 0; e < d; e++) {
            store_elem(pages, dtype, kofs + e, kr[h * d + e]);
            store_elem(pages, dtype, vofs + e, load_elem(v, io_dtype(dtype), h * d + e));
        }
    }
    free(kr);
}

void orc_paged_append_token(void *pages, int dtype, size_t n_kv, size_t P, size_t d,
                            const uint32_t *bt, size_t slot, const void *k_raw,
                            const void *v, const float *cos_row, const float *sin_row) {
    append_token_impl(pages, dtype, n_kv, P, d, bt, slot, k_raw, v, cos_row, sin_row, NULL, 0.f);
}

/* Tokens [t0, t1) of KV heads [h0, h1) of one sequence into fp32
 * [h1 - h0, t1 - t0, d]; pages marked ORC_PAGE_NONE read as zero. */
static void gather_range(const void *pages, int dtype, size_t n_kv, size_t P, size_t d,
                         const uint32_t *bt, size_t t0, size_t t1, size_t h0, size_t h1,
                         float *k_out, float *v_out) {
    size_t page_elems = 2 * n_kv * P * d;
    size_t n_tokens = t1 - t0;
    for (size_t t = t0; t < t1; t++) {
        uint32_t page = bt[t / P];
        size_t j = t % P;
        for (size_t h = h0; h < h1; h++) {
            float *kd = k_out + ((h - h0) * n_tokens + (t - t0)) * d;
            float *vd = v_out + ((h - h0) * n_tokens + (t - t0)) * d;
            if (page == ORC_PAGE_NONE) {
                memset(kd, 0, d * sizeof(float));
                memset(vd, 0, d * sizeof(float));
                continue;
            }
            if (is_quant(dtype)) {
                q_load_token((const uint8_t *)pages + (size_t)page * orc_page_bytes(dtype, n_kv, P, d), dtype, n_kv, P,
                             h, j, kd, vd);
                continue;
            }
            size_t kofs = (size_t)page * page_elems + (h * P + j) * d;
            size_t vofs = (size_t)page * page_elems + ((n_kv + h) * P + j) * d;
            for (size_t e = 0; e < d; e++) {
                kd[e] = load_elem(pages, dtype, kofs + e);
                vd[e] = load_elem(pages, dtype, vofs + e);
            }
        }
    }
}

void orc_paged_gather(const void *pages, int dtype, size_t n_kv, size_t P, size_t d,
                      const uint32_t *bt, size_t n_tokens, float *k_out, float *v_out) {
    gather_range(pages, dtype, n_kv, P, d, bt, 0, n_tokens, 0, n_kv, k_out, v_out);
}

/* q_norm non-NULL: lfm2.rs:797-804 rms_norm_heads on q (heads = n_q) first. */
static void paged_decode_impl(const void *pages, int dtype, size_t n_q, size_t n_kv, size_t P, size_t d,
                              const uint32_t *bt, size_t seq_len, size_t window, const void *q_raw,
                              const float *inv_freq, float *out, const float *q_norm, float eps) {
    if (seq_len == 0) { /* build-defined: an empty sequence attends to nothing */
        memset(out, 0, n_q * d * sizeof(float));
        return;
    }
    /* Keys below the window are masked (score -inf).  In attention_decode_cached
     * such a key leaves the max fold unchanged (fmaxf(m, -inf) = m), adds
     * expf(-inf) = +0 to the sum (x + 0 = x for the non-negative partial sums)
     * and is skipped by the PV loop (w == 0), so attending over the keys
     * [lo, seq_len) alone, in the same order, gives the same bits as the
     * masked row.  The gather then never touches evicted pages, and a 128k-token
     * session under a 32k window costs a quarter of the work. */
    size_t lo = (window > 0 && seq_len > window) ? seq_len - window : 0;
    size_t n_att = seq_len - lo;
    float *k = (float *)malloc(n_kv * n_att * d * sizeof(float));
    float *v = (float *)malloc(n_kv * n_att * d * sizeof(float));
    float *q = (float *)malloc(n_q * d * sizeof(float));
    float *cs = (float *)malloc(2 * d * sizeof(float));
    float *scores = (float *)malloc(n_q * n_att * sizeof(float));
    gather_range(pages, dtype, n_kv, P, d, bt, lo, seq_len, 0, n_kv, k, v);
    for (size_t i = 0; i < n_q * d; i++) q[i] = load_elem(q_raw, io_dtype(dtype), i);
    if (q_norm) orc_rms_norm(q, q_norm, eps, d, n_q, q);
    /* lfm2.rs:816-822: cos_sin at pos, RoPE on q with heads = n_q, tokens = 1 */
    orc_cos_sin(inv_freq, seq_len - 1, 1, d, cs, cs + d);
    orc_apply_rope_in_place(q, cs, cs + d, n_q, 1, d);
    orc_attention_decode_cached(q, k, v, n_q, n_kv, n_att, n_att, d, NULL, 0, scores, out);
    free(scores);
    free(cs);
    free(q);
    free(v);
    free(k);
}

void orc_paged_decode(const void *pages, int dtype, size_t n_q, size_t n_kv, size_t P,
                      size_t d, const uint32_t *bt, size_t seq_len, size_t window,
                      const void *q_raw, const float *inv_freq, float *out) {
    paged_decode_impl(pages, dtype, n_q, n_kv, P, d, bt, seq_len, window, q_raw, inv_freq, out, NULL, 0.f);
}

/* One sequence of orc_decode_step. */
typedef struct {
    void *pages;
    int dtype;
    size_t n_q, n_kv, P, d, bt_stride, n_seqs, window;
    const uint32_t *bt;
    const int32_t *seq_lens;
    const void *q_raw, *k_raw, *v;
    const float *inv_freq;
    float *out;
    atomic_long next;
    const float *q_norm, *k_norm;  /* NULL: no RMSNorm */
    float eps;
} step_job;

static void step_one(step_job *j, size_t s) {
    size_t esz = io_dtype(j->dtype) == ORC_BF16 ? 2 : 4;
    size_t len = (size_t)j->seq_lens[s];
    const uint32_t *row = j->bt + s * j->bt_stride;
    if (len > 0) {
        float cs[2 * 256];
        orc_cos_sin(j->inv_freq, len - 1, 1, j->d, cs, cs + j->d);
        append_token_impl(j->pages, j->dtype, j->n_kv, j->P, j->d, row, len - 1,
                          (const char *)j->k_raw + s * j->n_kv * j->d * esz,
                          (const char *)j->v + s * j->n_kv * j->d * esz, cs, cs + j->d, j->k_norm, j->eps);
    }
    paged_decode_impl(j->pages, j->dtype, j->n_q, j->n_kv, j->P, j->d, row, len, j->window,
                      (const char *)j->q_raw + s * j->n_q * j->d * esz, j->inv_freq,
                      j->out + s * j->n_q * j->d, j->q_norm, j->eps);
}

static void *step_worker(void *arg) {
    step_job *j = (step_job *)arg;
    for (;;) {
        long s = atomic_fetch_add(&j->next, 1);
        if (s >= (long)j->n_seqs) break;
        step_one(j, (size_t)s);
    }
    return NULL;
}

static void run_steps(step_job *j, int n_threads);

void orc_decode_step(void *pages, int dtype, size_t n_q, size_t n_kv, size_t P, size_t d,
                     const uint32_t *bt, size_t bt_stride, const int32_t *seq_lens,
                     size_t n_seqs, size_t window, const void *q_raw, const void *k_raw,
                     const void *v, const float *inv_freq, float *out, int n_threads) {
    step_job j = {pages, dtype, n_q, n_kv, P, d, bt_stride, n_seqs, window, bt, seq_lens,
                  q_raw, k_raw, v, inv_freq, out, 0, NULL, NULL, 0.f};
    run_steps(&j, n_threads);
}

void orc_decode_step_norm(void *pages, int dtype, size_t n_q, size_t n_kv, size_t P, size_t d,
                          const uint32_t *bt, size_t bt_stride, const int32_t *seq_lens,
                          size_t n_seqs, size_t window, const void *q_raw, const void *k_raw,
                          const void *v, const float *inv_freq, const float *q_norm,
                          const float *k_norm, float eps, float *out, int n_threads) {
    step_job j = {pages, dtype, n_q, n_kv, P, d, bt_stride, n_seqs, window, bt, seq_lens,
                  q_raw, k_raw, v, inv_freq, out, 0, q_norm, k_norm, eps};
    run_steps(&j, n_threads);
}

static void run_steps(step_job *j, int n_threads) {
    size_t n_seqs = j->n_seqs;
    int nt = n_threads > 0 ? n_threads : orc_max_threads();
    if (nt > (int)n_seqs) nt = (int)n_seqs;
    if (nt <= 1) {
        for (size_t s = 0; s < n_seqs; s++) step_one(j, s);
        return;
    }
    pthread_t *th = (pthread_t *)malloc((size_t)nt * sizeof(pthread_t));
    for (int i = 0; i < nt; i++) pthread_create(&th[i], NULL, step_worker, j);
    for (int i = 0; i < nt; i++) pthread_join(th[i], NULL);
    free(th);
}

/* ---- bulk helpers for large parity cases -------------------------------- */

/* Run fn(ctx, i) for i in [0, n) on nt POSIX threads (dynamic assignment). */
typedef struct {
    void (*fn)(void *, size_t);
    void *ctx;
    size_t n;
    atomic_long next;
} par_job;

static void *par_worker(void *arg) {
    par_job *j = (par_job *)arg;
    for (;;) {
        long i = atomic_fetch_add(&j->next, 1);
        if (i >= (long)j->n) break;
        j->fn(j->ctx, (size_t)i);
    }
    return NULL;
}

static void par_for(size_t n, int n_threads, void (*fn)(void *, size_t), void *ctx) {
    int nt = n_threads > 0 ? n_threads : orc_max_threads();
    if ((size_t)nt > n) nt = (int)n;
    if (nt <= 1) {
        for (size_t i = 0; i < n; i++) fn(ctx, i);
        return;
    }
    par_job j = {fn, ctx, n, 0};
    pthread_t *th = (pthread_t *)malloc((size_t)nt * sizeof(pthread_t));
    for (int i = 0; i < nt; i++) pthread_create(&th[i], NULL, par_worker, &j);
    for (int i = 0; i < nt; i++) pthread_join(th[i], NULL);
    free(th);
}

typedef struct {
    void *pages;
    int dtype;
    size_t n_kv, P, d, bt_stride;
    const uint32_t *bt;
    const int32_t *tok_row, *tok_slot, *tok_pos;
    const void *k_raw, *v;
    const float *inv_freq;
} append_bulk;

static void append_bulk_one(void *arg, size_t i) {
    const append_bulk *a = (const append_bulk *)arg;
    size_t esz = io_dtype(a->dtype) == ORC_BF16 ? 2 : 4;
    float cs[2 * 256];
    orc_cos_sin(a->inv_freq, (size_t)a->tok_pos[i], 1, a->d, cs, cs + a->d);
    append_token_impl(a->pages, a->dtype, a->n_kv, a->P, a->d, a->bt + (size_t)a->tok_row[i] * a->bt_stride,
                      (size_t)a->tok_slot[i], (const char *)a->k_raw + i * a->n_kv * a->d * esz,
                      (const char *)a->v + i * a->n_kv * a->d * esz, cs, cs + a->d, NULL, 0.f);
}

void orc_paged_append_tokens(void *pages, int dtype, size_t n_kv, size_t P, size_t d, const uint32_t *bt,
                             size_t bt_stride, const int32_t *tok_row, const int32_t *tok_slot,
                             const int32_t *tok_pos, size_t n_tokens, const void *k_raw, const void *v,
                             const float *inv_freq, int n_threads) {
    append_bulk a = {pages, dtype, n_kv, P, d, bt_stride, bt, tok_row, tok_slot, tok_pos, k_raw, v, inv_freq};
    par_for(n_tokens, n_threads, append_bulk_one, &a);
}

typedef struct {
    const void *pages;
    int dtype;
    size_t n_q, n_kv, P, d, bt_stride;
    const uint32_t *bt;
    const int32_t *cached, *q_off, *q_pos;
    const uint64_t *masks;
    const void *q_raw;
    const float *inv_freq;
    float *out;
} prefill_bulk;

/* One (sequence, KV head) of orc_paged_prefill: the head's K/V gathered once,
 * then each of its query heads through attention_one_head. */
static void prefill_one(void *arg, size_t job) {
    const prefill_bulk *a = (const prefill_bulk *)arg;
    size_t s = job / a->n_kv, kh = job % a->n_kv;
    size_t L = (size_t)a->cached[s];
    size_t q0 = (size_t)a->q_off[s], T = (size_t)a->q_off[s + 1] - q0;
    if (T == 0) return;
    size_t n = L + T, d = a->d, g = a->n_q / a->n_kv;
    float *kh_rows = (float *)malloc(n * d * sizeof(float));
    float *vh_rows = (float *)malloc(n * d * sizeof(float));
    float *q = (float *)malloc(T * d * sizeof(float));
    float *scores = (float *)malloc(T * n * sizeof(float));
    float cs[2 * 256];
    gather_range(a->pages, a->dtype, a->n_kv, a->P, d, a->bt + s * a->bt_stride, 0, n, kh, kh + 1, kh_rows,
                 vh_rows);
    mask_desc m = {MASK_PREFIX, NULL, 0, NULL, L, a->masks ? a->masks + q0 : NULL};
    for (size_t qh = kh * g; qh < (kh + 1) * g; qh++) {
        for (size_t t = 0; t < T; t++) {
            const void *src = a->q_raw;
            size_t base = ((q0 + t) * a->n_q + qh) * d;
            for (size_t e = 0; e < d; e++) q[t * d + e] = load_elem(src, io_dtype(a->dtype), base + e);
            /* RoPE of one token's head at its position (rope.rs:56-81, heads = tokens = 1) */
            orc_cos_sin(a->inv_freq, (size_t)a->q_pos[q0 + t], 1, d, cs, cs + d);
            orc_apply_rope_in_place(q + t * d, cs, cs + d, 1, 1, d);
        }
        attention_one_head(q, kh_rows, vh_rows, T, n, d, &m, scores,
                           a->out + (q0 * a->n_q + qh) * d, a->n_q * d);
    }
    free(scores);
    free(q);
    free(vh_rows);
    free(kh_rows);
}

void orc_paged_prefill(const void *pages, int dtype, size_t n_q, size_t n_kv, size_t P, size_t d,
                       const uint32_t *bt, size_t bt_stride, size_t n_seqs, const int32_t *cached,
                       const int32_t *q_off, const int32_t *q_pos, const uint64_t *masks, const void *q_raw,
                       const float *inv_freq, float *out, int n_threads) {
    prefill_bulk a = {pages, dtype, n_q, n_kv, P, d, bt_stride, bt, cached, q_off, q_pos, masks, q_raw,
                      inv_freq, out};
    par_for(n_seqs * n_kv, n_threads, prefill_one, &a);
}

int orc_max_threads(void) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}
