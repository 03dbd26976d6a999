/*
 * kv_oracle.h -- CPU oracle for the paged KV-cache path (TEST INFRASTRUCTURE).
 *
 * This library is the checker, never the product: only tests, the smoke check
 * and bench.py's CPU-baseline / reference arm may load it.  It restates, in C
 * with the same operation order, the reference's std-only Rust attention math:
 *
 *   rope.rs      crates/llm-cpu/src/rope.rs:6-81      inv_freq, cos_sin, rotate_half
 *   ops.rs       crates/llm-cpu/src/ops.rs:64-79      softmax_last_axis
 *   lfm2.rs      crates/llm-engine/src/lfm2.rs:1006-1111
 *                attention_decode_cached, attention_forward
 *
 * Rust's f32::{exp,cos,sin,powf} call the platform libm, so glibc's expf /
 * cosf / sinf / powf give the reference's own values on Linux-gnu.  Rust never
 * contracts a*b+c into an FMA, and f32::mul_add is fmaf: the library is built
 * with -ffp-contract=off and calls fmaf explicitly where the reference calls
 * mul_add.
 *
 * The paged helpers (orc_paged_*) are build-defined: the reference has no
 * paged KV (crates/llm-engine/src/cache.rs:1-51 is an occupancy placeholder).
 * They gather K/V through a block table into the reference's contiguous
 * [n_kv, cap, d] layout (lfm2.rs:188-203) and then call the restated
 * functions unchanged, so the paged result is the reference's result on the
 * gathered cache.
 */
#ifndef KV_ORACLE_H
#define KV_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Page storage.  ORC_F16: K and V as IEEE half in the bf16 page layout, with
 * bf16 k / v / q inputs (the library's KV_DTYPE_F16; the reference's tag F16). */
enum { ORC_F32 = 0, ORC_BF16 = 1, ORC_Q8 = 2, ORC_K8V4 = 3, ORC_F16 = 4 };
#define ORC_PAGE_NONE 0xFFFFFFFFu

/* bf16 <-> f32, round to nearest even (the build's bf16 storage rule). */
uint16_t orc_f32_to_bf16(float f);
float orc_bf16_to_f32(uint16_t h);

/* IEEE binary16 <-> binary32, round to nearest even. */
uint16_t orc_f32_to_f16(float f);
float orc_f16_to_f32(uint16_t h);
/* crates/llm-quant/src/lib.rs:26-36 and :63-78: one 32-element block. */
void orc_quantize_q8_0(const float *src, uint16_t *scale, int8_t *qs);
void orc_quantize_q4(const float *src, uint16_t *scale, uint8_t *qs);
/* Bytes of one page: quantised pages (ORC_Q8, ORC_K8V4) hold per (head,
 * token) the K codes, the V codes and two f16 scales each (see kv_oracle.c). */
size_t orc_page_bytes(int dtype, size_t n_kv, size_t P, size_t d);

/* rope.rs:6-14 */
void orc_inv_freq(size_t dim, float theta, float *out);
/* rope.rs:18-43 ; cos/sin are [tokens, dim] */
void orc_cos_sin(const float *inv_freq, size_t start, size_t tokens, size_t dim,
                 float *cos_out, float *sin_out);
/* rope.rs:46-81 ; states is [heads, tokens, dim] */
void orc_apply_rope_in_place(float *states, const float *cos_t, const float *sin_t,
                             size_t heads, size_t tokens, size_t dim);
/* ops.rs:64-79 ; logits is [len / n, n] */
void orc_softmax_last_axis(float *logits, size_t len, size_t n);

/* lfm2.rs:1006-1056.  key_valid may be NULL (all valid) or hold key_valid_len
 * flags; a position >= key_valid_len counts as valid (`key_valid.get(s)`).
 * scores is [n_q, kv_len] scratch; out is [n_q, dim]. */
void orc_attention_decode_cached(const float *q, const float *k_cache, const float *v_cache,
                                 size_t n_q, size_t n_kv, size_t kv_len, size_t kv_cap,
                                 size_t dim, const uint8_t *key_valid, size_t key_valid_len,
                                 float *scores, float *out);

/* lfm2.rs:1058-1111.  q [n_q, q_len, dim]; k/v [n_kv, kv_len, dim]; key_valid
 * NULL or [kv_len]; out [n_q, q_len, dim]. */
void orc_attention_forward(const float *q, const float *k, const float *v, size_t n_q,
                           size_t n_kv, size_t q_len, size_t kv_len, size_t dim, int causal,
                           const uint8_t *key_valid, float *out);

/* Same operation order as attention_forward, with an explicit [q_len, kv_len]
 * mask (1 = attend) in place of `causal` and `key_valid`.  This is how the
 * build states chunked-prefill masks (s > q_start + t masked) and tree-verify
 * masks (ancestor-or-self), which the reference does not have. */
void orc_attention_masked(const float *q, const float *k, const float *v, size_t n_q,
                          size_t n_kv, size_t q_len, size_t kv_len, size_t dim,
                          const uint8_t *mask, float *out);

/* ---- build-defined paged layout ------------------------------------------
 * Page p starts at element p * 2 * n_kv * P * d.  Inside a page: the K block
 * [n_kv][P][d] then the V block [n_kv][P][d].  Token t of a sequence lives in
 * page bt[t / P], slot t % P.                                                 */

/* Write one token's K/V.  k_raw/v are [n_kv, d] in the pool dtype (bf16 as
 * uint16).  K is rotated at rope_pos (cos/sin rows of length d) in fp32, then
 * stored (bf16: rounded to nearest even); V is stored as given. */
void orc_paged_append_token(void *pages, int dtype, size_t n_kv, size_t P, size_t d,
                            const uint32_t *bt, size_t slot, const void *k_raw,
                            const void *v, const float *cos_row, const float *sin_row);

/* Gather tokens [0, n_tokens) of one sequence into fp32 [n_kv, n_tokens, d].
 * Pages marked ORC_PAGE_NONE (evicted) read as zero. */
void orc_paged_gather(const void *pages, int dtype, size_t n_kv, size_t P, size_t d,
                      const uint32_t *bt, size_t n_tokens, float *k_out, float *v_out);

/* Decode attention of one sequence holding seq_len tokens (the new token is
 * already appended).  q_raw [n_q, d] in dtype, rotated at pos seq_len - 1.
 * window == 0: all keys; else keys s < seq_len - window are masked out (the
 * build's sliding window; masked keys contribute exact zeros, so only the
 * window's keys are gathered and attended).  out [n_q, d] fp32. */
void orc_paged_decode(const void *pages, int dtype, size_t n_q, size_t n_kv, size_t P,
                      size_t d, const uint32_t *bt, size_t seq_len, size_t window,
                      const void *q_raw, const float *inv_freq, float *out);

/* One decode step of one layer for n_seqs sequences: for each s, append the
 * token (k_raw[s], v[s]) at position seq_lens[s] - 1, then run
 * orc_paged_decode.  bt is [n_seqs, bt_stride].  Sequences run on n_threads
 * POSIX threads (0 = one per online CPU).  out [n_seqs, n_q, d] fp32. */
void orc_decode_step(void *pages, int dtype, size_t n_q, size_t n_kv, size_t P, size_t d,
                     const uint32_t *bt, size_t bt_stride, const int32_t *seq_lens,
                     size_t n_seqs, size_t window, const void *q_raw, const void *k_raw,
                     const void *v, const float *inv_freq, float *out, int n_threads);

/* Threads orc_decode_step uses with n_threads = 0 (online CPUs). */
int orc_max_threads(void);

/* RMSNorm over rows of `dim` values (crates/llm-cpu/src/ops.rs:8-23): the sum
 * of squares in double, scale = (float)(1 / sqrt(sumsq / dim + eps)),
 * out = w * (x * scale) as two float products.  out may alias x. */
void orc_rms_norm(const float *x, const float *weight, float eps, size_t dim, size_t rows, float *out);

/* orc_decode_step with the attention layer's per-head RMSNorm of q and k
 * before RoPE (lfm2.rs:797-812): q_norm, k_norm are [d] weights. */
void orc_decode_step_norm(void *pages, int dtype, size_t n_q, size_t n_kv, size_t P, size_t d,
                          const uint32_t *bt, size_t bt_stride, const int32_t *seq_lens,
                          size_t n_seqs, size_t window, const void *q_raw, const void *k_raw,
                          const void *v, const float *inv_freq, const float *q_norm,
                          const float *k_norm, float eps, float *out, int n_threads);

/* ---- bulk helpers for large parity cases (same arithmetic as above) ------ */

/* n_tokens calls of orc_paged_append_token: token i goes to row tok_row[i] of
 * bt ([rows, bt_stride]), slot tok_slot[i], rotated at position tok_pos[i];
 * k_raw / v are [n_tokens, n_kv, d].  Tokens must write distinct slots; they
 * are spread over n_threads threads (0 = one per online CPU). */
void orc_paged_append_tokens(void *pages, int dtype, size_t n_kv, size_t P, size_t d, const uint32_t *bt,
                             size_t bt_stride, const int32_t *tok_row, const int32_t *tok_slot,
                             const int32_t *tok_pos, size_t n_tokens, const void *k_raw, const void *v,
                             const float *inv_freq, int n_threads);

/* Chunked-prefill / tree-verify attention on paged K/V, the arithmetic of
 * attention_forward (lfm2.rs:1058-1111) with the build's masks: sequence s
 * has cached[s] committed tokens followed by the chunk's q_off[s+1] - q_off[s]
 * tokens (row s of bt).  Query token i (global index) is rotated at q_pos[i]
 * and sees every cached key, plus chunk key j when j <= its index in the chunk
 * (masks == NULL) or when bit j of masks[i] is set (ancestor-or-self).
 * q_raw [n_tok, n_q, d] in dtype; out [n_tok, n_q, d] fp32.  Work is spread
 * over (sequence, KV head) pairs on n_threads threads. */
void orc_paged_prefill(const void *pages, int dtype, size_t n_q, size_t n_kv, size_t P, size_t d,
                       const uint32_t *bt, size_t bt_stride, size_t n_seqs, const int32_t *cached,
                       const int32_t *q_off, const int32_t *q_pos, const uint64_t *masks, const void *q_raw,
                       const float *inv_freq, float *out, int n_threads);

#ifdef __cplusplus
}
#endif
#endif
