/*
 * llmhost_kv.h -- C ABI of the B200 paged KV-cache library (libllmhost_kv.so).
 *
 * This is the `extern "C"` surface a `crates/llm-cuda` backend binds with a
 * `#[link(name = "llmhost_kv")] extern "C" { ... }` block (style of
 * crates/llm-capi/src/lib.rs:12-15).  Plain pointers and sizes only:
 *   - device pointers are `void *` / typed pointers into CUDA device memory;
 *   - `stream` is a cudaStream_t passed as `void *` (NULL = legacy stream);
 *   - every call returns an int status (enum kv_status), 0 = OK.
 * Calls on one pool are externally serialised (the engine holds `&mut self`,
 * crates/llm-engine/src/batch.rs:173).  Hot calls never allocate: a pool owns
 * its pages, RoPE table and attention workspace, sized at kv_pool_create.
 *
 * Reference interfaces replaced (paths inside the llmhost project):
 *   kv_pool_create      Backend::alloc (crates/llm-core/src/backend.rs:11-12),
 *                       Lfm2Cache K/V buffers (crates/llm-engine/src/lfm2.rs:188-203)
 *   kv_append*          K/V append (lfm2.rs:828-832) with RoPE on k
 *                       (lfm2.rs:816-825, crates/llm-cpu/src/rope.rs:18-81),
 *                       prefill K/V store (lfm2.rs:751-761)
 *   kv_decode_attn      attention_decode_cached (lfm2.rs:1006-1056) with RoPE
 *                       on q (lfm2.rs:816-822) and the key mask (lfm2.rs:1032-1035)
 */
#ifndef LLMHOST_KV_H
#define LLMHOST_KV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KV_API_VERSION 1
#define KV_PAGE_NONE 0xFFFFFFFFu /* block-table entry of an evicted / absent page */

/* KV storage type.  The reference's KvDtype (crates/llm-quant/src/formats.rs:59-68)
 * tags F16/Q8/K8V4 and implements none; this library stores F32 and BF16. */
typedef enum { KV_DTYPE_F32 = 0, KV_DTYPE_BF16 = 1 } kv_dtype;

typedef enum {
    KV_OK = 0,
    KV_ERR_INVALID = 1,     /* bad argument: null pointer, shape, size */
    KV_ERR_BAD_PAGE = 2,    /* a page id out of range, or not allocated */
    KV_ERR_OOM = 3,         /* page pool or device memory exhausted */
    KV_ERR_TIMEOUT = 4,     /* a device-side wait ran past its time limit */
    KV_ERR_CUDA = 5,        /* a CUDA runtime / driver call failed */
    KV_ERR_UNSUPPORTED = 6, /* shape this build does not compile (see kv_pool_create) */
    KV_ERR_BAD_POS = 7      /* a RoPE position >= max_positions */
} kv_status;

typedef struct kv_pool kv_pool; /* opaque */

typedef struct {
    int32_t dtype;         /* kv_dtype */
    int32_t n_q_heads;     /* query heads; a multiple of n_kv_heads */
    int32_t n_kv_heads;    /* 1, 2, 4 or 8 */
    int32_t head_dim;      /* 64 */
    int32_t page_tokens;   /* 16 (reference KV_BLOCK_TOKENS, cache.rs:10) */
    uint32_t n_pages;      /* physical pages in the pool */
    float rope_theta;      /* e.g. 1e6 (crates/llm-core/src/config.rs:508) */
    int32_t max_positions; /* RoPE table length: positions 0 .. max_positions-1 */
    int32_t max_seqs;      /* most sequences one attention call may carry */
    int32_t device;        /* CUDA device ordinal */
} kv_pool_config;

/* Human-readable name of a status code (static string). */
const char *kv_status_str(int status);
/* KV_API_VERSION of the built library. */
int kv_api_version(void);

/* Create a pool: pages (zero-filled), the RoPE cos/sin table for positions
 * [0, max_positions) computed with the same libm calls as rope.rs:6-43, and
 * the decode workspace.  Sets *out on success. */
int kv_pool_create(const kv_pool_config *cfg, kv_pool **out);
int kv_pool_destroy(kv_pool *pool);
/* Device pointer to page 0 and the bytes of one page. */
void *kv_pool_pages(const kv_pool *pool);
size_t kv_pool_page_bytes(const kv_pool *pool);
/* Copy whole pages between the pool and host memory, synchronously: page
 * page_ids[i] <-> bytes [i * page_bytes, (i + 1) * page_bytes) of the host
 * buffer.  For tests, checkpoints and debugging; no reference counterpart
 * (the reference's KV lives in host Vec<f32>, lfm2.rs:194-197). */
int kv_pool_read_pages(kv_pool *pool, const uint32_t *page_ids, int32_t n, void *host_dst);
int kv_pool_write_pages(kv_pool *pool, const uint32_t *page_ids, int32_t n, const void *host_src);
/* Read and clear the device error word; returns the kv_status it maps to
 * (KV_OK if clear).  Synchronises the pool's device. */
int kv_last_error(kv_pool *pool);

/* Append tokens.  k, v: [n_tokens, n_kv_heads, head_dim] in the pool dtype.
 * Token i goes to sequence tok_seq[i] (row of block_tables, [n_seqs, bt_stride]
 * u32 page ids), storage slot tok_slot[i] (page bt[slot / P], slot % P), and
 * K is rotated at RoPE position tok_pos[i].  All arrays are device memory.
 * A sequence index outside [0, n_seqs), a slot past its row, a page id >=
 * n_pages or a position >= max_positions is skipped and flagged in the error
 * word (kv_last_error). */
int kv_append(kv_pool *pool, const void *k, const void *v, const int32_t *tok_seq,
              const int32_t *tok_slot, const int32_t *tok_pos, int32_t n_tokens,
              const uint32_t *block_tables, int32_t n_seqs, int32_t bt_stride, void *stream);

/* Decode append: one token per sequence s at position seq_lens[s] - 1, where
 * seq_lens already counts the new token.  k, v: [n_seqs, n_kv_heads, head_dim]. */
int kv_append_decode(kv_pool *pool, const void *k, const void *v, const uint32_t *block_tables,
                     int32_t bt_stride, const int32_t *seq_lens, int32_t n_seqs, void *stream);

/* Paged decode attention.  q: [n_seqs, n_q_heads, head_dim] (pool dtype,
 * before RoPE; rotated here at seq_lens[s] - 1).  Sequence s attends keys
 * [lo, seq_lens[s]) with lo = window > 0 ? max(0, seq_lens[s] - window) : 0.
 * out: [n_seqs, n_q_heads, head_dim] in the pool dtype.  A sequence with
 * seq_lens[s] == 0 gets zeros. */
int kv_decode_attn(kv_pool *pool, const void *q, const uint32_t *block_tables, int32_t bt_stride,
                   const int32_t *seq_lens, int32_t n_seqs, int32_t window, void *out,
                   void *stream);

/* Decode attention for callers that cannot allocate device memory.
 *
 * No counterpart in the reference.  Same arithmetic and arguments as
 * kv_decode_attn, but without a pool: some callers cannot call cudaMalloc
 * (their device memory all comes from a fixed arena they manage, or they may
 * not grow their footprint after start-up), so they cannot create a kv_pool.
 * They pass every buffer themselves: the pages (pool layout, n_pages of them,
 * dtype and head counts as in kv_pool_config), the RoPE table rope_cs
 * (float pairs (cos, sin) for positions [0, max_positions) and frequency
 * i < head_dim/2, as kv_pool_create builds it), q, the block tables, the
 * lengths, out, and `status`, one device int32 that receives the device
 * error bits of this call (1 bad page id, 2 wait timeout, 4 position out of
 * range; 0 when clean).
 *
 * The call itself allocates nothing.  Its scratch is one 4 MiB array in the
 * library's device image, held by every GPU that loads the library until
 * exit.  Limits: n_seqs <= 1024 and n_q_heads <= 32; larger calls return
 * KV_ERR_INVALID.  All calls on a device share that array: a call clears the
 * part that must start at zero, but two calls whose kernels overlap on the
 * GPU (different streams or threads) race on it, so serialise them.  The
 * first call on a device sets up with that device current (it looks up the
 * array's address); make that first call before any stream capture. */
int kv_decode_attn_noalloc(const void *pages, uint32_t n_pages, int32_t dtype, int32_t n_q_heads,
                           int32_t n_kv_heads, const void *rope_cs, int32_t max_positions,
                           const void *q, const uint32_t *block_tables, int32_t bt_stride,
                           const int32_t *seq_lens, int32_t n_seqs, int32_t window, void *out,
                           int32_t *status, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* LLMHOST_KV_H */
