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
 *   kv_append_decode_attn  the decode K/V store (lfm2.rs:828-832) and
 *                       attention_decode_cached in one launch
 *   kv_norm_append_decode_attn  the same with the q/k RMSNorm (lfm2.rs:797-812)
 *   kv_tree_*           validate_tree_for_tokens, validate_accept_path (tree.rs:48-123)
 *   kv_state_*          Engine::{open, forward, accept, rollback, committed,
 *                       session_kv} (batch.rs:128-297) and PagedKv (cache.rs:12-51),
 *                       with the page allocator, block tables, copy-on-write
 *                       fork, eviction and compaction the reference lacks
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
 * tags F16/Q8/K8V4 and implements none.  This library stores F32, BF16, F16
 * and the two quantised tags.
 *   KV_DTYPE_F16   K and V as IEEE half (the reference's default tag, "full
 *                  f16 keys and values") in the bf16 page layout; the appended
 *                  k / v, q and out are bf16 (K rotated in fp32, then K and V
 *                  rounded to half, to nearest even).  Every entry point but
 *                  kv_prefill_attn_shared and kv_decode_attn_noalloc; decode
 *                  runs on the tensor cores with f16 operands, prefill on the
 *                  CUDA cores in fp32.
 * The quantised tags use the block quantisers of the same crate
 * (crates/llm-quant/src/lib.rs:14-101, 32 elements and one f16 scale per
 * block, two blocks per 64-dim head row):
 *   KV_DTYPE_Q8    K and V as Q8_0 blocks (int8 codes, scale max|x| / 127)
 *   KV_DTYPE_K8V4  K as Q8_0, V as Q4 blocks (4-bit codes, scale max|x| / 8)
 * A quantised page is n_kv head blocks, each holding in order: K codes
 * [P][64] int8, V codes [P][64] int8 (Q8) or [P][32] packed nibbles (K8V4:
 * element 2i in the low nibble of byte i), scales [P][2 blocks][K, V] f16
 * (2176 or 1664 bytes a head at P = 16).  K is rotated (RoPE) in fp32 and then quantised.  For
 * quantised pools the appended k / v, q and out are bf16.  They take
 * appends, decode attention (kv_decode_attn, and kv_append_decode_attn as an
 * append launch followed by the attention launch; tensor cores, head layouts
 * as for bf16 pools), kv_prefill_attn (CUDA cores, on the dequantised keys and
 * values in fp32), kv_norm_append_decode_attn (the k norm in the append
 * launch, the q norm in the attention launch), page copies and token moves;
 * kv_prefill_attn_shared returns KV_ERR_UNSUPPORTED for them. */
typedef enum { KV_DTYPE_F32 = 0, KV_DTYPE_BF16 = 1, KV_DTYPE_Q8 = 2, KV_DTYPE_K8V4 = 3, KV_DTYPE_F16 = 4 } kv_dtype;

typedef enum {
    KV_OK = 0,
    KV_ERR_INVALID = 1,     /* bad argument: null pointer, shape, size */
    KV_ERR_BAD_PAGE = 2,    /* a page id out of range, or not allocated */
    KV_ERR_OOM = 3,         /* page pool or device memory exhausted */
    KV_ERR_TIMEOUT = 4,     /* a device-side wait ran past its time limit */
    KV_ERR_CUDA = 5,        /* a CUDA runtime / driver call failed */
    KV_ERR_UNSUPPORTED = 6, /* shape this build does not compile (see kv_pool_create) */
    KV_ERR_BAD_POS = 7,     /* a RoPE position >= max_positions */
    KV_ERR_UNKNOWN_SEQ = 8, /* EngineError::UnknownSeq (batch.rs:63) */
    KV_ERR_NO_PENDING = 9,  /* EngineError::NoPendingForward (batch.rs:64) */
    KV_ERR_INVALID_ACCEPT = 10, /* EngineError::InvalidAccept (batch.rs:65) */
    KV_ERR_TREE = 11        /* EngineError::Tree / a TreeError (tree.rs:11-19) */
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
    int32_t max_seqs;      /* most sequences one attention call may carry; the decode
                              kernel keeps a per-sequence table in shared memory, so
                              kv_pool_create returns KV_ERR_INVALID past a limit set
                              by the dtype and head layout: with 8 kv heads (group 4
                              to group 3) 1875-2219 for bf16 and f16, 851-1195 for Q8,
                              4947-5291 for K8V4, over 15000 for fp32 pools; higher
                              with fewer kv heads */
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

/* Append tokens.  k, v: [n_tokens, n_kv_heads, head_dim] in the pool dtype,
 * 16-byte aligned (KV_ERR_INVALID otherwise).
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
 * seq_lens already counts the new token.  k, v: [n_seqs, n_kv_heads, head_dim],
 * 16-byte aligned (as for kv_append). */
int kv_append_decode(kv_pool *pool, const void *k, const void *v, const uint32_t *block_tables,
                     int32_t bt_stride, const int32_t *seq_lens, int32_t n_seqs, void *stream);

/* Paged decode attention.  q: [n_seqs, n_q_heads, head_dim] (pool dtype,
 * before RoPE; rotated here at seq_lens[s] - 1), 16-byte aligned.  Sequence s attends keys
 * [lo, seq_lens[s]) with lo = window > 0 ? max(0, seq_lens[s] - window) : 0.
 * out: [n_seqs, n_q_heads, head_dim] in the pool dtype.  A sequence with
 * seq_lens[s] == 0 gets zeros. */
int kv_decode_attn(kv_pool *pool, const void *q, const uint32_t *block_tables, int32_t bt_stride,
                   const int32_t *seq_lens, int32_t n_seqs, int32_t window, void *out,
                   void *stream);

/* One decode step of an attention layer in one launch: kv_append_decode(k, v,
 * ...) followed by kv_decode_attn(q, ...) on the same block tables and
 * seq_lens, with the same results bit for bit (pages and out).  It replaces
 * the pair the reference runs per layer: the K/V store (lfm2.rs:828-832)
 * and attention_decode_cached (lfm2.rs:1006-1056).  The page holding each
 * sequence's new slot must belong to that sequence alone (copy-on-write
 * first), as it must for kv_append_decode: the new row is written into the
 * copy of the page this launch reads, not re-read from HBM. */
int kv_append_decode_attn(kv_pool *pool, const void *k, const void *v, const void *q,
                          const uint32_t *block_tables, int32_t bt_stride, const int32_t *seq_lens,
                          int32_t n_seqs, int32_t window, void *out, void *stream);

/* kv_append_decode_attn with the attention layer's per-head RMSNorm of q and
 * of the new k folded in, before RoPE (lfm2.rs:797-812, the norm of
 * crates/llm-cpu/src/ops.rs:8-23): x' = w * (x * s) with
 * s = 1 / sqrt(sum(x^2) / head_dim + eps), the sum in double.  q_norm and
 * k_norm are [head_dim] fp32 device weights, 16-byte aligned; eps >= 0.  The
 * stored K is the normalised, rotated k. */
int kv_norm_append_decode_attn(kv_pool *pool, const void *k, const void *v, const void *q, const float *q_norm,
                               const float *k_norm, float eps, const uint32_t *block_tables, int32_t bt_stride,
                               const int32_t *seq_lens, int32_t n_seqs, int32_t window, void *out, void *stream);

/* Chunked-prefill and tree-verify attention: attention_forward
 * (lfm2.rs:1058-1111) for T_s new query tokens of sequence s that follow
 * prefix_lens[s] = L_s cached tokens (the reference only prefills from
 * position 0, lfm2.rs:730).  The chunk's K/V must already be in the pages at
 * slots L_s .. L_s + T_s - 1 (kv_append).
 *   q          [total_q, n_q_heads, head_dim], pool dtype, before RoPE;
 *              sequence s owns rows q_offsets[s] .. q_offsets[s+1] - 1
 *   q_pos      [total_q] RoPE position of each query row
 *   tree_masks NULL: causal chunk (chunk token i sees chunk tokens j <= i);
 *              else [total_q] bit masks, bit j set when chunk token j is an
 *              ancestor-or-self of token i (speculative tree verify, T_s <= 64)
 *   out        [total_q, n_q_heads, head_dim], pool dtype
 * Every query also sees all L_s cached keys.  max_q_per_seq bounds T_s (the
 * launch covers that many tokens per sequence; a larger T_s, or T_s > 64 with
 * tree masks, is flagged in the error word as an invalid argument).  Slots
 * past L_s + T_s in the sequence's last page must hold finite values (as a
 * fresh pool and kv_append leave them).  bf16 pools run on the tcgen05
 * tensor cores, fp32 pools on the CUDA cores in fp32. */
int kv_prefill_attn(kv_pool *pool, const void *q, const int32_t *q_pos, const int32_t *q_offsets,
                    const int32_t *prefix_lens, const uint64_t *tree_masks,
                    const uint32_t *block_tables, int32_t bt_stride, int32_t n_seqs,
                    int32_t max_q_per_seq, void *out, void *stream);

/* Shared-prefix (cascade) form of kv_prefill_attn, for a batch whose
 * sequences all begin with the same shared_tokens tokens on the same pages
 * (block-table entries 0 .. shared_tokens / 16 - 1 equal in every row, as
 * after kv_state_fork of one prompt).  The shared keys are attended once for
 * all queries of the batch together (one dense pass over those pages, whose
 * unnormalised rows go to the workspace), then each sequence's remaining keys
 * (cached and chunk, with the same causal or tree masks), merged with the
 * first pass by the log-sum-exp identity.  Same arguments and results as
 * kv_prefill_attn (to rounding), plus
 *   shared_tokens  a multiple of 16, at most every prefix_lens[s] (a shorter
 *                  prefix is flagged in the error word as an invalid argument)
 *   workspace      16-byte aligned device memory of
 *                  kv_prefill_shared_workspace_bytes(pool, n_seqs, max_q_per_seq)
 *                  bytes, not shared with a launch still in flight
 * Two launches on the stream.  bf16 pools only (KV_ERR_UNSUPPORTED otherwise). */
size_t kv_prefill_shared_workspace_bytes(const kv_pool *pool, int32_t n_seqs, int32_t max_q_per_seq);
int kv_prefill_attn_shared(kv_pool *pool, const void *q, const int32_t *q_pos, const int32_t *q_offsets,
                           const int32_t *prefix_lens, const uint64_t *tree_masks,
                           const uint32_t *block_tables, int32_t bt_stride, int32_t n_seqs,
                           int32_t max_q_per_seq, int32_t shared_tokens, void *workspace, void *out,
                           void *stream);

/* One token's K/V (every head of one layer) from page slot to page slot. */
typedef struct {
    uint32_t src_page;
    int32_t src_slot;
    uint32_t dst_page;
    int32_t dst_slot;
} kv_token_move;

/* Page copies (copy-on-write, compaction): page src[i] -> dst[i], i < n, src and
 * dst device arrays.  The copies of one call must be independent (no page is
 * both a source and a destination).  Any n >= 0 (one launch per 65535). */
int kv_copy_pages(kv_pool *pool, const uint32_t *src, const uint32_t *dst, int32_t n, void *stream);
/* Token moves (commit of accepted draft tokens): moves is a device array of
 * n_moves; group g is moves[group_offsets[g] .. group_offsets[g+1]) (device
 * array of n_groups + 1), run in order a chunk at a time, every source of a
 * chunk read before any destination is written -- exact for the moves
 * kv_state_accept / kv_state_rollback produce.  Groups run in parallel and
 * must not touch the same slots. */
int kv_move_tokens(kv_pool *pool, const kv_token_move *moves, int32_t n_moves, const int32_t *group_offsets,
                   int32_t n_groups, void *stream);

/* ---- host-side KV state ----------------------------------------------------
 * Host-only (no CUDA calls).  It owns the page allocator and every sequence's
 * per-layer block tables, and mirrors llm-engine's Engine (batch.rs:128-297):
 * forward() stages draft tokens, accept()/rollback() commit a path of them.
 * Device work is returned as plans -- page copies (copy-on-write, compaction)
 * and token-slot moves (accepted draft tokens) -- that the caller runs with
 * kv_copy_pages / kv_move_slots before its next launch.  Allocation rules:
 * a LIFO free stack whose first pops follow alloc_order (NULL: 0, 1, 2, ...);
 * layers are walked in order; a write into a shared partial tail page copies
 * it first.  Output buffers are checked before the state changes. */

typedef struct kv_state kv_state; /* opaque */

enum {
    KV_TREE_OK = 0,
    KV_TREE_LENGTH_MISMATCH = 1,          /* TreeError::LengthMismatch { tree, tokens } */
    KV_TREE_PARENT_OUT_OF_RANGE = 2,      /* TreeError::ParentOutOfRange { child, parent } */
    KV_TREE_PARENT_DOES_NOT_PRECEDE = 3   /* TreeError::ParentDoesNotPrecede { child, parent } */
};

typedef struct {
    int32_t kind; /* KV_TREE_* */
    int64_t child;
    int64_t parent;
    int64_t tree;
    int64_t tokens;
} kv_tree_error;

/* tree.rs:66-73 validate_tree_for_tokens; KV_ERR_TREE with *err filled. */
int kv_tree_validate(const int32_t *tree, int32_t tree_len, int32_t tokens, kv_tree_error *err);
/* tree.rs:90-123 validate_accept_path. */
int kv_tree_validate_accept(const int32_t *tree, int32_t tree_len, const int64_t *accepted, int32_t n,
                            kv_tree_error *err);

int kv_state_create(uint32_t n_pages, int32_t n_layers, int32_t page_tokens, const uint32_t *alloc_order,
                    uint32_t n_order, kv_state **out);
int kv_state_destroy(kv_state *st);
/* Engine::open: a fresh, empty sequence (replaces existing state). */
int kv_state_open(kv_state *st, uint64_t seq_id);
/* Release a sequence and all its pages. */
int kv_state_close(kv_state *st, uint64_t seq_id);
/* New sequence dst sharing every committed page of src (copy-on-write). */
int kv_state_fork(kv_state *st, uint64_t src, uint64_t dst);
/* Commit n tokens (ids may be NULL) straight into the sequence's KV; cow_*
 * (capacity >= n_layers) receive the page copies to run first. */
int kv_state_append(kv_state *st, uint64_t seq_id, const uint32_t *tokens, int32_t n, uint32_t *cow_src,
                    uint32_t *cow_dst, int32_t cow_cap, int32_t *n_cow);
/* Engine::forward for one sequence: stage n draft tokens with parent array
 * tree (NULL: a chain).  slots[i] / positions[i] receive token i's storage
 * slot and RoPE position; cow_* the page copies to run before the append. */
int kv_state_forward(kv_state *st, uint64_t seq_id, const uint32_t *tokens, int32_t n, const int32_t *tree,
                     int32_t tree_len, int32_t *slots, int32_t *positions, uint32_t *cow_src, uint32_t *cow_dst,
                     int32_t cow_cap, int32_t *n_cow, kv_tree_error *err);
/* Engine::accept / Engine::rollback: commit a path of the staged tokens.
 * move_* (capacity >= staged tokens) receive the slot moves (accepted token
 * order[j] goes from slot L + order[j] to L + j).  tok_moves, if not NULL
 * (capacity >= staged tokens * n_layers), receives the same moves for every
 * layer addressed by page, taken before the commit frees the rejected pages:
 * run them with kv_move_tokens before the next launch.  *bad_index is set on
 * KV_ERR_INVALID_ACCEPT. */
int kv_state_accept(kv_state *st, uint64_t seq_id, const int64_t *accepted, int32_t n, int32_t *move_src,
                    int32_t *move_dst, int32_t move_cap, int32_t *n_moves, kv_token_move *tok_moves,
                    int32_t tok_cap, int32_t *n_tok_moves, int64_t *bad_index);
int kv_state_rollback(kv_state *st, uint64_t seq_id, const int64_t *rejected, int32_t n, int32_t *move_src,
                      int32_t *move_dst, int32_t move_cap, int32_t *n_moves, kv_token_move *tok_moves,
                      int32_t tok_cap, int32_t *n_tok_moves, int64_t *bad_index);
/* kv_state_forward for a batch of sequences, in order, flattened into the
 * arrays one kv_append and one kv_prefill_attn launch per layer take.
 * Sequence i stages tokens[tok_off[i] .. tok_off[i+1]) (tok_off: n_seqs + 1
 * entries, tok_off[0] = 0) with the parent array trees + tok_off[i] (trees
 * NULL: every draft a chain).  Outputs: tok_row / slots / positions [total
 * tokens] (batch row, storage slot, RoPE position of each token); prefix
 * [n_seqs] (committed tokens before each draft); masks [total tokens], if not
 * NULL, the ancestor-or-self bit masks kv_prefill_attn takes (every draft at
 * most 64 tokens); cow_* (capacity >= n_layers * n_seqs) the page copies to
 * run first, *n_cow of them; tables [n_layers][n_seqs][stride] the drafts'
 * block tables padded with KV_PAGE_NONE.  Sizes are checked before any state
 * changes; an error from sequence i (tree, OOM) returns with sequences
 * 0 .. i-1 staged, *n_done = i and *err filled for a tree error. */
int kv_state_forward_batch(kv_state *st, const uint64_t *seq_ids, int32_t n_seqs, const uint32_t *tokens,
                           const int32_t *tok_off, const int32_t *trees, int32_t *tok_row, int32_t *slots,
                           int32_t *positions, int32_t *prefix, uint64_t *masks, uint32_t *cow_src,
                           uint32_t *cow_dst, int32_t cow_cap, int32_t *n_cow, uint32_t *tables, int32_t stride,
                           int32_t *n_done, kv_tree_error *err);
/* kv_state_accept for a batch: sequence i commits paths[path_off[i] ..
 * path_off[i+1]).  tok_moves (capacity tok_cap >= staged tokens of all
 * sequences * n_layers; *tok_need receives that number, also when tok_cap is
 * too small and the call returns KV_ERR_INVALID with no change made)
 * receives the page-addressed token moves, one group per
 * (sequence, layer) in that order: group g is tok_moves[group_off[g] ..
 * group_off[g+1]), group_off having n_seqs * n_layers + 1 entries -- the
 * groups kv_move_tokens takes.  An error from sequence i returns with
 * sequences 0 .. i-1 committed, *n_done = i (*bad_index set on
 * KV_ERR_INVALID_ACCEPT). */
int kv_state_accept_batch(kv_state *st, const uint64_t *seq_ids, int32_t n_seqs, const int64_t *paths,
                          const int32_t *path_off, kv_token_move *tok_moves, int32_t tok_cap, int64_t *tok_need,
                          int32_t *group_off, int32_t *n_done, int64_t *bad_index);
/* Free the pages wholly below token_count - window (entries become KV_PAGE_NONE). */
int kv_state_evict_window(kv_state *st, uint64_t seq_id, int64_t window, int64_t *n_freed);
/* Move used pages into the lowest ids; *n_moves receives the count (also on
 * KV_ERR_INVALID when cap is too small, with no change made). */
int kv_state_compact(kv_state *st, uint32_t *src, uint32_t *dst, int32_t cap, int32_t *n_moves);
/* PagedKv::token_count (cache.rs:31-34). */
int kv_state_token_count(const kv_state *st, uint64_t seq_id, int64_t *n);
/* Engine::committed (batch.rs:162-165). */
int kv_state_committed(const kv_state *st, uint64_t seq_id, uint32_t *tokens, int64_t cap, int64_t *n);
/* One layer's block table; which = 0 committed, 1 the staged draft. */
int kv_state_table(const kv_state *st, uint64_t seq_id, int32_t layer, int32_t which, uint32_t *out,
                   int64_t cap, int64_t *n);
/* Rows of n_seqs tables for a kernel launch: out[i * stride + j], padded
 * with KV_PAGE_NONE. */
int kv_state_export_tables(const kv_state *st, const uint64_t *seq_ids, int32_t n_seqs, int32_t layer,
                           int32_t which, uint32_t *out, int32_t stride);
int kv_state_free_list(const kv_state *st, uint32_t *out, int64_t cap, int64_t *n);
int kv_state_refcount(const kv_state *st, uint32_t page, uint32_t *count);
/* Token count at which the staged draft starts (its first slot). */
int kv_state_pending_base(const kv_state *st, uint64_t seq_id, int64_t *base);

/* ---- the path's callers: draft trees and the batch scheduler ---------------
 * Host-only.  The reference has both as placeholders: a DraftModel hook that
 * returns tokens and a parent array (crates/llm-engine/src/draft.rs:9-23) and
 * a Scheduler of running sequence ids (crates/llm-engine/src/schedule.rs:8-48). */

/* The speculative tree from a draft model's candidates, best first:
 * candidate c has parent cand_parent[c] (-1: a root; parents precede their
 * children), token cand_token[c] and probability cand_prob[c] in [0, 1] given
 * its parent.  Its score is the product of the probabilities on its path.
 * Nodes are picked one at a time, the highest-scoring eligible candidate
 * next (ties to the lower index); a candidate is eligible once its parent is
 * picked (roots from the start) and if its depth (roots 0) is <= max_depth.
 * At most max_nodes are picked.  Out, in pick order: tokens, tree (parent as
 * an index into the output, -1 for roots: the DraftProposal form, valid for
 * kv_tree_validate) and, if not NULL, picked (candidate index); *n_out nodes. */
int kv_draft_tree_best_first(const int32_t *cand_parent, const uint32_t *cand_token, const double *cand_prob,
                             int32_t n_cand, int32_t max_nodes, int32_t max_depth, uint32_t *tokens, int32_t *tree,
                             int32_t *picked, int32_t *n_out);

typedef struct kv_sched kv_sched; /* opaque */
int kv_sched_create(kv_sched **out);
int kv_sched_destroy(kv_sched *s);
/* Scheduler::add (schedule.rs:23-27): appended once, in insertion order. */
int kv_sched_add(kv_sched *s, uint64_t seq_id);
/* Scheduler::remove (schedule.rs:29-31). */
int kv_sched_remove(kv_sched *s, uint64_t seq_id);
/* Scheduler::running / schedule (schedule.rs:34-47): the running ids in order. */
int kv_sched_running(const kv_sched *s, uint64_t *out, int64_t cap, int64_t *n);
/* Prompt tokens still to prefill for a running sequence (0: it decodes). */
int kv_sched_set_pending(kv_sched *s, uint64_t seq_id, int64_t prefill_tokens);
/* One step's batch under token_budget: first one decode token for every
 * running sequence with no prompt left, in running order, then prompt chunks
 * of up to chunk_tokens in running order while the budget lasts (the chunks
 * are taken off the sequences' pending counts).  Out: seq_ids, n_tokens,
 * is_prefill for *n_out entries (cap >= running sequences). */
int kv_sched_plan_step(kv_sched *s, int64_t token_budget, int32_t chunk_tokens, uint64_t *seq_ids,
                       int32_t *n_tokens, int32_t *is_prefill, int32_t cap, int32_t *n_out);
/* Longest-processing-time assignment of n items to n_bins (sessions to GPUs
 * by resident KV length): items by decreasing weight (ties to the lower
 * index), each to the currently lightest bin (ties to the lower bin). */
int kv_sched_lpt(const int64_t *weights, int32_t n, int32_t n_bins, int32_t *bins);

/* Decode attention for callers that cannot allocate device memory.
 *
 * No counterpart in the reference.  The arguments and results of
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
 * Kernel: both dtypes run the CUDA-core decode kernel (kv_decode_attn runs
 * it for fp32 pools only; its bf16 pools use the tensor-core kernel, which
 * rounds the probabilities to bf16 before P·V).  So fp32 results equal
 * kv_decode_attn's, and bf16 results differ from them by rounding, within
 * the bf16 tolerance (2e-2 normwise per row) of the reference arithmetic.
 * Head layouts: (n_kv_heads, n_q_heads / n_kv_heads) = (8, 3), (8, 4), (1, 4),
 * (2, 4), (4, 4); others return KV_ERR_UNSUPPORTED.
 *
 * The call itself allocates nothing.  Its scratch is one 4 MiB array in the
 * library's device image, held by every GPU that loads the library until
 * exit.  Limits: n_seqs <= 1024 and n_q_heads <= 32; larger calls return
 * KV_ERR_INVALID.  All calls on a device share that array: a call clears the
 * part that must start at zero, but two calls whose kernels overlap on the
 * GPU (different streams or threads) race on it, so serialise them.  The
 * first call on a device sets up with that device current (it looks up the
 * array's address); make that first call before any stream capture.  The
 * address is kept for the life of the process, so a device reset
 * (cudaDeviceReset, or a reset of the primary context) after the first call
 * on that device is not supported. */
int kv_decode_attn_noalloc(const void *pages, uint32_t n_pages, int32_t dtype, int32_t n_q_heads,
                           int32_t n_kv_heads, const void *rope_cs, int32_t max_positions,
                           const void *q, const uint32_t *block_tables, int32_t bt_stride,
                           const int32_t *seq_lens, int32_t n_seqs, int32_t window, void *out,
                           int32_t *status, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* LLMHOST_KV_H */
