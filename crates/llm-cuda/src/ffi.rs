//! Raw declarations of `include/llmhost_kv.h`, one per C function, in header
//! order.  Plain pointers, sizes and `i32` status codes (`KV_OK` = 0); the
//! safe wrappers live in `lib.rs`.  Device pointers are `*const c_void` /
//! typed raw pointers into CUDA memory, `stream` is a `cudaStream_t` (null =
//! the legacy stream).

#![allow(non_camel_case_types)]

use std::ffi::{c_char, c_void};

pub const KV_API_VERSION: i32 = 1;
/// Block-table entry of an evicted or absent page.
pub const KV_PAGE_NONE: u32 = 0xFFFF_FFFF;

pub const KV_DTYPE_F32: i32 = 0;
pub const KV_DTYPE_BF16: i32 = 1;
pub const KV_DTYPE_Q8: i32 = 2;
pub const KV_DTYPE_K8V4: i32 = 3;
pub const KV_DTYPE_F16: i32 = 4;

pub const KV_OK: i32 = 0;
pub const KV_ERR_INVALID: i32 = 1;
pub const KV_ERR_BAD_PAGE: i32 = 2;
pub const KV_ERR_OOM: i32 = 3;
pub const KV_ERR_TIMEOUT: i32 = 4;
pub const KV_ERR_CUDA: i32 = 5;
pub const KV_ERR_UNSUPPORTED: i32 = 6;
pub const KV_ERR_BAD_POS: i32 = 7;
pub const KV_ERR_UNKNOWN_SEQ: i32 = 8;
pub const KV_ERR_NO_PENDING: i32 = 9;
pub const KV_ERR_INVALID_ACCEPT: i32 = 10;
pub const KV_ERR_TREE: i32 = 11;

pub const KV_TREE_OK: i32 = 0;
pub const KV_TREE_LENGTH_MISMATCH: i32 = 1;
pub const KV_TREE_PARENT_OUT_OF_RANGE: i32 = 2;
pub const KV_TREE_PARENT_DOES_NOT_PRECEDE: i32 = 3;

/// Opaque device page pool (`kv_pool`).
#[repr(C)]
pub struct kv_pool {
    _opaque: [u8; 0],
}

/// Opaque host-side KV state: allocator and block tables (`kv_state`).
#[repr(C)]
pub struct kv_state {
    _opaque: [u8; 0],
}

/// Opaque continuous-batching scheduler (`kv_sched`).
#[repr(C)]
pub struct kv_sched {
    _opaque: [u8; 0],
}

/// `kv_pool_config`: field order and types as in the header.
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct kv_pool_config {
    pub dtype: i32,
    pub n_q_heads: i32,
    pub n_kv_heads: i32,
    pub head_dim: i32,
    pub page_tokens: i32,
    pub n_pages: u32,
    pub rope_theta: f32,
    pub max_positions: i32,
    pub max_seqs: i32,
    pub device: i32,
}

/// `kv_token_move`: one token's K/V (every head of one layer) between page slots.
#[repr(C)]
#[derive(Clone, Copy, Debug, Default, PartialEq, Eq)]
pub struct kv_token_move {
    pub src_page: u32,
    pub src_slot: i32,
    pub dst_page: u32,
    pub dst_slot: i32,
}

/// `kv_tree_error`: the data of a `TreeError` (crates/llm-engine/src/tree.rs:11-19).
#[repr(C)]
#[derive(Clone, Copy, Debug, Default, PartialEq, Eq)]
pub struct kv_tree_error {
    pub kind: i32,
    pub child: i64,
    pub parent: i64,
    pub tree: i64,
    pub tokens: i64,
}

#[link(name = "llmhost_kv")]
extern "C" {
    pub fn kv_status_str(status: i32) -> *const c_char;
    pub fn kv_api_version() -> i32;

    pub fn kv_pool_create(cfg: *const kv_pool_config, out: *mut *mut kv_pool) -> i32;
    pub fn kv_pool_destroy(pool: *mut kv_pool) -> i32;
    pub fn kv_pool_pages(pool: *const kv_pool) -> *mut c_void;
    pub fn kv_pool_page_bytes(pool: *const kv_pool) -> usize;
    pub fn kv_pool_read_pages(pool: *mut kv_pool, page_ids: *const u32, n: i32, host_dst: *mut c_void) -> i32;
    pub fn kv_pool_write_pages(pool: *mut kv_pool, page_ids: *const u32, n: i32, host_src: *const c_void) -> i32;
    pub fn kv_last_error(pool: *mut kv_pool) -> i32;

    pub fn kv_append(
        pool: *mut kv_pool,
        k: *const c_void,
        v: *const c_void,
        tok_seq: *const i32,
        tok_slot: *const i32,
        tok_pos: *const i32,
        n_tokens: i32,
        block_tables: *const u32,
        n_seqs: i32,
        bt_stride: i32,
        stream: *mut c_void,
    ) -> i32;
    pub fn kv_append_decode(
        pool: *mut kv_pool,
        k: *const c_void,
        v: *const c_void,
        block_tables: *const u32,
        bt_stride: i32,
        seq_lens: *const i32,
        n_seqs: i32,
        stream: *mut c_void,
    ) -> i32;
    pub fn kv_decode_attn(
        pool: *mut kv_pool,
        q: *const c_void,
        block_tables: *const u32,
        bt_stride: i32,
        seq_lens: *const i32,
        n_seqs: i32,
        window: i32,
        out: *mut c_void,
        stream: *mut c_void,
    ) -> i32;
    pub fn kv_append_decode_attn(
        pool: *mut kv_pool,
        k: *const c_void,
        v: *const c_void,
        q: *const c_void,
        block_tables: *const u32,
        bt_stride: i32,
        seq_lens: *const i32,
        n_seqs: i32,
        window: i32,
        out: *mut c_void,
        stream: *mut c_void,
    ) -> i32;
    pub fn kv_norm_append_decode_attn(
        pool: *mut kv_pool,
        k: *const c_void,
        v: *const c_void,
        q: *const c_void,
        q_norm: *const f32,
        k_norm: *const f32,
        eps: f32,
        block_tables: *const u32,
        bt_stride: i32,
        seq_lens: *const i32,
        n_seqs: i32,
        window: i32,
        out: *mut c_void,
        stream: *mut c_void,
    ) -> i32;
    pub fn kv_prefill_attn(
        pool: *mut kv_pool,
        q: *const c_void,
        q_pos: *const i32,
        q_offsets: *const i32,
        prefix_lens: *const i32,
        tree_masks: *const u64,
        block_tables: *const u32,
        bt_stride: i32,
        n_seqs: i32,
        max_q_per_seq: i32,
        out: *mut c_void,
        stream: *mut c_void,
    ) -> i32;
    pub fn kv_prefill_shared_workspace_bytes(pool: *const kv_pool, n_seqs: i32, max_q_per_seq: i32) -> usize;
    pub fn kv_prefill_attn_shared(
        pool: *mut kv_pool,
        q: *const c_void,
        q_pos: *const i32,
        q_offsets: *const i32,
        prefix_lens: *const i32,
        tree_masks: *const u64,
        block_tables: *const u32,
        bt_stride: i32,
        n_seqs: i32,
        max_q_per_seq: i32,
        shared_tokens: i32,
        workspace: *mut c_void,
        out: *mut c_void,
        stream: *mut c_void,
    ) -> i32;
    pub fn kv_copy_pages(pool: *mut kv_pool, src: *const u32, dst: *const u32, n: i32, stream: *mut c_void) -> i32;
    pub fn kv_move_tokens(
        pool: *mut kv_pool,
        moves: *const kv_token_move,
        n_moves: i32,
        group_offsets: *const i32,
        n_groups: i32,
        stream: *mut c_void,
    ) -> i32;

    pub fn kv_tree_validate(tree: *const i32, tree_len: i32, tokens: i32, err: *mut kv_tree_error) -> i32;
    pub fn kv_tree_validate_accept(
        tree: *const i32,
        tree_len: i32,
        accepted: *const i64,
        n: i32,
        err: *mut kv_tree_error,
    ) -> i32;

    pub fn kv_state_create(
        n_pages: u32,
        n_layers: i32,
        page_tokens: i32,
        alloc_order: *const u32,
        n_order: u32,
        out: *mut *mut kv_state,
    ) -> i32;
    pub fn kv_state_destroy(st: *mut kv_state) -> i32;
    pub fn kv_state_open(st: *mut kv_state, seq_id: u64) -> i32;
    pub fn kv_state_close(st: *mut kv_state, seq_id: u64) -> i32;
    pub fn kv_state_fork(st: *mut kv_state, src: u64, dst: u64) -> i32;
    pub fn kv_state_append(
        st: *mut kv_state,
        seq_id: u64,
        tokens: *const u32,
        n: i32,
        cow_src: *mut u32,
        cow_dst: *mut u32,
        cow_cap: i32,
        n_cow: *mut i32,
    ) -> i32;
    pub fn kv_state_forward(
        st: *mut kv_state,
        seq_id: u64,
        tokens: *const u32,
        n: i32,
        tree: *const i32,
        tree_len: i32,
        slots: *mut i32,
        positions: *mut i32,
        cow_src: *mut u32,
        cow_dst: *mut u32,
        cow_cap: i32,
        n_cow: *mut i32,
        err: *mut kv_tree_error,
    ) -> i32;
    pub fn kv_state_accept(
        st: *mut kv_state,
        seq_id: u64,
        accepted: *const i64,
        n: i32,
        move_src: *mut i32,
        move_dst: *mut i32,
        move_cap: i32,
        n_moves: *mut i32,
        tok_moves: *mut kv_token_move,
        tok_cap: i32,
        n_tok_moves: *mut i32,
        bad_index: *mut i64,
    ) -> i32;
    pub fn kv_state_rollback(
        st: *mut kv_state,
        seq_id: u64,
        rejected: *const i64,
        n: i32,
        move_src: *mut i32,
        move_dst: *mut i32,
        move_cap: i32,
        n_moves: *mut i32,
        tok_moves: *mut kv_token_move,
        tok_cap: i32,
        n_tok_moves: *mut i32,
        bad_index: *mut i64,
    ) -> i32;
    pub fn kv_state_forward_batch(
        st: *mut kv_state,
        seq_ids: *const u64,
        n_seqs: i32,
        tokens: *const u32,
        tok_off: *const i32,
        trees: *const i32,
        tok_row: *mut i32,
        slots: *mut i32,
        positions: *mut i32,
        prefix: *mut i32,
        masks: *mut u64,
        cow_src: *mut u32,
        cow_dst: *mut u32,
        cow_cap: i32,
        n_cow: *mut i32,
        tables: *mut u32,
        stride: i32,
        n_done: *mut i32,
        err: *mut kv_tree_error,
    ) -> i32;
    pub fn kv_state_accept_batch(
        st: *mut kv_state,
        seq_ids: *const u64,
        n_seqs: i32,
        paths: *const i64,
        path_off: *const i32,
        tok_moves: *mut kv_token_move,
        tok_cap: i32,
        tok_need: *mut i64,
        group_off: *mut i32,
        n_done: *mut i32,
        bad_index: *mut i64,
    ) -> i32;
    pub fn kv_state_evict_window(st: *mut kv_state, seq_id: u64, window: i64, n_freed: *mut i64) -> i32;
    pub fn kv_state_compact(st: *mut kv_state, src: *mut u32, dst: *mut u32, cap: i32, n_moves: *mut i32) -> i32;
    pub fn kv_state_token_count(st: *const kv_state, seq_id: u64, n: *mut i64) -> i32;
    pub fn kv_state_committed(st: *const kv_state, seq_id: u64, tokens: *mut u32, cap: i64, n: *mut i64) -> i32;
    pub fn kv_state_table(
        st: *const kv_state,
        seq_id: u64,
        layer: i32,
        which: i32,
        out: *mut u32,
        cap: i64,
        n: *mut i64,
    ) -> i32;
    pub fn kv_state_export_tables(
        st: *const kv_state,
        seq_ids: *const u64,
        n_seqs: i32,
        layer: i32,
        which: i32,
        out: *mut u32,
        stride: i32,
    ) -> i32;
    pub fn kv_state_free_list(st: *const kv_state, out: *mut u32, cap: i64, n: *mut i64) -> i32;
    pub fn kv_state_refcount(st: *const kv_state, page: u32, count: *mut u32) -> i32;
    pub fn kv_state_pending_base(st: *const kv_state, seq_id: u64, base: *mut i64) -> i32;

    pub fn kv_draft_tree_best_first(
        cand_parent: *const i32,
        cand_token: *const u32,
        cand_prob: *const f64,
        n_cand: i32,
        max_nodes: i32,
        max_depth: i32,
        tokens: *mut u32,
        tree: *mut i32,
        picked: *mut i32,
        n_out: *mut i32,
    ) -> i32;
    pub fn kv_sched_create(out: *mut *mut kv_sched) -> i32;
    pub fn kv_sched_destroy(s: *mut kv_sched) -> i32;
    pub fn kv_sched_add(s: *mut kv_sched, seq_id: u64) -> i32;
    pub fn kv_sched_remove(s: *mut kv_sched, seq_id: u64) -> i32;
    pub fn kv_sched_running(s: *const kv_sched, out: *mut u64, cap: i64, n: *mut i64) -> i32;
    pub fn kv_sched_set_pending(s: *mut kv_sched, seq_id: u64, prefill_tokens: i64) -> i32;
    pub fn kv_sched_plan_step(
        s: *mut kv_sched,
        token_budget: i64,
        chunk_tokens: i32,
        seq_ids: *mut u64,
        n_tokens: *mut i32,
        is_prefill: *mut i32,
        cap: i32,
        n_out: *mut i32,
    ) -> i32;
    pub fn kv_sched_lpt(weights: *const i64, n: i32, n_bins: i32, bins: *mut i32) -> i32;

    pub fn kv_decode_attn_noalloc(
        pages: *const c_void,
        n_pages: u32,
        dtype: i32,
        n_q_heads: i32,
        n_kv_heads: i32,
        rope_cs: *const c_void,
        max_positions: i32,
        q: *const c_void,
        block_tables: *const u32,
        bt_stride: i32,
        seq_lens: *const i32,
        n_seqs: i32,
        window: i32,
        out: *mut c_void,
        status: *mut i32,
        stream: *mut c_void,
    ) -> i32;
}

/// The CUDA runtime calls `DeviceBuffer` needs (libcudart).
#[link(name = "cudart")]
extern "C" {
    pub fn cudaMalloc(dev_ptr: *mut *mut c_void, size: usize) -> i32;
    pub fn cudaFree(dev_ptr: *mut c_void) -> i32;
    pub fn cudaMemset(dev_ptr: *mut c_void, value: i32, count: usize) -> i32;
    pub fn cudaSetDevice(device: i32) -> i32;
}
