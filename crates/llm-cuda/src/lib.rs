//! `llm-cuda`: the CUDA backend of llmhost's paged KV cache, for B200 (sm_100a).
//!
//! The kernels and the host KV state live in `libllmhost_kv.so` (built by
//! `build.rs` with nvcc); this crate binds its C ABI (`ffi`, one declaration
//! per function of `include/llmhost_kv.h`) and wraps it:
//!
//! * [`CudaBackend`] implements `llm_core::Backend` unchanged
//!   (crates/llm-core/src/backend.rs:4-13): `name()` is `"cuda"`, `alloc(len)`
//!   returns a zeroed device buffer of `len` f32.
//! * [`Pool`] owns one device page pool (pages, RoPE table, decode
//!   workspace); its methods are the hot calls: append, decode attention
//!   (plain, with the append fused, with the q/k RMSNorm fused), chunked
//!   prefill / tree verify, page copies and token moves.
//! * [`State`] owns the host-side allocator and every sequence's block
//!   tables: the rules behind `Engine::{open, forward, accept, rollback}`
//!   (crates/llm-engine/src/batch.rs:128-297) and `PagedKv`
//!   (crates/llm-engine/src/cache.rs:12-51), returning the page copies and
//!   token moves a [`Pool`] runs before its next launch.
//!
//! Device pointers are raw (`*const c_void`): the engine owns its device
//! tensors.  Calls on one pool or state are serialised by the caller (the
//! engine's `&mut self`, batch.rs:173), which is what makes the `Send`/`Sync`
//! impls below sound.

pub mod ffi;

use std::ffi::{c_void, CStr};
use std::fmt;
use std::ptr;

pub use ffi::{kv_token_move as TokenMove, KV_PAGE_NONE};

/// Tokens per KV page (the reference's `KV_BLOCK_TOKENS`, cache.rs:10).
pub const PAGE_TOKENS: usize = 16;

/// The data of a reference `TreeError` (crates/llm-engine/src/tree.rs:11-19).
#[derive(Clone, Copy, Debug, PartialEq, Eq)]
pub enum TreeError {
    LengthMismatch { tree: usize, tokens: usize },
    ParentOutOfRange { child: usize, parent: i32 },
    ParentDoesNotPrecede { child: usize, parent: i32 },
}

impl TreeError {
    fn from_ffi(e: &ffi::kv_tree_error) -> Option<Self> {
        match e.kind {
            ffi::KV_TREE_LENGTH_MISMATCH => Some(Self::LengthMismatch { tree: e.tree as usize, tokens: e.tokens as usize }),
            ffi::KV_TREE_PARENT_OUT_OF_RANGE => {
                Some(Self::ParentOutOfRange { child: e.child as usize, parent: e.parent as i32 })
            }
            ffi::KV_TREE_PARENT_DOES_NOT_PRECEDE => {
                Some(Self::ParentDoesNotPrecede { child: e.child as usize, parent: e.parent as i32 })
            }
            _ => None,
        }
    }
}

/// A failed library call.  The engine maps `UnknownSeq`, `NoPendingForward`,
/// `InvalidAccept` and `Tree` one-to-one onto its `EngineError`
/// (batch.rs:59-66); the rest are shape, page-table or device errors.
#[derive(Clone, Debug, PartialEq, Eq)]
pub enum KvError {
    Invalid,
    BadPage,
    Oom,
    Timeout,
    Cuda,
    Unsupported,
    BadPos,
    UnknownSeq(u64),
    NoPendingForward(u64),
    InvalidAccept { seq_id: u64, index: usize },
    Tree { seq_id: u64, error: TreeError },
    Other(i32),
}

impl fmt::Display for KvError {
    fn fmt(&self, f: &mut fmt::Formatter<'_>) -> fmt::Result {
        match self {
            Self::UnknownSeq(s) => write!(f, "unknown sequence {s}"),
            Self::NoPendingForward(s) => write!(f, "sequence {s} has no pending forward"),
            Self::InvalidAccept { seq_id, index } => write!(f, "invalid accept index {index} for sequence {seq_id}"),
            Self::Tree { seq_id, error } => write!(f, "bad tree for sequence {seq_id}: {error:?}"),
            other => write!(f, "{}", status_name(other.status())),
        }
    }
}

impl std::error::Error for KvError {}

impl KvError {
    fn status(&self) -> i32 {
        match self {
            Self::Invalid => ffi::KV_ERR_INVALID,
            Self::BadPage => ffi::KV_ERR_BAD_PAGE,
            Self::Oom => ffi::KV_ERR_OOM,
            Self::Timeout => ffi::KV_ERR_TIMEOUT,
            Self::Cuda => ffi::KV_ERR_CUDA,
            Self::Unsupported => ffi::KV_ERR_UNSUPPORTED,
            Self::BadPos => ffi::KV_ERR_BAD_POS,
            Self::UnknownSeq(_) => ffi::KV_ERR_UNKNOWN_SEQ,
            Self::NoPendingForward(_) => ffi::KV_ERR_NO_PENDING,
            Self::InvalidAccept { .. } => ffi::KV_ERR_INVALID_ACCEPT,
            Self::Tree { .. } => ffi::KV_ERR_TREE,
            Self::Other(s) => *s,
        }
    }
}

/// The library's name for a status code.
pub fn status_name(status: i32) -> String {
    // SAFETY: kv_status_str returns a static NUL-terminated string for any input.
    unsafe { CStr::from_ptr(ffi::kv_status_str(status)) }.to_string_lossy().into_owned()
}

fn check(status: i32) -> Result<(), KvError> {
    check_seq(status, u64::MAX, -1, None)
}

fn check_seq(status: i32, seq_id: u64, bad_index: i64, tree: Option<&ffi::kv_tree_error>) -> Result<(), KvError> {
    Err(match status {
        ffi::KV_OK => return Ok(()),
        ffi::KV_ERR_INVALID => KvError::Invalid,
        ffi::KV_ERR_BAD_PAGE => KvError::BadPage,
        ffi::KV_ERR_OOM => KvError::Oom,
        ffi::KV_ERR_TIMEOUT => KvError::Timeout,
        ffi::KV_ERR_CUDA => KvError::Cuda,
        ffi::KV_ERR_UNSUPPORTED => KvError::Unsupported,
        ffi::KV_ERR_BAD_POS => KvError::BadPos,
        ffi::KV_ERR_UNKNOWN_SEQ => KvError::UnknownSeq(seq_id),
        ffi::KV_ERR_NO_PENDING => KvError::NoPendingForward(seq_id),
        ffi::KV_ERR_INVALID_ACCEPT => KvError::InvalidAccept { seq_id, index: bad_index.max(0) as usize },
        ffi::KV_ERR_TREE => match tree.and_then(TreeError::from_ffi) {
            Some(error) => KvError::Tree { seq_id, error },
            None => KvError::Other(status),
        },
        other => KvError::Other(other),
    })
}

/// KV storage type (the reference's `KvDtype` tags F16/Q8/K8V4 and implements
/// none; `F16` here stores IEEE half, `Q8` and `K8V4` use llm-quant's Q8_0 /
/// Q4 block formats).  `llm_quant::KvDtype::F16` maps to `F16`.
#[derive(Clone, Copy, Debug, PartialEq, Eq)]
pub enum KvDtype {
    F32,
    Bf16,
    Q8,
    K8V4,
    F16,
}

/// Shape and size of a pool (`kv_pool_config`).
#[derive(Clone, Copy, Debug)]
pub struct PoolConfig {
    pub dtype: KvDtype,
    pub n_q_heads: i32,
    pub n_kv_heads: i32,
    pub n_pages: u32,
    pub rope_theta: f32,
    pub max_positions: i32,
    pub max_seqs: i32,
    pub device: i32,
}

impl PoolConfig {
    fn raw(&self) -> ffi::kv_pool_config {
        ffi::kv_pool_config {
            dtype: match self.dtype {
                KvDtype::F32 => ffi::KV_DTYPE_F32,
                KvDtype::Bf16 => ffi::KV_DTYPE_BF16,
                KvDtype::Q8 => ffi::KV_DTYPE_Q8,
                KvDtype::K8V4 => ffi::KV_DTYPE_K8V4,
                KvDtype::F16 => ffi::KV_DTYPE_F16,
            },
            n_q_heads: self.n_q_heads,
            n_kv_heads: self.n_kv_heads,
            head_dim: 64,
            page_tokens: PAGE_TOKENS as i32,
            n_pages: self.n_pages,
            rope_theta: self.rope_theta,
            max_positions: self.max_positions,
            max_seqs: self.max_seqs,
            device: self.device,
        }
    }
}

/// A device page pool.  Every method enqueues on `stream` (a `cudaStream_t`,
/// null for the legacy stream) and returns without waiting; device-side
/// errors (bad page ids, positions, timeouts) are read with
/// [`Pool::last_error`], off the hot path.
pub struct Pool {
    raw: *mut ffi::kv_pool,
}

// SAFETY: the pool handle is only used through &self / &mut self methods and
// the library serialises nothing itself; the engine serialises calls.
unsafe impl Send for Pool {}
unsafe impl Sync for Pool {}

impl Pool {
    pub fn new(cfg: &PoolConfig) -> Result<Self, KvError> {
        let raw_cfg = cfg.raw();
        let mut raw = ptr::null_mut();
        // SAFETY: both pointers are valid for the call.
        check(unsafe { ffi::kv_pool_create(&raw_cfg, &mut raw) })?;
        Ok(Self { raw })
    }

    /// Device address of page 0 and the size of one page in bytes.
    pub fn pages(&self) -> (*mut c_void, usize) {
        // SAFETY: self.raw is a live pool.
        unsafe { (ffi::kv_pool_pages(self.raw), ffi::kv_pool_page_bytes(self.raw)) }
    }

    /// Read and clear the device error word (synchronises the pool's device).
    pub fn last_error(&mut self) -> Result<(), KvError> {
        // SAFETY: self.raw is a live pool.
        check(unsafe { ffi::kv_last_error(self.raw) })
    }

    /// `kv_append`: K/V of n tokens into their slots, K rotated at `tok_pos`.
    ///
    /// # Safety
    /// Every pointer is device memory of the size the header states.
    #[allow(clippy::too_many_arguments)]
    pub unsafe fn append(
        &mut self,
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
    ) -> Result<(), KvError> {
        check(ffi::kv_append(self.raw, k, v, tok_seq, tok_slot, tok_pos, n_tokens, block_tables, n_seqs, bt_stride, stream))
    }

    /// `kv_append_decode_attn`: one decode step of a layer (the token's K/V
    /// store and attention_decode_cached, lfm2.rs:828-832 and :1006-1056).
    ///
    /// # Safety
    /// Every pointer is device memory of the size the header states.
    #[allow(clippy::too_many_arguments)]
    pub unsafe fn append_decode_attn(
        &mut self,
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
    ) -> Result<(), KvError> {
        check(ffi::kv_append_decode_attn(self.raw, k, v, q, block_tables, bt_stride, seq_lens, n_seqs, window, out, stream))
    }

    /// `kv_norm_append_decode_attn`: [`Pool::append_decode_attn`] with the
    /// layer's q/k RMSNorm (lfm2.rs:797-812) folded in.
    ///
    /// # Safety
    /// Every pointer is device memory of the size the header states.
    #[allow(clippy::too_many_arguments)]
    pub unsafe fn norm_append_decode_attn(
        &mut self,
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
    ) -> Result<(), KvError> {
        check(ffi::kv_norm_append_decode_attn(
            self.raw, k, v, q, q_norm, k_norm, eps, block_tables, bt_stride, seq_lens, n_seqs, window, out, stream,
        ))
    }

    /// `kv_decode_attn`: attention_decode_cached over paged K/V.
    ///
    /// # Safety
    /// Every pointer is device memory of the size the header states.
    #[allow(clippy::too_many_arguments)]
    pub unsafe fn decode_attn(
        &mut self,
        q: *const c_void,
        block_tables: *const u32,
        bt_stride: i32,
        seq_lens: *const i32,
        n_seqs: i32,
        window: i32,
        out: *mut c_void,
        stream: *mut c_void,
    ) -> Result<(), KvError> {
        check(ffi::kv_decode_attn(self.raw, q, block_tables, bt_stride, seq_lens, n_seqs, window, out, stream))
    }

    /// `kv_prefill_attn`: a causal chunk after a cached prefix, or a draft
    /// tree with ancestor-or-self masks (`tree_masks` non-null).
    ///
    /// # Safety
    /// Every pointer is device memory of the size the header states.
    #[allow(clippy::too_many_arguments)]
    pub unsafe fn prefill_attn(
        &mut self,
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
    ) -> Result<(), KvError> {
        check(ffi::kv_prefill_attn(
            self.raw, q, q_pos, q_offsets, prefix_lens, tree_masks, block_tables, bt_stride, n_seqs, max_q_per_seq, out, stream,
        ))
    }

    /// `kv_copy_pages`: copy-on-write and compaction copies (device arrays).
    ///
    /// # Safety
    /// `src` and `dst` are device arrays of `n` page ids.
    pub unsafe fn copy_pages(&mut self, src: *const u32, dst: *const u32, n: i32, stream: *mut c_void) -> Result<(), KvError> {
        check(ffi::kv_copy_pages(self.raw, src, dst, n, stream))
    }

    /// `kv_move_tokens`: the accepted draft tokens' moves, in groups.
    ///
    /// # Safety
    /// `moves` and `group_offsets` are device arrays of the stated lengths.
    pub unsafe fn move_tokens(
        &mut self,
        moves: *const TokenMove,
        n_moves: i32,
        group_offsets: *const i32,
        n_groups: i32,
        stream: *mut c_void,
    ) -> Result<(), KvError> {
        check(ffi::kv_move_tokens(self.raw, moves, n_moves, group_offsets, n_groups, stream))
    }
}

impl Drop for Pool {
    fn drop(&mut self) {
        // SAFETY: self.raw is live and dropped once.
        unsafe {
            ffi::kv_pool_destroy(self.raw);
        }
    }
}

/// What a staged draft needs on the device: copy-on-write pairs to run first,
/// then each token's storage slot and RoPE position.
#[derive(Clone, Debug, Default, PartialEq, Eq)]
pub struct ForwardPlan {
    pub slots: Vec<i32>,
    pub positions: Vec<i32>,
    pub cow: Vec<(u32, u32)>,
}

/// The host KV state: page allocator and block tables of every sequence.
pub struct State {
    raw: *mut ffi::kv_state,
    n_layers: usize,
}

// SAFETY: as for Pool; the engine serialises calls on one state.
unsafe impl Send for State {}
unsafe impl Sync for State {}

impl State {
    /// `alloc_order`: the order of the first page allocations (empty: 0, 1, 2, ...).
    pub fn new(n_pages: u32, n_layers: usize, alloc_order: &[u32]) -> Result<Self, KvError> {
        let mut raw = ptr::null_mut();
        let order = if alloc_order.is_empty() { ptr::null() } else { alloc_order.as_ptr() };
        // SAFETY: order points at alloc_order.len() ids or is null.
        check(unsafe {
            ffi::kv_state_create(n_pages, n_layers as i32, PAGE_TOKENS as i32, order, alloc_order.len() as u32, &mut raw)
        })?;
        Ok(Self { raw, n_layers })
    }

    pub fn open(&mut self, seq_id: u64) -> Result<(), KvError> {
        // SAFETY: self.raw is live.
        check_seq(unsafe { ffi::kv_state_open(self.raw, seq_id) }, seq_id, -1, None)
    }

    pub fn close(&mut self, seq_id: u64) -> Result<(), KvError> {
        // SAFETY: self.raw is live.
        check_seq(unsafe { ffi::kv_state_close(self.raw, seq_id) }, seq_id, -1, None)
    }

    /// A new sequence `dst` sharing every committed page of `src`.
    pub fn fork(&mut self, src: u64, dst: u64) -> Result<(), KvError> {
        // SAFETY: self.raw is live.
        check_seq(unsafe { ffi::kv_state_fork(self.raw, src, dst) }, src, -1, None)
    }

    /// Commit `tokens` straight into the sequence's KV; returns the page
    /// copies (copy-on-write) to run before the K/V append.
    pub fn append(&mut self, seq_id: u64, tokens: &[u32]) -> Result<Vec<(u32, u32)>, KvError> {
        let cap = self.n_layers.max(1);
        let (mut src, mut dst) = (vec![0u32; cap], vec![0u32; cap]);
        let mut n = 0i32;
        // SAFETY: buffers hold cap entries; tokens holds tokens.len().
        check_seq(
            unsafe {
                ffi::kv_state_append(self.raw, seq_id, tokens.as_ptr(), tokens.len() as i32, src.as_mut_ptr(), dst.as_mut_ptr(), cap as i32, &mut n)
            },
            seq_id,
            -1,
            None,
        )?;
        Ok(src.into_iter().zip(dst).take(n as usize).collect())
    }

    /// `Engine::forward` of a draft (batch.rs:173-222): `tree` is the parent
    /// array (`None`: a chain), validated as tree.rs:48-100 does.
    pub fn forward(&mut self, seq_id: u64, tokens: &[u32], tree: Option<&[i32]>) -> Result<ForwardPlan, KvError> {
        let n = tokens.len();
        let cap = self.n_layers.max(1);
        let mut plan = ForwardPlan { slots: vec![0; n], positions: vec![0; n], cow: Vec::new() };
        let (mut src, mut dst) = (vec![0u32; cap], vec![0u32; cap]);
        let (mut n_cow, mut err) = (0i32, ffi::kv_tree_error::default());
        let (tp, tl) = match tree {
            Some(t) => (t.as_ptr(), t.len() as i32),
            None => (ptr::null(), 0),
        };
        // SAFETY: every buffer is sized as the header asks.
        let rc = unsafe {
            ffi::kv_state_forward(
                self.raw,
                seq_id,
                tokens.as_ptr(),
                n as i32,
                tp,
                tl,
                plan.slots.as_mut_ptr(),
                plan.positions.as_mut_ptr(),
                src.as_mut_ptr(),
                dst.as_mut_ptr(),
                cap as i32,
                &mut n_cow,
                &mut err,
            )
        };
        check_seq(rc, seq_id, -1, Some(&err))?;
        plan.cow = src.into_iter().zip(dst).take(n_cow as usize).collect();
        Ok(plan)
    }

    fn commit(&mut self, seq_id: u64, idx: &[i64], accept: bool) -> Result<Vec<TokenMove>, KvError> {
        let mut base = 0i64;
        // SAFETY: self.raw is live.  Fails with NoPendingForward when nothing is staged.
        check_seq(unsafe { ffi::kv_state_pending_base(self.raw, seq_id, &mut base) }, seq_id, -1, None)?;
        // The draft table's page count bounds the staged tokens (the moves of
        // one layer); a null buffer with cap 0 asks for the count only.
        let mut draft_pages = 0i64;
        // SAFETY: self.raw is live; no buffer is written with cap 0.
        let rc = unsafe { ffi::kv_state_table(self.raw, seq_id, 0, 1, ptr::null_mut(), 0, &mut draft_pages) };
        if rc != ffi::KV_OK && rc != ffi::KV_ERR_INVALID {
            check_seq(rc, seq_id, -1, None)?;
        }
        let per = (draft_pages.max(0) as usize * PAGE_TOKENS).max(1);
        let cap = per * self.n_layers.max(1);
        let (mut ms, mut md) = (vec![0i32; per], vec![0i32; per]);
        let mut moves = vec![TokenMove::default(); cap];
        let (mut n_moves, mut n_tok, mut bad) = (0i32, 0i32, -1i64);
        // SAFETY: every buffer is sized above.
        let rc = unsafe {
            let f = if accept { ffi::kv_state_accept } else { ffi::kv_state_rollback };
            f(
                self.raw,
                seq_id,
                idx.as_ptr(),
                idx.len() as i32,
                ms.as_mut_ptr(),
                md.as_mut_ptr(),
                per as i32,
                &mut n_moves,
                moves.as_mut_ptr(),
                cap as i32,
                &mut n_tok,
                &mut bad,
            )
        };
        check_seq(rc, seq_id, bad, None)?;
        moves.truncate(n_tok as usize);
        Ok(moves)
    }

    /// `Engine::accept` (batch.rs:224-253): commit an accepted path of the
    /// staged draft; returns the token moves (every layer, addressed by page)
    /// to run with [`Pool::move_tokens`] before the next launch.
    pub fn accept(&mut self, seq_id: u64, accepted: &[usize]) -> Result<Vec<TokenMove>, KvError> {
        let idx: Vec<i64> = accepted.iter().map(|&i| i as i64).collect();
        self.commit(seq_id, &idx, true)
    }

    /// `Engine::rollback` (batch.rs:255-296): commit the complement of `rejected`.
    pub fn rollback(&mut self, seq_id: u64, rejected: &[usize]) -> Result<Vec<TokenMove>, KvError> {
        let idx: Vec<i64> = rejected.iter().map(|&i| i as i64).collect();
        self.commit(seq_id, &idx, false)
    }

    /// Free the pages wholly below `token_count - window`; returns how many.
    pub fn evict_window(&mut self, seq_id: u64, window: i64) -> Result<i64, KvError> {
        let mut n = 0i64;
        // SAFETY: self.raw is live.
        check_seq(unsafe { ffi::kv_state_evict_window(self.raw, seq_id, window, &mut n) }, seq_id, -1, None)?;
        Ok(n)
    }

    /// Move used pages into the lowest ids; returns the page copies to run
    /// (then re-export every table).
    pub fn compact(&mut self) -> Result<Vec<(u32, u32)>, KvError> {
        let mut n = 0i32;
        // SAFETY: a null buffer with cap 0 asks for the count only.
        let rc = unsafe { ffi::kv_state_compact(self.raw, ptr::null_mut(), ptr::null_mut(), 0, &mut n) };
        if rc != ffi::KV_OK && rc != ffi::KV_ERR_INVALID {
            check(rc)?;
        }
        let (mut src, mut dst) = (vec![0u32; n.max(1) as usize], vec![0u32; n.max(1) as usize]);
        // SAFETY: buffers hold n entries.
        check(unsafe { ffi::kv_state_compact(self.raw, src.as_mut_ptr(), dst.as_mut_ptr(), n, &mut n) })?;
        Ok(src.into_iter().zip(dst).take(n as usize).collect())
    }

    /// `PagedKv::token_count` (cache.rs:31-34).
    pub fn token_count(&self, seq_id: u64) -> Result<usize, KvError> {
        let mut n = 0i64;
        // SAFETY: self.raw is live.
        check_seq(unsafe { ffi::kv_state_token_count(self.raw, seq_id, &mut n) }, seq_id, -1, None)?;
        Ok(n as usize)
    }

    /// `PagedKv::allocated_blocks` (cache.rs:36-39).
    pub fn allocated_blocks(&self, seq_id: u64) -> Result<usize, KvError> {
        Ok(self.token_count(seq_id)?.div_ceil(PAGE_TOKENS))
    }

    /// Rows of block tables for one launch: `out[i * stride + j]`, padded
    /// with [`KV_PAGE_NONE`]; `draft` selects the staged draft's tables.
    pub fn export_tables(&self, seq_ids: &[u64], layer: usize, stride: usize, draft: bool) -> Result<Vec<u32>, KvError> {
        let mut out = vec![KV_PAGE_NONE; seq_ids.len() * stride];
        // SAFETY: out holds seq_ids.len() * stride entries.
        check(unsafe {
            ffi::kv_state_export_tables(
                self.raw,
                seq_ids.as_ptr(),
                seq_ids.len() as i32,
                layer as i32,
                i32::from(draft),
                out.as_mut_ptr(),
                stride as i32,
            )
        })?;
        Ok(out)
    }
}

impl Drop for State {
    fn drop(&mut self) {
        // SAFETY: self.raw is live and dropped once.
        unsafe {
            ffi::kv_state_destroy(self.raw);
        }
    }
}

/// Zeroed device storage of `len` f32 (`Backend::Buffer`).
pub struct DeviceBuffer {
    ptr: *mut c_void,
    len: usize,
}

// SAFETY: a device allocation has no thread affinity.
unsafe impl Send for DeviceBuffer {}
unsafe impl Sync for DeviceBuffer {}

impl DeviceBuffer {
    pub fn len(&self) -> usize {
        self.len
    }

    pub fn is_empty(&self) -> bool {
        self.len == 0
    }

    /// Device address of element 0 (null when empty).
    pub fn as_ptr(&self) -> *mut c_void {
        self.ptr
    }
}

impl Drop for DeviceBuffer {
    fn drop(&mut self) {
        if !self.ptr.is_null() {
            // SAFETY: ptr came from cudaMalloc and is freed once.
            unsafe {
                ffi::cudaFree(self.ptr);
            }
        }
    }
}

/// The CUDA backend of `llm_core::Backend` (crates/llm-core/src/backend.rs:4-13),
/// for one device; its KV pools are created with [`Pool::new`].
pub struct CudaBackend {
    device: i32,
}

impl CudaBackend {
    pub fn new(device: i32) -> Self {
        Self { device }
    }
}

impl llm_core::Backend for CudaBackend {
    type Buffer = DeviceBuffer;

    fn name(&self) -> &'static str {
        "cuda"
    }

    fn alloc(&self, len: usize) -> DeviceBuffer {
        if len == 0 {
            return DeviceBuffer { ptr: ptr::null_mut(), len: 0 };
        }
        let mut p = ptr::null_mut();
        let bytes = len * std::mem::size_of::<f32>();
        // SAFETY: p receives a fresh allocation of `bytes` on self.device.
        let ok = unsafe {
            ffi::cudaSetDevice(self.device) == 0 && ffi::cudaMalloc(&mut p, bytes) == 0 && ffi::cudaMemset(p, 0, bytes) == 0
        };
        assert!(ok, "cudaMalloc of {bytes} bytes on device {} failed", self.device);
        DeviceBuffer { ptr: p, len }
    }
}
