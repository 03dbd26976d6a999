"""Torch-facing wrapper of the C ABI: device tensors in, device tensors out.

`KvPool` is the object a `crates/llm-cuda` Backend would own (one pool of
physical pages shared by every attention layer).  All methods pass raw device
pointers of torch tensors straight to libllmhost_kv.so and launch on the
current torch CUDA stream; nothing is computed on the host.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _capi
from ._capi import KV_DTYPE_BF16, KV_DTYPE_F16, KV_DTYPE_F32, KV_DTYPE_K8V4, KV_DTYPE_Q8, KvPoolConfig, check
from .plans import tree_masks  # noqa: F401  (ancestor-or-self masks for prefill_attn)

# The dtype of k, v, q and out: quantised pools take bf16 and store codes.
_TORCH_DTYPE = {KV_DTYPE_F32: torch.float32, KV_DTYPE_BF16: torch.bfloat16, KV_DTYPE_Q8: torch.bfloat16,
                KV_DTYPE_K8V4: torch.bfloat16, KV_DTYPE_F16: torch.bfloat16}


def dtype_code(dtype) -> int:
    if dtype in ("bf16", torch.bfloat16, KV_DTYPE_BF16):
        return KV_DTYPE_BF16
    if dtype in ("f32", "fp32", torch.float32, KV_DTYPE_F32):
        return KV_DTYPE_F32
    if dtype in ("q8", KV_DTYPE_Q8):
        return KV_DTYPE_Q8
    if dtype in ("k8v4", KV_DTYPE_K8V4):
        return KV_DTYPE_K8V4
    if dtype in ("f16", KV_DTYPE_F16):  # half pages; k, v, q and out stay bf16
        return KV_DTYPE_F16
    raise ValueError(f"unsupported KV dtype {dtype!r}")


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream_ptr(stream) -> int | None:
    if stream is None:
        stream = torch.cuda.current_stream()
    return stream.cuda_stream


@dataclass(frozen=True)
class PoolShape:
    dtype: int
    n_q_heads: int
    n_kv_heads: int
    head_dim: int
    page_tokens: int
    n_pages: int

    @property
    def torch_dtype(self) -> torch.dtype:
        return _TORCH_DTYPE[self.dtype]

    @property
    def quantised(self) -> bool:
        return self.dtype in (KV_DTYPE_Q8, KV_DTYPE_K8V4)

    @property
    def page_elems(self) -> int:
        """Elements of one page: f32 / bf16 values, or bytes of a quantised page
        (per kv head: K codes, V codes, scales)."""
        if self.quantised:
            vrow = self.head_dim if self.dtype == KV_DTYPE_Q8 else self.head_dim // 2
            return self.n_kv_heads * self.page_tokens * (self.head_dim + vrow + 8)
        return 2 * self.n_kv_heads * self.page_tokens * self.head_dim


class KvPool:
    """A device page pool plus the RoPE table and attention workspace."""

    def __init__(self, *, dtype="bf16", n_q_heads=24, n_kv_heads=8, head_dim=64, page_tokens=16,
                 n_pages=4096, rope_theta=1e6, max_positions=1 << 17, max_seqs=1024, device=0):
        self._lib = _capi.lib()
        code = dtype_code(dtype)
        cfg = KvPoolConfig(code, n_q_heads, n_kv_heads, head_dim, page_tokens, n_pages,
                           float(rope_theta), max_positions, max_seqs, device)
        handle = _capi.c_void_p()
        check(self._lib.kv_pool_create(cfg, handle), "kv_pool_create")
        self._h = handle.value
        self.shape = PoolShape(code, n_q_heads, n_kv_heads, head_dim, page_tokens, n_pages)
        self.device = torch.device("cuda", device)
        self.max_positions = max_positions
        self.max_seqs = max_seqs
        self.page_bytes = int(self._lib.kv_pool_page_bytes(self._h))

    # -- lifetime ---------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "_h", None):
            check(self._lib.kv_pool_destroy(self._h), "kv_pool_destroy")
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def handle(self) -> int:
        return self._h

    # -- errors / page I/O ------------------------------------------------
    def last_error(self) -> int:
        return int(self._lib.kv_last_error(self._h))

    def check_device_error(self) -> None:
        check(self.last_error(), "device error word")

    def read_pages(self, page_ids) -> np.ndarray:
        """Pages as a host array [n, page_elems] (bf16 and f16 returned as
        uint16 bits, quantised pages as bytes)."""
        ids = np.ascontiguousarray(page_ids, dtype=np.uint32)
        np_dt = {KV_DTYPE_BF16: np.uint16, KV_DTYPE_F16: np.uint16, KV_DTYPE_F32: np.float32}.get(
            self.shape.dtype, np.uint8)
        out = np.empty((len(ids), self.shape.page_elems), dtype=np_dt)
        check(self._lib.kv_pool_read_pages(self._h, ids.ctypes.data, len(ids), out.ctypes.data),
              "kv_pool_read_pages")
        return out

    def write_pages(self, page_ids, data: np.ndarray) -> None:
        ids = np.ascontiguousarray(page_ids, dtype=np.uint32)
        data = np.ascontiguousarray(data)
        assert data.nbytes == len(ids) * self.page_bytes
        check(self._lib.kv_pool_write_pages(self._h, ids.ctypes.data, len(ids), data.ctypes.data),
              "kv_pool_write_pages")

    # -- hot path ---------------------------------------------------------
    def _check_tensor(self, t: torch.Tensor, name: str, dtype=None) -> None:
        if t.device != self.device:
            raise ValueError(f"{name} must live on {self.device}, got {t.device}")
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
        if dtype is not None and t.dtype != dtype:
            raise ValueError(f"{name} must be {dtype}, got {t.dtype}")

    def append(self, k, v, tok_seq, tok_slot, tok_pos, block_tables, stream=None) -> None:
        """K/V of n tokens into their slots; K rotated at tok_pos (kv_append)."""
        dt = self.shape.torch_dtype
        for t, nm in ((k, "k"), (v, "v")):
            self._check_tensor(t, nm, dt)
        for t, nm in ((tok_seq, "tok_seq"), (tok_slot, "tok_slot"), (tok_pos, "tok_pos")):
            self._check_tensor(t, nm, torch.int32)
        self._check_tensor(block_tables, "block_tables", torch.int32)
        n = tok_seq.numel()
        rows = block_tables.shape[0] if block_tables.dim() == 2 else 1
        check(self._lib.kv_append(self._h, _ptr(k), _ptr(v), _ptr(tok_seq), _ptr(tok_slot),
                                  _ptr(tok_pos), n, _ptr(block_tables), rows, block_tables.shape[-1],
                                  _stream_ptr(stream)), "kv_append")

    def append_decode(self, k, v, block_tables, seq_lens, stream=None) -> None:
        """One token per sequence at position seq_lens[s] - 1 (kv_append_decode)."""
        dt = self.shape.torch_dtype
        self._check_tensor(k, "k", dt)
        self._check_tensor(v, "v", dt)
        self._check_tensor(block_tables, "block_tables", torch.int32)
        self._check_tensor(seq_lens, "seq_lens", torch.int32)
        check(self._lib.kv_append_decode(self._h, _ptr(k), _ptr(v), _ptr(block_tables),
                                         block_tables.shape[-1], _ptr(seq_lens), seq_lens.numel(),
                                         _stream_ptr(stream)), "kv_append_decode")

    def copy_pages(self, src, dst, stream=None) -> None:
        """Independent page copies src[i] -> dst[i] (device int32 tensors; kv_copy_pages)."""
        self._check_tensor(src, "src", torch.int32)
        self._check_tensor(dst, "dst", torch.int32)
        check(self._lib.kv_copy_pages(self._h, _ptr(src), _ptr(dst), src.numel(), _stream_ptr(stream)),
              "kv_copy_pages")

    def move_tokens(self, moves, group_offsets, stream=None) -> None:
        """Token moves (device int32 tensor [n, 4] of src_page, src_slot, dst_page, dst_slot)
        in groups (device int32 tensor of n_groups + 1 offsets; kv_move_tokens)."""
        self._check_tensor(moves, "moves", torch.int32)
        self._check_tensor(group_offsets, "group_offsets", torch.int32)
        check(self._lib.kv_move_tokens(self._h, _ptr(moves), moves.shape[0], _ptr(group_offsets),
                                       group_offsets.numel() - 1, _stream_ptr(stream)), "kv_move_tokens")

    def decode_attn(self, q, block_tables, seq_lens, window: int = 0, out=None, stream=None):
        """Paged decode attention (kv_decode_attn); returns `out`."""
        dt = self.shape.torch_dtype
        self._check_tensor(q, "q", dt)
        self._check_tensor(block_tables, "block_tables", torch.int32)
        self._check_tensor(seq_lens, "seq_lens", torch.int32)
        if out is None:
            out = torch.empty_like(q)
        self._check_tensor(out, "out", dt)
        check(self._lib.kv_decode_attn(self._h, _ptr(q), _ptr(block_tables), block_tables.shape[-1],
                                       _ptr(seq_lens), seq_lens.numel(), int(window), _ptr(out),
                                       _stream_ptr(stream)), "kv_decode_attn")
        return out

    def append_decode_attn(self, k, v, q, block_tables, seq_lens, window: int = 0, out=None, stream=None):
        """append_decode then decode_attn in one launch (kv_append_decode_attn),
        bit-identical to the two calls; returns `out`."""
        dt = self.shape.torch_dtype
        self._check_tensor(k, "k", dt)
        self._check_tensor(v, "v", dt)
        self._check_tensor(q, "q", dt)
        self._check_tensor(block_tables, "block_tables", torch.int32)
        self._check_tensor(seq_lens, "seq_lens", torch.int32)
        if out is None:
            out = torch.empty_like(q)
        self._check_tensor(out, "out", dt)
        check(self._lib.kv_append_decode_attn(self._h, _ptr(k), _ptr(v), _ptr(q), _ptr(block_tables),
                                              block_tables.shape[-1], _ptr(seq_lens), seq_lens.numel(),
                                              int(window), _ptr(out), _stream_ptr(stream)),
              "kv_append_decode_attn")
        return out

    def norm_append_decode_attn(self, k, v, q, q_norm, k_norm, eps: float, block_tables, seq_lens,
                                window: int = 0, out=None, stream=None):
        """append_decode_attn with the per-head RMSNorm of q and k before RoPE
        (kv_norm_append_decode_attn); q_norm, k_norm: fp32 [head_dim] device
        tensors.  Returns `out`."""
        dt = self.shape.torch_dtype
        for t, name in ((k, "k"), (v, "v"), (q, "q")):
            self._check_tensor(t, name, dt)
        self._check_tensor(q_norm, "q_norm", torch.float32)
        self._check_tensor(k_norm, "k_norm", torch.float32)
        self._check_tensor(block_tables, "block_tables", torch.int32)
        self._check_tensor(seq_lens, "seq_lens", torch.int32)
        if out is None:
            out = torch.empty_like(q)
        self._check_tensor(out, "out", dt)
        check(self._lib.kv_norm_append_decode_attn(self._h, _ptr(k), _ptr(v), _ptr(q), _ptr(q_norm), _ptr(k_norm),
                                                   float(eps), _ptr(block_tables), block_tables.shape[-1],
                                                   _ptr(seq_lens), seq_lens.numel(), int(window), _ptr(out),
                                                   _stream_ptr(stream)), "kv_norm_append_decode_attn")
        return out

    def prefill_attn(self, q, q_pos, q_offsets, prefix_lens, block_tables, tree_masks=None,
                     max_q: int | None = None, out=None, stream=None):
        """Chunked-prefill / tree-verify attention (kv_prefill_attn); returns `out`.

        q [total_q, n_q, d] raw (RoPE applied here at q_pos), q_offsets [n_seqs + 1],
        prefix_lens [n_seqs] cached tokens before each chunk, tree_masks None (causal
        chunk) or int64 [total_q] ancestor-or-self bit masks.  max_q bounds the chunk
        length of every sequence; when None it is read from q_offsets (a device sync).
        """
        dt = self.shape.torch_dtype
        self._check_tensor(q, "q", dt)
        for t, nm in ((q_pos, "q_pos"), (q_offsets, "q_offsets"), (prefix_lens, "prefix_lens"),
                      (block_tables, "block_tables")):
            self._check_tensor(t, nm, torch.int32)
        if tree_masks is not None:
            self._check_tensor(tree_masks, "tree_masks", torch.int64)
        n_seqs = prefix_lens.numel()
        if q_offsets.numel() != n_seqs + 1:
            raise ValueError("q_offsets must hold n_seqs + 1 entries")
        if max_q is None:
            max_q = int((q_offsets[1:] - q_offsets[:-1]).max().item()) if n_seqs else 0
        if out is None:
            out = torch.empty_like(q)
        self._check_tensor(out, "out", dt)
        check(self._lib.kv_prefill_attn(self._h, _ptr(q), _ptr(q_pos), _ptr(q_offsets), _ptr(prefix_lens),
                                        _ptr(tree_masks), _ptr(block_tables), block_tables.shape[-1],
                                        n_seqs, int(max_q), _ptr(out), _stream_ptr(stream)),
              "kv_prefill_attn")
        return out

    def prefill_shared_workspace(self, n_seqs: int, max_q: int) -> torch.Tensor:
        """A workspace for prefill_attn_shared (device bytes)."""
        nbytes = int(self._lib.kv_prefill_shared_workspace_bytes(self._h, int(n_seqs), int(max_q)))
        return torch.empty(max(nbytes, 16), dtype=torch.uint8, device=self.device)

    def prefill_attn_shared(self, q, q_pos, q_offsets, prefix_lens, block_tables, shared_tokens: int, max_q: int,
                            tree_masks=None, workspace=None, out=None, stream=None):
        """prefill_attn for sequences that all begin with the same shared_tokens
        tokens on the same pages (kv_prefill_attn_shared): the shared keys in
        one pass for the whole batch, each sequence's own keys in a second,
        merged.  Returns `out`."""
        dt = self.shape.torch_dtype
        self._check_tensor(q, "q", dt)
        for t, nm in ((q_pos, "q_pos"), (q_offsets, "q_offsets"), (prefix_lens, "prefix_lens"),
                      (block_tables, "block_tables")):
            self._check_tensor(t, nm, torch.int32)
        if tree_masks is not None:
            self._check_tensor(tree_masks, "tree_masks", torch.int64)
        n_seqs = prefix_lens.numel()
        if q_offsets.numel() != n_seqs + 1:
            raise ValueError("q_offsets must hold n_seqs + 1 entries")
        if workspace is None:
            workspace = self.prefill_shared_workspace(n_seqs, max_q)
        if out is None:
            out = torch.empty_like(q)
        self._check_tensor(out, "out", dt)
        check(self._lib.kv_prefill_attn_shared(self._h, _ptr(q), _ptr(q_pos), _ptr(q_offsets), _ptr(prefix_lens),
                                               _ptr(tree_masks), _ptr(block_tables), block_tables.shape[-1],
                                               n_seqs, int(max_q), int(shared_tokens), _ptr(workspace), _ptr(out),
                                               _stream_ptr(stream)),
              "kv_prefill_attn_shared")
        return out

