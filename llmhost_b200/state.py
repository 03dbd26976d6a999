"""Python view of the host-side KV state (kv_state_* in include/llmhost_kv.h).

`KvState` mirrors llm-engine's `Engine` (crates/llm-engine/src/batch.rs:128-297)
and `PagedKv` (crates/llm-engine/src/cache.rs:12-51) with pages behind them:
`forward` stages draft tokens and returns where they go, `accept` / `rollback`
commit a path and return the slot moves to run on the device.  All logic
lives in the C++ library; this module only marshals arguments.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_int32, c_int64, c_uint32, c_uint64, c_void_p
from dataclasses import dataclass, field

import numpy as np

from . import _capi

PAGE_TOKENS = 16
TREE_KINDS = {1: "LengthMismatch", 2: "ParentOutOfRange", 3: "ParentDoesNotPrecede"}


class KvTreeError(ctypes.Structure):
    _fields_ = [("kind", c_int32), ("child", c_int64), ("parent", c_int64), ("tree", c_int64),
                ("tokens", c_int64)]


class TreeError(ValueError):
    """tree.rs:11-19: LengthMismatch { tree, tokens } / ParentOutOfRange /
    ParentDoesNotPrecede { child, parent }."""

    def __init__(self, e: KvTreeError):
        self.kind = TREE_KINDS.get(e.kind, str(e.kind))
        self.child, self.parent, self.tree, self.tokens = e.child, e.parent, e.tree, e.tokens
        if self.kind == "LengthMismatch":
            msg = f"tree length {self.tree} does not match token length {self.tokens}"
        elif self.kind == "ParentOutOfRange":
            msg = f"token {self.child} has out-of-range parent {self.parent}"
        else:
            msg = f"parent {self.parent} does not precede child {self.child}"
        super().__init__(msg)

    def key(self):
        if self.kind == "LengthMismatch":
            return (self.kind, self.tree, self.tokens)
        return (self.kind, self.child, self.parent)


class EngineError(RuntimeError):
    """batch.rs:59-66: Tree / UnknownSeq / NoPendingForward / InvalidAccept."""

    def __init__(self, kind: str, seq_id: int, index: int | None = None, tree: TreeError | None = None):
        self.kind, self.seq_id, self.index, self.tree = kind, seq_id, index, tree
        super().__init__(f"{kind}(seq {seq_id}" + (f", index {index}" if index is not None else "") + ")")


STATE_SIGNATURES = [
    ("kv_tree_validate", c_int32, [c_void_p, c_int32, c_int32, POINTER(KvTreeError)]),
    ("kv_tree_validate_accept", c_int32, [c_void_p, c_int32, c_void_p, c_int32, POINTER(KvTreeError)]),
    ("kv_state_create", c_int32, [c_uint32, c_int32, c_int32, c_void_p, c_uint32, POINTER(c_void_p)]),
    ("kv_state_destroy", c_int32, [c_void_p]),
    ("kv_state_open", c_int32, [c_void_p, c_uint64]),
    ("kv_state_close", c_int32, [c_void_p, c_uint64]),
    ("kv_state_fork", c_int32, [c_void_p, c_uint64, c_uint64]),
    ("kv_state_append", c_int32, [c_void_p, c_uint64, c_void_p, c_int32, c_void_p, c_void_p, c_int32,
                                  POINTER(c_int32)]),
    ("kv_state_forward", c_int32, [c_void_p, c_uint64, c_void_p, c_int32, c_void_p, c_int32, c_void_p,
                                   c_void_p, c_void_p, c_void_p, c_int32, POINTER(c_int32),
                                   POINTER(KvTreeError)]),
    ("kv_state_accept", c_int32, [c_void_p, c_uint64, c_void_p, c_int32, c_void_p, c_void_p, c_int32,
                                  POINTER(c_int32), c_void_p, c_int32, POINTER(c_int32), POINTER(c_int64)]),
    ("kv_state_rollback", c_int32, [c_void_p, c_uint64, c_void_p, c_int32, c_void_p, c_void_p, c_int32,
                                    POINTER(c_int32), c_void_p, c_int32, POINTER(c_int32), POINTER(c_int64)]),
    ("kv_state_evict_window", c_int32, [c_void_p, c_uint64, c_int64, POINTER(c_int64)]),
    ("kv_state_compact", c_int32, [c_void_p, c_void_p, c_void_p, c_int32, POINTER(c_int32)]),
    ("kv_state_token_count", c_int32, [c_void_p, c_uint64, POINTER(c_int64)]),
    ("kv_state_committed", c_int32, [c_void_p, c_uint64, c_void_p, c_int64, POINTER(c_int64)]),
    ("kv_state_table", c_int32, [c_void_p, c_uint64, c_int32, c_int32, c_void_p, c_int64, POINTER(c_int64)]),
    ("kv_state_export_tables", c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p, c_int32]),
    ("kv_state_free_list", c_int32, [c_void_p, c_void_p, c_int64, POINTER(c_int64)]),
    ("kv_state_refcount", c_int32, [c_void_p, c_uint32, POINTER(c_uint32)]),
    ("kv_state_pending_base", c_int32, [c_void_p, c_uint64, POINTER(c_int64)]),
    ("kv_state_forward_batch", c_int32, [c_void_p, c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_void_p,
                                         c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32,
                                         POINTER(c_int32), c_void_p, c_int32, POINTER(c_int32),
                                         POINTER(KvTreeError)]),
    ("kv_state_accept_batch", c_int32, [c_void_p, c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_int32,
                                        POINTER(c_int64), c_void_p, POINTER(c_int32), POINTER(c_int64)]),
]
_bound = False


def _lib():
    global _bound
    lib = _capi.lib()
    if not _bound:
        for name, res, args in STATE_SIGNATURES:
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _bound = True
    return lib


def _i32(a):
    return np.ascontiguousarray(a, dtype=np.int32)


def validate_tree(tree, tokens: int | None = None) -> None:
    """tree.rs:48-73; raises TreeError."""
    t = _i32(tree)
    err = KvTreeError()
    rc = _lib().kv_tree_validate(t.ctypes.data, len(t), len(t) if tokens is None else tokens, err)
    if rc == _capi_status("KV_ERR_TREE"):
        raise TreeError(err)
    _capi.check(rc, "kv_tree_validate")


def validate_accept_path(tree, accepted) -> None:
    """tree.rs:90-123; raises TreeError."""
    t = _i32(tree)
    a = np.ascontiguousarray(accepted, dtype=np.int64)
    err = KvTreeError()
    rc = _lib().kv_tree_validate_accept(t.ctypes.data, len(t), a.ctypes.data, len(a), err)
    if rc == _capi_status("KV_ERR_TREE"):
        raise TreeError(err)
    _capi.check(rc, "kv_tree_validate_accept")


def linear_tree(n: int) -> list[int]:
    """tree.rs:41-45."""
    return [-1 if i == 0 else i - 1 for i in range(n)]


def _capi_status(name: str) -> int:
    return {v: k for k, v in _capi.STATUS.items()}[name]


@dataclass
class ForwardPlan:
    slots: np.ndarray          # storage slot of each staged token
    positions: np.ndarray      # RoPE position of each staged token
    cow: list[tuple[int, int]] = field(default_factory=list)  # (src page, dst page) to copy first
    logits: list[list[float]] = field(default_factory=list)   # the reference's dummy logits (batch.rs:215)


class KvState:
    """Allocator + block tables + speculation state for n_layers attention layers."""

    def __init__(self, n_pages: int, n_layers: int, page_tokens: int = PAGE_TOKENS, alloc_order=None):
        self.lib = _lib()
        self.n_layers = n_layers
        self.page_tokens = page_tokens
        order = None if alloc_order is None else np.ascontiguousarray(alloc_order, dtype=np.uint32)
        h = c_void_p()
        _capi.check(self.lib.kv_state_create(n_pages, n_layers, page_tokens,
                                             None if order is None else order.ctypes.data,
                                             0 if order is None else len(order), h), "kv_state_create")
        self._h = h.value
        self.n_pages = n_pages
        self._accept_cap = 1024  # token-move buffer of accept_batch, grown on demand

    def close_all(self):
        if getattr(self, "_h", None):
            self.lib.kv_state_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close_all()
        except Exception:
            pass

    # -- sessions --------------------------------------------------------------
    def open(self, seq: int) -> None:
        _capi.check(self.lib.kv_state_open(self._h, seq), "kv_state_open")

    def close(self, seq: int) -> None:
        self._engine_check(self.lib.kv_state_close(self._h, seq), seq)

    def fork(self, src: int, dst: int) -> None:
        self._engine_check(self.lib.kv_state_fork(self._h, src, dst), src)

    def append(self, seq: int, n: int, tokens=None) -> list[tuple[int, int]]:
        cs = np.empty(self.n_layers, np.uint32)
        cd = np.empty(self.n_layers, np.uint32)
        nc = c_int32(0)
        tok = None if tokens is None else np.ascontiguousarray(tokens, dtype=np.uint32)
        rc = self.lib.kv_state_append(self._h, seq, None if tok is None else tok.ctypes.data, n,
                                      cs.ctypes.data, cd.ctypes.data, self.n_layers, nc)
        self._engine_check(rc, seq)
        return list(zip(cs[: nc.value].tolist(), cd[: nc.value].tolist()))

    def forward(self, seq: int, tokens, tree=None) -> ForwardPlan:
        tok = np.ascontiguousarray(tokens, dtype=np.uint32)
        n = len(tok)
        tr = None if tree is None else _i32(tree)
        slots = np.empty(max(n, 1), np.int32)
        pos = np.empty(max(n, 1), np.int32)
        cs = np.empty(self.n_layers, np.uint32)
        cd = np.empty(self.n_layers, np.uint32)
        nc = c_int32(0)
        err = KvTreeError()
        rc = self.lib.kv_state_forward(self._h, seq, tok.ctypes.data, n, None if tr is None else tr.ctypes.data,
                                       0 if tr is None else len(tr), slots.ctypes.data, pos.ctypes.data,
                                       cs.ctypes.data, cd.ctypes.data, self.n_layers, nc, err)
        if rc == _capi_status("KV_ERR_TREE"):
            raise EngineError("Tree", seq, tree=TreeError(err))
        self._engine_check(rc, seq)
        return ForwardPlan(slots[:n].copy(), pos[:n].copy(),
                           list(zip(cs[: nc.value].tolist(), cd[: nc.value].tolist())),
                           [[float(t)] for t in tok.tolist()])

    def _commit(self, fn, seq: int, idx, with_pages: bool):
        a = np.ascontiguousarray(idx, dtype=np.int64)
        cap = max(self.pending_size(seq), 1)
        ms = np.empty(cap, np.int32)
        md = np.empty(cap, np.int32)
        nm = c_int32(0)
        tm = np.empty((cap * self.n_layers, 4), np.int32) if with_pages else None
        ntm = c_int32(0)
        bad = c_int64(0)
        rc = fn(self._h, seq, a.ctypes.data if len(a) else None, len(a), ms.ctypes.data, md.ctypes.data, cap,
                nm, None if tm is None else tm.ctypes.data, 0 if tm is None else tm.shape[0], ntm, bad)
        if rc == _capi_status("KV_ERR_INVALID_ACCEPT"):
            raise EngineError("InvalidAccept", seq, index=int(bad.value))
        self._engine_check(rc, seq)
        moves = list(zip(ms[: nm.value].tolist(), md[: nm.value].tolist()))
        if with_pages:
            return moves, tm[: ntm.value].copy()
        return moves

    def accept(self, seq: int, accepted, with_pages: bool = False):
        """Commit a path; returns slot moves (and, with_pages, the per-layer
        page-addressed token moves [n, 4] to run with KvPool.move_tokens)."""
        return self._commit(self.lib.kv_state_accept, seq, accepted, with_pages)

    def rollback(self, seq: int, rejected, with_pages: bool = False):
        return self._commit(self.lib.kv_state_rollback, seq, rejected, with_pages)

    def forward_batch(self, seqs, tokens, trees, stride: int, masks: bool = True) -> dict:
        """forward() for every sequence in one native call (kv_state_forward_batch):
        tokens[i] / trees[i] (trees None: chains) of sequence seqs[i]; drafts of
        one length may come as [n_seqs, T] arrays.  Returns the flat launch
        arrays: tok_row, slots, positions, q_offsets, prefix, masks (int64 view;
        None unless masks), cow_src, cow_dst and tables [n_layers, n_seqs,
        stride].  A failing sequence raises like forward() with the sequences
        before it staged."""
        n = len(seqs)
        ids = np.ascontiguousarray(seqs, dtype=np.uint64)
        if isinstance(tokens, np.ndarray) and tokens.ndim == 2:
            if tokens.shape[0] != n:
                raise ValueError("tokens must have one row per sequence")
            off = np.arange(0, n * tokens.shape[1] + 1, tokens.shape[1], dtype=np.int32)
            tok = np.ascontiguousarray(tokens.reshape(-1) if tokens.size else np.zeros(1), dtype=np.uint32)
        else:
            lens = np.fromiter((len(t) for t in tokens), np.int64, n)
            off = np.zeros(n + 1, np.int32)
            np.cumsum(lens, out=off[1:])
            tok = np.ascontiguousarray(np.concatenate([np.asarray(t, np.uint32) for t in tokens]) if off[-1]
                                       else np.zeros(1, np.uint32), dtype=np.uint32)
        total = int(off[-1])
        tr = None
        if trees is not None:
            if isinstance(trees, np.ndarray) and trees.ndim == 2:
                if trees.shape[0] != n or trees.shape[1] != off[1] - off[0] or total != trees.size:
                    raise ValueError("trees must be [n_seqs, T] like tokens")
                tr = _i32(trees.reshape(-1) if total else np.zeros(1, np.int32))
            else:
                tr = _i32(np.concatenate([np.asarray(t, np.int32) for t in trees]) if total
                          else np.zeros(1, np.int32))
            if len(tr) < total:
                raise ValueError("every sequence needs a tree of its token count")
        k = max(total, 1)
        tok_row, slots, pos = np.empty(k, np.int32), np.empty(k, np.int32), np.empty(k, np.int32)
        prefix = np.empty(max(n, 1), np.int32)
        mk = np.empty(k, np.uint64) if masks else None
        cap = max(self.n_layers * n, 1)
        cs, cd = np.empty(cap, np.uint32), np.empty(cap, np.uint32)
        tables = np.empty((self.n_layers, max(n, 1), stride), np.uint32)
        nc, done, err = c_int32(0), c_int32(0), KvTreeError()
        rc = self.lib.kv_state_forward_batch(self._h, ids.ctypes.data, n, tok.ctypes.data, off.ctypes.data,
                                             None if tr is None else tr.ctypes.data, tok_row.ctypes.data,
                                             slots.ctypes.data, pos.ctypes.data, prefix.ctypes.data,
                                             None if mk is None else mk.ctypes.data, cs.ctypes.data,
                                             cd.ctypes.data, cap, nc, tables.ctypes.data, stride, done, err)
        if rc == _capi_status("KV_ERR_TREE"):
            raise EngineError("Tree", int(seqs[done.value]), tree=TreeError(err))
        self._engine_check(rc, int(seqs[done.value]) if done.value < n else -1)
        return {"tok_row": tok_row[:total], "slots": slots[:total], "positions": pos[:total], "q_offsets": off,
                "prefix": prefix[:n], "masks": None if mk is None else mk[:total].view(np.int64),
                "cow_src": cs[:nc.value], "cow_dst": cd[:nc.value], "tables": tables[:, :n]}

    def accept_batch(self, seqs, paths):
        """accept() for every sequence in one native call (kv_state_accept_batch).
        paths: one accepted path per sequence, or (flat int64 array, offsets
        [n_seqs + 1]).  Returns (token moves [n, 4] int32, group offsets
        [n_seqs * n_layers + 1]): one group per (sequence, layer), as
        KvPool.move_tokens takes them."""
        n = len(seqs)
        ids = np.ascontiguousarray(seqs, dtype=np.uint64)
        if isinstance(paths, tuple) and len(paths) == 2 and isinstance(paths[0], np.ndarray):
            off = np.ascontiguousarray(paths[1], dtype=np.int32)
            if len(off) != n + 1 or off[0] != 0:
                raise ValueError("path offsets must have n_seqs + 1 entries starting at 0")
            pa = np.ascontiguousarray(paths[0] if off[-1] else np.zeros(1), dtype=np.int64)
        else:
            off = np.zeros(n + 1, np.int32)
            np.cumsum([len(p) for p in paths], out=off[1:])
            pa = np.ascontiguousarray(np.concatenate([np.asarray(p, np.int64) for p in paths]) if off[-1]
                                      else np.zeros(1, np.int64), dtype=np.int64)
        groups = np.empty(n * self.n_layers + 1, np.int32)
        groups[0] = 0
        done, bad, need = c_int32(0), c_int64(0), c_int64(0)
        cap = max(self._accept_cap, 1)
        for _ in range(2):  # a second try when the staged drafts outgrew the last size
            tm = np.empty((cap, 4), np.int32)
            rc = self.lib.kv_state_accept_batch(self._h, ids.ctypes.data, n, pa.ctypes.data, off.ctypes.data,
                                                tm.ctypes.data, cap, need, groups.ctypes.data, done, bad)
            if need.value <= cap:
                break
            cap = self._accept_cap = int(need.value)
        if rc == _capi_status("KV_ERR_INVALID_ACCEPT"):
            raise EngineError("InvalidAccept", int(seqs[done.value]), index=int(bad.value))
        self._engine_check(rc, int(seqs[done.value]) if done.value < n else -1)
        return tm[:groups[-1]], groups

    def evict_window(self, seq: int, window: int) -> int:
        n = c_int64(0)
        self._engine_check(self.lib.kv_state_evict_window(self._h, seq, window, n), seq)
        return int(n.value)

    def compact(self) -> list[tuple[int, int]]:
        n = c_int32(0)
        rc = self.lib.kv_state_compact(self._h, None, None, 0, n)
        if rc == 0:
            return []
        src = np.empty(n.value, np.uint32)
        dst = np.empty(n.value, np.uint32)
        _capi.check(self.lib.kv_state_compact(self._h, src.ctypes.data, dst.ctypes.data, n.value, n), "compact")
        return list(zip(src.tolist(), dst.tolist()))

    # -- queries ---------------------------------------------------------------
    def token_count(self, seq: int) -> int:
        n = c_int64(0)
        self._engine_check(self.lib.kv_state_token_count(self._h, seq, n), seq)
        return int(n.value)

    def allocated_blocks(self, seq: int) -> int:
        """PagedKv::allocated_blocks = blocks_for(token_count) (cache.rs:36-50)."""
        return -(-self.token_count(seq) // self.page_tokens)

    def committed(self, seq: int) -> list[int]:
        n = c_int64(0)
        rc = self.lib.kv_state_committed(self._h, seq, None, 0, n)
        if rc == _capi_status("KV_ERR_UNKNOWN_SEQ"):
            raise EngineError("UnknownSeq", seq)
        out = np.empty(max(n.value, 1), np.uint32)
        _capi.check(self.lib.kv_state_committed(self._h, seq, out.ctypes.data, len(out), n), "committed")
        return out[: n.value].tolist()

    def table(self, seq: int, layer: int, draft: bool = False) -> list[int]:
        n = c_int64(0)
        rc = self.lib.kv_state_table(self._h, seq, layer, int(draft), None, 0, n)
        if rc not in (0, 1):
            self._engine_check(rc, seq)
        out = np.empty(max(n.value, 1), np.uint32)
        _capi.check(self.lib.kv_state_table(self._h, seq, layer, int(draft), out.ctypes.data, len(out), n), "table")
        return out[: n.value].tolist()

    def export_tables(self, seqs, layer: int, stride: int, draft: bool = False) -> np.ndarray:
        ids = np.ascontiguousarray(seqs, dtype=np.uint64)
        out = np.empty((len(ids), stride), np.uint32)
        self._engine_check(self.lib.kv_state_export_tables(self._h, ids.ctypes.data, len(ids), layer, int(draft),
                                                           out.ctypes.data, stride), -1)
        return out

    def free_list(self) -> list[int]:
        n = c_int64(0)
        self.lib.kv_state_free_list(self._h, None, 0, n)
        out = np.empty(max(n.value, 1), np.uint32)
        _capi.check(self.lib.kv_state_free_list(self._h, out.ctypes.data, len(out), n), "free_list")
        return out[: n.value].tolist()

    def refcount(self, page: int) -> int:
        c = c_uint32(0)
        _capi.check(self.lib.kv_state_refcount(self._h, page, c), "refcount")
        return int(c.value)

    def pending_base(self, seq: int) -> int:
        b = c_int64(0)
        self._engine_check(self.lib.kv_state_pending_base(self._h, seq, b), seq)
        return int(b.value)

    def pending_size(self, seq: int) -> int:
        try:
            self.pending_base(seq)
        except EngineError:
            return 0
        return len(self.table(seq, 0, draft=True)) * self.page_tokens  # an upper bound

    # -- errors ----------------------------------------------------------------
    def _engine_check(self, rc: int, seq: int) -> None:
        if rc == 0:
            return
        name = _capi.STATUS.get(rc)
        if name == "KV_ERR_UNKNOWN_SEQ":
            raise EngineError("UnknownSeq", seq)
        if name == "KV_ERR_NO_PENDING":
            raise EngineError("NoPendingForward", seq)
        _capi.check(rc)
