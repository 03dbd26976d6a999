"""The path's host-side callers over the C ABI: speculative draft trees and the
continuous-batching scheduler (kv_draft_tree_best_first, kv_sched_*).

The reference has both as placeholders: a DraftModel hook returning a token
list and a parent-index tree (crates/llm-engine/src/draft.rs:9-23) and a
Scheduler of running sequence ids packed into a ForwardBatch
(crates/llm-engine/src/schedule.rs:8-48).  The native versions keep those
semantics and add what the kernels need: the tree picked best first by
cumulative draft probability within a node and depth budget, a per-step
planner under a token budget (decode tokens first, then prompt chunks), and
LPT assignment of sessions to GPUs.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_double, c_int32, c_int64, c_uint32, c_uint64, c_void_p

import numpy as np

from . import _capi

SCHED_SIGNATURES = [
    ("kv_draft_tree_best_first", c_int32,
     [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p, POINTER(c_int32)]),
    ("kv_sched_create", c_int32, [POINTER(c_void_p)]),
    ("kv_sched_destroy", c_int32, [c_void_p]),
    ("kv_sched_add", c_int32, [c_void_p, c_uint64]),
    ("kv_sched_remove", c_int32, [c_void_p, c_uint64]),
    ("kv_sched_running", c_int32, [c_void_p, c_void_p, c_int64, POINTER(c_int64)]),
    ("kv_sched_set_pending", c_int32, [c_void_p, c_uint64, c_int64]),
    ("kv_sched_plan_step", c_int32,
     [c_void_p, c_int64, c_int32, c_void_p, c_void_p, c_void_p, c_int32, POINTER(c_int32)]),
    ("kv_sched_lpt", c_int32, [c_void_p, c_int32, c_int32, c_void_p]),
]
_bound = False


def _lib():
    global _bound
    lib = _capi.lib()
    if not _bound:
        for name, res, args in SCHED_SIGNATURES:
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _bound = True
    return lib


def draft_tree_best_first(parents, tokens, probs, max_nodes: int, max_depth: int):
    """The speculative tree from a draft model's candidates (candidate c: parent
    index or -1, token, probability given the parent; parents first).
    Returns (tokens, tree, picked): the DraftProposal form (draft.rs:14-17)
    with tree parents as output indices, and the candidate index of each node."""
    par = np.ascontiguousarray(parents, np.int32)
    tok = np.ascontiguousarray(tokens, np.uint32)
    pr = np.ascontiguousarray(probs, np.float64)
    n = len(par)
    if len(tok) != n or len(pr) != n:
        raise ValueError("parents, tokens and probs must have one entry per candidate")
    cap = max(max_nodes, 1)
    out_tok = np.empty(cap, np.uint32)
    out_tree = np.empty(cap, np.int32)
    picked = np.empty(cap, np.int32)
    m = c_int32(0)
    _capi.check(_lib().kv_draft_tree_best_first(par.ctypes.data, tok.ctypes.data, pr.ctypes.data, n, max_nodes,
                                                 max_depth, out_tok.ctypes.data, out_tree.ctypes.data,
                                                 picked.ctypes.data, ctypes.byref(m)), "kv_draft_tree_best_first")
    k = m.value
    return out_tok[:k].copy(), out_tree[:k].copy(), picked[:k].copy()


def lpt(weights, bins: int) -> np.ndarray:
    """LPT assignment (kv_sched_lpt): bin index of every item."""
    w = np.ascontiguousarray(weights, np.int64)
    out = np.empty(len(w), np.int32)
    _capi.check(_lib().kv_sched_lpt(w.ctypes.data, len(w), bins, out.ctypes.data), "kv_sched_lpt")
    return out


class Scheduler:
    """Running sequences in insertion order (schedule.rs:8-48) plus prompt
    tokens still to prefill and a per-step planner under a token budget."""

    def __init__(self):
        self.lib = _lib()
        h = c_void_p()
        _capi.check(self.lib.kv_sched_create(ctypes.byref(h)), "kv_sched_create")
        self._h = h.value

    def close(self):
        if getattr(self, "_h", None):
            self.lib.kv_sched_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def add(self, seq_id: int) -> None:
        _capi.check(self.lib.kv_sched_add(self._h, seq_id), "kv_sched_add")

    def remove(self, seq_id: int) -> None:
        _capi.check(self.lib.kv_sched_remove(self._h, seq_id), "kv_sched_remove")

    def running(self) -> list[int]:
        n = c_int64(0)
        self.lib.kv_sched_running(self._h, None, 0, ctypes.byref(n))
        out = np.empty(max(n.value, 1), np.uint64)
        _capi.check(self.lib.kv_sched_running(self._h, out.ctypes.data, len(out), ctypes.byref(n)), "kv_sched_running")
        return out[:n.value].tolist()

    def schedule(self) -> list[int]:
        """The batch schedule.rs:41-47 builds: one entry per running sequence, in order."""
        return self.running()

    def set_pending(self, seq_id: int, prefill_tokens: int) -> None:
        _capi.check(self.lib.kv_sched_set_pending(self._h, seq_id, prefill_tokens), "kv_sched_set_pending")

    def plan_step(self, token_budget: int, chunk_tokens: int):
        """[(seq_id, n_tokens, is_prefill)] of one step (kv_sched_plan_step)."""
        cap = max(len(self.running()), 1)
        ids = np.empty(cap, np.uint64)
        nt = np.empty(cap, np.int32)
        pf = np.empty(cap, np.int32)
        n = c_int32(0)
        _capi.check(self.lib.kv_sched_plan_step(self._h, token_budget, chunk_tokens, ids.ctypes.data, nt.ctypes.data,
                                                pf.ctypes.data, cap, ctypes.byref(n)), "kv_sched_plan_step")
        return [(int(ids[i]), int(nt[i]), bool(pf[i])) for i in range(n.value)]
