"""Device command plans for engine-level KV operations on a batch of sessions.

The reference's engine (crates/llm-engine/src/batch.rs:173-296) walks its
sessions one by one: `forward` stages draft tokens, `accept` / `rollback`
commit a path, and `PagedKv` only counts tokens (cache.rs:20-51).  Here the
host state (`KvState`, C++) decides where every token lives; this module turns
its per-session answers into the flat arrays one kernel launch per layer
consumes:

  ForwardBatch   a speculative round's staging for all sessions: copy-on-write
                 page copies, draft block tables, token slots and RoPE
                 positions, ancestor-or-self masks, the committed prefix of
                 each session (the cached keys every draft token sees)
  commit_moves   the accepted paths' token moves, grouped per (session, layer)
  DecodeStep     one decode token for every session under a sliding window:
                 the new pages to publish in the device block tables, pages
                 evicted below the window, and (every `compact_every` steps)
                 the compaction page moves

No device memory is touched here; callers copy the arrays and launch.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .state import KvState

PAGE_NONE = 0xFFFFFFFF


def tree_masks(parents) -> np.ndarray:
    """Ancestor-or-self bit masks (bit j of mask i: node j is i or an ancestor),
    int64 view of uint64; at most 64 nodes, parents[i] < i."""
    n = len(parents)
    if n > 64:
        raise ValueError("tree-verify chunks hold at most 64 tokens")
    m = np.zeros(n, np.uint64)
    for i, p in enumerate(parents):
        if not (-1 <= p < i):
            raise ValueError(f"parent {p} of node {i} does not precede it")
        m[i] = (m[p] if p >= 0 else np.uint64(0)) | np.uint64(1 << i)
    return m.view(np.int64)


@dataclass
class ForwardBatch:
    seqs: list
    cow_src: np.ndarray          # uint32 [n_cow]
    cow_dst: np.ndarray
    tok_seq: np.ndarray          # int32 [n_tok]: row of the batch (block-table row)
    slots: np.ndarray            # int32 [n_tok]
    positions: np.ndarray        # int32 [n_tok]
    q_offsets: np.ndarray        # int32 [n_seqs + 1]
    prefix: np.ndarray           # int32 [n_seqs]: committed tokens before the draft
    masks: np.ndarray            # int64 [n_tok]
    tables: np.ndarray           # uint32 [n_layers, n_seqs, stride]: draft tables
    max_q: int = 0

    @property
    def n_tokens(self) -> int:
        return len(self.slots)


def plan_forward(st: KvState, seqs, tokens, parents, stride: int) -> ForwardBatch:
    """KvState.forward for every session (tokens[i], parents[i]), flattened;
    one native call (kv_state_forward_batch).  Drafts of one length may come
    as [n, T] arrays."""
    f = st.forward_batch(seqs, tokens, parents, stride)
    qoff = f["q_offsets"]
    return ForwardBatch(list(seqs), f["cow_src"], f["cow_dst"], f["tok_row"], f["slots"], f["positions"], qoff,
                        f["prefix"], f["masks"], f["tables"], int(np.diff(qoff).max()) if len(seqs) else 0)


def commit_moves(st: KvState, seqs, paths):
    """KvState.accept for every session; the page-addressed token moves of all
    sessions and layers, one group per (session, layer), group offsets and the
    number of accepted tokens (one native call, kv_state_accept_batch).  paths:
    one accepted path per session, or (flat int64 array, offsets [n + 1])."""
    mv, offs = st.accept_batch(seqs, paths)
    accepted = int(paths[1][-1]) if isinstance(paths, tuple) else sum(len(p) for p in paths)
    return mv, offs, accepted


@dataclass
class DecodeStep:
    """What one windowed decode step changed in the block tables."""
    new_pages: list = field(default_factory=list)   # (layer, row, index, page)
    evicted: int = 0
    compaction: list = field(default_factory=list)  # (src page, dst page)


def plan_decode_step(st: KvState, seqs, window: int, compact: bool) -> DecodeStep:
    """Append one token to every session (a new page when it starts one),
    free the pages wholly below the window, and optionally compact the pool.
    After a compaction every table may have changed: re-export them all."""
    out = DecodeStep()
    for row, s in enumerate(seqs):
        cow = st.append(s, 1)
        if cow:
            raise RuntimeError("a windowed decode session shares no pages")
        n = st.token_count(s)
        if (n - 1) % st.page_tokens == 0:  # the token opened a page
            idx = (n - 1) // st.page_tokens
            for layer in range(st.n_layers):
                out.new_pages.append((layer, row, idx, st.table(s, layer)[idx]))
        if window:
            out.evicted += st.evict_window(s, window)
    if compact:
        out.compaction = st.compact()
    return out
