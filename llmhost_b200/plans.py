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
    """KvState.forward for every session (tokens[i], parents[i]), flattened."""
    cs, cd, tseq, slots, pos, qoff, prefix, masks = [], [], [], [], [], [0], [], []
    for row, s in enumerate(seqs):
        plan = st.forward(s, tokens[row], parents[row])
        for a, b in plan.cow:
            cs.append(a)
            cd.append(b)
        n = len(plan.slots)
        tseq.append(np.full(n, row, np.int32))
        slots.append(plan.slots.astype(np.int32))
        pos.append(plan.positions.astype(np.int32))
        qoff.append(qoff[-1] + n)
        prefix.append(st.pending_base(s))
        masks.append(tree_masks(parents[row]))
    tables = np.stack([st.export_tables(seqs, layer, stride, draft=True) for layer in range(st.n_layers)])
    return ForwardBatch(list(seqs), np.asarray(cs, np.uint32), np.asarray(cd, np.uint32),
                        np.concatenate(tseq), np.concatenate(slots), np.concatenate(pos),
                        np.asarray(qoff, np.int32), np.asarray(prefix, np.int32), np.concatenate(masks), tables,
                        max(np.diff(qoff)) if len(seqs) else 0)


def commit_moves(st: KvState, seqs, paths):
    """KvState.accept for every session; the page-addressed token moves of all
    sessions and layers, one group per (session, layer), and group offsets."""
    moves, offs = [], [0]
    accepted = 0
    for s, path in zip(seqs, paths):
        _, tm = st.accept(s, path, with_pages=True)
        accepted += len(path)
        per = len(tm) // st.n_layers
        for layer in range(st.n_layers):
            part = tm[layer * per:(layer + 1) * per]
            moves.append(part)
            offs.append(offs[-1] + len(part))
    mv = np.concatenate(moves).astype(np.int32) if moves else np.zeros((0, 4), np.int32)
    return mv.reshape(-1, 4), np.asarray(offs, np.int32), accepted


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
