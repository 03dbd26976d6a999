"""Seeded synthetic workloads with the shapes of the benchmark configurations.

The reference publishes no dataset for this path; inputs are N(0,1) draws from
numpy's PCG64 (`default_rng(seed)`), rounded to bf16 (nearest even) for the bf16
configurations, and page ids come from a seeded permutation of the pool.

Decode configuration ("bf16 batched decode"): 64 sessions with cached lengths
uniform in [128, 8192], page size 16, physical pages consumed in order from a
seeded permutation of a 2^20-page pool, 24 query / 8 KV heads, head_dim 64,
6 attention layers, one append plus one paged attention per layer per step.

The other configurations (one generator each below): an fp32 single session
(prefill 2048, then 256 decode steps), bf16 chunked prefill (16 sessions x 32
chunks of 512 tokens), a speculative tree step (32 sessions sharing a
4096-token prefix, 64-node trees of depth <= 6), and long context with a
sliding window (256 sessions, log-uniform lengths, LPT-partitioned over GPUs).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

PAGE_TOKENS = 16


def ceil_div(a, b):
    return -(-np.asarray(a) // b)


@dataclass
class DecodeWorkload:
    name: str
    dtype: str           # "bf16" or "f32"
    n_q: int
    n_kv: int
    head_dim: int
    n_layers: int
    l0: np.ndarray        # [n_seqs] tokens cached before step 0
    steps: int
    pool_pages: int
    block_tables: np.ndarray  # [n_layers, n_seqs, max_pages] uint32, pages for l0 + steps tokens
    window: int = 0
    rope_theta: float = 1e6

    @property
    def n_seqs(self) -> int:
        return len(self.l0)

    def seq_lens(self, step: int) -> np.ndarray:
        """Tokens per sequence after step `step`'s append (the attended length)."""
        return (self.l0 + step + 1).astype(np.int32)

    @property
    def elem_bytes(self) -> int:
        return 2 if self.dtype == "bf16" else 4

    def step_bytes(self, step: int) -> int:
        """Algorithmic HBM bytes of one decode step (all layers): cached K/V
        read, new k/v read, append write, q read, out write, block-table read."""
        e, d, nkv, nq = self.elem_bytes, self.head_dim, self.n_kv, self.n_q
        n = self.seq_lens(step).astype(np.int64)
        lo = np.maximum(n - self.window, 0) if self.window else np.zeros_like(n)
        cached = n - 1 - lo
        per_layer = (2 * nkv * d * e * cached + 2 * nkv * d * e * 2 + 2 * nq * d * e
                     + 4 * (ceil_div(n, PAGE_TOKENS) - lo // PAGE_TOKENS))
        return int(per_layer.sum()) * self.n_layers

    def attn_bytes(self, step: int) -> int:
        """Algorithmic bytes of one decode-attention launch (one layer): the
        attended K/V, q, out and block-table entries."""
        e, d, nkv, nq = self.elem_bytes, self.head_dim, self.n_kv, self.n_q
        n = self.seq_lens(step).astype(np.int64)
        lo = np.maximum(n - self.window, 0) if self.window else np.zeros_like(n)
        pages = ceil_div(n, PAGE_TOKENS) - lo // PAGE_TOKENS
        return int((2 * nkv * d * e * (n - lo) + 2 * nq * d * e + 4 * pages).sum())


def allocate_in_order(l0: np.ndarray, steps: int, n_layers: int, order: np.ndarray) -> np.ndarray:
    """Block tables when pages are taken in order from `order`: first the
    cached tokens (layer-major, then session), then one page whenever a
    decode step starts a new page (step, layer, session order)."""
    n = len(l0)
    final = l0 + steps
    max_pages = int(ceil_div(final.max(), PAGE_TOKENS))
    bt = np.full((n_layers, n, max_pages), 0xFFFFFFFF, dtype=np.uint32)
    cur = 0
    first = ceil_div(l0, PAGE_TOKENS)
    for layer in range(n_layers):
        for s in range(n):
            k = int(first[s])
            bt[layer, s, :k] = order[cur:cur + k]
            cur += k
    have = first.copy()
    for step in range(steps):
        pos = l0 + step  # position of this step's token
        need = pos // PAGE_TOKENS + 1
        grow = np.nonzero(need > have)[0]
        if len(grow) == 0:
            continue
        for layer in range(n_layers):
            for s in grow:
                bt[layer, s, have[s]] = order[cur]
                cur += 1
        have[grow] += 1
    return bt


def decode_config(steps: int = 512, seed: int = 1, n_seqs: int = 64, pool_pages: int = 1 << 20,
                  lo: int = 128, hi: int = 8192, dtype: str = "bf16", n_q: int = 24, n_kv: int = 8,
                  n_layers: int = 6, window: int = 0, world: int = 1, rank: int = 0) -> DecodeWorkload:
    """The batched-decode configuration (defaults) or a scaled variant of it.

    With world > 1 the job is n_seqs * world sessions: the configuration's
    n_seqs lengths once per GPU, split into world shares by LPT on cached
    length (the bytes a step reads).  LPT hands each share one session of
    every length, so each GPU's work is the configuration's exactly, at every
    world size (weak scaling with fixed work per GPU); this returns share
    `rank`.  Every share draws its pages from the same permutation of its own
    pool."""
    rng = np.random.default_rng(seed)
    lengths = rng.integers(lo, hi, endpoint=True, size=n_seqs).astype(np.int64)
    if world > 1:
        job = np.tile(lengths, world)
        l0 = job[lpt_partition(job.tolist(), world)[rank]]
    else:
        l0 = lengths
    order = rng.permutation(pool_pages).astype(np.uint32)
    bt = allocate_in_order(l0, steps, n_layers, order)
    return DecodeWorkload("bf16 batched decode" if dtype == "bf16" else "f32 batched decode",
                          dtype, n_q, n_kv, 64, n_layers, l0, steps, pool_pages, bt, window)


def normal_bits(rng: np.random.Generator, shape, dtype: str) -> np.ndarray:
    """N(0,1) fp32 draws; bf16 as uint16 bits (round to nearest even)."""
    x = rng.standard_normal(shape, dtype=np.float32)
    if dtype == "f32":
        return x
    # finite draws stay below 0xFF800000, so the 32-bit sum cannot wrap
    u = x.view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)


# ---- fp32 single session --------------------------------------------------------------
@dataclass
class SingleSessionWorkload:
    """One fp32 session: prefill `prefill` tokens, then `steps` decode steps.
    Block table of layer l is contiguous: page l * pages_per_layer + i."""
    name: str = "fp32 single session"
    dtype: str = "f32"
    n_q: int = 24
    n_kv: int = 8
    n_layers: int = 6
    prefill: int = 2048
    steps: int = 256
    rope_theta: float = 1e6

    @property
    def pages_per_layer(self) -> int:
        return int(ceil_div(self.prefill + self.steps, PAGE_TOKENS))

    @property
    def pool_pages(self) -> int:
        return self.n_layers * self.pages_per_layer

    def block_table(self, layer: int) -> np.ndarray:
        n = self.pages_per_layer
        return (layer * n + np.arange(n)).astype(np.uint32)

    def prefill_flops(self) -> float:
        """4 d per visible (query row, key) pair, causal, all layers."""
        t = self.prefill
        return 4.0 * 64 * self.n_q * (t * (t + 1) / 2) * self.n_layers


# ---- bf16 chunked prefill ---------------------------------------------------------------
@dataclass
class ChunkedPrefillWorkload:
    """Sessions append `chunk`-token chunks up to `total` tokens; chunk c of
    every session sees the c * chunk cached tokens plus a causal chunk."""
    name: str
    n_seqs: int
    chunk: int
    total: int
    n_q: int
    n_kv: int
    n_layers: int
    pool_pages: int
    block_tables: np.ndarray  # [n_layers, n_seqs, total / 16] uint32
    dtype: str = "bf16"
    rope_theta: float = 1e6

    @property
    def n_chunks(self) -> int:
        return self.total // self.chunk

    def chunk_flops(self, c: int) -> float:
        """Algorithmic FLOPs of chunk c for one layer and all sessions: 4 d per
        visible (query row, key) pair."""
        C = self.chunk
        pairs = C * (C * c) + C * (C + 1) / 2
        return 4.0 * 64 * self.n_q * pairs * self.n_seqs

    def total_flops(self) -> float:
        return sum(self.chunk_flops(c) for c in range(self.n_chunks)) * self.n_layers


def chunked_prefill_config(seed: int = 3, n_seqs: int = 16, chunk: int = 512, total: int = 16384,
                           n_q: int = 32, n_kv: int = 8, n_layers: int = 6,
                           pool_pages: int = 1 << 17) -> ChunkedPrefillWorkload:
    rng = np.random.default_rng(seed)
    order = rng.permutation(pool_pages).astype(np.uint32)
    per = total // PAGE_TOKENS
    need = n_layers * n_seqs * per
    if need > pool_pages:
        raise ValueError("pool too small for the chunked-prefill workload")
    bt = order[:need].reshape(n_layers, n_seqs, per)
    return ChunkedPrefillWorkload("bf16 chunked prefill", n_seqs, chunk, total, n_q, n_kv, n_layers,
                                  pool_pages, bt)


# ---- speculative tree --------------------------------------------------------------------
def draft_tree(rng: np.random.Generator, nodes: int = 64, depth: int = 6, fanout: int = 4):
    """A candidate tree built best-first by cumulative probability: every
    expanded node offers `fanout` children with Dirichlet(1) probabilities;
    the most probable open candidate is added next, until `nodes` nodes, no
    node deeper than `depth` (root at depth 0).  Returns (parents, children)
    where children[u] is the list of (probability, node index or -1 when the
    candidate was not added)."""
    import heapq

    parents = [-1]
    depth_of = [0]
    children: list[list[list]] = [[]]
    heap = []  # (-cumulative probability, tiebreak, parent, slot)
    tie = 0

    def expand(u, cum):
        nonlocal tie
        if depth_of[u] >= depth:
            return
        probs = rng.dirichlet(np.ones(fanout))
        for slot, p in enumerate(probs):
            children[u].append([float(p), -1])
            heapq.heappush(heap, (-cum * float(p), tie, u, slot))
            tie += 1

    expand(0, 1.0)
    while len(parents) < nodes and heap:
        negcum, _, u, slot = heapq.heappop(heap)
        v = len(parents)
        parents.append(u)
        depth_of.append(depth_of[u] + 1)
        children.append([])
        children[u][slot][1] = v
        expand(v, -negcum)
    return parents, children


def accept_path(rng: np.random.Generator, children) -> list[int]:
    """Walk from the root, sampling a child by its probability; stop at a
    candidate that is not in the tree.  The root is always accepted."""
    path = [0]
    u = 0
    while children[u]:
        probs = np.array([c[0] for c in children[u]])
        pick = int(rng.choice(len(probs), p=probs / probs.sum()))
        v = children[u][pick][1]
        if v < 0:
            break
        path.append(v)
        u = v
    return path


@dataclass
class SpecTreeWorkload:
    name: str = "bf16 speculative tree"
    n_seqs: int = 32
    prefix: int = 4096
    nodes: int = 64
    depth: int = 6
    steps: int = 64
    n_q: int = 24
    n_kv: int = 8
    n_layers: int = 6
    dtype: str = "bf16"
    pool_pages: int = 1 << 16
    seed: int = 4
    rope_theta: float = 1e6

    def plan(self):
        """Per step and session: (parents, accepted indices)."""
        rng = np.random.default_rng(self.seed)
        out = []
        for _ in range(self.steps):
            row = []
            for _ in range(self.n_seqs):
                parents, children = draft_tree(rng, self.nodes, self.depth)
                row.append((parents, accept_path(rng, children)))
            out.append(row)
        return out


# ---- long context with a sliding window ---------------------------------------------------
def lpt_partition(weights, bins: int) -> list[list[int]]:
    """Longest-processing-time-first: items in decreasing weight, each to the
    currently lightest bin (ties to the lowest bin index).  Deterministic."""
    order = sorted(range(len(weights)), key=lambda i: (-weights[i], i))
    load = [0] * bins
    out: list[list[int]] = [[] for _ in range(bins)]
    for i in order:
        b = min(range(bins), key=lambda k: (load[k], k))
        out[b].append(i)
        load[b] += weights[i]
    return [sorted(x) for x in out]


@dataclass
class LongContextWorkload:
    name: str
    lengths: np.ndarray      # [n_total] tokens cached before step 0, all sessions
    shard: list              # session indices of this GPU's share
    window: int
    steps: int
    compact_every: int
    n_q: int
    n_kv: int
    n_layers: int
    dtype: str = "bf16"
    rope_theta: float = 1e6
    long_session: int = 1 << 20

    @property
    def l0(self) -> np.ndarray:
        return self.lengths[self.shard]


def long_context_config(rank: int = 0, bins: int = 8, seed: int = 5, n_total: int = 256,
                        lo: int = 1024, hi: int = 131072, window: int = 32768, steps: int = 256,
                        compact_every: int = 64, n_q: int = 32, n_kv: int = 8,
                        n_layers: int = 6) -> LongContextWorkload:
    """256 sessions with lengths log-uniform in [lo, hi]; GPU `rank` of `bins`
    takes the LPT share by resident length min(L, window)."""
    rng = np.random.default_rng(seed)
    lengths = np.exp(rng.uniform(np.log(lo), np.log(hi), size=n_total)).astype(np.int64)
    resident = np.minimum(lengths, window)
    parts = lpt_partition(resident.tolist(), bins)
    return LongContextWorkload("bf16 long context, sliding window", lengths, parts[rank % bins], window, steps,
                               compact_every, n_q, n_kv, n_layers)

