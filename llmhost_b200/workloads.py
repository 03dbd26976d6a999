"""Seeded synthetic workloads with the shapes of the benchmark configurations.

The reference publishes no dataset for this path; inputs are N(0,1) draws from
numpy's PCG64 (`default_rng(seed)`), rounded to bf16 (nearest even) for the bf16
configurations, and page ids come from a seeded permutation of the pool.

Decode configuration ("bf16 batched decode"): 64 sessions with cached lengths
uniform in [128, 8192], page size 16, physical pages consumed in order from a
seeded permutation of a 2^20-page pool, 24 query / 8 KV heads, head_dim 64,
6 attention layers, one append plus one paged attention per layer per step.
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
                  n_layers: int = 6, window: int = 0) -> DecodeWorkload:
    """The batched-decode configuration (defaults) or a scaled variant of it."""
    rng = np.random.default_rng(seed)
    l0 = rng.integers(lo, hi, endpoint=True, size=n_seqs).astype(np.int64)
    order = rng.permutation(pool_pages).astype(np.uint32)
    bt = allocate_in_order(l0, steps, n_layers, order)
    return DecodeWorkload("bf16 batched decode" if dtype == "bf16" else "f32 batched decode",
                          dtype, n_q, n_kv, 64, n_layers, l0, steps, pool_pages, bt, window)


def normal_bits(rng: np.random.Generator, shape, dtype: str) -> np.ndarray:
    """N(0,1) fp32 draws; bf16 as uint16 bits (round to nearest even)."""
    x = rng.standard_normal(shape, dtype=np.float32)
    if dtype == "f32":
        return x
    u = x.view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
