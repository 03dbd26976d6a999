"""KV-head sharding of one long session over GPUs.

A session too long for one GPU's HBM (the 1M-token session: 256 MiB of K+V
per layer per KV head in bf16) is split by KV head: GPU r of W holds KV heads
[r n_kv / W, (r + 1) n_kv / W) and the query heads that read them (GQA group
g = n_q / n_kv), runs split-K decode attention over all of the session's pages
for its heads, and the per-head outputs are all-gathered (one collective per
step for all layers).  Heads are independent, so the gathered result equals
the unsharded computation exactly.

The reference has one contiguous KV buffer per layer and no multi-GPU path
(crates/llm-engine/src/lfm2.rs:188-203); this is build-defined.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class HeadShard:
    rank: int
    world: int
    kv_begin: int
    kv_end: int
    q_begin: int
    q_end: int

    @property
    def n_kv(self) -> int:
        return self.kv_end - self.kv_begin

    @property
    def n_q(self) -> int:
        return self.q_end - self.q_begin


def head_shard(rank: int, world: int, n_kv: int, n_q: int) -> HeadShard:
    """Contiguous KV-head ranges, equal per rank (world must divide n_kv)."""
    if world <= 0 or n_kv % world or n_q % n_kv:
        raise ValueError(f"cannot split {n_kv} KV heads / {n_q} q heads over {world} ranks")
    per = n_kv // world
    g = n_q // n_kv
    kb = rank * per
    return HeadShard(rank, world, kb, kb + per, kb * g, (kb + per) * g)


def assemble(gathered):
    """[world, layers, q heads per rank, d] (rank-major, as all_gather lays it
    out) -> [layers, n_q, d] in global head order."""
    w, layers, qh, d = gathered.shape
    if hasattr(gathered, "permute"):  # torch tensor (device or host)
        return gathered.permute(1, 0, 2, 3).reshape(layers, w * qh, d)
    return gathered.transpose(1, 0, 2, 3).reshape(layers, w * qh, d)
