"""kv_prefill_attn_shared: batches whose sequences begin with the same tokens on
the same pages (sessions forked from one prompt), against the CPU oracle.

The oracle runs the plain masked attention of every sequence through its own
block table (orc_paged_prefill); the library attends the shared pages once
for the whole batch and each sequence's remaining keys in a second launch,
merged by log-sum-exp.  Outputs within the bf16 tolerance (2e-2 normwise per
(token, query head) row), and close to kv_prefill_attn on the same inputs.
"""
import numpy as np
import pytest

from llmhost_b200.workloads import PAGE_TOKENS, normal_bits
from oracle import oracle as O
from paged_case import assert_close_rows, to_numpy_f32, to_torch

pytestmark = pytest.mark.gpu
NONE = 0xFFFFFFFF


def _depths(parents):
    d = []
    for p in parents:
        d.append(0 if p < 0 else d[p] + 1)
    return d


class SharedCase:
    """n sequences: the first S tokens shared (same pages, same K/V), then E_s
    private cached tokens, then a chunk (T_s causal tokens, or a tree given by
    its parent array)."""

    def __init__(self, n_q, n_kv, S, extra, chunks, seed=0):
        from llmhost_b200.kv import tree_masks

        rng = np.random.default_rng(seed)
        self.n_q, self.n_kv, self.S = n_q, n_kv, S
        n = len(extra)
        self.parents = [None if isinstance(c, int) else list(c) for c in chunks]
        self.tree = self.parents[0] is not None
        self.T = np.array([c if isinstance(c, int) else len(c) for c in chunks], np.int64)
        self.L = S + np.asarray(extra, np.int64)
        n_sh = S // PAGE_TOKENS
        own = -(-(self.L + self.T) // PAGE_TOKENS) - n_sh
        self.n_pages = n_sh + int(own.sum()) + 4
        perm = rng.permutation(self.n_pages).astype(np.uint32)
        width = n_sh + int(own.max())
        self.bt = np.full((n, width), NONE, np.uint32)
        cur = n_sh
        for s in range(n):
            self.bt[s, :n_sh] = perm[:n_sh]
            self.bt[s, n_sh:n_sh + own[s]] = perm[cur:cur + own[s]]
            cur += own[s]
        self.k_sh = normal_bits(rng, (S, n_kv, 64), "bf16")
        self.v_sh = normal_bits(rng, (S, n_kv, 64), "bf16")
        own_tok = self.L + self.T - S
        self.k = [normal_bits(rng, (int(t), n_kv, 64), "bf16") for t in own_tok]
        self.v = [normal_bits(rng, (int(t), n_kv, 64), "bf16") for t in own_tok]
        # positions of the private tokens: cached at their index, chunk i at L + depth(i) or L + i
        self.pos = []
        for s in range(n):
            chunk = _depths(self.parents[s]) if self.parents[s] is not None else list(range(int(self.T[s])))
            self.pos.append(np.concatenate([np.arange(S, self.L[s]), self.L[s] + np.array(chunk, np.int64)]))
        self.q = normal_bits(rng, (int(self.T.sum()), n_q, 64), "bf16")
        self.q_off = np.concatenate([[0], np.cumsum(self.T)]).astype(np.int32)
        self.q_pos = np.concatenate([p[int(L - S):] for p, L in zip(self.pos, self.L)]).astype(np.int32)
        self.masks = np.concatenate([tree_masks(p) for p in self.parents]) if self.tree else None
        self.max_q = int(self.T.max())
        self.max_pos = int(max(p.max(initial=0) for p in self.pos)) + 16

    def appends(self):
        """(rows, slots, positions, k, v) of every stored token: the shared ones once (row 0)."""
        n = len(self.L)
        rows = [np.zeros(self.S, np.int32)]
        slots = [np.arange(self.S, dtype=np.int32)]
        pos = [np.arange(self.S, dtype=np.int32)]
        for s in range(n):
            t = int(self.L[s] + self.T[s] - self.S)
            rows.append(np.full(t, s, np.int32))
            slots.append(np.arange(self.S, self.S + t, dtype=np.int32))
            pos.append(self.pos[s].astype(np.int32))
        k = np.concatenate([self.k_sh] + [a for a in self.k])
        v = np.concatenate([self.v_sh] + [a for a in self.v])
        return np.concatenate(rows), np.concatenate(slots), np.concatenate(pos), k, v

    def run_oracle(self):
        host = O.HostPages(self.n_pages, O.BF16, self.n_q, self.n_kv)
        rows, slots, pos, k, v = self.appends()
        host.append_tokens(self.bt, rows, slots, pos, k, v)
        return host.prefill(self.bt, self.L, self.q_off, self.q_pos, self.q, masks=self.masks)

    def run_gpu(self):
        import torch
        from llmhost_b200.kv import KvPool

        pool = KvPool(dtype="bf16", n_q_heads=self.n_q, n_kv_heads=self.n_kv, n_pages=self.n_pages,
                      max_positions=self.max_pos, max_seqs=len(self.L))
        dev = pool.device

        def i32(a):
            return torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(dev)

        rows, slots, pos, k, v = self.appends()
        bt = torch.from_numpy(self.bt.view(np.int32)).to(dev)
        pool.append(to_torch(k.reshape(-1), "bf16", dev), to_torch(v.reshape(-1), "bf16", dev), i32(rows), i32(slots),
                    i32(pos), bt)
        masks = None if self.masks is None else torch.from_numpy(self.masks).to(dev)
        q = to_torch(self.q, "bf16", dev)
        args = (q, i32(self.q_pos), i32(self.q_off), i32(self.L), bt)
        shared = pool.prefill_attn_shared(*args, shared_tokens=self.S, max_q=self.max_q, tree_masks=masks)
        again = pool.prefill_attn_shared(*args, shared_tokens=self.S, max_q=self.max_q, tree_masks=masks)
        plain = pool.prefill_attn(*args, tree_masks=masks, max_q=self.max_q)
        torch.cuda.synchronize()
        err = pool.last_error()
        pool.close()
        return to_numpy_f32(shared), to_numpy_f32(again), to_numpy_f32(plain), err


def check(case: SharedCase, what: str):
    ref = case.run_oracle()
    shared, again, plain, err = case.run_gpu()
    assert err == 0, f"device error word {err}"
    np.testing.assert_array_equal(shared, again, err_msg="repeated launches differ")
    assert_close_rows(shared, ref, 2e-2, what)
    assert_close_rows(shared, plain, 2e-2, what + " vs kv_prefill_attn")


def _tree(rng, n):
    return [-1] + [int(rng.integers(0, i)) for i in range(1, n)]


def test_shared_prefix_speculative_round(cuda):
    # the speculative configuration's verify: 32 sessions forked from a
    # 4096-token prompt, one 64-node tree each (the prefix pass is 2048 tokens
    # x 3 heads per kv head: the persistent schedule)
    rng = np.random.default_rng(7)
    case = SharedCase(24, 8, 4096, [0] * 32, [_tree(rng, 64) for _ in range(32)], seed=8)
    check(case, "shared 4096, 32 x 64-node trees")


def test_shared_prefix_ragged_private_keys(cuda):
    # private cached tokens after the shared ones (a later speculative round), ragged trees
    rng = np.random.default_rng(9)
    extra = [int(rng.integers(0, 300)) for _ in range(8)]
    case = SharedCase(24, 8, 512, extra, [_tree(rng, int(rng.integers(1, 65))) for _ in range(8)], seed=10)
    check(case, "shared 512, ragged")


def test_shared_prefix_causal_chunks(cuda):
    rng = np.random.default_rng(11)
    extra = [int(rng.integers(0, 200)) for _ in range(4)]
    case = SharedCase(32, 8, 1024, extra, [int(rng.integers(1, 120)) for _ in range(4)], seed=12)
    check(case, "shared 1024, causal chunks")


@pytest.mark.parametrize("n_q,n_kv", [(4, 1), (8, 2)])
def test_shared_prefix_kv_head_shards(cuda, n_q, n_kv):
    rng = np.random.default_rng(13 + n_kv)
    case = SharedCase(n_q, n_kv, 256, [0, 17, 40], [_tree(rng, n) for n in (5, 64, 33)], seed=14)
    check(case, f"shared 256, {n_q}q/{n_kv}kv")


def test_shared_prefix_longer_than_a_prefix_is_flagged(cuda):
    import torch

    rng = np.random.default_rng(15)
    case = SharedCase(24, 8, 256, [0, 0], [_tree(rng, 4), _tree(rng, 4)], seed=16)
    from llmhost_b200.kv import KvPool

    pool = KvPool(dtype="bf16", n_q_heads=24, n_kv_heads=8, n_pages=case.n_pages, max_positions=case.max_pos,
                  max_seqs=2)
    dev = pool.device

    def i32(a):
        return torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(dev)

    bt = torch.from_numpy(case.bt.view(np.int32)).to(dev)
    L = case.L.copy()
    L[1] = 128  # below the shared 256
    pool.prefill_attn_shared(to_torch(case.q, "bf16", dev), i32(case.q_pos), i32(case.q_off), i32(L), bt,
                             shared_tokens=256, max_q=case.max_q,
                             tree_masks=torch.from_numpy(case.masks).to(dev))
    torch.cuda.synchronize()
    assert pool.last_error() == 1  # KV_ERR_INVALID
    pool.close()
