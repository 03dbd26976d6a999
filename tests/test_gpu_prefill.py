"""Parity of chunked-prefill and tree-verify attention (kv_prefill_attn) against
the CPU oracle.

Each sequence has L cached tokens and a chunk of T new ones, all written with
kv_append (GPU) and orc_paged_append_token (oracle) from the same bits.  The
oracle gathers the stored K/V, rotates q at its position and runs
orc_attention_masked with the explicit mask: every cached key, plus chunk key
j for query i when j <= i (causal chunk) or j is an ancestor-or-self of i
(tree).  Tolerances normwise per (token, query head) row: 2e-2 for bf16 pools
(tcgen05 kernel), 1e-5 for fp32 pools (CUDA-core kernel).
"""
import numpy as np
import pytest

from llmhost_b200.workloads import PAGE_TOKENS, normal_bits
from oracle import oracle as O
from paged_case import PAGE_NONE, assert_close_rows, to_numpy_f32, to_torch

pytestmark = pytest.mark.gpu
RTOL = {"bf16": 2e-2, "f32": 1e-5}


def _depths(parents):
    d = []
    for p in parents:
        d.append(0 if p < 0 else d[p] + 1)
    return d


class PrefillCase:
    """seqs: list of (L, T) for a causal chunk or (L, parents) for a tree."""

    def __init__(self, n_q, n_kv, seqs, seed=0, extra_pages=4, dtype="bf16", store=None):
        from llmhost_b200.kv import tree_masks

        rng = np.random.default_rng(seed)
        self.n_q, self.n_kv, self.dtype = n_q, n_kv, dtype
        self.store = store or dtype  # the pool's storage type (quantised pools take bf16 q / k / v)
        self.L = np.array([s[0] for s in seqs], np.int64)
        self.parents = [None if isinstance(s[1], int) else list(s[1]) for s in seqs]
        self.T = np.array([s[1] if isinstance(s[1], int) else len(s[1]) for s in seqs], np.int64)
        self.tree = any(p is not None for p in self.parents)
        assert not self.tree or all(p is not None for p in self.parents)
        n = len(seqs)
        pages = -(-(self.L + self.T) // PAGE_TOKENS)
        self.n_pages = int(pages.sum()) + extra_pages
        perm = rng.permutation(self.n_pages).astype(np.uint32)
        self.bt = np.full((n, max(int(pages.max()), 1)), PAGE_NONE, np.uint32)
        cur = 0
        for s in range(n):
            self.bt[s, :pages[s]] = perm[cur:cur + pages[s]]
            cur += pages[s]
        tot = self.L + self.T
        # RoPE position of every stored token: cached t at t, chunk i at L + depth(i) (tree) or L + i
        self.pos = []
        for s in range(n):
            chunk = _depths(self.parents[s]) if self.parents[s] is not None else list(range(int(self.T[s])))
            self.pos.append(np.concatenate([np.arange(self.L[s]), self.L[s] + np.array(chunk, np.int64)]))
        self.k = [normal_bits(rng, (int(t), n_kv, 64), dtype) for t in tot]
        self.v = [normal_bits(rng, (int(t), n_kv, 64), dtype) for t in tot]
        self.q = normal_bits(rng, (int(self.T.sum()), n_q, 64), dtype)
        self.q_off = np.concatenate([[0], np.cumsum(self.T)]).astype(np.int32)
        self.q_pos = np.concatenate([p[int(L):] for p, L in zip(self.pos, self.L)]).astype(np.int32)
        self.masks = None
        if self.tree:
            self.masks = np.concatenate([tree_masks(p) for p in self.parents])
        self.max_pos = int(max((p.max(initial=0) for p in self.pos), default=0)) + 16

    def run_oracle(self):
        """Pages filled and attention computed by the oracle's bulk helpers
        (orc_paged_append_tokens, orc_paged_prefill), which
        tests/test_oracle_bulk.py pins bit for bit to the per-token append and
        orc_attention_masked with the explicit mask."""
        from paged_case import ORACLE_DTYPE

        host = O.HostPages(self.n_pages, ORACLE_DTYPE[self.store], self.n_q, self.n_kv)
        n = len(self.L)
        tot = self.L + self.T
        rows = np.repeat(np.arange(n, dtype=np.int32), tot)
        slots = np.concatenate([np.arange(int(t), dtype=np.int32) for t in tot]) if n else np.zeros(0, np.int32)
        pos = np.concatenate(self.pos).astype(np.int32) if n else np.zeros(0, np.int32)
        k = np.concatenate([a.reshape(-1, self.n_kv, 64) for a in self.k])
        v = np.concatenate([a.reshape(-1, self.n_kv, 64) for a in self.v])
        host.append_tokens(self.bt, rows, slots, pos, k, v)
        if self.q_off[-1] == 0:
            return host, np.zeros((0, self.n_q, 64), np.float32)
        out = host.prefill(self.bt, self.L, self.q_off, self.q_pos, self.q, masks=self.masks)
        return host, out

    def make_pool(self):
        from llmhost_b200.kv import KvPool

        return KvPool(dtype=self.store, n_q_heads=self.n_q, n_kv_heads=self.n_kv, n_pages=self.n_pages,
                      max_positions=self.max_pos, max_seqs=max(len(self.L), 1))

    def run_gpu(self, pool, max_q=None):
        import torch

        dev = pool.device
        n = len(self.L)
        tok_seq = np.concatenate([np.full(int(self.L[s] + self.T[s]), s, np.int32) for s in range(n)])
        tok_slot = np.concatenate([np.arange(int(self.L[s] + self.T[s]), dtype=np.int32) for s in range(n)])
        tok_pos = np.concatenate(self.pos).astype(np.int32)
        k = np.concatenate([a.reshape(-1) for a in self.k])
        v = np.concatenate([a.reshape(-1) for a in self.v])
        bt = torch.from_numpy(self.bt.view(np.int32)).to(dev)

        def i32(a):
            return torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(dev)

        pool.append(to_torch(k, self.dtype, dev), to_torch(v, self.dtype, dev), i32(tok_seq), i32(tok_slot),
                    i32(tok_pos), bt)
        masks = None if self.masks is None else torch.from_numpy(self.masks).to(dev)
        out = pool.prefill_attn(to_torch(self.q, self.dtype, dev), i32(self.q_pos), i32(self.q_off), i32(self.L), bt,
                                tree_masks=masks, max_q=max_q)
        torch.cuda.synchronize()
        return to_numpy_f32(out)


def check(case: PrefillCase, what: str):
    host, ref = case.run_oracle()
    with case.make_pool() as pool:
        out = case.run_gpu(pool)
        err = pool.last_error()
        ids = np.sort(case.bt[case.bt != PAGE_NONE])
        pages = pool.read_pages(ids)
    assert err == 0, f"device error word {err}"
    np.testing.assert_array_equal(pages, host.data[ids], err_msg="stored pages differ from the oracle")
    return assert_close_rows(out, ref, RTOL[case.dtype], what)


DTYPES = ["bf16", "f32"]


@pytest.mark.parametrize("dtype", DTYPES)
def test_prefill_causal_chunks_group3(cuda, dtype):
    # one token, chunks inside and across query tiles, prefixes that are and
    # are not multiples of the page size
    case = PrefillCase(24, 8, [(0, 1), (0, 37), (5, 16), (100, 50), (16, 128), (300, 200)], seed=11, dtype=dtype)
    check(case, f"{dtype} causal 24q/8kv")


@pytest.mark.parametrize("dtype", DTYPES)
def test_prefill_causal_chunks_group4(cuda, dtype):
    case = PrefillCase(32, 8, [(0, 33), (129, 7), (255, 129), (1000, 96)], seed=12, dtype=dtype)
    check(case, f"{dtype} causal 32q/8kv")


@pytest.mark.parametrize("dtype", DTYPES)
def test_prefill_from_position_zero_long(cuda, dtype):
    # a whole prompt in one chunk (the reference's attn_prefill case; the fp32
    # single-session workload prefills 2048 tokens of 24q/8kv)
    n_q, n = (32, 1024) if dtype == "bf16" else (24, 2048)
    case = PrefillCase(n_q, 8, [(0, n)], seed=13, dtype=dtype)
    check(case, f"{dtype} prompt {n}")


@pytest.mark.parametrize("dtype", DTYPES)
def test_prefill_single_kv_head(cuda, dtype):
    case = PrefillCase(4, 1, [(3000, 64), (0, 17)], seed=14, dtype=dtype)
    check(case, f"{dtype} 4q/1kv")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n_q", [24, 32])
def test_tree_verify(cuda, n_q, dtype):
    rng = np.random.default_rng(n_q)

    def rand_tree(n):
        return [-1] + [int(rng.integers(0, i)) for i in range(1, n)]

    seqs = [(37, rand_tree(20)), (0, rand_tree(64)), (200, [-1]), (16, list(range(-1, 15))), (513, rand_tree(43))]
    check(PrefillCase(n_q, 8, seqs, seed=15, dtype=dtype), f"{dtype} tree {n_q}q/8kv")


@pytest.mark.parametrize("dtype", DTYPES)
def test_prefill_empty_chunk_and_zero_seqs(cuda, dtype):
    case = PrefillCase(24, 8, [(10, 0), (0, 5), (20, 0)], seed=16, dtype=dtype)
    check(case, f"{dtype} empty chunks")
    import torch

    with case.make_pool() as pool:
        e = torch.empty(0, 24, 64, dtype=torch.bfloat16 if dtype == "bf16" else torch.float32, device=cuda)
        z = torch.zeros(1, dtype=torch.int32, device=cuda)
        pool.prefill_attn(e, z[:0], z, z[:0], torch.zeros(1, 1, dtype=torch.int32, device=cuda), max_q=0)
        assert pool.last_error() == 0


@pytest.mark.parametrize("dtype", DTYPES)
def test_prefill_chunk_longer_than_max_q_is_flagged(cuda, dtype):
    case = PrefillCase(24, 8, [(0, 50)], seed=17, dtype=dtype)
    with case.make_pool() as pool:
        case.run_gpu(pool, max_q=10)
        assert pool.last_error() == 1  # KV_ERR_INVALID
        assert pool.last_error() == 0  # the word was cleared


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n_q,n_kv", [(8, 2), (16, 4)])
def test_prefill_kv_head_shards(cuda, n_q, n_kv, dtype):
    # the per-GPU shapes of a KV-head-sharded session (group 4 over 2 and 4
    # kv heads): causal chunks and trees
    rng = np.random.default_rng(40 + n_q + n_kv)
    tree = [-1] + [int(rng.integers(0, i)) for i in range(1, 30)]
    check(PrefillCase(n_q, n_kv, [(0, 7), (130, 200), (17, 64)], seed=31, dtype=dtype), f"{dtype} {n_q}q/{n_kv}kv causal")
    check(PrefillCase(n_q, n_kv, [(40, tree), (0, [-1, 0, 0, 1])], seed=32, dtype=dtype), f"{dtype} {n_q}q/{n_kv}kv tree")


# ---- the persistent schedule (more (sequence, kv head, tile pair) units than SMs) ----------------
# Each CTA of the persistent grid takes an equal run of all units' key blocks;
# a unit cut between CTAs is computed in parts and merged by the last part.
# These cases reach its edges: a unit longer than several CTAs' runs (middle
# parts), units with no work (chunk shorter than the launch's max_q), fewer
# work positions than CTAs, tree masks, and launches repeated on the same
# pool (the merge counters must come back to zero).

def test_persistent_schedule_long_unit_split_many_ways(cuda):
    # 24 sequences x 8 kv heads = 192 units; one sequence has 20k cached keys,
    # so its units each span several CTAs' runs
    seqs = [(20000, 40)] + [(int(L), 30) for L in np.random.default_rng(50).integers(0, 600, size=23)]
    case = PrefillCase(24, 8, seqs, seed=51)
    host, ref = case.run_oracle()
    with case.make_pool() as pool:
        for rep in range(3):  # repeated launches on one pool
            out = case.run_gpu(pool)
            assert pool.last_error() == 0, rep
            assert_close_rows(out, ref, RTOL["bf16"], f"persistent long unit, launch {rep}")


def test_persistent_schedule_empty_units_and_few_positions(cuda):
    # max_q 256 at group 3 gives 4 tile pairs per (sequence, head): 5 x 8 x 4 =
    # 160 units, of which only the first tile pair of each holds tokens, so
    # the run list has fewer positions than the grid has CTAs
    seqs = [(0, 1), (5, 2), (100, 1), (0, 3), (17, 1)]
    case = PrefillCase(24, 8, seqs, seed=52)
    host, ref = case.run_oracle()
    with case.make_pool() as pool:
        for rep in range(2):
            out = case.run_gpu(pool, max_q=256)
            assert pool.last_error() == 0, rep
            assert_close_rows(out, ref, RTOL["bf16"], f"persistent sparse units, launch {rep}")


@pytest.mark.parametrize("n_q", [24, 32])
def test_persistent_schedule_tree_verify(cuda, n_q):
    # 32 sequences x 8 kv heads = 256 units: the speculative verify's launch
    # shape, with ragged prefixes and trees
    rng = np.random.default_rng(53 + n_q)

    def rand_tree(n):
        return [-1] + [int(rng.integers(0, i)) for i in range(1, n)]

    seqs = [(int(rng.integers(0, 3000)), rand_tree(int(rng.integers(1, 65)))) for _ in range(32)]
    check(PrefillCase(n_q, 8, seqs, seed=54), f"persistent tree verify {n_q}q/8kv")
