"""Plans of the host-side KV state run on the GPU, checked against a host replay.

A speculative round (prefill, copy-on-write fork, draft trees, accepted
paths) is planned by KvState; the GPU runs the plans with kv_append,
kv_copy_pages and kv_move_tokens, the oracle replays them on host pages.
Pages must match bit for bit, and decode attention over the committed
sequences must match the oracle within the bf16 tolerance.  The round runs on
bf16 pools and on both quantised pool types (whose token moves carry the code
rows and the scale rows of every head).
"""
import numpy as np
import pytest

from llmhost_b200.workloads import normal_bits
from oracle import oracle as O
from paged_case import ORACLE_DTYPE, assert_close_rows, to_numpy_f32, to_torch

pytestmark = pytest.mark.gpu
NONE = 0xFFFFFFFF


@pytest.mark.parametrize("store", ["bf16", "q8", "k8v4", "f16"])
def test_copy_pages_bit_exact(cuda, store):
    import torch
    from llmhost_b200.kv import KvPool

    rng = np.random.default_rng(0)
    with KvPool(dtype=store, n_q_heads=24, n_kv_heads=8, n_pages=64, max_positions=64, max_seqs=4) as pool:
        if store in ("bf16", "f16"):  # 16-bit elements, read back as uint16 bits
            data = rng.integers(0, 1 << 16, size=(64, 2 * 8 * 16 * 64), dtype=np.uint16)
        else:
            data = rng.integers(0, 256, size=(64, pool.page_bytes), dtype=np.uint8)
        pool.write_pages(np.arange(64), data)
        src = torch.tensor([3, 5, 7, 40], dtype=torch.int32, device=cuda)
        dst = torch.tensor([10, 11, 12, 63], dtype=torch.int32, device=cuda)
        pool.copy_pages(src, dst)
        torch.cuda.synchronize()
        got = pool.read_pages(np.arange(64))
        assert pool.last_error() == 0
    want = data.copy()
    want[[10, 11, 12, 63]] = data[[3, 5, 7, 40]]
    np.testing.assert_array_equal(got, want)


def _replay_moves(host, moves):
    """Host replay of page-addressed token moves, in order: a token is its
    (head, slot) row of every page section."""
    P, d, nkv = host.P, host.d, host.n_kv
    n = host.data.shape[0]
    if host.quant:  # head blocks of K codes, V codes, scales (bytes)
        rows = [d, d if host.dtype == O.Q8 else d // 2, 8]
        blocks = host.data.reshape(n, nkv, -1)
        views, at = [], 0
        for r in rows:
            views.append(blocks[:, :, at:at + P * r].reshape(n, nkv, P, r))
            at += P * r
        assert at == blocks.shape[2]
    else:
        views = [host.data.reshape(n, 2 * nkv, P, d)]
    for sp, ss, dp, ds in moves:
        for v in views:
            v[dp, :, ds, :] = v[sp, :, ss, :]


@pytest.mark.parametrize("seed,store", [(1, "bf16"), (2, "bf16"), (3, "q8"), (4, "k8v4"), (5, "f16")])
def test_speculative_round_matches_oracle(cuda, seed, store):
    import torch
    from llmhost_b200.kv import KvPool
    from llmhost_b200.state import KvState

    rng = np.random.default_rng(seed)
    L, n_q, n_kv, n_pages = 2, 24, 8, 256
    order = rng.permutation(n_pages).astype(np.uint32)
    st = KvState(n_pages, L, alloc_order=order)
    host = O.HostPages(n_pages, ORACLE_DTYPE[store], n_q, n_kv)
    pool = KvPool(dtype=store, n_q_heads=n_q, n_kv_heads=n_kv, n_pages=n_pages, max_positions=512, max_seqs=8)

    def dev_i32(a):
        return torch.from_numpy(np.ascontiguousarray(a, dtype=np.int64).astype(np.int32)).to(cuda)

    def append_tokens(seq, slots, positions, draft):
        """K/V of len(slots) tokens written on both sides, every layer."""
        for layer in range(L):
            bt = np.array(st.table(seq, layer, draft=draft), np.uint32)
            k = normal_bits(rng, (len(slots), n_kv, 64), "bf16")
            v = normal_bits(rng, (len(slots), n_kv, 64), "bf16")
            for i, (sl, po) in enumerate(zip(slots, positions)):
                host.append_token(bt, int(sl), int(po), k[i], v[i])
            bt_d = torch.from_numpy(bt.view(np.int32)).to(cuda)[None, :]
            zeros = torch.zeros(len(slots), dtype=torch.int32, device=cuda)
            pool.append(to_torch(k.reshape(-1), "bf16", cuda), to_torch(v.reshape(-1), "bf16", cuda), zeros,
                        dev_i32(slots), dev_i32(positions), bt_d)

    def run_copies(cow):
        if not cow:
            return
        src = np.array([c[0] for c in cow])
        dst = np.array([c[1] for c in cow])
        host.data[dst] = host.data[src]
        pool.copy_pages(dev_i32(src), dev_i32(dst))

    # prefill three sequences, fork a fourth from the first (shared, partial tail)
    lens = {1: 21, 2: 16, 3: 37}
    for s, n in lens.items():
        st.open(s)
        run_copies(st.append(s, n))
        append_tokens(s, list(range(n)), list(range(n)), draft=False)
    st.fork(1, 4)
    seqs = [1, 2, 3, 4]
    # one speculative round per sequence
    all_moves = []
    groups = [0]
    for s in seqs:
        n = int(rng.integers(3, 12))
        tree = [-1] + [int(rng.integers(0, i)) for i in range(1, n)]
        plan = st.forward(s, list(range(500, 500 + n)), tree)
        run_copies(plan.cow)
        append_tokens(s, plan.slots, plan.positions, draft=True)
        node = int(rng.integers(0, n))
        path = []
        while node != -1:
            path.append(node)
            node = tree[node]
        _, tok_moves = st.accept(s, sorted(path), with_pages=True)
        for layer in range(L):  # one group per (sequence, layer)
            part = tok_moves[layer * (len(tok_moves) // L):(layer + 1) * (len(tok_moves) // L)]
            all_moves.extend(part.tolist())
            groups.append(len(all_moves))
    _replay_moves(host, all_moves)
    if all_moves:
        pool.move_tokens(torch.tensor(all_moves, dtype=torch.int32, device=cuda),
                         torch.tensor(groups, dtype=torch.int32, device=cuda))
    torch.cuda.synchronize()
    assert pool.last_error() == 0
    used = sorted({p for s in seqs for layer in range(L) for p in st.table(s, layer) if p != NONE})
    np.testing.assert_array_equal(pool.read_pages(np.array(used)), host.data[used])

    # decode one more token per sequence over the committed tables, each layer
    stride = max(len(st.table(s, 0)) for s in seqs) + 1
    for s in seqs:
        run_copies(st.append(s, 1))  # reserve the decode token's slot (it may open a page)
    seq_lens = np.array([st.token_count(s) for s in seqs], np.int32)
    for layer in range(L):
        bt = st.export_tables(seqs, layer, stride)
        q = normal_bits(rng, (len(seqs), n_q, 64), "bf16")
        k = normal_bits(rng, (len(seqs), n_kv, 64), "bf16")
        v = normal_bits(rng, (len(seqs), n_kv, 64), "bf16")
        ref = host.decode_step(bt, seq_lens, 0, q, k, v)
        bt_d = torch.from_numpy(bt.view(np.int32)).to(cuda)
        lens_d = torch.from_numpy(seq_lens).to(cuda)
        pool.append_decode(to_torch(k, "bf16", cuda), to_torch(v, "bf16", cuda), bt_d, lens_d)
        out = pool.decode_attn(to_torch(q, "bf16", cuda), bt_d, lens_d)
        torch.cuda.synchronize()
        assert_close_rows(to_numpy_f32(out), ref, 2e-2, f"decode after commit, layer {layer}")
    assert pool.last_error() == 0
    pool.close()


def test_copy_pages_more_than_one_launch(cuda):
    # a compaction can move more pages than one launch's grid holds (65535)
    import torch
    from llmhost_b200.kv import KvPool

    n = 70000
    with KvPool(dtype="bf16", n_q_heads=4, n_kv_heads=1, n_pages=2 * n, max_positions=64, max_seqs=1) as pool:
        src_ids = np.arange(n, 2 * n)
        data = np.random.default_rng(3).integers(0, 1 << 16, size=(n, pool.shape.page_elems), dtype=np.uint16)
        pool.write_pages(src_ids, data)
        pool.copy_pages(torch.arange(n, 2 * n, dtype=torch.int32, device=cuda),
                        torch.arange(0, n, dtype=torch.int32, device=cuda))
        torch.cuda.synchronize()
        assert pool.last_error() == 0
        got = pool.read_pages(np.array([0, 65534, 65535, 65536, n - 1]))
    np.testing.assert_array_equal(got, data[[0, 65534, 65535, 65536, n - 1]])
