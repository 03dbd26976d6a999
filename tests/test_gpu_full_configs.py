"""Parity at the benchmark configurations' own sizes, through the C ABI.

Each test builds one configuration at the size the workload states (one layer
or two where every layer runs the same kernel on its own tables), runs it on
the GPU and replays it on the CPU oracle from the same seeded inputs:

* config 2, bf16 batched decode: the 64 sessions with lengths U[128, 8192]
  (seed 1) whose pages are drawn from a permutation of the 2^20-page pool;
  kv_append_decode_attn, kv_decode_attn and kv_norm_append_decode_attn; the
  same on Q8 and K8V4 pools (codes and scales bit-exact);
* config 3, bf16 chunked prefill: the last 512-token causal chunk after
  15 872 cached keys at 32q/8kv, beside the first chunk and a middle one;
* config 4, speculative tree: 32 sessions forked from a shared prefix, each
  with a 64-node tree of depth <= 6 from the workload's generator; the host
  state plans copy-on-write, the drafts are appended and verified with tree
  masks, the accepted paths are committed (kv_move_tokens) and the rejected
  pages freed; two rounds, then a decode step over the committed tables;
* config 5, long context: GPU 0's LPT share of the 256 sessions under a
  32 768-token window, 66 decode steps driven by plan_decode_step with its
  real evictions, new pages and one pool compaction (kv_copy_pages).

Bars: stored pages bit-identical to the oracle's, block tables, reference
counts and the free list identical to the independent Python model
(oracle/kvstate_model.py), attention within 2e-2 normwise per row (bf16).
The oracle fills pages with orc_paged_append_tokens and runs prefill with
orc_paged_prefill; tests/test_oracle_bulk.py pins both to the per-token
restatement bit for bit.
"""
import numpy as np
import pytest

from llmhost_b200.workloads import PAGE_TOKENS, normal_bits
from oracle import oracle as O
from paged_case import ORACLE_DTYPE, PAGE_NONE, assert_close_rows, to_numpy_f32, to_torch

pytestmark = pytest.mark.gpu
RTOL_BF16 = 2e-2


def _i32(a, dev):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a, np.int64).astype(np.int32)).to(dev)


def _u32(a, dev):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a, np.uint32).view(np.int32)).to(dev)


def _compact(bt):
    """Used page ids (sorted) and the block table renumbered 0..n-1 in that
    order, so the host copy holds only the pages the case touches."""
    ids = np.unique(bt[bt != PAGE_NONE])
    cbt = np.full_like(bt, PAGE_NONE)
    live = bt != PAGE_NONE
    cbt[live] = np.searchsorted(ids, bt[live]).astype(np.uint32)
    return ids, cbt


def _token_layout(lens):
    rows = np.repeat(np.arange(len(lens), dtype=np.int32), lens)
    slots = np.concatenate([np.arange(int(x), dtype=np.int32) for x in lens])
    return rows, slots


# ---- config 2 -----------------------------------------------------------------------
@pytest.mark.parametrize("store", ["bf16", "q8", "k8v4", "f16"])
def test_config2_batched_decode_full_size(cuda, store):
    import torch
    from llmhost_b200.kv import KvPool
    from llmhost_b200.workloads import decode_config

    wl = decode_config(steps=1, seed=1)  # the benchmark's sessions, lengths and page order
    assert wl.pool_pages == 1 << 20 and wl.n_seqs == 64
    bt = wl.block_tables[0]               # layer 0: the cached pages plus the decode token's page
    ids, cbt = _compact(bt)
    rng = np.random.default_rng(21)
    rows, slots = _token_layout(wl.l0)
    k = normal_bits(rng, (len(slots), wl.n_kv, 64), "bf16")
    v = normal_bits(rng, (len(slots), wl.n_kv, 64), "bf16")
    host = O.HostPages(len(ids), ORACLE_DTYPE[store], wl.n_q, wl.n_kv)
    host.append_tokens(cbt, rows, slots, slots, k, v)
    lens = wl.seq_lens(0)
    n = wl.n_seqs
    with KvPool(dtype=store, n_q_heads=wl.n_q, n_kv_heads=wl.n_kv, n_pages=wl.pool_pages,
                max_positions=int(lens.max()) + 16, max_seqs=n) as pool:
        bt_d = _u32(bt, cuda)
        pool.append(to_torch(k, "bf16", cuda), to_torch(v, "bf16", cuda), _i32(rows, cuda), _i32(slots, cuda),
                    _i32(slots, cuda), bt_d)
        del k, v
        lens_d = torch.from_numpy(lens).to(cuda)

        # 1. the benchmark's launch: append + attention in one kernel
        q = normal_bits(rng, (n, wl.n_q, 64), "bf16")
        kn = normal_bits(rng, (n, wl.n_kv, 64), "bf16")
        vn = normal_bits(rng, (n, wl.n_kv, 64), "bf16")
        out = pool.append_decode_attn(to_torch(kn, "bf16", cuda), to_torch(vn, "bf16", cuda), to_torch(q, "bf16", cuda),
                                      bt_d, lens_d)
        torch.cuda.synchronize()
        assert pool.last_error() == 0
        ref = host.decode_step(cbt, lens, 0, q, kn, vn)
        np.testing.assert_array_equal(pool.read_pages(ids), host.data, err_msg="config 2: stored pages differ")
        e1 = assert_close_rows(to_numpy_f32(out), ref, RTOL_BF16, "config 2 kv_append_decode_attn")

        # 2. attention alone on the same pages (kv_decode_attn), another q
        q2 = normal_bits(rng, (n, wl.n_q, 64), "bf16")
        out2 = pool.decode_attn(to_torch(q2, "bf16", cuda), bt_d, lens_d)
        torch.cuda.synchronize()
        assert pool.last_error() == 0
        ref2 = np.stack([host.decode(cbt[s], int(lens[s]), 0, q2[s]) for s in range(n)])
        e2 = assert_close_rows(to_numpy_f32(out2), ref2, RTOL_BF16, "config 2 kv_decode_attn")

        # 3. the layer's q/k RMSNorm folded in: the decode token's slot is written again
        qw = rng.uniform(0.5, 1.5, 64).astype(np.float32)
        kw = rng.uniform(0.5, 1.5, 64).astype(np.float32)
        q3 = normal_bits(rng, (n, wl.n_q, 64), "bf16")
        k3 = normal_bits(rng, (n, wl.n_kv, 64), "bf16")
        v3 = normal_bits(rng, (n, wl.n_kv, 64), "bf16")
        out3 = pool.norm_append_decode_attn(to_torch(k3, "bf16", cuda), to_torch(v3, "bf16", cuda),
                                            to_torch(q3, "bf16", cuda), torch.from_numpy(qw).to(cuda),
                                            torch.from_numpy(kw).to(cuda), 1e-5, bt_d, lens_d)
        torch.cuda.synchronize()
        assert pool.last_error() == 0
        ref3 = host.decode_step_norm(cbt, lens, 0, q3, k3, v3, qw, kw, 1e-5)
        tail = np.unique(bt[np.arange(n), (lens - 1) // PAGE_TOKENS])  # pages holding the decode token
        np.testing.assert_array_equal(pool.read_pages(tail), host.data[np.searchsorted(ids, tail)],
                                      err_msg="config 2: normalised K rows differ")
        e3 = assert_close_rows(to_numpy_f32(out3), ref3, RTOL_BF16, "config 2 kv_norm_append_decode_attn")
    print(f"config 2 {store} (64 sessions, {int(lens.sum())} keys, 2^20-page pool): worst row errors "
          f"{e1:.2e} / {e2:.2e} / {e3:.2e}")


# ---- config 3 -----------------------------------------------------------------------
def test_config3_chunked_prefill_full_size(cuda):
    import torch
    from llmhost_b200.kv import KvPool
    from llmhost_b200.workloads import chunked_prefill_config

    wl = chunked_prefill_config()  # 16 sessions x 32 chunks of 512, 32q/8kv, 2^17-page pool
    C = wl.chunk
    # (session, chunk index): four sessions at the last chunk (15 872 cached keys),
    # one at the first chunk and one in the middle, in one launch
    picks = [(0, 31), (5, 31), (10, 31), (15, 31), (3, 0), (7, 15)]
    sess = [s for s, _ in picks]
    cached = np.array([c * C for _, c in picks], np.int64)
    tot = cached + C
    bt = wl.block_tables[0][sess]
    bt = np.where(np.arange(bt.shape[1])[None, :] < (-(-tot // PAGE_TOKENS))[:, None], bt, PAGE_NONE).astype(np.uint32)
    ids, cbt = _compact(bt)
    rng = np.random.default_rng(23)
    rows, slots = _token_layout(tot)
    k = normal_bits(rng, (len(slots), wl.n_kv, 64), "bf16")
    v = normal_bits(rng, (len(slots), wl.n_kv, 64), "bf16")
    host = O.HostPages(len(ids), O.BF16, wl.n_q, wl.n_kv)
    host.append_tokens(cbt, rows, slots, slots, k, v)
    q_off = np.concatenate([[0], np.cumsum(np.full(len(picks), C))]).astype(np.int32)
    q_pos = np.concatenate([np.arange(c, c + C) for c in cached]).astype(np.int32)
    q = normal_bits(rng, (int(q_off[-1]), wl.n_q, 64), "bf16")
    with KvPool(dtype="bf16", n_q_heads=wl.n_q, n_kv_heads=wl.n_kv, n_pages=wl.pool_pages,
                max_positions=wl.total + 16, max_seqs=len(picks)) as pool:
        bt_d = _u32(bt, cuda)
        pool.append(to_torch(k, "bf16", cuda), to_torch(v, "bf16", cuda), _i32(rows, cuda), _i32(slots, cuda),
                    _i32(slots, cuda), bt_d)
        out = pool.prefill_attn(to_torch(q, "bf16", cuda), _i32(q_pos, cuda), _i32(q_off, cuda), _i32(cached, cuda),
                                bt_d, max_q=C)
        torch.cuda.synchronize()
        assert pool.last_error() == 0
        np.testing.assert_array_equal(pool.read_pages(ids), host.data, err_msg="config 3: stored pages differ")
        got = to_numpy_f32(out)
    ref = host.prefill(cbt, cached, q_off, q_pos, q)
    worst = assert_close_rows(got, ref, RTOL_BF16, "config 3 chunked prefill")
    print(f"config 3 (chunks after {cached.tolist()} keys): worst row error {worst:.2e}")


# ---- config 4 -----------------------------------------------------------------------
def _replay_moves(host, moves):
    """Page-addressed token moves, in order (kv_move_tokens' group order)."""
    pages = host.data.reshape(host.data.shape[0], 2 * host.n_kv, host.P, host.d)
    for sp, ss, dp, ds in np.asarray(moves).reshape(-1, 4):
        pages[dp, :, ds, :] = pages[sp, :, ss, :]


def _check_state(st, model, seqs, L, n_pages, draft=False):
    for s in seqs:
        for layer in range(L):
            assert st.table(s, layer, draft=draft) == model.table(s, layer, draft=draft), (s, layer, draft)
    assert st.free_list() == model.free_list()
    assert [st.refcount(p) for p in range(n_pages)] == model.ref


@pytest.mark.parametrize("prefix", [4096, 4101])
def test_config4_speculative_rounds_full_size(cuda, prefix):
    """prefix 4096 is the workload's (page-aligned: drafts open fresh pages);
    4101 leaves a shared partial tail page, so every session's first draft
    copies it before writing (copy-on-write)."""
    import torch
    from llmhost_b200.kv import KvPool
    from llmhost_b200.plans import commit_moves, plan_forward
    from llmhost_b200.state import KvState
    from llmhost_b200.workloads import SpecTreeWorkload
    from oracle.kvstate_model import Model

    wl = SpecTreeWorkload(prefix=prefix, steps=2)
    rounds = wl.plan()
    n, T, L = wl.n_seqs, wl.nodes, wl.n_layers
    n_pages = 8192  # a seeded permutation like the workload's 2^16-page pool, sized for two rounds
    order = np.random.default_rng(wl.seed).permutation(n_pages).astype(np.uint32)
    st = KvState(n_pages, L, alloc_order=order)
    model = Model(n_pages, L, order=order.tolist())
    host = O.HostPages(n_pages, O.BF16, wl.n_q, wl.n_kv)
    rng = np.random.default_rng(24 + prefix)
    max_tokens = prefix + (wl.depth + 1) * len(rounds) + T + 1
    stride = -(-max_tokens // PAGE_TOKENS) + 1
    pool = KvPool(dtype="bf16", n_q_heads=wl.n_q, n_kv_heads=wl.n_kv, n_pages=n_pages, max_positions=max_tokens + 16,
                  max_seqs=n)
    try:
        # the shared prefix: session 0 prefills it, the others fork (refcount n)
        st.open(0)
        model.open(0)
        st.append(0, prefix)
        model.append(0, prefix)
        pos = np.arange(prefix, dtype=np.int32)
        for layer in range(L):
            t0 = st.export_tables([0], layer, stride)
            k = normal_bits(rng, (prefix, wl.n_kv, 64), "bf16")
            v = normal_bits(rng, (prefix, wl.n_kv, 64), "bf16")
            pool.append(to_torch(k, "bf16", cuda), to_torch(v, "bf16", cuda), _i32(np.zeros(prefix), cuda),
                        _i32(pos, cuda), _i32(pos, cuda), _u32(t0, cuda))
            host.append_tokens(t0, np.zeros(prefix, np.int32), pos, pos, k, v)
        for s in range(1, n):
            st.fork(0, s)
            model.fork(0, s)
        seqs = list(range(n))
        _check_state(st, model, seqs, L, n_pages)
        tokens = np.tile(np.arange(1000, 1000 + T, dtype=np.uint32), (n, 1))
        check_layers = (0, L - 1)
        n_cow = 0
        for rnd, rows in enumerate(rounds):
            parents = np.array([r[0] for r in rows], np.int32)
            paths = [list(r[1]) for r in rows]
            fb = plan_forward(st, seqs, tokens, parents, stride)
            for s in seqs:
                model.forward(s, tokens[s].tolist(), parents[s].tolist())
            _check_state(st, model, seqs, L, n_pages, draft=True)
            n_cow += len(fb.cow_src)
            if len(fb.cow_src):
                pool.copy_pages(_u32(fb.cow_src, cuda), _u32(fb.cow_dst, cuda))
                host.data[fb.cow_dst] = host.data[fb.cow_src]
            ntok = fb.n_tokens
            assert ntok == n * T
            masks_d = torch.from_numpy(fb.masks).to(cuda)
            for layer in range(L):
                k = normal_bits(rng, (ntok, wl.n_kv, 64), "bf16")
                v = normal_bits(rng, (ntok, wl.n_kv, 64), "bf16")
                q = normal_bits(rng, (ntok, wl.n_q, 64), "bf16")
                tab = fb.tables[layer]
                tab_d = _u32(tab, cuda)
                pool.append(to_torch(k, "bf16", cuda), to_torch(v, "bf16", cuda), _i32(fb.tok_seq, cuda),
                            _i32(fb.slots, cuda), _i32(fb.positions, cuda), tab_d)
                host.append_tokens(tab, fb.tok_seq, fb.slots, fb.positions, k, v)
                out = pool.prefill_attn(to_torch(q, "bf16", cuda), _i32(fb.positions, cuda), _i32(fb.q_offsets, cuda),
                                        _i32(fb.prefix, cuda), tab_d, tree_masks=masks_d, max_q=T)
                torch.cuda.synchronize()
                assert pool.last_error() == 0
                if layer in check_layers:
                    ref = host.prefill(tab, fb.prefix, fb.q_offsets, fb.positions, q, masks=fb.masks)
                    assert_close_rows(to_numpy_f32(out), ref, RTOL_BF16, f"config 4 verify, round {rnd}, layer {layer}")
            mv, offs, acc = commit_moves(st, seqs, paths)
            for s in seqs:
                model.accept(s, paths[s])
            _check_state(st, model, seqs, L, n_pages)
            assert acc == sum(len(p) for p in paths)
            if len(mv):
                pool.move_tokens(_i32(np.asarray(mv).reshape(-1, 4), cuda), _i32(offs, cuda))
                _replay_moves(host, mv)
            torch.cuda.synchronize()
            assert pool.last_error() == 0
            live = sorted({p for s in seqs for layer in range(L) for p in st.table(s, layer) if p != PAGE_NONE})
            np.testing.assert_array_equal(pool.read_pages(np.array(live)), host.data[live],
                                          err_msg=f"config 4: pages after commit, round {rnd}")
        if prefix % PAGE_TOKENS:
            assert n_cow >= (n - 1) * L  # every forked session copied the shared tail page
        # a decode token per session over the committed tables (layer 0)
        for s in seqs:
            cow = st.append(s, 1)
            model.append(s, 1)
            for a, b in cow:
                pool.copy_pages(_u32([a], cuda), _u32([b], cuda))
                host.data[b] = host.data[a]
        _check_state(st, model, seqs, L, n_pages)
        lens = np.array([st.token_count(s) for s in seqs], np.int32)
        bt = st.export_tables(seqs, 0, stride)
        q = normal_bits(rng, (n, wl.n_q, 64), "bf16")
        kn = normal_bits(rng, (n, wl.n_kv, 64), "bf16")
        vn = normal_bits(rng, (n, wl.n_kv, 64), "bf16")
        out = pool.append_decode_attn(to_torch(kn, "bf16", cuda), to_torch(vn, "bf16", cuda), to_torch(q, "bf16", cuda),
                                      _u32(bt, cuda), _i32(lens, cuda))
        torch.cuda.synchronize()
        assert pool.last_error() == 0
        ref = host.decode_step(bt, lens, 0, q, kn, vn)
        assert_close_rows(to_numpy_f32(out), ref, RTOL_BF16, "config 4 decode after the rounds")
    finally:
        pool.close()
        st.close_all()


# ---- config 5 -----------------------------------------------------------------------
def test_config5_windowed_decode_evict_compact_full_size(cuda):
    import torch
    from llmhost_b200.kv import KvPool
    from llmhost_b200.plans import plan_decode_step
    from llmhost_b200.state import KvState
    from llmhost_b200.workloads import long_context_config

    wl = long_context_config(rank=0)  # GPU 0's LPT share of the 256 sessions
    W, every = wl.window, wl.compact_every
    L = 2  # every layer runs the same kernel on its own tables; two keep the page interleaving
    l0 = wl.l0
    n = len(l0)
    seqs = list(range(n))
    steps = every + 2  # one compaction (after step every-1) and two steps on the compacted pool
    resident = np.minimum(l0, W)
    # the window's pages, a new page per 16 steps, and one 8192-token piece of growth
    n_pages = int(L * (np.sum(-(-resident // PAGE_TOKENS)) + 2 * n + n * (steps // PAGE_TOKENS + 2) + 1024))
    order = np.random.default_rng(55).permutation(n_pages).astype(np.uint32)
    st = KvState(n_pages, L, alloc_order=order)
    # sessions grow in 8192-token pieces, evicting below the window as they go,
    # so the pool never holds more than the window plus one piece per session
    for s in seqs:
        st.open(s)
        left = int(l0[s])
        while left:
            c = min(left, 8192)
            st.append(s, c)
            st.evict_window(s, W)
            left -= c
    stride = -(-(int(l0.max()) + steps) // PAGE_TOKENS) + 1
    host = O.HostPages(n_pages, O.BF16, wl.n_q, wl.n_kv)
    rng = np.random.default_rng(25)
    pool = KvPool(dtype="bf16", n_q_heads=wl.n_q, n_kv_heads=wl.n_kv, n_pages=n_pages,
                  max_positions=int(l0.max()) + steps + 16, max_seqs=n)
    try:
        first = np.maximum(l0 - W, 0) // PAGE_TOKENS * PAGE_TOKENS  # first token of the first resident page
        rows = np.repeat(np.arange(n, dtype=np.int32), l0 - first)
        slots = np.concatenate([np.arange(a, b, dtype=np.int32) for a, b in zip(first, l0)])
        for layer in range(L):
            bt = st.export_tables(seqs, layer, stride)
            k = normal_bits(rng, (len(slots), wl.n_kv, 64), "bf16")
            v = normal_bits(rng, (len(slots), wl.n_kv, 64), "bf16")
            pool.append(to_torch(k, "bf16", cuda), to_torch(v, "bf16", cuda), _i32(rows, cuda), _i32(slots, cuda),
                        _i32(slots, cuda), _u32(bt, cuda))
            host.append_tokens(bt, rows, slots, slots, k, v)
            del k, v
        torch.cuda.synchronize()
        assert pool.last_error() == 0
        stats = {"evicted": 0, "moved": 0, "new_pages": 0}
        check_at = {0, 15, 31, every - 2, every - 1, every, every + 1}
        worst = 0.0
        for i in range(steps):
            ds = plan_decode_step(st, seqs, W, compact=(i % every == every - 1))
            stats["evicted"] += ds.evicted
            stats["new_pages"] += len(ds.new_pages)
            if ds.compaction:
                mv = np.asarray(ds.compaction, np.uint32)
                stats["moved"] += len(mv)
                pool.copy_pages(_u32(mv[:, 0], cuda), _u32(mv[:, 1], cuda))
                host.data[mv[:, 1]] = host.data[mv[:, 0]]
                # the compaction rule: afterwards the live pages are exactly ids [0, used)
                used = n_pages - len(st.free_list())
                live = np.unique(np.concatenate([st.export_tables(seqs, layer, stride).ravel() for layer in range(L)]))
                assert np.array_equal(live[live != PAGE_NONE], np.arange(used)), "compaction left holes"
            lens = np.array([st.token_count(s) for s in seqs], np.int32)
            for layer in range(L):
                bt = st.export_tables(seqs, layer, stride)
                q = normal_bits(rng, (n, wl.n_q, 64), "bf16")
                kn = normal_bits(rng, (n, wl.n_kv, 64), "bf16")
                vn = normal_bits(rng, (n, wl.n_kv, 64), "bf16")
                out = pool.append_decode_attn(to_torch(kn, "bf16", cuda), to_torch(vn, "bf16", cuda),
                                              to_torch(q, "bf16", cuda), _u32(bt, cuda), _i32(lens, cuda), window=W)
                if i in check_at and (layer == 0 or i == steps - 1):
                    ref = host.decode_step(bt, lens, W, q, kn, vn)
                    torch.cuda.synchronize()
                    assert pool.last_error() == 0, f"step {i}"
                    worst = max(worst, assert_close_rows(to_numpy_f32(out), ref, RTOL_BF16,
                                                         f"config 5 step {i} layer {layer}"))
                else:
                    host.append_tokens(bt, np.arange(n, dtype=np.int32), lens - 1, lens - 1, kn, vn)
        torch.cuda.synchronize()
        assert pool.last_error() == 0
        assert stats["moved"] > 0 and stats["evicted"] > 0 and stats["new_pages"] > 0, stats
        live = np.unique(np.concatenate([st.export_tables(seqs, layer, stride).ravel() for layer in range(L)]))
        live = live[live != PAGE_NONE]
        np.testing.assert_array_equal(pool.read_pages(live), host.data[live],
                                      err_msg="config 5: pages after eviction and compaction")
        print(f"config 5 ({n} sessions, {steps} steps): {stats}, worst row error {worst:.2e}")
    finally:
        pool.close()
        st.close_all()
