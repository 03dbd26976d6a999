"""Host-side step planners (llmhost_b200/plans.py) against per-session KvState
calls, and the workload generators' invariants.  No GPU needed."""
import numpy as np

from llmhost_b200.plans import PAGE_NONE, commit_moves, plan_decode_step, plan_forward
from llmhost_b200.state import KvState, validate_accept_path, validate_tree
from llmhost_b200.workloads import (SpecTreeWorkload, accept_path, chunked_prefill_config, draft_tree,
                                    long_context_config, lpt_partition)


def _two_states(n_pages=512, layers=2):
    order = np.random.default_rng(0).permutation(n_pages)
    return KvState(n_pages, layers, alloc_order=order), KvState(n_pages, layers, alloc_order=order)


def test_plan_forward_and_commit_match_per_session_calls():
    a, b = _two_states()
    for st in (a, b):
        st.open(0)
        st.append(0, 37)
        for s in (1, 2):
            st.fork(0, s)
    seqs = [0, 1, 2]
    rng = np.random.default_rng(1)
    trees = [draft_tree(rng, 9)[0], draft_tree(rng, 12)[0], [-1]]
    toks = [list(range(100, 100 + len(t))) for t in trees]
    fb = plan_forward(a, seqs, toks, trees, stride=16)
    cow, off = [], 0
    for row, s in enumerate(seqs):
        plan = b.forward(s, toks[row], trees[row])
        n = len(trees[row])
        assert fb.q_offsets[row] == off and fb.q_offsets[row + 1] == off + n
        np.testing.assert_array_equal(fb.slots[off:off + n], plan.slots)
        np.testing.assert_array_equal(fb.positions[off:off + n], plan.positions)
        assert (fb.tok_seq[off:off + n] == row).all()
        assert fb.prefix[row] == 37
        cow += plan.cow
        for layer in range(2):
            t = b.table(s, layer, draft=True)
            assert fb.tables[layer, row, :len(t)].tolist() == t
            assert (fb.tables[layer, row, len(t):] == PAGE_NONE).all()
        off += n
    assert list(zip(fb.cow_src.tolist(), fb.cow_dst.tolist())) == cow
    # all three sessions share the partial tail page (refcount 3), so each
    # copies it before its draft writes there, once per layer
    assert len(cow) == 3 * 2
    paths = [[0, 1], [0], [0]]
    mv, offs, acc = commit_moves(a, seqs, paths)
    assert acc == 4 and len(offs) == 1 + 3 * 2
    for s, p in zip(seqs, paths):
        _, tm = b.accept(s, p, with_pages=True)
    for s in seqs:
        assert a.committed(s) == b.committed(s)
        assert a.table(s, 0) == b.table(s, 0)


def test_forward_batch_masks_chains_and_errors():
    import pytest

    from llmhost_b200.plans import tree_masks
    from llmhost_b200.state import EngineError

    a, b = _two_states()
    for st in (a, b):
        for s in (0, 1, 2):
            st.open(s)
            st.append(s, 5 + 7 * s)
    rng = np.random.default_rng(3)
    trees = [draft_tree(rng, 20)[0], [-1, 0, 0, 1], list(range(-1, 63))]
    f = a.forward_batch([0, 1, 2], [list(range(len(t))) for t in trees], trees, stride=16)
    np.testing.assert_array_equal(f["masks"], np.concatenate([tree_masks(t) for t in trees]))
    np.testing.assert_array_equal(f["prefix"], [5, 12, 19])
    # no trees: chains, whose masks are the prefixes 0..i
    f = b.forward_batch([0, 1], [[1, 2, 3], [4]], None, stride=16)
    assert f["masks"].view(np.uint64).tolist() == [1, 3, 7, 1]
    np.testing.assert_array_equal(f["positions"], [5, 6, 7, 12])

    # a bad tree in the second sequence: the first is staged, the third is not
    c, _ = _two_states()
    for s in (0, 1, 2):
        c.open(s)
    with pytest.raises(EngineError) as e:
        c.forward_batch([0, 1, 2], [[1], [1, 2], [1]], [[-1], [-1, 1], [-1]], stride=4)
    assert e.value.kind == "Tree" and e.value.seq_id == 1
    assert c.pending_base(0) == 0
    with pytest.raises(EngineError) as e:
        c.pending_base(2)
    assert e.value.kind == "NoPendingForward"
    # tables wider than the stride: refused before any state changes
    d, _ = _two_states()
    d.open(0)
    d.append(0, 40)
    with pytest.raises(Exception):
        d.forward_batch([0], [list(range(30))], None, stride=4)  # 70 tokens need 5 pages
    with pytest.raises(EngineError):
        d.pending_base(0)
    # more than 64 tokens cannot be described by masks
    with pytest.raises(Exception):
        d.forward_batch([0], [list(range(65))], None, stride=16)


def test_accept_batch_grows_its_buffer_and_stops_at_a_bad_path():
    import pytest

    from llmhost_b200.state import EngineError

    a, b = _two_states()
    for st in (a, b):
        for s in (0, 1):
            st.open(s)
            st.append(s, 30)
    trees = [[-1, 0, 1, 1], [-1, 0]]
    toks = [[7, 8, 9, 10], [5, 6]]
    plan_forward(a, [0, 1], toks, trees, stride=16)
    for s in (0, 1):
        b.forward(s, toks[s], trees[s])
    a._accept_cap = 1  # too small: the call reports the size and runs again
    mv, offs, acc = commit_moves(a, [0, 1], [[0, 1, 3], [0]])
    assert acc == 4 and len(offs) == 1 + 2 * 2
    ref = [b.accept(s, p, with_pages=True)[1] for s, p in ((0, [0, 1, 3]), (1, [0]))]
    want = np.concatenate([r[layer * (len(r) // 2):(layer + 1) * (len(r) // 2)] for r in ref for layer in range(2)])
    np.testing.assert_array_equal(mv, want.reshape(-1, 4))
    for s in (0, 1):
        assert a.committed(s) == b.committed(s) and a.table(s, 1) == b.table(s, 1)
    # a path that is not closed under parents, in the second sequence
    plan_forward(a, [0, 1], toks, trees, stride=16)
    with pytest.raises(EngineError) as e:
        commit_moves(a, [0, 1], [[0], [1]])
    assert e.value.kind == "InvalidAccept" and e.value.seq_id == 1
    assert len(a.committed(0)) == 34  # the first sequence committed its path


def test_plan_decode_step_publishes_new_pages_and_evicts():
    st = KvState(256, 2)
    for s in (0, 1):
        st.open(s)
    st.append(0, 16)  # the next token opens page 1
    st.append(1, 40)
    step = plan_decode_step(st, [0, 1], window=0, compact=False)
    # session 0 opened its second page, session 1 did not
    assert [(l, r, i) for l, r, i, _ in step.new_pages] == [(0, 0, 1), (1, 0, 1)]
    for layer, row, idx, page in step.new_pages:
        assert st.table(row, layer)[idx] == page
    st.append(1, 100)
    step = plan_decode_step(st, [0, 1], window=32, compact=True)
    assert step.evicted > 0
    assert st.table(1, 0)[0] == PAGE_NONE
    # compaction moved pages into the holes the eviction left
    assert step.compaction and all(d < s for s, d in step.compaction)


def test_draft_trees_and_accepted_paths_are_valid():
    rng = np.random.default_rng(4)
    for _ in range(50):
        parents, children = draft_tree(rng, 64, 6)
        assert len(parents) == 64
        validate_tree(parents)
        depth = [0] * 64
        for i, p in enumerate(parents):
            if p >= 0:
                depth[i] = depth[p] + 1
        assert max(depth) <= 6
        path = accept_path(rng, children)
        validate_accept_path(parents, sorted(path))
        assert path[0] == 0 and len(path) <= 7
    plan = SpecTreeWorkload(steps=2).plan()
    assert len(plan) == 2 and len(plan[0]) == 32


def test_lpt_partition_balances_and_covers():
    w = [100, 90, 80, 70, 10, 10, 5]
    parts = lpt_partition(w, 3)
    assert sorted(i for p in parts for i in p) == list(range(len(w)))
    loads = [sum(w[i] for i in p) for p in parts]
    assert max(loads) - min(loads) <= max(w)
    lc = long_context_config(rank=0)
    allp = [i for r in range(8) for i in long_context_config(rank=r).shard]
    assert sorted(allp) == list(range(256))
    res = np.minimum(lc.lengths, lc.window)
    loads = [res[long_context_config(rank=r).shard].sum() for r in range(8)]
    assert max(loads) / min(loads) < 1.02


def test_chunked_prefill_flops_match_closed_form():
    wl = chunked_prefill_config()
    # 4 d n_q sum_c [C * 512 c + C (C + 1) / 2] per (session, layer)
    per = 4 * 64 * 32 * sum(512 * 512 * c + 512 * 513 / 2 for c in range(32))
    assert abs(wl.total_flops() - per * 16 * 6) < 1e3


def test_batched_calls_take_arrays_like_lists():
    a, b = _two_states()
    for st in (a, b):
        for s in (0, 1, 2):
            st.open(s)
            st.append(s, 20 + 9 * s)
    rng = np.random.default_rng(7)
    trees = [draft_tree(rng, 12)[0] for _ in range(3)]
    toks = [list(range(50 + 12 * i, 62 + 12 * i)) for i in range(3)]
    fa = a.forward_batch([0, 1, 2], toks, trees, stride=16)
    fb = b.forward_batch([0, 1, 2], np.array(toks, np.int64), np.array(trees, np.int32), stride=16)
    for k in fa:
        np.testing.assert_array_equal(fa[k], fb[k], err_msg=k)
    paths = [[0, 1], [0], [0, 2]]
    flat = np.array([0, 1, 0, 0, 2], np.int64)
    off = np.array([0, 2, 3, 5], np.int32)
    ma, ga, na = commit_moves(a, [0, 1, 2], paths)
    mb, gb, nb = commit_moves(b, [0, 1, 2], (flat, off))
    np.testing.assert_array_equal(ma, mb)
    np.testing.assert_array_equal(ga, gb)
    assert na == nb == 5
    for s in (0, 1, 2):
        assert a.committed(s) == b.committed(s)
