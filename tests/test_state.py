"""Host-side KV state: the reference's engine/tree/cache assertions, and the
C++ state against the independent Python model (oracle/kvstate_model.py),
bit-exact over random operation sequences.  No GPU needed.
"""
import random

import numpy as np
import pytest

from llmhost_b200.state import EngineError, KvState, TreeError, linear_tree, validate_accept_path, validate_tree
from oracle.kvstate_model import Model, ModelError, TreeErr

NONE = 0xFFFFFFFF


# ---- tree.rs:132-181 ---------------------------------------------------------------
def test_linear_chain_is_valid():
    tree = linear_tree(4)
    assert tree == [-1, 0, 1, 2]
    validate_tree(tree)


def test_branching_tree_parents_precede_children():
    tree = [-1, 0, 0, 1]
    validate_tree(tree)
    validate_accept_path(tree, [0, 1, 3])
    validate_accept_path(tree, [0, 2])
    with pytest.raises(TreeError):
        validate_accept_path(tree, [0, 3])


def test_parent_must_precede_child():
    with pytest.raises(TreeError) as e:
        validate_tree([-1, 2, 0])
    assert e.value.key() == ("ParentDoesNotPrecede", 1, 2)
    with pytest.raises(TreeError) as e:
        validate_tree([0])
    assert e.value.key() == ("ParentDoesNotPrecede", 0, 0)
    with pytest.raises(TreeError) as e:
        validate_tree([-1, -3])
    assert e.value.key() == ("ParentOutOfRange", 1, -3)
    with pytest.raises(TreeError) as e:
        validate_tree([-1, 0], tokens=3)
    assert e.value.key() == ("LengthMismatch", 2, 3)


def test_duplicate_accept_index_is_reported_like_reference():
    with pytest.raises(TreeError) as e:
        validate_accept_path([-1, 0, 1], [0, 1, 1])
    assert e.value.key() == ("ParentDoesNotPrecede", 1, -2)


# ---- cache.rs:139-151 ----------------------------------------------------------------
def test_paged_kv_uses_16_token_blocks():
    st = KvState(64, 1)
    st.open(1)
    assert st.allocated_blocks(1) == 0
    st.append(1, 1)
    assert st.allocated_blocks(1) == 1
    st.append(1, 15)
    assert st.allocated_blocks(1) == 1
    st.forward(1, [7], None)
    st.accept(1, [0])
    assert st.token_count(1) == 17 and st.allocated_blocks(1) == 2
    free_before = len(st.free_list())
    st.forward(1, [8])
    st.accept(1, [])  # nothing accepted: back to 17 tokens
    assert st.token_count(1) == 17
    assert len(st.free_list()) == free_before


# ---- batch.rs:311-414 --------------------------------------------------------------------
def test_forward_returns_logits_for_every_token():
    st = KvState(64, 6)
    st.open(1)
    a = st.forward(1, [10, 11, 12])
    b = st.forward(2, [20])  # an unknown sequence is opened by forward
    assert len(a.logits) == 3 and len(b.logits) == 1
    assert a.logits[2] == [12.0]


def test_accept_non_prefix_path_updates_kv():
    st = KvState(64, 6)
    st.open(7)
    st.forward(7, [100, 101, 102, 103], [-1, 0, 0, 1])
    assert st.committed(7) == []
    moves = st.accept(7, [0, 1, 3])
    assert st.committed(7) == [100, 101, 103]
    assert st.token_count(7) == 3 and st.allocated_blocks(7) == 1
    assert moves == [(3, 2)]  # token 3 moves from slot 3 to slot 2


def test_rollback_drops_rejected_indices():
    st = KvState(64, 6)
    st.open(3)
    st.forward(3, [1, 2, 3, 4])
    st.rollback(3, [2, 3])
    assert st.committed(3) == [1, 2]
    assert st.token_count(3) == 2


def test_reject_accept_that_is_not_a_path():
    st = KvState(64, 6)
    st.open(4)
    st.forward(4, [1, 2, 3], [-1, 0, 0])
    with pytest.raises(EngineError) as e:
        st.accept(4, [2])
    assert e.value.kind == "InvalidAccept" and e.value.seq_id == 4
    st.open(5)
    st.forward(5, [1, 2, 3])
    with pytest.raises(EngineError):
        st.accept(5, [0, 2])


def test_invalid_tree_fails_forward():
    st = KvState(64, 6)
    with pytest.raises(EngineError) as e:
        st.forward(1, [1, 2], [-1, 2])
    assert e.value.kind == "Tree"


def test_accept_without_forward_and_unknown_sequence():
    st = KvState(64, 2)
    with pytest.raises(EngineError) as e:
        st.accept(9, [0])
    assert e.value.kind == "UnknownSeq"
    st.open(9)
    with pytest.raises(EngineError) as e:
        st.accept(9, [0])
    assert e.value.kind == "NoPendingForward"


# ---- build-defined page rules --------------------------------------------------------------
def test_allocation_follows_the_given_order_and_reuses_lifo():
    order = [5, 3, 9, 1, 7, 0, 2, 4, 6, 8]
    st = KvState(10, 2, alloc_order=order)
    st.open(1)
    st.append(1, 17)  # 2 pages per layer: layer 0 then layer 1
    assert st.table(1, 0) == [5, 3] and st.table(1, 1) == [9, 1]
    st.close(1)  # layer 0 then layer 1, in table order -> 1 is on top
    assert st.free_list()[:4] == [1, 9, 3, 5]


def test_fork_shares_pages_and_copies_the_partial_tail_on_write():
    st = KvState(32, 2)
    st.open(1)
    st.append(1, 20)  # pages: layer0 [0,1], layer1 [2,3]; tail page half full
    st.fork(1, 2)
    assert st.refcount(1) == 2 and st.refcount(3) == 2
    cow = st.append(2, 1)
    assert cow == [(1, 4), (3, 5)]  # the shared tail pages are copied, once per layer
    assert st.table(2, 0) == [0, 4] and st.table(1, 0) == [0, 1]
    assert st.refcount(0) == 2 and st.refcount(1) == 1


def test_speculative_draft_never_writes_committed_pages():
    st = KvState(64, 1)
    st.open(1)
    st.append(1, 5)  # one page, partly filled
    plan = st.forward(1, [1, 2, 3], [-1, 0, 0])
    assert plan.cow == [(0, 1)]  # the draft copies the shared tail before writing
    assert list(plan.slots) == [5, 6, 7] and list(plan.positions) == [5, 6, 6]
    moves = st.accept(1, [0, 2])
    assert moves == [(7, 6)]
    assert st.table(1, 0) == [1] and st.refcount(0) == 0


def test_evict_window_and_compact():
    st = KvState(64, 1)
    st.open(1)
    st.append(1, 100)  # 7 pages: 0..6
    freed = st.evict_window(1, 40)  # window [60, 100): pages 0..2 wholly below
    assert freed == 3 and st.table(1, 0)[:4] == [NONE, NONE, NONE, 3]
    moves = st.compact()  # used: 3,4,5,6 -> move 4,5,6? no: U = 4, holes 0,1,2 <- movers 4,5,6
    assert moves == [(4, 0), (5, 1), (6, 2)]
    assert st.table(1, 0) == [NONE, NONE, NONE, 3, 0, 1, 2]
    assert st.free_list()[:3] == [4, 5, 6]


def test_oom_changes_nothing():
    st = KvState(3, 2)
    st.open(1)
    before = st.free_list()
    with pytest.raises(Exception):
        st.append(1, 40)  # needs 3 pages per layer
    assert st.free_list() == before and st.token_count(1) == 0


# ---- differential: library vs model ----------------------------------------------------------
def _snapshot(st, model, seqs, L):
    assert st.free_list() == model.free_list()
    for p in range(model.n_pages):
        assert st.refcount(p) == model.ref[p], p
    for s in seqs:
        if s not in model.sess:
            continue
        assert st.token_count(s) == model.sess[s]["n"]
        assert st.committed(s) == model.sess[s]["committed"]
        for layer in range(L):
            assert st.table(s, layer) == model.table(s, layer)
            if model.sess[s]["pending"]:
                assert st.table(s, layer, draft=True) == model.table(s, layer, draft=True)


def _rand_tree(rng, n):
    return [-1] + [rng.randrange(0, i) for i in range(1, n)]


def _rand_path(rng, tree):
    # a root-to-node path, sometimes with a missing parent (invalid)
    n = len(tree)
    node = rng.randrange(n)
    path = []
    while node != -1:
        path.append(node)
        node = tree[node]
    path = sorted(path)
    if rng.random() < 0.1 and len(path) > 1:
        path.pop(0)
    if rng.random() < 0.05:
        path = path + path[-1:]
    return path


@pytest.mark.parametrize("seed", range(12))
def test_library_matches_model(seed):
    rng = random.Random(seed)
    n_pages, L = rng.choice([40, 97, 300]), rng.choice([1, 2, 6])
    order = list(range(n_pages))
    rng.shuffle(order)
    st = KvState(n_pages, L, alloc_order=order)
    model = Model(n_pages, L, order=order)
    seqs = list(range(1, 6))
    for step in range(250):
        op = rng.choice(["open", "append", "forward", "accept", "rollback", "fork", "evict", "compact", "close"])
        s = rng.choice(seqs)
        got = exp = None
        try:
            if op == "open":
                exp = model.open(s)
            elif op == "append":
                n = rng.randrange(0, 40)
                exp = model.append(s, n, list(range(n)))
            elif op == "forward":
                n = rng.randrange(1, 20)
                tree = _rand_tree(rng, n) if rng.random() < 0.7 else None
                if tree is not None and rng.random() < 0.05:
                    tree[-1] = n + 3  # invalid
                exp = model.forward(s, list(range(1000, 1000 + n)), tree)
            elif op in ("accept", "rollback"):
                d = model.sess.get(s, {}).get("pending") if s in model.sess else None
                if op == "accept":
                    idx = _rand_path(rng, d["tree"]) if d else [0]
                    exp = model.accept(s, idx)
                else:
                    pop = len(d["tokens"]) if d else 1
                    idx = rng.sample(range(pop), k=min(pop, rng.randrange(0, 3))) if d else []
                    exp = model.rollback(s, idx)
            elif op == "fork":
                dst = rng.choice(seqs)
                exp = model.fork(s, dst)
            elif op == "evict":
                w = rng.randrange(1, 60)
                exp = model.evict_window(s, w)
            elif op == "compact":
                exp = model.compact()
            elif op == "close":
                exp = model.close(s)
        except (ModelError, TreeErr) as e:
            exp = ("error", type(e).__name__, getattr(e, "kind", None))
        try:
            if op == "open":
                got = st.open(s)
            elif op == "append":
                got = st.append(s, n, list(range(n)))
            elif op == "forward":
                p = st.forward(s, list(range(1000, 1000 + n)), tree)
                got = (p.slots.tolist(), p.positions.tolist(), p.cow)
            elif op == "accept":
                got = st.accept(s, idx)
            elif op == "rollback":
                got = st.rollback(s, idx)
            elif op == "fork":
                got = st.fork(s, dst)
            elif op == "evict":
                got = st.evict_window(s, w)
            elif op == "compact":
                got = st.compact()
            elif op == "close":
                got = st.close(s) if s in model.sess or True else None
        except EngineError as e:
            got = ("error", e.kind)
        except Exception as e:  # KvError from _capi.check (Invalid / Oom)
            got = ("error", type(e).__name__, getattr(e, "status", None))
        if isinstance(exp, tuple) and exp and exp[0] == "error":
            assert isinstance(got, tuple) and got[0] == "error", (step, op, exp, got)
        elif op == "close":
            pass
        else:
            if op == "forward":
                exp = (exp[0], exp[1], exp[2])
            assert got == exp, (step, op, s, got, exp)
        _snapshot(st, model, seqs, L)


def test_export_tables_pads_with_none():
    st = KvState(64, 2)
    st.open(1)
    st.open(2)
    st.append(1, 40)
    st.append(2, 5)
    rows = st.export_tables([1, 2], layer=1, stride=4)
    assert rows.shape == (2, 4)
    assert rows[0].tolist()[:3] == st.table(1, 1) and rows[0, 3] == NONE
    assert rows[1].tolist() == st.table(2, 1) + [NONE] * 3
    assert np.all(rows[1, 1:] == NONE)


# ---- tree-verify masks for kv_prefill_attn ----------------------------------------------------
def test_tree_masks_are_ancestor_or_self_sets():
    from llmhost_b200.kv import tree_masks

    rng = random.Random(7)
    for n in (1, 2, 17, 64):
        tree = _rand_tree(rng, n)
        m = tree_masks(tree).view(np.uint64)
        for i in range(n):
            anc, node = set(), i
            while node != -1:
                anc.add(node)
                node = tree[node]
            assert {j for j in range(n) if (int(m[i]) >> j) & 1} == anc
    with pytest.raises(ValueError):
        tree_masks([-1] * 65)
    with pytest.raises(ValueError):
        tree_masks([-1, 1])
