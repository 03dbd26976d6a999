"""The draft-tree builder and the batch scheduler (no GPU).

* The reference's own assertions: schedule.rs:49-66 (running set in insertion
  order, no duplicates, removal) and draft.rs:29-53 (a proposal of three
  tokens with tree [-1, 0, 0] is a valid tree).
* The native best-first tree builder against the workload generator's
  independent Python implementation (llmhost_b200.workloads.draft_tree), on
  the candidates that generator expanded: the same parent arrays.
* The step planner's budget rules and LPT against workloads.lpt_partition.
"""
import numpy as np
import pytest

from llmhost_b200 import _capi
from llmhost_b200.sched import Scheduler, draft_tree_best_first, lpt
from llmhost_b200.state import validate_tree
from llmhost_b200.workloads import draft_tree, lpt_partition


def test_reference_scheduler_kat():  # schedule.rs:49-66
    s = Scheduler()
    s.add(1)
    s.add(2)
    s.add(1)
    assert s.running() == [1, 2]
    batch = s.schedule()
    assert len(batch) == 2 and batch[0] == 1
    s.remove(1)
    assert s.running() == [2]


def test_reference_draft_kat():  # draft.rs:29-53: tokens [10, 11, 12], tree [-1, 0, 0]
    tokens, tree, picked = draft_tree_best_first([-1, 0, 0], [10, 11, 12], [1.0, 0.6, 0.4], max_nodes=8, max_depth=6)
    assert tokens.tolist() == [10, 11, 12] and tree.tolist() == [-1, 0, 0] and picked.tolist() == [0, 1, 2]
    validate_tree(tree.tolist(), len(tokens))


@pytest.mark.parametrize("seed", range(20))
@pytest.mark.parametrize("nodes,depth", [(64, 6), (16, 3), (5, 10)])
def test_best_first_matches_the_workload_generator(seed, nodes, depth):
    rng = np.random.default_rng(seed)
    parents, children = draft_tree(rng, nodes, depth)
    # the generator expands each node as it adds it, so listing every node's
    # candidate children in node order gives its candidate creation order
    # (the order its heap breaks ties by)
    order = list(range(len(parents)))
    par, prob, node = [-1], [1.0], [0]
    cand_of_node = {0: 0}
    for u in order:
        for p, v in children[u]:
            par.append(cand_of_node[u])
            prob.append(p)
            node.append(v)
            if v >= 0:
                cand_of_node[v] = len(par) - 1
    tokens = np.arange(len(par), dtype=np.uint32) + 1000
    _, tree, picked = draft_tree_best_first(par, tokens, prob, max_nodes=nodes, max_depth=depth)
    assert tree.tolist() == parents
    assert [node[c] for c in picked] == list(range(len(parents)))
    validate_tree(tree.tolist(), len(tree))


def test_best_first_budgets_and_ties():
    # depth limit: a chain of certain candidates stops at max_depth
    par = [-1, 0, 1, 2, 3]
    _, tree, _ = draft_tree_best_first(par, [1, 2, 3, 4, 5], [1.0] * 5, max_nodes=10, max_depth=2)
    assert tree.tolist() == [-1, 0, 1]
    # node budget and ties to the lower candidate index
    _, tree, picked = draft_tree_best_first([-1, 0, 0, 0], [1, 2, 3, 4], [1.0, 0.25, 0.5, 0.25], max_nodes=3,
                                            max_depth=6)
    assert picked.tolist() == [0, 2, 1] and tree.tolist() == [-1, 0, 0]
    # several roots; empty input
    _, tree, picked = draft_tree_best_first([-1, -1, 1], [7, 8, 9], [0.3, 0.7, 0.9], max_nodes=3, max_depth=6)
    assert picked.tolist() == [1, 2, 0] and tree.tolist() == [-1, 0, -1]
    assert draft_tree_best_first([], [], [], 4, 6)[0].size == 0


def test_best_first_rejects_bad_candidates():
    with pytest.raises(_capi.KvError):
        draft_tree_best_first([-1, 1], [1, 2], [1.0, 0.5], 4, 6)  # parent does not precede
    with pytest.raises(_capi.KvError):
        draft_tree_best_first([-1, 0], [1, 2], [1.0, 1.5], 4, 6)  # not a probability


def test_plan_step_budget_rules():
    s = Scheduler()
    for sid in (10, 11, 12, 13):
        s.add(sid)
    s.set_pending(11, 700)
    s.set_pending(13, 100)
    # decode tokens first (10, 12), then prompt chunks in running order
    assert s.plan_step(token_budget=600, chunk_tokens=512) == [(10, 1, False), (12, 1, False), (11, 512, True),
                                                               (13, 86, True)]
    # 11 has 188 left, 13 has 14
    assert s.plan_step(token_budget=100, chunk_tokens=512) == [(10, 1, False), (12, 1, False), (11, 98, True)]
    # 11 has 90 left
    assert s.plan_step(token_budget=1000, chunk_tokens=64) == [(10, 1, False), (12, 1, False), (11, 64, True),
                                                               (13, 14, True)]
    # 13 is done with its prompt: it decodes from now on
    assert s.plan_step(token_budget=1000, chunk_tokens=64) == [(10, 1, False), (12, 1, False), (13, 1, False),
                                                               (11, 26, True)]
    # so is 11; with a budget of 2 the first two in running order decode
    assert s.plan_step(token_budget=2, chunk_tokens=64) == [(10, 1, False), (11, 1, False)]
    assert s.plan_step(token_budget=0, chunk_tokens=64) == []
    with pytest.raises(_capi.KvError):
        s.set_pending(99, 5)  # not running
    s.remove(11)
    assert s.running() == [10, 12, 13]


@pytest.mark.parametrize("seed", range(10))
def test_lpt_matches_python_partition(seed):
    rng = np.random.default_rng(seed)
    w = rng.integers(1, 131072, size=int(rng.integers(1, 300)))
    bins = int(rng.integers(1, 9))
    got = lpt(w, bins)
    want = lpt_partition(w.tolist(), bins)
    for b in range(bins):
        assert sorted(np.nonzero(got == b)[0].tolist()) == want[b]
