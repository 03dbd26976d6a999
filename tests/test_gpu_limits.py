"""The max_seqs limit of a pool (kv_pool_config.max_seqs in include/llmhost_kv.h).

The tensor-core decode kernel keeps a call's per-sequence table in shared
memory beside its tile rings, so kv_pool_create refuses a max_seqs whose table
would not fit (KV_ERR_INVALID) rather than fail at the first launch.  The
header states the limits on a B200 (227 KiB of shared memory per block); here
each is checked at the boundary, and a decode call that uses the whole table
is checked against the oracle.
"""
import numpy as np
import pytest

from paged_case import DecodeCase, assert_close_rows, to_numpy_f32

pytestmark = pytest.mark.gpu

# (dtype, q heads, kv heads) -> largest max_seqs kv_pool_create accepts
LIMITS = {
    ("bf16", 24, 8): 2219,
    ("bf16", 32, 8): 1875,
    ("q8", 24, 8): 1195,
    ("q8", 32, 8): 851,
    ("k8v4", 24, 8): 5291,
    ("k8v4", 32, 8): 4947,
}


@pytest.mark.parametrize("key", list(LIMITS), ids=lambda k: f"{k[0]}-{k[1]}q{k[2]}kv")
def test_max_seqs_boundary(cuda, key):
    from llmhost_b200 import _capi
    from llmhost_b200.kv import KvPool

    dtype, n_q, n_kv = key
    limit = LIMITS[key]
    pool = KvPool(dtype=dtype, n_q_heads=n_q, n_kv_heads=n_kv, n_pages=16, max_positions=64, max_seqs=limit)
    pool.close()
    with pytest.raises(_capi.KvError) as e:
        KvPool(dtype=dtype, n_q_heads=n_q, n_kv_heads=n_kv, n_pages=16, max_positions=64, max_seqs=limit + 1)
    assert e.value.status == 1  # KV_ERR_INVALID


@pytest.mark.parametrize("store", ["bf16", "q8"])
def test_decode_with_a_full_sequence_table(cuda, store):
    # as many sequences as the pool allows, short and ragged (some empty), so
    # that every entry of the shared-memory table is used
    limit = LIMITS[(store, 24, 8)]
    rng = np.random.default_rng(17)
    lens = [int(x) for x in rng.integers(0, 40, limit)]
    case = DecodeCase("bf16", 24, 8, lens, seed=17, store=store)
    host, ref = case.run_oracle()
    with case.make_pool() as pool:
        assert pool.max_seqs == limit
        case.prefill_gpu(pool)
        out = to_numpy_f32(case.decode_gpu(pool))
        assert pool.last_error() == 0
        ids = case.used_pages()
        pages = pool.read_pages(ids)
    np.testing.assert_array_equal(pages, host.data[ids], err_msg="stored pages differ from the oracle")
    assert_close_rows(out, ref, 2e-2, f"{store}, {limit} sequences")
