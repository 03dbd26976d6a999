"""Quantised pools (KV_DTYPE_Q8, KV_DTYPE_K8V4) on the GPU against the oracle.

The reference tags these KvDtype variants (crates/llm-quant/src/formats.rs:
59-68) and quantises with BlockQ8_0 / BlockQ4 (crates/llm-quant/src/lib.rs:
14-101).  The append kernel must store the oracle's codes and f16 scales bit
for bit (K rotated in fp32, then quantised); decode attention over the
dequantised pages must match the oracle's fp32 attention on the same pages
within the bf16 tolerance, normwise per (sequence, query head) row.
"""
import numpy as np
import pytest

from paged_case import DecodeCase, assert_close_rows, to_numpy_f32, to_torch

pytestmark = pytest.mark.gpu
RTOL = 2e-2
STORES = ["q8", "k8v4"]


def run_case(case: DecodeCase, fused: bool = False, repeat: int = 1):
    host, ref = case.run_oracle()
    with case.make_pool() as pool:
        case.prefill_gpu(pool)
        out = case.decode_gpu(pool, fused=fused, repeat=repeat)
        err = pool.last_error()
        ids = case.used_pages()
        gpu_pages = pool.read_pages(ids)
    assert err == 0, f"device error word {err}"
    np.testing.assert_array_equal(gpu_pages, host.data[ids], err_msg="stored codes / scales differ from the oracle")
    return to_numpy_f32(out), ref


@pytest.mark.parametrize("store", STORES)
def test_quant_ragged_lengths(cuda, store):
    case = DecodeCase("bf16", 24, 8, [0, 1, 14, 15, 16, 17, 31, 100, 1000, 2999], seed=31, store=store)
    out, ref = run_case(case, repeat=2)
    assert_close_rows(out, ref, RTOL, f"{store} ragged")


@pytest.mark.parametrize("store", STORES)
@pytest.mark.parametrize("n_q,n_kv", [(4, 1), (8, 2), (16, 4), (32, 8), (24, 8)])
def test_quant_head_shapes(cuda, store, n_q, n_kv):
    # the tensor-core kernel's head layouts: group 3 and 4 at 8 kv heads and
    # the KV-head shards (1, 2, 4 kv heads) of a head-sharded session
    case = DecodeCase("bf16", n_q, n_kv, [3, 333, 2048, 47], seed=n_q * 10 + n_kv, store=store)
    out, ref = run_case(case)
    assert_close_rows(out, ref, RTOL, f"{store} {n_q}q/{n_kv}kv")


@pytest.mark.parametrize("store", STORES)
def test_quant_fused_append_decode_attn(cuda, store):
    # kv_append_decode_attn on a quantised pool: the append and the attention
    # as two launches, the same result as the separate calls
    case = DecodeCase("bf16", 24, 8, [5, 70, 4097], seed=41, store=store)
    out, ref = run_case(case, fused=True)
    assert_close_rows(out, ref, RTOL, f"{store} fused")


@pytest.mark.parametrize("store", STORES)
def test_quant_window_with_evicted_pages(cuda, store):
    # sliding window: pages wholly below the window are KV_PAGE_NONE in the
    # attention's block tables and must never be read
    case = DecodeCase("bf16", 24, 8, [10, 100, 511, 512, 513, 3000], seed=43, window=500,
                      evict_below_window=True, store=store)
    out, ref = run_case(case)
    assert_close_rows(out, ref, RTOL, f"{store} window")


@pytest.mark.parametrize("store", STORES)
def test_quant_long_single_head(cuda, store):
    # the long-context shard shape: one KV head, 40k keys in 16 splits
    case = DecodeCase("bf16", 4, 1, [40000], seed=47, store=store)
    out, ref = run_case(case)
    assert_close_rows(out, ref, RTOL, f"{store} 40k")


NORM_CASES = {
    "ragged": dict(n_q=24, n_kv=8, lens=[0, 1, 17, 300, 2999], seed=71),
    "group4": dict(n_q=32, n_kv=8, lens=[5, 700, 4097, 63], seed=72),
    "one kv head, long": dict(n_q=4, n_kv=1, lens=[20001], seed=73),
    "window, evicted": dict(n_q=24, n_kv=8, lens=[5000, 40, 1030], seed=74, window=1024, evict_below_window=True),
}


@pytest.mark.parametrize("store", STORES)
@pytest.mark.parametrize("name", list(NORM_CASES))
def test_quant_norm_decode_against_oracle(cuda, store, name):
    # kv_norm_append_decode_attn on a quantised pool: k normalised (sum of
    # squares in double), rotated and quantised by the append launch, q
    # normalised in the attention launch; codes and scales bit-exact
    c = dict(NORM_CASES[name])
    case = DecodeCase("bf16", c.pop("n_q"), c.pop("n_kv"), c.pop("lens"), store=store, **c)
    rng = np.random.default_rng(8)
    norm = (rng.uniform(0.5, 1.5, 64).astype(np.float32), rng.uniform(0.5, 1.5, 64).astype(np.float32), 1e-5)
    host, ref = case.run_oracle(norm=norm)
    with case.make_pool() as pool:
        case.prefill_gpu(pool)
        out = to_numpy_f32(case.decode_norm_gpu(pool, norm))
        assert pool.last_error() == 0
        ids = case.used_pages()
        pages = pool.read_pages(ids)
    np.testing.assert_array_equal(pages, host.data[ids], err_msg="stored codes / scales differ from the oracle")
    assert_close_rows(out, ref, RTOL, f"{store} norm {name}")


@pytest.mark.parametrize("store", STORES)
def test_quant_shared_prefill_refused(cuda, store):
    import torch
    from llmhost_b200 import _capi

    case = DecodeCase("bf16", 24, 8, [20], seed=1, store=store)
    with case.make_pool() as pool:
        dev = pool.device
        q = to_torch(case.q, "bf16", dev)
        k = to_torch(case.k_new, "bf16", dev)
        v = to_torch(case.v_new, "bf16", dev)
        bt = torch.from_numpy(case.bt.view(np.int32)).to(dev)
        lens = torch.from_numpy(case.seq_lens).to(dev)
        del k, v, lens
        qp = torch.zeros(1, dtype=torch.int32, device=dev)
        off = torch.tensor([0, 1], dtype=torch.int32, device=dev)
        sixteen = torch.full((1,), 16, dtype=torch.int32, device=dev)
        with pytest.raises(_capi.KvError) as e:
            pool.prefill_attn_shared(q[:1].contiguous(), qp, off, sixteen, bt, shared_tokens=16, max_q=1)
        assert e.value.status == 6  # KV_ERR_UNSUPPORTED
        assert pool.last_error() == 0


@pytest.mark.parametrize("store", STORES)
def test_quant_prefill_causal_chunks(cuda, store):
    # chunked prefill on a quantised pool: the CUDA-core kernel on the
    # dequantised keys and values; pages bit-exact, outputs within 2e-2
    import test_gpu_prefill as tp

    case = tp.PrefillCase(24, 8, [(0, 40), (100, 17), (300, 64), (31, 1)], seed=61, store=store)
    tp.check(case, f"{store} causal chunks")


@pytest.mark.parametrize("store", STORES)
def test_quant_tree_verify(cuda, store):
    import test_gpu_prefill as tp

    rng = np.random.default_rng(62)
    trees = [[-1] + [int(rng.integers(0, i)) for i in range(1, n)] for n in (1, 5, 64, 33)]
    case = tp.PrefillCase(32, 8, [(int(rng.integers(0, 700)), t) for t in trees], seed=63, store=store)
    tp.check(case, f"{store} tree verify")


@pytest.mark.parametrize("store", STORES)
def test_quant_group_without_kernel_is_refused(cuda, store):
    # as for bf16 pools, a head layout with no compiled kernel fails at pool
    # creation, not at the first launch
    from llmhost_b200 import _capi
    from llmhost_b200.kv import KvPool

    with pytest.raises(_capi.KvError) as e:
        KvPool(dtype=store, n_q_heads=8, n_kv_heads=8, n_pages=16, max_positions=64, max_seqs=4)
    assert e.value.status == 6  # KV_ERR_UNSUPPORTED


def test_quant_bad_page_is_flagged(cuda):
    # a block-table entry past the pool: the split that meets it skips the
    # page and sets the error word; the launch still completes
    import torch

    case = DecodeCase("bf16", 8, 2, [40], seed=2, store="q8")
    with case.make_pool() as pool:
        case.prefill_gpu(pool)
        bt = case.bt.copy()
        bt[0, 1] = case.n_pages + 5
        dev = pool.device
        pool.decode_attn(to_torch(case.q, "bf16", dev), torch.from_numpy(bt.view(np.int32)).to(dev),
                         torch.from_numpy(case.lens.astype(np.int32)).to(dev))
        torch.cuda.synchronize()
        assert pool.last_error() == 2  # KV_ERR_BAD_PAGE
