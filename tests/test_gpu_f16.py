"""Half-precision pools (KV_DTYPE_F16) on the GPU against the oracle.

F16 is the reference's default KvDtype tag ("full f16 keys and values",
crates/llm-quant/src/formats.rs:59-68; Engine::new(KvDtype::F16) in
crates/llm-engine/src/batch.rs:306).  The pool stores IEEE half in the bf16
page layout and takes bf16 k, v, q and out.  The append must store the
oracle's half bits exactly (K rotated in fp32, then K and V rounded to nearest
even); decode attention runs on the tensor cores with f16 operands, prefill
and tree verify on the CUDA cores, and both must match the oracle's fp32
attention over the same pages within 2e-2 normwise per (sequence or token,
query head) row.
"""
import numpy as np
import pytest

from paged_case import DecodeCase, assert_close_rows, to_numpy_f32, to_torch

pytestmark = pytest.mark.gpu
RTOL = 2e-2


def run_case(case: DecodeCase, fused: bool = False, repeat: int = 1):
    host, ref = case.run_oracle()
    with case.make_pool() as pool:
        case.prefill_gpu(pool)
        out = case.decode_gpu(pool, fused=fused, repeat=repeat)
        err = pool.last_error()
        ids = case.used_pages()
        gpu_pages = pool.read_pages(ids)
    assert err == 0, f"device error word {err}"
    np.testing.assert_array_equal(gpu_pages, host.data[ids], err_msg="stored half bits differ from the oracle")
    return to_numpy_f32(out), ref


def test_f16_ragged_lengths(cuda):
    case = DecodeCase("bf16", 24, 8, [0, 1, 14, 15, 16, 17, 31, 100, 1000, 2999], seed=131, store="f16")
    out, ref = run_case(case, repeat=2)
    assert_close_rows(out, ref, RTOL, "f16 ragged")


@pytest.mark.parametrize("n_q,n_kv", [(4, 1), (8, 2), (16, 4), (32, 8), (24, 8)])
def test_f16_head_shapes(cuda, n_q, n_kv):
    case = DecodeCase("bf16", n_q, n_kv, [3, 333, 2048, 47], seed=100 + n_q * 10 + n_kv, store="f16")
    out, ref = run_case(case)
    assert_close_rows(out, ref, RTOL, f"f16 {n_q}q/{n_kv}kv")


def test_f16_fused_append_decode_attn(cuda):
    # kv_append_decode_attn: the append folded into the attention launch, as
    # for bf16 pools; the stored token's half bits must match the oracle's
    case = DecodeCase("bf16", 24, 8, [5, 70, 4097, 0, 16], seed=141, store="f16")
    out, ref = run_case(case, fused=True)
    assert_close_rows(out, ref, RTOL, "f16 fused")


def test_f16_window_with_evicted_pages(cuda):
    case = DecodeCase("bf16", 24, 8, [10, 100, 511, 512, 513, 3000], seed=143, window=500,
                      evict_below_window=True, store="f16")
    out, ref = run_case(case)
    assert_close_rows(out, ref, RTOL, "f16 window")


def test_f16_long_single_head(cuda):
    case = DecodeCase("bf16", 4, 1, [40000], seed=147, store="f16")
    out, ref = run_case(case)
    assert_close_rows(out, ref, RTOL, "f16 40k")


@pytest.mark.parametrize("n_q,n_kv,lens", [(24, 8, [0, 1, 17, 300, 2999]), (4, 1, [20001])])
def test_f16_norm_decode_against_oracle(cuda, n_q, n_kv, lens):
    # kv_norm_append_decode_attn: q and the new k RMS-normalised in the same
    # launch; the stored K half bits exact
    case = DecodeCase("bf16", n_q, n_kv, lens, seed=171 + n_kv, store="f16")
    rng = np.random.default_rng(18)
    norm = (rng.uniform(0.5, 1.5, 64).astype(np.float32), rng.uniform(0.5, 1.5, 64).astype(np.float32), 1e-5)
    host, ref = case.run_oracle(norm=norm)
    with case.make_pool() as pool:
        case.prefill_gpu(pool)
        out = to_numpy_f32(case.decode_norm_gpu(pool, norm))
        assert pool.last_error() == 0
        ids = case.used_pages()
        pages = pool.read_pages(ids)
    np.testing.assert_array_equal(pages, host.data[ids], err_msg="stored half bits differ from the oracle")
    assert_close_rows(out, ref, RTOL, f"f16 norm {n_q}q/{n_kv}kv")


def test_f16_prefill_causal_chunks(cuda):
    import test_gpu_prefill as tp

    case = tp.PrefillCase(24, 8, [(0, 40), (100, 17), (300, 64), (31, 1)], seed=161, store="f16")
    tp.check(case, "f16 causal chunks")


def test_f16_tree_verify(cuda):
    import test_gpu_prefill as tp

    rng = np.random.default_rng(162)
    trees = [[-1] + [int(rng.integers(0, i)) for i in range(1, n)] for n in (1, 5, 64, 33)]
    case = tp.PrefillCase(32, 8, [(int(rng.integers(0, 700)), t) for t in trees], seed=163, store="f16")
    tp.check(case, "f16 tree verify")


def test_f16_shared_prefill_refused(cuda):
    import torch
    from llmhost_b200 import _capi

    case = DecodeCase("bf16", 24, 8, [20], seed=1, store="f16")
    with case.make_pool() as pool:
        dev = pool.device
        q = to_torch(case.q, "bf16", dev)
        bt = torch.from_numpy(case.bt.view(np.int32)).to(dev)
        qp = torch.zeros(1, dtype=torch.int32, device=dev)
        off = torch.tensor([0, 1], dtype=torch.int32, device=dev)
        sixteen = torch.full((1,), 16, dtype=torch.int32, device=dev)
        with pytest.raises(_capi.KvError) as e:
            pool.prefill_attn_shared(q[:1].contiguous(), qp, off, sixteen, bt, shared_tokens=16, max_q=1)
        assert e.value.status == 6  # KV_ERR_UNSUPPORTED
        assert pool.last_error() == 0
