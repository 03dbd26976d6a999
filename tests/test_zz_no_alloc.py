"""The allocation-free decode entry point, kv_decode_attn_noalloc.

It exists for callers that cannot call cudaMalloc (all their device memory
comes from an arena they manage, so they cannot create a kv_pool): they pass
every buffer, and the kernel's scratch lives in a fixed array inside the
library.  This file is collected last on purpose, so that a run stopping at
the first failure has already run every other test.  It checks, through the
C ABI, two calls in a row against the CPU oracle and against kv_decode_attn
on the same pages.  Both dtypes run the CUDA-core decode kernel here, so the
cases cover its sliding window (with the pages below it evicted) and the
KV-head-shard layouts as well as the full 8-KV-head ones.
"""
import numpy as np
import pytest

from paged_case import DecodeCase, assert_close_rows, to_numpy_f32, to_torch

pytestmark = pytest.mark.gpu

RTOL = {"f32": 1e-5, "bf16": 2e-2}


def rope_table(max_positions: int, theta: float = 1e6, dim: int = 64) -> np.ndarray:
    """(cos, sin) per position and frequency, the table kv_pool_create builds."""
    from oracle import oracle as O

    inv = O.inv_freq(dim, theta)
    c, s = O.cos_sin(inv, 0, max_positions, dim)  # [positions, dim], both halves equal
    return np.ascontiguousarray(np.stack([c[:, : dim // 2], s[:, : dim // 2]], axis=-1))


@pytest.mark.parametrize("dtype,n_q,n_kv,lens,window", [
    ("bf16", 24, 8, [0, 5, 17, 300, 2047, 4500], 0),
    ("f32", 32, 8, [1, 64, 1000], 0),
    ("bf16", 24, 8, [5000, 40, 1030, 2047], 1024),
    ("f32", 32, 8, [3000, 600], 512),
    ("bf16", 8, 2, [3000, 70, 0, 900], 0),
    ("bf16", 16, 4, [1500, 33, 4100], 700),
    ("f32", 4, 1, [2500, 16], 0),
])
def test_noalloc_matches_oracle_and_pool_entry_point(cuda, dtype, n_q, n_kv, lens, window):
    import torch
    from llmhost_b200 import _capi

    case = DecodeCase(dtype, n_q, n_kv, lens, seed=31, window=window, evict_below_window=window > 0)
    _, oracle_out = case.run_oracle()
    lib = _capi.lib()
    with case.make_pool() as pool:
        case.prefill_gpu(pool)
        ref = case.decode_gpu(pool)          # the pool entry point, kv_decode_attn
        assert pool.last_error() == 0
        ref_np = to_numpy_f32(ref)

        max_pos = pool.max_positions
        tab = torch.from_numpy(rope_table(max_pos)).to(cuda)
        q = to_torch(case.q, dtype, cuda)
        bt = torch.from_numpy(case.bt_attn.view(np.int32)).to(cuda)
        lens_d = torch.from_numpy(case.seq_lens).to(cuda)
        status = torch.full((1,), -1, dtype=torch.int32, device=cuda)
        code = _capi.KV_DTYPE_BF16 if dtype == "bf16" else _capi.KV_DTYPE_F32
        stream = torch.cuda.current_stream().cuda_stream
        for call in range(2):  # two calls in a row share the library's scratch
            out = torch.full_like(q, float("nan"))
            rc = lib.kv_decode_attn_noalloc(
                _capi.lib().kv_pool_pages(pool.handle), case.n_pages, code, n_q, n_kv, tab.data_ptr(),
                max_pos, q.data_ptr(), bt.data_ptr(), bt.shape[1], lens_d.data_ptr(), len(case.lens),
                case.window, out.data_ptr(), status.data_ptr(), stream)
            assert rc == 0, _capi.STATUS.get(rc, rc)
            torch.cuda.synchronize()
            assert int(status.item()) == 0, f"call {call}: device error bits {int(status.item())}"
            got = to_numpy_f32(out)
            assert_close_rows(got, oracle_out, RTOL[dtype], f"{dtype} no-alloc call {call} vs the oracle")
            assert_close_rows(got, ref_np, RTOL[dtype], f"{dtype} no-alloc call {call} vs kv_decode_attn")


def test_noalloc_rejects_sizes_beyond_its_limit(cuda):
    import torch
    from llmhost_b200 import _capi

    lib = _capi.lib()
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    dummy = torch.zeros(16, dtype=torch.int32, device=cuda)
    p = dummy.data_ptr()
    # 1025 sequences: more than the static scratch is sized for
    rc = lib.kv_decode_attn_noalloc(p, 1, 1, 24, 8, p, 16, p, p, 1, p, 1025, 0, p, status.data_ptr(), None)
    assert rc == 1
    # 64 query heads: above the 32-head limit
    rc = lib.kv_decode_attn_noalloc(p, 1, 1, 64, 8, p, 16, p, p, 1, p, 4, 0, p, status.data_ptr(), None)
    assert rc == 1
