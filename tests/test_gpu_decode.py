"""Parity of the CUDA append + paged decode attention against the CPU oracle.

Tolerances: attention outputs within 1e-5 relative for
fp32 and 2e-2 for bf16, checked normwise per (sequence, query head) row;
stored pages bit-exact (RoPE'd K uses the same libm cos/sin as the reference).
"""
import numpy as np
import pytest

from paged_case import DecodeCase, assert_close_rows, to_numpy_f32, to_torch

pytestmark = pytest.mark.gpu

RTOL = {"f32": 1e-5, "bf16": 2e-2}


def run_case(case: DecodeCase, repeat: int = 1, fused: bool = False):
    host, ref = case.run_oracle()
    with case.make_pool() as pool:
        case.prefill_gpu(pool)
        out = case.decode_gpu(pool, repeat=repeat, fused=fused)
        err = pool.last_error()
        ids = case.used_pages()
        gpu_pages = pool.read_pages(ids)
    assert err == 0, f"device error word {err}"
    np.testing.assert_array_equal(gpu_pages, host.data[ids], err_msg="stored pages differ from the oracle")
    return to_numpy_f32(out), ref


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_decode_ragged_lengths(cuda, dtype):
    case = DecodeCase(dtype, 24, 8, [0, 1, 14, 15, 16, 17, 31, 100, 1000, 2999], seed=3)
    out, ref = run_case(case)
    assert_close_rows(out, ref, RTOL[dtype], f"{dtype} ragged")


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_decode_group4(cuda, dtype):
    case = DecodeCase(dtype, 32, 8, [5, 700, 4097, 63], seed=4)
    out, ref = run_case(case)
    assert_close_rows(out, ref, RTOL[dtype], f"{dtype} 32q/8kv")


@pytest.mark.parametrize("dtype,length", [("bf16", 40000), ("f32", 12000)])
def test_decode_single_kv_head_long(cuda, dtype, length):
    # One KV head with 4 query heads (the per-GPU shard of the long-context
    # session): one sequence split over every CTA of the grid.
    case = DecodeCase(dtype, 4, 1, [length], seed=5)
    out, ref = run_case(case)
    assert_close_rows(out, ref, RTOL[dtype], f"{dtype} 4q/1kv long")


def test_decode_f32_long_against_exact(cuda):
    # At 40k keys the oracle's own sequential fp32 sums drift by ~1e-5
    # (lfm2.rs:1044-1054 accumulates in key order), so this case is judged
    # against float64 arithmetic on the same stored pages: the kernel must be
    # within 1e-5 of exact and no further from it than the oracle is (x1.5).
    from paged_case import truth_decode

    case = DecodeCase("f32", 4, 1, [40000], seed=5)
    host, ref = case.run_oracle()
    with case.make_pool() as pool:
        case.prefill_gpu(pool)
        out = to_numpy_f32(case.decode_gpu(pool))
        assert pool.last_error() == 0
    exact = truth_decode(host, case.bt_attn, case.seq_lens, case.window, case.q, "f32")
    from oracle import oracle as O

    e_gpu = O.rel_err_rows(out, exact).max()
    e_orc = O.rel_err_rows(ref, exact).max()
    assert e_gpu <= 1e-5, e_gpu
    assert e_gpu <= 1.5 * e_orc + 1e-7, (e_gpu, e_orc)


def test_decode_one_long_sequence_many_splits(cuda):
    case = DecodeCase("bf16", 24, 8, [60000], seed=6)
    out, ref = run_case(case, repeat=3)  # repeated calls: split counters reset
    assert_close_rows(out, ref, RTOL["bf16"], "bf16 one long sequence")


def test_decode_many_short_sequences(cuda):
    rng = np.random.default_rng(7)
    lens = rng.integers(0, 200, size=700)
    case = DecodeCase("bf16", 24, 8, lens, seed=7)
    out, ref = run_case(case)
    assert_close_rows(out, ref, RTOL["bf16"], "bf16 700 short sequences")


def test_decode_config_shaped_batch(cuda):
    # 64 sequences with lengths drawn like the batched-decode configuration
    # (uniform in [128, 8192]), scaled down 4x to keep the oracle quick.
    rng = np.random.default_rng(1)
    lens = rng.integers(128, 2048, endpoint=True, size=64)
    case = DecodeCase("bf16", 24, 8, lens, seed=8)
    out, ref = run_case(case)
    assert_close_rows(out, ref, RTOL["bf16"], "bf16 config-shaped")


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_decode_sliding_window_evicted_pages(cuda, dtype):
    # Pages wholly below the window are marked evicted (KV_PAGE_NONE): the
    # kernel must not read them (a read would set the bad-page error bit).
    case = DecodeCase(dtype, 24, 8, [5000, 40, 1030, 2047], seed=9, window=1024, evict_below_window=True)
    out, ref = run_case(case)
    assert_close_rows(out, ref, RTOL[dtype], f"{dtype} window")


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("lens", [[1, 64, 1000], [70], [0, 3, 9, 200]])
def test_decode_fewer_pages_than_ctas(cuda, dtype, lens):
    # Fewer pages than CTAs in the persistent grid: some CTA slices are empty
    # and a split sequence has one contributor per page.
    case = DecodeCase(dtype, 24, 8, lens, seed=12)
    out, ref = run_case(case, repeat=2)
    assert_close_rows(out, ref, RTOL[dtype], f"{dtype} sparse {lens}")


def test_zero_sequences_is_a_noop(cuda):
    import torch

    case = DecodeCase("bf16", 24, 8, [10], seed=10)
    with case.make_pool() as pool:
        empty_i = torch.zeros((0, 1), dtype=torch.int32, device=cuda)
        q = torch.zeros((0, 24, 64), dtype=torch.bfloat16, device=cuda)
        out = pool.decode_attn(q, empty_i, torch.zeros(0, dtype=torch.int32, device=cuda))
        assert out.shape == (0, 24, 64)
        assert pool.last_error() == 0


def test_bad_page_id_sets_error_word(cuda):
    import torch
    from llmhost_b200._capi import KV_PAGE_NONE

    case = DecodeCase("bf16", 24, 8, [100, 50], seed=11)
    with case.make_pool() as pool:
        case.prefill_gpu(pool)
        bt = case.bt.copy()
        bt[1, 1] = np.uint32(case.n_pages + 5)  # out of range: the kernel's bounds check flags it
        lens = torch.from_numpy(case.seq_lens).to(cuda)
        from paged_case import to_torch

        pool.decode_attn(to_torch(case.q, "bf16", cuda), torch.from_numpy(bt.view(np.int32)).to(cuda), lens)
        assert pool.last_error() == 2  # KV_ERR_BAD_PAGE
        bt[1, 1] = np.uint32(KV_PAGE_NONE)
        pool.decode_attn(to_torch(case.q, "bf16", cuda), torch.from_numpy(bt.view(np.int32)).to(cuda), lens)
        assert pool.last_error() == 2
        # the context stays usable
        assert pool.last_error() == 0


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("n_kv", [2, 4])
def test_decode_kv_head_shards(cuda, dtype, n_kv):
    # the shapes one GPU holds when a 32q/8kv session is split by KV head over 4 or 2 GPUs
    case = DecodeCase(dtype, 4 * n_kv, n_kv, [3, 900, 5000, 17], seed=6 + n_kv)
    out, ref = run_case(case)
    assert_close_rows(out, ref, RTOL[dtype], f"{dtype} {4 * n_kv}q/{n_kv}kv")


def test_pools_of_one_shape_with_different_workspaces(cuda):
    # The decode kernel's shared-memory limit is per device: creating a pool
    # with a smaller workspace must not break launches of an earlier pool.
    big = DecodeCase("bf16", 32, 8, [100, 2000] * 16, seed=21)
    host, ref = big.run_oracle()
    with big.make_pool(max_seqs=64) as p1:
        big.prefill_gpu(p1)
        from llmhost_b200.kv import KvPool

        with KvPool(dtype="bf16", n_q_heads=32, n_kv_heads=8, n_pages=16, max_positions=64, max_seqs=1):
            pass
        out = big.decode_gpu(p1)
        assert p1.last_error() == 0
    assert_close_rows(to_numpy_f32(out), ref, RTOL["bf16"], "first pool after a smaller one")


# ---- fused append + attention (kv_append_decode_attn) -----------------------

FUSED_CASES = {
    "ragged": dict(n_q=24, n_kv=8, lens=[0, 1, 14, 15, 16, 17, 31, 100, 1000, 2999], seed=21),
    "group4": dict(n_q=32, n_kv=8, lens=[5, 700, 4097, 63, 16, 33], seed=22),
    "one kv head, long": dict(n_q=4, n_kv=1, lens=[20001], seed=23),
    "two kv heads": dict(n_q=8, n_kv=2, lens=[1, 900, 3000], seed=24),
    "sparse": dict(n_q=24, n_kv=8, lens=[0, 3, 9, 200], seed=25),
    "window, evicted": dict(n_q=24, n_kv=8, lens=[5000, 40, 1030, 2047], seed=26, window=1024,
                            evict_below_window=True),
}


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("name", list(FUSED_CASES))
def test_fused_append_decode_against_oracle(cuda, dtype, name):
    c = dict(FUSED_CASES[name])
    case = DecodeCase(dtype, c.pop("n_q"), c.pop("n_kv"), c.pop("lens"), **c)
    out, ref = run_case(case, repeat=2, fused=True)  # then a plain decode over the appended pages
    assert_close_rows(out, ref, RTOL[dtype], f"{dtype} fused {name}")


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_fused_is_bit_identical_to_two_launches(cuda, dtype):
    # Same pages and the same output bits as kv_append_decode + kv_decode_attn,
    # including a sequence split over many CTAs and one-token sequences.
    import torch

    rng = np.random.default_rng(27)
    lens = np.concatenate([[1, 16, 17, 30000], rng.integers(1, 3000, size=60)])
    case = DecodeCase(dtype, 24, 8, lens, seed=27)
    outs, pages = [], []
    for fused in (False, True):
        with case.make_pool() as pool:
            case.prefill_gpu(pool)
            out = case.decode_gpu(pool, fused=fused)
            assert pool.last_error() == 0
            outs.append(out.view(torch.int16 if dtype == "bf16" else torch.int32).cpu().numpy())
            pages.append(pool.read_pages(case.used_pages()))
    np.testing.assert_array_equal(pages[1], pages[0])
    np.testing.assert_array_equal(outs[1], outs[0])


def test_fused_bad_position_stores_nothing(cuda):
    # A position past the RoPE table: flagged, and (as kv_append_decode) the
    # token is not stored; the other sequence is appended normally.
    import torch
    from paged_case import to_torch

    case = DecodeCase("bf16", 24, 8, [64, 40], seed=28)  # new tokens at positions 64 and 40
    with case.make_pool(max_positions=64) as pool:
        case.prefill_gpu(pool)
        torch.cuda.synchronize()
        assert pool.last_error() == 0
        ids = list(case.used_pages())
        before = pool.read_pages(ids)
        dev = pool.device
        pool.append_decode_attn(to_torch(case.k_new, "bf16", dev), to_torch(case.v_new, "bf16", dev),
                                to_torch(case.q, "bf16", dev), torch.from_numpy(case.bt.view(np.int32)).to(dev),
                                torch.from_numpy(case.seq_lens).to(dev))
        torch.cuda.synchronize()
        assert pool.last_error() == 7  # KV_ERR_BAD_POS
        after = pool.read_pages(ids)
    a_page = ids.index(int(case.bt[0, 64 // 16]))
    b_page = ids.index(int(case.bt[1, 40 // 16]))
    np.testing.assert_array_equal(after[a_page], before[a_page])  # position 64: nothing stored
    assert not np.array_equal(after[b_page], before[b_page])      # position 40: stored


def test_misaligned_k_is_rejected_before_launch(cuda):
    # k / v rows are read as 16-byte vectors: an unaligned pointer is refused
    # with KV_ERR_INVALID by every append entry point, with no launch.
    import torch
    from llmhost_b200._capi import KvError

    case = DecodeCase("bf16", 24, 8, [10, 20], seed=29)
    with case.make_pool() as pool:
        dev = pool.device
        buf = torch.zeros(2 * 8 * 64 + 1, dtype=torch.bfloat16, device=dev)
        k_bad = buf[1:].view(2, 8, 64)  # 2 bytes past an aligned base
        v = torch.zeros(2, 8, 64, dtype=torch.bfloat16, device=dev)
        q = torch.zeros(2, 24, 64, dtype=torch.bfloat16, device=dev)
        bt = torch.from_numpy(case.bt.view(np.int32)).to(dev)
        lens = torch.from_numpy(case.seq_lens).to(dev)
        for call in (lambda: pool.append_decode(k_bad, v, bt, lens),
                     lambda: pool.append_decode_attn(k_bad, v, q, bt, lens)):
            with pytest.raises(KvError) as e:
                call()
            assert e.value.status == 1  # KV_ERR_INVALID
        assert pool.last_error() == 0


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_empty_sequences_get_zeros(cuda, dtype):
    # seq_lens[s] == 0 (no token at all): the row of out is zeros, whatever it
    # held, and the other sequences are unaffected.
    import torch

    case = DecodeCase(dtype, 24, 8, [300, 40, 2000, 5], seed=32)
    host, ref = case.run_oracle()
    with case.make_pool() as pool:
        case.prefill_gpu(pool)
        case.decode_gpu(pool)  # appends the new tokens (ref covers them)
        dev = pool.device
        lens = case.seq_lens.copy()
        lens[[1, 3]] = 0
        q = to_torch(case.q, dtype, dev)
        out = torch.full_like(q, 7.0)
        pool.decode_attn(q, torch.from_numpy(case.bt_attn.view(np.int32)).to(dev),
                         torch.from_numpy(lens).to(dev), out=out)
        torch.cuda.synchronize()
        assert pool.last_error() == 0
        got = to_numpy_f32(out)
    assert np.all(got[[1, 3]] == 0)
    assert_close_rows(got[[0, 2]], ref[[0, 2]], RTOL[dtype], f"{dtype} rows beside empty ones")


@pytest.mark.parametrize("seed", range(6))
def test_fused_random_batches(cuda, seed):
    # Random batch shapes: sequence ends, CTA cuts and head-pair splits land
    # in different places for every seed.
    rng = np.random.default_rng(100 + seed)
    n = int(rng.integers(1, 90))
    lens = rng.integers(0, int(rng.choice([64, 700, 5000])), size=n)
    n_q, n_kv = [(24, 8), (32, 8), (8, 2), (16, 4), (4, 1)][seed % 5]
    case = DecodeCase("bf16", n_q, n_kv, lens, seed=200 + seed)
    out, ref = run_case(case, fused=True)
    assert_close_rows(out, ref, RTOL["bf16"], f"random batch {seed}")


# ---- q/k RMSNorm folded in (kv_norm_append_decode_attn) ----------------------

NORM_CASES = {
    "ragged": dict(n_q=24, n_kv=8, lens=[0, 1, 17, 300, 2999], seed=41),
    "group4": dict(n_q=32, n_kv=8, lens=[5, 700, 4097, 63], seed=42),
    "one kv head, long": dict(n_q=4, n_kv=1, lens=[20001], seed=43),
    "two kv heads": dict(n_q=8, n_kv=2, lens=[1, 900], seed=44),
    "window, evicted": dict(n_q=24, n_kv=8, lens=[5000, 40, 1030], seed=45, window=1024, evict_below_window=True),
}


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("name", list(NORM_CASES))
def test_norm_fused_decode_against_oracle(cuda, dtype, name):
    # Stored pages hold the normalised, rotated k bit for bit (the scale's sum
    # of squares is in double, as ops.rs:14-18); outputs within tolerance.
    c = dict(NORM_CASES[name])
    case = DecodeCase(dtype, c.pop("n_q"), c.pop("n_kv"), c.pop("lens"), **c)
    rng = np.random.default_rng(7)
    norm = (rng.uniform(0.5, 1.5, 64).astype(np.float32), rng.uniform(0.5, 1.5, 64).astype(np.float32), 1e-5)
    host, ref = case.run_oracle(norm=norm)
    with case.make_pool() as pool:
        case.prefill_gpu(pool)
        out = to_numpy_f32(case.decode_norm_gpu(pool, norm))
        assert pool.last_error() == 0
        ids = case.used_pages()
        pages = pool.read_pages(ids)
    np.testing.assert_array_equal(pages, host.data[ids], err_msg="stored pages differ from the oracle")
    assert_close_rows(out, ref, RTOL[dtype], f"{dtype} norm-fused {name}")


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_back_to_back_fused_steps(cuda, dtype):
    # Twenty decode steps enqueued without a host synchronisation: each launch
    # reads the K/V row the launch before it stored (steps cross page
    # boundaries at 16 and 32 tokens), so a launch that began reading before
    # its predecessor finished would show up here.  Every step's output
    # against the oracle's step-by-step run; the pages bit for bit.
    import torch

    from llmhost_b200.kv import KvPool
    from llmhost_b200.workloads import PAGE_TOKENS, normal_bits
    from oracle import oracle as O
    from paged_case import PAGE_NONE

    rng = np.random.default_rng(21)
    n_q, n_kv, steps = 24, 8, 20
    lens0 = np.array([0, 15, 16, 30, 100, 2047, 5000], np.int64)
    n = len(lens0)
    pages = -(-(lens0 + steps) // PAGE_TOKENS)
    n_pages = int(pages.sum()) + 4
    perm = rng.permutation(n_pages).astype(np.uint32)
    bt = np.full((n, int(pages.max())), PAGE_NONE, np.uint32)
    cur = 0
    for s in range(n):
        bt[s, :pages[s]] = perm[cur:cur + pages[s]]
        cur += pages[s]
    k_pre = [normal_bits(rng, (int(L), n_kv, 64), dtype) for L in lens0]
    v_pre = [normal_bits(rng, (int(L), n_kv, 64), dtype) for L in lens0]
    qs = [normal_bits(rng, (n, n_q, 64), dtype) for _ in range(steps)]
    ks = [normal_bits(rng, (n, n_kv, 64), dtype) for _ in range(steps)]
    vs = [normal_bits(rng, (n, n_kv, 64), dtype) for _ in range(steps)]

    host = O.HostPages(n_pages, O.BF16 if dtype == "bf16" else O.F32, n_q, n_kv)
    for s in range(n):
        for t in range(int(lens0[s])):
            host.append_token(bt[s], t, t, k_pre[s][t], v_pre[s][t])
    refs = [host.decode_step(bt, (lens0 + i + 1).astype(np.int32), 0, qs[i], ks[i], vs[i]) for i in range(steps)]

    with KvPool(dtype=dtype, n_q_heads=n_q, n_kv_heads=n_kv, n_pages=n_pages,
                max_positions=int(lens0.max()) + steps + 16, max_seqs=n) as pool:
        dev = pool.device
        bt_d = torch.from_numpy(bt.view(np.int32)).to(dev)
        tok_seq = np.concatenate([np.full(int(L), s, np.int32) for s, L in enumerate(lens0)])
        tok_slot = np.concatenate([np.arange(int(L), dtype=np.int32) for L in lens0])
        ts, tl = torch.from_numpy(tok_seq).to(dev), torch.from_numpy(tok_slot).to(dev)
        pool.append(to_torch(np.concatenate([a.reshape(-1) for a in k_pre]), dtype, dev),
                    to_torch(np.concatenate([a.reshape(-1) for a in v_pre]), dtype, dev), ts, tl, tl, bt_d)
        lens_d = [torch.from_numpy((lens0 + i + 1).astype(np.int32)).to(dev) for i in range(steps)]
        qd = [to_torch(x, dtype, dev) for x in qs]
        kd = [to_torch(x, dtype, dev) for x in ks]
        vd = [to_torch(x, dtype, dev) for x in vs]
        torch.cuda.synchronize()
        outs = [pool.append_decode_attn(kd[i], vd[i], qd[i], bt_d, lens_d[i]) for i in range(steps)]
        torch.cuda.synchronize()
        assert pool.last_error() == 0
        ids = np.sort(bt[bt != PAGE_NONE])
        np.testing.assert_array_equal(pool.read_pages(ids), host.data[ids], err_msg="stored pages differ")
        for i in range(steps):
            assert_close_rows(to_numpy_f32(outs[i]), refs[i], RTOL[dtype], f"{dtype} step {i}")
