"""The CPU oracle, pinned before it is trusted (no GPU needed).

1. Known-answer tests ported from the reference's own unit tests
   (crates/llm-cpu/src/rope.rs:87-109, crates/llm-cpu/src/ops.rs:120-126).
2. Golden vectors from Hugging Face transformers' LFM2 (fp32 eager attention),
   the upstream the reference's golden test compares against
   (crates/llm-engine/tests/lfm2_700m_golden.rs:1-17); see tests/golden/make_golden.py.
3. Internal identities of the restatement (decode == last causal row, paged ==
   contiguous, bf16 rounding == torch's).
"""
import json
from pathlib import Path

import numpy as np
import pytest

from llmhost_b200.workloads import normal_bits
from oracle import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden" / "golden.npz"


# ---- 1. reference KATs --------------------------------------------------------
def test_inv_freq_length_and_first():  # rope.rs:87-93
    f = O.inv_freq(64, 1_000_000.0)
    assert len(f) == 32
    assert abs(f[0] - 1.0) < 1e-6
    assert f[31] < f[0]


def test_rope_position_zero_is_identity():  # rope.rs:95-109
    inv = O.inv_freq(4, 10_000.0)
    c, s = O.cos_sin(inv, 0, 1, 4)
    q = np.array([1.0, 2.0, 3.0, 4.0], np.float32)
    O.apply_rope_in_place(q, c, s, 1, 1, 4)
    np.testing.assert_allclose(q, [1, 2, 3, 4], atol=1e-6)


def test_softmax_sums_to_one():  # ops.rs:120-126
    z = np.array([1.0, 3.0, 2.0], np.float32)
    O.softmax_last_axis(z, 3)
    assert abs(float(z.sum()) - 1.0) < 1e-6


def test_softmax_all_masked_row_is_nan_like_reference():
    # ops.rs:68-77: max = -inf, (-inf) - (-inf) = NaN, so the reference yields NaN.
    z = np.array([-np.inf, -np.inf], np.float32)
    O.softmax_last_axis(z, 2)
    assert np.all(np.isnan(z))


# ---- 2. golden vectors (HF transformers LFM2, fp32 eager) ------------------------
@pytest.fixture(scope="module")
def golden():
    g = np.load(GOLDEN)
    meta = json.loads(bytes(g["meta"]).decode())
    return g, meta


def test_golden_inv_freq(golden):
    g, meta = golden
    np.testing.assert_allclose(O.inv_freq(meta["d"], meta["theta"]), g["inv_freq"], rtol=2e-7)


def test_golden_rope_tables(golden):
    g, meta = golden
    inv = O.inv_freq(meta["d"], meta["theta"])
    for i, p in enumerate(meta["rope_positions"]):
        c, s = O.cos_sin(inv, p, 1, meta["d"])
        # torch and glibc cos/sin differ in the last bit; arguments reach 1e6 rad.
        np.testing.assert_allclose(c[0], g["rope_cos"][i], atol=2e-6, err_msg=f"cos pos {p}")
        np.testing.assert_allclose(s[0], g["rope_sin"][i], atol=2e-6, err_msg=f"sin pos {p}")


def _rope_heads(x, inv, positions, d):
    """Rotate [heads, T, d] rows at the given absolute positions (oracle)."""
    x = np.ascontiguousarray(x, np.float32).copy()
    c, s = O.cos_sin(inv, positions[0], len(positions), d)
    O.apply_rope_in_place(x, c, s, x.shape[0], x.shape[1], d)
    return x


def test_golden_decode_attention(golden):
    import tests_golden_inputs as gi

    g, meta = golden
    n_q, n_kv, d = meta["n_q"], meta["n_kv"], meta["d"]
    inv = O.inv_freq(d, meta["theta"])
    for seed, kv_len in meta["decode_cases"]:
        q, k, v = gi.inputs_decode(seed, kv_len, n_q, n_kv, d)
        k_rot = _rope_heads(k, inv, list(range(kv_len)), d)
        q_rot = _rope_heads(q[:, None, :], inv, [kv_len - 1], d)[:, 0, :]
        out = O.attention_decode_cached(q_rot, k_rot, v, n_q, n_kv, kv_len, kv_len, d)
        ref = g[f"decode_{seed}_{kv_len}"]
        assert O.rel_err_rows(out, ref).max() < 1e-5, f"decode seed {seed}"


def test_golden_prefill_attention(golden):
    import tests_golden_inputs as gi

    g, meta = golden
    n_q, n_kv, d = meta["n_q"], meta["n_kv"], meta["d"]
    inv = O.inv_freq(d, meta["theta"])
    for seed, t in meta["prefill_cases"]:
        q, k, v = gi.inputs_prefill(seed, t, n_q, n_kv, d)
        q_rot = _rope_heads(q, inv, list(range(t)), d)
        k_rot = _rope_heads(k, inv, list(range(t)), d)
        out = O.attention_forward(q_rot, k_rot, v, n_q, n_kv, t, t, d, causal=True)
        ref = g[f"prefill_{seed}_{t}"]
        assert O.rel_err_rows(out, ref).max() < 1e-5, f"prefill seed {seed}"


# ---- 3. identities of the restatement ---------------------------------------------
def test_decode_equals_last_causal_row_bit_exact():
    rng = np.random.default_rng(0)
    n_q, n_kv, d, L = 24, 8, 64, 37
    q = rng.standard_normal((n_q, L, d), dtype=np.float32)
    k = rng.standard_normal((n_kv, L, d), dtype=np.float32)
    v = rng.standard_normal((n_kv, L, d), dtype=np.float32)
    fw = O.attention_forward(q, k, v, n_q, n_kv, L, L, d, causal=True)
    dc = O.attention_decode_cached(np.ascontiguousarray(q[:, -1, :]), k, v, n_q, n_kv, L, L, d)
    np.testing.assert_array_equal(fw[:, -1, :], dc)


def test_key_valid_pad_mask_matches_explicit_mask():
    rng = np.random.default_rng(1)
    n_q, n_kv, d, L = 8, 2, 64, 20
    q = rng.standard_normal((n_q, L, d), dtype=np.float32)
    k = rng.standard_normal((n_kv, L, d), dtype=np.float32)
    v = rng.standard_normal((n_kv, L, d), dtype=np.float32)
    valid = np.ones(L, np.uint8)
    valid[[0, 3]] = 0
    a = O.attention_forward(q, k, v, n_q, n_kv, L, L, d, causal=True, key_valid=valid)
    mask = (np.tril(np.ones((L, L), np.uint8)) & valid[None, :]).astype(np.uint8)
    b = O.attention_masked(q, k, v, n_q, n_kv, L, L, d, mask)
    np.testing.assert_array_equal(np.nan_to_num(a), np.nan_to_num(b))


@pytest.mark.parametrize("dtype", [O.F32, O.BF16])
def test_paged_decode_equals_contiguous(dtype):
    rng = np.random.default_rng(2)
    n_q, n_kv, d, L = 24, 8, 64, 45
    name = "bf16" if dtype == O.BF16 else "f32"
    host = O.HostPages(16, dtype, n_q, n_kv)
    bt = np.array([7, 2, 11, 5], np.uint32)
    kr = normal_bits(rng, (L, n_kv, d), name)
    vr = normal_bits(rng, (L, n_kv, d), name)
    for t in range(L):
        host.append_token(bt, t, t, kr[t], vr[t])
    qr = normal_bits(rng, (n_q, d), name)
    out = host.decode(bt, L, 0, qr)
    # contiguous path: widen, rotate k at its own positions and q at L-1
    widen = (lambda a: O.bf16_bits_to_f32(a)) if dtype == O.BF16 else (lambda a: a)
    k = _rope_heads(widen(kr).transpose(1, 0, 2), host.inv, list(range(L)), d)
    if dtype == O.BF16:  # the pool stores rotated K in bf16
        k = O.bf16_bits_to_f32(O.f32_to_bf16_bits(k)).reshape(k.shape)
    v = np.ascontiguousarray(widen(vr).transpose(1, 0, 2))
    q = _rope_heads(widen(qr)[:, None, :], host.inv, [L - 1], d)[:, 0, :]
    ref = O.attention_decode_cached(q, k, v, n_q, n_kv, L, L, d)
    np.testing.assert_array_equal(out, ref)


def test_bf16_rounding_matches_torch():
    import torch

    rng = np.random.default_rng(3)
    x = np.concatenate([rng.standard_normal(10000, dtype=np.float32),
                        np.array([0.0, -0.0, 1e-40, 3.4e38, -3.4e38, np.inf, -np.inf], np.float32)])
    t = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(O.f32_to_bf16_bits(x), t)
    for xi in x[:50]:
        assert O.lib().orc_f32_to_bf16(float(xi)) == O.f32_to_bf16_bits(np.array([xi]))[0]


def test_decode_step_threads_agree():
    rng = np.random.default_rng(4)
    n = 9
    lens = rng.integers(1, 90, size=n).astype(np.int32)
    host1 = O.HostPages(128, O.BF16, 24, 8)
    bt = rng.permutation(128).astype(np.uint32)[: n * 8].reshape(n, 8)
    q = normal_bits(rng, (n, 24, 64), "bf16")
    k = normal_bits(rng, (n, 8, 64), "bf16")
    v = normal_bits(rng, (n, 8, 64), "bf16")
    host2 = O.HostPages(128, O.BF16, 24, 8, data=host1.data.copy())
    a = host1.decode_step(bt, lens, 0, q, k, v, n_threads=1)
    b = host2.decode_step(bt, lens, 0, q, k, v, n_threads=4)
    np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(host1.data, host2.data)


def test_rms_norm_known_answer():
    # ops.rs:108-117: x = [3, 4], unit weight, eps 0 -> x / sqrt(12.5)
    y = O.rms_norm(np.array([3.0, 4.0], np.float32), np.array([1.0, 1.0], np.float32), 0.0)
    rms = np.sqrt(np.float32(12.5))
    assert abs(y[0] - 3.0 / rms) < 1e-6 and abs(y[1] - 4.0 / rms) < 1e-6


def test_rms_norm_matches_sequential_double_restatement():
    # The same operations in plain Python (floats are doubles, the loop is
    # sequential like ops.rs:14-17): bit-exact.
    import math

    rng = np.random.default_rng(5)
    x = rng.standard_normal((6, 64)).astype(np.float32) * np.float32(3.0)
    w = rng.standard_normal(64).astype(np.float32)
    eps = 1e-5
    got = O.rms_norm(x, w, eps)
    for r in range(x.shape[0]):
        s = 0.0
        for v in x[r]:
            s += float(v) * float(v)
        scale = np.float32(1.0 / math.sqrt(s * (1.0 / 64) + float(np.float32(eps))))
        want = w * (x[r] * scale)
        np.testing.assert_array_equal(got[r], want)
