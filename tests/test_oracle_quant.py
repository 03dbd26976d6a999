"""The oracle's quantised KV formats, pinned before the kernels use them (no GPU).

KvDtype tags Q8 ("8-bit keys and values") and K8V4 ("8-bit keys and 4-bit
values") in crates/llm-quant/src/formats.rs:59-68 without kernels; the same
crate's block quantisers (BlockQ8_0, BlockQ4, crates/llm-quant/src/lib.rs:14-101)
are the arithmetic the build stores K/V with.  Pinned here:

1. the reference's own assertions on those quantisers (lib.rs:149-220);
2. the C restatement bit for bit against an independent numpy restatement
   of the same lines (f16 scale by round-to-nearest-even, round half away
   from zero, clamp), on random blocks and on edge values;
3. paged quantised pages: what append stores, gather dequantises (q * scale).
"""
import numpy as np
import pytest

from llmhost_b200.workloads import normal_bits
from oracle import oracle as O


def pattern():  # lib.rs:149-159
    src = np.array([i * 0.37 - 5.1 for i in range(32)], np.float32)
    src[0], src[1], src[2] = -6.0, 6.0, 0.0
    return src


def deq_q8(scale_bits, qs):
    return qs.astype(np.float32) * np.float32(O.f16_bits_to_f32(scale_bits))


def deq_q4(scale_bits, packed):
    lo = (packed & 0x0F).astype(np.int8)
    hi = (packed >> 4).astype(np.int8)
    nib = np.empty(32, np.int8)
    nib[0::2], nib[1::2] = lo, hi
    nib = ((nib.astype(np.int16) << 12).astype(np.int16) >> 12).astype(np.float32)  # sign-extend 4 bits
    return nib * np.float32(O.f16_bits_to_f32(scale_bits))


def test_q8_0_roundtrip():  # lib.rs:168-179
    src = pattern()
    back = deq_q8(*O.quantize_q8_0(src))
    amax = np.abs(src).max()
    assert np.abs(src - back).max() <= amax / 127.0 + 1e-3


def test_q4_roundtrip():  # lib.rs:181-196
    src = pattern()
    sc, packed = O.quantize_q4(src)
    back = deq_q4(sc, packed)
    amax = np.abs(src).max()
    assert np.abs(src - back).max() <= amax / 8.0 + 1e-3
    nib = np.concatenate([(packed & 0xF), (packed >> 4)]).astype(np.int8)
    nib = np.where(nib >= 8, nib - 16, nib)
    assert ((nib >= -8) & (nib <= 7)).all()


def test_zero_block():  # lib.rs:198-206
    z = np.zeros(32, np.float32)
    assert (deq_q8(*O.quantize_q8_0(z)) == 0).all()
    assert (deq_q4(*O.quantize_q4(z)) == 0).all()


def test_slices():  # lib.rs:208-220
    src = np.array([np.sin(np.float32(i)) * np.float32(3.0) for i in range(96)], np.float32)
    b8 = np.concatenate([deq_q8(*O.quantize_q8_0(src[32 * b:32 * b + 32])) for b in range(3)])
    b4 = np.concatenate([deq_q4(*O.quantize_q4(src[32 * b:32 * b + 32])) for b in range(3)])
    assert np.abs(src - b8).max() < 0.05
    assert np.abs(src - b4).max() < 0.5


def _np_quant(block, qmax, qmin, div):
    """lib.rs:26-36 / 63-78 in numpy, independently of the C restatement."""
    x = np.asarray(block, np.float32)
    amax = np.float32(np.max(np.abs(x))) if x.size else np.float32(0)
    scale = np.float16(amax / np.float32(div))
    sf = np.float32(scale)
    inv = np.float32(0) if sf == 0 else np.float32(1) / sf
    y = (x * inv).astype(np.float64)                    # the f32 product, exactly
    q = np.sign(y) * np.floor(np.abs(y) + 0.5)         # round half away from zero
    q = np.clip(q, qmin, qmax).astype(np.int8)
    return int(scale.view(np.uint16)), q


@pytest.mark.parametrize("seed", range(4))
def test_quantisers_match_an_independent_restatement(seed):
    rng = np.random.default_rng(seed)
    blocks = [rng.standard_normal(32).astype(np.float32) * np.float32(10.0 ** rng.integers(-4, 4)) for _ in range(300)]
    blocks += [np.full(32, 0.5, np.float32), np.full(32, -2.5, np.float32), np.linspace(-127, 127, 32, dtype=np.float32),
               np.zeros(32, np.float32), np.array([65504.0 * 127] + [1.0] * 31, np.float32)]
    for b in blocks:
        sc, qs = O.quantize_q8_0(b)
        ws, wq = _np_quant(b, 127, -127, 127.0)
        assert sc == ws and np.array_equal(qs, wq), b
        sc4, packed = O.quantize_q4(b)
        ws4, wq4 = _np_quant(b, 7, -8, 8.0)
        want = ((wq4[0::2].astype(np.uint8) & 0xF) | ((wq4[1::2].astype(np.uint8) & 0xF) << 4)).astype(np.uint8)
        assert sc4 == ws4 and np.array_equal(packed, want), b


@pytest.mark.parametrize("dtype", [O.Q8, O.K8V4])
def test_quantised_pages_store_and_gather(dtype):
    rng = np.random.default_rng(5 + dtype)
    n_kv, n_q, T = 8, 24, 40
    pages = -(-T // 16)
    bt = rng.permutation(pages + 2).astype(np.uint32)[:pages]
    host = O.HostPages(pages + 2, dtype, n_q, n_kv)
    assert host.page_elems == n_kv * 16 * (64 + (64 if dtype == O.Q8 else 32) + 8)
    k = normal_bits(rng, (T, n_kv, 64), "bf16")
    v = normal_bits(rng, (T, n_kv, 64), "bf16")
    slots = np.arange(T, dtype=np.int32)
    host.append_tokens(bt[None, :], np.zeros(T, np.int32), slots, slots, k, v)
    kk, vv = host.gather(bt, T)  # [n_kv, T, 64] dequantised
    # K: the bf16 row rotated in fp32 (as for bf16 pools), then Q8_0 per 32 dims
    for t in range(T):  # the fp32 rotation is quantised directly (no bf16 rounding between)
        c, s = O.cos_sin(host.inv, t, 1, 64)
        kr = O.bf16_bits_to_f32(k[t]).copy()
        O.apply_rope_in_place(kr, c, s, n_kv, 1, 64)
        for h in range(n_kv):
            for b in range(2):
                sc, qs = O.quantize_q8_0(kr[h, 32 * b:32 * b + 32])
                np.testing.assert_array_equal(kk[h, t, 32 * b:32 * b + 32], deq_q8(sc, qs))
                vb = O.bf16_bits_to_f32(v[t, h, 32 * b:32 * b + 32])
                want_v = deq_q8(*O.quantize_q8_0(vb)) if dtype == O.Q8 else deq_q4(*O.quantize_q4(vb))
                np.testing.assert_array_equal(vv[h, t, 32 * b:32 * b + 32], want_v)
    # decode on quantised pages = the fp32 attention on the dequantised K/V
    q = normal_bits(rng, (n_q, 64), "bf16")
    got = host.decode(bt, T, 0, q)
    qf = O.bf16_bits_to_f32(q).copy()
    c, s = O.cos_sin(host.inv, T - 1, 1, 64)
    O.apply_rope_in_place(qf, c, s, n_q, 1, 64)
    ref = O.attention_decode_cached(qf, kk, vv, n_q, n_kv, T, T, 64)
    np.testing.assert_array_equal(got, ref)
