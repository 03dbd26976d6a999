"""The oracle's half-precision pages (ORC_F16, the library's KV_DTYPE_F16), no GPU.

KvDtype::F16 ("full f16 keys and values", crates/llm-quant/src/formats.rs:
59-68) is the reference's default tag (crates/llm-engine/src/batch.rs:306,
cache.rs:145).  The build stores such a page in the bf16 layout with IEEE half
elements; k / v come in as bf16, K is rotated in fp32 and both are rounded to
half to nearest even.  Pinned here against numpy's own float16 rounding, and
attention over the half pages against fp32 pages holding the same rounded
values.
"""
import numpy as np

from llmhost_b200.workloads import normal_bits
from oracle import oracle as O


def _bf16_to_f32(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def _case(seed=3, n_tok=37, n_q=24, n_kv=8):
    rng = np.random.default_rng(seed)
    k = normal_bits(rng, (n_tok, n_kv, 64), "bf16")
    v = normal_bits(rng, (n_tok, n_kv, 64), "bf16")
    n_pages = 8
    bt = rng.permutation(n_pages).astype(np.uint32)[:4]
    return rng, k, v, bt, n_pages, n_q, n_kv


def test_half_pages_hold_the_rounded_fp32_values():
    rng, k, v, bt, n_pages, n_q, n_kv = _case()
    half = O.HostPages(n_pages, O.F16, n_q, n_kv)
    full = O.HostPages(n_pages, O.F32, n_q, n_kv)
    for t in range(k.shape[0]):
        half.append_token(bt, t, t, k[t], v[t])
        full.append_token(bt, t, t, _bf16_to_f32(k[t]), _bf16_to_f32(v[t]))
    # the same rotation in fp32, then numpy's float16 (round to nearest even)
    want = full.data[bt].astype(np.float16).view(np.uint16)
    np.testing.assert_array_equal(half.data[bt], want)
    # V needs no rotation: bf16 -> fp32 -> half
    vrows = half.data[bt].reshape(len(bt), 2, n_kv, 16, 64)[:, 1]
    v_pages = np.zeros((len(bt) * 16, n_kv, 64), np.uint16)
    v_pages[: k.shape[0]] = _bf16_to_f32(v).astype(np.float16).view(np.uint16)
    np.testing.assert_array_equal(vrows.transpose(0, 2, 1, 3).reshape(-1, n_kv, 64)[: k.shape[0]],
                                  v_pages[: k.shape[0]])


def test_decode_over_half_pages_equals_fp32_pages_of_the_same_values():
    rng, k, v, bt, n_pages, n_q, n_kv = _case(seed=4)
    half = O.HostPages(n_pages, O.F16, n_q, n_kv)
    for t in range(k.shape[0]):
        half.append_token(bt, t, t, k[t], v[t])
    # fp32 pages holding exactly the half values
    full = O.HostPages(n_pages, O.F32, n_q, n_kv,
                       data=half.data.view(np.float16).astype(np.float32).reshape(n_pages, -1))
    q = normal_bits(rng, (1, n_q, 64), "bf16")
    kn = normal_bits(rng, (1, n_kv, 64), "bf16")
    vn = normal_bits(rng, (1, n_kv, 64), "bf16")
    lens = np.array([k.shape[0] + 1], np.int32)
    out_h = half.decode_step(bt[None, :], lens, 0, q, kn, vn)
    out_f = full.decode_step(bt[None, :], lens, 0, _bf16_to_f32(q), _bf16_to_f32(kn),
                             _bf16_to_f32(vn).astype(np.float16).astype(np.float32))
    # the appended token: K rounded to half on one side and kept in fp32 on
    # the other, so the two agree to half precision, not bit for bit
    np.testing.assert_allclose(out_h, out_f, rtol=0, atol=2e-3)
