"""numpy/ctypes wrapper of the C oracle (oracle/kv_oracle.c) -- TEST INFRASTRUCTURE.

The oracle is the checker for the CUDA path, never the product.  Only tests/,
__graft_entry__.smoke() and bench.py's CPU baseline / reference arm use it.
Parity anchors: the restated functions follow crates/llm-cpu/src/rope.rs:6-81,
crates/llm-cpu/src/ops.rs:64-79 and crates/llm-engine/src/lfm2.rs:1006-1111 of
the reference; kv_oracle.c cites the line each C statement stands for.
"""
from __future__ import annotations

import ctypes
import subprocess
from ctypes import POINTER, c_float, c_int, c_int32, c_size_t, c_uint16, c_uint32, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libkv_oracle.so"

F32 = 0
BF16 = 1
Q8 = 2     # K and V as Q8_0 blocks (crates/llm-quant/src/lib.rs:14-46)
K8V4 = 3   # K as Q8_0, V as Q4 blocks (lib.rs:48-101)
F16 = 4    # K and V as IEEE half, bf16 layout; bf16 k / v / q in
PAGE_NONE = 0xFFFFFFFF

_lib = None


def build(force: bool = False) -> Path:
    """Compile the oracle with its Makefile (gcc, -ffp-contract=off)."""
    src = [HERE / "kv_oracle.c", HERE / "kv_oracle.h", HERE / "Makefile"]
    if force or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < max(p.stat().st_mtime for p in src):
        subprocess.run(["make", "-s", "-B" if force else "all"], cwd=HERE, check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        h = ctypes.CDLL(str(LIB_PATH))
        fp = POINTER(c_float)
        h.orc_f32_to_bf16.restype = c_uint16
        h.orc_f32_to_bf16.argtypes = [c_float]
        h.orc_bf16_to_f32.restype = c_float
        h.orc_bf16_to_f32.argtypes = [c_uint16]
        h.orc_inv_freq.argtypes = [c_size_t, c_float, fp]
        h.orc_cos_sin.argtypes = [fp, c_size_t, c_size_t, c_size_t, fp, fp]
        h.orc_apply_rope_in_place.argtypes = [fp, fp, fp, c_size_t, c_size_t, c_size_t]
        h.orc_softmax_last_axis.argtypes = [fp, c_size_t, c_size_t]
        h.orc_attention_decode_cached.argtypes = [fp, fp, fp, c_size_t, c_size_t, c_size_t, c_size_t,
                                                  c_size_t, c_void_p, c_size_t, fp, fp]
        h.orc_attention_forward.argtypes = [fp, fp, fp, c_size_t, c_size_t, c_size_t, c_size_t,
                                            c_size_t, c_int, c_void_p, fp]
        h.orc_attention_masked.argtypes = [fp, fp, fp, c_size_t, c_size_t, c_size_t, c_size_t,
                                           c_size_t, c_void_p, fp]
        h.orc_paged_append_token.argtypes = [c_void_p, c_int, c_size_t, c_size_t, c_size_t, c_void_p,
                                             c_size_t, c_void_p, c_void_p, fp, fp]
        h.orc_paged_gather.argtypes = [c_void_p, c_int, c_size_t, c_size_t, c_size_t, c_void_p,
                                       c_size_t, fp, fp]
        h.orc_paged_decode.argtypes = [c_void_p, c_int, c_size_t, c_size_t, c_size_t, c_size_t,
                                       c_void_p, c_size_t, c_size_t, c_void_p, fp, fp]
        h.orc_decode_step.argtypes = [c_void_p, c_int, c_size_t, c_size_t, c_size_t, c_size_t,
                                      c_void_p, c_size_t, c_void_p, c_size_t, c_size_t, c_void_p,
                                      c_void_p, c_void_p, fp, fp, c_int]
        h.orc_decode_step_norm.argtypes = [c_void_p, c_int, c_size_t, c_size_t, c_size_t, c_size_t,
                                           c_void_p, c_size_t, c_void_p, c_size_t, c_size_t, c_void_p,
                                           c_void_p, c_void_p, fp, fp, fp, c_float, fp, c_int]
        h.orc_rms_norm.argtypes = [fp, fp, c_float, c_size_t, c_size_t, fp]
        h.orc_paged_append_tokens.argtypes = [c_void_p, c_int, c_size_t, c_size_t, c_size_t, c_void_p,
                                              c_size_t, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p,
                                              c_void_p, fp, c_int]
        h.orc_paged_prefill.argtypes = [c_void_p, c_int, c_size_t, c_size_t, c_size_t, c_size_t, c_void_p,
                                        c_size_t, c_size_t, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                        fp, fp, c_int]
        h.orc_f32_to_f16.restype = c_uint16
        h.orc_f32_to_f16.argtypes = [c_float]
        h.orc_f16_to_f32.restype = c_float
        h.orc_f16_to_f32.argtypes = [c_uint16]
        h.orc_quantize_q8_0.argtypes = [fp, c_void_p, c_void_p]
        h.orc_quantize_q4.argtypes = [fp, c_void_p, c_void_p]
        h.orc_page_bytes.restype = c_size_t
        h.orc_page_bytes.argtypes = [c_int, c_size_t, c_size_t, c_size_t]
        h.orc_max_threads.restype = c_int
        _lib = h
    return _lib


def _f(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(POINTER(c_float))


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


# ---- bf16 (round to nearest even, same rule as orc_f32_to_bf16) -------------
def f32_to_bf16_bits(x) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(b) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---- restated reference functions ---------------------------------------------
def inv_freq(dim: int, theta: float) -> np.ndarray:
    out = np.empty(dim // 2, np.float32)
    lib().orc_inv_freq(dim, theta, _f(out))
    return out


def cos_sin(inv: np.ndarray, start: int, tokens: int, dim: int):
    c = np.empty((tokens, dim), np.float32)
    s = np.empty((tokens, dim), np.float32)
    lib().orc_cos_sin(_f(inv), start, tokens, dim, _f(c), _f(s))
    return c, s


def apply_rope_in_place(states: np.ndarray, c: np.ndarray, s: np.ndarray, heads, tokens, dim):
    lib().orc_apply_rope_in_place(_f(states), _f(c), _f(s), heads, tokens, dim)


def softmax_last_axis(logits: np.ndarray, n: int) -> None:
    lib().orc_softmax_last_axis(_f(logits), logits.size, n)


def attention_decode_cached(q, k_cache, v_cache, n_q, n_kv, kv_len, kv_cap, dim, key_valid=None):
    q, k_cache, v_cache = (np.ascontiguousarray(a, np.float32) for a in (q, k_cache, v_cache))
    kvm = None if key_valid is None else np.ascontiguousarray(key_valid, np.uint8)
    scores = np.empty(n_q * kv_len, np.float32)
    out = np.empty(n_q * dim, np.float32)
    lib().orc_attention_decode_cached(_f(q), _f(k_cache), _f(v_cache), n_q, n_kv, kv_len, kv_cap, dim,
                                      _p(kvm), 0 if kvm is None else kvm.size, _f(scores), _f(out))
    return out.reshape(n_q, dim)


def attention_forward(q, k, v, n_q, n_kv, q_len, kv_len, dim, causal=True, key_valid=None):
    q, k, v = (np.ascontiguousarray(a, np.float32) for a in (q, k, v))
    kvm = None if key_valid is None else np.ascontiguousarray(key_valid, np.uint8)
    out = np.empty(n_q * q_len * dim, np.float32)
    lib().orc_attention_forward(_f(q), _f(k), _f(v), n_q, n_kv, q_len, kv_len, dim, int(causal),
                                _p(kvm), _f(out))
    return out.reshape(n_q, q_len, dim)


def attention_masked(q, k, v, n_q, n_kv, q_len, kv_len, dim, mask):
    q, k, v = (np.ascontiguousarray(a, np.float32) for a in (q, k, v))
    m = np.ascontiguousarray(mask, np.uint8)
    out = np.empty(n_q * q_len * dim, np.float32)
    lib().orc_attention_masked(_f(q), _f(k), _f(v), n_q, n_kv, q_len, kv_len, dim, _p(m), _f(out))
    return out.reshape(n_q, q_len, dim)


# ---- paged layout ---------------------------------------------------------------
def quantize_q8_0(block) -> tuple[int, np.ndarray]:
    """One 32-element Q8_0 block (orc_quantize_q8_0): (f16 scale bits, int8 codes)."""
    x = np.ascontiguousarray(block, np.float32)
    assert x.size == 32
    sc = np.zeros(1, np.uint16)
    qs = np.zeros(32, np.int8)
    lib().orc_quantize_q8_0(_f(x), sc.ctypes.data, qs.ctypes.data)
    return int(sc[0]), qs


def quantize_q4(block) -> tuple[int, np.ndarray]:
    """One 32-element Q4 block (orc_quantize_q4): (f16 scale bits, 16 packed bytes)."""
    x = np.ascontiguousarray(block, np.float32)
    assert x.size == 32
    sc = np.zeros(1, np.uint16)
    qs = np.zeros(16, np.uint8)
    lib().orc_quantize_q4(_f(x), sc.ctypes.data, qs.ctypes.data)
    return int(sc[0]), qs


def f32_to_f16_bits(x: float) -> int:
    return int(lib().orc_f32_to_f16(x))


def f16_bits_to_f32(h: int) -> float:
    return float(lib().orc_f16_to_f32(h))


class HostPages:
    """A host copy of a page pool in the build's layout: [K|V][n_kv][P][d] per
    page for F32 / BF16; for the quantised types Q8 / K8V4 the page is bytes
    (K codes, V codes, K scales, V scales; see kv_oracle.c), and the appended
    k / v and the queries are bf16."""

    def __init__(self, n_pages: int, dtype: int, n_q: int, n_kv: int, page_tokens: int = 16,
                 head_dim: int = 64, theta: float = 1e6, data: np.ndarray | None = None):
        self.dtype, self.n_q, self.n_kv = dtype, n_q, n_kv
        self.P, self.d = page_tokens, head_dim
        self.quant = dtype in (Q8, K8V4)
        if self.quant:
            self.page_elems = int(lib().orc_page_bytes(dtype, n_kv, page_tokens, head_dim))
            np_dt = np.uint8
        else:
            self.page_elems = 2 * n_kv * page_tokens * head_dim
            np_dt = np.uint16 if dtype in (BF16, F16) else np.float32
        if data is None:
            data = np.zeros((n_pages, self.page_elems), np_dt)
        assert data.dtype == np_dt and data.shape == (n_pages, self.page_elems)
        self.data = np.ascontiguousarray(data)
        self.inv = inv_freq(head_dim, theta)

    def _raw(self, a) -> np.ndarray:
        np_dt = np.uint16 if self.dtype in (BF16, Q8, K8V4, F16) else np.float32
        a = np.ascontiguousarray(a)
        assert a.dtype == np_dt, (a.dtype, np_dt)
        return a

    def append_token(self, bt, slot: int, rope_pos: int, k_raw, v) -> None:
        bt = np.ascontiguousarray(bt, np.uint32)
        c, s = cos_sin(self.inv, rope_pos, 1, self.d)
        k_raw, v = self._raw(k_raw), self._raw(v)
        lib().orc_paged_append_token(self.data.ctypes.data, self.dtype, self.n_kv, self.P, self.d,
                                     bt.ctypes.data, slot, k_raw.ctypes.data, v.ctypes.data,
                                     _f(c), _f(s))

    def append_tokens(self, bt2d, tok_row, slots, positions, k_raw, v, n_threads: int = 0) -> None:
        """Many append_token calls in one (orc_paged_append_tokens): token i to
        row tok_row[i] of bt2d, slot slots[i], RoPE position positions[i];
        k_raw / v are [n_tokens, n_kv, d].  Slots must be distinct."""
        bt2d = np.ascontiguousarray(bt2d, np.uint32)
        if bt2d.ndim == 1:
            bt2d = bt2d[None, :]
        tok_row, slots, positions = (np.ascontiguousarray(a, np.int32) for a in (tok_row, slots, positions))
        n = len(slots)
        assert len(tok_row) == n and len(positions) == n
        k_raw, v = self._raw(k_raw), self._raw(v)
        assert k_raw.size == n * self.n_kv * self.d and v.size == k_raw.size
        if n == 0:
            return
        lib().orc_paged_append_tokens(self.data.ctypes.data, self.dtype, self.n_kv, self.P, self.d,
                                      bt2d.ctypes.data, bt2d.shape[1], tok_row.ctypes.data, slots.ctypes.data,
                                      positions.ctypes.data, n, k_raw.ctypes.data, v.ctypes.data, _f(self.inv),
                                      n_threads)

    def prefill(self, bt2d, cached, q_off, q_pos, q_raw, masks=None, n_threads: int = 0) -> np.ndarray:
        """Chunked-prefill (masks None: causal chunk) or tree-verify (masks:
        ancestor-or-self bits per query token) attention over the stored pages
        (orc_paged_prefill).  Returns [n_tok, n_q, d] float32."""
        bt2d = np.ascontiguousarray(bt2d, np.uint32)
        cached, q_off, q_pos = (np.ascontiguousarray(a, np.int32) for a in (cached, q_off, q_pos))
        q_raw = self._raw(q_raw)
        n_tok = int(q_off[-1])
        assert len(q_pos) == n_tok and q_raw.size == n_tok * self.n_q * self.d
        m = None if masks is None else np.ascontiguousarray(np.asarray(masks).view(np.uint64))
        out = np.zeros((n_tok, self.n_q, self.d), np.float32)
        lib().orc_paged_prefill(self.data.ctypes.data, self.dtype, self.n_q, self.n_kv, self.P, self.d,
                                bt2d.ctypes.data, bt2d.shape[1], len(cached), cached.ctypes.data,
                                q_off.ctypes.data, q_pos.ctypes.data, _p(m), q_raw.ctypes.data, _f(self.inv),
                                _f(out), n_threads)
        return out

    def gather(self, bt, n_tokens: int):
        bt = np.ascontiguousarray(bt, np.uint32)
        k = np.empty((self.n_kv, n_tokens, self.d), np.float32)
        v = np.empty((self.n_kv, n_tokens, self.d), np.float32)
        lib().orc_paged_gather(self.data.ctypes.data, self.dtype, self.n_kv, self.P, self.d,
                               bt.ctypes.data, n_tokens, _f(k), _f(v))
        return k, v

    def decode(self, bt, seq_len: int, window: int, q_raw) -> np.ndarray:
        bt = np.ascontiguousarray(bt, np.uint32)
        q_raw = self._raw(q_raw)
        out = np.empty((self.n_q, self.d), np.float32)
        lib().orc_paged_decode(self.data.ctypes.data, self.dtype, self.n_q, self.n_kv, self.P, self.d,
                               bt.ctypes.data, seq_len, window, q_raw.ctypes.data, _f(self.inv),
                               _f(out))
        return out

    def decode_step(self, bt2d, seq_lens, window: int, q_raw, k_raw, v, n_threads: int = 0):
        """Append one token per sequence then decode (orc_decode_step)."""
        bt2d = np.ascontiguousarray(bt2d, np.uint32)
        seq_lens = np.ascontiguousarray(seq_lens, np.int32)
        q_raw, k_raw, v = self._raw(q_raw), self._raw(k_raw), self._raw(v)
        n = len(seq_lens)
        out = np.empty((n, self.n_q, self.d), np.float32)
        lib().orc_decode_step(self.data.ctypes.data, self.dtype, self.n_q, self.n_kv, self.P, self.d,
                              bt2d.ctypes.data, bt2d.shape[1], seq_lens.ctypes.data, n, window,
                              q_raw.ctypes.data, k_raw.ctypes.data, v.ctypes.data, _f(self.inv),
                              _f(out), n_threads)
        return out

    def decode_step_norm(self, bt2d, seq_lens, window: int, q_raw, k_raw, v, q_norm, k_norm, eps: float,
                         n_threads: int = 0):
        """decode_step with the per-head RMSNorm of q and k before RoPE
        (orc_decode_step_norm, lfm2.rs:797-812)."""
        bt2d = np.ascontiguousarray(bt2d, np.uint32)
        seq_lens = np.ascontiguousarray(seq_lens, np.int32)
        q_raw, k_raw, v = self._raw(q_raw), self._raw(k_raw), self._raw(v)
        qn = np.ascontiguousarray(q_norm, np.float32)
        kn = np.ascontiguousarray(k_norm, np.float32)
        n = len(seq_lens)
        out = np.empty((n, self.n_q, self.d), np.float32)
        lib().orc_decode_step_norm(self.data.ctypes.data, self.dtype, self.n_q, self.n_kv, self.P, self.d,
                                   bt2d.ctypes.data, bt2d.shape[1], seq_lens.ctypes.data, n, window,
                                   q_raw.ctypes.data, k_raw.ctypes.data, v.ctypes.data, _f(self.inv),
                                   _f(qn), _f(kn), ctypes.c_float(eps), _f(out), n_threads)
        return out


def rms_norm(x, weight, eps: float) -> np.ndarray:
    """RMSNorm over the last axis (orc_rms_norm, ops.rs:8-23); float32 in and out."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(weight, np.float32)
    out = np.empty_like(x)
    lib().orc_rms_norm(_f(x), _f(w), ctypes.c_float(eps), w.size, x.size // w.size, _f(out))
    return out


def max_threads() -> int:
    return int(lib().orc_max_threads())


def rel_err_rows(got: np.ndarray, ref: np.ndarray) -> np.ndarray:
    """Normwise error per output row: max|got - ref| / max|ref| over the last axis."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    num = np.abs(got - ref).max(axis=-1)
    den = np.maximum(np.abs(ref).max(axis=-1), 1e-30)
    return num / den
