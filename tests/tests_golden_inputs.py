"""Inputs of the golden vectors, regenerated from their seeds.

Mirrors inputs_decode / inputs_prefill of tests/golden/make_golden.py, which
imports torch and transformers; tests only need numpy.
"""
import numpy as np


def inputs_decode(seed: int, kv_len: int, n_q: int, n_kv: int, d: int):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((n_q, d), dtype=np.float32)
    k = rng.standard_normal((n_kv, kv_len, d), dtype=np.float32)
    v = rng.standard_normal((n_kv, kv_len, d), dtype=np.float32)
    return q, k, v


def inputs_prefill(seed: int, tokens: int, n_q: int, n_kv: int, d: int):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((n_q, tokens, d), dtype=np.float32)
    k = rng.standard_normal((n_kv, tokens, d), dtype=np.float32)
    v = rng.standard_normal((n_kv, tokens, d), dtype=np.float32)
    return q, k, v
