"""Generate the golden vectors that pin the CPU oracle's attention and RoPE.

llmhost's own numeric gate (crates/llm-engine/tests/lfm2_700m_golden.rs:1-17)
compares its CPU path with Hugging Face transformers' LFM2 run in fp32 with
eager attention (tools/ref_dump.py:1-5).  This script runs the same upstream
functions -- `Lfm2RotaryEmbedding`, `apply_rotary_pos_emb` and
`eager_attention_forward` from transformers.models.lfm2.modeling_lfm2 -- on
seeded inputs and stores their outputs in golden.npz.  Inputs are not stored:
tests regenerate them from the seeds with numpy's PCG64 (`default_rng`).

    python tests/golden/make_golden.py     # rewrites tests/golden/golden.npz
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch
import transformers
from transformers.models.lfm2 import modeling_lfm2 as hf
from transformers.models.lfm2.configuration_lfm2 import Lfm2Config

HERE = Path(__file__).resolve().parent
OUT = HERE / "golden.npz"

# Shapes of the LFM2-700M attention layers (crates/llm-core/src/config.rs:494-525).
N_Q, N_KV, D, THETA = 24, 8, 64, 1e6
ROPE_POSITIONS = [0, 1, 17, 1000, 4095, 8191, 32767, 131071, 1048575]
DECODE_CASES = [(11, 1), (12, 129), (13, 700)]  # (seed, kv_len)
PREFILL_CASES = [(21, 33)]                     # (seed, tokens)


def inputs_decode(seed: int, kv_len: int):
    """Raw (pre-RoPE) q of the newest token and raw k/v of every position."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((N_Q, D), dtype=np.float32)
    k = rng.standard_normal((N_KV, kv_len, D), dtype=np.float32)
    v = rng.standard_normal((N_KV, kv_len, D), dtype=np.float32)
    return q, k, v


def inputs_prefill(seed: int, tokens: int):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((N_Q, tokens, D), dtype=np.float32)
    k = rng.standard_normal((N_KV, tokens, D), dtype=np.float32)
    v = rng.standard_normal((N_KV, tokens, D), dtype=np.float32)
    return q, k, v


class _Module(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.num_key_value_groups = N_Q // N_KV
        self.training = False


def _rotary():
    cfg = Lfm2Config(hidden_size=N_Q * D, num_attention_heads=N_Q, num_key_value_heads=N_KV,
                     rope_theta=THETA, max_position_embeddings=2 * 1048576)
    if getattr(cfg, "head_dim", None) is None:
        cfg.head_dim = D
    return hf.Lfm2RotaryEmbedding(cfg)


def _cos_sin(rot, positions):
    pos = torch.tensor([positions], dtype=torch.int64)
    dummy = torch.zeros(1, len(positions), D)
    cos, sin = rot(dummy, pos)
    return cos[0], sin[0]  # [T, D]


def main() -> None:
    torch.manual_seed(0)
    rot = _rotary()
    mod = _Module()
    out = {}
    out["inv_freq"] = rot.inv_freq.detach().numpy().astype(np.float32)
    cos, sin = _cos_sin(rot, ROPE_POSITIONS)
    out["rope_cos"] = cos.numpy()
    out["rope_sin"] = sin.numpy()

    for seed, kv_len in DECODE_CASES:
        q, k, v = inputs_decode(seed, kv_len)
        cos, sin = _cos_sin(rot, list(range(kv_len)))
        qt = torch.from_numpy(q)[None, :, None, :]           # [1, n_q, 1, d]
        kt = torch.from_numpy(k)[None]                       # [1, n_kv, T, d]
        vt = torch.from_numpy(v)[None]
        q_rot, _ = hf.apply_rotary_pos_emb(qt, qt, cos[-1:][None], sin[-1:][None])
        _, k_rot = hf.apply_rotary_pos_emb(kt, kt, cos[None], sin[None])
        o, _ = hf.eager_attention_forward(mod, q_rot, k_rot, vt, None, scaling=D ** -0.5)
        out[f"decode_{seed}_{kv_len}"] = o[0, 0].numpy()      # [n_q, d]

    for seed, t in PREFILL_CASES:
        q, k, v = inputs_prefill(seed, t)
        cos, sin = _cos_sin(rot, list(range(t)))
        qt, kt, vt = (torch.from_numpy(a)[None] for a in (q, k, v))
        q_rot, k_rot = hf.apply_rotary_pos_emb(qt, kt, cos[None], sin[None])
        mask = torch.full((t, t), float("-inf")).triu(1)[None, None]
        o, _ = hf.eager_attention_forward(mod, q_rot, k_rot, vt, mask, scaling=D ** -0.5)
        out[f"prefill_{seed}_{t}"] = o[0].transpose(0, 1).numpy()  # [n_q, T, d]

    meta = {"transformers": transformers.__version__, "torch": torch.__version__,
            "rope_positions": ROPE_POSITIONS, "decode_cases": DECODE_CASES,
            "prefill_cases": PREFILL_CASES, "n_q": N_Q, "n_kv": N_KV, "d": D, "theta": THETA}
    out["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
