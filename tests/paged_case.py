"""Seeded paged-KV cases run through both the CUDA library and the CPU oracle.

A case is a batch of sequences with `lens[s]` cached tokens, pages drawn from a
seeded permutation of a small pool.  The cached tokens are written with
kv_append (GPU) and orc_paged_append_token (oracle) from the same k/v bits;
then one decode step appends one more token per sequence and runs decode
attention.  The oracle is only the checker here.
"""
from __future__ import annotations

import numpy as np

from llmhost_b200.workloads import PAGE_TOKENS, normal_bits
from oracle import oracle as O

PAGE_NONE = 0xFFFFFFFF


def to_torch(bits: np.ndarray, dtype: str, device):
    import torch

    if dtype == "bf16":
        t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)
    else:
        t = torch.from_numpy(np.ascontiguousarray(bits, dtype=np.float32))
    return t.to(device)


def to_numpy_f32(t) -> np.ndarray:
    import torch

    return t.detach().to(torch.float32).cpu().numpy()


ORACLE_DTYPE = {"bf16": O.BF16, "f32": O.F32, "q8": O.Q8, "k8v4": O.K8V4, "f16": O.F16}


class DecodeCase:
    """`dtype` is the k / v / q type; `store` the pool's storage type when it
    differs (half pools "f16" and quantised pools "q8" / "k8v4" take bf16 k, v, q)."""

    def __init__(self, dtype: str, n_q: int, n_kv: int, lens, seed: int = 0, window: int = 0,
                 extra_pages: int = 8, evict_below_window: bool = False, store: str | None = None):
        rng = np.random.default_rng(seed)
        self.dtype, self.n_q, self.n_kv, self.window = dtype, n_q, n_kv, window
        self.store = store or dtype
        self.lens = np.asarray(lens, dtype=np.int64)
        n = len(self.lens)
        pages = -(-(self.lens + 1) // PAGE_TOKENS)
        self.n_pages = int(pages.sum()) + extra_pages
        perm = rng.permutation(self.n_pages).astype(np.uint32)
        self.max_pages = max(int(pages.max()) if n else 1, 1)
        self.bt = np.full((n, self.max_pages), PAGE_NONE, np.uint32)
        cur = 0
        for s in range(n):
            self.bt[s, :pages[s]] = perm[cur:cur + pages[s]]
            cur += pages[s]
        self.k_pre = [normal_bits(rng, (int(L), n_kv, 64), dtype) for L in self.lens]
        self.v_pre = [normal_bits(rng, (int(L), n_kv, 64), dtype) for L in self.lens]
        self.q = normal_bits(rng, (n, n_q, 64), dtype)
        self.k_new = normal_bits(rng, (n, n_kv, 64), dtype)
        self.v_new = normal_bits(rng, (n, n_kv, 64), dtype)
        self.seq_lens = (self.lens + 1).astype(np.int32)
        # Block table the kernels see: pages wholly below the window may be
        # marked evicted; attention must never touch them.
        self.bt_attn = self.bt.copy()
        if evict_below_window and window:
            for s in range(n):
                lo = max(int(self.seq_lens[s]) - window, 0)
                self.bt_attn[s, :lo // PAGE_TOKENS] = PAGE_NONE

    # ---- oracle -------------------------------------------------------------
    def run_oracle(self, norm=None):
        """norm = (q_norm, k_norm, eps): the decode step RMS-normalises q and
        the new k before RoPE (orc_decode_step_norm)."""
        host = O.HostPages(self.n_pages, ORACLE_DTYPE[self.store], self.n_q, self.n_kv)
        for s in range(len(self.lens)):
            for t in range(int(self.lens[s])):
                host.append_token(self.bt[s], t, t, self.k_pre[s][t], self.v_pre[s][t])
        if norm is None:
            out = host.decode_step(self.bt_attn, self.seq_lens, self.window, self.q, self.k_new, self.v_new)
        else:
            out = host.decode_step_norm(self.bt_attn, self.seq_lens, self.window, self.q, self.k_new, self.v_new,
                                        *norm)
        return host, out

    # ---- CUDA library ----------------------------------------------------------
    def make_pool(self, **kw):
        from llmhost_b200.kv import KvPool

        args = dict(dtype=self.store, n_q_heads=self.n_q, n_kv_heads=self.n_kv, n_pages=self.n_pages,
                    max_positions=int(self.seq_lens.max(initial=1)) + 16, max_seqs=max(len(self.lens), 1))
        args.update(kw)
        return KvPool(**args)

    def prefill_gpu(self, pool) -> None:
        import torch

        dev = pool.device
        if self.lens.sum() == 0:
            return
        tok_seq = np.concatenate([np.full(int(L), s, np.int32) for s, L in enumerate(self.lens)])
        tok_slot = np.concatenate([np.arange(int(L), dtype=np.int32) for L in self.lens])
        k = np.concatenate([a.reshape(-1) for a in self.k_pre])
        v = np.concatenate([a.reshape(-1) for a in self.v_pre])
        bt = torch.from_numpy(self.bt.view(np.int32)).to(dev)
        ts = torch.from_numpy(tok_seq).to(dev)
        tl = torch.from_numpy(tok_slot).to(dev)
        pool.append(to_torch(k, self.dtype, dev), to_torch(v, self.dtype, dev), ts, tl, tl, bt)

    def decode_norm_gpu(self, pool, norm):
        """kv_norm_append_decode_attn on the attention's block tables."""
        import torch

        dev = pool.device
        qw, kw, eps = norm
        out = pool.norm_append_decode_attn(
            to_torch(self.k_new, self.dtype, dev), to_torch(self.v_new, self.dtype, dev),
            to_torch(self.q, self.dtype, dev), torch.from_numpy(qw).to(dev), torch.from_numpy(kw).to(dev), eps,
            torch.from_numpy(self.bt_attn.view(np.int32)).to(dev), torch.from_numpy(self.seq_lens).to(dev),
            window=self.window)
        torch.cuda.synchronize()
        return out

    def decode_gpu(self, pool, repeat: int = 1, fused: bool = False):
        """Append the new token and attend; `fused` does both in one
        kv_append_decode_attn launch (on the attention's block tables: the
        new token's page is never below the window)."""
        import torch

        dev = pool.device
        bt = torch.from_numpy(self.bt.view(np.int32)).to(dev)
        bt_attn = torch.from_numpy(self.bt_attn.view(np.int32)).to(dev)
        lens = torch.from_numpy(self.seq_lens).to(dev)
        k = to_torch(self.k_new, self.dtype, dev)
        v = to_torch(self.v_new, self.dtype, dev)
        q = to_torch(self.q, self.dtype, dev)
        if fused:
            out = pool.append_decode_attn(k, v, q, bt_attn, lens, window=self.window)
            repeat -= 1
        else:
            pool.append_decode(k, v, bt, lens)
        for _ in range(repeat):
            out = pool.decode_attn(q, bt_attn, lens, window=self.window)
        torch.cuda.synchronize()
        return out

    def used_pages(self) -> np.ndarray:
        ids = self.bt[self.bt != PAGE_NONE]
        return np.sort(ids)


def truth_decode(host, bt, seq_lens, window, q_raw, dtype: str) -> np.ndarray:
    """float64 decode attention on the oracle's stored pages (q rotated by the
    oracle in fp32, as the kernels do), to measure how far each fp32 path is
    from exact arithmetic."""
    n = len(seq_lens)
    out = np.empty((n, host.n_q, host.d), np.float64)
    g = host.n_q // host.n_kv
    for s in range(n):
        L = int(seq_lens[s])
        k, v = host.gather(bt[s], L)
        q = (O.bf16_bits_to_f32(q_raw[s]) if dtype == "bf16" else np.asarray(q_raw[s], np.float32)).copy()
        c, sn = O.cos_sin(host.inv, L - 1, 1, host.d)
        O.apply_rope_in_place(q, c, sn, host.n_q, 1, host.d)
        lo = max(L - window, 0) if window else 0
        for h in range(host.n_q):
            kk = k[h // g, lo:L].astype(np.float64)
            vv = v[h // g, lo:L].astype(np.float64)
            sc = kk @ q[h].astype(np.float64) / np.sqrt(host.d)
            w = np.exp(sc - sc.max())
            out[s, h] = (w / w.sum()) @ vv
    return out


def assert_close_rows(got: np.ndarray, ref: np.ndarray, rtol: float, what: str = "") -> float:
    """Normwise per-row check: max|got-ref| <= rtol * max|ref| for every row."""
    got = np.asarray(got, np.float64).reshape(-1, ref.shape[-1])
    ref = np.asarray(ref, np.float64).reshape(-1, ref.shape[-1])
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    err = O.rel_err_rows(got, ref)
    worst = float(err.max(initial=0.0))
    assert worst <= rtol, f"{what}: worst normwise row error {worst:.3e} > {rtol:.1e} (row {int(err.argmax())})"
    return worst
