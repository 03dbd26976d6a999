"""Single-kernel timing cases: one seeded input per kernel, CUDA-event timed.

    python -m llmhost_b200.kernel_cases <case> [--reps N] [--warmup W]

Each case builds its input once, launches the kernel W times untimed, then N
times back to back between one pair of CUDA events on the launching stream,
and prints one JSON line: the mean launch time, the algorithmic bytes (or
FLOPs) per launch and what they give against the measured peak in
MEASURED_PEAKS.json when that file is present.  The same command lines,
under ncu with a kernel filter, give the per-kernel profiles.

Cases (sizes above L2, 126 MB, where the kernel streams; a few GB on the
device at most):

  append       kv_append: 65 536 tokens (32 sessions x 2048, a prompt store)
               into pages drawn from a permutation, bf16 24q/8kv
  copy         kv_copy_pages: 8192 page copies (copy-on-write / compaction
               moves), bf16 32 KiB pages
  move         kv_move_tokens: the accepted-path token moves of one speculative
               round (32 sessions x 6 layers, trees of the speculative config)
  decode_f32   kv_append_decode_attn on an fp32 pool: 64 sessions, lengths
               U[128, 2048] (the CUDA-core decode kernel)
  prefill_f32  kv_prefill_attn on an fp32 pool: one 2048-token causal prompt,
               24q/8kv (the fp32 single-session configuration's prefill)
  verify       kv_prefill_attn with ancestor masks: the speculative config's
               verify launch (32 sessions sharing a 4096-token prefix, one
               64-node tree each, 24q/8kv)
  verify_shared the same launch through kv_prefill_attn_shared: the 4096
               shared tokens in one pass for all 32 sessions, then each
               session's tree, merged
  decode_q8    kv_append_decode_attn on a Q8 pool (quantise-on-append, then
  decode_k8v4  tcgen05 decode of the converted tiles; K8V4: 4-bit V): the batched-decode
               configuration's 64 session lengths (U[128, 8192]) and six
               layers' block tables taken in turn, as bench.py does
  decode_f16   the same sessions on a half (KV_DTYPE_F16) pool: the append
               fused into the tcgen05 decode, f16 operands

Algorithmic bytes: append reads k, v and writes them (4 n_kv d e per token);
a page copy reads and writes a page; a token move reads and writes one
token's K and V rows; decode counts attended K/V, the new token's K/V read and
written, q, out and block-table entries (quantised pools: codes and scales of
every attended key, 136 bytes per key and head for Q8, 104 for K8V4, against
256 for bf16).  Algorithmic FLOPs (prefill,
verify): 4 d per visible (query row, key) pair.
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path

import numpy as np

from .workloads import PAGE_TOKENS, SpecTreeWorkload, normal_bits

ROOT = Path(__file__).resolve().parent.parent
NONE = 0xFFFFFFFF


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured (MEASURED_PEAKS.json)"
    return 6650.0, 1590.0, "fallback"


class _Dev:
    def __init__(self):
        import torch

        self.torch = torch
        self.dev = torch.device("cuda", 0)
        self.rng = np.random.default_rng(2025)

    def bf16(self, shape):
        t = self.torch.from_numpy(normal_bits(self.rng, shape, "bf16").view(np.int16))
        return t.view(self.torch.bfloat16).to(self.dev)

    def f32(self, shape):
        return self.torch.from_numpy(self.rng.standard_normal(shape, dtype=np.float32)).to(self.dev)

    def i32(self, a):
        return self.torch.from_numpy(np.ascontiguousarray(a, np.int64).astype(np.int32)).to(self.dev)

    def u32(self, a):
        return self.torch.from_numpy(np.ascontiguousarray(a, np.uint32).view(np.int32)).to(self.dev)


def _tables(rng, lens, n_pages):
    """Block tables for sequences of lens[s] tokens, pages from a permutation."""
    pages = -(-np.asarray(lens) // PAGE_TOKENS)
    perm = rng.permutation(n_pages).astype(np.uint32)
    bt = np.full((len(lens), max(int(pages.max()), 1)), NONE, np.uint32)
    cur = 0
    for s, p in enumerate(pages):
        bt[s, :p] = perm[cur:cur + p]
        cur += p
    return bt


def case_append(d: _Dev):
    from .kv import KvPool

    n_seq, T, n_q, n_kv = 32, 2048, 24, 8
    lens = np.full(n_seq, T)
    n_pages = int((-(-lens // PAGE_TOKENS)).sum()) + 64
    bt = _tables(d.rng, lens, n_pages)
    pool = KvPool(dtype="bf16", n_q_heads=n_q, n_kv_heads=n_kv, n_pages=n_pages, max_positions=T + 16,
                  max_seqs=n_seq)
    n = n_seq * T
    k, v = d.bf16((n, n_kv, 64)), d.bf16((n, n_kv, 64))
    rows = d.i32(np.repeat(np.arange(n_seq), T))
    slots = d.i32(np.tile(np.arange(T), n_seq))
    bt_d = d.u32(bt)

    def launch():
        pool.append(k, v, rows, slots, slots, bt_d)

    return pool, launch, {"kernel": "append_kernel (kv_append)", "bound": "hbm",
                          "bytes": 4 * n * n_kv * 64 * 2 + 4 * 3 * n, "tokens": n}


def case_copy(d: _Dev):
    from .kv import KvPool

    n_copy, n_pages = 8192, 32768
    pool = KvPool(dtype="bf16", n_q_heads=24, n_kv_heads=8, n_pages=n_pages, max_positions=64, max_seqs=1)
    perm = d.rng.permutation(n_pages)
    src, dst = d.i32(perm[:n_copy]), d.i32(perm[n_copy:2 * n_copy])

    def launch():
        pool.copy_pages(src, dst)

    return pool, launch, {"kernel": "copy_pages_kernel (kv_copy_pages)", "bound": "hbm",
                          "bytes": 2 * n_copy * pool.page_bytes + 8 * n_copy, "pages": n_copy}


def case_move(d: _Dev):
    from .kv import KvPool
    from .plans import commit_moves, plan_forward
    from .state import KvState

    wl = SpecTreeWorkload()
    rows = wl.plan()[0]
    n, T, L = wl.n_seqs, wl.nodes, wl.n_layers
    n_pages = 8192
    st = KvState(n_pages, L, alloc_order=d.rng.permutation(n_pages).astype(np.uint32))
    st.open(0)
    st.append(0, wl.prefix)
    for s in range(1, n):
        st.fork(0, s)
    seqs = list(range(n))
    stride = -(-(wl.prefix + T + 8) // PAGE_TOKENS) + 1
    parents = np.array([r[0] for r in rows], np.int32)
    plan_forward(st, seqs, np.tile(np.arange(1000, 1000 + T, dtype=np.uint32), (n, 1)), parents, stride)
    mv, offs, _ = commit_moves(st, seqs, [list(r[1]) for r in rows])
    st.close_all()
    pool = KvPool(dtype="bf16", n_q_heads=wl.n_q, n_kv_heads=wl.n_kv, n_pages=n_pages, max_positions=64,
                  max_seqs=n)
    moves, groups = d.i32(np.asarray(mv).reshape(-1, 4)), d.i32(offs)
    n_mv = int(moves.shape[0])
    tok_bytes = 2 * wl.n_kv * 64 * 2

    def launch():
        pool.move_tokens(moves, groups)

    return pool, launch, {"kernel": "move_tokens_kernel (kv_move_tokens)", "bound": "latency (a few MB per round)",
                          "bytes": 2 * n_mv * tok_bytes + 16 * n_mv, "moves": n_mv, "groups": len(offs) - 1}


def case_decode_f32(d: _Dev):
    from .kv import KvPool

    n_q, n_kv, n_seq = 24, 8, 64
    lens = d.rng.integers(128, 2048, endpoint=True, size=n_seq)
    n_pages = int((-(-(lens + 1) // PAGE_TOKENS)).sum()) + 64
    bt = _tables(d.rng, lens + 1, n_pages)
    pool = KvPool(dtype="f32", n_q_heads=n_q, n_kv_heads=n_kv, n_pages=n_pages, max_positions=int(lens.max()) + 32,
                  max_seqs=n_seq)
    tot = int(lens.sum())
    pool.append(d.f32((tot, n_kv, 64)), d.f32((tot, n_kv, 64)), d.i32(np.repeat(np.arange(n_seq), lens)),
                d.i32(np.concatenate([np.arange(x) for x in lens])),
                d.i32(np.concatenate([np.arange(x) for x in lens])), d.u32(bt))
    q, k, v = d.f32((n_seq, n_q, 64)), d.f32((n_seq, n_kv, 64)), d.f32((n_seq, n_kv, 64))
    seq_lens = d.i32(lens + 1)
    bt_d = d.u32(bt)
    out = d.torch.empty_like(q)
    e = 4
    n_tok = lens + 1
    byts = int((2 * n_kv * 64 * e * lens + 4 * n_kv * 64 * e + 2 * n_q * 64 * e + 4 * (-(-n_tok // 16))).sum())

    def launch():
        pool.append_decode_attn(k, v, q, bt_d, seq_lens, out=out)

    return pool, launch, {"kernel": "decode_kernel<float> (kv_append_decode_attn, fp32 pool)", "bound": "hbm",
                          "bytes": byts, "sessions": n_seq, "keys": int(n_tok.sum())}


def case_prefill_f32(d: _Dev):
    from .kv import KvPool

    n_q, n_kv, T = 24, 8, 2048
    pages = T // PAGE_TOKENS
    bt = d.rng.permutation(pages + 8).astype(np.uint32)[:pages][None, :]
    pool = KvPool(dtype="f32", n_q_heads=n_q, n_kv_heads=n_kv, n_pages=pages + 8, max_positions=T + 16, max_seqs=1)
    pos = d.i32(np.arange(T))
    bt_d = d.u32(bt)
    pool.append(d.f32((T, n_kv, 64)), d.f32((T, n_kv, 64)), d.i32(np.zeros(T)), pos, pos, bt_d)
    q = d.f32((T, n_q, 64))
    q_off, prefix = d.i32([0, T]), d.i32([0])
    out = d.torch.empty_like(q)
    flops = 4.0 * 64 * n_q * T * (T + 1) / 2

    def launch():
        pool.prefill_attn(q, pos, q_off, prefix, bt_d, max_q=T, out=out)

    return pool, launch, {"kernel": "prefill_f32_kernel (kv_prefill_attn, fp32 pool)", "bound": "fp32 CUDA cores",
                          "flops": flops, "tokens": T}


def case_verify(d: _Dev, shared_pass: bool = False):
    from .kv import KvPool, tree_masks

    wl = SpecTreeWorkload()
    rows = wl.plan()[0]
    n, T, P0 = wl.n_seqs, wl.nodes, wl.prefix
    shared = P0 // PAGE_TOKENS
    own = -(-T // PAGE_TOKENS)
    n_pages = shared + n * own + 8
    perm = d.rng.permutation(n_pages).astype(np.uint32)
    bt = np.full((n, shared + own), NONE, np.uint32)
    bt[:, :shared] = perm[:shared]
    bt[:, shared:] = perm[shared:shared + n * own].reshape(n, own)
    pool = KvPool(dtype="bf16", n_q_heads=wl.n_q, n_kv_heads=wl.n_kv, n_pages=n_pages, max_positions=P0 + T + 16,
                  max_seqs=n)
    bt_d = d.u32(bt)
    pos = np.arange(P0)
    pool.append(d.bf16((P0, wl.n_kv, 64)), d.bf16((P0, wl.n_kv, 64)), d.i32(np.zeros(P0)), d.i32(pos),
                d.i32(pos), bt_d)
    depth = []
    for parents, _ in rows:
        dd = []
        for p in parents:
            dd.append(0 if p < 0 else dd[p] + 1)
        depth.append(dd)
    tok_row = np.repeat(np.arange(n), T)
    slots = np.tile(np.arange(P0, P0 + T), n)
    q_pos = (P0 + np.array(depth)).reshape(-1)
    pool.append(d.bf16((n * T, wl.n_kv, 64)), d.bf16((n * T, wl.n_kv, 64)), d.i32(tok_row), d.i32(slots),
                d.i32(q_pos), bt_d)
    masks = np.concatenate([tree_masks(r[0]) for r in rows])
    q = d.bf16((n * T, wl.n_q, 64))
    q_pos_d, q_off = d.i32(q_pos), d.i32(np.arange(n + 1) * T)
    prefix = d.i32(np.full(n, P0))
    masks_d = d.torch.from_numpy(masks).to(d.dev)
    out = d.torch.empty_like(q)
    ones = np.unpackbits(masks.view(np.uint8)).reshape(-1, 64).sum(axis=1)
    flops = 4.0 * 64 * wl.n_q * float((P0 + ones).sum())
    kv_bytes = 2 * wl.n_kv * 64 * 2 * (P0 * n + n * T)

    if shared_pass:
        ws = pool.prefill_shared_workspace(n, T)

        def launch():
            pool.prefill_attn_shared(q, q_pos_d, q_off, prefix, bt_d, shared_tokens=shared * PAGE_TOKENS, max_q=T,
                                     tree_masks=masks_d, workspace=ws, out=out)

        return pool, launch, {"kernel": "prefill_kernel x 2 (kv_prefill_attn_shared: shared-prefix pass, then "
                                        "each session's keys merged)", "bound": "tensor", "flops": flops,
                              "kv_bytes_streamed": 2 * wl.n_kv * 64 * 2 * (P0 + n * T), "sessions": n, "nodes": T}

    def launch():
        pool.prefill_attn(q, q_pos_d, q_off, prefix, bt_d, tree_masks=masks_d, max_q=T, out=out)

    return pool, launch, {"kernel": "prefill_kernel (kv_prefill_attn, tree masks, tcgen05)", "bound": "tensor",
                          "flops": flops, "kv_bytes_streamed": kv_bytes, "sessions": n, "nodes": T}


def case_verify_shared(d: _Dev):
    return case_verify(d, shared_pass=True)


def _decode_quant(d: _Dev, store: str):
    from .kv import KvPool
    from .workloads import decode_config

    wl = decode_config()
    n_q, n_kv, n_seq, n_layers = wl.n_q, wl.n_kv, wl.n_seqs, wl.n_layers
    lens = np.asarray(wl.l0, np.int64)
    per_layer = int((-(-(lens + 1) // PAGE_TOKENS)).sum())
    n_pages = n_layers * per_layer + 64
    perm = d.rng.permutation(n_pages).astype(np.uint32)
    pool = KvPool(dtype=store, n_q_heads=n_q, n_kv_heads=n_kv, n_pages=n_pages, max_positions=int(lens.max()) + 32,
                  max_seqs=n_seq)
    tot = int(lens.sum())
    rows = d.i32(np.repeat(np.arange(n_seq), lens))
    slots = d.i32(np.concatenate([np.arange(x) for x in lens]))
    tables = []
    for layer in range(n_layers):  # disjoint pages per layer
        bt = _tables(np.random.default_rng(layer), lens + 1, per_layer)
        bt = np.where(bt == NONE, NONE, perm[layer * per_layer:(layer + 1) * per_layer][np.minimum(bt, per_layer - 1)])
        tables.append(d.u32(bt))
        k, v = d.bf16((tot, n_kv, 64)), d.bf16((tot, n_kv, 64))
        pool.append(k, v, rows, slots, slots, tables[-1])
        del k, v
    q, k, v = d.bf16((n_seq, n_q, 64)), d.bf16((n_seq, n_kv, 64)), d.bf16((n_seq, n_kv, 64))
    seq_lens = d.i32(lens + 1)
    out = d.torch.empty_like(q)
    n_tok = lens + 1
    if store == "f16":  # half pages: the bf16 byte count (the fused append reads and writes the new row)
        byts = int((n_kv * 256 * n_tok + 2 * n_kv * 64 * 4 + 2 * n_q * 64 * 2 + 4 * (-(-n_tok // 16))).sum())
    else:
        key_bytes = 64 + (64 if store == "q8" else 32) + 8
        byts = int((n_kv * key_bytes * n_tok + 2 * n_kv * 64 * 2 + 2 * n_q * 64 * 2
                    + 4 * (-(-n_tok // 16))).sum())
    state = {"i": 0}

    def launch():
        pool.append_decode_attn(k, v, q, tables[state["i"] % n_layers], seq_lens, out=out)
        state["i"] += 1

    kernel = ("decode_tc_kernel, append fused, f16 operands (f16 pool)" if store == "f16" else
              f"append_q_kernel + decode_tc_kernel with converter warps ({store} pool)")
    return pool, launch, {"kernel": kernel,
                          "bound": "hbm", "bytes": byts, "sessions": n_seq, "keys": int(n_tok.sum()),
                          "layers_in_turn": n_layers, "bf16_equivalent_bytes":
                              int((n_kv * 256 * n_tok + 2 * n_kv * 64 * 4 + 2 * n_q * 64 * 2
                                   + 4 * (-(-n_tok // 16))).sum())}


def case_decode_q8(d: _Dev):
    return _decode_quant(d, "q8")


def case_decode_k8v4(d: _Dev):
    return _decode_quant(d, "k8v4")


def case_decode_f16(d: _Dev):
    return _decode_quant(d, "f16")


CASES = {"append": case_append, "copy": case_copy, "move": case_move, "decode_f32": case_decode_f32,
         "prefill_f32": case_prefill_f32, "verify": case_verify, "verify_shared": case_verify_shared,
         "decode_q8": case_decode_q8,
         "decode_k8v4": case_decode_k8v4, "decode_f16": case_decode_f16}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=sorted(CASES))
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args()
    d = _Dev()
    torch = d.torch
    pool, launch, info = CASES[args.case](d)
    torch.cuda.synchronize()
    pool.check_device_error()
    for _ in range(args.warmup):
        launch()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream()
    e0.record(stream)
    for _ in range(args.reps):
        launch()
    e1.record(stream)
    torch.cuda.synchronize()
    pool.check_device_error()
    us = e0.elapsed_time(e1) * 1e3 / max(args.reps, 1)
    hbm, tflops, kind = _peaks()
    line = {"case": args.case, "launch_us": us, "reps": args.reps, "warmup": args.warmup, **info}
    if "bytes" in info:
        gbs = info["bytes"] / (us * 1e-6) / 1e9
        line.update(achieved_gbs=gbs, hbm_peak_gbs=hbm, frac_of_hbm=gbs / hbm, peak_kind=kind)
    if "flops" in info:
        tf = info["flops"] / (us * 1e-6) / 1e12
        line.update(achieved_tflops=tf)
        if info["bound"] == "tensor":
            line.update(bf16_peak_tflops=tflops, frac_of_tensor=tf / tflops, peak_kind=kind)
    if "kv_bytes_streamed" in info:
        line.update(kv_gbs=info["kv_bytes_streamed"] / (us * 1e-6) / 1e9)
    print(json.dumps(line), flush=True)
    pool.close()


if __name__ == "__main__":
    main()
