"""Benchmark: paged decode attention + append on the batched-decode workload.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (one GPU's share; sessions are independent, so N GPUs run N
independent batches -- weak scaling, no collective on the data path):
64 sessions, cached lengths uniform in [128, 8192] (seed 1 + 1000*rank), bf16,
24 query / 8 KV heads, head_dim 64, page 16, pages drawn in order from a seeded
permutation of a 2^20-page pool, 6 attention layers.  A step is one token per
session through all 6 layers: per layer one kv_append_decode plus one
kv_decode_attn.  The 512-step schedule is replayed cyclically when K + W > 512.

Reported: tokens/s over all ranks (value), the device-timed step, the
decode-attention kernel's achieved HBM GB/s against MEASURED_PEAKS.json
(roofline), an end-to-end pass through the public API with pinned host inputs
and outputs (e2e), and the CPU oracle timed on this host (cpu_baseline).
The K/V working set (~3.5 GB per step) is far larger than L2 (126 MB), so no
explicit flush is needed between steps.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode attn+append tokens/s and HBM GB/s (% peak) at 1/2/4/8 B200 vs CPU path"
UNIT = "tokens/s"
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1024)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=12.0, help="seconds of CPU-baseline work")
    ap.add_argument("--schedule", type=int, default=512, help="decode steps in the workload")
    ap.add_argument("--layers", type=int, default=6, help="attention layers (6 in the workload)")
    ap.add_argument("--pool-pages", type=int, default=1 << 20,
                    help="pool size in pages (2^20 in the workload; smaller only for profiling)")
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def load_traffic_ratio():
    """DRAM bytes / algorithmic bytes of the decode kernel from the committed ncu summary."""
    p = ROOT / "profiles" / "decode_attn_traffic.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["dram_bytes_per_launch"]) / float(d["algorithmic_bytes_per_launch"]), d
    return None, None


# ---------------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------------
def cpu_baseline(wl, budget_s: float, max_steps: int | None = None, sessions_per_step: int | None = None):
    """The CPU oracle (restated reference attention) on a bounded sample of the
    workload: one layer of the first decode step for `sessions_per_step`
    sessions, repeated until `budget_s` elapses (or max_steps), on every host
    thread.  Returns tokens/s extrapolated to the 6-layer step."""
    from oracle import oracle as O
    from llmhost_b200.workloads import normal_bits

    rng = np.random.default_rng(99)
    n = wl.n_seqs
    sessions_per_step = sessions_per_step or n
    lens0 = wl.seq_lens(0)
    need = -(-lens0 // 16)
    total = int(need.sum())
    # compact host pool for layer 0 of every session
    bt = np.full((n, int(need.max())), 0xFFFFFFFF, np.uint32)
    cur = 0
    for s in range(n):
        bt[s, :need[s]] = np.arange(cur, cur + need[s], dtype=np.uint32)
        cur += need[s]
    dt = O.BF16 if wl.dtype == "bf16" else O.F32
    host = O.HostPages(total, dt, wl.n_q, wl.n_kv, theta=wl.rope_theta,
                       data=normal_bits(rng, (total, 2 * wl.n_kv * 16 * 64), wl.dtype))
    q = normal_bits(rng, (n, wl.n_q, 64), wl.dtype)
    k = normal_bits(rng, (n, wl.n_kv, 64), wl.dtype)
    v = normal_bits(rng, (n, wl.n_kv, 64), wl.dtype)
    threads = O.max_threads()
    done_tokens, elapsed, steps = 0, 0.0, 0
    start = 0
    while True:
        idx = (np.arange(sessions_per_step) + start) % n
        start += sessions_per_step
        t0 = time.perf_counter()
        host.decode_step(bt[idx], lens0[idx], wl.window, q[idx], k[idx], v[idx], n_threads=threads)
        elapsed += time.perf_counter() - t0
        done_tokens += len(idx)
        steps += 1
        if (max_steps and steps >= max_steps) or (not max_steps and elapsed >= budget_s):
            break
    tokens_per_s = done_tokens / (elapsed * wl.n_layers)
    sample = (f"{steps} x [{sessions_per_step} sessions x 1 layer] of decode step 0 "
              f"(append + attention, lengths {int(lens0.min())}-{int(lens0.max())}), "
              f"extrapolated to {wl.n_layers} layers")
    return tokens_per_s, threads, sample, elapsed


def host_info():
    cpu = ""
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                cpu = ln.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    try:
        load = float(open("/proc/loadavg").read().split()[0])
    except OSError:
        load = None
    return {"cpu_model": cpu, "nproc": os.cpu_count(), "loadavg": load}


# ---------------------------------------------------------------------------------
def run_reference(args, rank: int, world: int):
    from llmhost_b200.workloads import decode_config

    if rank != 0:
        return
    wl = decode_config(steps=args.schedule, seed=1)
    # Size one reference step so that the whole run stays within ~2 minutes.
    probe_tps, threads, _, probe_el = cpu_baseline(wl, 0.0, max_steps=1, sessions_per_step=8)
    per_session = probe_el / 8
    total_steps = args.steps + args.warmup
    sps = int(max(1, min(wl.n_seqs, 120.0 / max(total_steps * per_session, 1e-9))))
    if args.warmup:
        cpu_baseline(wl, 0.0, max_steps=args.warmup, sessions_per_step=sps)
    tps, threads, sample, elapsed = cpu_baseline(wl, 0.0, max_steps=args.steps, sessions_per_step=sps)
    line = {
        "impl": "reference", "metric": METRIC, "value": tps, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": elapsed / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": wl.dtype, "data": "synthetic",
        "config": {"workload": wl.name, "sessions": wl.n_seqs, "layers": wl.n_layers,
                   "q_heads": wl.n_q, "kv_heads": wl.n_kv, "head_dim": 64, "page_tokens": 16},
        "cpu_baseline": {"value": tps, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": tps, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "host": host_info(),
        "note": "reference is Rust with no toolchain here; this is the C restatement of its CPU attention",
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------
def run_ours(args, rank: int, world: int, local_rank: int):
    import torch
    import torch.distributed as dist

    from llmhost_b200.kv import KvPool
    from llmhost_b200.workloads import decode_config

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    wl = decode_config(steps=args.schedule, seed=1 + 1000 * rank, n_layers=args.layers,
                       pool_pages=args.pool_pages)
    n, L = wl.n_seqs, wl.n_layers
    S = wl.steps
    max_pos = int(wl.l0.max()) + S + 16
    pool = KvPool(dtype=wl.dtype, n_q_heads=wl.n_q, n_kv_heads=wl.n_kv, n_pages=wl.pool_pages,
                  rope_theta=wl.rope_theta, max_positions=max_pos, max_seqs=n, device=local_rank)
    tdt = pool.shape.torch_dtype
    bt_dev = [torch.from_numpy(wl.block_tables[l].view(np.int32)).to(dev) for l in range(L)]
    lens_dev = torch.from_numpy(np.stack([wl.seq_lens(t) for t in range(S)])).to(dev)  # [S, n]

    # Fill the cached K/V of every layer through kv_append (prefill path).
    gen = torch.Generator(device=dev)
    gen.manual_seed(7 + rank)
    chunk_tokens = 1 << 16
    tok_seq = torch.from_numpy(np.concatenate([np.full(int(x), s, np.int32) for s, x in enumerate(wl.l0)])).to(dev)
    tok_pos = torch.from_numpy(np.concatenate([np.arange(int(x), dtype=np.int32) for x in wl.l0])).to(dev)
    for l in range(L):
        for a in range(0, tok_seq.numel(), chunk_tokens):
            b = min(a + chunk_tokens, tok_seq.numel())
            k = torch.randn((b - a, wl.n_kv, 64), generator=gen, device=dev, dtype=torch.float32).to(tdt)
            v = torch.randn((b - a, wl.n_kv, 64), generator=gen, device=dev, dtype=torch.float32).to(tdt)
            pool.append(k, v, tok_seq[a:b], tok_pos[a:b], tok_pos[a:b], bt_dev[l])
    torch.cuda.synchronize()
    pool.check_device_error()

    # Device-resident per-step inputs (a ring of n_sets distinct steps).
    n_sets = min(64, S)
    qkv_shape = (n_sets, L, n, wl.n_q + 2 * wl.n_kv, 64)
    qkv = torch.randn(qkv_shape, generator=gen, device=dev, dtype=torch.float32).to(tdt)
    q_in = qkv[..., :wl.n_q, :]
    k_in = qkv[..., wl.n_q:wl.n_q + wl.n_kv, :]
    v_in = qkv[..., wl.n_q + wl.n_kv:, :]
    q_c = [[q_in[i, l].contiguous() for l in range(L)] for i in range(n_sets)]
    k_c = [[k_in[i, l].contiguous() for l in range(L)] for i in range(n_sets)]
    v_c = [[v_in[i, l].contiguous() for l in range(L)] for i in range(n_sets)]
    out = [torch.empty((n, wl.n_q, 64), device=dev, dtype=tdt) for _ in range(L)]
    stream = torch.cuda.current_stream()

    def step(t, ev=None):
        i = t % n_sets
        lens = lens_dev[t % S]
        for l in range(L):
            pool.append_decode(k_c[i][l], v_c[i][l], bt_dev[l], lens, stream=stream)
            if ev is not None:
                ev[l][0].record(stream)
            pool.decode_attn(q_c[i][l], bt_dev[l], lens, out=out[l], stream=stream)
            if ev is not None:
                ev[l][1].record(stream)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # warm-up
    for t in range(args.warmup):
        step(t)
    torch.cuda.synchronize()
    pool.check_device_error()

    # ---- device-timed region ----
    K = args.steps
    kev = [[[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in range(L)]
           for _ in range(K)]
    sampler = ClockSampler(local_rank)
    sampler.start()
    barrier()
    torch.cuda.synchronize()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(K):
        step(args.warmup + i, kev[i])
    t_end.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    pool.check_device_error()
    ms_local = t_start.elapsed_time(t_end)
    ms = max_over_ranks(ms_local)
    kernel_ms = [kev[i][l][0].elapsed_time(kev[i][l][1]) for i in range(K) for l in range(L)]
    attn_bytes = [wl.attn_bytes((args.warmup + i) % S) for i in range(K) for _ in range(L)]
    step_bytes = [wl.step_bytes((args.warmup + i) % S) for i in range(K)]
    tokens = n * K * world
    value = tokens / (ms / 1e3)
    ms_per_step = ms / K

    hbm, peak_kind = peaks()
    mean_kernel_s = float(np.mean(kernel_ms)) / 1e3
    mean_attn_bytes = float(np.mean(attn_bytes))
    achieved = mean_attn_bytes / mean_kernel_s / 1e9
    ratio, prof = load_traffic_ratio()
    roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                "traffic": (ratio * mean_attn_bytes) if ratio else None,
                "kernel": "decode_kernel (kv_decode_attn)",
                "algorithmic_bytes_per_launch": mean_attn_bytes,
                "mean_launch_us": mean_kernel_s * 1e6,
                "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                else "fallback 6.65 TB/s"}
    step_gbs = float(np.mean(step_bytes)) / (ms_per_step / 1e3) / 1e9

    # ---- end-to-end pass through the public API with host buffers ----
    e2e = None
    if not args.no_e2e:
        Ke = min(K, 256)
        pin_q = [[q_c[i % n_sets][l].cpu().pin_memory() for l in range(L)] for i in range(n_sets)]
        pin_k = [[k_c[i % n_sets][l].cpu().pin_memory() for l in range(L)] for i in range(n_sets)]
        pin_v = [[v_c[i % n_sets][l].cpu().pin_memory() for l in range(L)] for i in range(n_sets)]
        pin_lens = torch.from_numpy(np.stack([wl.seq_lens(t) for t in range(S)])).pin_memory()
        pin_out = [torch.empty((n, wl.n_q, 64), dtype=tdt).pin_memory() for _ in range(L)]
        dq = [torch.empty_like(q_c[0][0]) for _ in range(L)]
        dk = [torch.empty_like(k_c[0][0]) for _ in range(L)]
        dv = [torch.empty_like(v_c[0][0]) for _ in range(L)]
        dlens = torch.empty(n, dtype=torch.int32, device=dev)

        def e2e_step(t):
            i = t % n_sets
            dlens.copy_(pin_lens[t % S], non_blocking=True)
            for l in range(L):
                dq[l].copy_(pin_q[i][l], non_blocking=True)
                dk[l].copy_(pin_k[i][l], non_blocking=True)
                dv[l].copy_(pin_v[i][l], non_blocking=True)
                pool.append_decode(dk[l], dv[l], bt_dev[l], dlens, stream=stream)
                pool.decode_attn(dq[l], bt_dev[l], dlens, out=out[l], stream=stream)
                pin_out[l].copy_(out[l], non_blocking=True)

        for t in range(3):
            e2e_step(t)
        torch.cuda.synchronize()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(Ke):
            e2e_step(args.warmup + i)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        e_ms = max_over_ranks(e0.elapsed_time(e1))
        esz = pool.shape.torch_dtype.itemsize
        h2d = L * n * (wl.n_q + 2 * wl.n_kv) * 64 * esz + n * 4
        d2h = L * n * wl.n_q * 64 * esz
        e2e = {"value": n * Ke * world / (e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "steps": Ke,
               "path": "pinned host q/k/v -> KvPool.append_decode + decode_attn (C ABI) -> pinned host out"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tps, threads, sample, _ = cpu_baseline(wl, args.cpu_budget)
        cpu = {"value": tps, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample,
               "host": host_info()}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": wl.name if (L == 6 and wl.pool_pages == 1 << 20) else
                       f"{wl.name} (reduced: {L} layers, {wl.pool_pages} pages)",
                       "sessions_per_gpu": n, "layers": L, "q_heads": wl.n_q,
                       "kv_heads": wl.n_kv, "head_dim": 64, "page_tokens": 16,
                       "pool_pages": wl.pool_pages, "schedule_steps": S,
                       "lengths": "uniform [128, 8192] + step",
                       "l2": "no flush: K/V read per step (~3.5 GB) >> 126 MB L2",
                       "parallelism": f"batch-sharded x{world} (independent sessions per GPU)"},
            "step_gbs": step_gbs, "step_frac_of_peak": step_gbs / hbm,
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": K * L * 2, "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    pool.close()


def main():
    args = parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
