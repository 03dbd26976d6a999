"""Benchmark: paged decode attention + append on the batched-decode workload.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (one GPU's share; sessions are independent, so N GPUs run N
batches -- weak scaling, no collective on the data path): 64 sessions per
GPU, cached lengths uniform in [128, 8192] (seed 1; the job holds those 64
lengths once per GPU and LPT on length hands each GPU one session of every
length, so per-GPU work is the same at every N), bf16,
24 query / 8 KV heads, head_dim 64, page 16, pages drawn in order from a seeded
permutation of a 2^20-page pool, 6 attention layers.  A step is one token per
session through all 6 layers: per layer one kv_append_decode_attn (the
token's K/V append and the attention in one launch; --unfused runs
kv_append_decode then kv_decode_attn).  The 512-step schedule is replayed
cyclically when K + W > 512.

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

# NCCL's log lines go to stderr unless the caller chose a file (read when NCCL
# first initialises, which importing torch.distributed can trigger)
os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")


class _stdout_to_stderr:
    """File descriptor 1 redirected to descriptor 2 for the duration (output
    written by native code included)."""

    def __enter__(self):
        sys.stdout.flush()
        self.saved = os.dup(1)
        os.dup2(2, 1)
        return self

    def __exit__(self, *exc):
        sys.stdout.flush()
        os.dup2(self.saved, 1)
        os.close(self.saved)
        return False


ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode attn+append tokens/s and HBM GB/s (% peak) at 1/2/4/8 B200 vs CPU path"
UNIT = "tokens/s"
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--workload", choices=["decode", "single", "prefill", "spec", "longctx"], default="decode",
                    help="decode: the headline batched decode; single: fp32 single session (prefill 2048 + "
                         "256 decode); prefill: bf16 chunked prefill; spec: speculative tree rounds; "
                         "longctx: long context with a sliding window (+ the 1M-token session shard)")
    ap.add_argument("--steps", type=int, default=None, help="timed steps (default per workload)")
    ap.add_argument("--warmup", type=int, default=None, help="untimed warm-up steps (default per workload)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--unfused", action="store_true",
                    help="decode workloads: kv_append_decode + kv_decode_attn as two launches per layer")
    ap.add_argument("--qk-norm", action="store_true",
                    help="decode workload: kv_norm_append_decode_attn (the layer's q/k RMSNorm folded in)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=12.0, help="seconds of CPU-baseline work")
    ap.add_argument("--schedule", type=int, default=512, help="decode steps in the workload")
    ap.add_argument("--layers", type=int, default=6, help="attention layers (6 in the workload)")
    ap.add_argument("--prefill-start-chunk", type=int, default=0,
                    help="prefill workload: chunk of the first warm-up step (profiling a long-prefix chunk)")
    ap.add_argument("--pool-pages", type=int, default=1 << 20,
                    help="pool size in pages (2^20 in the workload; smaller only for profiling)")
    args = ap.parse_args()
    defaults = {"decode": (1024, 16), "single": (5, 3), "prefill": (32, 3), "spec": (64, 3), "longctx": (256, 8)}
    k, w = defaults[args.workload]
    args.steps = k if args.steps is None else args.steps
    args.warmup = w if args.warmup is None else args.warmup
    return args


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
    wl = decode_config(steps=args.schedule, seed=1, n_layers=args.layers, pool_pages=args.pool_pages,
                       world=world, rank=rank)
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

    fused = not args.unfused
    qk_norm = args.qk_norm and fused
    if qk_norm:  # per-layer RMSNorm weights, as the attention layer's q_norm / k_norm
        qn_w = [torch.empty(64, device=dev).uniform_(0.5, 1.5, generator=gen) for _ in range(L)]
        kn_w = [torch.empty(64, device=dev).uniform_(0.5, 1.5, generator=gen) for _ in range(L)]

    def step(t, ev=None):
        i = t % n_sets
        lens = lens_dev[t % S]
        for l in range(L):
            if fused:
                if ev is not None:
                    ev[l][0].record(stream)
                if qk_norm:
                    pool.norm_append_decode_attn(k_c[i][l], v_c[i][l], q_c[i][l], qn_w[l], kn_w[l], 1e-5, bt_dev[l],
                                                 lens, out=out[l], stream=stream)
                else:
                    pool.append_decode_attn(k_c[i][l], v_c[i][l], q_c[i][l], bt_dev[l], lens, out=out[l],
                                            stream=stream)
            else:
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
    # Nothing but the decode launches goes into the stream between the two
    # events, so the launches run back to back as in serving (each one's
    # set-up overlaps the previous one's tail through programmatic dependent
    # launch) and the region's time per launch is the kernel's own.
    K = args.steps
    sampler = ClockSampler(local_rank)
    sampler.start()
    barrier()
    torch.cuda.synchronize()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(K):
        step(args.warmup + i)
    t_end.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    pool.check_device_error()
    ms_local = t_start.elapsed_time(t_end)
    ms = max_over_ranks(ms_local)
    launches = K * L * (1 if fused else 2)
    # The fused launch moves the whole layer's algorithmic bytes (append
    # included); the plain decode launch only the attention's.
    step_bytes = [wl.step_bytes((args.warmup + i) % S) for i in range(K)]
    attn_bytes = [(step_bytes[i] / L if fused else wl.attn_bytes((args.warmup + i) % S)) for i in range(K)]
    tokens = n * K * world
    value = tokens / (ms / 1e3)
    ms_per_step = ms / K

    # Per-rank figures (all ranks take part in the same collective).
    per_rank = [[float(sum(step_bytes)) / K, ms_local, float(n)]]
    if world > 1:
        mine = torch.tensor(per_rank[0], device=dev, dtype=torch.float64)
        allr = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(allr, mine)
        per_rank = [t.tolist() for t in allr]

    hbm, peak_kind = peaks()
    launch_s = ms_local / 1e3 / launches if fused else None
    mean_attn_bytes = float(np.mean(attn_bytes))
    # A separate, untimed pass brackets single launches with events: a note
    # only, since an event between two launches stops the next one's set-up
    # from overlapping (the sampled launches read a little long).
    n_sample = min(16, K)
    kev = [[[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in range(L)]
           for _ in range(n_sample)]
    for i in range(n_sample):
        step(args.warmup + K + i, kev[i])
    torch.cuda.synchronize()
    pool.check_device_error()
    sampled_us = float(np.mean([e[0].elapsed_time(e[1]) for r in kev for e in r])) * 1e3
    if not fused:  # two launches per layer: the decode launch's time comes from the sampled pass
        launch_s = sampled_us / 1e6
    achieved = mean_attn_bytes / launch_s / 1e9
    ratio, prof = load_traffic_ratio()
    roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                "traffic": (ratio * mean_attn_bytes) if ratio else None,
                "kernel": ("decode_tc_kernel (kv_norm_append_decode_attn: q/k RMSNorm + append + attention, "
                           "one launch per layer)") if qk_norm
                else "decode_tc_kernel (kv_append_decode_attn: append + attention, one launch per layer)"
                if fused else "decode_tc_kernel (kv_decode_attn)",
                "algorithmic_bytes_per_launch": mean_attn_bytes,
                "mean_launch_us": launch_s * 1e6,
                "launch_time": ("timed region / launches: the region holds only these launches, back to back"
                                if fused else "sampled launches (events around each decode launch)"),
                "launches_timed": launches,
                "sampled_launch_us": sampled_us,
                "sampled_note": f"{n_sample} untimed steps with events around every launch (breaks the "
                                "launch overlap, so a little long)",
                "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                else "fallback 6.65 TB/s"}
    step_gbs = float(np.mean(step_bytes)) / (ms_per_step / 1e3) / 1e9

    # ---- end-to-end pass through the public API with host buffers ----
    # Each step's inputs for all layers sit in one pinned block ([layer][q | k
    # | v] and the step's seq_lens) and go over in one copy; the outputs of all
    # layers come back in one copy.  A copy stream moves step t+1's inputs and
    # step t-1's outputs while step t computes (two device buffers each way).
    e2e = None
    if not args.no_e2e:
        Ke = min(K, 256)
        qn, kn = n * wl.n_q * 64, n * wl.n_kv * 64
        per_layer = qn + 2 * kn
        pin_in = []
        for i in range(n_sets):
            blk = torch.empty(L * per_layer, dtype=tdt).pin_memory()
            for l in range(L):
                b0 = l * per_layer
                blk[b0:b0 + qn].copy_(q_c[i][l].reshape(-1).cpu())
                blk[b0 + qn:b0 + qn + kn].copy_(k_c[i][l].reshape(-1).cpu())
                blk[b0 + qn + kn:b0 + per_layer].copy_(v_c[i][l].reshape(-1).cpu())
            pin_in.append(blk)
        pin_lens = torch.from_numpy(np.stack([wl.seq_lens(t) for t in range(S)])).pin_memory()
        pin_out = torch.empty((L, n, wl.n_q, 64), dtype=tdt).pin_memory()
        dev_in = [torch.empty(L * per_layer, dtype=tdt, device=dev) for _ in range(2)]
        dev_lens = [torch.empty(n, dtype=torch.int32, device=dev) for _ in range(2)]
        dev_out = [torch.empty((L, n, wl.n_q, 64), dtype=tdt, device=dev) for _ in range(2)]
        cstream = torch.cuda.Stream(device=dev)
        h2d_done = [torch.cuda.Event() for _ in range(2)]
        comp_done = [torch.cuda.Event() for _ in range(2)]
        d2h_done = [torch.cuda.Event() for _ in range(2)]

        def h2d(t, first):
            b = t % 2
            with torch.cuda.stream(cstream):
                if not first:
                    cstream.wait_event(comp_done[b])  # step t-2 is done with buffer b
                dev_in[b].copy_(pin_in[t % n_sets], non_blocking=True)
                dev_lens[b].copy_(pin_lens[t % S], non_blocking=True)
                h2d_done[b].record(cstream)

        def compute(t, first):
            b = t % 2
            stream.wait_event(h2d_done[b])
            if not first:
                stream.wait_event(d2h_done[b])  # step t-2's outputs are read back
            for l in range(L):
                b0 = l * per_layer
                dq = dev_in[b][b0:b0 + qn].view(n, wl.n_q, 64)
                dk = dev_in[b][b0 + qn:b0 + qn + kn].view(n, wl.n_kv, 64)
                dv = dev_in[b][b0 + qn + kn:b0 + per_layer].view(n, wl.n_kv, 64)
                if fused:
                    pool.append_decode_attn(dk, dv, dq, bt_dev[l], dev_lens[b], out=dev_out[b][l], stream=stream)
                else:
                    pool.append_decode(dk, dv, bt_dev[l], dev_lens[b], stream=stream)
                    pool.decode_attn(dq, bt_dev[l], dev_lens[b], out=dev_out[b][l], stream=stream)
            comp_done[b].record(stream)

        def d2h(t):
            b = t % 2
            with torch.cuda.stream(cstream):
                cstream.wait_event(comp_done[b])
                pin_out.copy_(dev_out[b], non_blocking=True)
                d2h_done[b].record(cstream)

        def e2e_run(t0, steps):
            cstream.wait_stream(stream)
            h2d(t0, True)
            for j in range(steps):
                if j + 1 < steps:
                    h2d(t0 + j + 1, j + 1 < 2)
                compute(t0 + j, j < 2)
                d2h(t0 + j)
            stream.wait_stream(cstream)

        e2e_run(0, 3)
        torch.cuda.synchronize()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        e2e_run(args.warmup, Ke)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        e_ms = max_over_ranks(e0.elapsed_time(e1))
        esz = pool.shape.torch_dtype.itemsize
        h2d_bytes = L * per_layer * esz + n * 4
        d2h_bytes = L * n * wl.n_q * 64 * esz
        e2e = {"value": n * Ke * world / (e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d_bytes,
               "d2h_bytes_per_step": d2h_bytes, "steps": Ke,
               "path": ("pinned host q/k/v (one block per step) -> KvPool.append_decode_attn per layer (C ABI) -> "
                        "pinned host out (one block per step); copies on a second stream, one step ahead/behind")
               if fused else "pinned host q/k/v -> KvPool.append_decode + decode_attn (C ABI) -> pinned host out"}

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
                       "lengths": "uniform [128, 8192] + step" + (
                           f"; the 64 lengths once per GPU, LPT shares by length (one of each per GPU)" if world > 1 else ""),
                       "l2": "no flush: K/V read per step (~3.5 GB) >> 126 MB L2",
                       "parallelism": f"batch-sharded x{world} (independent sessions per GPU)"},
            "step_gbs": step_gbs, "step_frac_of_peak": step_gbs / hbm,
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": launches, "clocks": clocks,
            "per_rank": [{"rank": r, "sessions": int(x[2]), "bytes_per_step": x[0], "ms": x[1],
                          "gbs": x[0] * K / (x[1] / 1e3) / 1e9} for r, x in enumerate(per_rank)],
        }
        print(json.dumps(line), flush=True)
    pool.close()


# =====================================================================================
# The other workloads (--workload single | prefill | spec | longctx).  Each prints
# one JSON line with the keys of the headline line; its metric names the workload.
# =====================================================================================
def tensor_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["bf16_tflops_sustained"]), "measured sustained (MEASURED_PEAKS.json bf16_tflops_sustained)"
    return 1400.0, "fallback sustained 1.4 PFLOP/s"


class Ctx:
    """Device, stream and rank plumbing shared by the workload runners."""

    def __init__(self, rank: int, world: int, local_rank: int):
        import torch
        import torch.distributed as dist

        self.torch, self.dist = torch, dist
        self.rank, self.world, self.local_rank = rank, world, local_rank
        torch.cuda.set_device(local_rank)
        self.dev = torch.device("cuda", local_rank)
        self.stream = torch.cuda.current_stream()

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max_over_ranks(self, x: float) -> float:
        if self.world == 1:
            return x
        t = self.torch.tensor([x], device=self.dev, dtype=self.torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def events(self):
        ev = self.torch.cuda.Event
        return ev(enable_timing=True), ev(enable_timing=True)

    def timed(self, step, first: int, count: int, clocks: bool = True):
        """Device time in ms (max over ranks) of step(first) .. step(first + count - 1)."""
        torch = self.torch
        sampler = ClockSampler(self.local_rank) if clocks else None
        if sampler:
            sampler.start()
        self.barrier()
        torch.cuda.synchronize()
        e0, e1 = self.events()
        e0.record(self.stream)
        for i in range(count):
            step(first + i)
        e1.record(self.stream)
        torch.cuda.synchronize()
        self.barrier()
        clk = sampler.stop() if sampler else None
        return self.max_over_ranks(e0.elapsed_time(e1)), clk

    def i32(self, a):
        return self.torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(self.dev)


def _line(args, ctx, metric, value, unit, ms_per_step, dtype, config, roofline, cpu, e2e, launches, clocks,
          scaling="weak", **extra):
    d = {"metric": metric, "value": value, "unit": unit, "n_gpus": ctx.world, "steps": args.steps,
         "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": scaling,
         "vs_baseline": None, "dtype": dtype, "data": "synthetic", "config": config, "roofline": roofline,
         "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches, "clocks": clocks}
    d.update(extra)
    return d


def _cpu_threads_map(fn, items, threads):
    """fn over items on `threads` host threads (the oracle releases the GIL)."""
    from concurrent.futures import ThreadPoolExecutor

    with ThreadPoolExecutor(max_workers=threads) as ex:
        return list(ex.map(fn, items))


# ---- fp32 single session -------------------------------------------------------------
METRIC_SINGLE = "fp32 single-session prefill 2048 + 256 decode tokens/s (6 layers, 24q/8kv)"


def cpu_single(budget_s: float):
    """Oracle on one layer: causal prefill attention over 2048 tokens plus
    decode steps at lengths 2049.., one thread (the reference runs one session
    on one thread); extrapolated to the 6-layer job."""
    from oracle import oracle as O
    from llmhost_b200.workloads import SingleSessionWorkload, normal_bits

    wl = SingleSessionWorkload()
    rng = np.random.default_rng(0)
    T = wl.prefill
    q = rng.standard_normal((wl.n_q, T, 64), dtype=np.float32)
    k = rng.standard_normal((wl.n_kv, T, 64), dtype=np.float32)
    v = rng.standard_normal((wl.n_kv, T, 64), dtype=np.float32)
    t0 = time.perf_counter()
    O.attention_forward(q, k, v, wl.n_q, wl.n_kv, T, T, 64, causal=True)
    t_pre = time.perf_counter() - t0
    npages = wl.pages_per_layer
    host = O.HostPages(npages, O.F32, wl.n_q, wl.n_kv, data=normal_bits(rng, (npages, 2 * wl.n_kv * 16 * 64), "f32"))
    bt = np.arange(npages, dtype=np.uint32)[None, :]
    qd = rng.standard_normal((1, wl.n_q, 64), dtype=np.float32)
    kd = rng.standard_normal((1, wl.n_kv, 64), dtype=np.float32)
    n_dec, t_dec = 0, 0.0
    while t_dec < max(budget_s - t_pre, 0.5) and n_dec < wl.steps:
        lens = np.array([T + n_dec + 1], np.int32)
        t0 = time.perf_counter()
        host.decode_step(bt, lens, 0, qd, kd, kd, n_threads=1)
        t_dec += time.perf_counter() - t0
        n_dec += 1
    job_s = wl.n_layers * (t_pre + t_dec / n_dec * wl.steps)
    sample = (f"1 layer: causal prefill attention over {T} tokens + {n_dec} decode steps (append + attention), "
              f"one thread, extrapolated to {wl.n_layers} layers and {wl.steps} steps")
    return (T + wl.steps) / job_s, 1, sample


def run_single(args, ctx):
    torch = ctx.torch
    from llmhost_b200.kv import KvPool
    from llmhost_b200.workloads import SingleSessionWorkload

    wl = SingleSessionWorkload()
    L, T, D = wl.n_layers, wl.prefill, wl.steps
    dev, st = ctx.dev, ctx.stream
    pool = KvPool(dtype="f32", n_q_heads=wl.n_q, n_kv_heads=wl.n_kv, n_pages=wl.pool_pages,
                  rope_theta=wl.rope_theta, max_positions=T + D + 16, max_seqs=1, device=ctx.local_rank)
    gen = torch.Generator(device=dev)
    gen.manual_seed(11 + ctx.rank)

    def rnd(*shape):
        return torch.randn(shape, generator=gen, device=dev, dtype=torch.float32)

    bt = [torch.from_numpy(wl.block_table(l).view(np.int32)).to(dev)[None, :] for l in range(L)]
    qp, kp, vp = rnd(L, T, wl.n_q, 64), rnd(L, T, wl.n_kv, 64), rnd(L, T, wl.n_kv, 64)
    qd, kd, vd = rnd(L, D, 1, wl.n_q, 64), rnd(L, D, 1, wl.n_kv, 64), rnd(L, D, 1, wl.n_kv, 64)
    zeros = torch.zeros(T, dtype=torch.int32, device=dev)
    pos = torch.arange(T, dtype=torch.int32, device=dev)
    qoff = ctx.i32([0, T])
    pre0 = ctx.i32([0])
    lens = torch.arange(T + 1, T + D + 1, dtype=torch.int32, device=dev).view(D, 1)
    outp = torch.empty_like(qp[0])
    outd = torch.empty(1, wl.n_q, 64, device=dev)
    rec = {"pre": [], "dec": []}

    def job(i, record=False, src=None):
        q_p, k_p, v_p, q_d, k_d, v_d = src or (qp, kp, vp, qd, kd, vd)
        for l in range(L):
            pool.append(k_p[l], v_p[l], zeros, pos, pos, bt[l], stream=st)
            e = ctx.events() if record else None
            if e:
                e[0].record(st)
            pool.prefill_attn(q_p[l], pos, qoff, pre0, bt[l], max_q=T, out=outp, stream=st)
            if e:
                e[1].record(st)
                rec["pre"].append(e)
        for t in range(D):
            for l in range(L):
                e = ctx.events() if record and t % 8 == 0 else None
                if e:
                    e[0].record(st)
                pool.append_decode_attn(k_d[l, t], v_d[l, t], q_d[l, t], bt[l], lens[t], out=outd, stream=st)
                if e:
                    e[1].record(st)
                    rec["dec"].append((e, T + t + 1))

    for w in range(args.warmup):
        job(w)
    torch.cuda.synchronize()
    pool.check_device_error()
    ms, clocks = ctx.timed(lambda i: job(i, record=True), 0, args.steps)
    pool.check_device_error()
    pre_ms = float(np.mean([a.elapsed_time(b) for a, b in rec["pre"]]))
    dec = [(a.elapsed_time(b), n) for (a, b), n in rec["dec"]]
    dec_bytes = [2 * wl.n_kv * 64 * 4 * n + 2 * wl.n_q * 64 * 4 + 4 * (-(-n // 16)) for _, n in dec]
    dec_us = float(np.mean([t for t, _ in dec])) * 1e3
    achieved = float(np.mean(dec_bytes)) / (dec_us * 1e-6) / 1e9
    hbm, kind = peaks()
    roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                "traffic": None, "kernel": "decode_kernel (kv_append_decode_attn, fp32 CUDA cores, 1 session)",
                "algorithmic_bytes_per_launch": float(np.mean(dec_bytes)), "mean_launch_us": dec_us,
                "peak_kind": kind,
                "note": "one session: a launch moves ~4.5 MB, so the kernel is latency-bound, not HBM-bound"}
    tok = (T + D) * args.steps * ctx.world
    value = tok / (ms / 1e3)
    # end to end: pinned host inputs, outputs read back after every layer's attention
    e2e = None
    if not args.no_e2e:
        hp = [x.cpu().pin_memory() for x in (qp, kp, vp, qd, kd, vd)]
        dp = [torch.empty_like(x) for x in (qp, kp, vp, qd, kd, vd)]
        host_out = torch.empty(L, D, 1, wl.n_q, 64).pin_memory()
        host_pre = torch.empty(L, T, wl.n_q, 64).pin_memory()

        def e2e_job(i):
            for h, d in zip(hp, dp):
                d.copy_(h, non_blocking=True)
            q_p, k_p, v_p, q_d, k_d, v_d = dp
            for l in range(L):
                pool.append(k_p[l], v_p[l], zeros, pos, pos, bt[l], stream=st)
                pool.prefill_attn(q_p[l], pos, qoff, pre0, bt[l], max_q=T, out=outp, stream=st)
                host_pre[l].copy_(outp, non_blocking=True)
            for t in range(D):
                for l in range(L):
                    pool.append_decode_attn(k_d[l, t], v_d[l, t], q_d[l, t], bt[l], lens[t], out=outd,
                                            stream=st)
                    host_out[l, t].copy_(outd, non_blocking=True)

        e2e_job(0)
        torch.cuda.synchronize()
        e_ms, _ = ctx.timed(e2e_job, 0, max(1, args.steps // 2), clocks=False)
        h2d = sum(x.numel() * 4 for x in hp)
        e2e = {"value": (T + D) * max(1, args.steps // 2) * ctx.world / (e_ms / 1e3), "unit": "tokens/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": (host_out.numel() + host_pre.numel()) * 4,
               "path": "pinned host q/k/v -> KvPool.append/prefill_attn/append_decode/decode_attn -> pinned out"}
    cpu = None
    if ctx.rank == 0 and ctx.world == 1 and not args.no_cpu_baseline:
        v_cpu, cores, sample = cpu_single(args.cpu_budget)
        cpu = {"value": v_cpu, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample,
               "host": host_info()}
    if ctx.rank == 0:
        cfg = {"workload": wl.name, "sessions": 1, "prefill_tokens": T, "decode_steps": D, "layers": L,
               "q_heads": wl.n_q, "kv_heads": wl.n_kv, "head_dim": 64, "page_tokens": 16,
               "block_table": "contiguous (page = layer * 144 + i)",
               "l2": "no flush: a step is a whole job; the 70 MB of K/V stays in L2 (it would on the reference too)",
               "parallelism": f"independent replica per GPU x{ctx.world}"}
        print(json.dumps(_line(args, ctx, METRIC_SINGLE, value, "tokens/s", ms / args.steps, "f32", cfg, roofline,
                               cpu, e2e, args.steps * (L * 2 + D * L * 2), clocks,
                               prefill_attn_ms_per_layer=pre_ms,
                               prefill_attn_tflops=wl.prefill_flops() / L / (pre_ms / 1e3) / 1e12)), flush=True)
    pool.close()


# ---- bf16 chunked prefill ------------------------------------------------------------
METRIC_PREFILL = "bf16 chunked prefill tokens/s and attention TFLOP/s (% tensor peak), 16 sessions x 32 chunks"


def cpu_prefill(budget_s: float, wl):
    """Oracle masked attention for (session, layer) chunks of the job, all host
    threads in parallel (one chunk per thread), until the budget; returns the
    job's tokens/s at the measured CPU FLOP rate."""
    from oracle import oracle as O

    threads = O.max_threads()
    C = wl.chunk
    c = wl.n_chunks // 2  # a middle chunk: L = 8192
    Lk = c * C
    rng = np.random.default_rng(3)
    q = rng.standard_normal((wl.n_q, C, 64), dtype=np.float32)
    k = rng.standard_normal((wl.n_kv, Lk + C, 64), dtype=np.float32)
    v = rng.standard_normal((wl.n_kv, Lk + C, 64), dtype=np.float32)
    mask = np.zeros((C, Lk + C), np.uint8)
    mask[:, :Lk] = 1
    mask[:, Lk:] = np.tril(np.ones((C, C), np.uint8))
    done, t0 = 0, time.perf_counter()
    while True:
        _cpu_threads_map(lambda _: O.attention_masked(q, k, v, wl.n_q, wl.n_kv, C, Lk + C, 64, mask),
                         range(threads), threads)
        done += threads
        if time.perf_counter() - t0 >= budget_s:
            break
    el = time.perf_counter() - t0
    flop_rate = done * wl.chunk_flops(c) / wl.n_seqs / el
    job_tokens = wl.n_seqs * wl.total
    value = job_tokens / (wl.total_flops() / flop_rate)
    sample = (f"{done} x [1 session x 1 layer] chunk {c} (L = {Lk}, 512 queries, 32q/8kv) on {threads} threads; "
              f"job time = job FLOPs / measured FLOP rate")
    return value, threads, sample


def run_prefill(args, ctx):
    torch = ctx.torch
    from llmhost_b200.kv import KvPool
    from llmhost_b200.workloads import chunked_prefill_config

    wl = chunked_prefill_config(seed=3 + 1000 * ctx.rank)
    L, n, C = wl.n_layers, wl.n_seqs, wl.chunk
    dev, st = ctx.dev, ctx.stream
    pool = KvPool(dtype="bf16", n_q_heads=wl.n_q, n_kv_heads=wl.n_kv, n_pages=wl.pool_pages,
                  rope_theta=wl.rope_theta, max_positions=wl.total + 16, max_seqs=n, device=ctx.local_rank)
    bt = [torch.from_numpy(wl.block_tables[l].view(np.int32)).to(dev) for l in range(L)]
    gen = torch.Generator(device=dev)
    gen.manual_seed(13 + ctx.rank)
    n_sets = 2

    def rnd(*shape):
        return torch.randn(shape, generator=gen, device=dev, dtype=torch.float32).to(torch.bfloat16)

    qs = [rnd(L, n * C, wl.n_q, 64) for _ in range(n_sets)]
    ks = [rnd(L, n * C, wl.n_kv, 64) for _ in range(n_sets)]
    vs = [rnd(L, n * C, wl.n_kv, 64) for _ in range(n_sets)]
    tok_seq = ctx.i32(np.repeat(np.arange(n), C))
    q_off = ctx.i32(np.arange(0, n * C + 1, C))
    slots = [ctx.i32(np.tile(np.arange(c * C, (c + 1) * C), n)) for c in range(wl.n_chunks)]
    prefix = [ctx.i32(np.full(n, c * C)) for c in range(wl.n_chunks)]
    out = torch.empty(n * C, wl.n_q, 64, device=dev, dtype=torch.bfloat16)
    rec = []

    def step(i, record=False, src=None):
        c = i % wl.n_chunks
        q, k, v = src or (qs[i % n_sets], ks[i % n_sets], vs[i % n_sets])
        for l in range(L):
            pool.append(k[l], v[l], tok_seq, slots[c], slots[c], bt[l], stream=st)
            e = ctx.events() if record else None
            if e:
                e[0].record(st)
            pool.prefill_attn(q[l], slots[c], q_off, prefix[c], bt[l], max_q=C, out=out, stream=st)
            if e:
                e[1].record(st)
                rec.append((e, c))

    c0 = args.prefill_start_chunk
    for w in range(args.warmup):
        step(c0 + w)
    torch.cuda.synchronize()
    pool.check_device_error()
    ms, clocks = ctx.timed(lambda i: step(i, record=True), c0 + args.warmup, args.steps)
    pool.check_device_error()
    launch = [(a.elapsed_time(b), c) for (a, b), c in rec]
    flops = sum(wl.chunk_flops(c) for _, c in launch)
    kern_s = sum(t for t, _ in launch) / 1e3
    achieved = flops / kern_s / 1e12
    peak, kind = tensor_peak()
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                "traffic": None, "kernel": "prefill_kernel (kv_prefill_attn, tcgen05)",
                "algorithmic_flops_per_launch": flops / len(launch),
                "mean_launch_us": kern_s / len(launch) * 1e6, "peak_kind": kind,
                "flops_rule": "4 * head_dim per visible (query row, key) pair"}
    tokens = n * C * args.steps * ctx.world
    value = tokens / (ms / 1e3)
    e2e = None
    if not args.no_e2e:
        hq = qs[0].cpu().pin_memory()
        hk = ks[0].cpu().pin_memory()
        hv = vs[0].cpu().pin_memory()
        dq, dk, dv = torch.empty_like(qs[0]), torch.empty_like(ks[0]), torch.empty_like(vs[0])
        hout = torch.empty(L, n * C, wl.n_q, 64, dtype=torch.bfloat16).pin_memory()

        def e2e_step(i):
            c = i % wl.n_chunks
            dq.copy_(hq, non_blocking=True)
            dk.copy_(hk, non_blocking=True)
            dv.copy_(hv, non_blocking=True)
            for l in range(L):
                pool.append(dk[l], dv[l], tok_seq, slots[c], slots[c], bt[l], stream=st)
                pool.prefill_attn(dq[l], slots[c], q_off, prefix[c], bt[l], max_q=C, out=out, stream=st)
                hout[l].copy_(out, non_blocking=True)

        e2e_step(0)
        torch.cuda.synchronize()
        ke = min(args.steps, wl.n_chunks)
        e_ms, _ = ctx.timed(e2e_step, 0, ke, clocks=False)
        e2e = {"value": n * C * ke * ctx.world / (e_ms / 1e3), "unit": "tokens/s",
               "h2d_bytes_per_step": (hq.numel() + hk.numel() + hv.numel()) * 2,
               "d2h_bytes_per_step": hout.numel() * 2,
               "path": "pinned host q/k/v -> KvPool.append + prefill_attn (C ABI) per layer -> pinned out"}
    cpu = None
    if ctx.rank == 0 and ctx.world == 1 and not args.no_cpu_baseline:
        v_cpu, cores, sample = cpu_prefill(args.cpu_budget, wl)
        cpu = {"value": v_cpu, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample,
               "host": host_info()}
    if ctx.rank == 0:
        covered = sorted({(c0 + args.warmup + i) % wl.n_chunks for i in range(args.steps)})
        cfg = {"workload": wl.name, "sessions_per_gpu": n, "chunk": C, "total_tokens": wl.total, "layers": L,
               "q_heads": wl.n_q, "kv_heads": wl.n_kv, "head_dim": 64, "page_tokens": 16,
               "chunks_timed": f"{len(covered)} of {wl.n_chunks}",
               "l2": "no flush: each step reads 16 sessions' prefix K/V (up to 512 MB per layer) >> L2",
               "parallelism": f"batch-sharded x{ctx.world}"}
        print(json.dumps(_line(args, ctx, METRIC_PREFILL, value, "tokens/s", ms / args.steps, "bf16", cfg, roofline,
                               cpu, e2e, args.steps * L * 2, clocks, attention_tflops=achieved,
                               step_tflops=sum(wl.chunk_flops((c0 + args.warmup + i) % wl.n_chunks)
                                               for i in range(args.steps)) * L * ctx.world / (ms / 1e3) / 1e12)),
              flush=True)
    pool.close()


# ---- speculative tree rounds ------------------------------------------------------------
METRIC_SPEC = "speculative tree rounds: verified tree tokens/s (32 sessions x 64-node trees, COW fork, commit)"


class _Staging:
    """Double-buffered pinned staging for per-step host arrays copied to the
    device: every array of a step is packed into one pinned buffer (256-byte
    aligned slots) and moved with one host-to-device copy."""

    def __init__(self, torch, dev, sizes: dict):
        self.torch = torch
        self.layout, off = {}, 0
        for k, (shape, dt) in sizes.items():
            shape = shape if isinstance(shape, tuple) else (shape,)
            itemsize = torch.empty((), dtype=dt).element_size()
            nbytes = int(np.prod(shape)) * itemsize
            self.layout[k] = (off, shape, dt, itemsize)
            off += -(-nbytes // 256) * 256
        self.total = off
        self.host = [torch.empty(off, dtype=torch.uint8).pin_memory() for _ in range(2)]
        self.dev = torch.empty(off, dtype=torch.uint8, device=dev)
        self.done = [None, None]
        self.cur = 0

    def put(self, arrays: dict):
        """Copy numpy arrays (first dim may be shorter) to the device; returns device views."""
        torch = self.torch
        if self.done[self.cur] is not None:
            self.done[self.cur].synchronize()
        hbuf = self.host[self.cur].numpy()
        out, start, end = {}, self.total, 0
        for k, a in arrays.items():
            off, shape, dt, itemsize = self.layout[k]
            a = np.ascontiguousarray(a)
            nbytes = a.size * a.itemsize
            hbuf[off:off + nbytes] = a.reshape(-1).view(np.uint8)
            n = a.shape[0]
            out[k] = self.dev[off:off + nbytes].view(dt).view((n,) + shape[1:])
            start, end = min(start, off), max(end, off + nbytes)
        if end > start:  # only this call's slots: the other arrays' device copies stay as they are
            self.dev[start:end].copy_(self.host[self.cur][start:end], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self.done[self.cur] = ev
        self.cur ^= 1
        return out


def cpu_spec(budget_s: float, wl):
    """Oracle tree-masked attention for one (session, layer) verify of 64 nodes
    over the 4096-token prefix, all host threads in parallel; extrapolated to
    the step (sessions x layers)."""
    from oracle import oracle as O
    from llmhost_b200.plans import tree_masks
    from llmhost_b200.workloads import draft_tree

    threads = O.max_threads()
    rng = np.random.default_rng(4)
    parents, _ = draft_tree(rng, wl.nodes, wl.depth)
    T, Lp = wl.nodes, wl.prefix
    m = tree_masks(parents).view(np.uint64)
    mask = np.zeros((T, Lp + T), np.uint8)
    mask[:, :Lp] = 1
    for i in range(T):
        mask[i, Lp:] = [(int(m[i]) >> j) & 1 for j in range(T)]
    q = rng.standard_normal((wl.n_q, T, 64), dtype=np.float32)
    k = rng.standard_normal((wl.n_kv, Lp + T, 64), dtype=np.float32)
    v = rng.standard_normal((wl.n_kv, Lp + T, 64), dtype=np.float32)
    done, t0 = 0, time.perf_counter()
    while True:
        _cpu_threads_map(lambda _: O.attention_masked(q, k, v, wl.n_q, wl.n_kv, T, Lp + T, 64, mask),
                         range(threads), threads)
        done += threads
        if time.perf_counter() - t0 >= budget_s:
            break
    per_verify = (time.perf_counter() - t0) / done
    step_s = per_verify * wl.n_seqs * wl.n_layers
    sample = (f"{done} x [1 session x 1 layer] tree verify ({T} nodes over a {Lp}-token prefix, 24q/8kv) on "
              f"{threads} threads; step = {wl.n_seqs} sessions x {wl.n_layers} layers of it")
    return wl.n_seqs * wl.nodes / step_s, threads, sample


def run_spec(args, ctx):
    torch = ctx.torch
    from llmhost_b200.kv import KvPool
    from llmhost_b200.plans import commit_moves, plan_forward
    from llmhost_b200.state import KvState
    from llmhost_b200.workloads import SpecTreeWorkload

    wl = SpecTreeWorkload(seed=4 + 1000 * ctx.rank)
    plan = wl.plan()
    # the plan's trees and accepted paths as arrays, made before the timed region
    plan_np = []
    for rows in plan:
        parents = np.array([r[0] for r in rows], np.int32)
        lens = [len(r[1]) for r in rows]
        offs = np.zeros(len(rows) + 1, np.int32)
        np.cumsum(lens, out=offs[1:])
        flat = np.concatenate([np.asarray(r[1], np.int64) for r in rows])
        plan_np.append((parents, (flat, offs)))
    L, n, T = wl.n_layers, wl.n_seqs, wl.nodes
    dev, stm = ctx.dev, ctx.stream
    total_steps = args.warmup + args.steps
    max_tokens = wl.prefix + (wl.depth + 1) * total_steps + T
    stride = -(-max_tokens // 16) + 1
    order = np.random.default_rng(wl.seed).permutation(wl.pool_pages).astype(np.uint32)
    st = KvState(wl.pool_pages, L, alloc_order=order)
    pool = KvPool(dtype="bf16", n_q_heads=wl.n_q, n_kv_heads=wl.n_kv, n_pages=wl.pool_pages,
                  rope_theta=wl.rope_theta, max_positions=max_tokens + 16, max_seqs=n, device=ctx.local_rank)
    gen = torch.Generator(device=dev)
    gen.manual_seed(17 + ctx.rank)

    def rnd(*shape):
        return torch.randn(shape, generator=gen, device=dev, dtype=torch.float32).to(torch.bfloat16)

    # the shared prefix: session 0 prefills it, sessions 1.. fork (refcount n)
    st.open(0)
    st.append(0, wl.prefix)
    pos = ctx.i32(np.arange(wl.prefix))
    zeros = ctx.i32(np.zeros(wl.prefix))
    for l in range(L):
        t0 = torch.from_numpy(st.export_tables([0], l, stride).view(np.int32)).to(dev)
        pool.append(rnd(wl.prefix, wl.n_kv, 64), rnd(wl.prefix, wl.n_kv, 64), zeros, pos, pos, t0)
    for s in range(1, n):
        st.fork(0, s)
    torch.cuda.synchronize()
    pool.check_device_error()
    seqs = list(range(n))
    # device-resident per-step inputs (a ring of 4 sets)
    qs = [rnd(L, n * T, wl.n_q, 64) for _ in range(4)]
    ks = [rnd(L, n * T, wl.n_kv, 64) for _ in range(4)]
    vs = [rnd(L, n * T, wl.n_kv, 64) for _ in range(4)]
    out = torch.empty(n * T, wl.n_q, 64, device=dev, dtype=torch.bfloat16)
    tokens = np.tile(np.arange(1000, 1000 + T, dtype=np.uint32), (n, 1))
    i32, i64 = torch.int32, torch.int64
    stage = _Staging(torch, dev, {"tables": ((L, n, stride), i32), "cow_src": (L * n, i32), "cow_dst": (L * n, i32),
                                  "tok_seq": (n * T, i32), "slots": (n * T, i32), "pos": (n * T, i32),
                                  "q_off": (n + 1, i32), "prefix": (n, i32), "masks": (n * T, i64),
                                  "moves": ((L * n * (wl.depth + 1), 4), i32), "groups": (L * n + 1, i32)})
    rec = []
    stats = {"accepted": 0, "verified": 0, "cow": 0, "flops": []}

    def step(i, record=False, src=None):
        parents, paths = plan_np[i % len(plan_np)]
        fb = plan_forward(st, seqs, tokens, parents, stride)
        d = stage.put({"tables": fb.tables.view(np.int32), "cow_src": fb.cow_src.view(np.int32),
                       "cow_dst": fb.cow_dst.view(np.int32), "tok_seq": fb.tok_seq, "slots": fb.slots,
                       "pos": fb.positions, "q_off": fb.q_offsets, "prefix": fb.prefix, "masks": fb.masks})
        if len(fb.cow_src):
            pool.copy_pages(d["cow_src"], d["cow_dst"], stream=stm)
        q, k, v = src or (qs[i % 4], ks[i % 4], vs[i % 4])
        ntok = fb.n_tokens
        for l in range(L):
            pool.append(k[l, :ntok], v[l, :ntok], d["tok_seq"], d["slots"], d["pos"], d["tables"][l], stream=stm)
            e = ctx.events() if record and i % 4 == 0 else None  # every 4th step's launches
            if e:
                e[0].record(stm)
            pool.prefill_attn(q[l, :ntok], d["pos"], d["q_off"], d["prefix"], d["tables"][l], tree_masks=d["masks"],
                              max_q=T, out=out[:ntok], stream=stm)
            if e:
                e[1].record(stm)
                rec.append(e)
        mv, offs, acc = commit_moves(st, seqs, paths)
        dm = stage.put({"moves": mv, "groups": offs})
        if len(mv):
            pool.move_tokens(dm["moves"], dm["groups"], stream=stm)
        if record:
            stats["accepted"] += acc
            stats["verified"] += ntok
            stats["cow"] += len(fb.cow_src)
            ones = np.unpackbits(fb.masks.view(np.uint8)).reshape(-1, 64).sum(axis=1)  # popcount per mask
            vis = fb.prefix[fb.tok_seq] + ones
            stats["flops"].append(4.0 * 64 * wl.n_q * float(vis.sum()))

    for w in range(args.warmup):
        step(w)
    torch.cuda.synchronize()
    pool.check_device_error()
    ms, clocks = ctx.timed(lambda i: step(i, record=True), args.warmup, args.steps)
    pool.check_device_error()
    kt = [a.elapsed_time(b) for a, b in rec]
    flops_per_launch = float(np.mean(stats["flops"]))
    achieved = flops_per_launch / (float(np.mean(kt)) / 1e3) / 1e12
    peak, kind = tensor_peak()
    kv_bytes = 2 * wl.n_kv * 64 * 2 * (wl.prefix * n + n * T)
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                "traffic": None, "kernel": "prefill_kernel (kv_prefill_attn, tree masks, tcgen05)",
                "algorithmic_flops_per_launch": flops_per_launch, "mean_launch_us": float(np.mean(kt)) * 1e3,
                "peak_kind": kind,
                "hbm_view": {"bytes_per_launch": kv_bytes,
                             "achieved_gbs": kv_bytes / (float(np.mean(kt)) / 1e3) / 1e9}}
    value = stats["verified"] * ctx.world / (ms / 1e3)
    cpu = None
    if ctx.rank == 0 and ctx.world == 1 and not args.no_cpu_baseline:
        v_cpu, cores, sample = cpu_spec(args.cpu_budget, wl)
        cpu = {"value": v_cpu, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample,
               "host": host_info()}
    if ctx.rank == 0:
        cfg = {"workload": wl.name, "sessions_per_gpu": n, "shared_prefix": wl.prefix, "tree_nodes": T,
               "tree_depth": wl.depth, "layers": L, "q_heads": wl.n_q, "kv_heads": wl.n_kv, "head_dim": 64,
               "page_tokens": 16, "tree": "best-first by cumulative Dirichlet(1) probability, 4 candidates/node",
               "l2": "no flush: the 32 sessions' prefix K/V (~50 MB per layer) is re-read each layer",
               "parallelism": f"batch-sharded x{ctx.world}"}
        e2e = {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": None, "d2h_bytes_per_step": 0,
               "note": "the timed step already runs through the public API with its host planning and per-step "
                       "host->device copies of tables, slots, masks and moves; q/k/v are device-resident"}
        print(json.dumps(_line(args, ctx, METRIC_SPEC, value, "tokens/s", ms / args.steps, "bf16", cfg, roofline,
                               cpu, e2e, args.steps * (L * 2 + 2), clocks,
                               accepted_tokens_per_s=stats["accepted"] * ctx.world / (ms / 1e3),
                               mean_accepted_per_session=stats["accepted"] / (args.steps * n),
                               cow_copies=stats["cow"])), flush=True)
    pool.close()
    st.close_all()


# ---- long context with a sliding window -------------------------------------------------
METRIC_LONGCTX = ("long-context decode tokens/s (window 32k, evict + compact) and the 1M-token session "
                  "(KV-head sharded, NCCL all-gather) step time")


def cpu_longctx(budget_s: float, wl):
    """Oracle decode steps (append + windowed attention, one layer) over the
    GPU's share of sessions at their resident lengths, all host threads."""
    from oracle import oracle as O
    from llmhost_b200.workloads import normal_bits

    rng = np.random.default_rng(5)
    lens = np.minimum(wl.l0, wl.window).astype(np.int32) + 1
    need = -(-lens // 16)
    bt = np.full((len(lens), int(need.max())), 0xFFFFFFFF, np.uint32)
    cur = 0
    for s in range(len(lens)):
        bt[s, :need[s]] = np.arange(cur, cur + need[s], dtype=np.uint32)
        cur += need[s]
    host = O.HostPages(cur, O.BF16, wl.n_q, wl.n_kv, data=normal_bits(rng, (cur, 2 * wl.n_kv * 16 * 64), "bf16"))
    q = normal_bits(rng, (len(lens), wl.n_q, 64), "bf16")
    k = normal_bits(rng, (len(lens), wl.n_kv, 64), "bf16")
    threads = O.max_threads()
    steps, t0 = 0, time.perf_counter()
    while True:
        host.decode_step(bt, lens, wl.window, q, k, k, n_threads=threads)
        steps += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    el = time.perf_counter() - t0
    sample = (f"{steps} x [{len(lens)} sessions x 1 layer] decode step at resident lengths (<= window {wl.window}), "
              f"{threads} threads, extrapolated to {wl.n_layers} layers")
    return len(lens) * steps / (el * wl.n_layers), threads, sample


def run_longctx(args, ctx):
    torch = ctx.torch
    from llmhost_b200.kv import KvPool
    from llmhost_b200.plans import plan_decode_step
    from llmhost_b200.state import KvState
    from llmhost_b200.workloads import long_context_config

    if ctx.world > 8 or 8 % ctx.world:
        raise SystemExit("longctx runs on 1, 2, 4 or 8 GPUs")
    wl = long_context_config(rank=ctx.rank)
    L, W = wl.n_layers, wl.window
    seqs = list(range(len(wl.shard)))
    l0 = wl.l0
    n = len(seqs)
    dev, stm = ctx.dev, ctx.stream
    total_steps = args.warmup + args.steps
    pool_pages = 1 << 19
    order = np.random.default_rng(5 + ctx.rank).permutation(pool_pages)
    st = KvState(pool_pages, L, alloc_order=order.astype(np.uint32))
    pool = KvPool(dtype="bf16", n_q_heads=wl.n_q, n_kv_heads=wl.n_kv, n_pages=pool_pages, rope_theta=wl.rope_theta,
                  max_positions=int(l0.max()) + total_steps + 16, max_seqs=n, device=ctx.local_rank)
    gen = torch.Generator(device=dev)
    gen.manual_seed(19 + ctx.rank)

    def rnd(*shape):
        return torch.randn(shape, generator=gen, device=dev, dtype=torch.float32).to(torch.bfloat16)

    stride = -(-(int(l0.max()) + total_steps) // 16) + 1
    for s in seqs:
        st.open(s)
        st.append(s, int(l0[s]))
    # K/V only for the resident window (from the first page that the window touches)
    for l in range(L):
        tables = torch.from_numpy(st.export_tables(seqs, l, stride).view(np.int32)).to(dev)
        for s in seqs:
            a = max(0, int(l0[s]) - W) // 16 * 16
            cnt = int(l0[s]) - a
            idx = np.arange(a, int(l0[s]), dtype=np.int32)
            pool.append(rnd(cnt, wl.n_kv, 64), rnd(cnt, wl.n_kv, 64), ctx.i32(np.full(cnt, s)), ctx.i32(idx),
                        ctx.i32(idx), tables)
    for s in seqs:
        st.evict_window(s, W)
    dtables = torch.stack([torch.from_numpy(st.export_tables(seqs, l, stride).view(np.int32)) for l in range(L)]).to(dev)
    lens = ctx.i32(l0)  # becomes the attended length after each step's append
    torch.cuda.synchronize()
    pool.check_device_error()
    # the 1M-token session: this GPU's KV heads (8 / world of them) and their q heads
    from llmhost_b200.shard import assemble, head_shard

    shard = head_shard(ctx.rank, ctx.world, wl.n_kv, wl.n_q)
    hpr = shard.n_kv
    big_len = wl.long_session
    big_pages = L * (-(-(big_len + total_steps) // 16)) + 64
    big = KvPool(dtype="bf16", n_q_heads=4 * hpr, n_kv_heads=hpr, n_pages=big_pages, rope_theta=wl.rope_theta,
                 max_positions=big_len + total_steps + 16, max_seqs=1, device=ctx.local_rank)
    per_layer = -(-(big_len + total_steps) // 16)
    big_order = np.random.default_rng(7).permutation(big_pages).astype(np.uint32)
    big_bt = [torch.from_numpy(big_order[l * per_layer:(l + 1) * per_layer].view(np.int32)).to(dev)[None, :]
              for l in range(L)]
    chunk = 1 << 16
    for l in range(L):
        for a in range(0, big_len, chunk):
            idx = torch.arange(a, a + chunk, dtype=torch.int32, device=dev)
            big.append(rnd(chunk, hpr, 64), rnd(chunk, hpr, 64), torch.zeros(chunk, dtype=torch.int32, device=dev),
                       idx, idx, big_bt[l])
    big_len_dev = ctx.i32([big_len])
    torch.cuda.synchronize()
    big.check_device_error()
    qs = rnd(4, L, n, wl.n_q, 64)
    ks = rnd(4, L, n, wl.n_kv, 64)
    vs = rnd(4, L, n, wl.n_kv, 64)
    bq = rnd(4, L, 1, 4 * hpr, 64)
    bk = rnd(4, L, 1, hpr, 64)
    bv = rnd(4, L, 1, hpr, 64)
    out = torch.empty(n, wl.n_q, 64, device=dev, dtype=torch.bfloat16)
    bout = torch.empty(L, 4 * hpr, 64, device=dev, dtype=torch.bfloat16)
    gathered = torch.empty(ctx.world, L, 4 * hpr, 64, device=dev, dtype=torch.bfloat16)
    rec, brec, grec = [], [], []
    stats = {"evicted": 0, "compactions": 0, "moved": 0, "new_pages": 0}

    def step(i, record=False):
        ds = plan_decode_step(st, seqs, W, compact=(i % wl.compact_every == wl.compact_every - 1))
        if ds.new_pages:
            a = np.asarray(ds.new_pages, np.int64)
            vals = torch.from_numpy(a[:, 3].astype(np.uint32).view(np.int32)).to(dev, non_blocking=True)
            dtables[a[:, 0], a[:, 1], a[:, 2]] = vals
        if ds.compaction:
            mv = np.asarray(ds.compaction, np.uint32)
            pool.copy_pages(ctx.i32(mv[:, 0].view(np.int32)), ctx.i32(mv[:, 1].view(np.int32)), stream=stm)
            dtables.copy_(torch.stack([torch.from_numpy(st.export_tables(seqs, l, stride).view(np.int32))
                                       for l in range(L)]).to(dev, non_blocking=True))
        lens.add_(1)
        j = i % 4
        for l in range(L):
            e = ctx.events() if record else None
            if e:
                e[0].record(stm)
            pool.append_decode_attn(ks[j, l], vs[j, l], qs[j, l], dtables[l], lens, window=W, out=out, stream=stm)
            if e:
                e[1].record(stm)
                rec.append(e)
        big_len_dev.add_(1)
        eb = ctx.events() if record else None
        if eb:
            eb[0].record(stm)
        for l in range(L):
            big.append_decode_attn(bk[j, l], bv[j, l], bq[j, l], big_bt[l], big_len_dev, out=bout[l], stream=stm)
        if eb:
            eb[1].record(stm)
            brec.append(eb)
        if ctx.world > 1:
            eg = ctx.events() if record else None
            if eg:
                eg[0].record(stm)
            ctx.dist.all_gather_into_tensor(gathered, bout)
            assemble(gathered)  # [layers, 32 q heads, d] in global head order
            if eg:
                eg[1].record(stm)
                grec.append(eg)
        if record:
            stats["evicted"] += ds.evicted
            stats["moved"] += len(ds.compaction)
            stats["compactions"] += int(bool(ds.compaction))
            stats["new_pages"] += len(ds.new_pages)

    for w in range(args.warmup):
        step(w)
    torch.cuda.synchronize()
    pool.check_device_error()
    big.check_device_error()
    ms, clocks = ctx.timed(lambda i: step(i, record=True), args.warmup, args.steps)
    pool.check_device_error()
    big.check_device_error()
    kt = float(np.mean([a.elapsed_time(b) for a, b in rec]))
    lens_h = lens.cpu().numpy().astype(np.int64)
    att = np.minimum(lens_h - args.steps // 2, W)  # attended keys, mid-run
    abytes = float((2 * wl.n_kv * 64 * 2 * att + 2 * wl.n_q * 64 * 2 + 4 * (-(-att // 16) + 1)).sum())
    hbm, kind = peaks()
    achieved = abytes / (kt / 1e3) / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                "traffic": None, "kernel": "decode_tc_kernel (kv_append_decode_attn, window 32768)",
                "algorithmic_bytes_per_launch": abytes, "mean_launch_us": kt * 1e3, "peak_kind": kind}
    big_ms = float(np.mean([a.elapsed_time(b) for a, b in brec]))
    big_bytes = L * (2 * hpr * 64 * 2 * big_len)
    value = n * args.steps * ctx.world / (ms / 1e3)
    cpu = None
    if ctx.rank == 0 and ctx.world == 1 and not args.no_cpu_baseline:
        v_cpu, cores, sample = cpu_longctx(args.cpu_budget, wl)
        cpu = {"value": v_cpu, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample,
               "host": host_info()}
    if ctx.rank == 0:
        cfg = {"workload": wl.name, "sessions_total": len(wl.lengths), "sessions_per_gpu": n,
               "lengths": "log-uniform [1024, 131072], LPT-partitioned by resident length into 8 shares",
               "window": W, "compact_every": wl.compact_every, "layers": L, "q_heads": wl.n_q, "kv_heads": wl.n_kv,
               "head_dim": 64, "page_tokens": 16, "long_session_tokens": big_len,
               "long_session_kv_heads_per_gpu": hpr,
               "l2": "no flush: each step reads ~6 GB of windowed K/V >> L2",
               "parallelism": f"batch share {ctx.rank} of 8 per GPU x{ctx.world}; 1M session KV-head sharded"}
        e2e = {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": None, "d2h_bytes_per_step": 0,
               "note": "the timed step runs through the public API with host-side eviction, compaction and "
                       "block-table publishing; q/k/v are device-resident"}
        print(json.dumps(_line(args, ctx, METRIC_LONGCTX, value, "tokens/s", ms / args.steps, "bf16", cfg, roofline,
                               cpu, e2e, args.steps * L * 4, clocks,
                               scaling="weak (batch share); the 1M session is split over the GPUs",
                               long_session_ms_per_step=big_ms,
                               long_session_gbs=big_bytes / (big_ms / 1e3) / 1e9,
                               allgather_ms_per_step=float(np.mean([a.elapsed_time(b) for a, b in grec]))
                               if grec else None,
                               evicted_pages=stats["evicted"], compactions=stats["compactions"],
                               compaction_page_moves=stats["moved"])), flush=True)
    big.close()
    pool.close()
    st.close_all()


RUNNERS = {"single": (run_single, cpu_single, METRIC_SINGLE), "prefill": (run_prefill, cpu_prefill, METRIC_PREFILL),
           "spec": (run_spec, cpu_spec, METRIC_SPEC), "longctx": (run_longctx, cpu_longctx, METRIC_LONGCTX)}


def run_reference_workload(args, rank, world):
    """The CPU oracle arm for the non-headline workloads (rank 0 only)."""
    from llmhost_b200.workloads import (SpecTreeWorkload, chunked_prefill_config, long_context_config)

    if rank != 0:
        return
    _, cpu_fn, metric = RUNNERS[args.workload]
    budget = max(2.0, 100.0 / max(args.steps + args.warmup, 1))
    wl = {"single": None, "prefill": chunked_prefill_config(), "spec": SpecTreeWorkload(),
          "longctx": long_context_config(rank=0)}[args.workload]
    t0 = time.perf_counter()
    value, threads, sample = cpu_fn(budget) if wl is None else cpu_fn(budget, wl)
    el = time.perf_counter() - t0
    line = {"impl": "reference", "metric": metric, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32" if args.workload == "single" else "bf16",
            "data": "synthetic", "config": {"workload": args.workload},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "host": host_info(), "seconds": el,
            "note": "reference is Rust with no toolchain here; this is the C restatement of its CPU attention"}
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if args.workload == "decode":
            run_reference(args, rank, world)
        else:
            run_reference_workload(args, rank, world)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        # NCCL may print (its version line, at communicator set-up) on file
        # descriptor 1, which carries the one JSON result line: set the group
        # and its communicator up with descriptor 1 pointing at stderr
        with _stdout_to_stderr():
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", local_rank))
            dist.barrier()
    try:
        if args.workload == "decode":
            run_ours(args, rank, world, local_rank)
        else:
            RUNNERS[args.workload][0](args, Ctx(rank, world, local_rank))
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
