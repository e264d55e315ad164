"""Benchmark of the B200 flash-attention forward (the not-cute-zig `flash` path).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload c4|c2|c5|c5d16] [--no-e2e] [--no-cpu]

One step = one launch of the hot path over one batch of synthetic input
(default: BASELINE config 4 -- batch_heads 64, seq_len 8192, head_dim 64,
causal, f16 Q/K/V N(0,1) with K x2, f32 O -- per GPU).  For N > 1 the script
runs under torch.distributed.run, one rank per GPU; every rank owns its own
64 slices (weak scaling, no collective on the data path), and the step time
is the max over ranks of the CUDA-event time.

Metric: the reference's FLOP formula (src/main.zig:843-844) per second,
whole job.  The JSON line also carries the roofline of the kernel against
the measured B200 peak, an end-to-end number through the C ABI with host
buffers (H2D of Q/K/V and D2H of O inside the timed region), a CPU baseline
(the oracle, a restatement of src/main.zig:1271-1307, on a bounded sample)
and the SM clocks sampled during the timed region.

--impl reference times the reference's CPU attention (the oracle port; the
Zig original cannot be built here) on the host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import ctypes
import importlib
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "flash fwd TFLOP/s & % f16 tensor peak, d=64 causal, at 1/2/4/8 B200"
NOMINAL_F16_TFLOPS = 2250.0
FALLBACK_TFLOPS = 1590.0

WORKLOADS = {
    # name: (batch_heads per GPU, seq_len, head_dim, causal, std, k_mul, seed, O dtype, description)
    "c4": (64, 8192, 64, True, 1.0, 2.0, 3, "f32", "config4_long_causal bh=64 S=8192 d=64 causal N(0,1) Kx2"),
    "c2": (8, 1024, 64, True, 0.5, 1.0, 1, "f16", "config2_profile bh=8 S=1024 d=64 causal N(0,.25) f16 O"),
    "c5": (1024, 2048, 64, False, 0.5, 1.0, 4, "f32", "config5_sweep bh=1024 S=2048 d=64 non-causal N(0,.25)"),
    "c5d16": (1024, 2048, 16, False, 0.5, 1.0, 5, "f32", "config5_sweep bh=1024 S=2048 d=16 non-causal N(0,.25)"),
    "c3": (512, 128, 32, False, None, None, 2, "f32",
           "config3_padded bh=512 S=128 d=32 non-causal, Q/K/V row stride 40 (NaN padding), U(-1,1)"),
}
# Workloads with padded Q/K/V rows (`row` elements apart, NaN in the padding,
# O contiguous) and U(lo, hi) values; their roofline is HBM bandwidth.
PADDED = {"c3": {"row": 40, "lo": -1.0, "hi": 1.0}}
FALLBACK_HBM_GBS = 6650.0
L2_BYTES = 126 * 1024 * 1024


def flops_of(bh, s, d, causal):
    eff = s * (s + 1) // 2 if causal else s * s
    return bh * 4 * eff * d


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            pk = json.load(f)
        return float(pk["bf16_tflops"]), float(pk["bf16_tflops_sustained"]), "measured"
    except Exception:
        return FALLBACK_TFLOPS, FALLBACK_TFLOPS, "fallback"


def load_hbm():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def load_traffic(workload):
    """DRAM bytes per launch from the committed ncu summary (or None)."""
    path = os.path.join(ROOT, "profiles", f"flash_fwd_{workload}_traffic.txt")
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    return float(line.split(":", 1)[1].split()[0])
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clock / throttle sampling around the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.file = tempfile.NamedTemporaryFile(mode="w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(gpu_index)], stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        rows = [r.split(",") for r in self.file.read().strip().splitlines() if r.strip()]
        os.unlink(self.file.name)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for name, val in zip(names, r[5:9]):
                    if val.strip().lower() == "active":
                        reasons.add(name)
            except (ValueError, IndexError):
                continue
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def make_inputs(oracle, bh, s, d, std, k_mul, seed):
    n = bh * s * d
    q = oracle.fill_normal(n, seed * 3 + 0, 0.0, std)
    k = oracle.fill_normal(n, seed * 3 + 1, 0.0, std * k_mul)
    v = oracle.fill_normal(n, seed * 3 + 2, 0.0, std)
    return q, k, v


# ---------------------------------------------------------------------------
# CPU leg: the oracle (restated reference CPU attention) on a bounded sample
# ---------------------------------------------------------------------------
def make_padded_inputs(oracle, bh, s, d, row, lo, hi, seed):
    """Q, K, V of bh slices of s rows `row` elements apart: U(lo, hi) values
    (seeds seed*3 + 0..2), NaN in each row's padding columns."""
    out = []
    for i in range(3):
        a = oracle.fill_uniform(bh * s * row, seed * 3 + i, lo, hi)
        oracle.fill_row_padding(a, bh, s, d, s * row, row)
        out.append(a)
    return out


def host_threads(oracle):
    """All host threads this process may run on (torchrun sets OMP_NUM_THREADS=1
    for its workers; the CPU legs use every core they are allowed)."""
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:
        n = os.cpu_count() or 1
    return max(n, oracle.max_threads())


class _StdoutToStderr:
    """Sends C-level writes to stdout (the NCCL version banner) to stderr, so
    rank 0's stdout carries only the JSON line."""

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


def cpu_sample(oracle, q, k, v, s, d, causal, scale, target_s, threads=0, bh=1):
    """Times the oracle on a bounded sample of the workload sized to about
    target_s seconds: the last rows of slice 0 (the heaviest rows under causal
    masking) when one slice is enough, else whole slices 0..m-1.  Returns
    (TFLOP/s, seconds, description, flops, threads)."""
    import numpy as np

    threads = threads or host_threads(oracle)

    def run_rows(rows):
        out = np.zeros(s * d, dtype=np.float32)
        r0 = s - rows
        t0 = time.perf_counter()
        oracle.flash_reference(q[: s * d], k[: s * d], v[: s * d], batch_heads=1, seq_len=s, head_dim=d,
                               q_stride=s * d, k_stride=s * d, v_stride=s * d, o_stride=s * d, scale=scale,
                               causal=causal, out=out, rows=(r0, s), threads=threads)
        dt = time.perf_counter() - t0
        keys = sum((r + 1) if causal else s for r in range(r0, s))
        return dt, 4 * keys * d

    def run_slices(m):
        out = np.zeros(m * s * d, dtype=np.float32)
        t0 = time.perf_counter()
        oracle.flash_reference(q[: m * s * d], k[: m * s * d], v[: m * s * d], batch_heads=m, seq_len=s,
                               head_dim=d, q_stride=s * d, k_stride=s * d, v_stride=s * d, o_stride=s * d,
                               scale=scale, causal=causal, out=out, threads=threads)
        dt = time.perf_counter() - t0
        keys = (s * (s + 1) // 2) if causal else s * s
        return dt, 4 * m * keys * d

    rows = min(s, max(threads, 8))
    dt, fl = run_rows(rows)
    while dt < 0.5 and rows < s:
        rows = min(s, rows * 4)
        dt, fl = run_rows(rows)
    if rows < s:
        rows = min(s, max(threads, int(rows * target_s / max(dt, 1e-6))))
    if rows < s:
        dt, fl = run_rows(rows)
        return fl / dt / 1e12, dt, f"rows {s - rows}..{s - 1} of slice 0", fl, threads, rows
    dt1, _ = run_slices(1)
    m = max(1, min(bh, int(target_s / max(dt1, 1e-6))))
    dt, fl = run_slices(m)
    return fl / dt / 1e12, dt, f"slices 0..{m - 1} (all rows)", fl, threads, s


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def reference_arm(args):
    """--impl reference: the reference's CPU attention (oracle port), rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import oracle

    bh, s, d, causal, std, k_mul, seed, o_dtype, desc = WORKLOADS[args.workload]
    pad = PADDED.get(args.workload)
    if pad:  # the oracle reads the same values with the padding removed
        q, k, v = (a.reshape(s, pad["row"])[:, :d].reshape(-1).copy()
                   for a in make_padded_inputs(oracle, 1, s, d, pad["row"], pad["lo"], pad["hi"], seed))
    else:
        q, k, v = make_inputs(oracle, 1, s, d, std, k_mul, seed)
    scale = 1.0 / math.sqrt(d)
    threads = host_threads(oracle)
    budget = 90.0  # seconds of CPU work for the whole --steps/--warmup run
    _, dt_cal, _, _, _, rows_cal = cpu_sample(oracle, q, k, v, s, d, causal, scale, 1.0, threads)
    per_row = dt_cal / rows_cal
    rows = max(threads, int(budget / (args.steps + args.warmup) / per_row))
    rows = min(rows, s)
    import numpy as np

    out = np.zeros(s * d, dtype=np.float32)
    r0 = s - rows
    keys = sum((r + 1) if causal else s for r in range(r0, s))
    step_flops = 4 * keys * d
    times = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        oracle.flash_reference(q, k, v, batch_heads=1, seq_len=s, head_dim=d, q_stride=s * d, k_stride=s * d,
                               v_stride=s * d, o_stride=s * d, scale=scale, causal=causal, out=out,
                               rows=(r0, s), threads=threads)
        if i >= args.warmup:
            times.append(time.perf_counter() - t0)
    total = sum(times)
    value = step_flops * len(times) / total / 1e12
    sample = (f"rows {r0}..{s - 1} of one slice per step ({rows} rows, {step_flops / 1e9:.3f} GFLOP), "
              f"oracle restatement of src/main.zig:1271-1307, {threads} threads, {cpu_model()}")
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total / len(times) * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": desc, "batch_heads": bh, "seq_len": s, "head_dim": d, "causal": causal,
                   "parallelism": "cpu (rank 0 only)"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="c4")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--gather", action="store_true",
                    help="N > 1: also time gathering every rank's O shard on rank 0 (NCCL over NVLink), "
                         "separately from the metric")
    ap.add_argument("--splits", type=int, default=None,
                    help="force the split-KV count (ncz_flash_fwd_splits: 1 = none); default: automatic")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        return reference_arm(args)

    import numpy as np
    import torch

    import oracle

    ncz = importlib.import_module("not-cute-zig_b200")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        with _StdoutToStderr():
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
            dist.barrier()

    bh, s, d, causal, std, k_mul, seed, o_dtype, desc = WORKLOADS[args.workload]
    scale = 1.0 / math.sqrt(d)
    n = bh * s * d
    pad = PADDED.get(args.workload)
    row = pad["row"] if pad else d
    n_in = bh * s * row  # elements of each of Q, K, V (padding included)
    row_strides = (row, row, row, d) if pad else None
    # Weak scaling: every rank owns its own bh slices (seeded by rank).
    if pad:
        hq, hk, hv = make_padded_inputs(oracle, bh, s, d, row, pad["lo"], pad["hi"], seed + 1000 * rank)
    else:
        hq, hk, hv = make_inputs(oracle, bh, s, d, std, k_mul, seed + 1000 * rank)
    q = torch.from_numpy(hq).to(dev)
    k = torch.from_numpy(hk).to(dev)
    v = torch.from_numpy(hv).to(dev)
    tdt = torch.float16 if o_dtype == "f16" else torch.float32
    o = torch.empty(n, dtype=tdt, device=dev)
    working_set = 3 * n_in * 2 + n * o.element_size()
    # Inputs + O smaller than L2: flush L2 before every timed step (memset of a
    # 256 MB buffer, outside the timed intervals).
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev) if working_set <= L2_BYTES else None
    opts = ncz.Options(seq_len=s, head_dim=d, q_stride=s * row, k_stride=s * row, v_stride=s * row,
                       o_stride=s * d, scale=scale, batch_heads=bh, causal=causal)
    stream = torch.cuda.current_stream(dev)
    step_flops = flops_of(bh, s, d, causal)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def step():
        if args.splits is not None:
            ncz.launch_splits(q, k, v, o, opts, args.splits, row_strides=row_strides, stream=stream)
        elif o_dtype == "f16" or pad:
            ncz.launch_ex(q, k, v, o, opts, row_strides=row_strides, stream=stream)
        else:
            ncz.launch(q, k, v, o, opts, stream=stream)

    for _ in range(args.warmup):
        step()
    ncz.sync_status(device=local, stream=stream)
    barrier()
    sampler = ClockSampler(local)
    time.sleep(0.3)  # let the sampler start
    barrier()
    launches0 = ncz.flash.launch_count()
    if flush is None:
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(args.steps):
            step()
        end.record(stream)
        barrier()
        ms = start.elapsed_time(end)
    else:
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for e0, e1 in evs:
            flush.zero_()
            e0.record(stream)
            step()
            e1.record(stream)
        barrier()
        ms = sum(e0.elapsed_time(e1) for e0, e1 in evs)
    clocks = sampler.stop()
    launches = ncz.flash.launch_count() - launches0
    ncz.sync_status(device=local, stream=stream)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    ms_step = ms_max / args.steps
    value = world * step_flops * args.steps / (ms_max / 1e3) / 1e12
    per_gpu = step_flops / (ms_step / 1e3) / 1e12
    assert np.isfinite(o[: s * d].float().cpu().numpy()).all()

    # e2e through the C ABI with pinned host buffers: ncz_flash_fwd_host uploads
    # Q/K/V, runs the forward and downloads O in slice chunks on three streams.
    e2e = None
    if not args.no_e2e:
        pq, pk_, pv = (torch.from_numpy(a).pin_memory() for a in (hq, hk, hv))
        po = torch.empty(n, dtype=tdt).pin_memory()
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)

        def e2e_step():
            ncz.launch_host(pq, pk_, pv, po, dq, dk, dv, o, opts, row_strides=row_strides, stream=stream)

        for _ in range(3):
            e2e_step()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.e2e_steps):
            e2e_step()
        e1.record(stream)
        barrier()
        et = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
        if dist is not None:
            dist.all_reduce(et, op=dist.ReduceOp.MAX)
        e2e = {"value": world * step_flops * args.e2e_steps / (float(et.item()) / 1e3) / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": 3 * n_in * 2, "d2h_bytes_per_step": n * o.element_size(), "steps": args.e2e_steps,
               "api": "flash.launch_host -> ncz_flash_fwd_host (C ABI), default chunking"}

    # Optional O gather to rank 0 over NVLink (NCCL), off the timed metric.
    gather = None
    if args.gather and dist is not None:
        parts = [torch.empty_like(o) for _ in range(world)] if rank == 0 else None
        for _ in range(2):
            dist.gather(o, parts, dst=0)
        barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 5
        g0.record(stream)
        for _ in range(reps):
            dist.gather(o, parts, dst=0)
        g1.record(stream)
        barrier()
        gt = torch.tensor([g0.elapsed_time(g1) / reps], dtype=torch.float64, device=dev)
        dist.all_reduce(gt, op=dist.ReduceOp.MAX)
        gms = float(gt.item())
        moved = (world - 1) * n * o.element_size()
        gather = {"ms": gms, "bytes_to_rank0": moved, "gbps_into_rank0": moved / (gms * 1e6),
                  "how": "torch.distributed.gather of each rank's O shard to rank 0 (NCCL), max over ranks"}
        del parts

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cq, ck, cv = (a.reshape(bh, s, row)[:, :, :d].reshape(-1).copy() for a in (hq, hk, hv)) if pad else (hq, hk, hv)
        tf, dt, what, fl, thr, _ = cpu_sample(oracle, cq, ck, cv, s, d, causal, scale, args.cpu_seconds, bh=bh)
        cpu = {"value": tf, "unit": "TFLOP/s", "cores": thr, "kind": "port",
               "sample": f"oracle (restatement of src/main.zig:1271-1307) on {what} "
                         f"({fl / 1e9:.2f} GFLOP in {dt:.1f} s), {cpu_model()}"}

    if dist is not None:
        dist.barrier()
    if rank == 0:
        burst, sustained, src = load_peaks()
        timed_s = ms_max / 1e3
        peak = sustained if timed_s > 1.0 else burst
        traffic = load_traffic(args.workload)
        if pad:
            # HBM-bound: algorithmic bytes by the reference formula
            # (bh*S*d*(3*2 + O bytes), src/main.zig:845) per launch over its time.
            hbm, hsrc = load_hbm()
            gbs = n * (3 * 2 + o.element_size()) / (ms_step / 1e3) / 1e9
            roofline = {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                        "traffic": traffic, "peak_source": f"{hsrc} HBM copy",
                        "kernel": f"ncz::flash_fwd_sm100<{d},true,false>"}
        else:
            roofline = {"bound": "tensor", "achieved": per_gpu, "peak": peak, "unit": "TFLOP/s",
                        "frac": per_gpu / peak, "traffic": traffic,
                        "peak_source": f"{src} bf16 {'sustained' if peak == sustained else 'burst'}",
                        "kernel": f"ncz::flash_fwd_sm100<{d},true,false>"}
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": desc, "batch_heads_per_gpu": bh, "batch_heads_total": bh * world,
                       "seq_len": s, "head_dim": d, "causal": causal, "o_dtype": o_dtype,
                       "parallelism": f"slices sharded x{world}, no collective", "split_kv": "auto" if args.splits is None else args.splits,
                       "l2": ("inputs 3x%.1f MB + O %.1f MB > 126 MB L2; no flush" if flush is None else
                              "inputs 3x%.1f MB + O %.1f MB fit in L2: 256 MB memset before every timed step, "
                              "outside the timed intervals") % (n_in * 2 / 1e6, n * o.element_size() / 1e6)},
            "pct_peak_nominal": per_gpu / NOMINAL_F16_TFLOPS,
            "pct_peak_measured": per_gpu / peak,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "o_gather": gather,
            "gpu_launches": launches,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
