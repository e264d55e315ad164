"""Benchmark of the B200 flash-attention forward (the not-cute-zig `flash` path).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload c4|c2|c3|c5|c5d16] [--scaling strong|weak]
                  [--no-e2e] [--no-cpu] [--no-secondary]

One step = one launch of the hot path over one batch of synthetic input.
Headline (default): BASELINE config 4 -- batch_heads 64, seq_len 8192,
head_dim 64, causal, f16 Q/K/V N(0,1) with K x2, f32 O.  For N > 1 the script
runs under torch.distributed.run, one rank per GPU, and the workload's slices
are split across the ranks (strong scaling, slice ranges of shard.slice_range:
8 slices per GPU at N=8; the partition of src/flash.zig:49-53, slice =
grid.y); no collective on the data path.  --scaling weak gives every rank its
own full workload instead.  The step time is the max over ranks of the
CUDA-event time.

Metric: the reference's FLOP formula (src/main.zig:843-844) per second,
whole job.  The JSON line also carries the roofline of the kernel against
the measured B200 peak, an end-to-end number through the C ABI with host
buffers (H2D of Q/K/V and D2H of O inside the timed region), a CPU baseline
(the oracle, a restatement of src/main.zig:1271-1307, on a bounded sample),
the SM clocks sampled during the timed region, a parity record per rank
(the oracle as checker on one slice per rank, after the timed region), and,
unless --no-secondary, the other BASELINE configs (5 d=64, 5 d=16, 3, 2)
timed briefly after the headline as `workloads`.

--impl reference times the reference's CPU attention (the oracle port; the
Zig original cannot be built here) on the host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import hashlib
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
    # name: (batch_heads in total, seq_len, head_dim, causal, std, k_mul, seed, O dtype, description)
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
# The other BASELINE configs, timed after the headline (fewer steps).
SECONDARY = ("c5", "c5d16", "c3", "c2")
SECONDARY_STEPS = {"c5": 100, "c5d16": 100, "c3": 300, "c2": 300}
FALLBACK_HBM_GBS = 6650.0
L2_BYTES = 126 * 1024 * 1024
# Parity bounds (north star): max |gpu - oracle| and the per-element relative
# error |gpu - oracle| / max(|oracle|, REL_FLOOR).
ATOL, RTOL, REL_FLOOR = 2e-3, 1e-2, 1e-3
P_UNIT = 2.0 ** -11  # unit roundoff of P rounded to f16 before PV (src/flash_h64_bn32.zig:185)
PARITY_ROWS = 128  # rows at the head and at the tail of the checked slice
# Sources the committed ncu traffic figures were measured on (their hash is
# recorded in each profiles/flash_fwd_<workload>_traffic.txt).
KERNEL_SOURCES = ("not-cute-zig_b200/csrc/flash_fwd_sm100.cuh", "not-cute-zig_b200/csrc/sm100_ptx.cuh",
                  "not-cute-zig_b200/csrc/flash_api.cu")


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


def kernel_sources_hash():
    """sha256 (first 16 hex digits) of the kernel sources, in KERNEL_SOURCES order."""
    h = hashlib.sha256()
    for rel in KERNEL_SOURCES:
        with open(os.path.join(ROOT, rel), "rb") as f:
            h.update(f.read())
    return h.hexdigest()[:16]


def load_traffic(workload):
    """DRAM bytes per launch from the committed ncu summary, with where it came
    from: (bytes or None, {"file", "kernel_sources_sha256", "current", "stale"}).
    A summary measured on other kernel sources than the ones built now is
    reported as stale."""
    rel = os.path.join("profiles", f"flash_fwd_{workload}_traffic.txt")
    traffic, recorded = None, None
    try:
        with open(os.path.join(ROOT, rel)) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    traffic = float(line.split(":", 1)[1].split()[0])
                elif line.startswith("kernel_sources_sha256:"):
                    recorded = line.split(":", 1)[1].strip()
    except OSError:
        return None, None
    cur = kernel_sources_hash()
    return traffic, {"file": rel, "kernel_sources_sha256": recorded, "current": cur, "stale": recorded != cur}


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


def make_inputs(oracle, bh, s, d, std, k_mul, seed, first_slice=0):
    """Q, K, V of slices first_slice .. first_slice+bh-1 of a workload's seeded
    N(0, std^2) streams (K scaled by k_mul): the same bits whatever the shard."""
    n, first = bh * s * d, first_slice * s * d
    q = oracle.fill_normal(n, seed * 3 + 0, 0.0, std, first=first)
    k = oracle.fill_normal(n, seed * 3 + 1, 0.0, std * k_mul, first=first)
    v = oracle.fill_normal(n, seed * 3 + 2, 0.0, std, first=first)
    return q, k, v


def make_padded_inputs(oracle, bh, s, d, row, lo, hi, seed, first_slice=0):
    """Q, K, V of bh slices of s rows `row` elements apart: U(lo, hi) values
    (seeds seed*3 + 0..2), NaN in each row's padding columns; slices
    first_slice .. first_slice+bh-1 of the workload's streams."""
    out = []
    for i in range(3):
        a = oracle.fill_uniform(bh * s * row, seed * 3 + i, lo, hi, first=first_slice * s * row)
        oracle.fill_row_padding(a, bh, s, d, s * row, row)
        out.append(a)
    return out


def workload_inputs(oracle, name, lo, hi, seed_shift=0):
    """Host Q, K, V of slices [lo, hi) of workload `name` (seed + seed_shift)."""
    _, s, d, _, std, k_mul, seed, _, _ = WORKLOADS[name]
    pad = PADDED.get(name)
    if pad:
        return make_padded_inputs(oracle, hi - lo, s, d, pad["row"], pad["lo"], pad["hi"], seed + seed_shift, lo)
    return make_inputs(oracle, hi - lo, s, d, std, k_mul, seed + seed_shift, lo)


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


# ---------------------------------------------------------------------------
# CPU leg: the oracle (restated reference CPU attention) on a bounded sample
# ---------------------------------------------------------------------------
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


def parity_check(oracle, name, hq, hk, hv, o_host, lo, hi, rows=PARITY_ROWS, threads=0):
    """The oracle as checker on one slice of this rank's shard (the middle one),
    rows [0, rows) and [S - rows, S).  Per element: |gpu - oracle| <= ATOL
    (plus half an f16 ulp of |O| for f16 O) and |gpu - oracle| <= RTOL *
    max(|oracle|, REL_FLOOR) + P_UNIT * mag, where mag = sum_k w_k |v_k| (from
    the oracle) bounds what the reference's rounding of P to f16
    (src/flash_h64_bn32.zig:185) can change.  Also reported: the plain
    per-element relative error and how many elements exceed RTOL by it, and the
    norm-relative error max|gpu - oracle| / max|oracle|."""
    import numpy as np

    _, s, d, causal, _, _, _, o_dtype, _ = WORKLOADS[name]
    pad = PADDED.get(name)
    row = pad["row"] if pad else d
    local = (hi - lo) // 2
    st = s * row
    q, k, v = (a[local * st:(local + 1) * st] for a in (hq, hk, hv))
    got = o_host.reshape(hi - lo, s, d)[local].astype(np.float64)
    bands = [(0, min(rows, s))] + ([(max(rows, s - rows), s)] if s > rows else [])
    max_abs = max_rel = norm_num = norm_den = ratio = 0.0
    viol = rel_over = 0
    for r0, r1 in bands:
        want = np.zeros(s * d, dtype=np.float32)
        mag = np.zeros(s * d, dtype=np.float32)
        oracle.flash_reference(q, k, v, batch_heads=1, seq_len=s, head_dim=d, q_stride=st, k_stride=st,
                               v_stride=st, o_stride=s * d, scale=1.0 / math.sqrt(d), causal=causal,
                               row_strides=(row, row, row, d), out=want, rows=(r0, r1), threads=threads, mag=mag)
        w = want.reshape(s, d)[r0:r1].astype(np.float64)
        mg = mag.reshape(s, d)[r0:r1].astype(np.float64)
        g = got[r0:r1]
        err = np.abs(g - w)
        o_unit = 2.0 ** -11 if o_dtype == "f16" else 0.0
        floor = np.maximum(np.abs(w), REL_FLOOR)
        rel = err / floor
        allow = RTOL * floor + P_UNIT * mg
        max_abs = max(max_abs, float(err.max()))
        max_rel = max(max_rel, float(rel.max()))
        ratio = max(ratio, float((err / allow).max()))
        norm_num, norm_den = max(norm_num, float(err.max())), max(norm_den, float(np.abs(w).max()))
        viol += int((err > ATOL + o_unit * np.abs(w)).sum() + (err > allow).sum())
        rel_over += int((rel > RTOL).sum())
    finite = bool(np.isfinite(o_host).all())
    return {"slice": lo + local, "rows": [list(b) for b in bands], "max_abs": max_abs, "max_rel": max_rel,
            "rel_over": rel_over, "allowance_ratio": ratio, "norm_rel": norm_num / max(norm_den, 1e-30),
            "violations": viol, "finite": finite, "ok": finite and viol == 0}


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
        "scaling": args.scaling, "vs_baseline": None, "dtype": "f32", "data": "synthetic",
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
class Ctx:
    """Per-process state shared by the workloads of one run."""

    def __init__(self, args, torch, dist, ncz, oracle, world, rank, local):
        self.args, self.torch, self.dist, self.ncz, self.oracle = args, torch, dist, ncz, oracle
        self.world, self.rank, self.local = world, rank, local
        self.dev = torch.device("cuda", local)
        self.stream = torch.cuda.current_stream(self.dev)

    def barrier(self):
        if self.dist is not None:
            self.dist.barrier()
        self.torch.cuda.synchronize(self.dev)

    def max_over_ranks(self, x):
        t = self.torch.tensor([float(x)], dtype=self.torch.float64, device=self.dev)
        if self.dist is not None:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def gather_rows(self, vals):
        """Every rank's list of floats, on every rank (a collective: all ranks call it)."""
        t = self.torch.tensor([float(x) for x in vals], dtype=self.torch.float64, device=self.dev)
        if self.dist is None:
            return [[float(x) for x in t.tolist()]]
        out = self.torch.empty(self.world * t.numel(), dtype=self.torch.float64, device=self.dev)
        self.dist.all_gather_into_tensor(out, t)
        return [list(map(float, r)) for r in out.view(self.world, -1).tolist()]


def run_workload(cx, name, steps, warmup, *, e2e_steps=0, cpu=False, gather=False):
    """Times one workload on this rank's slices; every rank calls it with the
    same arguments (the collectives inside line up).  Returns the record on
    rank 0, None elsewhere."""
    import numpy as np

    torch, ncz, oracle, args = cx.torch, cx.ncz, cx.oracle, cx.args
    bh_total, s, d, causal, std, k_mul, seed, o_dtype, desc = WORKLOADS[name]
    scale = 1.0 / math.sqrt(d)
    pad = PADDED.get(name)
    row = pad["row"] if pad else d
    weak = args.scaling == "weak"
    if weak:  # every rank owns a whole workload of its own (seeded by rank)
        lo, hi, shift = 0, bh_total, 1000 * cx.rank
    else:
        shard = importlib.import_module("not-cute-zig_b200.shard")
        lo, hi = shard.slice_range(bh_total, cx.world, cx.rank)
        shift = 0
    bh = hi - lo  # slices on this rank (>= 1: bh_total >= world is checked by the caller)
    job_slices = bh_total * cx.world if weak else bh_total
    job_flops = flops_of(job_slices, s, d, causal)
    hq, hk, hv = workload_inputs(oracle, name, lo, hi, shift)
    n_in = bh * s * row
    n = bh * s * d
    q, k, v = (torch.from_numpy(a).to(cx.dev) for a in (hq, hk, hv))
    tdt = torch.float16 if o_dtype == "f16" else torch.float32
    o = torch.empty(n, dtype=tdt, device=cx.dev)
    working_set = 3 * n_in * 2 + n * o.element_size()
    # Inputs + O smaller than L2: flush L2 before every timed step (memset of a
    # 256 MB buffer, outside the timed intervals).
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=cx.dev) if working_set <= L2_BYTES else None
    opts = ncz.Options(seq_len=s, head_dim=d, q_stride=s * row, k_stride=s * row, v_stride=s * row,
                       o_stride=s * d, scale=scale, batch_heads=bh, causal=causal)
    row_strides = (row, row, row, d) if pad else None
    stream = cx.stream

    def step():
        if args.splits is not None:
            ncz.launch_splits(q, k, v, o, opts, args.splits, row_strides=row_strides, stream=stream)
        elif o_dtype == "f16" or pad:
            ncz.launch_ex(q, k, v, o, opts, row_strides=row_strides, stream=stream)
        else:
            ncz.launch(q, k, v, o, opts, stream=stream)

    for _ in range(warmup):
        step()
    ncz.sync_status(device=cx.local, stream=stream)
    cx.barrier()
    sampler = ClockSampler(cx.local)
    time.sleep(0.3)  # let the sampler start
    cx.barrier()
    launches0 = ncz.flash.launch_count()
    if flush is None:
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(steps):
            step()
        end.record(stream)
        cx.barrier()
        ms = start.elapsed_time(end)
    else:
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for e0, e1 in evs:
            flush.zero_()
            e0.record(stream)
            step()
            e1.record(stream)
        cx.barrier()
        ms = sum(e0.elapsed_time(e1) for e0, e1 in evs)
    clocks = sampler.stop()
    launches = ncz.flash.launch_count() - launches0
    status = ncz.sync_status(device=cx.local, stream=stream)
    ms_max = cx.max_over_ranks(ms)
    ms_step = ms_max / steps
    value = job_flops * steps / (ms_max / 1e3) / 1e12
    per_gpu = value / cx.world

    # Parity after the timed region: the oracle checks one slice of this rank's shard.
    par = parity_check(oracle, name, hq, hk, hv, o.float().cpu().numpy(), lo, hi,
                       threads=max(1, host_threads(oracle) // cx.world))
    par["status"] = status
    per_rank = cx.gather_rows([par["slice"], par["max_abs"], par["max_rel"], par["norm_rel"], par["violations"],
                               par["rel_over"], par["allowance_ratio"], 1.0 if par["ok"] and status == 0 else 0.0])

    # e2e through the C ABI with pinned host buffers: ncz_flash_fwd_host uploads
    # Q/K/V, runs the forward and downloads O in slice chunks on three streams.
    e2e = None
    if e2e_steps > 0:
        pq, pk_, pv = (torch.from_numpy(a).pin_memory() for a in (hq, hk, hv))
        po = torch.empty(n, dtype=tdt).pin_memory()
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)

        def e2e_step():
            ncz.launch_host(pq, pk_, pv, po, dq, dk, dv, o, opts, row_strides=row_strides, stream=stream)

        for _ in range(3):
            e2e_step()
        cx.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        e1.record(stream)
        cx.barrier()
        et = cx.max_over_ranks(e0.elapsed_time(e1))
        h2d, d2h = 3 * n_in * 2, n * o.element_size()
        e2e = {"value": job_flops * e2e_steps / (et / 1e3) / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": e2e_steps,
               "ms_per_step": et / e2e_steps,
               "host_copy_gbs_all_ranks": cx.world * (h2d + d2h) * e2e_steps / (et / 1e3) / 1e9,
               "api": "flash.launch_host -> ncz_flash_fwd_host (C ABI), default chunking"}
        del pq, pk_, pv, po, dq, dk, dv

    # Optional O gather to rank 0 over NVLink (NCCL), off the timed metric.
    og = None
    if gather and cx.dist is not None and not weak and bh_total % cx.world == 0:
        dist = cx.dist
        parts = [torch.empty_like(o) for _ in range(cx.world)] if cx.rank == 0 else None
        for _ in range(2):
            dist.gather(o, parts, dst=0)
        cx.barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 5
        g0.record(stream)
        for _ in range(reps):
            dist.gather(o, parts, dst=0)
        g1.record(stream)
        cx.barrier()
        gms = cx.max_over_ranks(g0.elapsed_time(g1) / reps)
        moved = (cx.world - 1) * n * o.element_size()
        og = {"ms": gms, "bytes_to_rank0": moved, "gbps_into_rank0": moved / (gms * 1e6),
              "how": "torch.distributed.gather of each rank's O shard to rank 0 (NCCL), max over ranks"}
        del parts

    cpu_rec = None
    if cpu and cx.rank == 0 and cx.world == 1 and not args.no_cpu:
        cq, ck, cv = ((a.reshape(bh, s, row)[:, :, :d].reshape(-1).copy() for a in (hq, hk, hv)) if pad
                      else (hq, hk, hv))
        tf, dt, what, fl, thr, _ = cpu_sample(oracle, cq, ck, cv, s, d, causal, scale, args.cpu_seconds, bh=bh)
        cpu_rec = {"value": tf, "unit": "TFLOP/s", "cores": thr, "kind": "port",
                   "sample": f"oracle (restatement of src/main.zig:1271-1307) on {what} "
                             f"({fl / 1e9:.2f} GFLOP in {dt:.1f} s), {cpu_model()}"}
    flushed = flush is not None
    del q, k, v, o, flush
    torch.cuda.empty_cache()
    if cx.rank != 0:
        return None

    burst, sustained, src = load_peaks()
    peak = sustained if ms_max / 1e3 > 1.0 else burst
    traffic, traffic_src = load_traffic(name)
    kernel = f"ncz::flash_fwd_sm100<{d},true,false>"
    if pad:
        # HBM-bound: algorithmic bytes by the reference formula
        # (bh*S*d*(3*2 + O bytes), src/main.zig:845) per launch over its time.
        hbm, hsrc = load_hbm()
        gbs = n * (3 * 2 + (2 if o_dtype == "f16" else 4)) / (ms_step / 1e3) / 1e9
        roofline = {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                    "traffic": traffic, "traffic_source": traffic_src, "peak_source": f"{hsrc} HBM copy",
                    "kernel": kernel}
    else:
        roofline = {"bound": "tensor", "achieved": per_gpu, "peak": peak, "unit": "TFLOP/s",
                    "frac": per_gpu / peak, "traffic": traffic, "traffic_source": traffic_src,
                    "peak_source": f"{src} bf16 {'sustained' if peak == sustained else 'burst'}", "kernel": kernel}
    ranks = [{"rank": i, "slice": int(r[0]), "max_abs": r[1], "max_rel": r[2], "norm_rel": r[3],
              "violations": int(r[4]), "rel_over": int(r[5]), "allowance_ratio": r[6], "ok": bool(r[7])}
             for i, r in enumerate(per_rank)]
    parity = {"checker": "oracle (restatement of src/main.zig:1271-1307), after the timed region",
              "rows_per_slice": par["rows"], "atol": ATOL, "rel": f"|a-b|/max(|b|,{REL_FLOOR:g})",
              "gate": f"|a-b| <= {ATOL:g} and |a-b| <= {RTOL:g}*max(|b|,{REL_FLOOR:g}) + 2^-11*sum_k w_k|v_k|",
              "max_abs": max(r["max_abs"] for r in ranks), "max_rel": max(r["max_rel"] for r in ranks),
              "rel_over": sum(r["rel_over"] for r in ranks),
              "allowance_ratio": max(r["allowance_ratio"] for r in ranks),
              "norm_rel": max(r["norm_rel"] for r in ranks), "ok": all(r["ok"] for r in ranks), "ranks": ranks}
    return {
        "value": value, "ms_per_step": ms_step, "steps": steps, "warmup": warmup, "per_gpu": per_gpu,
        "gpu_launches": launches, "clocks": clocks, "roofline": roofline, "parity": parity, "e2e": e2e,
        "o_gather": og, "cpu_baseline": cpu_rec,
        "config": {"workload": desc, "batch_heads": job_slices, "batch_heads_per_gpu": bh, "seq_len": s,
                   "head_dim": d, "causal": causal, "o_dtype": o_dtype,
                   "parallelism": (f"every rank its own {bh_total} slices x{cx.world}, no collective" if weak else
                                   f"{bh_total} slices split over {cx.world} GPU(s) (shard.slice_range), "
                                   "no collective"),
                   "split_kv": "auto" if args.splits is None else args.splits,
                   "l2": ("inputs 3x%.1f MB + O %.1f MB > 126 MB L2; no flush" if not flushed else
                          "inputs 3x%.1f MB + O %.1f MB fit in L2: 256 MB memset before every timed step, "
                          "outside the timed intervals") % (n_in * 2 / 1e6, n * (2 if o_dtype == "f16" else 4) / 1e6)},
        "pct_peak_nominal": per_gpu / NOMINAL_F16_TFLOPS,
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="c4")
    ap.add_argument("--scaling", choices=["strong", "weak"], default="strong",
                    help="strong: the workload's slices split over the ranks; weak: every rank its own workload")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-secondary", action="store_true",
                    help="time the headline workload only (not the other BASELINE configs)")
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

    import torch

    import oracle

    ncz = importlib.import_module("not-cute-zig_b200")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        with _StdoutToStderr():
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", local))
            dist.barrier()
    cx = Ctx(args, torch, dist, ncz, oracle, world, rank, local)

    head = run_workload(cx, args.workload, args.steps, args.warmup, e2e_steps=0 if args.no_e2e else args.e2e_steps,
                        cpu=True, gather=args.gather)
    secondary = {}
    if not args.no_secondary and args.workload == "c4" and args.splits is None:
        for name in SECONDARY:
            if args.scaling == "strong" and WORKLOADS[name][0] < world:
                continue  # fewer slices than GPUs: nothing to split
            rec = run_workload(cx, name, SECONDARY_STEPS[name], args.warmup)
            if rank == 0:
                secondary[name] = {key: rec[key] for key in ("value", "ms_per_step", "steps", "per_gpu",
                                                             "gpu_launches", "clocks", "roofline", "parity",
                                                             "config", "pct_peak_nominal")}

    if dist is not None:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": METRIC, "value": head["value"], "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True,
            "scaling": args.scaling, "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": head["config"],
            "pct_peak_nominal": head["pct_peak_nominal"],
            "pct_peak_measured": head["roofline"]["frac"] if head["roofline"]["bound"] == "tensor" else None,
            "roofline": head["roofline"],
            "cpu_baseline": head["cpu_baseline"],
            "e2e": head["e2e"],
            "parity": head["parity"],
            "o_gather": head["o_gather"],
            "gpu_launches": head["gpu_launches"],
            "clocks": head["clocks"],
            "workloads": secondary or None,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
