"""Event-timed benchmarking and JSONL records, after src/benchmark.zig and the
compare records of src/main.zig:859-881.

run_kernel mirrors benchmark.runKernel (src/benchmark.zig:35-92): W warm-up
launches, a synchronize, then I launches each bracketed by its own event pair
(record start, launch, record stop, wait for stop), reporting mean/min/max in
milliseconds and, given the algorithmic bytes / FLOPs, GB/s and TFLOP/s from
the mean.  run_multi is the multi-device form: per device its own event pair
per iteration, the iteration time is the slowest device, and the host
wall-clock of the all-device launch is reported beside it.
"""
from __future__ import annotations

import json
import logging
import os
import time
from dataclasses import dataclass, field
from typing import Callable, List, Optional, Sequence

log = logging.getLogger("not-cute-zig_b200")


@dataclass
class BenchmarkResult:
    """src/benchmark.zig:6-23."""

    mean_ms: float
    min_ms: float
    max_ms: float
    throughput_gbps: Optional[float] = None
    tflops: Optional[float] = None
    device_ms: List[float] = field(default_factory=list)  # per device (run_multi), mean over iterations
    host_ms: Optional[float] = None                       # host wall-clock per iteration (run_multi)

    def print(self, name: str) -> None:
        log.info("--- Benchmark: %s ---", name)
        log.info("  Time: mean=%.3fms, min=%.3fms, max=%.3fms", self.mean_ms, self.min_ms, self.max_ms)
        if self.throughput_gbps is not None:
            log.info("  Bandwidth: %.2f GB/s", self.throughput_gbps)
        if self.tflops is not None:
            log.info("  Compute:   %.2f TFLOPs", self.tflops)

    def record(self, kernel: str, implementation: str, shape: str, correct: bool, bytes_: int, flops: int,
               max_abs_error: Optional[float] = None, **extra) -> dict:
        """One compare record (src/main.zig:859-881 field order), plus `extra`
        fields (gpus, device_ms, pct_peak_nominal, pct_peak_measured,
        max_rel_error, host_cores, ...)."""
        rec = {"kernel": kernel, "implementation": implementation, "shape": shape, "correct": bool(correct),
               "mean_ms": self.mean_ms, "min_ms": self.min_ms, "max_ms": self.max_ms,
               "gbps": self.throughput_gbps or 0.0, "tflops": self.tflops or 0.0, "bytes": int(bytes_),
               "flops": int(flops)}
        if max_abs_error is not None:
            rec["max_abs_error"] = float(max_abs_error)
        rec.update(extra)
        return rec


def _rates(mean_ms: float, bytes_processed: Optional[int], flops_processed: Optional[int]):
    # src/benchmark.zig:79-86: GB/s = bytes / (mean_ms * 1e6); TFLOP/s = flops / (mean_ms * 1e9)
    gbps = bytes_processed / (mean_ms * 1e6) if bytes_processed is not None else None
    tflops = flops_processed / (mean_ms * 1e9) if flops_processed is not None else None
    return gbps, tflops


def summarize(times_ms: Sequence[float], bytes_processed: Optional[int] = None,
              flops_processed: Optional[int] = None) -> BenchmarkResult:
    """mean/min/max and rates of per-iteration times (no device work; tested on CPU)."""
    if not times_ms:
        raise ValueError("no iterations")
    mean = sum(times_ms) / len(times_ms)
    gbps, tflops = _rates(mean, bytes_processed, flops_processed)
    return BenchmarkResult(mean, min(times_ms), max(times_ms), gbps, tflops)


def run_kernel(launch: Callable[[], None], *, warmup_iters: int = 3, iters: int = 10,
               bytes_processed: Optional[int] = None, flops_processed: Optional[int] = None,
               stream=None) -> BenchmarkResult:
    """benchmark.runKernel: `launch` enqueues one launch on `stream` (default:
    the current torch stream of the current device)."""
    import torch

    stream = stream or torch.cuda.current_stream()
    for _ in range(warmup_iters):
        launch()
    stream.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = []
    for _ in range(iters):
        start.record(stream)
        launch()
        stop.record(stream)
        stop.synchronize()
        times.append(start.elapsed_time(stop))
    return summarize(times, bytes_processed, flops_processed)


def run_multi(launches: Sequence[Callable[[], None]], streams: Sequence, *, warmup_iters: int = 3,
              iters: int = 10, bytes_processed: Optional[int] = None,
              flops_processed: Optional[int] = None) -> BenchmarkResult:
    """Multi-device runKernel: launches[i] enqueues device i's share on
    streams[i] (a stream of that device).  Per iteration every device has its
    own event pair; the iteration time is the slowest device; bytes/FLOPs are
    the whole job's.  device_ms holds each device's mean, host_ms the mean host
    wall-clock from the first launch to the last device's completion."""
    import torch

    if len(launches) != len(streams) or not launches:
        raise ValueError("one stream per launch")
    for _ in range(warmup_iters):
        for fn in launches:
            fn()
    for s in streams:
        s.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in streams]
    per_iter, per_dev, host = [], [[] for _ in streams], []
    for _ in range(iters):
        t0 = time.perf_counter()
        for (e0, e1), s, fn in zip(evs, streams, launches):
            e0.record(s)
            fn()
            e1.record(s)
        for _, e1 in evs:
            e1.synchronize()
        host.append((time.perf_counter() - t0) * 1e3)
        ms = [e0.elapsed_time(e1) for e0, e1 in evs]
        for i, v in enumerate(ms):
            per_dev[i].append(v)
        per_iter.append(max(ms))
    res = summarize(per_iter, bytes_processed, flops_processed)
    res.device_ms = [sum(v) / len(v) for v in per_dev]
    res.host_ms = sum(host) / len(host)
    return res


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def emit(records: Sequence[dict], path: Optional[str] = None) -> None:
    """Writes JSONL: one record per line, to `path` (appended) or stdout."""
    lines = "".join(json.dumps(r) + "\n" for r in records)
    if path:
        with open(path, "a") as f:
            f.write(lines)
    else:
        print(lines, end="", flush=True)
