"""Flash-attention compare / benchmark harness with the reference's JSONL records.

Mirrors compareFlash (src/main.zig:975-1041) and benchmarkFlash
(src/main.zig:790-856): fillFlashInput inputs (src/main.zig:1207-1211),
5 warm-up + 20 timed launches through benchmark.run_kernel, algorithmic
bytes and FLOPs by the reference formulas (src/main.zig:843-845), and one
JSONL record per shape in the reference's field order (src/main.zig:873-881)
plus gpus, device_ms, pct_peak_nominal, pct_peak_measured, max_rel_error,
host_cores, cpu_ms (with --cpu-ms: the same fp32 attention timed on the host
CPU) and label.  Correctness is checked against plain fp32 attention in
torch on the same device (max-abs <= 0.02, the reference's compare bound,
src/main.zig:1042); rel = |a - b| / max(|b|, 1e-3).

    python not-cute-zig_b200/compare.py                  # the 15 reference shapes
    python not-cute-zig_b200/compare.py --shape 8,1024,64,1 --gpus 2 --jsonl out.jsonl
    python not-cute-zig_b200/compare.py --shape 4,1000,32,1 --row-stride 40 --in-dtype bf16 --o-dtype f16 --seed 7
    python not-cute-zig_b200/compare.py --mma        # GEMM + epilogue (compareMma, src/main.zig:953-975)
    python not-cute-zig_b200/compare.py --join ours.jsonl sdpa.jsonl cuda.jsonl   # joined table

--join reads JSONL records of several harnesses (this one, the reference's
tools/cuda_baselines.cu and tools/pytorch_baselines.py) and prints, per
(kernel, shape), this library's time against every other implementation's,
as the reference's modal_run.py:34-69 joins them.
"""
from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import sys
from typing import List, Optional, Tuple

_HERE = os.path.dirname(os.path.abspath(__file__))
if os.path.dirname(_HERE) not in sys.path:
    sys.path.insert(0, os.path.dirname(_HERE))

# compareFlash calls, src/main.zig:141-170: (batch_heads, seq_len, head_dim, causal)
REFERENCE_SHAPES: List[Tuple[int, int, int, bool]] = [
    (2, 32, 16, False), (2, 32, 32, True), (2, 64, 16, False), (2, 64, 32, True), (2, 128, 32, True),
    (8, 128, 16, False), (8, 128, 32, True), (8, 256, 16, False), (8, 256, 32, True), (16, 256, 32, False),
    (16, 512, 32, True), (8, 256, 64, False), (8, 512, 64, True), (16, 512, 64, False), (8, 1024, 64, True),
]
NOMINAL_F16_TFLOPS = 2250.0


def fill_flash_input(n: int, mul: int, add: int, scale: float):
    """fillFlashInput: f16(((i * mul + add) % 17) * scale), src/main.zig:1207-1211."""
    import numpy as np

    i = np.arange(n, dtype=np.int64)
    return (((i * mul + add) % 17).astype(np.float32) * np.float32(scale)).astype(np.float16)


def torch_attention(q, k, v, bh: int, s: int, d: int, scale: float, causal: bool, row: int = 0):
    """fp32 attention in torch (cross-check only): softmax(QK^T * scale, causal
    top-left) V, per slice; rows `row` elements apart (0 = d), flat result of
    bh * s * d elements."""
    import torch

    row = row or d
    qf, kf, vf = (t.view(bh, s, row)[:, :, :d].float() for t in (q, k, v))
    scores = torch.matmul(qf, kf.transpose(1, 2)) * scale
    if causal:
        mask = torch.ones(s, s, dtype=torch.bool, device=q.device).triu(1)
        scores = scores.masked_fill(mask, float("-inf"))
    return torch.matmul(torch.softmax(scores, dim=-1), vf).reshape(-1)


def host_reference_ms(q, k, v, bh: int, s: int, d: int, scale: float, causal: bool, row: int = 0) -> float:
    """Wall time (ms) of the fp32 cross-check attention computed on the host
    CPU with torch's threads: the cpu_ms field of a record."""
    import time

    qc, kc, vc = (t.detach().cpu() for t in (q, k, v))
    t0 = time.perf_counter()
    torch_attention(qc, kc, vc, bh, s, d, scale, causal, row)
    return (time.perf_counter() - t0) * 1e3


def measured_peak() -> Optional[float]:
    path = os.path.join(os.path.dirname(_HERE), "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        return None


IN_DTYPES = {"f16": "float16", "bf16": "bfloat16"}
O_DTYPES = {"f32": ("float32", 4), "f16": ("float16", 2), "bf16": ("bfloat16", 2)}


def compare_shape(ncz, bh: int, s: int, d: int, causal: bool, gpus: int = 1, *, seed: Optional[int] = None,
                  in_dtype: str = "f16", o_dtype: str = "f32", row_stride: int = 0, cpu_ms: bool = False) -> dict:
    """One compareFlash record.  Defaults are the reference's: fillFlashInput
    inputs, f16 Q/K/V, f32 O, rows of head_dim elements, through flash.launch.
    `seed` draws N(0, 1) inputs instead; `in_dtype` / `o_dtype` / `row_stride`
    (elements between rows, >= head_dim; the padding of O must stay untouched)
    go through the extended descriptor (flash.launch_ex)."""
    import numpy as np
    import torch

    from importlib import import_module

    bench = import_module("not-cute-zig_b200.benchmark")
    shard = import_module("not-cute-zig_b200.shard")
    row = row_stride or d
    if row < d:
        raise ValueError(f"row stride {row} < head_dim {d}")
    extended = row != d or in_dtype != "f16" or o_dtype != "f32"
    in_torch = getattr(torch, IN_DTYPES[in_dtype])
    o_name, o_bytes = O_DTYPES[o_dtype]
    o_torch = getattr(torch, o_name)
    stride = s * row
    n = bh * stride
    scale = 1.0 / math.sqrt(d)
    if seed is None:
        hq, hk, hv = (fill_flash_input(n, 3, 1, 0.125), fill_flash_input(n, 5, 2, 0.0625),
                      fill_flash_input(n, 7, 3, 0.03125))
    else:
        rng = np.random.default_rng(seed)
        hq, hk, hv = (rng.standard_normal(n, dtype=np.float32) for _ in range(3))
    flops = bh * (4 * ((s * (s + 1)) // 2 if causal else s * s) * d)
    bytes_ = bh * s * d * (2 * 3 + o_bytes)
    gpus = max(1, min(gpus, torch.cuda.device_count(), bh))
    launches, streams, outs = [], [], []
    for g in range(gpus):
        lo, hi = shard.slice_range(bh, gpus, g)
        dev = torch.device("cuda", g)
        q, k, v = (torch.from_numpy(h[lo * stride:hi * stride]).to(dev).to(in_torch) for h in (hq, hk, hv))
        o = torch.zeros((hi - lo) * stride, dtype=o_torch, device=dev)
        st = torch.cuda.Stream(dev)
        opts = ncz.Options(seq_len=s, head_dim=d, q_stride=stride, k_stride=stride, v_stride=stride,
                           o_stride=stride, scale=scale, batch_heads=hi - lo, causal=causal)
        if extended:
            launches.append(lambda q=q, k=k, v=v, o=o, opts=opts, st=st: ncz.launch_ex(
                q, k, v, o, opts, row_strides=(row,) * 4, stream=st))
        else:
            launches.append(lambda q=q, k=k, v=v, o=o, opts=opts, st=st: ncz.launch(q, k, v, o, opts, stream=st))
        streams.append(st)
        outs.append((q, k, v, o, lo, hi))
    if gpus == 1:
        res = bench.run_kernel(launches[0], warmup_iters=5, iters=20, bytes_processed=bytes_,
                               flops_processed=flops, stream=streams[0])
        res.device_ms = [res.mean_ms]
    else:
        res = bench.run_multi(launches, streams, warmup_iters=5, iters=20, bytes_processed=bytes_,
                              flops_processed=flops)
    max_abs, max_rel, padding_kept = 0.0, 0.0, True
    cpu_total = 0.0 if cpu_ms else None
    for (q, k, v, o, lo, hi), st in zip(outs, streams):
        st.synchronize()
        ncz.sync_status(device=q.device.index, stream=st)
        want = torch_attention(q, k, v, hi - lo, s, d, scale, causal, row)
        got = o.view(hi - lo, s, row)
        diff = (got[:, :, :d].float().reshape(-1) - want).abs()
        max_abs = max(max_abs, float(diff.max()))
        max_rel = max(max_rel, float((diff / want.abs().clamp_min(1e-3)).max()))
        padding_kept = padding_kept and bool((got[:, :, d:] == 0).all())
        if cpu_ms:
            cpu_total += host_reference_ms(q, k, v, hi - lo, s, d, scale, causal, row)
    peak = measured_peak()
    shape = f"batch_heads={bh},seq={s},head={d},causal={str(causal).lower()}"
    if extended:
        shape += f",row_stride={row},in={in_dtype},o={o_dtype}"
    if seed is not None:
        shape += f",seed={seed}"
    label = ncz.select_kernel(ncz.Options(seq_len=s, head_dim=d, q_stride=stride, k_stride=stride,
                                          v_stride=stride, o_stride=stride, scale=scale, batch_heads=bh,
                                          causal=causal)).label
    return res.record("flash_attention", "not_cute_zig_b200", shape, max_abs <= 0.02 and padding_kept, bytes_,
                      flops, max_abs,
                      gpus=gpus, device_ms=res.device_ms, host_ms=res.host_ms,
                      pct_peak_nominal=(res.tflops or 0.0) / NOMINAL_F16_TFLOPS,
                      pct_peak_measured=((res.tflops or 0.0) / peak) if peak else None,
                      max_rel_error=max_rel, host_cores=bench.host_cores(), cpu_ms=cpu_total, label=label)


def measured_hbm() -> Optional[float]:
    path = os.path.join(os.path.dirname(_HERE), "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return None


def torch_gemm(a, b, c, batches: int, k_iters: int, alpha: float, beta: float, epilogue: int, b_col: bool):
    """fp32 D = act(alpha * A B + beta * C) per batch in torch (cross-check
    only), the activations written as src/device.zig:57-80 writes them (exp2
    forms; silu and gelu give NaN where exp2 overflows, as there)."""
    import torch

    am = a.view(batches, k_iters, 16, 16).float().permute(0, 2, 1, 3).reshape(batches, 16, 16 * k_iters)
    if b_col:
        bm = b.view(batches, k_iters, 8, 16).float().transpose(2, 3).reshape(batches, 16 * k_iters, 8)
    else:
        bm = b.view(batches, k_iters, 16, 8).float().reshape(batches, 16 * k_iters, 8)
    out = alpha * torch.bmm(am, bm) + beta * c.view(batches, 16, 8)
    log2e = 1.4426950408889634
    if epilogue == 1:
        out = torch.relu(out)
    elif epilogue == 2:
        e = torch.exp2(out * log2e)
        out = out * (e / (1.0 + e))
    elif epilogue == 3:
        e = torch.exp2(2.0 * (0.7978845608 * (out + 0.044715 * out * out * out)) * log2e)
        out = 0.5 * out * (1.0 + (e - 1.0) / (e + 1.0))
    return out.reshape(-1)


def compare_mma(ncz, batches: int, k_iters: int, epilogue: int) -> dict:
    """compareMma (src/main.zig:953-975) for batches = k_iters = 1 (mma_matmul,
    16x8x16, alpha 1, beta 0); otherwise pipelined_mma_matmul over `batches`
    batches (the reference runs one): 5 warm-up + 20 timed launches,
    algorithmic bytes = A, B f16 read + C f32 read + D f32 written."""
    import torch

    bench = importlib.import_module("not-cute-zig_b200.benchmark")
    single = batches == 1 and k_iters == 1
    g = torch.Generator(device="cuda")
    g.manual_seed(batches * 31 + k_iters)
    a = (torch.rand(batches * k_iters * 256, generator=g, device="cuda") * 2 - 1).half()
    b = (torch.rand(batches * k_iters * 128, generator=g, device="cuda") * 2 - 1).half()
    c = torch.rand(batches * 128, generator=g, device="cuda") * 2 - 1
    d = torch.empty_like(c)
    alpha, beta = (1.0, 0.0) if single else (1.0, 0.5)
    stream = torch.cuda.current_stream()
    if single:
        launch = lambda: ncz.mma.mma_matmul(a, b, c, d, alpha, beta, stream=stream)  # noqa: E731
    else:
        launch = lambda: ncz.mma.pipelined_mma_matmul(a, b, c, d, alpha, beta, k_iters * 256, k_iters * 128,  # noqa: E731
                                                      128, k_iters, epilogue, batches, stream=stream)
    bytes_ = ncz.mma.bytes_moved(k_iters, batches)
    flops = ncz.mma.flops(k_iters, batches)
    res = bench.run_kernel(launch, warmup_iters=5, iters=20, bytes_processed=bytes_, flops_processed=flops,
                           stream=stream)
    ncz.mma.sync_status()
    want = torch_gemm(a, b, c, batches, k_iters, alpha, beta, 0 if single else epilogue, single)
    nan_match = bool(torch.equal(torch.isnan(d), torch.isnan(want)))
    ok = ~torch.isnan(want)
    err = float((d[ok] - want[ok]).abs().max()) if nan_match else float("nan")
    peak = measured_hbm()
    shape = "16x8x16" if single else f"batches={batches},k_iters={k_iters},16x8,epilogue={int(epilogue)}"
    return res.record("mma_gemm", "not_cute_zig_b200", shape, nan_match and err <= 1e-3, bytes_, flops, err,
                      pct_hbm_measured=(res.throughput_gbps / peak) if peak else None, host_cores=bench.host_cores(),
                      label="mma_gemm_sm100a")


MMA_SHAPES = [(1, 1, 0), (1 << 21, 1, 1), (1 << 20, 4, 2), (1 << 18, 16, 3)]
OURS = "not_cute_zig_b200"


def read_records(paths: List[str]) -> List[dict]:
    """JSON records, one per line, of every file (other lines are skipped)."""
    out = []
    for path in paths:
        with open(path) as f:
            for line in f:
                line = line.strip()
                if line.startswith("{"):
                    try:
                        out.append(json.loads(line))
                    except json.JSONDecodeError:
                        continue
    return out


def join_table(records: List[dict]) -> List[str]:
    """Markdown rows: per (kernel, shape) with a record of this library, one row
    per other implementation: both mean times, their ratio (other / ours) and
    whether both records are correct (the reference's join, modal_run.py:34-69)."""
    by_case: dict = {}
    for r in records:
        if r.get("gpus", 1) not in (1, None):
            continue
        by_case.setdefault((r.get("kernel"), r.get("shape")), {})[r.get("implementation")] = r
    rows = ["| kernel | shape | baseline | ours ms | baseline ms | baseline / ours | both correct |",
            "|---|---|---|---|---|---|---|"]
    for (kernel, shape), impls in sorted(by_case.items(), key=lambda kv: (str(kv[0][0]), str(kv[0][1]))):
        ours = impls.get(OURS)
        if ours is None:
            continue
        for name in sorted(impls):
            if name == OURS:
                continue
            other = impls[name]
            ratio = other["mean_ms"] / ours["mean_ms"] if ours["mean_ms"] else 0.0
            ok = "yes" if ours.get("correct") and other.get("correct") else "no"
            rows.append(f"| {kernel} | {shape} | {name} | {ours['mean_ms']:.4f} | {other['mean_ms']:.4f} | "
                        f"{ratio:.2f}x | {ok} |")
    return rows


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--shape", action="append", default=[],
                    help="bh,seq,head,causal (repeatable); default: the 15 reference compare shapes")
    ap.add_argument("--gpus", type=int, default=1, help="shard slices across this many devices")
    ap.add_argument("--seed", type=int, default=None,
                    help="N(0,1) inputs from this seed instead of the reference's fillFlashInput pattern")
    ap.add_argument("--in-dtype", choices=sorted(IN_DTYPES), default="f16", help="Q/K/V element type")
    ap.add_argument("--o-dtype", choices=sorted(O_DTYPES), default="f32", help="O element type")
    ap.add_argument("--row-stride", type=int, default=0,
                    help="elements between rows of Q/K/V/O (>= head_dim; 0 = head_dim)")
    ap.add_argument("--cpu-ms", action="store_true",
                    help="also time the fp32 cross-check attention on the host CPU (cpu_ms)")
    ap.add_argument("--jsonl", default=None, help="append records to this file instead of stdout")
    ap.add_argument("--mma", action="store_true",
                    help="the GEMM + epilogue records instead: compareMma's 16x8x16 and batched throughput shapes")
    ap.add_argument("--mma-shape", action="append", default=[],
                    help="batches,k_iters,epilogue (repeatable; implies --mma)")
    ap.add_argument("--join", nargs="+", default=None, metavar="JSONL",
                    help="print the joined table of these record files (no GPU work)")
    args = ap.parse_args(argv)
    if args.join:
        print("\n".join(join_table(read_records(args.join))))
        return 0
    ncz = importlib.import_module("not-cute-zig_b200")
    bench = importlib.import_module("not-cute-zig_b200.benchmark")
    if args.mma or args.mma_shape:
        shapes = [tuple(int(x) for x in spec.split(",")) for spec in args.mma_shape] or MMA_SHAPES
        records = [compare_mma(ncz, nb, k, e) for nb, k, e in shapes]
        bench.emit(records, args.jsonl)
        return 0 if all(r["correct"] for r in records) else 1
    shapes = REFERENCE_SHAPES
    if args.shape:
        shapes = []
        for spec in args.shape:
            bh, s, d, c = (int(x) for x in spec.split(","))
            shapes.append((bh, s, d, bool(c)))
    records = [compare_shape(ncz, bh, s, d, c, args.gpus, seed=args.seed, in_dtype=args.in_dtype,
                             o_dtype=args.o_dtype, row_stride=args.row_stride, cpu_ms=args.cpu_ms)
               for bh, s, d, c in shapes]
    bench.emit(records, args.jsonl)
    return 0 if all(r["correct"] for r in records) else 1


if __name__ == "__main__":
    sys.exit(main())
