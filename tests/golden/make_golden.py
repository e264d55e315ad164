"""Generates tests/golden/reference_tiled.npz on a GPU box -- the oracle's pin.

Runs the reference's OWN attention kernel flash_tiled_kernel
(tools/cuda_baselines.cu:200-307, compiled unmodified into
oracle/_ref/libncz_ref.so by oracle/build.py) on the reference's own test
inputs: fillFlashInput data (src/main.zig:219-221) for the four smoke cases
with odd slice strides (src/main.zig:190-193) and the fifteen compare shapes
(src/main.zig:141-170).  That kernel computes in f32 (scores, online softmax
with expf, f32 PV), so it agrees with the reference CPU attention to f32
round-off; the CPU test tests/test_oracle.py checks the oracle against it.

Stored per case: the full active output for cases up to 65536 output
elements, otherwise 4096 active elements at fixed seeded positions plus the
float64 sum and sum of squares over all active elements.

Usage (GPU box): python tests/golden/make_golden.py
"""
from __future__ import annotations

import ctypes
import math
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from oracle import build as obuild  # noqa: E402
from tests import cases as C  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_tiled.npz")
FULL_LIMIT = 65536
SAMPLE = 4096


def main():
    import torch

    lib = ctypes.CDLL(obuild.REF_SO)
    fn = lib.ncz_ref_flash_tiled
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 7 + [ctypes.c_float, ctypes.c_int]
    dev = torch.device("cuda:0")
    store = {}
    cases = [("smoke", c[0], c[1], c[2], c[3], c[4]) for c in C.SMOKE_CASES]
    cases += [("compare", c[0], c[1], c[2], (c[1] * c[2],) * 4, c[3]) for c in C.COMPARE_CASES]
    for i, (kind, bh, s, d, strides, causal) in enumerate(cases):
        p = C.pattern_problem(bh, s, d, strides, causal, oracle)
        q, k, v = (torch.from_numpy(a).to(dev) for a in (p.q, p.k, p.v))
        o = torch.zeros(bh * strides[3], dtype=torch.float32, device=dev)
        err = fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), bh, s, d, *strides,
                 ctypes.c_float(1.0 / math.sqrt(d)), int(causal))
        assert err == 0, f"reference kernel failed: cuda error {err}"
        got = o.cpu().numpy()
        idx = C.active_index(p)
        vals = got[idx]
        key = f"c{i:02d}"
        store[f"{key}_meta"] = np.array([bh, s, d, *strides, int(causal), int(kind == "smoke")], dtype=np.int64)
        if idx.size <= FULL_LIMIT:
            store[f"{key}_idx"] = idx.astype(np.int64)
            store[f"{key}_val"] = vals
        else:
            rng = np.random.default_rng(1000 + i)
            pick = np.sort(rng.choice(idx.size, SAMPLE, replace=False))
            store[f"{key}_idx"] = idx[pick].astype(np.int64)
            store[f"{key}_val"] = vals[pick]
        store[f"{key}_sum"] = np.array([vals.astype(np.float64).sum(), (vals.astype(np.float64) ** 2).sum()])
        print(f"{key} {kind} bh={bh} S={s} d={d} causal={causal} stored={store[f'{key}_idx'].size}")
    np.savez_compressed(OUT, **store)
    print("wrote", OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main()
