"""Fixtures of the GEMM + epilogue path, shared by the CPU and GPU tests.

The reference's own fixtures for its mma demo kernels, restated:
  fill_pipeline_inputs  fillPipelineInputs  src/main.zig:1163-1182 (epilogue and
                        pipelined demos: runEpilogueDemo :289, runPipelinedMma :343)
  fill_mma_inputs       fillMmaInputs       src/main.zig:1119-1144 (runBatchedMma
                        :396, runMmaMatmul :1049 with alpha 1.25, beta 0.5)
  gemm_baseline_inputs  run_gemm            tools/cuda_baselines.cu:580-589
All their values are small multiples of powers of two, so every product and
partial sum is exact in f32: exact_gemm (float64) gives the answer the oracle
and the kernel must reproduce bit for bit (the reference's demos accept
|diff| <= 0.001, src/main.zig:333).
"""
from __future__ import annotations

import numpy as np

TILE_A, TILE_B, TILE_C = 256, 128, 128


def fill_pipeline_inputs(k_iters: int):
    a = np.empty(k_iters * TILE_A, np.float16)
    b = np.empty(k_iters * TILE_B, np.float16)
    for tile in range(k_iters):
        i = np.arange(TILE_A)
        a[tile * TILE_A:(tile + 1) * TILE_A] = (((i + tile) % 5) * 0.125).astype(np.float16)
        i = np.arange(TILE_B)
        b[tile * TILE_B:(tile + 1) * TILE_B] = (((i * 3 + tile) % 7) * 0.0625).astype(np.float16)
    c = ((np.arange(TILE_C) % 13) * 0.03125).astype(np.float32)
    return a, b, c


def fill_mma_inputs(seed: int):
    """A row-major 16x16, B column-major 16x8 (element (k, n) at n*16 + k), C row-major."""
    row, col = np.meshgrid(np.arange(16), np.arange(16), indexing="ij")
    a = (((row + col + seed) % 5) * 0.25).astype(np.float16).reshape(-1)
    k, n = np.meshgrid(np.arange(16), np.arange(8), indexing="ij")  # B[k][n]
    b = np.empty(TILE_B, np.float16)
    b[n.reshape(-1) * 16 + k.reshape(-1)] = (((k * 2 + n + seed) % 7) * 0.125).astype(np.float16).reshape(-1)
    r, cc = np.meshgrid(np.arange(16), np.arange(8), indexing="ij")
    c = (((r + cc * 3 + seed) % 11) * 0.03125).astype(np.float32).reshape(-1)
    return a, b, c


def gemm_baseline_inputs():
    a = ((np.arange(TILE_A) % 5) * 0.25).astype(np.float16)
    b = ((np.arange(TILE_B) % 7) * 0.125).astype(np.float16)  # row-major K x N (B[kk * n + c])
    return a, b, np.zeros(TILE_C, np.float32)


def exact_gemm(a, b, c, *, alpha, beta, k_iters, batches=1, sa=None, sb=None, sc=None, b_col=False, relu=False):
    """float64 D = alpha * (A B) + beta * C per batch (relu optional); exact for
    the dyadic fixtures above."""
    sa = k_iters * TILE_A if sa is None else sa
    sb = k_iters * TILE_B if sb is None else sb
    sc = TILE_C if sc is None else sc
    d = np.asarray(c, np.float64).copy()
    for bt in range(batches):
        acc = np.zeros((16, 8))
        for t in range(k_iters):
            at = np.asarray(a[bt * sa + t * TILE_A: bt * sa + (t + 1) * TILE_A], np.float64).reshape(16, 16)
            bt_ = np.asarray(b[bt * sb + t * TILE_B: bt * sb + (t + 1) * TILE_B], np.float64)
            bm = bt_.reshape(8, 16).T if b_col else bt_.reshape(16, 8)
            acc += at @ bm
        cm = np.asarray(c[bt * sc: bt * sc + TILE_C], np.float64).reshape(16, 8)
        out = alpha * acc + beta * cm
        if relu:
            out = np.maximum(out, 0.0)
        d[bt * sc: bt * sc + TILE_C] = out.reshape(-1)
    return d


def silu64(x):
    x = np.asarray(x, np.float64)
    e = np.exp2(x * np.log2(np.e))
    return x * (e / (1.0 + e))


def gelu64(x):
    x = np.asarray(x, np.float64)
    inner = 0.7978845608 * (x + 0.044715 * x * x * x)
    e = np.exp2(2.0 * inner * np.log2(np.e))
    return 0.5 * x * (1.0 + (e - 1.0) / (e + 1.0))
