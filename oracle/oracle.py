"""numpy front end of the C oracle (flash_oracle.c) -- TEST INFRASTRUCTURE ONLY.

Restates the reference CPU attention computeFlashReferenceOne
(src/main.zig:1271-1307) and its input generator fillFlashInput
(src/main.zig:1207-1211); see flash_oracle.c for the line-by-line mapping.
f16 arrays are numpy float16; outputs are float32.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import build as _build

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        srcs = [p for p in _build.oracle_sources() if os.path.exists(p)]
        if not os.path.exists(_build.ORACLE_SO) or any(
                os.path.getmtime(p) > os.path.getmtime(_build.ORACLE_SO) for p in srcs):
            _build.build_oracle()
        h = ctypes.CDLL(_build.ORACLE_SO)
        sz, vp = ctypes.c_size_t, ctypes.c_void_p
        h.ncz_oracle_flash.restype = None
        h.ncz_oracle_flash.argtypes = [sz, sz, sz, vp, sz, sz, vp, sz, sz, vp, sz, sz, vp, sz, sz,
                                       ctypes.c_float, ctypes.c_uint32, sz, sz, ctypes.c_int]
        h.ncz_oracle_flash_bf16.restype = None
        h.ncz_oracle_flash_bf16.argtypes = h.ncz_oracle_flash.argtypes
        h.ncz_oracle_flash_mag.restype = None
        h.ncz_oracle_flash_mag.argtypes = [sz, sz, sz, vp, sz, sz, vp, sz, sz, vp, sz, sz, vp, vp, sz, sz,
                                           ctypes.c_float, ctypes.c_uint32, sz, sz, ctypes.c_int, ctypes.c_int]
        h.ncz_oracle_fill_normal_bf16.restype = None
        h.ncz_oracle_fill_normal_bf16.argtypes = [vp, sz, ctypes.c_uint64, ctypes.c_float, ctypes.c_float]
        h.ncz_oracle_fill_pattern.restype = None
        h.ncz_oracle_fill_pattern.argtypes = [vp, sz, sz, sz, sz, ctypes.c_float]
        h.ncz_oracle_fill_normal.restype = None
        h.ncz_oracle_fill_normal.argtypes = [vp, sz, ctypes.c_uint64, ctypes.c_float, ctypes.c_float]
        h.ncz_oracle_fill_uniform.restype = None
        h.ncz_oracle_fill_uniform.argtypes = [vp, sz, ctypes.c_uint64, ctypes.c_float, ctypes.c_float]
        h.ncz_oracle_fill_normal_range.restype = None
        h.ncz_oracle_fill_normal_range.argtypes = [vp, sz, ctypes.c_uint64, sz, ctypes.c_float, ctypes.c_float]
        h.ncz_oracle_fill_uniform_range.restype = None
        h.ncz_oracle_fill_uniform_range.argtypes = [vp, sz, ctypes.c_uint64, sz, ctypes.c_float, ctypes.c_float]
        h.ncz_oracle_fill_row_padding.restype = None
        h.ncz_oracle_fill_row_padding.argtypes = [vp, sz, sz, sz, sz, sz, ctypes.c_uint16]
        h.ncz_oracle_max_threads.restype = ctypes.c_int
        h.ncz_oracle_max_threads.argtypes = []
        h.ncz_oracle_mma.restype = None
        h.ncz_oracle_mma.argtypes = [vp, vp, vp, vp, ctypes.c_float, ctypes.c_float, sz, sz, sz, sz, ctypes.c_uint32,
                                     sz, ctypes.c_int]
        _lib = h
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def fill_pattern(n: int, mul: int, add: int, scale: float, modulus: int = 17) -> np.ndarray:
    """fillFlashInput (src/main.zig:1207-1211): f16(((i*mul+add) % modulus) * scale)."""
    out = np.empty(n, dtype=np.float16)
    lib().ncz_oracle_fill_pattern(_ptr(out), n, mul, add, modulus, scale)
    return out


def fill_normal(n: int, seed: int, mean: float = 0.0, std: float = 1.0, first: int = 0) -> np.ndarray:
    """f16(mean + std * N(0,1)) from splitmix64(seed) + Box-Muller: elements
    first .. first+n-1 of the stream (the same bits as a longer fill's slice)."""
    out = np.empty(n, dtype=np.float16)
    lib().ncz_oracle_fill_normal_range(_ptr(out), n, seed, first, mean, std)
    return out


def fill_uniform(n: int, seed: int, lo: float = -1.0, hi: float = 1.0, first: int = 0) -> np.ndarray:
    """f16(U(lo, hi)) from splitmix64(seed): elements first .. first+n-1 of the stream."""
    out = np.empty(n, dtype=np.float16)
    lib().ncz_oracle_fill_uniform_range(_ptr(out), n, seed, first, lo, hi)
    return out


def fill_row_padding(a: np.ndarray, batch_heads: int, seq_len: int, head_dim: int, slice_stride: int,
                     row_stride: int, value=np.float16(np.nan)) -> None:
    """Writes `value` into every padding element (column >= head_dim) of a strided view."""
    bits = np.array([value], dtype=np.float16).view(np.uint16)[0]
    lib().ncz_oracle_fill_row_padding(_ptr(a), batch_heads, seq_len, head_dim, slice_stride, row_stride,
                                      int(bits))


def flash_reference(q: np.ndarray, k: np.ndarray, v: np.ndarray, *, batch_heads: int, seq_len: int,
                    head_dim: int, q_stride: int, k_stride: int, v_stride: int, o_stride: int,
                    scale: float, causal: bool, row_strides=None, out: np.ndarray | None = None,
                    rows: tuple[int, int] | None = None, threads: int = 0,
                    mag: np.ndarray | None = None) -> np.ndarray:
    """The reference CPU attention over all slices (computeFlashReferenceSlices,
    src/main.zig:1242-1269), with optional per-row strides (default head_dim).

    Returns a float32 array of batch_heads * o_stride elements (unwritten
    elements are 0, as the reference's `expected` buffer is zero-filled).
    `mag` (float32, laid out like out) receives sum_k w_k |v_k| per output
    element: the scale of the error that rounding the weights P (relative
    error <= u each) can cause, at most u * mag."""
    qr, kr, vr, orow = row_strides if row_strides is not None else (head_dim,) * 4
    bf16 = q.dtype == np.uint16  # bf16 bit patterns (numpy has no bf16 type)
    for a in (q, k, v):
        assert a.dtype == (np.uint16 if bf16 else np.float16) and a.flags.c_contiguous
    if out is None:
        out = np.zeros(batch_heads * o_stride, dtype=np.float32)
    r0, r1 = rows if rows is not None else (0, seq_len)
    if mag is not None:
        assert mag.dtype == np.float32 and mag.size >= out.size
        lib().ncz_oracle_flash_mag(batch_heads, seq_len, head_dim, _ptr(q), q_stride, qr, _ptr(k), k_stride, kr,
                                   _ptr(v), v_stride, vr, _ptr(out), _ptr(mag), o_stride, orow, float(scale),
                                   int(bool(causal)), r0, r1, threads, int(bf16))
        return out
    fn = lib().ncz_oracle_flash_bf16 if bf16 else lib().ncz_oracle_flash
    fn(batch_heads, seq_len, head_dim, _ptr(q), q_stride, qr, _ptr(k), k_stride, kr,
       _ptr(v), v_stride, vr, _ptr(out), o_stride, orow, float(scale), int(bool(causal)), r0, r1, threads)
    return out


def fill_normal_bf16(n: int, seed: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    """bf16(mean + std * N(0,1)) bit patterns (uint16) from splitmix64(seed) + Box-Muller,
    the same stream as fill_normal."""
    out = np.empty(n, dtype=np.uint16)
    lib().ncz_oracle_fill_normal_bf16(_ptr(out), n, seed, mean, std)
    return out


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def max_threads() -> int:
    return int(lib().ncz_oracle_max_threads())


def mma_reference(a: np.ndarray, b: np.ndarray, c: np.ndarray, *, alpha: float, beta: float, batch_stride_a: int,
                  batch_stride_b: int, batch_stride_c: int, k_iters: int, epilogue: int, batches: int,
                  b_col: bool = False) -> np.ndarray:
    """GEMM + epilogue oracle (mma_oracle.c: computePipelineReference,
    src/main.zig:1184-1204, and computeMmaReference, :1146-1162, generalised
    to batches, strides and the silu / gelu activations of src/device.zig).
    Returns D as float32 with C's shape (entries outside the batches' tiles are
    copied from C)."""
    a = np.ascontiguousarray(a, dtype=np.float16)
    b = np.ascontiguousarray(b, dtype=np.float16)
    c = np.ascontiguousarray(c, dtype=np.float32)
    d = c.copy()
    lib().ncz_oracle_mma(_ptr(a), _ptr(b), _ptr(c), _ptr(d), alpha, beta, batch_stride_a, batch_stride_b,
                         batch_stride_c, k_iters, epilogue, batches, 1 if b_col else 0)
    return d
