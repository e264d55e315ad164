"""Batched 16x8 GEMM with fused epilogue on sm_100a, behind the argument tuples
of the reference's mma demo kernels (src/kernels.zig):

    pipelined_mma_matmul(a, b, c, d, alpha, beta, batch_stride_a, batch_stride_b,
                         batch_stride_c, k_iters, epilogue_kind)    :33-141
    batched_mma_matmul(a, b, c, d, alpha, beta, batch_stride_a, batch_stride_b,
                       batch_stride_c)                               :301-319
    mma_matmul(a, b, c, d, alpha, beta)                              :290-299

The reference takes the batch count from grid.y; here it is `batches`.  Per
batch, D = epilogue(alpha * (A B) + beta * C) on one 16x8 f32 tile; A and B
are f16.  Tensors are torch CUDA tensors (a, b float16; c, d float32) or raw
device addresses (int); sizes are checked for tensors (the reference, taking
raw pointers, checks nothing).  Errors raise FlashError with the library's
status code.
"""
from __future__ import annotations

import ctypes
from enum import IntEnum
from typing import Optional

from . import flash

_VP, _SZ = ctypes.c_void_p, ctypes.c_size_t
_SIGNATURES = {
    "ncz_mma_matmul_pipelined": (
        ctypes.c_int,
        [_VP, _VP, _VP, _VP, ctypes.c_float, ctypes.c_float, _SZ, _SZ, _SZ, _SZ, ctypes.c_uint32, _SZ, _VP],
    ),
    "ncz_mma_matmul_batched": (
        ctypes.c_int,
        [_VP, _VP, _VP, _VP, ctypes.c_float, ctypes.c_float, _SZ, _SZ, _SZ, _SZ, _VP],
    ),
    "ncz_mma_matmul": (ctypes.c_int, [_VP, _VP, _VP, _VP, ctypes.c_float, ctypes.c_float, _VP]),
    "ncz_mma_sync_status": (ctypes.c_int, [ctypes.c_int]),
    "ncz_mma_test_set_wait_limit": (ctypes.c_int, [ctypes.c_int, ctypes.c_uint64]),
    "ncz_mma_test_drop_copy": (ctypes.c_int, [ctypes.c_int, ctypes.c_int]),
}
_bound = False

TILE_A = 16 * 16  # elements of one A tile
TILE_B = 16 * 8   # elements of one B tile
TILE_C = 16 * 8   # elements of one C / D tile


class Epilogue(IntEnum):
    """kernels.Epilogue (src/kernels.zig:26-31)."""

    NONE = 0
    RELU = 1
    SILU = 2
    GELU = 3


def lib() -> ctypes.CDLL:
    global _bound
    handle = flash.lib()
    if not _bound:
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _bound = True
    return handle


def _addr(t, dtype_name: str, need: int, what: str) -> int:
    if isinstance(t, int):
        return t
    import torch

    if not t.is_cuda or t.dtype != getattr(torch, dtype_name):
        raise flash.FlashError(5, f"{what}: expected a CUDA {dtype_name} tensor")
    if not t.is_contiguous() or t.numel() < need:
        raise flash.FlashError(5, f"{what}: needs a contiguous tensor of at least {need} elements")
    return t.data_ptr()


def _extent(batches: int, stride: int, per_batch: int) -> int:
    return 0 if batches == 0 else (batches - 1) * stride + per_batch


def pipelined_mma_matmul(a, b, c, d, alpha: float, beta: float, batch_stride_a: int, batch_stride_b: int,
                         batch_stride_c: int, k_iters: int, epilogue: int = Epilogue.NONE, batches: int = 1,
                         stream=None) -> None:
    """src/kernels.zig:33-141: A_b k_iters row-major 16x16 tiles, B_b k_iters
    row-major 16x8 (K x N) tiles, C_b / D_b row-major 16x8 (stride batch_stride_c)."""
    pa = _addr(a, "float16", _extent(batches, batch_stride_a, k_iters * TILE_A), "a")
    pb = _addr(b, "float16", _extent(batches, batch_stride_b, k_iters * TILE_B), "b")
    pc = _addr(c, "float32", _extent(batches, batch_stride_c, TILE_C), "c")
    pd = _addr(d, "float32", _extent(batches, batch_stride_c, TILE_C), "d")
    flash._check(
        lib().ncz_mma_matmul_pipelined(pa, pb, pc, pd, alpha, beta, batch_stride_a, batch_stride_b, batch_stride_c,
                                       k_iters, int(epilogue), batches, flash._stream_handle(stream)),
        "pipelined_mma_matmul",
    )


def batched_mma_matmul(a, b, c, d, alpha: float, beta: float, batch_stride_a: int, batch_stride_b: int,
                       batch_stride_c: int, batches: int = 1, stream=None) -> None:
    """src/kernels.zig:301-319: one row-major 16x16 A tile and one column-major
    16x8 B tile (element (k, n) at n * 16 + k) per batch."""
    pa = _addr(a, "float16", _extent(batches, batch_stride_a, TILE_A), "a")
    pb = _addr(b, "float16", _extent(batches, batch_stride_b, TILE_B), "b")
    pc = _addr(c, "float32", _extent(batches, batch_stride_c, TILE_C), "c")
    pd = _addr(d, "float32", _extent(batches, batch_stride_c, TILE_C), "d")
    flash._check(
        lib().ncz_mma_matmul_batched(pa, pb, pc, pd, alpha, beta, batch_stride_a, batch_stride_b, batch_stride_c,
                                     batches, flash._stream_handle(stream)),
        "batched_mma_matmul",
    )


def mma_matmul(a, b, c, d, alpha: float, beta: float, stream=None) -> None:
    """src/kernels.zig:290-299: one 16x8x16 tile, B column-major."""
    pa = _addr(a, "float16", TILE_A, "a")
    pb = _addr(b, "float16", TILE_B, "b")
    pc = _addr(c, "float32", TILE_C, "c")
    pd = _addr(d, "float32", TILE_C, "d")
    flash._check(lib().ncz_mma_matmul(pa, pb, pc, pd, alpha, beta, flash._stream_handle(stream)), "mma_matmul")


def sync_status(device: Optional[int] = None) -> int:
    """Synchronises `device` and raises FlashError(DeviceTimeout) when a GEMM
    kernel's bounded wait for a staged tile ran out."""
    st = lib().ncz_mma_sync_status(-1 if device is None else device)
    flash._check(st, "mma sync_status")
    return st


def flops(k_iters: int, batches: int) -> int:
    """2 * 16 * 8 * 16 * k_iters per batch (the reference counts 2*m*n*k,
    tools/cuda_baselines.cu:616)."""
    return 2 * 16 * 8 * 16 * k_iters * batches


def bytes_moved(k_iters: int, batches: int) -> int:
    """A and B f16 read, C f32 read, D f32 written, per batch."""
    return batches * (k_iters * (TILE_A + TILE_B) * 2 + 2 * TILE_C * 4)
