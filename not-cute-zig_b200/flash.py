"""Host-side mirror of not-cute-zig's `flash` module (src/flash.zig) over the
B200 C ABI in libncz_flash.so (include/ncz_flash.h).

Same names, argument meaning and error behaviour as the reference:

  Options / Options.validate   src/flash.zig:5-28
  launch (+ requireLen)        src/flash.zig:31-70, 98-100
  KernelSelection/select_kernel src/flash.zig:72-96
  FlashError codes             src/cuda.zig:134-151 (CudaError), plus
                               DeviceTimeout and Misaligned

Buffers are torch CUDA tensors (Q/K/V float16, O float32 -- or float16
through launch_ex); pointers and element counts are taken from them, so the
reference's slice-length checks (requireLen) apply to tensor.numel().

There is no CPU path: if the shared library is missing every call raises.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import Optional, Sequence

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libncz_flash.so")

STATUS_NAMES = {
    0: "Success",
    1: "OutOfMemory",
    2: "Overflow",
    3: "SharedObjectInitFailed",
    4: "NotFound",
    5: "InvalidValue",
    6: "InvalidContext",
    7: "InvalidDevice",
    8: "InvalidImage",
    9: "ContextIsDestroyed",
    10: "LaunchFailed",
    11: "LaunchOutOfResources",
    12: "LaunchTimeout",
    13: "IllegalAddress",
    14: "NoDevice",
    15: "NotInitialized",
    16: "UnknownError",
    17: "DeviceTimeout",
    18: "Misaligned",
}

DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2
STATIC_SCRATCH_BYTES = 16 << 20  # NCZ_STATIC_SCRATCH_BYTES: ncz_flash_fwd_static's fixed scratch per device
PRODUCERS = {"auto": 0, "tma": 1, "lsu": 2}


class FlashError(RuntimeError):
    """A non-zero status from the C ABI; `.name` is the reference's CudaError name."""

    def __init__(self, status: int, what: str = ""):
        self.status = int(status)
        self.name = STATUS_NAMES.get(self.status, f"Status{self.status}")
        super().__init__(f"{what}: {self.name} ({self.status})" if what else f"{self.name} ({self.status})")


class _Desc(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("o", ctypes.c_void_p),
        ("batch_heads", ctypes.c_size_t),
        ("seq_len", ctypes.c_size_t),
        ("head_dim", ctypes.c_size_t),
        ("q_stride", ctypes.c_size_t),
        ("k_stride", ctypes.c_size_t),
        ("v_stride", ctypes.c_size_t),
        ("o_stride", ctypes.c_size_t),
        ("q_row_stride", ctypes.c_size_t),
        ("k_row_stride", ctypes.c_size_t),
        ("v_row_stride", ctypes.c_size_t),
        ("o_row_stride", ctypes.c_size_t),
        ("scale", ctypes.c_float),
        ("causal", ctypes.c_uint32),
        ("o_dtype", ctypes.c_int32),
        ("producer", ctypes.c_int32),
        ("device", ctypes.c_int32),
        ("stream", ctypes.c_void_p),
        ("in_dtype", ctypes.c_int32),
    ]


_SZ = ctypes.c_size_t
_VP = ctypes.c_void_p
_SIGNATURES = {
    "ncz_init": (ctypes.c_int, []),
    "ncz_shutdown": (ctypes.c_int, []),
    "ncz_flash_validate": (ctypes.c_int, [_SZ] * 7),
    "ncz_flash_validate_ex": (ctypes.c_int, [ctypes.POINTER(_Desc)]),
    "ncz_flash_select": (
        ctypes.c_int,
        [_SZ, _SZ, _SZ, ctypes.c_uint32, ctypes.c_char_p, _SZ, ctypes.POINTER(ctypes.c_uint32)],
    ),
    "ncz_flash_fwd": (
        ctypes.c_int,
        [_VP, _VP, _VP, _VP] + [_SZ] * 7 + [ctypes.c_float, ctypes.c_uint32, _VP],
    ),
    "ncz_flash_launch": (
        ctypes.c_int,
        [_VP, _SZ, _VP, _SZ, _VP, _SZ, _VP, _SZ] + [_SZ] * 7 + [ctypes.c_float, ctypes.c_uint32, _VP],
    ),
    "ncz_flash_fwd_ex": (ctypes.c_int, [ctypes.POINTER(_Desc)]),
    "ncz_flash_fwd_named": (
        ctypes.c_int,
        [ctypes.c_char_p, _VP, _VP, _VP, _VP] + [_SZ] * 7 + [ctypes.c_float, ctypes.c_uint32, _VP],
    ),
    "ncz_flash_kernel_info": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint32),
                                             ctypes.POINTER(ctypes.c_uint32)]),
    "ncz_flash_fwd_multi": (ctypes.c_int, [ctypes.POINTER(_Desc), ctypes.c_int]),
    "ncz_flash_fwd_host": (ctypes.c_int, [ctypes.POINTER(_Desc), _VP, _VP, _VP, _VP, _SZ]),
    "ncz_flash_fwd_splits": (ctypes.c_int, [ctypes.POINTER(_Desc), ctypes.c_int]),
    "ncz_flash_fwd_static": (ctypes.c_int, [ctypes.POINTER(_Desc), ctypes.c_int]),
    "ncz_flash_sync_status": (ctypes.c_int, [ctypes.c_int, _VP, ctypes.POINTER(ctypes.c_uint32)]),
    "ncz_test_set_wait_limit": (ctypes.c_int, [ctypes.c_int, ctypes.c_uint64]),
    "ncz_test_set_qsplit": (ctypes.c_int, [ctypes.c_int]),
    "ncz_test_set_qsplit_groups": (ctypes.c_int, [ctypes.c_int]),
    "ncz_test_set_twin": (ctypes.c_int, [ctypes.c_int]),
    "ncz_test_tile_shape": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int32)]),
    "ncz_test_twin_work": (ctypes.c_int, [_SZ, _SZ, ctypes.c_uint32, ctypes.c_int, ctypes.POINTER(ctypes.c_int32)]),
    "ncz_test_qsplit_work": (ctypes.c_int, [_SZ, _SZ, ctypes.c_uint32, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                            ctypes.POINTER(ctypes.c_int32)]),
    "ncz_test_qsplit_plan": (ctypes.c_int, [_SZ, _SZ, _SZ, ctypes.POINTER(ctypes.c_int32)]),
    "ncz_test_drop_arrive": (ctypes.c_int, [ctypes.c_int, ctypes.c_int]),
    "ncz_test_item_work": (ctypes.c_int, [_SZ, _SZ, ctypes.c_uint32, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                          ctypes.POINTER(ctypes.c_int32)]),
    "ncz_test_split_plan": (ctypes.c_int, [_SZ, _SZ, ctypes.c_int, _SZ, ctypes.POINTER(ctypes.c_int32)]),
    "ncz_test_chunk_plan": (ctypes.c_int, [_SZ, _SZ, ctypes.c_int, ctypes.POINTER(ctypes.c_size_t), _SZ,
                                           ctypes.POINTER(ctypes.c_size_t)]),
    "ncz_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "ncz_launch_count": (ctypes.c_uint64, []),
    "ncz_umma_smem_desc": (ctypes.c_uint64, [ctypes.c_uint32] * 4),
    "ncz_umma_instr_desc_f16": (ctypes.c_uint32, [ctypes.c_uint32] * 4),
    "ncz_umma_instr_desc_bf16": (ctypes.c_uint32, [ctypes.c_uint32] * 4),
    "ncz_tma_swizzle_offset": (ctypes.c_uint32, [ctypes.c_uint32] * 2),
}

_lib: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    """Loads libncz_flash.so (built in-tree by __graft_entry__.build())."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FlashError(15, f"{LIB_PATH} is not built (run __graft_entry__.build())")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def _check(status: int, what: str) -> None:
    if status != 0:
        raise FlashError(status, what)


@dataclass
class Options:
    """flash.Options (src/flash.zig:5-15); strides are elements per slice."""

    seq_len: int
    head_dim: int
    q_stride: int
    k_stride: int
    v_stride: int
    o_stride: int
    scale: float
    batch_heads: int = 1
    causal: bool = False

    def validate(self) -> None:
        """src/flash.zig:16-28; raises FlashError(InvalidValue)."""
        _check(
            lib().ncz_flash_validate(
                self.batch_heads, self.seq_len, self.head_dim,
                self.q_stride, self.k_stride, self.v_stride, self.o_stride,
            ),
            "Options.validate",
        )


@dataclass(frozen=True)
class KernelSelection:
    """flash.KernelSelection (src/flash.zig:72-76)."""

    name: str
    label: str
    threads: int


def select_kernel(opts: Options) -> KernelSelection:
    """flash.selectKernel (src/flash.zig:78-96): one sm_100a kernel family."""
    buf = ctypes.create_string_buffer(64)
    threads = ctypes.c_uint32(0)
    _check(
        lib().ncz_flash_select(opts.batch_heads, opts.seq_len, opts.head_dim, int(bool(opts.causal)),
                               buf, 64, ctypes.byref(threads)),
        "select_kernel",
    )
    label = buf.value.decode()
    return KernelSelection(name=label, label=label, threads=threads.value)


def _stream_handle(stream) -> Optional[int]:
    if stream is None:
        import torch

        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def _require(t, dtype_name: str, what: str) -> None:
    import torch

    want = getattr(torch, dtype_name)
    if not t.is_cuda:
        raise FlashError(5, f"{what} must be a CUDA tensor")
    if t.dtype != want:
        raise FlashError(5, f"{what} must be {dtype_name}, got {t.dtype}")
    if not t.is_contiguous():
        raise FlashError(5, f"{what} must be contiguous (strides are given in Options)")


def launch(q, k, v, o, opts: Options, stream=None) -> None:
    """flash.launch (src/flash.zig:31-70): validate, requireLen, launch (async).

    q/k/v: float16 CUDA tensors, o: float32 CUDA tensor, each holding at least
    batch_heads * stride elements.  The C call launches on the current device,
    so q's device is made current for it (tensors carry their device here).
    """
    import torch

    _require(q, "float16", "q")
    _require(k, "float16", "k")
    _require(v, "float16", "v")
    _require(o, "float32", "o")
    if not (k.device == v.device == o.device == q.device):
        raise FlashError(5, "q, k, v and o must be on one device")
    with torch.cuda.device(q.device):
        status = lib().ncz_flash_launch(
            q.data_ptr(), q.numel(), k.data_ptr(), k.numel(), v.data_ptr(), v.numel(),
            o.data_ptr(), o.numel(),
            opts.batch_heads, opts.seq_len, opts.head_dim,
            opts.q_stride, opts.k_stride, opts.v_stride, opts.o_stride,
            float(opts.scale), int(bool(opts.causal)), _stream_handle(stream),
        )
    _check(status, "flash.launch")


# The reference's exported flash kernels (src/main_device.zig:41-47), all
# accepted by launch_named, as are the labels select_kernel returns.
REFERENCE_KERNELS = (
    "flash_attention_fwd", "flash_attention_fwd_opt", "flash_attention_fwd_v2", "flash_attention_fwd_h64",
    "flash_attention_fwd_h64_bn32", "flash_attention_fwd_h64_causal",
)


def kernel_info(name: str):
    """(head dims the kernel name accepts, always causal) for a name
    launch_named accepts; FlashError(NotFound) for any other."""
    dims, causal = ctypes.c_uint32(0), ctypes.c_uint32(0)
    _check(lib().ncz_flash_kernel_info(name.encode(), ctypes.byref(dims), ctypes.byref(causal)), f"kernel {name!r}")
    return tuple(d for bit, d in ((1, 16), (2, 32), (4, 64)) if dims.value & bit), bool(causal.value)


def launch_named(kernel: str, q, k, v, o, opts: Options, stream=None) -> None:
    """module.getFunction(kernel) + Function.launch with the 12-argument tuple
    and grid.y = batch_heads (src/main.zig:93-94, :820-852): `kernel` is one of
    REFERENCE_KERNELS or a select_kernel label.  As the named kernel does, a
    head_dim it does not take (the h64 kernels take 64 only) or seq_len 0
    returns without writing O; flash_attention_fwd_h64_causal is causal
    whatever opts.causal says.  Unknown names raise FlashError(NotFound)."""
    import torch

    _require(q, "float16", "q")
    _require(k, "float16", "k")
    _require(v, "float16", "v")
    _require(o, "float32", "o")
    if not (k.device == v.device == o.device == q.device):
        raise FlashError(5, "q, k, v and o must be on one device")
    with torch.cuda.device(q.device):
        status = lib().ncz_flash_fwd_named(
            kernel.encode(), q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
            opts.batch_heads, opts.seq_len, opts.head_dim,
            opts.q_stride, opts.k_stride, opts.v_stride, opts.o_stride,
            float(opts.scale), int(bool(opts.causal)), _stream_handle(stream),
        )
    _check(status, f"launch_named({kernel})")


def make_desc(q, k, v, o, opts: Options, *, row_strides: Optional[Sequence[int]] = None,
              producer: str = "auto", device: Optional[int] = None, stream=None) -> _Desc:
    """Extended descriptor (ncz_flash_desc): row strides (default head_dim),
    Q/K/V float16 or bfloat16 and O float32, float16 or bfloat16 (taken from
    the tensors' dtypes), producer override, device."""
    import torch

    if q.dtype not in (torch.float16, torch.bfloat16):
        raise FlashError(5, "q must be float16 or bfloat16")
    in_name = "float16" if q.dtype == torch.float16 else "bfloat16"
    _require(q, in_name, "q")
    _require(k, in_name, "k")
    _require(v, in_name, "v")
    o_types = {torch.float32: DTYPE_F32, torch.float16: DTYPE_F16, torch.bfloat16: DTYPE_BF16}
    if o.dtype not in o_types:
        raise FlashError(5, "o must be float32, float16 or bfloat16")
    _require(o, str(o.dtype).replace("torch.", ""), "o")
    rs = list(row_strides) if row_strides is not None else [0, 0, 0, 0]
    d = _Desc()
    d.q, d.k, d.v, d.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr()
    d.batch_heads, d.seq_len, d.head_dim = opts.batch_heads, opts.seq_len, opts.head_dim
    d.q_stride, d.k_stride, d.v_stride, d.o_stride = opts.q_stride, opts.k_stride, opts.v_stride, opts.o_stride
    d.q_row_stride, d.k_row_stride, d.v_row_stride, d.o_row_stride = rs
    d.scale = float(opts.scale)
    d.causal = int(bool(opts.causal))
    d.o_dtype = o_types[o.dtype]
    d.in_dtype = DTYPE_F16 if q.dtype == torch.float16 else DTYPE_BF16
    d.producer = PRODUCERS[producer]
    d.device = q.device.index if device is None else device
    d.stream = _stream_handle(stream)
    # requireLen for the extended layout: the last element a slice touches.
    for t, stride, name in ((q, opts.q_stride, "q"), (k, opts.k_stride, "k"), (v, opts.v_stride, "v"),
                            (o, opts.o_stride, "o")):
        if t.numel() < opts.batch_heads * stride:
            raise FlashError(5, f"{name} holds {t.numel()} elements, needs {opts.batch_heads * stride}")
    return d


def launch_ex(q, k, v, o, opts: Options, *, row_strides: Optional[Sequence[int]] = None,
              producer: str = "auto", device: Optional[int] = None, stream=None) -> None:
    """ncz_flash_fwd_ex: the reference launch plus the layout extensions."""
    d = make_desc(q, k, v, o, opts, row_strides=row_strides, producer=producer, device=device, stream=stream)
    _check(lib().ncz_flash_fwd_ex(ctypes.byref(d)), "flash.launch_ex")


def launch_splits(q, k, v, o, opts: Options, splits: int, *, row_strides: Optional[Sequence[int]] = None,
                  producer: str = "auto", stream=None) -> None:
    """ncz_flash_fwd_splits: launch_ex with an explicit split-KV request
    (0 = automatic, 1 = no split, n = up to n K ranges merged by a second kernel)."""
    d = make_desc(q, k, v, o, opts, row_strides=row_strides, producer=producer, stream=stream)
    _check(lib().ncz_flash_fwd_splits(ctypes.byref(d), int(splits)), "flash.launch_splits")


def launch_static(q, k, v, o, opts: Options, splits: int = 0, *, row_strides: Optional[Sequence[int]] = None,
                  producer: str = "auto", stream=None) -> None:
    """ncz_flash_fwd_static: launch_splits for callers that cannot let the
    library allocate device memory.  The split-KV partials go to a fixed
    STATIC_SCRATCH_BYTES array of the library's device image; splits = 0 takes
    the largest count that fits, an explicit count that does not fit raises
    FlashError(OutOfMemory) before any launch.  All such calls on a device
    share the array: order them (one stream or event-ordered streams), and
    make the first one on a device before any stream capture (it looks up the
    array's address)."""
    d = make_desc(q, k, v, o, opts, row_strides=row_strides, producer=producer, stream=stream)
    _check(lib().ncz_flash_fwd_static(ctypes.byref(d), int(splits)), "flash.launch_static")


def launch_host(q_host, k_host, v_host, o_host, q, k, v, o, opts: Options, *, chunk_slices: int = 0,
                row_strides: Optional[Sequence[int]] = None, producer: str = "auto", stream=None) -> None:
    """ncz_flash_fwd_host: forward on HOST buffers (q_host .. o_host, CPU tensors,
    pinned for overlap) staged through the device buffers q .. o of the same
    layout; uploads, forwards and downloads are pipelined in chunks of
    chunk_slices slices (0 = automatic).  O is in o_host once `stream` reaches
    the point after this call (e.g. after stream.synchronize())."""
    d = make_desc(q, k, v, o, opts, row_strides=row_strides, producer=producer, stream=stream)
    for h, t, name in ((q_host, q, "q"), (k_host, k, "k"), (v_host, v, "v"), (o_host, o, "o")):
        if h.device.type != "cpu":
            raise FlashError(5, f"{name}_host must be a host (CPU) tensor")
        if h.dtype != t.dtype or h.numel() < t.numel() or not h.is_contiguous():
            raise FlashError(5, f"{name}_host must be a contiguous {t.dtype} tensor of >= {t.numel()} elements")
    _check(lib().ncz_flash_fwd_host(ctypes.byref(d), q_host.data_ptr(), k_host.data_ptr(), v_host.data_ptr(),
                                    o_host.data_ptr(), int(chunk_slices)), "flash.launch_host")


def launch_multi(descs: Sequence[_Desc]) -> None:
    """ncz_flash_fwd_multi: one call launching per-device slice shards."""
    arr = (_Desc * len(descs))(*descs)
    _check(lib().ncz_flash_fwd_multi(arr, len(descs)), "flash.launch_multi")


def sync_status(device: Optional[int] = None, stream=None) -> int:
    """Synchronises the stream and raises FlashError(DeviceTimeout) if a
    bounded in-kernel wait expired since the last call; returns the raw word."""
    detail = ctypes.c_uint32(0)
    handle = 0 if stream is None else _stream_handle(stream)
    st = lib().ncz_flash_sync_status(-1 if device is None else device, handle, ctypes.byref(detail))
    if st != 0:
        raise FlashError(st, f"sync_status (word {detail.value:#x})")
    return detail.value


def shutdown() -> int:
    """ncz_shutdown: releases the library's pools, streams and events on every
    device and drops its caches (the next call initialises again); returns
    the first release error (0 = none).  Work in flight is not waited for."""
    return int(lib().ncz_shutdown())


def launch_count() -> int:
    """Kernel launches issued by this library in this process."""
    return int(lib().ncz_launch_count())


def flops(batch_heads: int, seq_len: int, head_dim: int, causal: bool) -> int:
    """Reference FLOP formula (src/main.zig:843-844): bh * 4 * eff * d,
    eff = S(S+1)/2 causal, S^2 otherwise."""
    eff = seq_len * (seq_len + 1) // 2 if causal else seq_len * seq_len
    return batch_heads * 4 * eff * head_dim


def bytes_moved(batch_heads: int, seq_len: int, head_dim: int, o_bytes: int = 4) -> int:
    """Reference byte formula (src/main.zig:845): Q, K, V f16 read + O written."""
    return batch_heads * seq_len * head_dim * (3 * 2 + o_bytes)
