"""The driver-call table of libncz_flash.so (include/ncz_driver.h) from Python.

Every CUDA call of the C ABI goes through one table of C function pointers;
`install` puts Python callables in its place (host tests: a fake of N
devices that fails chosen calls on chosen devices), `install(None)` restores
the CUDA runtime.  Each entry returns a CUDA runtime error number (0 =
success).  The installed callables must stay alive while the table is in use;
this module keeps them until the next `install`.
"""
from __future__ import annotations

import ctypes
from typing import Callable, Dict, Optional

from . import flash

_I, _VP, _SZ = ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t
_PI = ctypes.POINTER(ctypes.c_int)
_PVP = ctypes.POINTER(ctypes.c_void_p)

COPY_HOST_TO_DEVICE, COPY_DEVICE_TO_HOST = 1, 2

# (entry, argument types) in the order of ncz_driver_table; all return int.
ENTRIES = [
    ("get_device_count", [_PI]),
    ("get_device", [_PI]),
    ("set_device", [_I]),
    ("sm_count", [_I, _PI]),
    ("load_tensor_map_encoder", []),
    ("encode_tensor_map", [_VP, _I, _VP, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64),
                           ctypes.POINTER(ctypes.c_uint32), ctypes.c_uint32]),
    ("set_max_dynamic_smem", [_VP, _I]),
    ("launch_kernel", [_VP, ctypes.c_uint32, ctypes.c_uint32, _SZ, _VP, _PVP]),
    ("stream_create", [_PVP]),
    ("stream_destroy", [_VP]),
    ("event_create", [_PVP]),
    ("event_destroy", [_VP]),
    ("event_record", [_VP, _VP]),
    ("stream_wait_event", [_VP, _VP]),
    ("stream_synchronize", [_VP]),
    ("device_synchronize", []),
    ("memcpy_async", [_VP, _VP, _SZ, _I, _VP]),
    ("symbol_read", [_VP, _VP, _SZ]),
    ("symbol_write", [_VP, _VP, _SZ]),
    ("symbol_address", [_PVP, _VP]),
    ("pool_create", [_PVP, _I, ctypes.c_uint64]),
    ("pool_destroy", [_VP]),
    ("pool_alloc_async", [_PVP, _SZ, _VP, _VP]),
    ("free_async", [_VP, _VP]),
]
PROTOTYPES = {name: ctypes.CFUNCTYPE(_I, *args) for name, args in ENTRIES}


class DriverTable(ctypes.Structure):
    """ncz_driver_table."""

    _fields_ = [("size", _SZ)] + [(name, PROTOTYPES[name]) for name, _ in ENTRIES]


_SIGNATURES = {
    "ncz_set_driver": (ctypes.c_int, [ctypes.POINTER(DriverTable), ctypes.POINTER(ctypes.c_int)]),
    "ncz_get_driver": (ctypes.c_int, [ctypes.POINTER(DriverTable)]),
    "ncz_kernel_label": (ctypes.c_int, [_VP, ctypes.c_char_p, _SZ]),
}
_bound = False
_installed: Optional[DriverTable] = None  # keeps the callbacks of an installed table alive


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


def make_table(entries: Dict[str, Callable[..., int]]) -> DriverTable:
    """A table of the given callables (every entry of ENTRIES is required)."""
    missing = [name for name, _ in ENTRIES if name not in entries]
    if missing:
        raise ValueError(f"driver table lacks {missing}")
    t = DriverTable()
    t.size = ctypes.sizeof(DriverTable)
    for name, _ in ENTRIES:
        setattr(t, name, PROTOTYPES[name](entries[name]))
    return t


def install(entries: Optional[Dict[str, Callable[..., int]]]) -> int:
    """ncz_set_driver: installs a table of `entries` (None = the CUDA runtime)
    and returns the first error of releasing the library's objects through
    the previous table (0 = none); the table is installed either way."""
    global _installed
    table = None if entries is None else make_table(entries)
    released = ctypes.c_int(0)
    st = lib().ncz_set_driver(None if table is None else ctypes.byref(table), ctypes.byref(released))
    flash._check(st, "driver.install")
    _installed = table
    return released.value


def current() -> DriverTable:
    """ncz_get_driver: a copy of the table in use."""
    t = DriverTable()
    t.size = ctypes.sizeof(DriverTable)
    flash._check(lib().ncz_get_driver(ctypes.byref(t)), "driver.current")
    return t


def kernel_label(kernel: int) -> Optional[str]:
    """ncz_kernel_label: the library's name for the kernel at host address
    `kernel` (as launch_kernel receives it), or None."""
    buf = ctypes.create_string_buffer(64)
    if lib().ncz_kernel_label(kernel, buf, len(buf)) != 0:
        return None
    return buf.value.decode()
