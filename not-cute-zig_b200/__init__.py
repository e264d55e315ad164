"""not-cute-zig B200: an sm_100a flash-attention forward behind the reference's
`flash` module API (src/flash.zig), and the batched 16x8 GEMM with fused
epilogue behind its mma demo kernels (src/kernels.zig; module `mma`).  Module
`driver` swaps the table of CUDA calls the library makes (host tests fake devices
through it).  The package directory name is not a
Python identifier, so import it with importlib.import_module("not-cute-zig_b200").
"""
from . import driver  # noqa: F401
from . import flash  # noqa: F401
from . import mma  # noqa: F401
from .flash import (  # noqa: F401
    FlashError,
    KernelSelection,
    Options,
    launch,
    launch_ex,
    launch_host,
    launch_multi,
    launch_named,
    launch_splits,
    launch_static,
    select_kernel,
    sync_status,
)
