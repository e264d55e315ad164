"""Build recipe for libncz_flash.so (sm_100a only), in-tree: the flash-attention
forward (csrc/flash_api.cu), the batched GEMM with epilogue (csrc/mma_api.cu)
and the driver-call table both of them call CUDA through (csrc/driver.cu).

libncz_flash_debug.so is the same sources with NCZ_DEBUG_ITEM_VISITS: the
forward also counts, per work item, the CTAs that started it (a check of the
launch-control item walk; not for production use).

nvcc -gencode arch=compute_100a,code=sm_100a -O3 -lineinfo -shared -fPIC,
static cudart (the library resolves cuTensorMapEncodeTiled at run time, so
it has no link-time dependency on libcuda and loads on machines without a
GPU driver).
"""
from __future__ import annotations

import glob
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libncz_flash.so")
DEBUG_LIB = os.path.join(HERE, "libncz_flash_debug.so")
NVCC = os.environ.get("NVCC", "nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
         "-shared", "-I", os.path.join(ROOT, "include")]


def sources():
    return [os.path.join(HERE, "csrc", f) for f in ("flash_api.cu", "mma_api.cu", "driver.cu")]


def deps():
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*")) + glob.glob(os.path.join(ROOT, "include", "*.h")))


def _build(out: str, extra, force: bool, verbose: bool) -> str:
    if not force and os.path.exists(out):
        t = os.path.getmtime(out)
        if all(os.path.getmtime(p) <= t for p in deps()):
            return out
    cmd = [NVCC] + FLAGS + list(extra) + (["-Xptxas", "-v"] if verbose else []) + sources() + ["-o", out]
    subprocess.run(cmd, check=True)
    return out


def build(force: bool = False, verbose: bool = False) -> str:
    """The product library."""
    return _build(LIB, [], force, verbose)


def build_debug(force: bool = False, verbose: bool = False) -> str:
    """The item-visit debug library (tests only)."""
    return _build(DEBUG_LIB, ["-DNCZ_DEBUG_ITEM_VISITS"], force, verbose)


if __name__ == "__main__":
    print(build(force=True, verbose=True))
