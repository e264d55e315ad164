"""Build recipe for libncz_flash.so (sm_100a only), in-tree: the flash-attention
forward (csrc/flash_api.cu), the batched GEMM with epilogue (csrc/mma_api.cu)
and the driver-call table both of them call CUDA through (csrc/driver.cu).

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
NVCC = os.environ.get("NVCC", "nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
         "-shared", "-I", os.path.join(ROOT, "include")]


def sources():
    return [os.path.join(HERE, "csrc", f) for f in ("flash_api.cu", "mma_api.cu", "driver.cu")]


def deps():
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*")) + glob.glob(os.path.join(ROOT, "include", "*.h")))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and os.path.exists(LIB):
        t = os.path.getmtime(LIB)
        if all(os.path.getmtime(p) <= t for p in deps()):
            return LIB
    cmd = [NVCC] + FLAGS + (["-Xptxas", "-v"] if verbose else []) + sources() + ["-o", LIB]
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(force=True, verbose=True))
