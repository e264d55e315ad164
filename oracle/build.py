"""Build recipes for the test oracle (TEST INFRASTRUCTURE ONLY).

- liboracle.so: the plain-C restatements of the reference CPU attention
  (oracle/flash_oracle.c) and of its CPU GEMM references (oracle/mma_oracle.c),
  gcc -O2 -fno-fast-math -fopenmp.
- _ref/libncz_ref.so and _ref/cuda_baselines: the reference's own
  tools/cuda_baselines.cu compiled from where it lies in the reference tree
  (only when that tree is present); they travel to GPU boxes as built files.
- _ref/pytorch_baselines.py: the reference's SDPA comparator
  (tools/pytorch_baselines.py) staged unmodified beside them, so a GPU box can
  run it (`python oracle/_ref/pytorch_baselines.py`); its JSONL joins with
  compare.py's records (`compare.py --join`).
"""
from __future__ import annotations

import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_DIR = os.path.join(HERE, "_ref")
REF_SO = os.path.join(REF_DIR, "libncz_ref.so")
REF_BIN = os.path.join(REF_DIR, "cuda_baselines")
REF_SDPA = os.path.join(REF_DIR, "pytorch_baselines.py")
# The reference checkout sits beside this repository ("reference/" next to the
# repository root) unless NCZ_REFERENCE_ROOT names another place.
REFERENCE_ROOT = os.environ.get("NCZ_REFERENCE_ROOT",
                                os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))
NVCC = os.environ.get("NVCC", "nvcc")


def _run(cmd):
    subprocess.run(cmd, check=True)


def _stale(out, srcs):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(s) > t for s in srcs)


def oracle_sources():
    return [os.path.join(HERE, "flash_oracle.c"), os.path.join(HERE, "mma_oracle.c")]


def build_oracle(force: bool = False) -> str:
    srcs = oracle_sources()
    if force or _stale(ORACLE_SO, srcs):
        _run(["gcc", "-O2", "-fno-fast-math", "-fopenmp", "-fPIC", "-shared", "-std=c11"] + srcs + ["-o", ORACLE_SO,
              "-lm"])
    return ORACLE_SO


def build_reference(force: bool = False) -> bool:
    """Builds oracle/_ref from the reference sources; False when they are absent."""
    tools = os.path.join(REFERENCE_ROOT, "tools")
    src = os.path.join(tools, "cuda_baselines.cu")
    if not os.path.exists(src) or shutil.which(NVCC) is None:
        return False
    os.makedirs(REF_DIR, exist_ok=True)
    harness = os.path.join(HERE, "ref_harness.cu")
    if force or _stale(REF_SO, [src, harness]):
        _run([NVCC, "-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-Xcompiler", "-fPIC",
              "-shared", "-Dmain=ncz_reference_baselines_main", "-I", tools, harness, "-lcublas", "-o", REF_SO])
    if force or _stale(REF_BIN, [src]):
        _run([NVCC, "-O3", "-std=c++17", "-arch=sm_100a", src, "-lcublas", "-o", REF_BIN])
    sdpa = os.path.join(tools, "pytorch_baselines.py")
    if os.path.exists(sdpa) and (force or _stale(REF_SDPA, [sdpa])):
        shutil.copyfile(sdpa, REF_SDPA)
    return True


if __name__ == "__main__":
    print(build_oracle(force=True))
    print("reference built:", build_reference(force=True))
