"""The public headers from plain C and from C++: tests/c_abi/consumer.c is
compiled as C99 and as C++17 with -Wall -Wextra -Werror -pedantic against
include/*.h, linked with
libncz_flash.so and run.  It installs a driver-call table written in C (one
fake device), launches through ncz_flash_fwd, ncz_flash_fwd_named and
ncz_mma_matmul_pipelined, and checks grids and kernel labels.  This is the
shape of binding a Zig or C host uses; no GPU is involved."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("compiler,lang", [("gcc", ["-std=c99"]), ("g++", ["-std=c++17", "-x", "c++"])])
def test_consumer_builds_and_runs(ncz, tmp_path, compiler, lang):
    cc = shutil.which(compiler)
    if cc is None:
        pytest.skip(f"no {compiler}")
    libdir = os.path.dirname(ncz.flash.LIB_PATH)
    exe = tmp_path / "consumer"
    build = subprocess.run([cc] + lang + ["-Wall", "-Wextra", "-Werror", "-pedantic", "-I",
                                          os.path.join(ROOT, "include"),
                                          os.path.join(ROOT, "tests", "c_abi", "consumer.c"), "-x", "none",
                                          "-L", libdir, "-lncz_flash", f"-Wl,-rpath,{libdir}", "-o", str(exe)],
                           capture_output=True, text=True)
    assert build.returncode == 0, build.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stderr
    assert "c abi consumer: ok" in run.stdout
