"""Build-quality guard, no GPU needed: every sm_100a kernel compiles with the
library's flags and ptxas reports no register spills, except the one known
small spill listed below.  ptxas resource lines (registers, stack, spills) are
compiler output about this repository's own kernels."""
from __future__ import annotations

import concurrent.futures
import pathlib
import re
import shutil
import subprocess

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
KERNELS = sorted((ROOT / "tsac-metal_b200" / "csrc" / "kernels").glob("*.cu"))
FLAGS = ["-std=c++20", "-O3", "-gencode", "arch=compute_100a,code=sm_100a", "-fmad=false", "-ftz=false",
         "-prec-div=true", "-prec-sqrt=true", "-I", str(ROOT / "tsac-metal_b200" / "csrc"),
         "-I", str(ROOT / "include"), "-Xptxas", "-v", "-c", "-o", "/dev/null"]
# Known: the 64-channel exact-convolution tile keeps 32 prefetch registers of
# inputs at its 128-register cap (two CTAs per SM) and spills one word.
ALLOWED_SPILLS = {"conv1d_kernelILi64ELi256E": (4, 16)}


def _spills(source):
    out = subprocess.run(["nvcc", *FLAGS, str(source)], capture_output=True, text=True)
    assert out.returncode == 0, out.stderr[-2000:]
    found, current = {}, None
    for line in out.stderr.splitlines():
        m = re.search(r"Compiling entry function '([^']+)'", line)
        if m:
            current = m.group(1)
        m = re.search(r"(\d+) bytes spill stores, (\d+) bytes spill loads", line)
        if m and current:
            found[current] = (int(m.group(1)), int(m.group(2)))
    return source.name, found


@pytest.mark.slow
@pytest.mark.skipif(shutil.which("nvcc") is None, reason="nvcc not installed")
def test_kernels_compile_without_new_spills():
    with concurrent.futures.ThreadPoolExecutor(8) as pool:
        results = list(pool.map(_spills, KERNELS))
    entries = 0
    for name, found in results:
        entries += len(found)
        for function, (stores, loads) in found.items():
            allowed = next((v for k, v in ALLOWED_SPILLS.items() if k in function), (0, 0))
            assert stores <= allowed[0] and loads <= allowed[1], f"{name}: {function} spills {stores}/{loads} bytes"
    assert entries >= 20
