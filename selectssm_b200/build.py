"""Builds ``libselectssm_b200.so`` (the C-ABI library) in-tree with nvcc for sm_100a.

Usage: ``python -m selectssm_b200.build`` (or ``__graft_entry__.build()``).
The library links the CUDA runtime statically and resolves the driver's
``cuTensorMapEncodeTiled`` at run time, so it needs no libcuda at link time.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libselectssm_b200.so")
SOURCES = ["scan.cu", "conv1d.cu", "noalloc.cu", "rmsnorm.cu", "selftest.cu"]
HEADERS = ["common.cuh", "scan_kernels.cuh", "scan_bwd.cuh", "scan_fwd.cuh", "scan_fwd_lane.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _inputs():
    inc = os.path.join(os.path.dirname(HERE), "include", "selectssm_b200.h")
    return [os.path.join(CSRC, f) for f in SOURCES + HEADERS] + [inc]


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(f) <= t for f in _inputs())


def build(force: bool = False, verbose: bool = False, extra_flags=None) -> str:
    """Compile the library unless it is newer than all its sources; returns its path."""
    if not force and up_to_date():
        return LIB
    cmd = [nvcc_path(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
           "-DSSM_BUILD", "-o", LIB + ".tmp"]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    cmd += list(extra_flags or [])
    cmd += [os.path.join(CSRC, f) for f in SOURCES]
    res = subprocess.run(cmd, cwd=CSRC, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + res.stdout + res.stderr)
    if verbose:
        sys.stderr.write(res.stdout + res.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
