"""Builds libp2p_b200.so in this package directory with nvcc for sm_100a (B200) only.

    python -m p2pllm_b200.build [--force]

The library is plain C ABI (include/p2p_b200.h): no torch headers, no pybind. Python reaches it through ctypes
(p2pllm_b200._lib), other hosts through the header.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libp2p_b200.so")
SOURCES = sorted(glob.glob(os.path.join(HERE, "csrc", "*.cu")))
DEPS = SOURCES + sorted(glob.glob(os.path.join(HERE, "csrc", "*.cuh"))) + [os.path.join(ROOT, "include", "p2p_b200.h")]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", "-Xptxas", "-v"]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(found):
        raise RuntimeError("nvcc not found: the p2p_b200 CUDA library cannot be built here")
    return found


def stale() -> bool:
    if not os.path.exists(LIB):
        return True
    built = os.path.getmtime(LIB)
    return any(os.path.getmtime(p) > built for p in DEPS)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compiles every csrc/*.cu into libp2p_b200.so (objects in _build/); returns the library path."""
    if not force and not stale():
        return LIB
    out_dir = os.path.join(ROOT, "_build")
    os.makedirs(out_dir, exist_ok=True)
    objs = []
    for src in SOURCES:
        obj = os.path.join(out_dir, os.path.basename(src).replace(".cu", ".o"))
        cmd = [nvcc(), *ARCH, *FLAGS, "-I", os.path.join(ROOT, "include"), "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode:
            raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stderr[-6000:]}")
        if verbose:
            sys.stderr.write(r.stderr)
        objs.append(obj)
    tmp = LIB + ".tmp"
    r = subprocess.run([nvcc(), *ARCH, "-shared", "-o", tmp, *objs], capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError(f"nvcc link failed:\n{r.stderr[-4000:]}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
