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


OPS_SRC = os.path.join(HERE, "torch_ops", "ops.cpp")
OPS_LIB = os.path.join(HERE, "libp2p_torch_ops.so")


def build_ops(force: bool = False, verbose: bool = False) -> str:
    """Compiles the torch custom operators (torch_ops/ops.cpp, TORCH_LIBRARY p2p_b200) over the C ABI into
    libp2p_torch_ops.so. It leaves the p2p_* symbols undefined: _lib loads libp2p_b200.so into the global scope first."""
    deps = [OPS_SRC, os.path.join(ROOT, "include", "p2p_b200.h")]
    if not force and os.path.exists(OPS_LIB) and all(os.path.getmtime(d) <= os.path.getmtime(OPS_LIB) for d in deps):
        return OPS_LIB
    import torch
    from torch.utils import cpp_extension
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    torch_lib = os.path.join(os.path.dirname(torch.__file__), "lib")
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
           *[f"-I{p}" for p in cpp_extension.include_paths()], f"-I{os.path.join(cuda_home, 'include')}",
           f"-I{os.path.join(ROOT, 'include')}", OPS_SRC, f"-L{torch_lib}", "-lc10", "-ltorch_cpu", "-ltorch",
           "-lc10_cuda", f"-Wl,-rpath,{torch_lib}", "-o", OPS_LIB + ".tmp"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError(f"g++ failed on torch_ops/ops.cpp:\n{r.stderr[-6000:]}")
    if verbose:
        sys.stderr.write(r.stderr)
    os.replace(OPS_LIB + ".tmp", OPS_LIB)
    return OPS_LIB


def build(force: bool = False, verbose: bool = False) -> str:
    """Compiles every csrc/*.cu into libp2p_b200.so (objects in _build/); returns the library path."""
    if not force and not stale():
        return LIB
    out_dir = os.path.join(ROOT, "_build")
    os.makedirs(out_dir, exist_ok=True)
    headers = [p for p in DEPS if not p.endswith(".cu")]
    newest_header = max(os.path.getmtime(p) for p in headers)

    def compile_one(src: str) -> str:
        obj = os.path.join(out_dir, os.path.basename(src).replace(".cu", ".o"))
        # An object newer than its source and every header is reused (each .cu includes only the headers listed).
        if not force and os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), newest_header):
            return obj
        cmd = [nvcc(), *ARCH, *FLAGS, "-I", os.path.join(ROOT, "include"), "-c", src, "-o", obj + ".tmp"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode:
            raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stderr[-6000:]}")
        if verbose:
            sys.stderr.write(r.stderr)
        os.replace(obj + ".tmp", obj)
        return obj

    # The sources compile side by side (nvcc is single-threaded; the largest files take minutes each).
    from concurrent.futures import ThreadPoolExecutor
    with ThreadPoolExecutor(max_workers=max(1, min(len(SOURCES), os.cpu_count() or 1))) as pool:
        objs = list(pool.map(compile_one, SOURCES))
    tmp = LIB + ".tmp"
    r = subprocess.run([nvcc(), *ARCH, "-shared", "-o", tmp, *objs], capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError(f"nvcc link failed:\n{r.stderr[-4000:]}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
    print(build_ops(force="--force" in sys.argv, verbose="-v" in sys.argv))
