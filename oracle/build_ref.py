"""Test infrastructure, not product: builds the reference's own GPU kernel (p2p/compact.cu, a torch extension) from its
source where it lies in the reference tree, into oracle/_ref/, for sm_100a.

The reference builds it the same way at first use (p2p/compact.py:22-33: torch.utils.cpp_extension.load of compact.cu
with -O3); here the architecture is pinned to sm_100a and the build directory is oracle/_ref/, so the module travels
with the repository to a GPU machine that has no reference tree. Nothing of the reference is copied: the compiler reads
the one source file in place.

    python -m oracle.build_ref [REFERENCE_ROOT]
"""
from __future__ import annotations

import glob
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
NAME = "p2p_compact"


def built() -> str | None:
    """The built module's path, or None."""
    hits = sorted(glob.glob(os.path.join(OUT, NAME + "*.so")))
    return hits[0] if hits else None


def build(reference_root: str) -> str | None:
    src = os.path.join(reference_root, "p2p", "compact.cu")
    if not os.path.exists(src):
        return None
    os.makedirs(OUT, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    os.environ.setdefault("MAX_JOBS", "4")
    from torch.utils.cpp_extension import load
    load(NAME, [src], extra_cuda_cflags=["-O3", "-lineinfo"], build_directory=OUT, verbose=False)
    return built()


def load_module():
    """The reference kernel module built by build(); raises if absent."""
    import importlib.util

    import torch  # noqa: F401  (the extension links against torch's libraries)
    path = built()
    if path is None:
        raise RuntimeError("the reference kernel is not built (python -m oracle.build_ref <reference root>)")
    spec = importlib.util.spec_from_file_location(NAME, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else os.path.join(os.sep, "root", "reference")))
