import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a) and the built libp2p_b200.so")


def golden(name: str) -> dict:
    with np.load(os.path.join(GOLDEN, name)) as f:
        return {k: f[k] for k in f.files}


@pytest.fixture(scope="session")
def select_cases():
    return golden("select_cases.npz")


@pytest.fixture(scope="session")
def config1_golden():
    return golden("config1.npz")


@pytest.fixture(scope="session")
def combine_golden():
    return golden("combine_cases.npz")


@pytest.fixture(scope="session")
def expert_golden():
    return golden("expert_case.npz")


@pytest.fixture(scope="session")
def tiles_golden():
    return golden("tiles_cases.npz")


def tiles_blocks(cases: dict, name: str):
    """The block list (p2p/prepare.py:201-206 form) of a tiles_cases.npz module, as torch tensors on the CPU."""
    import torch
    n_blocks, cols = int(cases[name + "_meta"][0]), int(cases[name + "_meta"][1])
    dt = torch.float16 if name == "b" else torch.bfloat16
    blocks = []
    for j in range(n_blocks):
        if f"{name}_b{j}_dense" in cases:
            w = torch.from_numpy(cases[f"{name}_b{j}_dense"].view(np.int16).copy()).view(dt)
            blocks.append(("dense", w))
        else:
            v = torch.from_numpy(cases[f"{name}_b{j}_values"].view(np.int16).copy()).view(dt)
            blocks.append(("sparse", v, torch.from_numpy(cases[f"{name}_b{j}_words"]), cols))
    return blocks
