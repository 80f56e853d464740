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
