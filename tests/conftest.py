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
def llama_select():
    return golden("llama_select.npz")


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


# --- replica files: the small fake layer of tests/golden/make_golden.py (replica_case), rebuilt from its weights ------

REPLICA_KEEP = {"q": 33, "k": 40, "v": 100, "o": 33, "gate": 36, "up": 95, "down": 36}
REPLICA_SIZES = {"self_attn.qkv_proj": ((64, 16, 16), 64), "self_attn.o_proj": ((64,), 64),
                 "mlp.gate_up_proj": ((128, 128), 64), "mlp.down_proj": ((64,), 128)}


def _fake_linear(sizes, w):
    import torch

    class Linear(torch.nn.Module):
        """A linear module with the attributes SGLang's fused linear layers carry; runs its quant_method once a replica
        is installed, as SGLang's layers do (p2p/compact.py:205-218)."""

        def __init__(self):
            super().__init__()
            self.output_sizes, self.output_partition_sizes = list(sizes), list(sizes)
            self.output_size, self.input_size = sum(sizes), w.shape[1]
            self.weight = torch.nn.Parameter(w, requires_grad=False)

        def forward(self, x):
            if hasattr(self, "quant_method"):
                return self.quant_method.apply(self, x, None)
            return torch.nn.functional.linear(x, self.weight)

    return Linear()


def replica_model(case: dict, device="cpu"):
    """A one-layer model (model.layers[0]) with the fake layer's weights from replica_case.npz."""
    import torch
    layer = torch.nn.Module()
    layer.self_attn, layer.mlp = torch.nn.Module(), torch.nn.Module()
    for path, (sizes, cols) in REPLICA_SIZES.items():
        w = torch.from_numpy(case[f"w:{path}"].view(np.int16).copy()).view(torch.bfloat16).to(device)
        parent, name = path.split(".")
        setattr(getattr(layer, parent), name, _fake_linear(sizes, w))
    model = torch.nn.Module()
    model.layers = torch.nn.ModuleList([layer])
    return model


@pytest.fixture(scope="session")
def replica_golden():
    return golden("replica_case.npz")
