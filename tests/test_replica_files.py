"""Replica files (p2p/prepare.py:42-119): the file the reference's prepare.write made for a small layer
(tests/golden/replica_layer0.safetensors) loads with its tensors and metadata, saves back byte for byte, is written
again bit for bit by this package's GPU selection, and installs as compact modules whose outputs match the dense
pruned layer's."""
import json
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, REPLICA_KEEP, replica_model
from p2pllm_b200 import prepare

FILE = os.path.join(GOLDEN, "replica_layer0.safetensors")


def test_load_reads_the_reference_file():
    tensors, meta = prepare.load(FILE)
    assert meta["layer"] == 0 and meta["keep"] == REPLICA_KEEP
    blocks = {key: [b[0] for b in info["blocks"]] for key, info in meta["modules"].items()}
    assert blocks == {"self_attn.qkv_proj": ["q", "k", "v"], "self_attn.o_proj": ["o"],
                      "mlp.gate_up_proj": ["gate", "up"], "mlp.down_proj": ["down"]}
    for key, info in meta["modules"].items():
        for name, rows, k in info["blocks"]:
            if k == 0:
                assert tensors[f"{key}:{name}:dense"].shape == (rows, info["cols"])
            else:
                assert tensors[f"{key}:{name}:values"].shape == (rows, k)
                assert tensors[f"{key}:{name}:mask"].dtype == torch.int32
                assert tensors[f"{key}:{name}:mask"].shape == (rows, -(-info["cols"] // 32))
    # keep 100 is stored whole; keep 95 too (compact would take more than 0.9 of its dense bytes)
    assert "self_attn.qkv_proj:v:dense" in tensors and "mlp.gate_up_proj:up:dense" in tensors


def test_save_round_trip_is_byte_exact(tmp_path):
    tensors, meta = prepare.load(FILE)
    out = tmp_path / "layer0.safetensors"
    prepare.save(tensors, meta, str(out))
    assert out.read_bytes() == open(FILE, "rb").read()


@pytest.mark.gpu
def test_write_reproduces_the_reference_file(replica_golden, tmp_path):
    model = replica_model(replica_golden, "cuda")
    sums = {(0, k[5:]): torch.from_numpy(v) for k, v in replica_golden.items() if k.startswith("sums:")}
    path, = prepare.write(model.layers, {"keep": {"0": dict(REPLICA_KEEP)}}, sums, [0], str(tmp_path))
    got, got_meta = prepare.load(path)
    want, want_meta = prepare.load(FILE)
    assert got_meta == want_meta and sorted(got) == sorted(want)
    for k in want:
        assert torch.equal(got[k].view(torch.int16) if got[k].dtype == torch.bfloat16 else got[k],
                           want[k].view(torch.int16) if want[k].dtype == torch.bfloat16 else want[k]), k
    assert open(path, "rb").read() == open(FILE, "rb").read()


@pytest.mark.gpu
@pytest.mark.parametrize("form", ["compact", "dense"])
def test_install_replica_runs_the_pruned_layer(replica_golden, form):
    from p2pllm_b200 import compact
    model = replica_model(replica_golden, "cuda")
    tensors, meta = prepare.load(FILE)
    prepare.install_replica(model, FILE, form)
    layer = model.layers[0]
    g = torch.Generator(device="cuda").manual_seed(0)
    for key, info in meta["modules"].items():
        module = dict(layer.named_modules())[key]
        assert (hasattr(module, "quant_method") and module.weight.shape[1] == 0) == (form == "compact")
        blocks = [b for _, b in prepare.blocks_of(tensors, key, info, "cuda", torch.bfloat16)]
        dense = torch.cat([compact.expand(b) for b in blocks]).float()
        x = torch.randn(17, info["cols"], generator=g, device="cuda").bfloat16()
        y = module(x).float()
        want = x.float() @ dense.T
        assert float((y - want).norm() / want.norm()) <= 1e-2
