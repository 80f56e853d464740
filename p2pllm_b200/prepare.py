"""Replica files: the on-disk form of a pruned layer, as p2p/prepare.py writes and installs it, with the selection and
the GEMM on B200.

File format (p2p/prepare.py:42-84), one safetensors file a layer, dir/layer<i>.safetensors:

    "<module key>:<projection>:values"  [rows, k]                 the kept weights of each row, in column order
    "<module key>:<projection>:mask"    [rows, ceil(cols / 32)]   int32 words, bit c % 32 of word c // 32: column c kept
    "<module key>:<projection>:dense"   [rows, cols]              a block stored whole (keep 100, or compact would
                                                                   take more than SAVES of its dense bytes)
    metadata "p2p": JSON {"layer": i, "keep": {projection: keep},
                          "modules": {module key: {"cols": cols, "blocks": [[projection, rows, k (0: dense)], ...]}}}

Routed experts carry a leading expert dimension on every tensor. The format is the reference's, so files written by
either side install on the other; write() makes its selection on the GPU (Wanda top-k, ties to the lower column) and
install_replica() hands the blocks to compact.Compact / compact.CompactMoE (or, with form "grouped", routed experts to
moe.GroupedMoE, which multiplies them compact instead of expanding them every pass).
"""
from __future__ import annotations

import json
import os

import torch
from safetensors import safe_open
from safetensors.torch import save_file

from . import compact, family, wanda

SAVES = 0.9            # a pruned block is stored compact only if that takes at most this share of its dense bytes


def _on_gpu(t: torch.Tensor) -> torch.Tensor:
    return t if t.is_cuda else t.cuda()


def write(layers, plan: dict, sums: dict, which: list, out: str) -> list:
    """dir/layer<i>.safetensors for each layer in `which`: per projection its row blocks, each kept whole or pruned to
    plan["keep"][str(i)][projection] percent and packed (p2p/prepare.py:42-73). sums: {(layer, module key): channel
    sums}, as wanda.Calibration.finish returns them. Returns the paths written."""
    paths = []
    for i in which:
        layer, keep = layers[i], plan["keep"][str(i)]
        modules, projections = dict(layer.named_modules()), family.projections(layer)
        tensors, meta = {}, {}
        for name, p in projections.items():
            module = modules[p.path]
            w = getattr(module, p.param).data
            block, cols = w[p.rows], w.shape[-1]
            entry = meta.setdefault(p.key, {"cols": cols, "blocks": []})["blocks"]
            if keep[name] >= 100:
                tensors[f"{p.key}:{name}:dense"] = block
                entry.append([name, block.shape[-2], 0])
                continue
            group = family.split_group(module, p)
            gw = _on_gpu(w)
            norms = wanda.channel_norms(sums[i, p.key], gw, group)
            pruned, mask = wanda.prune(_on_gpu(block), keep[name], norms, group, with_mask=True)
            values, words = compact.pack(pruned.reshape(-1, cols), mask.reshape(-1, cols))
            if values.nbytes + words.nbytes > SAVES * block.nbytes:   # compact would save too little: keep it dense
                tensors[f"{p.key}:{name}:dense"] = pruned
                entry.append([name, block.shape[-2], 0])
                continue
            lead = block.shape[:-1]
            tensors[f"{p.key}:{name}:values"] = values.view(*lead, -1)
            tensors[f"{p.key}:{name}:mask"] = words.view(*lead, -1)
            entry.append([name, block.shape[-2], values.shape[-1]])
        path = os.path.join(out, f"layer{i}.safetensors")
        save(tensors, {"layer": i, "keep": keep, "modules": meta}, path)
        paths.append(path)
    return paths


def save(tensors: dict, meta: dict, path: str) -> None:
    """The tensors (on the host, contiguous) and the metadata under "p2p" (p2p/prepare.py:76-77)."""
    save_file({k: v.contiguous().cpu() for k, v in tensors.items()}, path, metadata={"p2p": json.dumps(meta)})


def load(path: str) -> tuple:
    """(tensors, metadata) that save wrote (p2p/prepare.py:80-83)."""
    with safe_open(path, "pt") as h:
        return {k: h.get_tensor(k) for k in h.keys()}, json.loads(h.metadata()["p2p"])


def blocks_of(tensors: dict, key: str, info: dict, device=None, dtype=None) -> list:
    """One module's row blocks from a replica file, in the order the metadata lists them: ("dense", W) or
    ("sparse", values, mask words, cols) (p2p/prepare.py:97-101)."""
    out = []
    for p, rows, k in info["blocks"]:
        if k == 0:
            block = ("dense", tensors[f"{key}:{p}:dense"])
        else:
            block = ("sparse", tensors[f"{key}:{p}:values"], tensors[f"{key}:{p}:mask"], info["cols"])
        out.append((p, tuple(t.to(device, dtype if t.is_floating_point() else t.dtype) if torch.is_tensor(t) else t
                             for t in block)))
    return out


def install_replica(model, file: str, form: str = "compact") -> dict:
    """Replace a copied layer's projections with the replica in `file` and return its metadata: compact as their
    modules' quant_method (the module's weight becomes an empty [rows, 0] tensor), or expanded back into the weight
    (form "dense", a check) (p2p/prepare.py:86-119). Form "grouped" is "compact" with routed experts run by
    moe.GroupedMoE (gated SiLU) instead of compact.CompactMoE."""
    import torch.nn as nn
    tensors, meta = load(file)
    layer = family.layers(model)[meta["layer"]]
    modules, projections = dict(layer.named_modules()), family.projections(layer)
    where = {p.key: (p.path, p.param) for p in projections.values()}
    experts = {}

    def first_row(p):                    # where a projection starts in its module's tensor
        rows = p.rows[-1] if isinstance(p.rows, tuple) else p.rows
        return rows.start or 0

    for key, info in meta["modules"].items():
        path, param = where[key]
        module = modules[path]
        w = getattr(module, param)
        parts = blocks_of(tensors, key, info, w.device, w.dtype)
        parts = [b for _, b in sorted(parts, key=lambda nb: first_row(projections[nb[0]]))]
        if form == "dense" or all(b[0] == "dense" for b in parts):     # nothing compact: the layer's own method runs
            w.data.copy_(torch.cat([compact.expand(b) for b in parts], dim=-2))
        elif param == "weight":
            module.quant_method = compact.Compact(parts)
            module.weight = nn.Parameter(w.new_empty(w.shape[0], 0), requires_grad=False)
        else:
            experts.setdefault(path, {})[param] = parts
    for path, weights in experts.items():
        module = modules[path]
        if form == "grouped":
            from . import moe
            module.quant_method = moe.GroupedMoE(module.quant_method, weights)
        else:
            module.quant_method = compact.CompactMoE(module.quant_method, weights)
        for param in weights:
            setattr(module, param, nn.Parameter(getattr(module, param).new_empty(0), requires_grad=False))
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
    return meta
