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
from dataclasses import dataclass

import torch
from safetensors import safe_open
from safetensors.torch import save_file

from . import compact, family, wanda

# Largest ratio of compact bytes (values + mask words) to dense bytes at which a replica file keeps a pruned block in
# compact form; above it the block is written dense (the same rule as the reference's writer, so files match).
SAVES = 0.9


def _on_gpu(t: torch.Tensor) -> torch.Tensor:
    return t if t.is_cuda else t.cuda()


@dataclass
class StoredBlock:
    """How one projection's rows are stored in a replica file: whole ("dense": {"dense": W}, k = 0) or compact
    ({"values": [.., rows, k], "mask": [.., rows, ceil(cols / 32)]})."""
    projection: str
    rows: int
    k: int
    tensors: dict


def _store_projection(module, proj: family.Projection, name: str, keep: float, sums) -> StoredBlock:
    """The stored form of one projection at `keep` percent (p2p/prepare.py:42-73 decides the same way): keep >= 100 is
    stored whole; otherwise the Wanda selection (on the GPU) and the reference's packing, unless values + mask words
    would take more than SAVES of the dense bytes -- then the pruned rows are stored whole."""
    weight = getattr(module, proj.param).data
    rows, cols = weight[proj.rows], weight.shape[-1]
    n_rows = rows.shape[-2]
    if keep >= 100:
        return StoredBlock(name, n_rows, 0, {"dense": rows})
    norms = wanda.channel_norms(sums, _on_gpu(weight), family.split_group(module, proj))
    pruned, mask = wanda.prune(_on_gpu(rows), keep, norms, family.split_group(module, proj), with_mask=True)
    values, words = compact.pack(pruned.reshape(-1, cols), mask.reshape(-1, cols))
    if values.nbytes + words.nbytes > SAVES * rows.nbytes:
        return StoredBlock(name, n_rows, 0, {"dense": pruned})
    lead = rows.shape[:-1]
    return StoredBlock(name, n_rows, values.shape[-1], {"values": values.view(*lead, -1), "mask": words.view(*lead, -1)})


def plan_layer(layer, keep: dict, sums: dict, index: int) -> dict:
    """{module key: {"cols": cols, "blocks": [StoredBlock, ...]}} of one layer, modules and blocks in the order the
    layer's projections are listed."""
    by_path = dict(layer.named_modules())
    plan: dict = {}
    for name, proj in family.projections(layer).items():
        module = by_path[proj.path]
        cols = getattr(module, proj.param).shape[-1]
        entry = plan.setdefault(proj.key, {"cols": cols, "blocks": []})
        sums_of = sums[index, proj.key] if keep[name] < 100 else None
        entry["blocks"].append(_store_projection(module, proj, name, keep[name], sums_of))
    return plan


def serialise(index: int, keep: dict, plan: dict) -> tuple:
    """(tensors, metadata) of a planned layer in the file format above."""
    tensors, modules = {}, {}
    for key, entry in plan.items():
        listed = []
        for block in entry["blocks"]:
            for kind, t in block.tensors.items():
                tensors[f"{key}:{block.projection}:{kind}"] = t
            listed.append([block.projection, block.rows, block.k])
        modules[key] = {"cols": entry["cols"], "blocks": listed}
    return tensors, {"layer": index, "keep": keep, "modules": modules}


def write(layers, plan: dict, sums: dict, which: list, out: str) -> list:
    """dir/layer<i>.safetensors for each layer in `which`, its projections pruned to plan["keep"][str(i)] percent
    (p2p/prepare.py:42-73). sums: {(layer, module key): channel sums}, as wanda.Calibration.finish returns them.
    Returns the paths written."""
    paths = []
    for i in which:
        keep = plan["keep"][str(i)]
        tensors, meta = serialise(i, keep, plan_layer(layers[i], keep, sums, i))
        path = os.path.join(out, f"layer{i}.safetensors")
        save(tensors, meta, path)
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


def _first_row(proj: family.Projection) -> int:
    """Where a projection's rows start in its module's tensor."""
    rows = proj.rows[-1] if isinstance(proj.rows, tuple) else proj.rows
    return rows.start or 0


def _attach_experts(module, weights: dict, form: str) -> None:
    """Routed experts run compact: the layer's own MoE method over the used experts, expanded each pass
    (compact.CompactMoE), or, form "grouped", multiplied compact (moe.GroupedMoE); the module's expert tensors become
    empty."""
    import torch.nn as nn
    if form == "grouped":
        from . import moe
        module.quant_method = moe.GroupedMoE(module.quant_method, weights)
    else:
        module.quant_method = compact.CompactMoE(module.quant_method, weights)
    for param in weights:
        setattr(module, param, nn.Parameter(getattr(module, param).new_empty(0), requires_grad=False))


def install_replica(model, file: str, form: str = "compact") -> dict:
    """Replaces a copied layer's projections with the replica in `file` and returns its metadata (p2p/prepare.py:86-119
    has the same contract). Compact blocks make the module's quant_method a compact.Compact, its weight an empty
    [rows, 0] tensor; a module stored whole, or form "dense" (a check), gets the dense rows written back into its
    weight. Form "grouped" is "compact" with routed experts run by moe.GroupedMoE."""
    import torch.nn as nn
    tensors, meta = load(file)
    layer = family.layers(model)[meta["layer"]]
    by_path, projections = dict(layer.named_modules()), family.projections(layer)
    owner = {proj.key: proj for proj in projections.values()}
    routed: dict = {}
    for key, info in meta["modules"].items():
        proj = owner[key]
        module = by_path[proj.path]
        weight = getattr(module, proj.param)
        named = blocks_of(tensors, key, info, weight.device, weight.dtype)
        ordered = [block for _, block in sorted(named, key=lambda nb: _first_row(projections[nb[0]]))]
        if form == "dense" or all(block[0] == "dense" for block in ordered):
            weight.data.copy_(torch.cat([compact.expand(block) for block in ordered], dim=-2))
        elif proj.param == "weight":
            module.quant_method = compact.Compact(ordered)
            module.weight = nn.Parameter(weight.new_empty(weight.shape[0], 0), requires_grad=False)
        else:
            routed.setdefault(proj.path, {})[proj.param] = ordered
    for path, weights in routed.items():
        _attach_experts(by_path[path], weights, form)
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
    return meta
