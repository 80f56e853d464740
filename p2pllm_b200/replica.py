"""Replica groups on B200: the combine of p2p/replica.py on plain torch decoder layers.

A group of layers runs in parallel on decode and verify passes. Every member reads the group's input h; the last one
reads h~ = copy(h) from a pruned copy of the member before it. The next step reads

    h' = l_0(h) + sum_{0<k<n-1} (l_k(h) - h) + (l_last(h~) - h~)

in fp32, each difference rounded to the model's dtype first (p2p/replica.py:1-13, 81-85). The sum is one CUDA kernel
(kernels.combine). A layer here is any module whose forward(h) returns the layer's output with its residual added.
"""
from __future__ import annotations

import functools

import torch
import torch.nn as nn

from . import compact, family, kernels, wanda


def combine(parts: list, h: torch.Tensor, h_copy: torch.Tensor) -> torch.Tensor:
    """h' from the members' outputs (parts[k] = l_k(x_k)); p2p/replica.py:81-85."""
    return kernels.combine(parts, h, h_copy)


def _sharing_clone(module: nn.Module) -> nn.Module:
    """A new tree of module objects over the same tensors: every clone has parameter, buffer and child tables of its
    own, so replacing a tensor (or installing a quant_method) in the clone leaves the original untouched, while no
    tensor is copied."""
    twin = nn.Module.__new__(type(module))
    twin.__dict__.update(module.__dict__)
    for table in ("_parameters", "_buffers"):
        twin.__dict__[table] = dict(module.__dict__[table])
    twin.__dict__["_modules"] = {name: _sharing_clone(child) for name, child in module.__dict__["_modules"].items()}
    return twin


def shrink(layer: nn.Module, keep: dict, sums: dict, i: int, form: str = "dense") -> nn.Module:
    """A copy of layer i keeping `keep[projection]` percent of each projection's weights (p2p/replica.py:34-49).
    form "dense": pruned weights in place, as the reference's scan does; "compact": each pruned projection module
    multiplies through a Compact (values + column indices) instead of its dense weight."""
    c = _sharing_clone(layer)
    c.__dict__.pop("forward", None)
    modules = dict(c.named_modules())
    blocks: dict = {}
    pruned: set = set()                  # module tensors with a projection below keep 100; the rest stay shared
    for name, p in family.projections(layer).items():
        module = modules[p.path]
        w = getattr(module, p.param).data
        if keep[name] >= 100:
            blocks.setdefault((p.path, p.param), []).append((p.rows, ("dense", w[p.rows])))
            continue
        pruned.add((p.path, p.param))
        norms = wanda.channel_norms(sums[i, p.key], w, family.split_group(module, p))
        if form == "dense":
            blocks.setdefault((p.path, p.param), []).append((p.rows, ("dense", wanda.prune(w[p.rows], keep[name], norms))))
        else:
            values, idx = wanda.select(w[p.rows], keep[name], norms)
            blocks.setdefault((p.path, p.param), []).append((p.rows, ("compact", values, idx, w.shape[-1])))
    for (path, param), parts in blocks.items():
        if (path, param) not in pruned:
            continue
        module = modules[path]
        parts = [b for _, b in sorted(parts, key=lambda rb: _first_row(rb[0]))]
        if form == "dense" or param != "weight":
            setattr(module, param, nn.Parameter(torch.cat([compact.expand(b) for b in parts], dim=-2),
                                                requires_grad=False))
        else:
            method = compact.Compact(parts)
            bias = getattr(module, "bias", None)
            module.quant_method = method
            module.forward = functools.partial(_compact_forward, method, bias)
    return c


def _first_row(rows) -> int:
    """Where a projection starts in its module's tensor (routed experts: the slice after the expert axis)."""
    rows = rows[-1] if isinstance(rows, tuple) else rows
    return rows.start or 0


def _compact_forward(method, bias, x):
    return method.apply(None, x, bias)


def _run(module: nn.Module, x: torch.Tensor) -> torch.Tensor:
    """A layer's own forward, past any forward installed on the instance."""
    return type(module).forward(module, x)


def _member(group: list, replica: nn.Module, k: int, h: torch.Tensor, mode: str = "decode"):
    """Member k of a group on one pass (p2p/replica.py:69-85): on decode / verify passes member 0 runs the whole group
    and combines, the others pass h on; prefill runs each layer alone."""
    if mode not in ("decode", "verify"):
        return _run(group[k], h)
    if k:
        return h
    h_copy = _run(replica, h)
    outs = [_run(group[0], h)] + [_run(m, h) for m in group[1:-1]] + [_run(group[-1], h_copy)]
    return combine(outs, h, h_copy)


def install(layers: nn.ModuleList, plan: dict, sums: dict, groups: "list | None" = None, form: str = "dense",
            mode: str = "decode") -> None:
    """Apply a plan ({"groups": [[layer ids]], "keep": {layer: {projection: percent}}}), replacing any installed
    before; only `groups` of it, if given (p2p/replica.py:88-96)."""
    remove(layers)
    for group in plan["groups"] if groups is None else groups:
        copied = group[-2]
        replica = shrink(layers[copied], plan["keep"][str(copied)], sums, copied, form)
        members = [layers[i] for i in group]
        for k, layer in enumerate(members):
            layer.forward = functools.partial(_member, members, replica, k, mode=mode)


def remove(layers: nn.ModuleList) -> None:
    for layer in layers:
        layer.__dict__.pop("forward", None)
