"""Where a decoder layer's projections sit inside its modules: the projection -> row-slice mapping of p2p/family.py.

Only what the replica path needs is kept: the name table, Projection, layers(), projections() and split_group(). A
fused module (qkv_proj, gate_up_proj) is cut by its `output_sizes`, a plain torch Linear counts as one projection named
by its attribute, and routed experts ([expert, 2 * rows, hidden] gate + up, [expert, hidden, rows] down) give
egate / eup / edown.
"""
from __future__ import annotations

from typing import NamedTuple

import torch.nn as nn

TABLE = {"qkv_proj": ("q", "k", "v"), "in_proj_qkvz": ("q", "k", "v", "z"), "o_proj": ("o",), "out_proj": ("out",),
         "gate_up_proj": ("gate", "up"), "down_proj": ("down",),
         # plain torch layers name each projection on its own
         "q_proj": ("q",), "k_proj": ("k",), "v_proj": ("v",), "gate_proj": ("gate",), "up_proj": ("up",)}


class Projection(NamedTuple):
    """One projection of a decoder layer. The field names and `key` are the calib.pt interface shared with p2p/family.py
    (calibration sums and replica files are keyed by them)."""
    path: str                # dotted path of the owning module, from the layer
    rows: "slice | tuple"    # index of this projection's rows in the module's tensor as this rank holds it
    shape: list              # [rows, cols] of the whole projection, every rank's share together
    param: str = "weight"    # attribute name of the module's tensor

    @property
    def key(self) -> str:
        """The calib.pt key: the module path for a linear module's weight, "<path>.<tensor>" for routed experts."""
        return self.path if self.param == "weight" else f"{self.path}.{self.param}"


def _is_layer(m: nn.Module) -> bool:
    names = {path.rsplit(".", 1)[-1] for path, _ in m.named_modules()}
    return "down_proj" in names and bool({"gate_up_proj", "gate_proj"} & names)


def layers(model: nn.Module) -> nn.ModuleList:
    """The decoder layers: the longest module list whose first entry holds an MLP named in TABLE."""
    found = [m for m in model.modules() if isinstance(m, nn.ModuleList) and len(m) and _is_layer(m[0])]
    if not found:
        raise ValueError(f"{type(model).__name__}: add its projections to p2pllm_b200.family.TABLE")
    return max(found, key=len)


def projections(layer: nn.Module) -> dict:
    """{projection name: Projection} of a decoder layer (p2p/family.py:40-56)."""
    out = {}
    for path, m in layer.named_modules():
        names = TABLE.get(path.rsplit(".", 1)[-1])
        if names and hasattr(m, "weight"):
            sizes = getattr(m, "output_partition_sizes", None) or getattr(m, "output_sizes", None) or [m.weight.shape[0]]
            totals = getattr(m, "output_sizes", None) or sizes
            cols = getattr(m, "input_size", None) or m.weight.shape[-1]
            if len(sizes) != len(names):
                raise ValueError(f"{path}: {len(sizes)} row blocks for {names}")
            start = 0
            for name, total, rows in zip(names, totals, sizes):
                out[name] = Projection(path, slice(start, start + rows), [total, cols])
                start += rows
        elif hasattr(m, "w13_weight") and hasattr(m, "w2_weight"):
            n_exp, two_r, hidden = m.w13_weight.shape
            r = two_r // 2
            out["egate"] = Projection(path, (slice(None), slice(0, r)), [n_exp * r, hidden], "w13_weight")
            out["eup"] = Projection(path, (slice(None), slice(r, 2 * r)), [n_exp * r, hidden], "w13_weight")
            out["edown"] = Projection(path, (slice(None), slice(None)), [n_exp * hidden, r], "w2_weight")
    return out


def split_group(module: nn.Module, p: Projection):
    """The TP group whose ranks each hold only some of this projection's columns, or None if this rank holds them all
    (p2p/family.py:82-89). Modules outside SGLang carry theirs as `tp_group`."""
    if getattr(module, p.param).shape[-1] == p.shape[1]:
        return None
    return getattr(module, "tp_group", None)
