"""Wanda calibration and pruning on B200: the operator API of p2p/wanda.py.

Score |w_ij| * ||x_j|| in each row and keep the `keep` percent that score highest. Calibration sums and the per-row
selection run as CUDA kernels (libp2p_b200.so); `select` returns the compact form directly (values + column indices),
`prune` the reference's (pruned, mask).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import family, kernels


def k_of(keep: float, cols: int) -> int:
    """Weights a row keeps: max(1, round(keep / 100 * cols)), Python's round-half-even on the float (p2p/wanda.py:82;
    p2p/search.py:30 uses the same expression)."""
    return max(1, round(keep / 100 * cols))


def expert_inputs(m, x: torch.Tensor, ids: torch.Tensor) -> tuple:
    """Sums of squares of what a FusedMoE's experts read, per channel and over the tokens routed to each (each token
    once): for gate and up [expert, hidden], for down [expert, rows]. ids: each token's experts; ids outside
    [0, experts) are skipped. p2p/wanda.py:10-20."""
    n_exp, hidden = m.w13_weight.shape[0], m.w13_weight.shape[-1]
    into = torch.zeros(n_exp, hidden, dtype=torch.float64, device=x.device)
    gated = torch.zeros(m.w2_weight.shape[0], m.w2_weight.shape[-1], dtype=torch.float64, device=x.device)
    x2 = x.reshape(-1, hidden)
    kernels.expert_sumsq(x2, ids.reshape(x2.shape[0], -1), into)
    xf = x2.float()
    flat = ids.reshape(x2.shape[0], -1)
    for e in torch.unique(flat[(flat >= 0) & (flat < n_exp)]).tolist():
        routed = xf[(flat == e).any(-1)]
        gate, up = (routed @ m.w13_weight[e].float().T).chunk(2, -1)       # an fp32 library GEMM per expert
        kernels.sumsq_cols(F.silu(gate) * up, gated[e])
    return into, gated


class Calibration:
    """Per-channel sums of squares of every projection's input, collected through forward pre-hooks
    (p2p/wanda.py:23-60). Each hook call adds x.float().pow(2).sum(0).double() on the GPU."""

    def __init__(self, layers):
        self.sums, self.handles = {}, []
        for i, layer in enumerate(layers):
            modules = dict(layer.named_modules())
            for path in {p.path for p in family.projections(layer).values()}:
                hook = self._experts if hasattr(modules[path], "w13_weight") else self._linear
                self.handles.append(modules[path].register_forward_pre_hook(hook(i, path)))

    def _linear(self, i, path):
        def hook(module, args):
            x = args[0]
            sums = self.sums.get((i, path))
            if sums is None:
                sums = self.sums[i, path] = torch.zeros(x.shape[-1], dtype=torch.float64, device=x.device)
            kernels.sumsq_cols(x, sums)
        return hook

    def _experts(self, i, path):
        def hook(module, args):
            into, gated = expert_inputs(module, args[0], args[1].topk_ids)
            for key, v in (((i, f"{path}.w13_weight"), into), ((i, f"{path}.w2_weight"), gated)):
                self.sums[key] = self.sums[key] + v if key in self.sums else v
        return hook

    def finish(self, layers) -> dict:
        """Stop collecting. {(layer, projection key): sums over all ranks} on the CPU."""
        for h in self.handles:
            h.remove()
        out = {}
        for i, layer in enumerate(layers):
            modules = dict(layer.named_modules())
            for key, p in {p.key: p for p in family.projections(layer).values()}.items():
                if (i, key) in self.sums:
                    x, group = self.sums[i, key], family.split_group(modules[p.path], p)
                    out[i, key] = (group.all_gather(x, dim=x.dim() - 1) if group else x).cpu()
        return out


def channel_norms(sums: torch.Tensor, w: torch.Tensor, group=None) -> torch.Tensor:
    """||x_j|| for the columns of w this rank holds: [columns], or [expert, 1, columns] for experts, where an expert no
    token reached gets norms of one. group: as family.split_group. p2p/wanda.py:63-73."""
    sums = sums.to(w.device)
    if group:
        cols = w.shape[-1]
        sums = sums[..., group.rank_in_group * cols: (group.rank_in_group + 1) * cols]
    return kernels.channel_norms(sums)


def _full_rows(w: torch.Tensor, norms: torch.Tensor, group) -> tuple:
    """w and norms over all of a split projection's columns (the reference gathers scores, p2p/wanda.py:81; gathering
    the weights and norms gives the same scores)."""
    if not group:
        return w, norms
    return group.all_gather(w, dim=w.dim() - 1), group.all_gather(norms, dim=norms.dim() - 1)


def select(w: torch.Tensor, keep: float, norms: torch.Tensor, group=None, idx_dtype=None) -> tuple:
    """(values [.., k], idx [.., k]): the kept weights of each row and their columns, ascending; ties at the k-th score
    go to the lower column. The compact form of prune's choice."""
    full_w, full_n = _full_rows(w, norms, group)
    k = k_of(keep, full_w.shape[-1])
    out = kernels.wanda_select(full_w, full_n, k, idx_dtype=idx_dtype)
    return out["values"], out["idx"]


def prune(w: torch.Tensor, keep: float, norms: torch.Tensor, group=None, with_mask: bool = False):
    """w with zeros everywhere but the `keep` percent of each row's weights that score highest (and, with_mask, which
    those are: the same number in every row). A projection split across ranks compares scores across them, so the
    choice does not depend on the TP size. p2p/wanda.py:76-87."""
    full_w, full_n = _full_rows(w, norms, group)
    k = k_of(keep, full_w.shape[-1])
    out = kernels.wanda_select(full_w, full_n, k, values=False, idx=False, mask=True, pruned=True)
    pruned, mask = out["pruned"], out["mask"]
    if group:
        start = group.rank_in_group * w.shape[-1]
        pruned, mask = pruned[..., start: start + w.shape[-1]], mask[..., start: start + w.shape[-1]]
    return (pruned, mask) if with_mask else pruned
