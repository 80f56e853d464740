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


def _gated_layout(m):
    """The module's gate + up experts as one grouped layout whose GEMM squares and sums the gated activations (dense
    rows: every weight kept), built at the first calibration call and kept on the module while its weights stay; None
    when the shapes or dtypes do not fit the tensor-core kernel."""
    from . import moe
    w = m.w13_weight
    key = (w.data_ptr(), tuple(w.shape), w.dtype)
    cached = getattr(m, "_p2p_gated_layout", None)
    if cached is not None and cached[0] == key:
        return cached[1]
    tiles = None
    if (w.is_cuda and w.dtype in (torch.bfloat16, torch.float16) and w.dim() == 3 and w.shape[1] % 128 == 0
            and w.shape[2] % 8 == 0 and w.shape[2] <= 256 * 64):
        r = w.shape[1] // 2
        tiles = moe.ExpertTiles([("dense", w[:, :r]), ("dense", w[:, r:])], gated=True)
    m._p2p_gated_layout = (key, tiles)
    return tiles


def _distinct_experts(ids: torch.Tensor, n_exp: int) -> torch.Tensor:
    """ids [T, K] with each token's repeated experts, and ids outside [0, n_exp), replaced by -1: a token counts once
    for each expert it reaches."""
    s = ids.sort(-1).values
    bad = (s < 0) | (s >= n_exp)
    bad[:, 1:] |= s[:, 1:] == s[:, :-1]
    return torch.where(bad, torch.full_like(s, -1), s)


def expert_inputs(m, x: torch.Tensor, ids: torch.Tensor) -> tuple:
    """Sums of squares of what a FusedMoE's experts read, per channel and over the tokens routed to each (each token
    once): for gate and up [expert, hidden], for down [expert, rows]. ids: each token's experts; ids outside
    [0, experts) are skipped. p2p/wanda.py:10-20.

    The gated half runs on the grouped tensor-core GEMM when the experts are bf16 / f16 and x has their dtype: the
    routed tokens sorted by expert (moe.route), one launch over all experts whose epilogue squares silu(g) * u and sums
    it per item (fp32, the products exact), the items of an expert added in fp64. Otherwise an fp32 GEMM per expert."""
    n_exp, hidden = m.w13_weight.shape[0], m.w13_weight.shape[-1]
    into = torch.zeros(n_exp, hidden, dtype=torch.float64, device=x.device)
    gated = torch.zeros(m.w2_weight.shape[0], m.w2_weight.shape[-1], dtype=torch.float64, device=x.device)
    x2 = x.reshape(-1, hidden)
    kernels.expert_sumsq(x2, ids.reshape(x2.shape[0], -1), into)
    tiles = _gated_layout(m) if x2.dtype == m.w13_weight.dtype else None
    if tiles is not None:
        from . import moe
        flat = _distinct_experts(ids.reshape(x2.shape[0], -1), n_exp)
        r = moe.route(flat, n_exp)
        if r["order"].numel():
            xs = x2.index_select(0, r["order"] // flat.shape[1]).contiguous()
            sums = torch.empty(r["items"].shape[0], tiles.rows // 2, dtype=torch.float32, device=x.device)
            tiles.gated_sums(xs, r["items"], r["most"], sums)
            gated.index_add_(0, r["items"][:, 0].long(), sums.double())
        return into, gated
    xf = x2.float()
    flat = ids.reshape(x2.shape[0], -1)
    for e in torch.unique(flat[(flat >= 0) & (flat < n_exp)]).tolist():
        routed = xf[(flat == e).any(-1)]
        gate, up = (routed @ m.w13_weight[e].float().T).chunk(2, -1)       # an fp32 library GEMM per expert
        kernels.sumsq_cols(F.silu(gate) * up, gated[e])
    return into, gated


class Calibration:
    """Calibration of a model's layers for Wanda: while it is active, every module a projection reads its input from
    adds the per-channel sum of squares of that input, in fp64, to an accumulator on the GPU (the package's calibration
    kernel, one call per forward). Routed-expert modules add their per-expert sums (expert_inputs).

    Accumulators are keyed as p2p/wanda.py:23-60 keys them, so finish() returns what calib.pt holds: (layer index,
    projection key), the key being the module's path for a linear module and "<path>.w13_weight" /
    "<path>.w2_weight" for the routed experts' two tensors."""

    def __init__(self, layers):
        self._acc: dict = {}
        self._hooks: list = []
        for index, layer in enumerate(layers):
            by_path = dict(layer.named_modules())
            for path in sorted({proj.path for proj in family.projections(layer).values()}):
                module = by_path[path]
                make = self._routed_hook if hasattr(module, "w13_weight") else self._input_hook
                self._hooks.append(module.register_forward_pre_hook(make(index, path)))

    def _accumulator(self, key: tuple, shape, device) -> torch.Tensor:
        acc = self._acc.get(key)
        if acc is None:
            acc = self._acc[key] = torch.zeros(shape, dtype=torch.float64, device=device)
        return acc

    def _input_hook(self, index: int, path: str):
        def hook(module, args):
            x = args[0]
            kernels.sumsq_cols(x, self._accumulator((index, path), (x.shape[-1],), x.device))
        return hook

    def _routed_hook(self, index: int, path: str):
        def hook(module, args):
            into, gated = expert_inputs(module, args[0], args[1].topk_ids)
            for tensor_name, sums in (("w13_weight", into), ("w2_weight", gated)):
                self._accumulator((index, f"{path}.{tensor_name}"), sums.shape, sums.device).add_(sums)
        return hook

    def finish(self, layers) -> dict:
        """Removes the hooks and returns {(layer index, projection key): fp64 sums on the CPU}; a projection whose
        columns are split over a TP group gets the sums of all its columns (gathered from the group's ranks)."""
        for handle in self._hooks:
            handle.remove()
        self._hooks = []
        result = {}
        for index, layer in enumerate(layers):
            by_path = dict(layer.named_modules())
            for proj in family.projections(layer).values():
                key = (index, proj.key)
                if key in result or key not in self._acc:
                    continue
                sums = self._acc[key]
                group = family.split_group(by_path[proj.path], proj)
                if group:
                    sums = group.all_gather(sums, dim=sums.dim() - 1)
                result[key] = sums.cpu()
        return result


def channel_norms(sums: torch.Tensor, w: torch.Tensor, group=None) -> torch.Tensor:
    """The input-channel norms sqrt(sums) (fp32) that w's columns on this rank are scored with: [cols], or
    [experts, 1, cols] for routed experts, an expert that saw no token getting norms of one. With a TP group splitting
    w's columns (family.split_group), this rank's share of the sums is taken first (p2p/wanda.py:63-73)."""
    sums = sums.to(w.device)
    if group:
        width = w.shape[-1]
        first = group.rank_in_group * width
        sums = sums[..., first:first + width]
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
    """The dense form of the selection (p2p/wanda.py:76-87): w where a weight is among its row's k = k_of(keep, cols)
    best scores |w| * norms and zero elsewhere, plus, with_mask, the bool mask of the kept weights (k in every row).
    For columns split over a TP group the scores of the whole row decide, and each rank gets its own columns back, so
    the result does not depend on how many ranks hold the projection."""
    full_w, full_n = _full_rows(w, norms, group)
    k = k_of(keep, full_w.shape[-1])
    out = kernels.wanda_select(full_w, full_n, k, values=False, idx=False, mask=True, pruned=True)
    pruned, mask = out["pruned"], out["mask"]
    if group:
        start = group.rank_in_group * w.shape[-1]
        pruned, mask = pruned[..., start: start + w.shape[-1]], mask[..., start: start + w.shape[-1]]
    return (pruned, mask) if with_mask else pruned
