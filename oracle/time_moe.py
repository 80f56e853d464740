"""Test infrastructure, not product: config 4's routed experts (128 experts, top-8, hidden 2048, intermediate 768,
keep 30, bf16, 272 tokens) timed two ways from the same compact blocks, on one GPU:

  grouped    this package's moe.GroupedMoE (the experts multiplied compact, p2p_spmm_tc_grouped)
  reference  the reference's path (p2p/compact.py:241-256, CompactMoE): every used expert expanded to dense each pass,
             then a fused dense MoE -- vLLM's Triton fused_experts standing in for SGLang's (not installable here)

Both outputs are checked against an fp32 MoE on the dense pruned weights (rel-L2 <= 1e-2). Median CUDA-event time of
`--passes` passes, each queued behind a spin kernel.

    python -m oracle.time_moe [--passes 20]
"""
from __future__ import annotations

import argparse
import statistics
from typing import NamedTuple

import torch
import torch.nn.functional as F


class TopK(NamedTuple):
    topk_weights: torch.Tensor
    topk_ids: torch.Tensor


class Dispatch(NamedTuple):
    hidden_states: torch.Tensor
    topk_output: TopK


def reference_moe(x, ids, weights, w13, w2):
    """fp32 gated-SiLU MoE on dense weights, expert by expert."""
    xf, out = x.float(), torch.zeros(x.shape[0], w2.shape[1], device=x.device)
    R = w13.shape[1] // 2
    for e in ids[ids >= 0].unique().tolist():
        t, j = (ids == e).nonzero(as_tuple=True)
        gu = xf[t] @ w13[e].float().T
        out.index_add_(0, t, weights[t, j].float().unsqueeze(1) * ((F.silu(gu[:, :R]) * gu[:, R:]) @ w2[e].float().T))
    return out


def experts(E, R, H, keep, g):
    """Compact blocks {"w13_weight": [gate, up], "w2_weight": [down]} of random experts and their dense pruned forms."""
    from p2pllm_b200 import wanda

    def prune(w):
        norms = torch.rand(w.shape[0], w.shape[2], generator=g, device="cuda") + 0.1
        vals, idxs = zip(*(wanda.select(w[e], keep, norms[e]) for e in range(w.shape[0])))
        values, idx = torch.stack(vals), torch.stack(idxs)
        dense = torch.zeros_like(w).scatter_(2, idx.long(), values)
        return ("compact", values, idx, w.shape[2]), dense

    w13 = (torch.randn(E, 2 * R, H, generator=g, device="cuda") * 0.05).bfloat16()
    w2 = (torch.randn(E, H, R, generator=g, device="cuda") * 0.05).bfloat16()
    (gate, dg), (up, du), (down, dd) = prune(w13[:, :R].contiguous()), prune(w13[:, R:].contiguous()), prune(w2)
    return {"w13_weight": [gate, up], "w2_weight": [down]}, torch.cat([dg, du], 1), dd


class DenseMethod:
    """The layer's own method the reference's CompactMoE hands the expanded experts to."""

    def apply(self, layer, d):
        from vllm.model_executor.layers.fused_moe import fused_experts
        t = d.topk_output
        return fused_experts(d.hidden_states, layer.w13_weight, layer.w2_weight, t.topk_weights, t.topk_ids)


def timed(fn, passes):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    out = []
    for _ in range(passes):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(4_000_000)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        out.append(a.elapsed_time(b) * 1e3)
    return statistics.median(out)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--passes", type=int, default=20)
    args = ap.parse_args()
    from p2pllm_b200 import compact, moe
    E, R, H, T, K = 128, 768, 2048, 272, 8
    g = torch.Generator(device="cuda").manual_seed(1)
    blocks, w13, w2 = experts(E, R, H, 30, g)
    w, ids = torch.randn(T, E, generator=g, device="cuda").softmax(-1).topk(K, dim=-1)
    x = torch.randn(T, H, generator=g, device="cuda").bfloat16()
    d = Dispatch(x, TopK(w, ids))
    want = reference_moe(x, ids, w, w13, w2)
    empty = torch.nn.Module()
    for name in ("w13_weight", "w2_weight"):
        empty.register_parameter(name, torch.nn.Parameter(x.new_empty(0), requires_grad=False))
    grouped = moe.GroupedMoE(None, blocks)
    expand = compact.CompactMoE(DenseMethod(), blocks)
    for name, fn in (("grouped", lambda: grouped.apply(None, d)), ("reference", lambda: expand.apply(empty, d))):
        y = fn()
        rel = float((y.float() - want).norm() / want.norm())
        assert rel <= 1e-2, (name, rel)
        us = timed(fn, args.passes)
        print(f"{name}: {us:.1f} us a pass, {T / us * 1e6:.0f} tokens/s, rel-L2 {rel:.2e}", flush=True)


if __name__ == "__main__":
    main()
