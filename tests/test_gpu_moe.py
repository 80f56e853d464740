"""The grouped MoE path (moe.GroupedMoE: the routed experts multiplied compact, no per-pass expansion) against a
plain fp32 MoE on the dense pruned weights: the reference's own MoE test case (tests/test_compact.py:80-126, f16) and
a config-4-shaped layer (128 experts, top-8, hidden 2048, intermediate 768, keep 30, bf16, 272 tokens) with tokens
routed nowhere, an expert past one grouped item (>256 tokens) and experts no token reaches. rel-L2 <= 1e-2."""
from typing import NamedTuple

import pytest
import torch
import torch.nn.functional as F

from p2pllm_b200 import compact, moe, wanda

pytestmark = pytest.mark.gpu


class TopK(NamedTuple):
    topk_weights: torch.Tensor
    topk_ids: torch.Tensor


class Dispatch(NamedTuple):
    hidden_states: torch.Tensor
    topk_output: TopK


def _reference_moe(x, ids, weights, w13, w2):
    """fp32 gated-SiLU MoE on dense weights, expert by expert; ids < 0 route nowhere."""
    xf, out = x.float(), torch.zeros(x.shape[0], w2.shape[1], device=x.device)
    R = w13.shape[1] // 2
    for e in ids[ids >= 0].unique().tolist():
        t, j = (ids == e).nonzero(as_tuple=True)
        gu = xf[t] @ w13[e].float().T
        h = F.silu(gu[:, :R]) * gu[:, R:]
        out.index_add_(0, t, weights[t, j].float().unsqueeze(1) * (h @ w2[e].float().T))
    return out


def _prune_experts(w, keep, g, form):
    """Per-expert Wanda selection of w [E, r, C]: the block and the dense pruned weights."""
    E, r, C = w.shape
    norms = torch.rand(E, C, generator=g, device="cuda") + 0.1
    vals, idxs = zip(*(wanda.select(w[e], keep, norms[e]) for e in range(E)))
    values, idx = torch.stack(vals), torch.stack(idxs)
    dense = torch.zeros_like(w)
    dense.scatter_(2, idx.long(), values)
    if form == "sparse":
        _, words = compact.pack(dense.reshape(-1, C), dense.reshape(-1, C) != 0)
        return ("sparse", values, words.view(E, r, -1), C), dense
    return ("compact", values, idx, C), dense


def _layer(E, R, H, keep, dtype, seed, form="compact"):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w13 = (torch.randn(E, 2 * R, H, generator=g, device="cuda") * 0.05).to(dtype)
    w2 = (torch.randn(E, H, R, generator=g, device="cuda") * 0.05).to(dtype)
    gate, dg = _prune_experts(w13[:, :R].contiguous(), keep, g, form)
    up, du = _prune_experts(w13[:, R:].contiguous(), keep, g, form)
    down, dd = _prune_experts(w2, keep, g, form)
    return {"w13_weight": [gate, up], "w2_weight": [down]}, torch.cat([dg, du], 1), dd, g


def _check(got, want):
    rel = float((got.float() - want).norm() / want.norm())
    assert rel <= 1e-2, rel


def test_the_reference_moe_case():
    """E 16, R 32, H 64, 5 tokens, 2 experts a token (5 of 16 used), keep 40, f16, the reference's packed blocks."""
    blocks, w13, w2, g = _layer(16, 32, 64, 40, torch.float16, 0, form="sparse")
    ids = torch.tensor([[3, 11], [11, 0], [7, 3], [15, 7], [0, 11]], device="cuda")
    x = torch.randn(5, 64, generator=g, device="cuda").half()
    w = torch.rand(5, 2, generator=g, device="cuda")
    got = moe.GroupedMoE(None, blocks).apply(None, Dispatch(x, TopK(w, ids)))
    assert got.dtype == torch.float16 and got.shape == (5, 64)
    _check(got, _reference_moe(x, ids, w, w13, w2))


def test_a_config4_layer_with_skewed_routing():
    E, R, H, T, K = 128, 768, 2048, 272, 8
    blocks, w13, w2, g = _layer(E, R, H, 30, torch.bfloat16, 1)
    logits = torch.randn(T, E, generator=g, device="cuda")
    logits[:, 120:] = -1e9                                   # experts 120.. never reached
    logits[:, 0] += 10                                       # every token to expert 0: 272 > 256 tokens, two items
    w, ids = logits.softmax(-1).topk(K, dim=-1)
    ids = ids.clone()
    ids[::17, -1] = -1                                       # some slots routed nowhere
    x = torch.randn(T, H, generator=g, device="cuda").bfloat16()
    layer = moe.GroupedMoE(None, blocks)
    got = layer.apply(None, Dispatch(x, TopK(w, ids)))
    _check(got, _reference_moe(x, ids, w, w13, w2))
    again = layer.apply(None, Dispatch(x, TopK(w, ids)))
    assert torch.equal(got, again)                           # fixed order: the same bits every pass


def test_no_routed_tokens_give_zeros():
    blocks, _, _, g = _layer(4, 64, 64, 50, torch.bfloat16, 2)
    x = torch.randn(3, 64, generator=g, device="cuda").bfloat16()
    ids = torch.full((3, 2), -1, device="cuda")
    got = moe.GroupedMoE(None, blocks).apply(None, Dispatch(x, TopK(torch.ones(3, 2, device="cuda"), ids)))
    assert torch.equal(got, torch.zeros_like(got))


@pytest.mark.parametrize("T,K,E", [(272, 8, 128), (5, 2, 16), (3000, 4, 64), (1, 1, 1)])
def test_route_is_a_stable_sort_by_expert(T, K, E):
    """p2p_moe_route against torch: pairs sorted by expert (ties by pair index), places, counts, items of <= 256."""
    g = torch.Generator(device="cuda").manual_seed(T)
    ids = torch.randint(-1, E, (T, K), generator=g, device="cuda")
    ids[0, 0] = 0
    r = moe.route(ids, E)
    flat = ids.reshape(-1)
    key = torch.where(flat >= 0, flat, torch.full_like(flat, E))
    want = torch.argsort(key, stable=True)[: int((flat >= 0).sum())]
    assert torch.equal(r["order"], want)
    where = torch.full_like(flat, -1)
    where[want] = torch.arange(want.numel(), device="cuda")
    assert torch.equal(r["where"], where)
    counts = torch.bincount(flat[flat >= 0], minlength=E)
    assert torch.equal(r["counts"].long(), counts)
    items = r["items"].cpu().tolist()
    start, k = 0, 0
    for e, c in enumerate(counts.tolist()):
        for s in range(0, c, 256):
            assert items[k] == [e, start + s, min(256, c - s), 0]
            k += 1
        start += c
    assert k == len(items) and r["most"] == max((it[2] for it in items), default=0)


def test_grouped_gate_in_the_epilogue_matches_silu_between_launches():
    """Config-4 shapes (R = 768): the gate/up launch with SiLU(gate) * up in its epilogue against the same pass with
    the activation between the two launches (rel-L2 1e-3: only the epilogue's exp may differ in the last fp32 bit)."""
    E, R, H, T, K = 128, 768, 2048, 272, 8
    blocks, w13, w2, g = _layer(E, R, H, 30, torch.bfloat16, 5)
    fused = moe.GroupedMoE(None, blocks)
    assert fused.w13.gated
    unfused = moe.GroupedMoE(None, blocks)
    unfused.w13 = moe.ExpertTiles(blocks["w13_weight"])
    assert not unfused.w13.gated
    logits = torch.randn(T, E, generator=g, device="cuda")
    w, ids = logits.softmax(-1).topk(K, dim=-1)
    x = torch.randn(T, H, generator=g, device="cuda").bfloat16()
    got = fused.apply(None, Dispatch(x, TopK(w, ids)))
    want = unfused.apply(None, Dispatch(x, TopK(w, ids)))
    rel = float((got.double() - want.double()).norm() / want.double().norm())
    assert rel <= 1e-3, rel
    _check(got, _reference_moe(x, ids, w, w13, w2))


def test_gated_expert_calibration_on_the_grouped_kernel():
    """wanda.expert_inputs' gated half on the grouped GEMM (bf16 experts) against p2p/wanda.py:16-19 restated in torch
    fp32 (a token routed twice to one expert counts once; experts past 120 never reached; one expert with more than 256
    tokens, so two items)."""
    import types
    from p2pllm_b200 import wanda
    E, R, H, T, K = 128, 768, 2048, 300, 8
    g = torch.Generator(device="cuda").manual_seed(11)
    w13 = (torch.randn(E, 2 * R, H, generator=g, device="cuda") * 0.05).bfloat16()
    m = types.SimpleNamespace(w13_weight=w13, w2_weight=torch.zeros(E, H, R, device="cuda").bfloat16())
    logits = torch.randn(T, E, generator=g, device="cuda")
    logits[:, 120:] = -1e9
    logits[:, 0] += 10
    ids = logits.topk(K, dim=-1).indices
    ids[::7, 1] = ids[::7, 0]                                # a repeated expert in some tokens
    ids[::11, -1] = -1                                       # and slots routed nowhere
    x = torch.randn(T, H, generator=g, device="cuda").bfloat16()
    into, gated = wanda.expert_inputs(m, x, ids)
    assert wanda._gated_layout(m) is not None
    want = torch.zeros(E, R, dtype=torch.float64, device="cuda")
    xf = x.float()
    for e in range(E):
        routed = xf[(ids == e).any(-1)]
        if routed.shape[0] == 0:
            continue
        gate, up = (routed @ w13[e].float().T).chunk(2, -1)
        want[e] = (torch.nn.functional.silu(gate) * up).pow(2).sum(0).double()
    assert torch.allclose(gated, want, rtol=1e-4, atol=1e-9), float(((gated - want).abs() / want.abs().clamp_min(1e-9)).max())
    assert (gated[120:] == 0).all()
