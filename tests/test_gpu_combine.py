"""The group-combine epilogue and the spread-step parts on the GPU, bit for bit against the reference's outputs
(fixtures made by running p2p.replica._member and p2p.route._summed)."""
import numpy as np
import pytest
import torch

import oracle
from p2pllm_b200 import kernels, replica, route

pytestmark = pytest.mark.gpu

TORCH_DT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def _t(bits, dt):
    if dt == "f32":
        return torch.from_numpy(bits.copy()).cuda()
    return torch.from_numpy(bits.view(np.int16).copy()).view(TORCH_DT[dt]).cuda()


def _bits(t):
    t = t.cpu()
    return t.view(torch.int16).numpy().view(np.uint16) if t.dtype != torch.float32 else t.numpy()


@pytest.mark.parametrize("dt", ["bf16", "f32", "f16"])
@pytest.mark.parametrize("n", [2, 3, 5])
def test_combine_and_summed_are_bit_exact(combine_golden, n, dt):
    key = f"n{n}_{dt}"
    parts = [_t(combine_golden[key + f"_p{j}"], dt) for j in range(n)]
    h, hc = _t(combine_golden[key + "_h"], dt), _t(combine_golden[key + "_hc"], dt)
    out = replica.combine(parts, h, hc)
    assert np.array_equal(_bits(out).view(np.uint8), combine_golden[key + "_out"].view(np.uint8))
    s = route.summed(parts)
    assert np.array_equal(_bits(s).view(np.uint8), combine_golden[key + "_summed"].view(np.uint8))


@pytest.mark.parametrize("numel", [1, 7, 8, 4096 * 17, 4096 * 64 + 3])
@pytest.mark.parametrize("dt", ["bf16", "f32"])
def test_combine_any_size_against_the_oracle(numel, dt):
    g = torch.Generator(device="cuda").manual_seed(numel)
    mk = lambda: torch.randn(numel, generator=g, device="cuda").to(TORCH_DT[dt])
    h, hc, parts = mk(), mk(), [mk() for _ in range(4)]
    out = kernels.combine(parts, h, hc)
    want = oracle.combine([_bits(p) for p in parts], _bits(h), _bits(hc), dt)
    assert np.array_equal(_bits(out).view(np.uint8), want.view(np.uint8))
    part = route.member_part(1, parts[1], h)
    assert np.array_equal(_bits(part).view(np.uint8), oracle.member_part(_bits(parts[1]), _bits(h), dt).view(np.uint8))
    assert route.member_part(0, parts[0], h) is parts[0]


def test_misaligned_views_take_the_scalar_path():
    base = torch.randn(4 * 4096 + 1, device="cuda").bfloat16()
    h = base[1:]                                    # 2 bytes past a 16-byte boundary
    parts = [torch.randn(4 * 4096, device="cuda").bfloat16() for _ in range(3)]
    out = kernels.combine(parts, h, h)
    want = oracle.combine([_bits(p) for p in parts], _bits(h), _bits(h), "bf16")
    assert np.array_equal(_bits(out), want)


class _Block(torch.nn.Module):
    """A synthetic Llama-shaped decoder block standing in for attention + MLP: h + down(silu(gate h) * up h)."""

    def __init__(self, hidden, inter, seed):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.gate_proj = torch.nn.Linear(hidden, inter, bias=False)
        self.up_proj = torch.nn.Linear(hidden, inter, bias=False)
        self.down_proj = torch.nn.Linear(inter, hidden, bias=False)
        for m in (self.gate_proj, self.up_proj, self.down_proj):
            m.weight.data = torch.randn(m.weight.shape, generator=g) * 0.02

    def forward(self, h):
        return h + self.down_proj(torch.nn.functional.silu(self.gate_proj(h)) * self.up_proj(h))


def test_group_install_matches_the_formula():
    """replica.install on plain layers: decode runs the group through member 0, the others pass h on, prefill runs
    each layer alone (tests/test_sglang.py:224-240 on real, shaped layers)."""
    hidden, inter = 256, 512
    layers = torch.nn.ModuleList([_Block(hidden, inter, s) for s in range(3)]).cuda().bfloat16()
    sums = {(1, p): torch.rand(hidden if p != "down_proj" else inter, dtype=torch.float64) + 0.1
            for p in ("gate_proj", "up_proj", "down_proj")}
    plan = {"groups": [[0, 1, 2]], "keep": {"1": {"gate": 40, "up": 40, "down": 40}}}
    h = torch.randn(8, hidden, device="cuda").bfloat16()
    with torch.no_grad():
        copy = replica.shrink(layers[1], plan["keep"]["1"], sums, 1, form="dense")
        want = replica.combine([layers[0](h), layers[1](h), layers[2](copy(h))], h, copy(h))
        for form in ("dense", "compact"):
            replica.install(layers, plan, sums, form=form)
            got = layers[0](h)
            assert layers[1](got) is got and layers[2](got) is got
            if form == "dense":
                assert torch.equal(got, want)
            else:
                assert (got.float() - want.float()).norm() / want.float().norm() <= 1e-2
        replica.remove(layers)
        assert torch.equal(layers[1](h), _Block.forward(layers[1], h))


def test_shrink_prunes_routed_experts_per_projection():
    """p2p/replica.py:34-49 on a layer with routed experts: gate, up and down of every expert pruned on their own
    (per-expert channel norms from [E, C] sums), the rest of the layer shared; the compact form expands experts."""
    import torch.nn as nn

    from p2pllm_b200 import wanda

    E, R, H = 4, 32, 64
    g = torch.Generator(device="cuda").manual_seed(0)

    class Experts(nn.Module):
        def __init__(self):
            super().__init__()
            self.w13_weight = nn.Parameter(torch.randn(E, 2 * R, H, generator=g, device="cuda").bfloat16(), False)
            self.w2_weight = nn.Parameter(torch.randn(E, H, R, generator=g, device="cuda").bfloat16(), False)

    class Mlp(nn.Module):
        def __init__(self):
            super().__init__()
            self.experts = Experts()
            self.down_proj = nn.Linear(R, H, bias=False, device="cuda", dtype=torch.bfloat16)
            self.gate_proj = nn.Linear(H, R, bias=False, device="cuda", dtype=torch.bfloat16)

    class Layer(nn.Module):
        def __init__(self):
            super().__init__()
            self.mlp = Mlp()

    layer = Layer()
    sums = {(0, "mlp.experts.w13_weight"): torch.rand(E, H, generator=g, device="cuda").double() + 0.1,
            (0, "mlp.experts.w2_weight"): torch.rand(E, R, generator=g, device="cuda").double() + 0.1}
    sums[0, "mlp.experts.w2_weight"][2] = 0                    # an expert no token reached: norms of one
    keep = {"egate": 30, "eup": 50, "edown": 40, "down": 100, "gate": 100}
    for form in ("dense", "compact"):
        c = replica.shrink(layer, keep, sums, 0, form=form)
        w13, w2 = layer.mlp.experts.w13_weight, layer.mlp.experts.w2_weight
        n13 = wanda.channel_norms(sums[0, "mlp.experts.w13_weight"], w13)
        n2 = wanda.channel_norms(sums[0, "mlp.experts.w2_weight"], w2)
        want13 = torch.cat([wanda.prune(w13[:, :R], 30, n13), wanda.prune(w13[:, R:], 50, n13)], dim=1)
        assert torch.equal(c.mlp.experts.w13_weight, want13)
        assert torch.equal(c.mlp.experts.w2_weight, wanda.prune(w2, 40, n2))
        assert (c.mlp.experts.w13_weight != 0).sum() == E * R * (round(0.3 * H) + round(0.5 * H))
        assert c.mlp.down_proj.weight is layer.mlp.down_proj.weight   # keep 100: shared, untouched
        assert layer.mlp.experts.w13_weight is w13 and torch.equal(w13, layer.mlp.experts.w13_weight)
