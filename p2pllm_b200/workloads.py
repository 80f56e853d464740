"""Seeded synthetic workloads with the shapes and value distributions of the five benchmark configurations.

No checkpoints or datasets are used: weights are N(0, 0.02), calibration and forward activations are N(0, 1) scaled
per input channel by lognormal(0, 1), generated from fixed seeds, on the CPU generator (reproducible on any machine
with the same torch) or on the device for the large configurations.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class Projection:
    name: str
    rows: int
    cols: int
    keep: float


# Llama-3-8B: q, o 4096x4096; k, v 1024x4096 (GQA, 8 KV heads); gate, up 14336x4096; down 4096x14336.
LLAMA3_8B = (
    Projection("q", 4096, 4096, 33), Projection("k", 1024, 4096, 33), Projection("v", 1024, 4096, 33),
    Projection("o", 4096, 4096, 33), Projection("gate", 14336, 4096, 36), Projection("up", 14336, 4096, 36),
    Projection("down", 4096, 14336, 36),
)

# Qwen2.5-32B: hidden 5120, intermediate 27648, 40 query / 8 KV heads of 128.
QWEN25_32B = (
    Projection("q", 5120, 5120, 40), Projection("k", 1024, 5120, 40), Projection("v", 1024, 5120, 40),
    Projection("o", 5120, 5120, 40), Projection("gate", 27648, 5120, 40), Projection("up", 27648, 5120, 40),
    Projection("down", 5120, 27648, 40),
)


def channel_scale(cols: int, generator: torch.Generator, device="cpu") -> torch.Tensor:
    """lognormal(0, 1) per input channel."""
    return torch.exp(torch.randn(cols, generator=generator, device=device))


@dataclass
class Config1:
    """CPU-runnable single projection: W [2048, 2048] fp32 ~ N(0, 0.02), keep 40, a 17-token forward batch, calibration
    from 128 x 512 tokens in 16 calls of 4096 tokens; seed 0."""
    w: torch.Tensor
    scale: torch.Tensor
    x: torch.Tensor
    seed: int
    keep: float = 40.0
    calib_tokens: int = 128 * 512
    calib_call: int = 4096

    def calib_chunks(self, device="cpu"):
        """The calibration activations, one hook call at a time."""
        g = torch.Generator().manual_seed(self.seed + 1)
        for _ in range(self.calib_tokens // self.calib_call):
            yield (torch.randn(self.calib_call, self.w.shape[1], generator=g) * self.scale).to(device)


def config1(seed: int = 0, rows: int = 2048, cols: int = 2048, tokens: int = 17) -> Config1:
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(rows, cols, generator=g) * 0.02
    scale = channel_scale(cols, g)
    x = torch.randn(tokens, cols, generator=g) * scale
    return Config1(w=w, scale=scale, x=x, seed=seed)


def projection_weights(p: Projection, seed: int, device, dtype=torch.bfloat16) -> torch.Tensor:
    """W [rows, cols] ~ N(0, 0.02) in dtype, generated on `device`."""
    g = torch.Generator(device=device).manual_seed(seed)
    return (torch.randn(p.rows, p.cols, generator=g, device=device) * 0.02).to(dtype)


def activations(cols: int, tokens: int, seed: int, device, dtype=torch.bfloat16, scale=None) -> torch.Tensor:
    """x [tokens, cols] ~ N(0, 1) times a per-channel lognormal scale (its own, from `seed`, unless given)."""
    g = torch.Generator(device=device).manual_seed(seed)
    if scale is None:
        scale = channel_scale(cols, g, device)
    return (torch.randn(tokens, cols, generator=g, device=device) * scale).to(dtype)


def selection_case(p: Projection, index: int, calib_tokens: int = 4096):
    """(w [rows, cols] bf16 ~ N(0, 0.02), calibration activations [calib_tokens, cols] bf16, lognormal-scaled) of one
    projection of the full-size selection check, from the CPU generator, so the reference's selection computed on one
    machine and this package's on another see the same inputs."""
    g = torch.Generator().manual_seed(7000 + index)
    w = (torch.randn(p.rows, p.cols, generator=g) * 0.02).bfloat16()
    scale = channel_scale(p.cols, g)
    x = (torch.randn(calib_tokens, p.cols, generator=g) * scale).bfloat16()
    return w, x


def calibrate(cols: int, generator: torch.Generator, scale: torch.Tensor, calib_tokens: int, device, calls: int = 16):
    """The benchmark's calibration of one projection input: calib_tokens lognormal-scaled bf16 tokens drawn from
    `generator` on `device`, reduced by the package's calibration kernel in `calls` hook calls. Returns (sums fp64
    [cols], the kernel's milliseconds, the bytes it read)."""
    from . import kernels
    sums = torch.zeros(cols, dtype=torch.float64, device=device)
    chunk = max(1, calib_tokens // calls)
    ms, nbytes = 0.0, 0
    for _ in range(max(1, calib_tokens // chunk)):
        xc = (torch.randn(chunk, cols, generator=generator, device=device) * scale).bfloat16()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        kernels.sumsq_cols(xc, sums)
        b.record()
        b.synchronize()
        ms += a.elapsed_time(b)
        nbytes += xc.numel() * 2
        del xc
    return sums, ms, nbytes


# The benchmark layer's linear modules as SGLang holds them (fused q/k/v and gate/up), the input each reads, and the
# projections they hold.
LAYER_MODULES = {"qkv_proj": ("attn_in", ("q", "k", "v")), "o_proj": ("attn_out", ("o",)),
                 "gate_up_proj": ("mlp_in", ("gate", "up")), "down_proj": ("mlp_mid", ("down",))}


def layer_seeds(seed: int, projections=LLAMA3_8B) -> dict:
    """{module: (calibration generator seed, {projection name: weight seed})} of the benchmark layer of rank seed."""
    names = [p.name for p in projections]
    return {module: (seed * 1000 + gi, {n: seed * 1000 + 17 * (names.index(n) + 1) for n in proj})
            for gi, (module, (_, proj)) in enumerate(LAYER_MODULES.items())}


# ---- config 5: a layer-parallel plan on a Qwen2.5-32B-shaped model ----------------------------------------------------

CFG5_LAYERS = 64
CFG5_GROUPS = [[2 * s, 2 * s + 1] for s in range(CFG5_LAYERS // 2)]     # 32 pair-steps, each with a keep-40 replica


def rms_norm(h: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """h / rms(h) per row, in fp32, back in h's dtype (unit norm weights)."""
    hf = h.float()
    return (hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + eps)).to(h.dtype)


class DecoderBlock:
    """A Qwen2.5-32B-shaped decoder layer as a function of the hidden state h [T, hidden]: RMSNorm, q/k/v, causal
    attention of the pass's own tokens (GQA: 40 query heads over 8 KV heads of 128; no KV cache of earlier tokens and no
    rotary embedding -- this package has neither), o, residual; RMSNorm, SiLU(gate) * up, down, residual. Each of the
    four linear modules (qkv, o, gate_up, down) is a callable x -> y: a dense bf16 weight (torch linear) for an exact
    layer, a compact.Compact for a replica. A module "gated" in place of "gate_up" returns SiLU(gate) * up itself
    (compact.GatedTiles: the activation in the GEMM's epilogue)."""

    def __init__(self, modules: dict, heads: int = 40, kv_heads: int = 8, head_dim: int = 128):
        self.m = modules
        self.heads, self.kv_heads, self.d = heads, kv_heads, head_dim

    def __call__(self, h: torch.Tensor) -> torch.Tensor:
        import torch.nn.functional as F
        T = h.shape[0]
        qkv = self.m["qkv"](rms_norm(h))
        q, k, v = qkv.split([self.heads * self.d, self.kv_heads * self.d, self.kv_heads * self.d], dim=-1)
        q = q.view(T, self.heads, self.d).transpose(0, 1).unsqueeze(0)
        k = k.reshape(T, self.kv_heads, self.d).transpose(0, 1).unsqueeze(0)
        v = v.reshape(T, self.kv_heads, self.d).transpose(0, 1).unsqueeze(0)
        a = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
        h = h + self.m["o"](a.squeeze(0).transpose(0, 1).reshape(T, self.heads * self.d))
        if "gated" in self.m:
            return h + self.m["down"](self.m["gated"](rms_norm(h)))
        gu = self.m["gate_up"](rms_norm(h))
        gate, up = gu.chunk(2, dim=-1)
        return h + self.m["down"]((F.silu(gate.float()) * up.float()).to(h.dtype))


CFG5_MODULES = {"qkv": ("q", "k", "v"), "o": ("o",), "gate_up": ("gate", "up"), "down": ("down",)}


def cfg5_weights(layer: int, device, seed: int = 5, projections=QWEN25_32B) -> dict:
    """{projection name: W [rows, cols] bf16 ~ N(0, 0.02)} of layer `layer` of the config-5 model, from its own seeds."""
    return {p.name: projection_weights(p, seed * 100_000 + layer * 100 + i, device)
            for i, p in enumerate(projections)}


def cfg5_norms(layer: int, device, seed: int = 5, projections=QWEN25_32B) -> dict:
    """{module: input-channel norms} that a layer's replica is selected with: a lognormal(0, 1) scale per channel
    (the synthetic activations' spread), in place of calibration sums."""
    by = {p.name: p for p in projections}
    g = torch.Generator(device=device).manual_seed(seed * 100_000 + layer * 100 + 99)
    return {m: channel_scale(by[names[0]].cols, g, device) for m, names in CFG5_MODULES.items()}


def cfg5_exact(layer: int, device, seed: int = 5) -> DecoderBlock:
    """Layer `layer` of the config-5 model with dense bf16 projections (fused qkv and gate_up weights)."""
    import torch.nn.functional as F
    w = cfg5_weights(layer, device, seed)
    mods = {}
    for m, names in CFG5_MODULES.items():
        W = torch.cat([w.pop(n) for n in names]) if len(names) > 1 else w.pop(names[0])
        mods[m] = (lambda W: lambda x: F.linear(x, W))(W)
    return DecoderBlock(mods)


def cfg5_replica(layer: int, device, seed: int = 5, layout: str | None = None) -> tuple:
    """(the keep-40 replica of layer `layer` as a DecoderBlock over compact.Compact modules, its weight bytes): every
    projection pruned by the Wanda selection on the GPU, the dense weights dropped. In the tensor-core layout the gate
    and up projections form one compact.GatedTiles (SiLU * up in the GEMM's epilogue)."""
    from . import compact, wanda
    norms = cfg5_norms(layer, device, seed)
    keep = {p.name: p.keep for p in QWEN25_32B}
    mods, nbytes = {}, 0
    w = cfg5_weights(layer, device, seed)
    for m, names in CFG5_MODULES.items():
        blocks = []
        for n in names:
            values, idx = wanda.select(w.pop(n), keep[n], norms[m])
            blocks.append(("compact", values, idx, QWEN25_32B_COLS[n]))
        if m == "gate_up" and (layout or compact.DEFAULT_LAYOUT) == "tc":
            gt = compact.GatedTiles(blocks)
            nbytes += gt.nbytes()
            mods["gated"] = gt
            continue
        c = compact.Compact.__new__(compact.Compact)
        c.tiles = compact.Tiles(blocks, layout=layout)
        nbytes += c.nbytes()
        mods[m] = (lambda c: lambda x: c.apply(None, x))(c)
    return DecoderBlock(mods), nbytes


QWEN25_32B_COLS = {p.name: p.cols for p in QWEN25_32B}


def cfg5_input(pass_index: int, tokens: int, device, seed: int = 5, hidden: int = 5120) -> torch.Tensor:
    """The hidden state entering the first step on pass `pass_index`: N(0, 1) rows, RMS-normalised, bf16."""
    g = torch.Generator(device=device).manual_seed(seed * 7919 + pass_index)
    return rms_norm(torch.randn(tokens, hidden, generator=g, device=device)).bfloat16()
