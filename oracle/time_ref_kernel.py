"""Test infrastructure, not product: the reference's GPU kernel (p2p/compact.cu, built into oracle/_ref/ by
oracle/build_ref.py, driven by oracle/ref_tiles.py) timed beside this library's compact GEMM on the same replica
layer, the same selection and the same inputs, on one GPU.

The layer is the bench's: Llama-3-8B projections (q, k, v, o keep 33; gate, up, down keep 36) as SGLang fuses them
(qkv_proj, o_proj, gate_up_proj, down_proj), Wanda-selected on the GPU from synthetic calibration. Each side runs
its own public call per module (the reference: Tiles.__call__, p2p/compact.py:195-201, with its timed split choice;
this library: Compact.apply). A pass over the four modules moves about 310 MB of weights, more than the 126 MB L2, so
no pass finds the previous one's weights in cache. Each module's time is the median over passes of its CUDA-event
duration, with the pass queued ahead of the GPU (a spin kernel first) so that host launch cost is not counted on
either side. The two outputs are compared with each other and must agree within the bf16 tolerance (rel-L2 1e-2).

    python -m oracle.time_ref_kernel [--tokens 17 272] [--passes 30]
"""
from __future__ import annotations

import argparse
import json
import statistics

import torch

from oracle import build_ref, ref_tiles

MODULES = {"qkv_proj": ("q", "k", "v"), "o_proj": ("o",), "gate_up_proj": ("gate", "up"), "down_proj": ("down",)}
# A spin of a few milliseconds queued ahead of each timed pass: the host enqueues the pass's launches while the GPU
# spins, so each module's events measure the GPU's time for it, not the host's time to issue it.
HEAD_START_CYCLES = 8_000_000


def words_of(idx: torch.Tensor, cols: int) -> torch.Tensor:
    """The reference's mask words (p2p/compact.py:36-45: bit c % 32 of word c // 32, int32 two's complement)."""
    n_words = -(-cols // 32)
    mask = torch.zeros(idx.shape[0], n_words * 32, dtype=torch.int64, device=idx.device)
    mask.scatter_(1, idx.long(), 1)
    w = (mask.view(idx.shape[0], n_words, 32) << torch.arange(32, device=idx.device)).sum(-1)
    return torch.where(w >= 2 ** 31, w - 2 ** 32, w).to(torch.int32)


def layer(seed: int, device) -> dict:
    from p2pllm_b200 import kernels, wanda, workloads
    proj = {p.name: p for p in workloads.LLAMA3_8B}
    out = {}
    for gi, (module, names) in enumerate(MODULES.items()):
        cols = proj[names[0]].cols
        g = torch.Generator(device=device).manual_seed(seed * 1000 + gi)
        scale = workloads.channel_scale(cols, g, device)
        sums = torch.zeros(cols, dtype=torch.float64, device=device)
        for _ in range(4):
            kernels.sumsq_cols((torch.randn(16384, cols, generator=g, device=device) * scale).bfloat16(), sums)
        norms = kernels.channel_norms(sums)
        blocks = []
        for n in names:
            p = proj[n]
            w = workloads.projection_weights(p, seed * 1000 + 17 * (list(proj).index(n) + 1), device)
            values, idx = wanda.select(w, p.keep, norms)
            blocks.append((values, idx, cols))
        out[module] = (blocks, scale)
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, nargs="+", default=[17, 272])
    ap.add_argument("--passes", type=int, default=30)
    args = ap.parse_args()
    from p2pllm_b200 import compact
    dev = torch.device("cuda", 0)
    ext = build_ref.load_module()
    lay = layer(0, dev)
    ours, refs, nbytes = {}, {}, {}
    for module, (blocks, _) in lay.items():
        ours[module] = compact.Compact([("compact", v, i, c) for v, i, c in blocks])
        refs[module] = ref_tiles.RefTiles([("sparse", v, words_of(i, c), c) for v, i, c in blocks], ext)
        nbytes[module] = sum(v.numel() * 4 for v, _, _ in blocks)
    g = torch.Generator(device=dev).manual_seed(5)
    report = {}
    for tokens in args.tokens:
        xs = {m: (torch.randn(tokens, lay[m][0][0][2], generator=g, device=dev) * lay[m][1]).bfloat16() for m in lay}
        side = {"b200": lambda m, x: ours[m].apply(None, x), "reference": lambda m, x: refs[m](x)}
        times = {s: {m: [] for m in lay} for s in side}
        outs = {}
        for s, call in side.items():
            for m in lay:
                outs[s, m] = call(m, xs[m])                              # warm-up and the outputs compared below
            for _ in range(args.passes):
                evs = []
                torch.cuda._sleep(HEAD_START_CYCLES)           # the GPU waits while the host queues the whole pass
                for m in lay:
                    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    a.record()
                    call(m, xs[m])
                    b.record()
                    evs.append((m, a, b))
                torch.cuda.synchronize(dev)
                for m, a, b in evs:
                    times[s][m].append(a.elapsed_time(b) * 1e3)
        row = {}
        for m in lay:
            y0, y1 = outs["b200", m].double(), outs["reference", m].double()
            rel = float((y0 - y1).norm() / y1.norm())
            assert rel <= 1e-2, (m, tokens, rel)
            t0, t1 = statistics.median(times["b200"][m]), statistics.median(times["reference"][m])
            row[m] = {"b200_us": round(t0, 2), "reference_us": round(t1, 2), "speedup": round(t1 / t0, 2),
                      "weights_MB": round(nbytes[m] / 1e6, 1), "rel_l2": rel,
                      "reference_splits": refs[m].splits(min(tokens, 64))}
        lt0 = sum(r["b200_us"] for r in row.values())
        lt1 = sum(r["reference_us"] for r in row.values())
        row["layer"] = {"b200_us": round(lt0, 2), "reference_us": round(lt1, 2), "speedup": round(lt1 / lt0, 2),
                        "b200_tokens_per_s": round(tokens / lt0 * 1e6), "reference_tokens_per_s": round(tokens / lt1 * 1e6)}
        report[f"T={tokens}"] = row
        print(json.dumps({f"T={tokens}": row}), flush=True)


if __name__ == "__main__":
    main()
