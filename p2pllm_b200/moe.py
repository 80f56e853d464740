"""Routed experts run compact: a FusedMoE quant_method that multiplies the experts' pruned weights where they lie,
instead of expanding every used expert to dense on every pass (p2p/compact.py:227-262, CompactMoE).

    ExpertTiles   one routed-expert tensor (row blocks with a leading expert dimension) in one tensor-core layout,
                  each expert starting on a 128-row tile
    GroupedMoE    quant_method.apply(layer, dispatch_output): gated-SiLU experts (w13 = gate then up, w2 = down)

A pass: one kernel (p2p_moe_route) sorts the routed (token, slot) pairs by expert (stable) and writes the grouped
GEMM's items; x's rows are gathered in that order; one grouped launch of the compact GEMM (p2p_spmm_tc_grouped_gated:
a CTA takes one row tile of one expert's run of up to 256 tokens, the expert's gate and up rows interleaved 64 and 64
so that its epilogue writes SiLU(gate) * up, in fp32 from the rounded outputs, rounded to x's dtype); a second grouped
launch gives down; p2p_moe_combine weights each token's outputs by its routing
weights and adds them in slot order in fp32 (deterministic). Three numbers (pairs, items, the largest item) are read
back once a pass to size the launches (the reference's CompactMoE also syncs, on torch.unique).
"""
from __future__ import annotations

import torch

from . import kernels
from ._lib import P2PError, call, dtype_code, ptr, require_cuda, stream_of
from .compact import _cols, gate_up_rows, to_compact

ITEM_TOKENS = 256                       # tokens one grouped CTA takes (an accumulator of at most 256 columns)


class ExpertTiles:
    """A routed-expert tensor [E, rows, cols] from its row blocks (each ("dense", W [E, r, C]) or ("sparse" |
    "compact", values [E, r, k], words | idx [E, r, ...], C), in row order), laid out for the grouped GEMM: expert
    e's rows start at row tile e * item_row_tiles. Built once at load (one layout build an expert)."""

    def __init__(self, blocks: list, gated: bool = False):
        self.gated = gated
        if gated:                               # gate rows then up rows, interleaved: one compact (or dense) block
            values, idx = gate_up_rows(blocks)
            blocks = [("compact", values, idx, _cols(blocks[0])) if idx is not None else ("dense", values)]
        blocks = [to_compact(b) for b in blocks]
        self.cols = _cols(blocks[0])
        self.experts = blocks[0][1].shape[0]
        self.rows = sum(b[1].shape[-2] for b in blocks)
        self.dtype, self.device = blocks[0][1].dtype, blocks[0][1].device
        if self.dtype not in (torch.bfloat16, torch.float16) or self.cols % 8:
            raise P2PError("grouped experts need bf16 / f16 weights with columns in multiples of 8")
        self.item_row_tiles = -(-self.rows // 128)
        words, segs, base = [], [], 0
        for e in range(self.experts):
            row_blocks, row0 = [], 0
            for b in blocks:
                v = b[1][e].contiguous()
                idx = b[2][e].contiguous() if b[0] == "compact" else None
                row_blocks.append((row0, v, idx))
                row0 += v.shape[0]
            w, seg, _ = kernels.tiles_build(row_blocks, self.cols)
            total = int(seg[-1].item())
            words.append(w[:total])
            segs.append(seg[:-1] + base)
            base += total
        self.words = torch.cat(words) if base else torch.zeros(4, dtype=torch.int32, device=self.device)
        self.seg = torch.cat(segs + [torch.tensor([base], dtype=torch.int64, device=self.device)])
        self.seg_cap = int((self.seg[1:] - self.seg[:-1]).max().item())
        self.layout_row_tiles = self.experts * self.item_row_tiles

    def __call__(self, x: torch.Tensor, items: torch.Tensor, max_tokens: int, out: torch.Tensor) -> torch.Tensor:
        """out [P, rows] rows s.. of an item = x rows s.. times the item's expert (items: int32 [n, 4] on the GPU);
        gated: out [P, rows / 2] = dtype(silu(gate) * up) of them, applied in the GEMM's epilogue."""
        call("p2p_spmm_tc_grouped_gated" if self.gated else "p2p_spmm_tc_grouped", ptr(x), dtype_code(x), x.shape[0], self.cols, x.stride(0), ptr(self.words),
             ptr(self.seg), self.layout_row_tiles, self.rows, self.item_row_tiles, self.seg_cap, ptr(items),
             items.shape[0], max_tokens, ptr(out), out.stride(0), stream_of(x))
        if kernels.CHECK_WAITS:
            kernels.spmm_tc_status(x.device)
        return out

    def gated_sums(self, x: torch.Tensor, items: torch.Tensor, max_tokens: int, out: torch.Tensor) -> torch.Tensor:
        """out [n_items, rows / 2] fp32: per item, the column sums over its tokens of (silu(g) * u)^2, g and u this
        gated layout's unrounded products (p2p_spmm_tc_grouped_gated_sums)."""
        if not self.gated:
            raise P2PError("gated sums need the interleaved gate / up layout")
        call("p2p_spmm_tc_grouped_gated_sums", ptr(x), dtype_code(x), x.shape[0], self.cols, x.stride(0),
             ptr(self.words), ptr(self.seg), self.layout_row_tiles, self.rows, self.item_row_tiles, self.seg_cap,
             ptr(items), items.shape[0], max_tokens, ptr(out), out.stride(0), stream_of(x))
        return out

    def nbytes(self) -> int:
        return self.words.numel() * 4 + self.seg.numel() * 8


def route(ids: torch.Tensor, experts: int) -> dict:
    """The pass's routing on the GPU (p2p_moe_route): order [P] (pairs sorted by expert, stable), where [T K] (each
    pair's place, -1 if routed nowhere), counts [E], items [n, 4] ({expert, first place, places, 0}), and on the host
    P, the item count and the largest item."""
    require_cuda(ids)
    flat = ids.reshape(-1).to(torch.int64).contiguous()
    n = flat.numel()
    dev = flat.device
    max_items = -(-n // ITEM_TOKENS) + experts
    order = torch.empty(max(n, 1), dtype=torch.int64, device=dev)
    where = torch.empty(max(n, 1), dtype=torch.int64, device=dev)
    counts = torch.empty(experts, dtype=torch.int32, device=dev)
    items = torch.empty(max_items, 4, dtype=torch.int32, device=dev)
    meta = torch.empty(3, dtype=torch.int64, device=dev)
    call("p2p_moe_route", ptr(flat), n, experts, ptr(order), ptr(where), ptr(counts), ptr(items), max_items, ptr(meta),
         stream_of(flat))
    pairs, n_items, most = meta.tolist()
    return {"order": order[:pairs], "where": where[:n], "counts": counts, "items": items[:n_items], "most": most}


class GroupedMoE(torch.nn.Module):
    """A FusedMoE's quant_method for compact routed experts, gated SiLU: weights {"w13_weight": blocks of [E, 2R, H]
    (gate rows, then up rows), "w2_weight": blocks of [E, H, R]}. apply(layer, dispatch_output) returns the layer's
    output [T, H] in x's dtype. Other attributes are the layer's own method's."""

    def __init__(self, method, weights: dict):
        super().__init__()
        self.method = method
        two_r = sum(b[1].shape[-2] for b in weights["w13_weight"])
        # SiLU(gate) * up inside the gate/up launch when the rows allow it (R a multiple of 64, one k)
        try:
            self.w13 = ExpertTiles(weights["w13_weight"], gated=two_r % 128 == 0)
        except P2PError:
            self.w13 = ExpertTiles(weights["w13_weight"])
        self.w2 = ExpertTiles(weights["w2_weight"])
        if self.w13.rows % 2 or self.w2.cols != self.w13.rows // 2 or self.w2.rows != self.w13.cols:
            raise P2PError("w13 [E, 2R, H] and w2 [E, H, R] do not match")

    def __getattr__(self, name):
        try:
            return super().__getattr__(name)
        except AttributeError:
            return getattr(super().__getattr__("method"), name)

    def apply(self, layer, dispatch_output):
        x = dispatch_output.hidden_states
        topk = dispatch_output.topk_output
        ids, weights = topk.topk_ids, topk.topk_weights
        T, K = ids.shape
        x2 = x.reshape(-1, x.shape[-1])
        if x2.dtype != self.w13.dtype:
            raise P2PError(f"x is {x2.dtype}, the experts {self.w13.dtype}")
        r = route(ids, self.w13.experts)
        P = r["order"].numel()
        out = torch.empty(T, self.w2.rows, dtype=x2.dtype, device=x.device)
        if P == 0:
            return out.zero_().reshape(*x.shape[:-1], self.w2.rows)
        xs = x2.index_select(0, r["order"] // K).contiguous()
        R = self.w13.rows // 2
        if self.w13.gated:
            h = self.w13(xs, r["items"], r["most"], torch.empty(P, R, dtype=x2.dtype, device=x.device))
        else:
            gu = self.w13(xs, r["items"], r["most"], torch.empty(P, self.w13.rows, dtype=x2.dtype, device=x.device))
            h = (torch.nn.functional.silu(gu[:, :R].float()) * gu[:, R:].float()).to(x2.dtype).contiguous()
        down = self.w2(h, r["items"], r["most"], torch.empty(P, self.w2.rows, dtype=x2.dtype, device=x.device))
        w = weights.reshape(-1).float().contiguous()
        call("p2p_moe_combine", ptr(down), dtype_code(down), down.stride(0), ptr(r["where"]), ptr(w), T, K,
             self.w2.rows, ptr(out), out.stride(0), stream_of(down))
        return out.reshape(*x.shape[:-1], self.w2.rows)

    def process_weights_after_loading(self, layer) -> None:
        pass

    def nbytes(self) -> int:
        return self.w13.nbytes() + self.w2.nbytes()
