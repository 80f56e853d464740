"""Pruned weights stored and multiplied compactly on B200: the operator API of p2p/compact.py.

A replica's projection keeps the same number k of weights in every row (Wanda). The reference stores each row's kept
values plus a 1-bit-per-weight mask and multiplies 8 x 8 pieces on mma.sync tensor cores; here each row keeps its
values plus their column indices (int16 while cols <= 32767), and the GEMM y[t, r] = sum_j v[r, j] * x[t, idx[r, j]]
runs as hand-written sm_100a kernels (libp2p_b200.so). The reference's block lists and mask words are accepted as they
are and converted on the GPU at load.

Block list (p2p/compact.py:88-97, prepare.py:201-203), in row order:
    ("dense", W [rows, cols])                                  kept whole
    ("sparse", values [rows, k], words [rows, ceil(cols/32)], cols)   the reference's packed form
    ("compact", values [rows, k], idx [rows, k], cols)          this package's form (values + column indices)
each with an optional leading expert dimension for routed experts.
"""
from __future__ import annotations

import os

import torch

from . import kernels
from ._lib import P2PError, idx_dtype

__all__ = ["pack", "unpack", "expand", "to_compact", "Tiles", "GatedTiles", "Compact", "CompactMoE"]

# The layout bf16 / f16 modules take unless asked otherwise: "tc" (values + positions, 4 bytes a kept weight, one
# 16-bit store a weight into a shared-memory tile) or "mask" (values + one bit a weight, the reference's storage,
# tiles rebuilt in registers into tensor memory). P2P_LAYOUT=tc|mask overrides it.
DEFAULT_LAYOUT = os.environ.get("P2P_LAYOUT", "tc")


def pack(w: torch.Tensor, mask: torch.Tensor) -> tuple:
    """(values [rows, k], words [rows, ceil(cols / 32)] int32) of w where mask, which keeps the same k in every row.
    p2p/compact.py:36-45."""
    return kernels.pack_mask(w, mask)


def unpack(values: torch.Tensor, words: torch.Tensor, cols: int) -> torch.Tensor:
    """The dense matrix pack stored. p2p/compact.py:48-61 (its Triton kernel _unpack, 64-85, is replaced by a CUDA one)."""
    return kernels.unpack(values, cols, words=words)


def _cols(block: tuple) -> int:
    return block[3] if block[0] in ("sparse", "compact") else block[1].shape[-1]


def expand(block: tuple, experts=None) -> torch.Tensor:
    """A stored row block as a dense matrix, each with a leading expert dimension for routed experts; of those, only
    `experts` (ids), if given. p2p/compact.py:88-97."""
    if block[0] == "dense":
        return block[1] if experts is None else block[1][experts]
    kind, values, meta, cols = block
    if experts is not None:
        values, meta = values[experts], meta[experts]
    lead = values.shape[:-1]
    v2 = values.reshape(-1, values.shape[-1])
    m2 = meta.reshape(-1, meta.shape[-1])
    dense = kernels.unpack(v2, cols, words=m2) if kind == "sparse" else kernels.unpack(v2, cols, idx=m2)
    return dense.view(*lead, cols)


def to_compact(block: tuple) -> tuple:
    """A block as ("dense", W) or ("compact", values, idx, cols): mask words become column indices (on the GPU,
    checking that every row keeps k); column indices are range-checked once here, so the GEMMs need not."""
    if block[0] == "dense":
        return block
    kind, values, meta, cols = block
    if kind == "sparse":
        k = values.shape[-1]
        idx = kernels.words_to_idx(meta.reshape(-1, meta.shape[-1]), cols, k).view(*values.shape[:-1], k)
        return ("compact", values, idx, cols)
    if kind == "compact":
        kernels.check_idx(meta, cols)
        return block
    raise P2PError(f"unknown block kind {kind!r}")


def _nbytes(blocks) -> int:
    return sum(t.numel() * t.element_size() for b in blocks for t in b[1:] if torch.is_tensor(t))


class Tiles:
    """A module's row blocks on the GPU, as the compact GEMM reads them; calling it multiplies tokens by them.
    The B200 counterpart of p2p/compact.py:113-202 (Tiles). bf16 / f16 modules whose columns are a multiple of 8 are
    re-laid once into (128-row x 64-column) segments of packed (value, row, column) words and multiplied on tcgen05
    tensor cores; fp32 modules (and others) keep rows of values + column indices for the CUDA-core kernel."""

    @staticmethod
    def usable(blocks: list) -> bool:
        """CUDA tensors of bf16, f16 or f32, 2-D blocks (p2p/compact.py:117-122 asks for the same, less fp32, plus
        columns in multiples of 8, which only the tensor-core layout needs)."""
        t = blocks[0][1]
        return t.is_cuda and t.dtype in (torch.bfloat16, torch.float16, torch.float32) and t.dim() == 2

    def __init__(self, blocks: list, layout: str | None = None):
        if not blocks:
            raise P2PError("a module needs at least one row block")
        blocks = [to_compact(b) for b in blocks]
        self.cols = _cols(blocks[0])
        self.dtype = blocks[0][1].dtype
        self.device = blocks[0][1].device
        rows_blocks, row0 = [], 0
        kinds = set()
        for b in blocks:
            if _cols(b) != self.cols:
                raise P2PError("every block of a module has the same columns")
            if b[1].dtype != self.dtype or b[1].dim() != 2:
                raise P2PError("blocks share one dtype and are 2-D")
            values = b[1].contiguous()
            idx = b[2].contiguous() if b[0] == "compact" else None
            if idx is not None:
                kinds.add(idx.dtype)
            rows_blocks.append((row0, values, idx))
            row0 += values.shape[0]
        if len(kinds) > 1:                        # one index width for the whole module
            want = idx_dtype(self.cols)
            rows_blocks = [(r, v, None if i is None else i.to(want)) for r, v, i in rows_blocks]
        self.rows = row0
        tc_ok = self.dtype in (torch.bfloat16, torch.float16) and self.cols % 8 == 0
        self.layout = layout or (DEFAULT_LAYOUT if tc_ok else "rows")
        if self.layout in ("tc", "mask") and not tc_ok:
            raise P2PError("the tensor-core layouts hold bf16 / f16 modules with columns in multiples of 8")
        if self.layout == "tc":
            self.words, self.seg, self.seg_cap = kernels.tiles_build(rows_blocks, self.cols)
            self.blocks = None
        elif self.layout == "mask":
            self.data, self.seg = kernels.mask_build(rows_blocks, self.cols)
            self.blocks = None
        elif self.layout == "rows":
            self.blocks = rows_blocks
        else:
            raise P2PError(f"unknown layout {self.layout!r}")

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """x [T, cols] @ W.T: [T, rows]. Any T (the reference launches at most 64 tokens at a time)."""
        if x.dtype != self.dtype:
            raise P2PError(f"x is {x.dtype}, the weights {self.dtype}")
        if self.layout == "mask":
            return kernels.spmm_mask(x, self.data, self.seg, self.rows, self.cols, out=out)
        if self.layout == "tc":
            return kernels.spmm_tc(x, self.words, self.seg, self.rows, self.cols, self.seg_cap, out=out)
        return kernels.spmm_rows(x, self.blocks, self.cols, self.rows, out=out)

    def nbytes(self) -> int:
        if self.layout == "mask":
            return self.data.numel() + self.seg.numel() * 8
        if self.layout == "tc":
            return self.words.numel() * 4 + self.seg.numel() * 8
        return sum(t.numel() * t.element_size() for _, v, i in self.blocks for t in (v, i) if t is not None)


def interleave_gate_up(t: torch.Tensor) -> torch.Tensor:
    """Rows [.., 2R, k] of a gated MLP's input projection (gate rows, then up rows) reordered so that every 128 rows
    hold 64 gate rows and the same 64 units' up rows: the layout of the gated GEMM."""
    r2, k = t.shape[-2], t.shape[-1]
    lead = t.shape[:-2]
    return t.reshape(*lead, 2, r2 // 128, 64, k).transpose(-4, -3).reshape(*lead, r2, k)


def gate_up_rows(blocks: list) -> tuple:
    """(values [.., 2R, k], idx [.., 2R, k] or None for dense rows) of a gate + up module's row blocks, in row order
    (all compact with one k, or all dense), interleaved for the gated GEMM. Raises if the blocks do not fit it."""
    blocks = [to_compact(b) for b in blocks]
    kinds = {b[0] for b in blocks}
    if len(kinds) != 1 or len({b[1].shape[-1] for b in blocks}) != 1:
        raise P2PError("a gated module's blocks are all compact with one k, or all dense")
    values = torch.cat([b[1] for b in blocks], dim=-2)
    idx = torch.cat([b[2] for b in blocks], dim=-2) if blocks[0][0] == "compact" else None
    if values.shape[-2] % 128 or values.dtype not in (torch.bfloat16, torch.float16) or _cols(blocks[0]) % 8:
        raise P2PError("a gated module needs bf16 / f16 rows, 2R with R a multiple of 64, columns in multiples of 8")
    return interleave_gate_up(values).contiguous(), None if idx is None else interleave_gate_up(idx).contiguous()


class GatedTiles:
    """A gated MLP's gate and up projections as one tensor-core module whose GEMM also applies the gate: calling it on
    x [T, cols] returns dtype(silu(g) * u) [T, R], g and u being the projections' outputs rounded to the model dtype
    -- what SGLang's SiluAndMul makes of the gate_up projection's output, without writing it (p2p/compact.py:205-224
    multiplies the two projections; the activation is the model's own). Blocks: the gate rows, then the up rows."""

    def __init__(self, blocks: list):
        values, idx = gate_up_rows(blocks)
        self.cols = _cols(to_compact(blocks[0]))
        self.dtype, self.device = values.dtype, values.device
        self.layout_rows = values.shape[-2]
        self.rows = self.layout_rows // 2
        self.layout = "tc"
        self.words, self.seg, self.seg_cap = kernels.tiles_build([(0, values, idx)], self.cols)

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        if x.dtype != self.dtype:
            raise P2PError(f"x is {x.dtype}, the weights {self.dtype}")
        return kernels.spmm_tc_gated(x, self.words, self.seg, self.layout_rows, self.cols, self.seg_cap, out=out)

    def nbytes(self) -> int:
        return self.words.numel() * 4 + self.seg.numel() * 8


class Compact:
    """A linear module's quant_method for a replica: its row blocks as Tiles. SGLang's linear layers call
    quant_method.apply(layer, x, bias). p2p/compact.py:205-224."""

    def __init__(self, blocks: list):
        assert Tiles.usable(blocks), ("a compact replica needs CUDA tensors of bfloat16, float16 or float32 and "
                                      "libp2p_b200.so")
        self.tiles = Tiles(blocks)

    def apply(self, layer, x: torch.Tensor, bias=None) -> torch.Tensor:
        out = self.tiles(x.reshape(-1, x.shape[-1]))
        if bias is not None:
            out = out + bias
        return out.reshape(*x.shape[:-1], out.shape[-1])

    def process_weights_after_loading(self, layer) -> None:
        pass

    def nbytes(self) -> int:
        return self.tiles.nbytes()


class CompactMoE(torch.nn.Module):
    """A FusedMoE's quant_method for compact routed experts ({weight name: row blocks with a leading expert
    dimension}): each pass expands only the experts in use, and the layer's own method runs them.
    p2p/compact.py:227-262, with the expansion on this package's CUDA kernel instead of Triton."""

    def __init__(self, method, weights: dict):
        super().__init__()
        self.method, self.weights = method, weights

    def __getattr__(self, name):
        try:
            return super().__getattr__(name)
        except AttributeError:
            return getattr(super().__getattr__("method"), name)

    def apply(self, layer, dispatch_output):
        topk = dispatch_output.topk_output
        ids = topk.topk_ids
        used = torch.unique(ids[ids >= 0])                     # sorted ids of the experts this pass reaches
        # Each routed id becomes its position among the used experts; -1 (no expert) stays -1.
        local = torch.searchsorted(used, ids.clamp(min=0)).to(ids.dtype)
        local = torch.where(ids >= 0, local, ids)
        swapped = {name: torch.nn.Parameter(torch.cat([expand(b, used) for b in blocks], dim=-2), requires_grad=False)
                   for name, blocks in self.weights.items()}
        saved = {name: layer._parameters[name] for name in swapped}
        layer._parameters.update(swapped)
        try:
            routed = dispatch_output._replace(topk_output=topk._replace(topk_ids=local))
            return self.method.apply(layer, routed)
        finally:
            layer._parameters.update(saved)              # the layer's own (empty) weights are back

    def process_weights_after_loading(self, layer) -> None:
        pass

    def nbytes(self) -> int:
        return sum(_nbytes(blocks) for blocks in self.weights.values())
