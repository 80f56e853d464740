"""Row sharding of a compact module over the GPUs of one node.

Wanda keeps the top-k of each output row on its own (p2p/wanda.py:83), so a module's rows split across ranks with no
exchange at selection time: every rank holds a contiguous run of whole 128-row tiles (the GEMM's unit) and the full x,
computes its rows of y, and one all-gather over NCCL (NVLink) assembles y [T, rows] on every rank. Runs of rows are as
equal as whole tiles allow, earlier ranks taking the extra tile.

    row_ranges(rows, world)          [(start, stop)] per rank
    shard_blocks(blocks, start, stop)  the part of a module's block list covering rows [start, stop)
    ShardedCompact                   a rank's Compact over its rows, with the all-gather of y
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import compact

TILE_ROWS = 128


def row_ranges(rows: int, world: int) -> list:
    """[(start, stop)] of each rank: whole 128-row tiles, as even as they divide, the remainder to the first ranks; the
    last range ends at `rows`. Ranks past the tiles get empty ranges."""
    if rows < 0 or world < 1:
        raise ValueError(f"row_ranges: rows {rows}, world {world}")
    tiles = -(-rows // TILE_ROWS)
    base, extra = divmod(tiles, world)
    out, t = [], 0
    for r in range(world):
        n = base + (1 if r < extra else 0)
        out.append((min(t * TILE_ROWS, rows), min((t + n) * TILE_ROWS, rows)))
        t += n
    return out


def _rows(block: tuple) -> int:
    return block[1].shape[-2]


def _take(block: tuple, a: int, b: int) -> tuple:
    if block[0] == "dense":
        return ("dense", block[1][..., a:b, :])
    kind, values, meta, cols = block
    return (kind, values[..., a:b, :], meta[..., a:b, :], cols)


def shard_blocks(blocks: list, start: int, stop: int) -> list:
    """The blocks (a module's block list, in row order) cut to rows [start, stop) of the whole module."""
    out, r0 = [], 0
    for b in blocks:
        n = _rows(b)
        a, z = max(start, r0), min(stop, r0 + n)
        if a < z:
            out.append(_take(b, a - r0, z - r0))
        r0 += n
    return out


class ShardedCompact:
    """One rank's share of a compact module: its rows as a Compact, and apply() returning the whole y on every rank.
    The rank's GEMM writes its rows straight into its slot of the all-gather buffer; one all_gather_into_tensor over the
    process group (NCCL on GPUs) collects every rank's slot, and the slots are laid side by side into y [T, rows]."""

    def __init__(self, blocks: list, group=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.rows = sum(_rows(b) for b in blocks)
        self.ranges = row_ranges(self.rows, self.world)
        start, stop = self.ranges[self.rank]
        self.local = compact.Compact(shard_blocks(blocks, start, stop)) if stop > start else None
        self.width = max(b - a for a, b in self.ranges)
        self.mine = stop - start

    def local_part(self, x2: torch.Tensor, part: torch.Tensor) -> torch.Tensor:
        """This rank's rows of y into part [T, width] (columns past its rows zeroed)."""
        if self.local is not None:
            self.local.tiles(x2, out=part[:, :self.mine])
        if self.mine < self.width:
            part[:, self.mine:].zero_()
        return part

    def gather(self, part: torch.Tensor) -> torch.Tensor:
        """y [T, rows] from every rank's part."""
        if self.world == 1:
            return part[:, :self.rows]
        T = part.shape[0]
        slots = torch.empty(self.world * T, self.width, dtype=part.dtype, device=part.device)
        dist.all_gather_into_tensor(slots, part.contiguous(), group=self.group)
        slots = slots.view(self.world, T, self.width)
        if all(b - a == self.width for a, b in self.ranges):
            return slots.permute(1, 0, 2).reshape(T, self.world * self.width)
        return torch.cat([slots[r, :, :b - a] for r, (a, b) in enumerate(self.ranges)], dim=1)

    def apply(self, layer, x: torch.Tensor, bias=None) -> torch.Tensor:
        x2 = x.reshape(-1, x.shape[-1])
        part = torch.empty(x2.shape[0], self.width, dtype=x.dtype, device=x.device)
        y = self.gather(self.local_part(x2, part))
        if bias is not None:
            y = y + bias
        return y.reshape(*x.shape[:-1], self.rows)
