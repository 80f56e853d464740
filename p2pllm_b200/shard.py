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
    """One rank's share of a compact module: its rows as a Compact, and apply() returning the whole y on every rank
    (an all-gather of the ranks' row runs over the process group, NCCL on GPUs)."""

    def __init__(self, blocks: list, group=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.rows = sum(_rows(b) for b in blocks)
        self.ranges = row_ranges(self.rows, self.world)
        start, stop = self.ranges[self.rank]
        self.local = compact.Compact(shard_blocks(blocks, start, stop)) if stop > start else None
        self.width = max(b - a for a, b in self.ranges)

    def apply(self, layer, x: torch.Tensor, bias=None) -> torch.Tensor:
        x2 = x.reshape(-1, x.shape[-1])
        start, stop = self.ranges[self.rank]
        part = torch.zeros(x2.shape[0], self.width, dtype=x.dtype, device=x.device)
        if self.local is not None:
            part[:, :stop - start] = self.local.apply(None, x2)
        if self.world == 1:
            y = part[:, :self.rows]
        else:
            pieces = [torch.empty_like(part) for _ in range(self.world)]
            dist.all_gather(pieces, part, group=self.group)
            y = torch.cat([p[:, :b - a] for p, (a, b) in zip(pieces, self.ranges)], dim=1)
        if bias is not None:
            y = y + bias
        return y.reshape(*x.shape[:-1], self.rows)
