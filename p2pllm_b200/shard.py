"""Row sharding of a compact module over the GPUs of one node.

Wanda keeps the top-k of each output row on its own (p2p/wanda.py:83), so a module's rows split across ranks with no
exchange at selection time: every rank holds a contiguous run of whole 128-row tiles (the GEMM's unit) and the full x,
computes its rows of y, and y [T, rows] is assembled on every rank. Runs of rows are as equal as whole tiles allow,
earlier ranks taking the extra tile.

Two ways to assemble y:
  fused (the default on GPUs of one node): the rank's tensor-core GEMM writes its rows of y into its own y buffer and
      a push kernel (p2p_peer_push, all SMs, 16-byte stores) writes them into every other rank's -- or, push=False,
      the GEMM's epilogue stores each value straight into every rank's y buffer; y buffers in symmetric memory, plain
      stores over NVLink, then a bounded peer barrier (PeerGroup) makes them visible: no NCCL call, no copy engine;
  "nccl": the rank's GEMM writes its slot of a gather buffer, one NCCL all_gather_into_tensor collects the slots.

    row_ranges(rows, world)          [(start, stop)] per rank
    shard_blocks(blocks, start, stop)  the part of a module's block list covering rows [start, stop)
    PeerGroup                        flag arrays in peer memory and the barrier over them
    ShardedCompact                   a rank's Compact over its rows, with y assembled on every rank
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib, compact, kernels
from ._lib import P2PError

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


def _cols(block: tuple) -> int:
    return block[3] if block[0] in ("sparse", "compact") else block[1].shape[-1]


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


def _symmetric(shape, dtype, device, group):
    """A tensor in symmetric memory and the device addresses of every rank's copy of it (ctypes array, rank order)."""
    import torch.distributed._symmetric_memory as symm_mem
    t = symm_mem.empty(*shape, dtype=dtype, device=device)
    handle = symm_mem.rendezvous(t, group if group is not None else dist.group.WORLD)
    ptrs = list(handle.buffer_ptrs)
    return t, (ctypes.c_void_p * len(ptrs))(*ptrs)


class PeerGroup:
    """Flag arrays in peer memory (one per rank, 8 slots each) and the barrier over them (p2p_peer_barrier): after
    barrier(), every store the ranks' streams made before it is visible on every rank. Created by all ranks together."""

    def __init__(self, group=None, device=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.flags, self.ptrs = _symmetric((8,), torch.int32, self.device, group)
        self.flags.zero_()
        torch.cuda.synchronize(self.device)
        dist.barrier(group)                         # every rank's flags are zero before the first barrier
        self.epoch = 0

    def barrier(self, timeout_us: int = 5_000_000) -> None:
        self.epoch += 1
        _lib.call("p2p_peer_barrier", self.ptrs, self.world, self.rank, self.epoch, timeout_us,
                  torch.cuda.current_stream(self.device).cuda_stream)

    def status(self) -> None:
        """Raises if a barrier gave up waiting for a rank. Syncs."""
        _lib.call("p2p_peer_status", 1, torch.cuda.current_stream(self.device).cuda_stream)


class ShardedCompact:
    """One rank's share of a compact module: its rows as a Compact, and apply() returning the whole y on every rank.

    fused (the default with more than one rank): the rank's GEMM (the tensor-core layout `layout`, the package's
    default unless given) writes its rows of y into its own y buffer and a push kernel stores them into every other
    rank's over NVLink (push=False: the GEMM's epilogue stores them into every rank's), then a peer barrier; y is a view of one of two symmetric buffers, used in turn, so it
    stays valid until this module's next-but-one apply. Otherwise ("nccl"): the GEMM writes its slot of a gather
    buffer, and one all_gather_into_tensor over the process group collects the slots into y."""

    def __init__(self, blocks: list, group=None, fused: bool | None = None, peers: PeerGroup | None = None,
                 layout: str | None = None, push: bool | None = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.rows = sum(_rows(b) for b in blocks)
        self.cols = _cols(blocks[0])
        self.ranges = row_ranges(self.rows, self.world)
        start, stop = self.ranges[self.rank]
        self.fused = (self.world > 1) if fused is None else fused
        mine = shard_blocks(blocks, start, stop)
        self.local = None
        if stop > start:
            self.local = compact.Compact.__new__(compact.Compact)
            self.local.tiles = compact.Tiles(mine, layout=layout)
        self.width = max(b - a for a, b in self.ranges)
        self.mine = stop - start
        self.peers = peers
        # fused: by default the GEMM writes its rows into its own y buffer (TMA stores) and one push kernel over all
        # SMs stores them into every peer's; push=False stores every value to every rank's y from the GEMM's
        # epilogue instead (N stores a value on the epilogue's critical path; measured slower at 2 ranks)
        self.push = True if push is None else push
        self._bufs, self._turn, self._cap = [], 0, 0

    # ---- fused: y stored into every rank's buffer by the GEMM ----------------------------------------------------------

    def prepare(self, tokens: int, dtype=torch.bfloat16, device=None) -> None:
        """Symmetric y buffers for up to `tokens` rows (every rank calls it with the same tokens, together)."""
        device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        if self.peers is None:
            self.peers = PeerGroup(self.group, device)
        self._bufs = [_symmetric((tokens, self.rows), dtype, device, self.group) for _ in range(2)]
        self._others = [(ctypes.c_void_p * max(self.world - 1, 1))(*[ptrs[r] for r in range(self.world) if r != self.rank])
                        for _, ptrs in self._bufs]
        self._cap = tokens

    def apply_fused(self, x2: torch.Tensor, sync: bool = True) -> torch.Tensor:
        T = x2.shape[0]
        if T > self._cap:
            self.prepare(T, x2.dtype, x2.device)
        buf, ptrs = self._bufs[self._turn]
        others = self._others[self._turn]
        self._turn ^= 1
        if self.local is not None and self.push:
            a, b = self.ranges[self.rank]
            self.local.tiles(x2, out=buf[:T, a:b])
            _lib.call("p2p_peer_push", buf.data_ptr(), others, self.world - 1, T, a, b - a, self.rows,
                      _lib.dtype_code(buf), torch.cuda.current_stream(buf.device).cuda_stream)
        elif self.local is not None:
            t = self.local.tiles
            if t.layout == "tc":
                kernels.spmm_tc_peers(x2, t.words, t.seg, self.mine, self.cols, t.seg_cap, ptrs, self.world,
                                      self.ranges[self.rank][0], self.rows)
            elif t.layout == "mask":
                kernels.spmm_mask_peers(x2, t.data, t.seg, self.mine, self.cols, ptrs, self.world,
                                        self.ranges[self.rank][0], self.rows)
            else:
                raise P2PError("the fused all-gather needs a tensor-core layout (tc or mask)")
        if sync:
            self.peers.barrier()
        return buf[:T]

    # ---- nccl: a gather buffer and one all-gather ----------------------------------------------------------------------

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

    def apply(self, layer, x: torch.Tensor, bias=None, sync: bool = True) -> torch.Tensor:
        x2 = x.reshape(-1, x.shape[-1])
        if self.fused and self.world > 1:
            y = self.apply_fused(x2, sync)
        else:
            part = torch.empty(x2.shape[0], self.width, dtype=x.dtype, device=x.device)
            y = self.gather(self.local_part(x2, part))
        if bias is not None:
            y = y + bias
        return y.reshape(*x.shape[:-1], self.rows)
