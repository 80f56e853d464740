"""Host logic of the multi-GPU paths on CPU: two gloo ranks in child processes (127.0.0.1). The NCCL hop's framing
(route.send_piece / recv_parts: each destination gets the piece, the receiver takes parts in member order) and the row
sharding's partition (shard.row_ranges / shard_blocks: whole 128-row tiles, every row once) and its all-gather
assembly."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from p2pllm_b200 import route, shard


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(rank, world, port, fn, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        q.put((rank, fn(rank, world)))
    finally:
        dist.destroy_process_group()


def _spawn(fn, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, world, port, fn, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return out


def _hop(rank, world):
    # rank 0 and rank 1 are members of a spread step; both send their part to both ranks, which add them in order
    piece = torch.full((3, 5), float(rank + 1)) * torch.arange(5.0)
    works = route.send_piece(piece, [r for r in range(world) if r != rank])
    parts = route.recv_parts([r for r in range(world) if r != rank], piece)
    for w in works:
        w.wait()
    got = [piece if r == rank else parts.pop(0) for r in range(world)]
    return [g.tolist() for g in got]


def _exchange(rank, world):
    piece = torch.full((2, 3), float(rank + 1))
    peers = [r for r in range(world) if r != rank]
    got = route.exchange(piece, peers, peers)
    return [g.tolist() for g in got]


def test_exchange_batches_both_directions():
    out = _spawn(_exchange)
    assert out[0] == [[[2.0] * 3] * 2] and out[1] == [[[1.0] * 3] * 2]


def test_hop_delivers_every_members_part_in_order():
    out = _spawn(_hop)
    want = [(torch.full((3, 5), float(r + 1)) * torch.arange(5.0)).tolist() for r in range(2)]
    assert out[0] == want and out[1] == want


@pytest.mark.parametrize("rows,world", [(1, 2), (127, 2), (128, 2), (129, 2), (4096, 8), (14336, 8), (5120, 3),
                                        (300, 4), (0, 2)])
def test_row_ranges_cover_every_row_once_in_whole_tiles(rows, world):
    ranges = shard.row_ranges(rows, world)
    assert len(ranges) == world and ranges[0][0] == 0 and ranges[-1][1] == rows
    for (a, b), (c, d) in zip(ranges, ranges[1:]):
        assert b == c and a <= b
    assert all(a % 128 == 0 for a, _ in ranges if a < rows)
    tiles = [-(-(b - a) // 128) for a, b in ranges]
    assert max(tiles) - min(tiles) <= 1


def test_shard_blocks_cut_mixed_blocks():
    w = torch.arange(10 * 4.0).view(10, 4)
    v = torch.arange(6 * 2.0).view(6, 2)
    idx = torch.tensor([[0, 3]] * 6)
    blocks = [("dense", w), ("compact", v, idx, 4)]
    got = shard.shard_blocks(blocks, 8, 13)
    assert got[0][0] == "dense" and torch.equal(got[0][1], w[8:10])
    assert got[1][0] == "compact" and torch.equal(got[1][1], v[0:3]) and torch.equal(got[1][2], idx[0:3])


def _gather(rank, world):
    # ShardedCompact.gather on CPU parts: each rank's run of rows, padded to the widest run; 300 rows split unevenly
    # (256 + 44), 256 rows evenly (128 + 128)
    out = {}
    for rows in (300, 256):
        sc = object.__new__(shard.ShardedCompact)
        sc.group, sc.world, sc.rank, sc.rows = None, world, rank, rows
        sc.ranges = shard.row_ranges(rows, world)
        sc.width = max(b - a for a, b in sc.ranges)
        a, b = sc.ranges[rank]
        part = torch.zeros(2, sc.width)
        part[:, :b - a] = torch.arange(a, b, dtype=torch.float32)
        y = sc.gather(part)
        out[rows] = (tuple(y.shape), y.tolist())
    return out


def test_gather_assembles_rows_in_order():
    out = _spawn(_gather)
    for rows in (300, 256):
        want = torch.arange(float(rows)).expand(2, rows).tolist()
        assert out[0][rows] == ((2, rows), want) and out[1][rows] == ((2, rows), want)