"""The spread-step hop of p2p/route.py on B200: members on different GPUs send their parts of a step to the next
step's ranks over NCCL (NVLink), and the receiver adds them in fp32 in member order.

    member_part   p2p/route.py:1254-1274   l(h) for member 0, dtype(l(h) - h) for the others
    send_piece    p2p/route.py:800-810     one NCCL isend per destination rank
    exchange      a rank's sends and receives of one step as one NCCL batch
    summed        p2p/route.py:825-831     dtype(sum of the parts in fp32, member order)

The SGLang pipeline plumbing around them (stage layout, request framing, KV updates) is not part of this package.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import kernels


def member_part(k: int, y: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """Member k's part of a step: y itself for the first member, dtype(float(y) - float(x)) for the others."""
    return y if k == 0 else kernels.member_part(y, x)


def summed(parts: list, dtype=None) -> torch.Tensor:
    """One step input from its members' parts, added in fp32 in member order."""
    out = kernels.sum_parts(parts)
    return out if dtype is None or out.dtype == dtype else out.to(dtype)


def send_piece(t: torch.Tensor, dsts: list, group=None) -> list:
    """t to every rank in dsts, one NCCL isend each, once the current stream has made it. Returns the works; keep t
    alive until they complete."""
    t = t.contiguous()
    return [dist.isend(t, dst, group=group) for dst in dsts]


def recv_parts(srcs: list, like: torch.Tensor, group=None) -> list:
    """One part from each rank in srcs (member order), received into new tensors shaped like `like`. For a rank that
    only receives; a rank that also sends in the same step uses exchange()."""
    bufs = [torch.empty_like(like) for _ in srcs]
    works = [dist.irecv(b, src, group=group) for b, src in zip(bufs, srcs)]
    for w in works:
        w.wait()
    return bufs


def exchange(piece: torch.Tensor, dsts: list, srcs: list, group=None) -> list:
    """Send piece to every rank in dsts and receive one part from every rank in srcs (member order), as one batch:
    NCCL runs a rank's sends and receives of a step together, so two ranks sending to each other cannot each wait for
    the other's receive. Returns the received parts."""
    piece = piece.contiguous()
    bufs = [torch.empty_like(piece) for _ in srcs]
    ops = [dist.P2POp(dist.isend, piece, d, group=group) for d in dsts]
    ops += [dist.P2POp(dist.irecv, b, s, group=group) for b, s in zip(bufs, srcs)]
    if ops:
        for w in dist.batch_isend_irecv(ops):
            w.wait()
    return bufs
