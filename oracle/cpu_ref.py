"""Oracle (test infrastructure only): the reference's CPU path for a compact projection, for the timed CPU baseline.

The reference has no CPU sparse kernel (p2p/compact.py:117-122: Tiles needs CUDA); its CPU path expands the packed
rows (p2p/compact.py:57-61, the CPU branch of unpack) and runs the dense masked matmul F.linear(x, W), as its tests
do (tests/test_compact.py:52). Its one-time work on a replica's load is the Wanda selection (p2p/wanda.py:76-87) and
the packing (p2p/compact.py:36-45). This module restates those steps with torch on the CPU, the library the reference
itself uses there, so they can be timed on a machine without the reference.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def unpack_rows(values: torch.Tensor, idx: torch.Tensor, cols: int) -> torch.Tensor:
    """Dense rows with the kept values in place and zeros elsewhere (p2p/compact.py:57-61, from column indices)."""
    out = torch.zeros(values.shape[0], cols, dtype=values.dtype)
    out.scatter_(1, idx.to(torch.int64), values)
    return out


def forward(x: torch.Tensor, dense: torch.Tensor) -> torch.Tensor:
    """y = x @ W.T on the CPU (F.linear of the unpacked matrix), in the weights' dtype."""
    return F.linear(x, dense)


def prune(w: torch.Tensor, keep: float, norms: torch.Tensor) -> tuple:
    """(pruned, mask) of p2p/wanda.py:76-87 (no TP group), with the torch CPU operations it is made of: fp32 scores
    |w| * norms, torch.topk of k = max(1, round(keep / 100 * cols)) per row, a bool mask set at the winners, w kept
    where the mask is set."""
    cols = w.shape[-1]
    k = max(1, round(keep / 100 * cols))
    winners = (w.float().abs() * norms).topk(k, dim=-1).indices
    mask = torch.zeros(w.shape, dtype=torch.bool)
    mask.scatter_(-1, winners, True)
    return torch.where(mask, w.float(), 0.0).to(w.dtype), mask


def pack(w: torch.Tensor, mask: torch.Tensor) -> tuple:
    """(values [rows, k], words [rows, ceil(cols / 32)] int32) of p2p/compact.py:36-45: the kept values in column
    order, and each group of 32 columns as one word with bit j set where column 32 i + j is kept (two's complement)."""
    rows, cols = w.shape
    n_words = -(-cols // 32)
    kept = torch.zeros(rows, n_words * 32, dtype=torch.int64)
    kept[:, :cols] = mask
    weights = torch.ones(32, dtype=torch.int64) << torch.arange(32)
    words = (kept.view(rows, n_words, 32) * weights).sum(-1)
    words = words - (words >> 31) * (1 << 32)                     # to the signed 32-bit range
    return w[mask].reshape(rows, -1), words.to(torch.int32)


def unpack_words(values: torch.Tensor, words: torch.Tensor, cols: int) -> torch.Tensor:
    """The dense matrix of values and mask words (p2p/compact.py:57-61, the CPU branch)."""
    rows = values.shape[0]
    shifts = torch.arange(32)
    bits = (words.to(torch.int64)[:, :, None] >> shifts) & 1
    kept = bits.reshape(rows, -1)[:, :cols].to(torch.bool)
    dense = torch.zeros(rows, cols, dtype=values.dtype)
    dense[kept] = values.flatten()
    return dense
