"""Oracle (test infrastructure only): the reference's CPU forward of a compact projection, for the timed CPU baseline.

The reference has no CPU sparse kernel (p2p/compact.py:117-122: Tiles needs CUDA); its CPU path expands the packed
rows (p2p/compact.py:57-61, the CPU branch of unpack) and runs the dense masked matmul F.linear(x, W), as its tests
do (tests/test_compact.py:52). This module restates that path with torch on the CPU, the library the reference itself
uses there.
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
