"""Oracle (test infrastructure only): the compact formats and the compact forward, restated in numpy."""
from __future__ import annotations

import numpy as np

from .wanda_oracle import as_f32


def pack(w: np.ndarray, mask: np.ndarray):
    """(values [rows, k], words [rows, ceil(cols/32)] int32) of p2p/compact.py:36-45: the kept values in column order
    and bit c%32 of word c/32 set where kept (two's-complement int32)."""
    rows, cols = mask.shape
    k = int(mask[0].sum())
    assert (mask.sum(-1) == k).all(), "every row must keep the same number of weights"
    values = w[mask].reshape(rows, k)
    n = (cols + 31) // 32
    bits = np.zeros((rows, 32 * n), dtype=np.uint64)
    bits[:, :cols] = mask
    words = (bits.reshape(rows, n, 32) << np.arange(32, dtype=np.uint64)).sum(-1)
    return values, words.astype(np.uint32).view(np.int32)


def words_to_idx(words: np.ndarray, cols: int) -> np.ndarray:
    """Column indices [rows, k] of the set bits of the mask words, ascending."""
    bits = (words.astype(np.uint32)[..., None] >> np.arange(32, dtype=np.uint32)) & 1
    mask = bits.reshape(words.shape[0], -1)[:, :cols].astype(bool)
    k = int(mask[0].sum()) if mask.shape[0] else 0
    return np.nonzero(mask)[1].reshape(mask.shape[0], k)


def unpack(values: np.ndarray, words: np.ndarray, cols: int) -> np.ndarray:
    """The dense matrix pack stored (p2p/compact.py:57-61, the CPU branch)."""
    rows = values.shape[0]
    bits = (words.astype(np.uint32)[..., None] >> np.arange(32, dtype=np.uint32)) & 1
    mask = bits.reshape(rows, -1)[:, :cols].astype(bool)
    out = np.zeros((rows, cols), dtype=values.dtype)
    out[mask] = values.reshape(-1)
    return out


def expand_idx(values: np.ndarray, idx: np.ndarray, cols: int) -> np.ndarray:
    """Dense rows from values + column indices."""
    out = np.zeros((values.shape[0], cols), dtype=values.dtype)
    np.put_along_axis(out, np.asarray(idx, dtype=np.int64), values, axis=-1)
    return out


def forward(x: np.ndarray, values: np.ndarray, idx: np.ndarray, cols: int, dtype: str = "f32") -> np.ndarray:
    """y [T, rows] = x @ W.T for the W that values + idx hold, in float64: the dense masked matmul the reference's
    tests compare its kernel with (tests/test_compact.py:52, `x.float() @ w.float().T`), without fp32 rounding."""
    w = expand_idx(as_f32(values, dtype), idx, cols).astype(np.float64)
    return as_f32(x, dtype).astype(np.float64) @ w.T


def forward_blocks(x: np.ndarray, blocks: list, cols: int, dtype: str = "f32") -> np.ndarray:
    """y for a module's row blocks in row order, each ("dense", W) or ("compact", values, idx) (p2p/compact.py:205-218
    keeps the blocks in row order, tests/test_compact.py:27-36)."""
    outs = []
    for b in blocks:
        if b[0] == "dense":
            outs.append(as_f32(x, dtype).astype(np.float64) @ as_f32(b[1], dtype).astype(np.float64).T)
        else:
            outs.append(forward(x, b[1], b[2], cols, dtype))
    return np.concatenate(outs, axis=-1)
