"""Oracle (test infrastructure only): Wanda calibration and selection, restated in numpy.

bf16 tensors are held as uint16 bit patterns (numpy has no bfloat16); f16 and f32 as numpy's own types.
"""
from __future__ import annotations

import numpy as np


def bf16_to_f32(u16: np.ndarray) -> np.ndarray:
    """bf16 bit patterns -> float32 (exact)."""
    return (np.asarray(u16, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(f: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even; NaN stays NaN (quiet)."""
    f = np.ascontiguousarray(f, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(f)
    if nan.any():
        rounded = np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), rounded)
    return rounded


def as_f32(a: np.ndarray, dtype: str) -> np.ndarray:
    """Values of a tensor of `dtype` ("bf16", "f16", "f32") as float32."""
    if dtype == "bf16":
        return bf16_to_f32(a)
    a = np.asarray(a)
    if dtype == "f16" and a.dtype == np.uint16:          # f16 bit patterns
        a = a.view(np.float16)
    return a.astype(np.float32)


def k_of(keep: float, cols: int) -> int:
    """Weights kept per row: max(1, round(keep / 100 * cols)) with Python's round-half-even on the float
    (p2p/wanda.py:82)."""
    return max(1, round(keep / 100 * cols))


def sumsq_cols(x: np.ndarray, dtype: str = "f32") -> np.ndarray:
    """x.float().pow(2).sum(0).double() (p2p/wanda.py:39): squares in fp32, the column sum rounded to fp32, as float64.
    The sum itself is taken in float64 and rounded once, so the result is the correctly rounded fp32 column sum."""
    xf = as_f32(x, dtype)
    sq = (xf * xf).astype(np.float32)
    return sq.astype(np.float64).sum(0).astype(np.float32).astype(np.float64)


def channel_norms(sums: np.ndarray) -> np.ndarray:
    """sums.sqrt().float(), and for expert sums [E, C] a row of zeros becomes ones, shaped [E, 1, C]
    (p2p/wanda.py:63-73, without the TP slice)."""
    norms = np.sqrt(np.asarray(sums, dtype=np.float64)).astype(np.float32)
    if norms.ndim == 2:
        zero = ~(norms.sum(-1, keepdims=True, dtype=np.float32) > 0)
        norms = np.where(zero, np.float32(1.0), norms)[:, None, :]
    return norms


def scores(w: np.ndarray, norms: np.ndarray, dtype: str = "f32") -> np.ndarray:
    """w.float().abs() * norms in fp32 (p2p/wanda.py:80)."""
    return (np.abs(as_f32(w, dtype)) * np.asarray(norms, dtype=np.float32)).astype(np.float32)


def select(score: np.ndarray, k: int) -> np.ndarray:
    """Column indices [rows, k], ascending, of each row's k highest scores; ties go to the lower column.
    The reference's choice is the top-k of p2p/wanda.py:83 (torch.topk, tie order unspecified); this is a stable
    descending sort, which agrees with it on every row whose k-th and (k+1)-th scores differ."""
    s = np.asarray(score, dtype=np.float32)
    s = np.where(s == 0, np.float32(0), s)                       # -0 ranks as +0
    order = np.argsort(-s, axis=-1, kind="stable")[..., :k]
    return np.sort(order, axis=-1)


def tie_rows(score: np.ndarray, k: int) -> np.ndarray:
    """Rows whose k-th and (k+1)-th highest scores are equal: where the reference's topk may choose otherwise."""
    s = np.sort(np.asarray(score, dtype=np.float32), axis=-1)[..., ::-1]
    if k >= s.shape[-1]:
        return np.zeros(s.shape[:-1], dtype=bool)
    return s[..., k - 1] == s[..., k]


def prune(w: np.ndarray, keep: float, norms: np.ndarray, dtype: str = "f32"):
    """(pruned, mask) of p2p/wanda.py:76-87 with with_mask=True, no TP group: w where kept, w.float() * 0 elsewhere."""
    s = scores(w, norms, dtype)
    k = k_of(keep, s.shape[-1])
    idx = select(s, k)
    mask = np.zeros(s.shape, dtype=bool)
    np.put_along_axis(mask, idx, True, axis=-1)
    wf = as_f32(w, dtype)
    pruned = (wf * mask).astype(np.float32)
    if dtype == "bf16":
        pruned = f32_to_bf16(pruned)
    elif dtype == "f16":
        pruned = pruned.astype(np.float16).view(np.uint16)
    return pruned, mask


def expert_inputs(x: np.ndarray, ids: np.ndarray, w13: np.ndarray, w2_cols: int, dtype: str = "f32"):
    """(into [E, hidden], gated [E, rows]) of p2p/wanda.py:10-20: for each expert, over the tokens routed to it (each
    token once), the fp32 column sums of x^2 and of (silu(gate) * up)^2 with gate, up = x @ w13[e].T, as float64.
    w13: [E, 2 * rows, hidden] float32 values."""
    xf = as_f32(x, dtype)
    n_exp = w13.shape[0]
    into = np.zeros((n_exp, xf.shape[-1]), dtype=np.float64)
    gated = np.zeros((n_exp, w2_cols), dtype=np.float64)
    for e in np.unique(ids):
        if e < 0:
            continue
        routed = xf[(ids == e).any(-1)]
        into[e] = sumsq_cols(routed)
        gu = (routed.astype(np.float64) @ w13[e].astype(np.float64).T).astype(np.float32)
        gate, up = np.split(gu, 2, axis=-1)
        act = (gate / (1 + np.exp(-gate.astype(np.float64)))).astype(np.float32) * up
        gated[e] = sumsq_cols(act.astype(np.float32))
    return into, gated
