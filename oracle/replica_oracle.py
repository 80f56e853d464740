"""Oracle (test infrastructure only): the group combine and the spread-step parts, restated in numpy."""
from __future__ import annotations

import numpy as np

from .wanda_oracle import as_f32, f32_to_bf16


def _round(v: np.ndarray, dtype: str) -> np.ndarray:
    """v (float32) rounded to `dtype` and back to float32."""
    if dtype == "bf16":
        from .wanda_oracle import bf16_to_f32
        return bf16_to_f32(f32_to_bf16(v))
    if dtype == "f16":
        return v.astype(np.float16).astype(np.float32)
    return v.astype(np.float32)


def _out(v: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return f32_to_bf16(v)
    if dtype == "f16":
        return v.astype(np.float16).view(np.uint16)
    return v.astype(np.float32)


def combine(parts: list, h: np.ndarray, h_copy: np.ndarray, dtype: str) -> np.ndarray:
    """p2p/replica.py:81-85: total = float(l_0(h)); for the middle members total += dtype(float(l_k(h)) - float(h));
    total += dtype(float(l_last(h~)) - float(h~)); the result in dtype. parts[k]: member k's output."""
    total = as_f32(parts[0], dtype).copy()
    hf = as_f32(h, dtype)
    for p in parts[1:-1]:
        total += _round(as_f32(p, dtype) - hf, dtype)
    total += _round(as_f32(parts[-1], dtype) - as_f32(h_copy, dtype), dtype)
    return _out(total, dtype)


def summed(parts: list, dtype: str) -> np.ndarray:
    """p2p/route.py:825-831: the parts added in float32 in member order, the sum in dtype."""
    total = as_f32(parts[0], dtype).copy()
    for p in parts[1:]:
        total += as_f32(p, dtype)
    return _out(total, dtype)


def member_part(y: np.ndarray, x: np.ndarray, dtype: str) -> np.ndarray:
    """p2p/route.py:1268-1274: a member's part (float(y) - float(x)) in dtype."""
    return _out(as_f32(y, dtype) - as_f32(x, dtype), dtype)
