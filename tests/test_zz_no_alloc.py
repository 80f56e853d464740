"""p2p_sumsq_cols_noalloc: the calibration reduction for callers that cannot allocate device memory.

A calibration hook runs inside the serving engine's forward pass, after the engine (SGLang) has reserved its share of
GPU memory for weights and the KV pool; asking the driver for scratch memory there can fail or fragment what is left.
This entry point keeps its scratch in a fixed array inside the library and allocates nothing. The test calls it
through the C ABI, twice in a row on the same and on different inputs, and checks each result against the
workspace-taking p2p_sumsq_cols, within the same tolerance the other calibration tests use (relative 1e-6: the column
totals are rounded to fp32 once per call)."""
import ctypes

import numpy as np
import pytest
import torch

from p2pllm_b200 import _lib, kernels

pytestmark = pytest.mark.gpu

DTYPE = {torch.bfloat16: _lib.BF16, torch.float16: _lib.F16, torch.float32: _lib.F32}


def _noalloc(x: torch.Tensor, sums: torch.Tensor) -> int:
    lib = _lib.load()
    return lib.p2p_sumsq_cols_noalloc(ctypes.c_void_p(x.data_ptr()), DTYPE[x.dtype], x.shape[0], x.shape[1],
                                      x.stride(0), ctypes.c_void_p(sums.data_ptr()),
                                      ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("dtype,shape", [(torch.bfloat16, (100000, 4096)), (torch.float32, (30000, 16384)),
                                         (torch.float16, (5000, 1000)), (torch.bfloat16, (7, 33))])
def test_two_calls_match_the_workspace_entry_point(dtype, shape):
    g = torch.Generator(device="cuda").manual_seed(shape[0])
    for call in range(2):                       # the built-in scratch keeps the last call's contents
        x = (torch.randn(*shape, generator=g, device="cuda") * (1 + call)).to(dtype)
        want = torch.zeros(shape[1], dtype=torch.float64, device="cuda")
        kernels.sumsq_cols(x, want)
        got = torch.zeros(shape[1], dtype=torch.float64, device="cuda")
        assert _noalloc(x, got) == 0, _lib.load().p2p_last_error().decode()
        torch.cuda.synchronize()
        assert np.allclose(got.cpu().numpy(), want.cpu().numpy(), rtol=1e-6, atol=0)


def test_it_accumulates_like_the_hook():
    """Calls add into sums, as the reference's hook accumulates call after call (p2p/wanda.py:34-40)."""
    x = torch.randn(20000, 2048, device="cuda").bfloat16()
    want = torch.zeros(2048, dtype=torch.float64, device="cuda")
    got = torch.zeros(2048, dtype=torch.float64, device="cuda")
    for _ in range(2):
        kernels.sumsq_cols(x, want)
        assert _noalloc(x, got) == 0
    torch.cuda.synchronize()
    assert np.allclose(got.cpu().numpy(), want.cpu().numpy(), rtol=1e-6, atol=0)


def test_more_columns_than_its_scratch_holds_are_refused():
    x = torch.zeros(4, 16385, device="cuda", dtype=torch.bfloat16)
    sums = torch.zeros(16385, dtype=torch.float64, device="cuda")
    assert _noalloc(x, sums) == -2
    assert b"16384" in _lib.load().p2p_last_error()
