"""The gated GEMM (SiLU(gate) * up in the compact GEMM's epilogue) against the unfused path it replaces -- the
gate_up projection's output rounded to the model dtype, then silu(gate) * up in fp32, rounded -- on the plain
tensor-core launch (one split, cluster-reduced splits, workspace-reduced splits); routed experts are covered in
test_gpu_moe.py. The epilogue's exp may differ from torch's in the last fp32 bit, so outputs agree to rel-L2 1e-3 and
almost all bits."""
import pytest
import torch
import torch.nn.functional as F

from p2pllm_b200 import compact, wanda
from p2pllm_b200._lib import P2PError

pytestmark = pytest.mark.gpu


def _unfused(tiles: compact.Tiles, x: torch.Tensor, R: int) -> torch.Tensor:
    gu = tiles(x)
    return (F.silu(gu[:, :R].float()) * gu[:, R:].float()).to(x.dtype)


def _close(got, want):
    rel = float((got.double() - want.double()).norm() / want.double().norm())
    same = float((got == want).float().mean())
    return rel, same


def _blocks(R, H, keep, dtype, seed, dense=False):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = (torch.randn(2 * R, H, generator=g, device="cuda") * 0.05).to(dtype)
    if dense:
        return [("dense", w[:R]), ("dense", w[R:])]
    norms = torch.rand(H, generator=g, device="cuda") + 0.1
    v, i = wanda.select(w, keep, norms)
    return [("compact", v[:R], i[:R], H), ("compact", v[R:], i[R:], H)]


@pytest.mark.parametrize("T", [1, 17, 64, 272])
@pytest.mark.parametrize("R,H", [(768, 2048), (14336, 4096), (256, 27648)])
def test_gated_module_is_silu_of_gate_times_up(T, R, H):
    blocks = _blocks(R, H, 36, torch.bfloat16, seed=R + T)
    gated = compact.GatedTiles(blocks)
    plain = compact.Tiles(blocks, layout="tc")
    x = torch.randn(T, H, generator=torch.Generator(device="cuda").manual_seed(T), device="cuda").bfloat16()
    got = gated(x)
    assert got.shape == (T, R)
    rel, same = _close(got, _unfused(plain, x, R))
    assert rel <= 1e-3 and same >= 0.98, (rel, same)


def test_gated_dense_rows_and_f16_and_out():
    blocks = _blocks(512, 1024, 100, torch.float16, seed=3, dense=True)
    gated = compact.GatedTiles(blocks)
    plain = compact.Tiles(blocks, layout="tc")
    x = torch.randn(17, 1024, device="cuda").half()
    wide = torch.full((17, 700), 3.0, device="cuda").half()
    got = gated(x, out=wide[:, 100:612])
    rel, same = _close(got, _unfused(plain, x, 512))
    assert rel <= 1e-3 and same >= 0.98
    assert (wide[:, :100] == 3).all() and (wide[:, 612:] == 3).all()


def test_gated_layout_refuses_rows_it_cannot_pair():
    blocks = _blocks(96, 256, 50, torch.bfloat16, seed=4)        # R = 96 is not a multiple of 64
    with pytest.raises(P2PError, match="multiple of 64"):
        compact.GatedTiles(blocks)
