"""The reference's own GPU kernel (p2p/compact.cu, built into oracle/_ref/ by oracle/build_ref.py) on the layouts
its Tiles built (tests/golden/tiles_cases.npz) and on this library's selections: within the reference's tolerance of
the oracle's dense forward, and of this library's compact GEMM on the same weights. Skipped where the reference kernel
was not built (it needs the reference tree at build time)."""
import numpy as np
import pytest
import torch

import oracle
from conftest import tiles_blocks
from oracle import build_ref, ref_tiles

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(build_ref.built() is None, reason="reference kernel not built into oracle/_ref")]


@pytest.fixture(scope="module")
def ext():
    return build_ref.load_module()


def _dense(blocks, cols):
    dense, _ = ref_tiles._dense_and_kept(blocks, cols, blocks[0][1].dtype, "cpu")
    return dense


@pytest.mark.parametrize("name", ["a", "b", "c"])
@pytest.mark.parametrize("tokens", [1, 17, 64, 100])
def test_reference_kernel_on_its_own_layouts(ext, tiles_golden, name, tokens):
    blocks = tiles_blocks(tiles_golden, name)
    cols = int(tiles_golden[name + "_meta"][1])
    cuda_blocks = [tuple(t.cuda() if torch.is_tensor(t) else t for t in b) for b in blocks]
    tiles = ref_tiles.RefTiles(cuda_blocks, ext, tune=False)
    g = torch.Generator().manual_seed(tokens)
    x = torch.randn(tokens, cols, generator=g).to(blocks[0][1].dtype)
    y = tiles(x.cuda()).cpu().double()
    want = x.double() @ _dense(blocks, cols).double().T
    rel = float((y - want).norm() / want.norm())
    assert rel <= 1e-2, rel


@pytest.mark.parametrize("rows,cols,keep,tokens", [(1024, 4096, 33, 17), (640, 1024, 36, 272)])
def test_reference_kernel_agrees_with_ours(ext, rows, cols, keep, tokens):
    from p2pllm_b200 import compact, wanda
    g = torch.Generator(device="cuda").manual_seed(rows)
    w = (torch.randn(rows, cols, generator=g, device="cuda") * 0.02).bfloat16()
    norms = torch.rand(cols, generator=g, device="cuda") + 0.1
    values, idx = wanda.select(w, keep, norms)
    x = torch.randn(tokens, cols, generator=g, device="cuda").bfloat16()
    ref = ref_tiles.RefTiles([("sparse", values, ref_tiles.words_of(idx, cols), cols)], ext)(x).double()
    ours = compact.Compact([("compact", values, idx, cols)]).apply(None, x).double()
    bits = lambda t: t.cpu().view(torch.int16).numpy().view(np.uint16)
    want = oracle.forward(bits(x), bits(values), idx.cpu().numpy().astype(np.int64), cols, "bf16")
    for y in (ref, ours):
        rel = np.linalg.norm(y.cpu().numpy() - want) / np.linalg.norm(want)
        assert rel <= 1e-2, rel
