"""The compact sparse GEMM and the compact formats on the GPU, against the oracle's dense masked matmul (the check of
the reference's tests/test_compact.py) and the reference's pack/unpack semantics."""
import numpy as np
import pytest
import torch

import oracle
from p2pllm_b200 import P2PError, compact, kernels, wanda

pytestmark = pytest.mark.gpu


def _pruned(rows, cols, keep, dtype=torch.float16, seed=0):
    """tests/test_compact.py:11-16: a pruned matrix and its mask from seeded weights and norms rand + 0.1."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = torch.randn(rows, cols, generator=g, device="cuda").to(dtype)
    norms = torch.rand(cols, generator=g, device="cuda") + 0.1
    return wanda.prune(w, keep, norms, with_mask=True), w, norms


def _rel_l2(got, want):
    got, want = got.double(), want.double()
    return (torch.linalg.norm(got - want) / torch.linalg.norm(want)).item()


@pytest.mark.parametrize("rows,cols,keep", [(64, 64, 50), (100, 77, 7), (256, 5120, 40), (130, 1000, 90), (8, 33, 5)])
def test_pack_round_trips(rows, cols, keep):
    """tests/test_compact.py:19-24."""
    (w, mask), _, _ = _pruned(rows, cols, keep)
    values, words = compact.pack(w, mask)
    assert values.shape == (rows, max(1, round(keep / 100 * cols))) and words.dtype == torch.int32
    assert torch.equal(compact.unpack(values, words, cols), w)
    v2, words2 = oracle.pack(w.cpu().float().numpy(), mask.cpu().numpy())
    assert np.array_equal(words.cpu().numpy(), words2)


def test_pack_refuses_rows_of_unequal_length():
    w = torch.randn(4, 16, device="cuda")
    mask = torch.zeros(4, 16, dtype=torch.bool, device="cuda")
    mask[:, :3] = True
    mask[2, 5] = True
    with pytest.raises(AssertionError):
        compact.pack(w, mask)


def test_compact_method_puts_blocks_in_row_order():
    """tests/test_compact.py:27-36: a sparse block then a dense one."""
    (a, ma), _, _ = _pruned(48, 96, 30)
    (b, _), _, _ = _pruned(32, 96, 100, seed=1)
    method = compact.Compact([("sparse", *compact.pack(a, ma), 96), ("dense", b)])
    x = torch.randn(2, 5, 96, device="cuda").half()
    want = x.float() @ torch.cat([a, b]).float().T
    got = method.apply(None, x).float()
    assert got.shape == (2, 5, 80) and (got - want).abs().max() <= 1e-2 * want.abs().max()


@pytest.mark.parametrize("layout", [None, "rows"])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("t", [1, 3, 17, 32, 64, 100, 272])
@pytest.mark.parametrize("rows,cols,keep", [(512, 5120, 40), (300, 1000, 7), (96, 80, 90), (1024, 2048, 25), (17, 8, 50),
                                            (5000, 256, 30)])
def test_tiles_match_a_dense_matmul(layout, dtype, t, rows, cols, keep):
    """tests/test_compact.py:44-56 (its tolerance max|d| <= 1e-2 max|want|), plus rel-L2 <= 1e-2 for bf16/f16 and
    <= 1e-5 for fp32, any shape and any token count, in either layout (bf16/f16 default to the tensor-core one)."""
    if layout is not None and dtype == torch.float32:
        pytest.skip("fp32 has the row layout only")
    (w, mask), _, _ = _pruned(rows, cols, keep, dtype)
    tiles = compact.Tiles([("sparse", *compact.pack(w, mask), cols)], layout=layout)
    x = torch.randn(t, cols, device="cuda").to(dtype)
    want = x.double() @ w.double().T
    got = tiles(x)
    assert got.shape == (t, rows) and got.dtype == dtype
    assert (got.double() - want).abs().max() <= 1e-2 * want.abs().max()
    assert _rel_l2(got, want) <= (1e-5 if dtype == torch.float32 else 1e-2)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_rows_layout_against_the_oracle_with_int32_indices(dtype):
    """cols above 32767 take int32 indices."""
    rows, cols, keep = 40, 40000, 10
    (w, mask), _, _ = _pruned(rows, cols, keep, dtype, seed=5)
    values, idx = wanda.select(w, keep, torch.rand(cols, device="cuda") + 0.1)
    assert idx.dtype == torch.int32
    x = torch.randn(9, cols, device="cuda").to(dtype)
    got = compact.Tiles([("compact", values, idx, cols)])(x)
    bits = values.cpu().float().numpy()
    want = oracle.forward(x.cpu().float().numpy(), bits, idx.cpu().numpy(), cols)
    rel = np.linalg.norm(got.cpu().double().numpy() - want) / np.linalg.norm(want)
    assert rel <= (1e-5 if dtype == torch.float32 else 1e-2)


def test_dense_and_compact_blocks_of_mixed_keep():
    """A fused module (q, k, v) whose blocks keep different k, one of them dense."""
    cols = 512
    g = torch.Generator(device="cuda").manual_seed(3)
    norms = torch.rand(cols, generator=g, device="cuda") + 0.1
    ws = [torch.randn(r, cols, generator=g, device="cuda").bfloat16() for r in (128, 64, 64)]
    blocks = [("compact", *wanda.select(ws[0], 33, norms), cols), ("dense", ws[1]),
              ("compact", *wanda.select(ws[2], 60, norms), cols)]
    tiles = compact.Tiles(blocks)
    x = torch.randn(17, cols, device="cuda").bfloat16()
    dense = torch.cat([compact.expand(b) for b in blocks])
    want = x.double() @ dense.double().T
    assert _rel_l2(tiles(x), want) <= 1e-2


def test_zero_tokens_and_empty_blocks():
    (w, mask), _, _ = _pruned(64, 128, 30, torch.bfloat16)
    tiles = compact.Tiles([("sparse", *compact.pack(w, mask), 128)])
    assert tiles(torch.empty(0, 128, device="cuda", dtype=torch.bfloat16)).shape == (0, 64)


def test_bad_indices_are_refused_at_load():
    values = torch.randn(4, 3, device="cuda").bfloat16()
    idx = torch.tensor([[0, 1, 2]] * 3 + [[0, 1, 9]], dtype=torch.int16, device="cuda")
    with pytest.raises(P2PError, match="outside"):
        compact.Tiles([("compact", values, idx, 8)])


def test_words_with_the_wrong_count_are_refused():
    values = torch.randn(2, 3, device="cuda")
    words = torch.tensor([[0b111], [0b1111]], dtype=torch.int32, device="cuda")   # 3 and 4 bits
    with pytest.raises(P2PError, match="exactly"):
        compact.Tiles([("sparse", values, words, 8)])


def test_no_cpu_fallback():
    with pytest.raises(P2PError, match="CUDA"):
        kernels.sumsq_cols(torch.randn(4, 4), torch.zeros(4, dtype=torch.float64))


def test_expand_experts_and_compact_moe_match_a_reference_moe():
    """tests/test_compact.py:80-126: CompactMoE expands only the routed experts, renumbers their ids and hands both to
    the layer's own method; the result equals the method on the dense pruned weights."""
    from typing import NamedTuple

    import torch.nn as nn
    import torch.nn.functional as F

    class TopK(NamedTuple):
        topk_weights: torch.Tensor
        topk_ids: torch.Tensor

    class Dispatch(NamedTuple):
        hidden_states: torch.Tensor
        topk_output: TopK

    class Method:
        def apply(self, layer, d):
            x, t, out = d.hidden_states.float(), d.topk_output, 0
            for j in range(t.topk_ids.shape[1]):
                gate, up = torch.einsum("trh,th->tr", layer.w13_weight[t.topk_ids[:, j]].float(), x).chunk(2, -1)
                out = out + t.topk_weights[:, j:j + 1] * torch.einsum(
                    "thr,tr->th", layer.w2_weight[t.topk_ids[:, j]].float(), F.silu(gate) * up)
            return out

    E, R, H, T = 16, 32, 64, 5
    g = torch.Generator(device="cuda").manual_seed(0)
    w13 = torch.randn(E, 2 * R, H, generator=g, device="cuda").half()
    w2 = torch.randn(E, H, R, generator=g, device="cuda").half()
    blocks, pruned = {"w13_weight": [], "w2_weight": []}, {}
    for name, w, rows in (("w13_weight", w13, (slice(0, R), slice(R, 2 * R))), ("w2_weight", w2, (slice(None),))):
        parts = []
        for r in rows:
            norms = torch.rand(E, 1, w.shape[-1], generator=g, device="cuda") + 0.1
            p, mask = wanda.prune(w[:, r].contiguous(), 40, norms, with_mask=True)
            values, words = compact.pack(p.reshape(-1, w.shape[-1]), mask.reshape(-1, w.shape[-1]))
            blocks[name].append(("sparse", values.view(E, p.shape[1], -1), words.view(E, p.shape[1], -1), w.shape[-1]))
            parts.append(p)
        pruned[name] = torch.cat(parts, dim=1)
    dense, empty = nn.Module(), nn.Module()
    for name in pruned:
        dense.register_parameter(name, nn.Parameter(pruned[name], requires_grad=False))
        empty.register_parameter(name, nn.Parameter(pruned[name].new_empty(0), requires_grad=False))
    ids = torch.tensor([[3, 11], [11, 0], [7, 3], [15, 7], [0, 11]], device="cuda")
    d = Dispatch(torch.randn(T, H, generator=g, device="cuda").half(), TopK(torch.rand(T, 2, device="cuda"), ids))
    got = compact.CompactMoE(Method(), blocks).apply(empty, d)
    assert torch.equal(got, Method().apply(dense, d))
    assert all(empty._parameters[name].numel() == 0 for name in pruned)


def test_out_is_checked_and_may_be_a_column_slice():
    """A caller's out: the wrong shape or dtype is refused; a column slice of a wider buffer is written in place."""
    (w, mask), _, _ = _pruned(256, 512, 30, torch.bfloat16, seed=4)
    for layout in ("tc", "rows"):
        tiles = compact.Tiles([("sparse", *compact.pack(w, mask), 512)], layout=layout)
        x = torch.randn(17, 512, device="cuda").bfloat16()
        wide = torch.full((17, 400), 7.0, device="cuda").bfloat16()
        got = tiles(x, out=wide[:, 16:272])
        assert got.data_ptr() == wide[:, 16:272].data_ptr()
        assert torch.equal(wide[:, 16:272], tiles(x))
        assert (wide[:, :16] == 7).all() and (wide[:, 272:] == 7).all()
        with pytest.raises(P2PError, match="wanted"):
            tiles(x, out=torch.empty(17, 255, device="cuda", dtype=torch.bfloat16))
        with pytest.raises(P2PError, match="wanted"):
            tiles(x, out=torch.empty(17, 256, device="cuda", dtype=torch.float16))
        with pytest.raises(P2PError, match="strides"):
            tiles(x, out=torch.empty(256, 17, device="cuda", dtype=torch.bfloat16).T)
