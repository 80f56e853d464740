"""The bitmask layout (the reference's storage: values + one bit a weight) and its tcgen05 GEMM with the weight tiles
in tensor memory, on the GPU: the layout decodes back to the selection bit for bit, and the GEMM matches the oracle's
dense masked matmul (rel-L2 <= 1e-2 for bf16/f16, and the reference test's max|d| <= 1e-2 max|want|) over token counts
1..600, odd shapes, mixed dense/compact blocks, the reference's own block form, split columns and every Llama-3-8B
projection; repeated calls give the same bits."""
import numpy as np
import pytest
import torch

import oracle
from p2pllm_b200 import compact, kernels, wanda

pytestmark = pytest.mark.gpu

# piece p, bit -> (row in its 16-row block, column in its 64-column tile); the layout's definition
P = np.arange(16)[:, None]
BIT = np.arange(64)[None, :]
PIECE_ROW = 8 * ((P >> 1) & 1) + (BIT >> 3)
PIECE_COL = 16 * (P >> 2) + 4 * ((BIT >> 1) & 3) + 2 * (P & 1) + (BIT & 1)


def _bits(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def _module(rows, cols, keep, dtype=torch.bfloat16, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = (torch.randn(rows, cols, generator=g, device="cuda") * 0.02).to(dtype)
    norms = torch.rand(cols, generator=g, device="cuda") + 0.1
    return wanda.select(w, keep, norms)


def _check(got, want):
    got = got.double().cpu().numpy() if torch.is_tensor(got) else got
    rel = np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30)
    assert rel <= 1e-2, rel
    assert np.abs(got - want).max() <= 1e-2 * np.abs(want).max()


def decode(data: np.ndarray, seg: np.ndarray, rows: int, cols: int):
    """(values [rows, cols] uint16, kept [rows, cols] bool) of a bitmask layout, checking its header, the start
    offsets of every half-piece and the sizes."""
    n_ct = -(-cols // 64)
    n_rt = -(-rows // 128)
    vals = np.zeros((n_rt * 128, n_ct * 64), np.uint16)
    kept = np.zeros(vals.shape, bool)
    for sg in range(len(seg) - 1):
        rt, ct = divmod(sg, n_ct)
        assert seg[sg] % 16 == 0
        b = data[seg[sg]:seg[sg + 1]]
        hdr = b[:16].view(np.uint16).astype(np.int64)
        blocks = b[16:1552].reshape(8, 192)
        lo = blocks[:, :64].copy().view(np.uint32)                                 # [block, piece]
        hi = blocks[:, 64:128].copy().view(np.uint32)
        olo = blocks[:, 128:160].copy().view(np.uint16).astype(np.int64)
        ohi = blocks[:, 160:192].copy().view(np.uint16).astype(np.int64)
        words = np.stack([lo, hi], axis=-1).copy().view(np.uint8).reshape(8, 16, 8)
        bits = np.unpackbits(words, axis=-1, bitorder="little").astype(bool)      # [block, piece, bit]
        n_lo = bits[:, :, :32].sum(-1)
        n_all = bits.sum(-1)
        starts = np.concatenate([[0], np.cumsum(n_all.reshape(-1))[:-1]]).reshape(8, 16)
        assert np.array_equal(olo, 2 * starts) and np.array_equal(ohi, 2 * (starts + n_lo))     # byte offsets
        assert np.array_equal(np.cumsum(n_all.sum(-1)), hdr)
        n = int(hdr[-1])
        assert len(b) == (1552 + 2 * n + 15) // 16 * 16
        assert not b[1552 + 2 * n:].any()                                          # zero padding
        v = b[1552:1552 + 2 * n].view(np.uint16)
        blk, p, bit = np.nonzero(bits)                                             # in the layout's value order
        r = rt * 128 + 16 * blk + PIECE_ROW[p, bit]
        c = ct * 64 + PIECE_COL[p, bit]
        assert not kept[r, c].any()
        kept[r, c] = True
        vals[r, c] = v
    return vals[:rows, :cols], kept[:rows, :cols]


@pytest.mark.parametrize("rows,cols,keep", [(128, 64, 36), (300, 1000, 7), (1024, 4096, 33), (17, 8, 50),
                                            (200, 5120, 90), (130, 2048, 100)])
def test_mask_layout_decodes_to_the_selection(rows, cols, keep):
    values, idx = _module(rows, cols, keep)
    data, seg = kernels.mask_build([(0, values, idx)], cols)
    got, kept = decode(data.cpu().numpy(), seg.cpu().numpy(), rows, cols)
    want = np.zeros((rows, cols), np.uint16)
    np.put_along_axis(want, idx.cpu().numpy().astype(np.int64), _bits(values), axis=1)
    mask = np.zeros((rows, cols), bool)
    np.put_along_axis(mask, idx.cpu().numpy().astype(np.int64), True, axis=1)
    assert np.array_equal(kept, mask)
    assert np.array_equal(np.where(kept, got, 0), want)
    assert data.numel() >= int(seg[-1])


def test_mask_layout_bytes_per_weight():
    """2 bytes a kept weight plus one bit a weight (the reference's storage), plus a 16-bit offset per 32 bits of mask,
    a 16-byte header a 128 x 64 segment and its padding."""
    values, idx = _module(4096, 4096, 33)
    data, seg = kernels.mask_build([(0, values, idx)], 4096)
    kept = values.numel()
    ref = kept * 2 + 4096 * 4096 // 8
    n_seg = seg.numel() - 1
    assert ref + 512 * n_seg <= int(seg[-1]) <= ref + (512 + 32) * n_seg


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("t", [1, 3, 16, 17, 31, 64, 100, 128, 129, 255, 256, 257, 272, 288, 289, 512, 600])
@pytest.mark.parametrize("rows,cols,keep", [(512, 5120, 40), (300, 1000, 7), (1024, 2048, 25), (17, 8, 50),
                                            (200, 5120, 95)])
def test_mask_matches_the_dense_matmul(dtype, t, rows, cols, keep):
    values, idx = _module(rows, cols, keep, dtype, seed=t)
    tiles = compact.Tiles([("compact", values, idx, cols)], layout="mask")
    x = torch.randn(t, cols, device="cuda").to(dtype)
    y = tiles(x)
    kernels.spmm_mask_status()
    assert y.shape == (t, rows) and y.dtype == dtype
    dt = "bf16" if dtype == torch.bfloat16 else "f16"
    _check(y, oracle.forward(_bits(x), _bits(values), idx.cpu().numpy(), cols, dt))


def test_mask_and_tc_layouts_agree_and_repeat_bit_for_bit():
    values, idx = _module(4096, 4096, 33, seed=11)
    mk = compact.Tiles([("compact", values, idx, 4096)], layout="mask")
    tc = compact.Tiles([("compact", values, idx, 4096)], layout="tc")
    for t in (17, 272):
        x = torch.randn(t, 4096, device="cuda").bfloat16()
        a, b = mk(x), mk(x)
        kernels.spmm_mask_status()
        assert torch.equal(a, b)
        r = tc(x)
        assert ((a.float() - r.float()).norm() / r.float().norm()).item() <= 1e-2


def test_mask_mixed_dense_and_compact_blocks_and_reference_blocks():
    cols = 1024
    g = torch.Generator(device="cuda").manual_seed(3)
    norms = torch.rand(cols, generator=g, device="cuda") + 0.1
    ws = [torch.randn(r, cols, generator=g, device="cuda").bfloat16() for r in (200, 72, 130)]
    w2, mask2 = wanda.prune(ws[2], 60, norms, with_mask=True)
    blocks = [("compact", *wanda.select(ws[0], 33, norms), cols), ("dense", ws[1]),
              ("sparse", *compact.pack(w2, mask2), cols)]
    tiles = compact.Tiles(blocks, layout="mask")
    assert tiles.rows == 402
    base = torch.randn(40, 2 * cols, device="cuda").bfloat16()
    x = base[:, cols // 2: cols // 2 + cols]                         # a strided view
    dense = torch.cat([compact.expand(b) for b in blocks])
    _check(tiles(x), x.double().cpu().numpy() @ dense.double().cpu().numpy().T)
    kernels.spmm_mask_status()


def test_mask_llama_shapes_at_17_and_272_tokens():
    from p2pllm_b200 import workloads
    for p in workloads.LLAMA3_8B:
        values, idx = _module(p.rows, p.cols, p.keep, seed=p.rows + p.cols)
        tiles = compact.Tiles([("compact", values, idx, p.cols)], layout="mask")
        for t in (17, 272):
            x = torch.randn(t, p.cols, device="cuda").bfloat16()
            y = tiles(x)
            kernels.spmm_mask_status()
            sample = torch.arange(0, p.rows, 97, device="cuda")
            want = oracle.forward(_bits(x), _bits(values[sample]), idx[sample].cpu().numpy(), p.cols, "bf16")
            _check(y[:, sample], want)


def test_mask_dependent_launches_see_the_previous_kernels_output():
    g = torch.Generator(device="cuda").manual_seed(9)
    mods = [compact.Tiles([("compact", *_module(4096, 4096, 33, seed=s), 4096)], layout="mask") for s in (1, 2, 3)]
    x = torch.randn(17, 4096, generator=g, device="cuda").bfloat16()
    want = x
    for m in mods:
        want = m(want)
        torch.cuda.synchronize()
    for _ in range(3):
        torch.cuda._sleep(2_000_000)
        y = x
        for m in mods:
            y = m(y)
        torch.cuda.synchronize()
        assert torch.equal(y, want)


def test_mask_on_the_benchmark_layer_at_17_and_272_tokens():
    """The benchmark's own layer (fused qkv / gate_up modules, selections from lognormal-scaled calibrations, so column
    tiles of very different density and segments of very different size): against the 4-byte layout, and sampled rows
    against the oracle. Segment sizes here once made the ring's producer place a segment at the ring's very end
    without wrapping."""
    from p2pllm_b200 import workloads
    dev = torch.device("cuda", 0)
    seeds = workloads.layer_seeds(0)
    proj = {p.name: p for p in workloads.LLAMA3_8B}
    for module, (_, names) in workloads.LAYER_MODULES.items():
        cols = proj[names[0]].cols
        g = torch.Generator(device=dev).manual_seed(seeds[module][0])
        scale = workloads.channel_scale(cols, g, dev)
        sums, _, _ = workloads.calibrate(cols, g, scale, 128 * 2048, dev)
        norms = kernels.channel_norms(sums)
        blocks = []
        for n in names:
            w = workloads.projection_weights(proj[n], seeds[module][1][n], dev)
            blocks.append(("compact", *wanda.select(w, proj[n].keep, norms), cols))
        mk = compact.Tiles(blocks, layout="mask")
        tc = compact.Tiles(blocks, layout="tc")
        values = torch.cat([b[1] for b in blocks])
        idx = torch.cat([b[2] for b in blocks])
        for t in (17, 272):
            x = (torch.randn(t, cols, generator=g, device=dev) * scale).bfloat16()
            a, b = mk(x), tc(x)
            kernels.spmm_mask_status()
            assert ((a.float() - b.float()).norm() / b.float().norm()).item() <= 1e-2
            sample = torch.arange(0, values.shape[0], 89, device=dev)
            want = oracle.forward(_bits(x), _bits(values[sample]), idx[sample].cpu().numpy(), cols, "bf16")
            _check(a[:, sample], want)
