"""The tensor-core layout and the tcgen05 compact GEMM on the GPU: the layout decodes back to the oracle's selection
bit for bit, and the GEMM matches the oracle's dense masked matmul (rel-L2 <= 1e-2 for bf16/f16, the reference's
max|d| <= 1e-2 max|want| too) over token counts 1..600, odd shapes, mixed dense/compact blocks and split columns."""
import numpy as np
import pytest
import torch

import oracle
from p2pllm_b200 import _lib, compact, kernels, wanda

pytestmark = pytest.mark.gpu


def _bits(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def _module(rows, cols, keep, dtype=torch.bfloat16, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = (torch.randn(rows, cols, generator=g, device="cuda") * 0.02).to(dtype)
    norms = torch.rand(cols, generator=g, device="cuda") + 0.1
    values, idx = wanda.select(w, keep, norms)
    return values, idx


def _check(got, want, dtype):
    got = got.double().cpu().numpy() if torch.is_tensor(got) else got
    rel = np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30)
    assert rel <= 1e-2, rel
    assert np.abs(got - want).max() <= 1e-2 * np.abs(want).max()


@pytest.mark.parametrize("rows,cols,keep", [(128, 64, 36), (300, 1000, 7), (1024, 4096, 33), (17, 8, 50),
                                            (200, 5120, 90)])
def test_layout_decodes_to_the_selection(rows, cols, keep):
    """Every segment: a header of cumulative 8-row-group counts, then one word per kept weight holding its value and
    its swizzled byte offset in the 128 x 64 tile, 32-row slice after slice, each slice dealt to the GEMM's store rounds
    so that each store round holds as few entries of any one shared-memory bank as the slice's remaining entries allow
    (the smallest m with sum over banks of min(left, m) >= the round's places); decoded, the layout is the selection,
    bit for bit."""
    values, idx = _module(rows, cols, keep)
    words, seg, cap = kernels.tiles_build([(0, values, idx)], cols)
    w = words.cpu().numpy().view(np.uint32)
    s = seg.cpu().numpy()
    n_ct = -(-cols // 64)
    got = np.zeros((rows, cols), np.uint16)
    seen = np.zeros((rows, cols), np.int32)
    for i in range(len(s) - 1):
        assert s[i] % 4 == 0 and s[i + 1] >= s[i] + 8
        rt, ct = divmod(i, n_ct)
        hdr = np.stack([w[s[i]:s[i] + 8] & 0xFFFF, w[s[i]:s[i] + 8] >> 16], axis=1).reshape(16)
        assert (np.diff(hdr) >= 0).all()
        count = int(hdr[15])
        assert s[i + 1] - s[i] == 8 + ((count + 3) & ~3)
        ents = w[s[i] + 8:s[i] + 8 + count].astype(np.int64)
        off = ents & 0x3FFF
        assert (off % 2 == 0).all()
        r = off >> 7
        c = ((((off >> 4) & 7) ^ (r & 7)) << 3) | ((off & 15) >> 1)
        sl = r // 32
        e = np.arange(count)
        bounds = np.concatenate([[0], hdr[3::4]])                   # slice s: [hdr[4s-1], hdr[4s+3])
        assert ((bounds[sl] <= e) & (e < bounds[sl + 1])).all()
        bank = (off >> 2) & 31
        for q in range(4):                                          # each slice's store rounds, in order
            first = s[i] + 8 + bounds[q]
            pr = np.arange(bounds[q + 1] - bounds[q]) + (first & 3)  # places above the 4-word boundary
            rnd = np.where(pr < 1024, (pr >> 7) * 4 + (pr & 3), 32 + ((pr - 1024) >> 5))
            b = bank[bounds[q]:bounds[q + 1]]
            left = np.bincount(b, minlength=32)
            for R in np.unique(rnd):
                here = np.bincount(b[rnd == R], minlength=32)
                m = 1
                while np.minimum(left, m).sum() < here.sum():
                    m += 1
                assert here.max() == m
                left -= here
        np.add.at(seen, (rt * 128 + r, ct * 64 + c), 1)
        got[rt * 128 + r, ct * 64 + c] = (ents >> 16).astype(np.uint16)
    assert cap == int(np.diff(s).max())
    want = np.zeros((rows, cols), np.uint16)
    np.put_along_axis(want, idx.cpu().numpy().astype(np.int64), _bits(values), axis=1)
    mask = np.zeros((rows, cols), bool)
    np.put_along_axis(mask, idx.cpu().numpy().astype(np.int64), True, axis=1)
    assert np.array_equal(seen, mask.astype(np.int32))
    assert np.array_equal(got, want)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("t", [1, 3, 16, 17, 31, 64, 100, 255, 256, 257, 272, 512, 513, 600])
@pytest.mark.parametrize("rows,cols,keep", [(512, 5120, 40), (300, 1000, 7), (1024, 2048, 25), (17, 8, 50),
                                            (200, 5120, 95)])
def test_tc_matches_the_dense_matmul(dtype, t, rows, cols, keep):
    values, idx = _module(rows, cols, keep, dtype, seed=t)
    tiles = compact.Tiles([("compact", values, idx, cols)])
    assert tiles.layout == "tc"
    x = torch.randn(t, cols, device="cuda").to(dtype)
    y = tiles(x)
    kernels.spmm_tc_status()
    assert y.shape == (t, rows) and y.dtype == dtype
    dt = "bf16" if dtype == torch.bfloat16 else "f16"
    want = oracle.forward(_bits(x), _bits(values), idx.cpu().numpy(), cols, dt)
    _check(y, want, dtype)


def test_tc_and_rows_layouts_agree_and_repeat_bit_for_bit():
    values, idx = _module(4096, 4096, 33, seed=11)
    tc = compact.Tiles([("compact", values, idx, 4096)])
    rows = compact.Tiles([("compact", values, idx, 4096)], layout="rows")
    for t in (17, 272):
        x = torch.randn(t, 4096, device="cuda").bfloat16()
        a, b = tc(x), tc(x)
        kernels.spmm_tc_status()
        assert torch.equal(a, b)                                   # split partials are added in a fixed order
        r = rows(x)
        assert ((a.float() - r.float()).norm() / r.float().norm()).item() <= 1e-2


def test_tc_mixed_dense_and_compact_blocks_in_row_order():
    """A fused qkv-like module: compact, dense and compact blocks of different k (tests/test_compact.py:27-36)."""
    cols = 1024
    g = torch.Generator(device="cuda").manual_seed(3)
    norms = torch.rand(cols, generator=g, device="cuda") + 0.1
    ws = [torch.randn(r, cols, generator=g, device="cuda").bfloat16() for r in (200, 72, 130)]
    blocks = [("compact", *wanda.select(ws[0], 33, norms), cols), ("dense", ws[1]),
              ("compact", *wanda.select(ws[2], 60, norms), cols)]
    tiles = compact.Tiles(blocks)
    assert tiles.layout == "tc" and tiles.rows == 402
    x = torch.randn(40, cols, device="cuda").bfloat16()
    dense = torch.cat([compact.expand(b) for b in blocks])
    want = x.double().cpu().numpy() @ dense.double().cpu().numpy().T
    _check(tiles(x), want, torch.bfloat16)
    kernels.spmm_tc_status()


def test_tc_reference_blocks_and_strided_x():
    """The reference's ("sparse", values, words, cols) blocks load into the tensor-core layout; x may be a strided view."""
    (w, mask) = wanda.prune(torch.randn(256, 2048, device="cuda").bfloat16(), 36,
                            torch.rand(2048, device="cuda") + 0.1, with_mask=True)
    values, words = compact.pack(w, mask)
    tiles = compact.Tiles([("sparse", values, words, 2048)])
    base = torch.randn(17, 4096, device="cuda").bfloat16()
    x = base[:, 1024:3072]                                         # row stride 4096
    want = x.double().cpu().numpy() @ w.double().cpu().numpy().T
    _check(tiles(x), want, torch.bfloat16)
    kernels.spmm_tc_status()


def test_llama_shapes_at_17_and_272_tokens():
    """The configuration the bench runs: each Llama-3-8B projection shape at keep 33/36, against the oracle on a
    sample of rows (every token)."""
    from p2pllm_b200 import workloads
    for p in workloads.LLAMA3_8B:
        values, idx = _module(p.rows, p.cols, p.keep, seed=p.rows + p.cols)
        tiles = compact.Tiles([("compact", values, idx, p.cols)])
        for t in (17, 272):
            x = torch.randn(t, p.cols, device="cuda").bfloat16()
            y = tiles(x)
            kernels.spmm_tc_status()
            sample = torch.arange(0, p.rows, 97, device="cuda")
            want = oracle.forward(_bits(x), _bits(values[sample]), idx[sample].cpu().numpy(), p.cols, "bf16")
            _check(y[:, sample], want, torch.bfloat16)


@pytest.mark.parametrize("t", [1, 17, 100, 256, 272, 300])
@pytest.mark.parametrize("rows,cols,keep", [(19000, 1000, 7), (28772, 640, 40), (40000, 64, 50), (20000, 200, 30)])
def test_persistent_runs_match_the_dense_matmul(t, rows, cols, keep):
    """Modules of more row tiles than SMs run as one CTA an SM, each a contiguous run of (row tile, column tile) units
    across row tiles: runs shorter and longer than a row tile, a ragged last row tile, a single column tile (every row
    tile whole in its run), both accumulator layouts (N <= 256: one per issuer; above: one shared). Against the oracle
    on a sample of rows and the last rows; a second call repeats the first bit for bit (the shared row tiles' partials
    are added in run order, and their tickets are left zero)."""
    values, idx = _module(rows, cols, keep, seed=rows + t)
    tiles = compact.Tiles([("compact", values, idx, cols)])
    x = torch.randn(t, cols, device="cuda").bfloat16()
    y = tiles(x)
    kernels.spmm_tc_status()
    sample = torch.cat([torch.arange(0, rows, 37, device="cuda"), torch.arange(rows - 130, rows, device="cuda")])
    want = oracle.forward(_bits(x), _bits(values[sample]), idx[sample].cpu().numpy(), cols, "bf16")
    _check(y[:, sample], want, torch.bfloat16)
    assert torch.equal(tiles(x), y)
    kernels.spmm_tc_status()


@pytest.mark.parametrize("t", [17, 64])
def test_persistent_runs_in_f16(t):
    """The run instantiation for f16 weights (a module of 160 row tiles, ragged last one), against the oracle."""
    rows, cols = 20400, 512
    values, idx = _module(rows, cols, 33, torch.float16, seed=t)
    tiles = compact.Tiles([("compact", values, idx, cols)])
    x = torch.randn(t, cols, device="cuda").half()
    y = tiles(x)
    kernels.spmm_tc_status()
    sample = torch.cat([torch.arange(0, rows, 29, device="cuda"), torch.arange(rows - 70, rows, device="cuda")])
    want = oracle.forward(_bits(x), _bits(values[sample]), idx[sample].cpu().numpy(), cols, "f16")
    _check(y[:, sample], want, torch.float16)


def test_split_launches_of_different_shapes_share_a_workspace():
    """Column-split launches with few row tiles, then many: each finds its ticket counters zero."""
    for rows, cols in ((256, 4096), (14336, 4096), (512, 14336), (28672, 4096)):
        values, idx = _module(rows, cols, 36, seed=rows)
        tiles = compact.Tiles([("compact", values, idx, cols)])
        x = torch.randn(17, cols, device="cuda").bfloat16()
        y = tiles(x)
        kernels.spmm_tc_status()
        sample = torch.arange(0, rows, 61, device="cuda")
        want = oracle.forward(_bits(x), _bits(values[sample]), idx[sample].cpu().numpy(), cols, "bf16")
        _check(y[:, sample], want, torch.bfloat16)


def test_dependent_launches_see_the_previous_kernels_output():
    """Each launch is a programmatic dependent of the stream's previous kernel and may start before it ends; its x
    loads wait for it. Chained modules (B on A's output) and x rewritten in place just before a launch must give the
    same bits as runs separated by a synchronize."""
    g = torch.Generator(device="cuda").manual_seed(9)
    mods = []
    for seed in (1, 2, 3):
        values, idx = _module(4096, 4096, 33, seed=seed)
        mods.append(compact.Compact([("compact", values, idx, 4096)]))
    x = torch.randn(17, 4096, generator=g, device="cuda").bfloat16()
    want = x
    steps = []
    for m in mods:                                          # the reference: one module at a time, synchronised
        want = m.apply(None, want)
        torch.cuda.synchronize()
        steps.append(want.clone())
    for _ in range(3):
        torch.cuda._sleep(2_000_000)                        # the host queues the chain while the GPU is busy
        y = x
        for m in mods:
            y = m.apply(None, y)
        torch.cuda.synchronize()
        assert torch.equal(y, steps[-1])
    # an in-place torch kernel on x right before a launch
    m = mods[0]
    for scale in (2.0, -0.5, 3.0):
        x2 = x.clone()
        torch.cuda.synchronize()
        torch.cuda._sleep(1_000_000)
        x2.mul_(scale)
        got = m.apply(None, x2)
        torch.cuda.synchronize()
        assert torch.equal(got, m.apply(None, (x * scale)))


@pytest.mark.parametrize("tokens", [17, 100])
def test_a_withheld_tile_in_persistent_runs_ends_with_an_error_status(tokens):
    """The give-up path of the persistent runs (a module of 149 row tiles, one CTA an SM): every run withholds its
    first x tile, so its MMAs, the zero copies into the A slots, the expanders and the row tiles' read-outs all stop
    at bounded waits. The launch ends by itself, the status names a wait, and the next launch through the same
    workspace (re-zeroed by the status check: a stopped run may leave a row tile's ticket taken) is right and
    repeats bit for bit."""
    import time
    from p2pllm_b200._lib import P2PError
    rows, cols = 19000, 1024
    values, idx = _module(rows, cols, 36, seed=11)
    tiles = compact.Tiles([("compact", values, idx, cols)])
    x = torch.randn(tokens, cols, device="cuda").bfloat16()
    y = tiles(x)                                                    # the workspace cached for this stream
    kernels.spmm_tc_status(reset=True)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    kernels.spmm_tc_withhold(x, tiles.words, tiles.seg, tiles.rows, tiles.cols, tiles.seg_cap, hold_tile=0,
                             wait_us=20000)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 1.0
    with pytest.raises(P2PError, match="timed out"):
        kernels.spmm_tc_status(reset=True)
    kernels.spmm_tc_status()
    need = _lib.load().p2p_spmm_tc_workspace(rows, cols, tokens)
    assert need > 0                                                 # the runs' ticket counters and partials
    assert int(torch.count_nonzero(kernels._workspace(x.device, need, "spmm_tc"))) == 0
    again = tiles(x)
    kernels.spmm_tc_status()
    assert torch.equal(again, y)
    sample = torch.cat([torch.arange(0, rows, 41, device="cuda"), torch.arange(rows - 130, rows, device="cuda")])
    want = oracle.forward(_bits(x), _bits(values[sample]), idx[sample].cpu().numpy(), cols, "bf16")
    _check(again[:, sample], want, torch.bfloat16)


@pytest.mark.parametrize("tokens", [17, 272])
def test_a_withheld_tile_ends_the_launch_with_an_error_status(tokens):
    """Failure detection without a fault: every CTA withholds one x tile (it is never loaded), so the waits for it run
    out after 20 ms of %globaltimer. The launch must end by itself (drained: no copy or MMA left in flight), the status
    must name the wait that gave up, and the context must stay usable: the next ordinary launch gives the right
    product, and a wait of that launch is not cut short by the earlier give-up."""
    import time
    from p2pllm_b200._lib import P2PError
    values, idx = _module(256, 1024, 36, seed=5)
    tiles = compact.Tiles([("compact", values, idx, 1024)])
    x = torch.randn(tokens, 1024, device="cuda").bfloat16()
    kernels.spmm_tc_status(reset=True)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    kernels.spmm_tc_withhold(x, tiles.words, tiles.seg, tiles.rows, tiles.cols, tiles.seg_cap, hold_tile=0,
                             wait_us=20000)
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert elapsed < 1.0, elapsed                                   # the 20 ms limit, plus the drain, not 2 s
    with pytest.raises(P2PError, match="timed out"):
        kernels.spmm_tc_status(reset=True)
    kernels.spmm_tc_status()                                        # reset: clean again
    y = tiles(x)
    kernels.spmm_tc_status()
    want = oracle.forward(_bits(x), _bits(values), idx.cpu().numpy(), 1024, "bf16")
    _check(y, want, torch.bfloat16)
