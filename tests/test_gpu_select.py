"""Wanda calibration and selection on the GPU against the oracle and the reference's fixtures: selected indices
bit-exact (ties to the lower column), calibration sums within fp32 rounding."""
import hashlib

import numpy as np
import pytest
import torch

import oracle
from p2pllm_b200 import kernels, wanda, workloads

pytestmark = pytest.mark.gpu

TORCH_DT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def _to_torch(bits: np.ndarray, dt: str, device="cuda") -> torch.Tensor:
    if dt == "f32":
        return torch.from_numpy(bits.copy()).to(device)
    return torch.from_numpy(bits.view(np.int16).copy()).view(TORCH_DT[dt]).to(device)


def _bits(t: torch.Tensor) -> np.ndarray:
    t = t.cpu()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


@pytest.mark.parametrize("dt", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("i", range(10))
def test_select_is_bit_exact(select_cases, i, dt):
    key = f"c{i}_{dt}"
    rows, cols, keep, k = (int(v) if j != 2 else float(v) for j, v in enumerate(select_cases[key + "_meta"]))
    w_bits, norms = select_cases[key + "_w"], select_cases[key + "_norms"]
    w = _to_torch(w_bits, dt)
    n = torch.from_numpy(norms).cuda()
    out = kernels.wanda_select(w, n, k, words=True, mask=True, pruned=True)
    # the oracle's stable choice, on every row
    idx = oracle.select(oracle.scores(w_bits, norms, dt), k)
    assert np.array_equal(out["idx"].cpu().numpy().astype(np.int64), idx)
    assert np.array_equal(_bits(out["values"]), np.take_along_axis(w_bits, idx, axis=1))
    mask = np.zeros((rows, cols), bool)
    np.put_along_axis(mask, idx, True, axis=1)
    assert np.array_equal(out["mask"].cpu().numpy(), mask)
    _, words = oracle.pack(w_bits, mask)
    assert np.array_equal(out["words"].cpu().numpy(), words)
    pruned, _ = oracle.prune(w_bits, keep, norms, dt)
    assert np.array_equal(_bits(out["pruned"]).view(np.uint8), pruned.view(np.uint8))
    # and the reference's own words on rows without a tie at the k-th score
    clean = ~select_cases[key + "_ties"]
    assert np.array_equal(out["words"].cpu().numpy()[clean], select_cases[key + "_words"][clean])
    if key + "_pruned" in select_cases and clean.all():
        assert np.array_equal(_bits(out["pruned"]).view(np.uint8), select_cases[key + "_pruned"].view(np.uint8))


def test_reference_unit_vectors_on_the_gpu():
    """tests/test_wanda.py:20-33 and 104-108 through the GPU prune."""
    w = torch.tensor([[1.0, -5.0, 2.0, 3.0], [4.0, 1.5, -1.0, 0.5]], device="cuda")
    assert wanda.prune(w, 50, torch.ones(4, device="cuda")).tolist() == [[0.0, -5.0, 0.0, 3.0], [4.0, 1.5, 0.0, 0.0]]
    assert (wanda.prune(torch.ones(3, 10, device="cuda"), 30, torch.ones(10, device="cuda")) != 0).sum(1).tolist() == [3] * 3
    assert wanda.prune(torch.tensor([[1.0, 2.0]], device="cuda"), 50,
                       torch.tensor([10.0, 1.0], device="cuda")).tolist() == [[1.0, 0.0]]
    w3 = torch.tensor([[[1.0, 3.0, 2.0]], [[1.0, 3.0, 2.0]]], device="cuda")
    sums = torch.tensor([[100.0, 1.0, 1.0], [0.0, 0.0, 0.0]], dtype=torch.float64, device="cuda")
    assert wanda.prune(w3, 34, wanda.channel_norms(sums, w3)).tolist() == [[[1.0, 0.0, 0.0]], [[0.0, 3.0, 0.0]]]
    w4 = torch.ones(2, 3, 4, device="cuda")
    s4 = torch.tensor([[9.0, 1, 1, 1], [1, 1, 1, 9.0]], dtype=torch.float64, device="cuda")
    got = wanda.prune(w4, 25, wanda.channel_norms(s4, w4))
    assert got.sum().item() == 6 and got[0, :, 0].sum().item() == 3 and got[1, :, 3].sum().item() == 3


class FakeGroup:
    """all_gather across ranks living in this process (tests/test_wanda.py:10-17)."""

    def __init__(self, parts, rank):
        self.parts, self.rank_in_group = parts, rank

    def all_gather(self, x, dim=0):
        return torch.cat([x if r == self.rank_in_group else p for r, p in enumerate(self.parts)], dim)


def test_row_parallel_ranks_choose_as_one_matrix():
    """tests/test_wanda.py:45-53: a projection split over TP ranks prunes as the whole."""
    g = torch.Generator(device="cuda").manual_seed(1)
    w, norms = torch.randn(20, 100, generator=g, device="cuda"), torch.rand(100, generator=g, device="cuda")
    whole = wanda.prune(w, 33, norms)
    cols = [w[:, :50].contiguous(), w[:, 50:].contiguous()]
    ns = [norms[:50].contiguous(), norms[50:].contiguous()]
    got = []
    for r in range(2):
        # the fake group gathers whatever it is given per rank: weights, then norms
        class G(FakeGroup):
            def all_gather(self, x, dim=0, _r=r):
                src = cols if x.shape[-1] == 50 and x.dim() == 2 else ns
                return torch.cat([x if q == _r else src[q] for q in range(2)], dim)
        got.append(wanda.prune(cols[r], 33, ns[r], G(None, r)))
    assert torch.equal(torch.cat(got, 1), whole)


def test_config1_on_the_gpu_matches_the_reference(config1_golden):
    """calibration on the GPU (16 hook calls), norms, the selection's mask words and values hashed
    against the reference's, and the fp32 forward within rel-L2 1e-5 of the reference's F.linear."""
    cfg = workloads.config1(seed=0)
    sums = torch.zeros(cfg.w.shape[1], dtype=torch.float64, device="cuda")
    for chunk in cfg.calib_chunks("cuda"):
        kernels.sumsq_cols(chunk, sums)
    ref_sums = config1_golden["sums"]
    got = sums.cpu().numpy()
    assert np.allclose(got, ref_sums, rtol=1e-6, atol=0)
    norms = wanda.channel_norms(torch.from_numpy(ref_sums), cfg.w.cuda())
    assert np.array_equal(norms.cpu().numpy(), config1_golden["norms"])
    w = cfg.w.cuda()
    k = int(config1_golden["k"])
    out = kernels.wanda_select(w, norms, k, words=True)
    assert hashlib.sha256(out["words"].cpu().numpy().tobytes()).hexdigest() == str(config1_golden["words_sha256"])
    assert hashlib.sha256(out["values"].cpu().numpy().tobytes()).hexdigest() == str(config1_golden["values_sha256"])
    y = kernels.spmm_rows(cfg.x.cuda(), [(0, out["values"], out["idx"])], w.shape[1], w.shape[0])
    want = config1_golden["y"].astype(np.float64)
    rel = np.linalg.norm(y.cpu().numpy() - want) / np.linalg.norm(want)
    assert rel <= 1e-5, rel


@pytest.mark.parametrize("dt", ["bf16", "f32", "f16"])
@pytest.mark.parametrize("shape", [(1, 7), (3, 4096), (1000, 4096), (70000, 2048), (5, 9), (257, 1000)])
def test_sumsq_matches_the_oracle(dt, shape):
    g = torch.Generator(device="cuda").manual_seed(shape[0])
    x = (torch.randn(*shape, generator=g, device="cuda") * 3).to(TORCH_DT[dt])
    sums = torch.zeros(shape[1], dtype=torch.float64, device="cuda")
    kernels.sumsq_cols(x, sums)
    kernels.sumsq_cols(x, sums)                   # a second call adds, and finds its workspace zeroed again
    want = 2 * oracle.sumsq_cols(_bits(x), dt)
    assert np.allclose(sums.cpu().numpy(), want, rtol=2e-6, atol=0)


def test_sumsq_strided_and_misaligned_rows():
    x = torch.randn(300, 515, device="cuda")[:, 3:]          # row stride 515, start off 16-byte alignment
    sums = torch.zeros(512, dtype=torch.float64, device="cuda")
    kernels.sumsq_cols(x, sums)
    assert np.allclose(sums.cpu().numpy(), oracle.sumsq_cols(x.cpu().numpy()), rtol=1e-6)


def test_sumsq_calls_of_different_shapes_share_a_workspace():
    """A call with more column strips after one with fewer must find its counters zero (they live apart from the
    partials)."""
    shapes = [(100000, 4096, torch.bfloat16), (30000, 16384, torch.float32), (50000, 1024, torch.float16),
              (30000, 16384, torch.float32)]
    for rows, cols, dt in shapes:
        x = torch.randn(rows, cols, device="cuda").to(dt)
        sums = torch.zeros(cols, dtype=torch.float64, device="cuda")
        kernels.sumsq_cols(x, sums)
        want = x.double().pow(2).sum(0)
        assert torch.allclose(sums, want, rtol=1e-5, atol=0), (rows, cols, dt)


def test_sumsq_is_deterministic():
    x = torch.randn(100000, 1024, device="cuda").bfloat16()
    a = torch.zeros(1024, dtype=torch.float64, device="cuda")
    b = torch.zeros(1024, dtype=torch.float64, device="cuda")
    kernels.sumsq_cols(x, a)
    kernels.sumsq_cols(x, b)
    assert torch.equal(a, b)


def test_expert_inputs_match_the_reference(expert_golden):
    import types
    g = expert_golden
    m = types.SimpleNamespace(w13_weight=torch.from_numpy(g["w13"]).cuda(),
                              w2_weight=torch.zeros(g["w13"].shape[0], g["w13"].shape[2], g["gated"].shape[1],
                                                    device="cuda"))
    into, gated = wanda.expert_inputs(m, torch.from_numpy(g["x"]).cuda(), torch.from_numpy(g["ids"]).cuda())
    assert np.allclose(into.cpu().numpy(), g["into"], rtol=1e-6, atol=0)
    assert np.allclose(gated.cpu().numpy(), g["gated"], rtol=1e-5, atol=1e-9)


def test_calibration_hooks_collect_sums():
    class Layer(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.q_proj = torch.nn.Linear(64, 64, bias=False)
            self.gate_proj = torch.nn.Linear(64, 128, bias=False)
            self.up_proj = torch.nn.Linear(64, 128, bias=False)
            self.down_proj = torch.nn.Linear(128, 64, bias=False)

        def forward(self, h):
            return h + self.down_proj(self.gate_proj(h) * self.up_proj(self.q_proj(h)))

    layers = torch.nn.ModuleList([Layer(), Layer()]).cuda()
    cal = wanda.Calibration(layers)
    xs = [torch.randn(16, 64, device="cuda") for _ in range(3)]
    with torch.no_grad():
        for x in xs:
            for layer in layers:
                x = layer(x)
    sums = cal.finish(layers)
    assert set(sums) == {(i, p) for i in range(2) for p in ("q_proj", "gate_proj", "up_proj", "down_proj")}
    x0 = torch.cat(xs).float()
    assert torch.allclose(sums[0, "q_proj"], x0.pow(2).sum(0).double().cpu(), rtol=1e-5)
