"""Selection at BASELINE config 2's full sizes (every Llama-3-8B projection, keep 33 / 36), on the GPU:

* against the reference itself: tests/golden/llama_select.npz holds the reference's norms and the digest of each row's
  mask words from its wanda.prune + compact.pack on CPU-seeded weights (tests/golden/make_golden.py); this package's
  words must give the same digest on every row whose k-th and (k+1)-th scores differ, and the rows that tie must be the
  same rows;
* against the oracle on every row, including the ties (lower column first), both on those weights and on the weights
  and calibration the benchmark itself builds (its own calibration kernel over 128 x 2048 lognormal-scaled tokens).
The tie counts are printed (pytest -s)."""
import hashlib

import numpy as np
import pytest
import torch

import oracle
from p2pllm_b200 import kernels, wanda, workloads

pytestmark = pytest.mark.gpu


def _bits(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def _digests(words: np.ndarray) -> np.ndarray:
    words = np.ascontiguousarray(words)
    return np.array([int.from_bytes(hashlib.blake2b(r.tobytes(), digest_size=8).digest(), "little") for r in words],
                    dtype=np.uint64)


@pytest.mark.parametrize("index", range(len(workloads.LLAMA3_8B)))
def test_full_size_selection_matches_the_reference(llama_select, index):
    p = workloads.LLAMA3_8B[index]
    w_cpu, x_cpu = workloads.selection_case(p, index)
    w, x = w_cpu.cuda(), x_cpu.cuda()
    # The calibration kernel at this width, against the reference's sums (fp32 column totals, within an fp32 rounding).
    sums = torch.zeros(p.cols, dtype=torch.float64, device="cuda")
    kernels.sumsq_cols(x, sums)
    assert np.allclose(sums.cpu().numpy(), llama_select[p.name + "_sums"], rtol=1e-6, atol=0)
    norms = torch.from_numpy(llama_select[p.name + "_norms"]).cuda()
    k = int(llama_select[p.name + "_k"])
    assert k == oracle.k_of(p.keep, p.cols)
    out = kernels.wanda_select(w, norms, k, values=True, idx=True, words=True)
    score = oracle.scores(_bits(w), llama_select[p.name + "_norms"], "bf16")
    want_idx = oracle.select(score, k)
    assert np.array_equal(out["idx"].cpu().numpy().astype(np.int64), want_idx)            # every row, ties included
    ties = np.nonzero(oracle.tie_rows(score, k))[0]
    assert np.array_equal(ties, llama_select[p.name + "_tie_rows"])
    same = _digests(out["words"].cpu().numpy()) == llama_select[p.name + "_words_b2"]
    free = np.ones(p.rows, bool)
    free[ties] = False
    assert same[free].all(), np.nonzero(~same & free)[0][:10]
    print(f"{p.name} [{p.rows} x {p.cols}] keep {p.keep}: k {k}, rows tied at the k-th score {len(ties)}, "
          f"rows equal to the reference's words {int(same.sum())} of {p.rows}")


def test_the_benchmark_layers_selection_matches_the_oracle_on_every_row():
    """The selection bench.py measures: its calibration (the package's kernel over 128 x 2048 lognormal-scaled tokens
    per module input, seeded on the device) and its weights, every row against the oracle."""
    dev = torch.device("cuda", 0)
    seeds = workloads.layer_seeds(0)
    proj = {p.name: p for p in workloads.LLAMA3_8B}
    for module, (_, names) in workloads.LAYER_MODULES.items():
        cols = proj[names[0]].cols
        g = torch.Generator(device=dev).manual_seed(seeds[module][0])
        scale = workloads.channel_scale(cols, g, dev)
        sums, _, _ = workloads.calibrate(cols, g, scale, 128 * 2048, dev)
        norms = kernels.channel_norms(sums)
        for n in names:
            p = proj[n]
            w = workloads.projection_weights(p, seeds[module][1][n], dev)
            values, idx = wanda.select(w, p.keep, norms)
            score = oracle.scores(_bits(w), norms.cpu().numpy(), "bf16")
            k = oracle.k_of(p.keep, p.cols)
            assert np.array_equal(idx.cpu().numpy().astype(np.int64), oracle.select(score, k))
            want_vals = np.take_along_axis(_bits(w), idx.cpu().numpy().astype(np.int64), axis=1)
            assert np.array_equal(_bits(values), want_vals)
            print(f"bench {n} [{p.rows} x {p.cols}] keep {p.keep}: rows tied at the k-th score "
                  f"{int(oracle.tie_rows(score, k).sum())}")
