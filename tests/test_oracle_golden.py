"""The CPU oracle pinned against the reference: its own unit-test vectors and the fixtures tests/golden/make_golden.py
made by running the reference's p2p.wanda / p2p.compact / p2p.replica / p2p.route. No GPU."""
import hashlib

import numpy as np
import pytest
import torch

import oracle
from p2pllm_b200 import workloads

N_SELECT = 10


def _case(cases, i, dt):
    key = f"c{i}_{dt}"
    rows, cols, keep, k = cases[key + "_meta"]
    return key, int(rows), int(cols), float(keep), int(k)


# --- the reference's own vectors: tests/test_wanda.py ----------------------------------------------------------------

def test_keeps_the_top_scores_in_each_row():
    """tests/test_wanda.py:20-23."""
    w = np.array([[1.0, -5.0, 2.0, 3.0], [4.0, 1.5, -1.0, 0.5]], dtype=np.float32)
    pruned, _ = oracle.prune(w, 50, np.ones(4, np.float32))
    assert pruned.tolist() == [[0.0, -5.0, 0.0, 3.0], [4.0, 1.5, 0.0, 0.0]]


def test_ties_keep_exactly_k_weights():
    """tests/test_wanda.py:26-28, and which ones: the lowest columns."""
    pruned, mask = oracle.prune(np.ones((3, 10), np.float32), 30, np.ones(10, np.float32))
    assert (pruned != 0).sum(1).tolist() == [3, 3, 3]
    assert mask[:, :3].all() and not mask[:, 3:].any()


def test_norms_change_what_is_kept():
    """tests/test_wanda.py:31-33."""
    pruned, _ = oracle.prune(np.array([[1.0, 2.0]], np.float32), 50, np.array([10.0, 1.0], np.float32))
    assert pruned.tolist() == [[1.0, 0.0]]


def test_each_expert_is_pruned_on_its_own_inputs():
    """tests/test_wanda.py:60-64."""
    w = np.ones((2, 3, 4), np.float32)
    sums = np.array([[9.0, 1, 1, 1], [1, 1, 1, 9.0]])
    pruned, _ = oracle.prune(w, 25, oracle.channel_norms(sums))
    assert pruned.sum() == 6 and pruned[0, :, 0].sum() == 3 and pruned[1, :, 3].sum() == 3


def test_an_expert_no_token_reached_keeps_its_largest_weights():
    """tests/test_wanda.py:104-108."""
    w = np.array([[[1.0, 3.0, 2.0]], [[1.0, 3.0, 2.0]]], np.float32)
    sums = np.array([[100.0, 1.0, 1.0], [0.0, 0.0, 0.0]])
    pruned, _ = oracle.prune(w, 34, oracle.channel_norms(sums))
    assert pruned.tolist() == [[[1.0, 0.0, 0.0]], [[0.0, 3.0, 0.0]]]


def test_row_parallel_norms_slice():
    """tests/test_wanda.py:55-58: norms are sqrt of the sums."""
    assert oracle.channel_norms(np.array([1.0, 4.0, 9.0, 16.0]))[2:].tolist() == [3.0, 4.0]


@pytest.mark.parametrize("keep,cols,k", [(33, 200, 66), (40, 2048, 819), (33, 4096, 1352), (36, 4096, 1475),
                                         (36, 14336, 5161), (40, 5120, 2048), (40, 27648, 11059), (30, 2048, 614),
                                         (30, 768, 230), (50, 5, 2), (50, 3, 2), (5, 10, 1), (0.1, 10, 1)])
def test_k_follows_python_round(keep, cols, k):
    """k = max(1, round(keep / 100 * cols)) with banker's rounding (p2p/wanda.py:82); the figures of the configs."""
    assert oracle.k_of(keep, cols) == k


# --- fixtures made by the reference ---------------------------------------------------------------------------------

@pytest.mark.parametrize("dt", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("i", range(N_SELECT))
def test_select_matches_the_reference_prune_and_pack(select_cases, i, dt):
    """The oracle's selection, values and mask words equal wanda.prune + compact.pack on every row without a tie at
    the k-th place; on tie rows it keeps the same number and the lower columns."""
    key, rows, cols, keep, k = _case(select_cases, i, dt)
    w = select_cases[key + "_w"]
    norms = select_cases[key + "_norms"]
    ties = select_cases[key + "_ties"]
    assert oracle.k_of(keep, cols) == k
    s = oracle.scores(w, norms, dt)
    idx = oracle.select(s, k)
    assert idx.shape == (rows, k) and (np.diff(idx, axis=1) > 0).all()
    ref_idx = oracle.words_to_idx(select_cases[key + "_words"], cols)
    clean = ~ties
    assert np.array_equal(idx[clean], ref_idx[clean])
    # The same kept values on clean rows, in column order.
    values = np.take_along_axis(w, idx, axis=1)
    assert np.array_equal(values[clean], select_cases[key + "_values"][clean])
    # Mask words of the oracle's own choice round-trip through pack / unpack.
    mask = np.zeros((rows, cols), bool)
    np.put_along_axis(mask, idx, True, axis=1)
    v2, words = oracle.pack(w, mask)
    assert np.array_equal(v2, values)
    assert np.array_equal(words[clean], select_cases[key + "_words"][clean])
    assert np.array_equal(oracle.words_to_idx(words, cols), idx)
    if key + "_pruned" in select_cases and clean.all():
        pruned, _ = oracle.prune(w, keep, norms, dt)
        assert np.array_equal(pruned.view(np.uint8), select_cases[key + "_pruned"].view(np.uint8))


def test_ties_are_exercised(select_cases):
    """The coarse-norm cases really do tie at the k-th place somewhere, so the tie rule is tested."""
    n = sum(int(select_cases[f"c{i}_{dt}_ties"].sum()) for i in range(N_SELECT) for dt in ("f32", "bf16", "f16"))
    assert n > 0


def test_config1_selection_and_forward_match_the_reference(config1_golden):
    """BASELINE config 1 end to end on the CPU: calibration sums, norms, selection (hash of the reference's mask words
    and values) and the forward against the reference's F.linear of the unpacked matrix."""
    cfg = workloads.config1(seed=0)
    sums = np.zeros(cfg.w.shape[1])
    for chunk in cfg.calib_chunks():
        sums += oracle.sumsq_cols(chunk.numpy())
    ref_sums = config1_golden["sums"]
    assert np.allclose(sums, ref_sums, rtol=1e-6, atol=0)
    norms = oracle.channel_norms(ref_sums)
    assert np.array_equal(norms, config1_golden["norms"])
    w = cfg.w.numpy()
    k = int(config1_golden["k"])
    assert k == oracle.k_of(cfg.keep, w.shape[1]) == 819
    s = oracle.scores(w, norms)
    assert int(config1_golden["tie_rows"]) == int(oracle.tie_rows(s, k).sum()) == 0
    idx = oracle.select(s, k)
    mask = np.zeros(w.shape, bool)
    np.put_along_axis(mask, idx, True, axis=1)
    values, words = oracle.pack(w, mask)
    assert hashlib.sha256(words.tobytes()).hexdigest() == str(config1_golden["words_sha256"])
    assert hashlib.sha256(values.tobytes()).hexdigest() == str(config1_golden["values_sha256"])
    y = oracle.forward(cfg.x.numpy(), values, idx, w.shape[1])
    want = config1_golden["y"].astype(np.float64)
    assert np.linalg.norm(y - want) / np.linalg.norm(want) <= 1e-5


@pytest.mark.parametrize("dt", ["bf16", "f32", "f16"])
@pytest.mark.parametrize("n", [2, 3, 5])
def test_combine_and_summed_match_the_reference(combine_golden, n, dt):
    """replica._member's combine (p2p/replica.py:81-85) and route._summed (p2p/route.py:825-831), bit for bit."""
    key = f"n{n}_{dt}"
    parts = [combine_golden[key + f"_p{j}"] for j in range(n)]
    out = oracle.combine(parts, combine_golden[key + "_h"], combine_golden[key + "_hc"], dt)
    assert np.array_equal(out.view(np.uint8), combine_golden[key + "_out"].view(np.uint8))
    s = oracle.summed(parts, dt)
    assert np.array_equal(s.view(np.uint8), combine_golden[key + "_summed"].view(np.uint8))


def test_expert_inputs_match_the_reference(expert_golden):
    """wanda.expert_inputs: a token routed twice counts once, an unrouted expert stays zero."""
    g = expert_golden
    into, gated = oracle.expert_inputs(g["x"], g["ids"], g["w13"], g["gated"].shape[1])
    assert np.allclose(into, g["into"], rtol=1e-6, atol=0)
    assert np.allclose(gated, g["gated"], rtol=1e-5, atol=1e-9)
    assert (into[-1] == 0).all() and (g["into"][-1] == 0).all()


def test_bf16_conversions_round_to_nearest_even():
    f = np.array([1.0, 1.00390625, 1.01171875, -3.5, 65504.0, np.inf, -0.0], np.float32)
    assert np.array_equal(oracle.f32_to_bf16(f), torch.tensor(f).bfloat16().view(torch.int16).numpy().view(np.uint16))
    r = np.random.default_rng(0).standard_normal(10000).astype(np.float32)
    assert np.array_equal(oracle.f32_to_bf16(r), torch.tensor(r).bfloat16().view(torch.int16).numpy().view(np.uint16))


def test_oracle_selection_at_full_size_matches_the_reference_words(llama_select):
    """The oracle against the reference's own full-size selection (tests/golden/llama_select.npz): on the k projection
    (1024 x 4096, keep 33) every row's mask words, rebuilt from the oracle's indices, digest the same as the
    reference's, except the rows that tie at the k-th score."""
    import hashlib
    import torch
    from p2pllm_b200 import workloads
    index = [p.name for p in workloads.LLAMA3_8B].index("k")
    p = workloads.LLAMA3_8B[index]
    w, _ = workloads.selection_case(p, index)
    bits = w.view(torch.int16).numpy().view(np.uint16)
    score = oracle.scores(bits, llama_select["k_norms"], "bf16")
    k = int(llama_select["k_k"])
    idx = oracle.select(score, k)
    mask = np.zeros((p.rows, p.cols), bool)
    np.put_along_axis(mask, idx, True, axis=1)
    _, words = oracle.pack(bits, mask)
    dig = np.array([int.from_bytes(hashlib.blake2b(np.ascontiguousarray(r).tobytes(), digest_size=8).digest(),
                                   "little") for r in words], dtype=np.uint64)
    ties = set(llama_select["k_tie_rows"].tolist())
    same = dig == llama_select["k_words_b2"]
    assert all(same[r] for r in range(p.rows) if r not in ties)
    assert set(np.nonzero(oracle.tie_rows(score, k))[0].tolist()) == ties
