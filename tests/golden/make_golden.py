"""Writes the golden fixtures of tests/golden/ by running the reference p2pLLM itself (p2p.wanda, p2p.compact,
p2p.replica, p2p.route) on seeded inputs. Runs only where the reference source tree is present:

    P2P_REFERENCE=<path to the p2pLLM checkout> python tests/golden/make_golden.py

p2p.replica imports SGLang's residual-stream helper at module level; a stub providing the two calls it makes is put in
sys.modules, as the reference's own tests/test_sglang.py:214-218 monkeypatches them (set_written returns x,
stream_of(...).export returns (out, None)).
"""
from __future__ import annotations

import hashlib
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from p2pllm_b200 import workloads  # noqa: E402


def _reference():
    root = os.environ.get("P2P_REFERENCE")
    if not root or not os.path.isdir(os.path.join(root, "p2p")):
        raise SystemExit("set P2P_REFERENCE to the p2pLLM source tree")
    sys.path.insert(0, root)
    stream = types.SimpleNamespace(export=lambda out: (out, None))
    batch = types.SimpleNamespace(set_written=lambda x, fb: x, stream_of=lambda fb: stream)
    for name in ("sglang", "sglang.srt", "sglang.srt.layers", "sglang.srt.layers.layer_boundary"):
        sys.modules.setdefault(name, types.ModuleType(name))
    residual = types.ModuleType("sglang.srt.layers.layer_boundary.residual")
    residual.batch = batch
    sys.modules["sglang.srt.layers.layer_boundary.residual"] = residual
    from p2p import compact, replica, route, wanda
    return wanda, compact, replica, route


def bits(t: torch.Tensor) -> np.ndarray:
    """A tensor's raw storage: bf16/f16 as uint16, fp32 as float32."""
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


DT = {torch.float32: "f32", torch.bfloat16: "bf16", torch.float16: "f16"}

# (rows, cols, keep) of the reference's tests/test_compact.py:19 and :46, plus shapes with ties and odd sizes.
SELECT_SHAPES = [(64, 64, 50), (100, 77, 7), (30, 1000, 90), (8, 33, 5), (17, 8, 50), (40, 1000, 7), (96, 80, 90),
                 (64, 512, 33), (32, 1000, 36), (2, 40000, 40)]


def select_cases(wanda, compact) -> dict:
    out = {}
    for i, (rows, cols, keep) in enumerate(SELECT_SHAPES):
        for dtype in (torch.float32, torch.bfloat16, torch.float16):
            g = torch.Generator().manual_seed(1000 + i)
            w = torch.randn(rows, cols, generator=g).to(dtype)
            norms = torch.rand(cols, generator=g) + 0.1
            if i % 3 == 1:                       # coarse norms: many equal scores, so ties at the k-th place
                norms = (norms * 4).round() / 4 + 0.25
            pruned, mask = wanda.prune(w, keep, norms, with_mask=True)
            values, words = compact.pack(pruned, mask)
            score = w.float().abs() * norms
            k = max(1, round(keep / 100 * cols))
            srt = score.sort(dim=-1, descending=True).values
            ties = (srt[:, k - 1] == srt[:, k]).numpy() if k < cols else np.zeros(rows, bool)
            key = f"c{i}_{DT[dtype]}"
            out[key + "_w"] = bits(w)
            out[key + "_norms"] = norms.numpy()
            out[key + "_meta"] = np.array([rows, cols, keep, k], dtype=np.float64)
            out[key + "_words"] = words.numpy()
            out[key + "_values"] = bits(values)
            if rows * cols <= 8192:
                out[key + "_pruned"] = bits(pruned)
            out[key + "_ties"] = ties
            assert torch.equal(compact.unpack(values, words, cols), pruned)
    return out


def config1_case(wanda, compact) -> dict:
    """W [2048, 2048] fp32, keep 40, calibration 128 x 512 tokens, 17-token forward, seed 0."""
    cfg = workloads.config1(seed=0)
    sums = 0
    for chunk in cfg.calib_chunks():
        sums = sums + chunk.float().pow(2).sum(0).double()           # wanda.py:39 and _add at :34-35
    norms = wanda.channel_norms(sums, cfg.w)
    pruned, mask = wanda.prune(cfg.w, cfg.keep, norms, with_mask=True)
    values, words = compact.pack(pruned, mask)
    y = torch.nn.functional.linear(cfg.x, compact.unpack(values, words, cfg.w.shape[1]))
    score = cfg.w.float().abs() * norms
    k = max(1, round(cfg.keep / 100 * cfg.w.shape[1]))
    srt = score.sort(dim=-1, descending=True).values
    return {
        "sums": sums.numpy(),
        "norms": norms.numpy(),
        "k": np.array(k),
        "words_sha256": np.array(hashlib.sha256(words.numpy().tobytes()).hexdigest()),
        "values_sha256": np.array(hashlib.sha256(values.numpy().tobytes()).hexdigest()),
        "y": y.numpy(),
        "tie_rows": np.array(int((srt[:, k - 1] == srt[:, k]).sum())),
    }


class _Layer(torch.nn.Module):
    """The reference's own fake layer of tests/test_sglang.py:205-211: scale * h + h^2."""

    def __init__(self, scale: float):
        super().__init__()
        self.scale = scale

    def forward(self, hidden_states, forward_batch):
        return self.scale * hidden_states + hidden_states ** 2


def combine_cases(replica, route) -> dict:
    out = {}
    decode = types.SimpleNamespace(forward_mode=types.SimpleNamespace(is_decode=lambda: True,
                                                                      is_target_verify=lambda: False))
    for dtype in (torch.bfloat16, torch.float32, torch.float16):
        for n in (2, 3, 5):
            g = torch.Generator().manual_seed(7 + n)
            h = torch.randn(8, 96, generator=g).to(dtype)
            members = [_Layer(0.3 + 0.1 * j) for j in range(n)]
            copy = _Layer(0.85)
            got = replica._member(members, copy, 0, h, decode)
            hc = copy(h, None)
            parts = [m(h, None) for m in members[:-1]] + [members[-1](hc, None)]
            key = f"n{n}_{DT[dtype]}"
            out[key + "_h"] = bits(h)
            out[key + "_hc"] = bits(hc)
            for j, p in enumerate(parts):
                out[key + f"_p{j}"] = bits(p)
            out[key + "_out"] = bits(got)
            summed = route._summed([{"hidden_states": p} for p in parts], dtype)["hidden_states"]
            out[key + "_summed"] = bits(summed)
    return out


def expert_case(wanda) -> dict:
    """wanda.expert_inputs (p2p/wanda.py:10-20) on a small routed batch with a duplicate id and an unused expert."""
    g = torch.Generator().manual_seed(3)
    E, R, H, T, K = 6, 8, 32, 40, 2
    m = types.SimpleNamespace(w13_weight=torch.randn(E, 2 * R, H, generator=g), w2_weight=torch.randn(E, H, R, generator=g))
    x = torch.randn(T, H, generator=g)
    ids = torch.randint(0, E - 1, (T, K), generator=g)          # expert E-1 never routed
    ids[3] = torch.tensor([2, 2])                              # a token routed twice to one expert
    into, gated = wanda.expert_inputs(m, x, ids)
    return {"w13": m.w13_weight.numpy(), "x": x.numpy(), "ids": ids.numpy(), "into": into.numpy(),
            "gated": gated.numpy()}


def tiles_cases(wanda, compact) -> dict:
    """The reference kernel's layout (p2p.compact.Tiles, p2p/compact.py:124-174) of small modules, built on the CPU with
    compact.cu's default shape (RT 128, KCOLS 64, WARPS 4); Tiles' timing-based split choice needs the GPU and is left
    out (it does not change the layout)."""
    compact._EXT = types.SimpleNamespace(RT=128, KCOLS=64, WARPS=4)
    compact.Tiles._tune = lambda self: {}
    cases = {"a": (torch.bfloat16, [("sparse", 300, 36)], 200),
             "b": (torch.float16, [("dense", 64, 0), ("sparse", 100, 20), ("sparse", 40, 50)], 128),
             "c": (torch.bfloat16, [("sparse", 130, 90)], 64)}
    out = {}
    for name, (dtype, spec, cols) in cases.items():
        g = torch.Generator().manual_seed(len(name) + ord(name))
        blocks = []
        for j, (kind, rows, keep) in enumerate(spec):
            w = torch.randn(rows, cols, generator=g).to(dtype)
            if kind == "dense":
                blocks.append(("dense", w))
                out[f"{name}_b{j}_dense"] = bits(w)
                continue
            pruned, mask = wanda.prune(w, keep, torch.rand(cols, generator=g) + 0.1, with_mask=True)
            values, words = compact.pack(pruned, mask)
            blocks.append(("sparse", values, words, cols))
            out[f"{name}_b{j}_values"] = bits(values)
            out[f"{name}_b{j}_words"] = words.numpy()
        t = compact.Tiles(blocks)
        out[f"{name}_meta"] = np.array([len(spec), cols, t.rows, t.vcap, t.tiles, t.chunks], dtype=np.int64)
        out[f"{name}_vals"] = bits(t.vals)
        out[f"{name}_masks"] = t.masks.numpy()
        out[f"{name}_woff"] = t.woff.numpy()
    compact._EXT = None
    return out


class _Linear(torch.nn.Module):
    """A linear module with the attributes SGLang's fused linear layers carry (output_sizes, output_partition_sizes,
    input_size), which the reference's family.projections reads."""

    def __init__(self, sizes, cols, g, dtype):
        super().__init__()
        self.output_sizes, self.output_size, self.input_size = list(sizes), sum(sizes), cols
        self.output_partition_sizes = list(sizes)                   # one rank holds them all
        self.weight = torch.nn.Parameter((torch.randn(sum(sizes), cols, generator=g) * 0.02).to(dtype),
                                         requires_grad=False)


def replica_layer(g, dtype=torch.bfloat16, hidden=64, kv=16, inter=128):
    layer = torch.nn.Module()
    layer.self_attn, layer.mlp = torch.nn.Module(), torch.nn.Module()
    layer.self_attn.qkv_proj = _Linear((hidden, kv, kv), hidden, g, dtype)
    layer.self_attn.o_proj = _Linear((hidden,), hidden, g, dtype)
    layer.mlp.gate_up_proj = _Linear((inter, inter), hidden, g, dtype)
    layer.mlp.down_proj = _Linear((hidden,), inter, g, dtype)
    return layer


# Keeps per projection: compact ones, one kept whole (100) and one where compact would save too little (95).
REPLICA_KEEP = {"q": 33, "k": 40, "v": 100, "o": 33, "gate": 36, "up": 95, "down": 36}


def replica_case(out_dir: str) -> dict:
    """p2p.prepare.write (p2p/prepare.py:42-73) on one small fake layer: the file it writes goes to
    tests/golden/replica_layer0.safetensors; its inputs (weights, sums, plan) to replica_case.npz."""
    import shutil
    import tempfile
    sys.modules.setdefault("sglang.srt.plugins", types.ModuleType("sglang.srt.plugins"))
    from p2p import prepare
    g = torch.Generator().manual_seed(11)
    layer = replica_layer(g)
    keys = {"self_attn.qkv_proj": 64, "self_attn.o_proj": 64, "mlp.gate_up_proj": 64, "mlp.down_proj": 128}
    sums = {(0, k): (torch.rand(c, generator=g, dtype=torch.float64) * 100 + 1) for k, c in keys.items()}
    plan = {"keep": {"0": dict(REPLICA_KEEP)}}
    with tempfile.TemporaryDirectory() as tmp:
        prepare.write([layer], plan, sums, [0], tmp)
        shutil.copy(os.path.join(tmp, "layer0.safetensors"), os.path.join(out_dir, "replica_layer0.safetensors"))
    out = {f"w:{path}": bits(m.weight.data) for path, m in layer.named_modules() if hasattr(m, "weight")}
    out |= {f"sums:{k}": v.numpy() for (_, k), v in sums.items()}
    return out


def row_hashes(words: np.ndarray) -> np.ndarray:
    """An 8-byte BLAKE2b digest of each row of mask words, as uint64 (a full-size selection stored compactly)."""
    words = np.ascontiguousarray(words)
    return np.array([int.from_bytes(hashlib.blake2b(r.tobytes(), digest_size=8).digest(), "little") for r in words],
                    dtype=np.uint64)


def llama_select_case(wanda, compact) -> dict:
    """The reference's selection at BASELINE config 2's full sizes: each Llama-3-8B projection (keep 33 / 36) on
    CPU-seeded weights, with norms from a lognormal-scaled calibration (wanda.py:39, channel_norms), pruned and packed
    by the reference (wanda.prune with_mask, compact.pack). Stored: the norms, each row's mask-word digest and the rows
    whose k-th and (k+1)-th scores tie (where torch.topk's choice is unspecified)."""
    out = {}
    for i, p in enumerate(workloads.LLAMA3_8B):
        w, x = workloads.selection_case(p, i)
        sums = x.float().pow(2).sum(0).double()
        norms = wanda.channel_norms(sums, w)
        pruned, mask = wanda.prune(w, p.keep, norms, with_mask=True)
        _, words = compact.pack(pruned, mask)
        score = w.float().abs() * norms
        k = max(1, round(p.keep / 100 * p.cols))
        srt = score.sort(dim=-1, descending=True).values
        out[p.name + "_norms"] = norms.numpy()
        out[p.name + "_sums"] = sums.numpy()
        out[p.name + "_words_b2"] = row_hashes(words.numpy())
        out[p.name + "_tie_rows"] = np.nonzero((srt[:, k - 1] == srt[:, k]).numpy())[0].astype(np.int64)
        out[p.name + "_k"] = np.array(k)
        print(p.name, "k", k, "tie rows", len(out[p.name + "_tie_rows"]), flush=True)
    return out


def main() -> None:
    wanda, compact, replica, route = _reference()
    torch.manual_seed(0)
    np.savez_compressed(os.path.join(HERE, "select_cases.npz"), **select_cases(wanda, compact))
    np.savez_compressed(os.path.join(HERE, "config1.npz"), **config1_case(wanda, compact))
    np.savez_compressed(os.path.join(HERE, "combine_cases.npz"), **combine_cases(replica, route))
    np.savez_compressed(os.path.join(HERE, "expert_case.npz"), **expert_case(wanda))
    np.savez_compressed(os.path.join(HERE, "tiles_cases.npz"), **tiles_cases(wanda, compact))
    np.savez_compressed(os.path.join(HERE, "replica_case.npz"), **replica_case(HERE))
    np.savez_compressed(os.path.join(HERE, "llama_select.npz"), **llama_select_case(wanda, compact))
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
