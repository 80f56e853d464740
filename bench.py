#!/usr/bin/env python
"""Replica sparse-GEMM throughput on B200: one Llama-3-8B-shaped replica layer.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--tokens T]

A step is one forward pass of the replica layer's compact projections (q, k, v, o at keep 33; gate, up, down at keep
36; 4 bytes a kept weight) over a batch of T = 272 tokens (16 sequences x 17 draft-pass tokens), module by module as
SGLang holds them: qkv_proj, o_proj, gate_up_proj, down_proj, each one Compact (one kernel launch).
Weights are N(0, 0.02), activations N(0, 1) times a lognormal per-channel scale, all seeded and synthetic; the
calibration sums come from 128 x 2048 synthetic tokens per projection input through the package's own calibration
kernel, and the selection from its Wanda top-k kernel.

value: tokens/s of the whole job (N ranks, each with its own replica layer: weak scaling, no data-path collective),
device-timed with CUDA events, the max over ranks. e2e: the same through the public API (Compact.apply) with the
inputs copied from pinned host memory and the outputs read back inside the timed region. roofline: the compact GEMM's
algorithmic bytes (values + indices + x + y, each once) per launch over its event-timed duration, against the measured
HBM copy bandwidth. cpu_baseline: the reference's CPU forward (dense masked F.linear of the unpacked rows) on the
host's cores, on a bounded sample of the same layer.

--impl reference times that CPU path alone (rank 0; other ranks exit) and prints the same metric with impl=reference.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from p2pllm_b200 import workloads  # noqa: E402

METRIC = "replica sparse-GEMM tokens/s (Llama-3-8B replica layer, keep 33/36, T=272)"
UNIT = "tokens/s"
# The layer's linear modules as SGLang holds them (fused q/k/v and gate/up), the input each reads, and their blocks.
MODULES = workloads.LAYER_MODULES
INPUT_OF = {n: group for group, names in MODULES.values() for n in names}
L2_BYTES = 126 * 1024 * 1024
# A spin queued just before a device-timed region: the host enqueues the region's launches while the GPU spins, so
# the events time the GPU's work rather than the host's launch cost (the spin itself is outside the region).
HEAD_START_CYCLES = 20_000_000


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", default="b200", choices=["b200", "reference"])
    p.add_argument("--tokens", type=int, default=272)
    p.add_argument("--calib-tokens", type=int, default=128 * 2048)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--workload", default="cfg2", choices=["cfg2", "cfg1", "cfg3", "cfg4", "cfg5", "module"],
                   help="cfg2 (default): the headline line. cfg1, cfg3, cfg5: one extra line each on one GPU (config "
                        "1's fp32 projection; config 3's replica block + group combine at T = 1, 8, 32, 64; a "
                        "Qwen2.5-32B replica layer at keep 40). module: one module of the cfg2 layer (--module, "
                        "--layout), --steps launches, for profiling")
    p.add_argument("--module", default="gate_up_proj", choices=list(MODULES))
    p.add_argument("--layout", default=None, choices=["tc", "mask"],
                   help="the tensor-core layout of the compact modules (default: the package's)")
    p.add_argument("--push", default="auto", choices=["auto", "on", "off"],
                   help="row sharding: the rank's rows to its peers by a push kernel after the GEMM (on, the "
                        "default), or from the GEMM's epilogue (off)")
    p.add_argument("--pass-tokens", type=int, default=17,
                   help="cfg5: tokens of a pass (a draft pass of 16 + 1 by default)")
    p.add_argument("--cfg5-single-layer", action="store_true",
                   help="cfg5: time one replica layer on one GPU instead of the layer-parallel plan")
    return p.parse_args()


def measured_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


# ---------------------------------------------------------------------------------------------------------- clocks --

_REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
            0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting", 0x10: "sync_boost"}


class ClockSampler:
    """SM clock and clock-event reasons of this rank's GPU through NVML, every few ms while running."""

    def __init__(self, device: int, period_s: float = 0.005):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self.period, self._stop, self._thread = period_s, threading.Event(), None
        try:
            import pynvml
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            try:
                self.h = pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + uuid) if not uuid.startswith("GPU-") else uuid)
            except Exception:
                self.h = pynvml.nvmlDeviceGetHandleByIndex(device)
            self.nvml = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self._reason_fn = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                getattr(pynvml, "nvmlDeviceGetCurrentClocksThrottleReasons")
        except Exception as e:                                         # no NVML: report that, keep going
            self.nvml, self.error = None, str(e)

    def _run(self):
        while not self._stop.is_set():
            self.sample()
            time.sleep(self.period)

    def sample(self):
        if self.nvml is None:
            return
        try:
            self.samples.append(self.nvml.nvmlDeviceGetClockInfo(self.h, self.nvml.NVML_CLOCK_SM))
            bits = self._reason_fn(self.h)
            self.reasons |= {name for bit, name in _REASONS.items() if bits & bit}
        except Exception:
            pass

    def __enter__(self):
        self.sample()
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        self.sample()
        self._stop.set()
        self._thread.join()

    def summary(self) -> dict:
        if self.nvml is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "error": getattr(self, "error", "")}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ------------------------------------------------------------------------------------------------------- the layer --

class ReplicaLayer:
    """A Llama-3-8B replica layer's four linear modules, each a Compact over its projections' blocks, calibrated and
    selected on the GPU."""

    def __init__(self, seed: int, tokens: int, calib_tokens: int, device: torch.device, projections=None):
        from p2pllm_b200 import compact, kernels, wanda
        self.device, self.tokens = device, tokens
        self.proj = {p.name: p for p in (projections or workloads.LLAMA3_8B)}
        self.inputs, self.methods, self.k, self.selected = {}, {}, {}, {}
        calib_ms, select_ms, calib_bytes = 0.0, 0.0, 0
        ev = lambda: torch.cuda.Event(enable_timing=True)
        seeds = workloads.layer_seeds(seed, tuple(self.proj.values()))
        for module, (group, names) in MODULES.items():
            cols = self.proj[names[0]].cols
            g = torch.Generator(device=device).manual_seed(seeds[module][0])
            scale = workloads.channel_scale(cols, g, device)
            # Calibration: the hook's reduction over 128 x 2048 synthetic tokens, in 16 calls.
            sums, ms, nb = workloads.calibrate(cols, g, scale, calib_tokens, device)
            calib_ms, calib_bytes = calib_ms + ms, calib_bytes + nb
            norms = kernels.channel_norms(sums)
            self.inputs[group] = (torch.randn(tokens, cols, generator=g, device=device) * scale).bfloat16()
            blocks = []
            for n in names:
                p = self.proj[n]
                w = workloads.projection_weights(p, seeds[module][1][n], device)
                a, b = ev(), ev()
                a.record()
                values, idx = wanda.select(w, p.keep, norms)
                b.record()
                b.synchronize()
                select_ms += a.elapsed_time(b)
                del w
                self.k[n] = values.shape[1]
                self.selected[n] = (values, idx)
                blocks.append(("compact", values, idx, p.cols))
            self.methods[module] = compact.Compact(blocks)
        self.calib_ms, self.select_ms, self.calib_bytes = calib_ms, select_ms, calib_bytes
        torch.cuda.synchronize(device)

    def rows(self, module: str) -> int:
        return sum(self.proj[n].rows for n in MODULES[module][1])

    def cols(self, module: str) -> int:
        return self.proj[MODULES[module][1][0]].cols

    def algorithmic_bytes(self, module: str, tokens: int) -> int:
        """Values + indices (2 + 2 bytes a kept weight), x and y, each once."""
        weights = sum(self.proj[n].rows * self.k[n] * 4 for n in MODULES[module][1])
        return weights + tokens * self.cols(module) * 2 + tokens * self.rows(module) * 2

    def flops(self, module: str, tokens: int) -> int:
        return sum(2 * self.proj[n].rows * self.k[n] * tokens for n in MODULES[module][1])

    def mask_format_bytes(self, module: str) -> int:
        return sum(self.proj[n].rows * self.k[n] * 2 + self.proj[n].rows * ((self.proj[n].cols + 31) // 32) * 4
                   for n in MODULES[module][1])

    def step(self, events=None, x=None):
        """One pass of the layer; with events, records (start, end) around each module's launch."""
        x = x or self.inputs
        outs = {}
        for i, (module, (group, _)) in enumerate(MODULES.items()):
            if events is not None:
                events[i][0].record()
            outs[module] = self.methods[module].apply(None, x[group])
            if events is not None:
                events[i][1].record()
        return outs


def cpu_model() -> str:
    """The host CPU's model name (from /proc/cpuinfo), or the platform's processor string."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


class ReferenceCPU:
    """The reference's CPU path for a whole Llama-3-8B replica layer, on all host cores: at load, per projection, the
    Wanda selection (torch.topk of |w| * norms, p2p/wanda.py:76-87), the packing into values + mask words
    (p2p/compact.py:36-45) and the expansion back to a dense matrix (compact.unpack's CPU branch, p2p/compact.py:57-61)
    -- timed once, as `setup` -- and per step the forward F.linear(x, W) of every projection (the reference's only CPU
    forward: compact.Tiles needs CUDA). All 218 M weights of the layer, bf16, seeded synthetic weights and norms. Used by
    both the headline's cpu_baseline and the --impl reference arm, so the two report the same measurement."""

    def __init__(self, tokens: int):
        from oracle import cpu_ref
        self.cpu_ref = cpu_ref
        torch.set_num_threads(os.cpu_count() or 1)
        self.cores = torch.get_num_threads()
        self.cpu = cpu_model()
        self.tokens = tokens
        g = torch.Generator().manual_seed(0)
        self.projs = list(workloads.LLAMA3_8B)
        self.mats, self.xs = {}, {}
        setup = {"prune_s": 0.0, "pack_s": 0.0, "unpack_s": 0.0}
        for p in self.projs:
            w = (torch.randn(p.rows, p.cols, generator=g) * 0.02).bfloat16()
            norms = torch.rand(p.cols, generator=g) * workloads.channel_scale(p.cols, g) + 1e-3
            t0 = time.perf_counter()
            pruned, mask = cpu_ref.prune(w, p.keep, norms)
            t1 = time.perf_counter()
            values, words = cpu_ref.pack(pruned, mask)
            t2 = time.perf_counter()
            self.mats[p.name] = cpu_ref.unpack_words(values, words, p.cols)
            t3 = time.perf_counter()
            setup["prune_s"] += t1 - t0
            setup["pack_s"] += t2 - t1
            setup["unpack_s"] += t3 - t2
            del w, pruned, mask, values, words
            if INPUT_OF[p.name] not in self.xs:
                self.xs[INPUT_OF[p.name]] = (torch.randn(tokens, p.cols, generator=g)
                                             * workloads.channel_scale(p.cols, g)).bfloat16()
        self.setup = setup
        self.sample = (f"the whole layer (all {sum(p.rows * p.cols for p in self.projs) / 1e6:.0f} M weights of the 7 "
                       f"projections), {tokens} tokens, bf16 F.linear of the unpacked matrices; median of the steps "
                       "after warm-up")

    def step(self) -> float:
        """Seconds of one layer pass."""
        t0 = time.perf_counter()
        for p in self.projs:
            self.cpu_ref.forward(self.xs[INPUT_OF[p.name]], self.mats[p.name])
        return time.perf_counter() - t0

    def layer_seconds(self, steps: int, warmup: int) -> float:
        for _ in range(max(1, warmup)):
            self.step()
        return statistics.median(self.step() for _ in range(max(10, steps)))

    def summary(self, value: float) -> dict:
        return {"value": value, "unit": UNIT, "cores": self.cores, "cpu": self.cpu, "kind": "port",
                "sample": self.sample, "setup": {k: round(v, 3) for k, v in self.setup.items()}}


# ---------------------------------------------------------------------------------------------------------- driver --

def dist_env():
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    return rank, world, local


def max_over_ranks(v: float, world: int, device) -> float:
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def run_reference(args, rank, world):
    """The reference's CPU forward on the host cores, rank 0 only."""
    if rank != 0:
        return
    ref = ReferenceCPU(args.tokens)
    layer_s = ref.layer_seconds(args.steps, args.warmup)
    value = args.tokens / layer_s
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": layer_s * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "cfg2 Llama-3-8B replica layer (q,k,v,o keep 33; gate,up,down keep 36), T=%d"
                               % args.tokens,
                   "tokens": args.tokens, "path": "reference CPU forward (oracle port of compact.unpack + F.linear)"},
        "cpu_baseline": ref.summary(value),
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# Traffic of the compact GEMM per algorithmic byte, from one ncu capture of each kernel on the bench's gate_up module
# (dram__bytes_read.sum + dram__bytes_write.sum over the launch's algorithmic bytes); the files under profiles/ named
# in each entry hold the capture and its command.
TRAFFIC_RATIO = {"tc": (0.942, "profiles/spmm_tc_gate_up_T17_T272.md"),
                 "mask": (1.03, "profiles/spmm_mask_gate_up_T17.md")}


def _events():
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def _region_ms(fn, steps: int, stream) -> float:
    """Device milliseconds of `steps` calls of fn as one region, queued behind a spin (the host's launch cost is off the
    clock): only the two bracketing events, so the launches' programmatic overlap stays."""
    a, b = _events()
    torch.cuda._sleep(HEAD_START_CYCLES)
    a.record(stream)
    for _ in range(steps):
        fn()
    b.record(stream)
    b.synchronize()
    return a.elapsed_time(b)


def _module_tiles(layer, layout: str) -> dict:
    """The layer's modules in one tensor-core layout: {module: Tiles}."""
    from p2pllm_b200 import compact
    out = {}
    for module, (group, names) in MODULES.items():
        blocks = [("compact", *layer.selected[n], layer.proj[n].cols) for n in names]
        out[module] = compact.Tiles(blocks, layout=layout)
    return out


def _format_line(layer, tiles: dict, layout: str, steps: int, stream, peak: float) -> dict:
    """Device time of a layer step in one layout at the bench's T and at 17 tokens, with that layout's bytes."""
    res = {}
    for T in (layer.tokens, 17):
        xs = {g: t[:T].contiguous() for g, t in layer.inputs.items()}
        step = lambda: [tiles[m](xs[g]) for m, (g, _) in MODULES.items()]
        for _ in range(3):
            step()
        ms = _region_ms(step, steps, stream) / steps
        nbytes = sum(t.nbytes() for t in tiles.values()) + sum(T * (layer.cols(m) + layer.rows(m)) * 2 for m in MODULES)
        res[f"T{T}"] = {"ms_per_step": ms, "tokens_per_s": T / (ms / 1e3), "bytes_per_step": nbytes,
                        "hbm_gbs": nbytes / (ms / 1e3) / 1e9, "frac": nbytes / (ms / 1e3) / 1e9 / peak}
    res["weights_bytes"] = sum(t.nbytes() for t in tiles.values())
    res["bytes_per_kept_weight"] = res["weights_bytes"] / sum(layer.proj[n].rows * layer.k[n] for n in layer.proj)
    return res


def _host_us_per_call(method, x, calls: int = 200) -> float:
    """Host microseconds of one Compact.apply call (launch only; the GPU is kept busy by a spin meanwhile)."""
    torch.cuda._sleep(HEAD_START_CYCLES * 4)
    t0 = time.perf_counter()
    for _ in range(calls):
        method.apply(None, x)
    dt = time.perf_counter() - t0
    torch.cuda.synchronize()
    return dt / calls * 1e6


def _gpu_reference(layer, stream) -> dict | None:
    """A baseline leg: the reference's own GPU kernel (p2p/compact.cu built for sm_100a into oracle/_ref by build())
    on the same selections, laid out and split-tuned as its Tiles does, timed on the same layer at the bench's T and at
    17 tokens. None when the module was not built."""
    from oracle import build_ref, ref_tiles
    if build_ref.built() is None:
        return None
    ext = build_ref.load_module()
    mods = {}
    for module, (group, names) in MODULES.items():
        blocks = []
        for n in names:
            values, idx = layer.selected[n]
            blocks.append(("sparse", values, ref_tiles.words_of(idx, layer.proj[n].cols), layer.proj[n].cols))
        mods[module] = ref_tiles.RefTiles(blocks, ext, tune=True)
    out = {}
    for T in (layer.tokens, 17):
        xs = {g: t[:T].contiguous() for g, t in layer.inputs.items()}
        step = lambda: [mods[m](xs[g]) for m, (g, _) in MODULES.items()]
        for _ in range(2):
            step()
        ms = _region_ms(step, 5, stream) / 5
        out[f"T{T}"] = {"ms_per_step": ms, "tokens_per_s": T / (ms / 1e3)}
    out["how"] = ("reference compact.Tiles kernel (p2p/compact.cu, mma.sync on its bitmask format), built for sm_100a "
                  "from the reference source; same weights and selections; split tuned as Tiles._tune does")
    return out


def run_b200(args, rank, world, local):
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    peaks = measured_peaks()
    # every rank builds the same layer (same seeds): with N GPUs it is row-sharded across them
    layer = ReplicaLayer(seed=0, tokens=args.tokens, calib_tokens=args.calib_tokens, device=device)
    if world == 1:
        run_single(args, layer, device, peaks)
    else:
        run_sharded(args, layer, rank, world, device, peaks)


def run_single(args, layer, device, peaks):
    from p2pllm_b200 import compact
    stream = torch.cuda.current_stream(device)
    names = list(MODULES)
    n_proj = len(names)
    for _ in range(args.warmup):
        layer.step()
    torch.cuda.synchronize(device)

    # timed region: exactly K steps, only the two bracketing events. The four launches of a step are the same kernel,
    # each a programmatic dependent of the one before (it starts on SMs the previous one frees and streams its weights
    # while that one drains); an event recorded between launches would stop that overlap, so the roofline's per-launch
    # figure is the region's: bytes of a step over its time (= bytes a launch over the mean launch time).
    start, end = _events()
    torch.cuda.synchronize(device)
    clocks = ClockSampler(device.index)
    with clocks:
        torch.cuda._sleep(HEAD_START_CYCLES)
        start.record(stream)
        for s in range(args.steps):
            layer.step()
        end.record(stream)
        torch.cuda.synchronize(device)
    total_ms = start.elapsed_time(end)
    ms_per_step = total_ms / args.steps
    value = args.tokens * args.steps / (total_ms / 1e3)
    layout = layer.methods[names[0]].tiles.layout

    # per-module breakdown, a separate pass: events around each launch (serialised, so a little slower than a step)
    events = [[list(_events()) for _ in range(n_proj)] for _ in range(20)]
    torch.cuda._sleep(HEAD_START_CYCLES // 4)
    for s in range(20):
        layer.step(events[s])
    torch.cuda.synchronize(device)
    launch_ms = {n: statistics.median(events[s][i][0].elapsed_time(events[s][i][1]) for s in range(20))
                 for i, n in enumerate(names)}

    # both tensor-core layouts of the same selections, each with its own bytes
    formats = {}
    for L in ("tc", "mask"):
        tiles = {m: layer.methods[m].tiles for m in names} if L == layout else _module_tiles(layer, L)
        formats[L] = _format_line(layer, tiles, L, max(10, args.steps), stream, peaks["hbm_gbs"])
        del tiles
    fmt = formats[layout]
    achieved = fmt[f"T{args.tokens}"]["bytes_per_step"] / (ms_per_step / 1e3) / 1e9
    flops = sum(layer.flops(n, args.tokens) for n in names)
    ratio, ratio_src = TRAFFIC_RATIO[layout]
    traffic = None if ratio is None else ratio * fmt[f"T{args.tokens}"]["bytes_per_step"]

    # e2e through the public API at the bench's T and at 17 tokens
    e2e = _e2e(layer, args.tokens, args.steps, args.warmup, device, stream)
    e2e17 = _e2e(layer, 17, args.steps, args.warmup, device, stream)
    host_us = _host_us_per_call(layer.methods["o_proj"], layer.inputs["attn_out"][:17].contiguous())

    gpu_ref = _gpu_reference(layer, stream)
    cpu = None
    if not args.no_cpu_baseline:
        ref = ReferenceCPU(args.tokens)
        cpu = ref.summary(args.tokens / ref.layer_seconds(steps=10, warmup=2))

    out = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,0.02) weights, lognormal-scaled "
                                                      "N(0,1) activations; no checkpoint or dataset)",
        "config": {"workload": "cfg2 Llama-3-8B replica layer (q,k,v,o keep 33; gate,up,down keep 36), "
                               f"T={args.tokens}", "tokens": args.tokens, "layout": layout,
                   "format": {"tc": "bf16 values + 16-bit positions (4 bytes a kept weight)",
                              "mask": "bf16 values + 1 bit a weight + 16-bit offsets (the reference's storage)"}[layout],
                   "weights_bytes_per_gpu": fmt["weights_bytes"],
                   "l2": "inputs larger than L2: %.0f MB of weights streamed per step vs %d MB L2"
                         % (fmt["weights_bytes"] / 1e6, L2_BYTES >> 20),
                   "parallelism": "one GPU, the whole layer"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "traffic": traffic, "traffic_source": ratio_src,
                     "peak_source": peaks["source"], "kernel": f"spmm ({layout} layout; one launch per module, 4 a step)",
                     "algorithmic_bytes_per_step": fmt[f"T{args.tokens}"]["bytes_per_step"],
                     "algorithmic_flops_per_step": flops,
                     "achieved_tflops": flops / (ms_per_step / 1e3) / 1e12,
                     "timing": "CUDA events around the K-step region on the launching stream; per launch = "
                               "step bytes over step time (4 launches of this kernel a step)"},
        "formats": formats,
        "per_module_us": {n: launch_ms[n] * 1e3 for n in names},
        "per_module_note": "a separate pass with an event around each launch, which stops the launches' overlap",
        "t17": formats[layout]["T17"],
        "setup": {"calib_ms": layer.calib_ms, "select_ms": layer.select_ms,
                  "calib_gbs": layer.calib_bytes / (layer.calib_ms / 1e3) / 1e9},
        "e2e": dict(e2e, t17=e2e17),
        "host_us_per_call": host_us,
        "gpu_launches": args.steps * n_proj,
        "clocks": clocks.summary(),
        "cpu_baseline": cpu,
        "gpu_reference": gpu_ref,
    }
    print(json.dumps(out), flush=True)


def _e2e(layer, T: int, steps: int, warmup: int, device, stream) -> dict:
    """Tokens/s through Compact.apply with pinned host inputs copied in and every output copied back each step,
    pipelined as a serving loop runs it: step s's inputs go in on an input stream (double-buffered), the modules run on
    the compute stream once they have landed, and the outputs go back on an output stream as soon as the step ends."""
    names = list(MODULES)
    host_x = {g: t[:T].contiguous().cpu().pin_memory() for g, t in layer.inputs.items()}
    host_y = {n: torch.empty(T, layer.rows(n), dtype=torch.bfloat16).pin_memory() for n in names}
    h2d = sum(t.numel() * t.element_size() for t in host_x.values())
    d2h = sum(t.numel() * t.element_size() for t in host_y.values())
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    dev_x2 = [{g: torch.empty_like(t, device=device) for g, t in host_x.items()} for _ in range(2)]
    landed = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]
    for ev in consumed:
        ev.record(stream)

    def run(n):
        for k in range(n):
            buf = k % 2
            with torch.cuda.stream(s_in):
                s_in.wait_event(consumed[buf])                 # the step two back has read this buffer
                for g in host_x:
                    dev_x2[buf][g].copy_(host_x[g], non_blocking=True)
                landed[buf].record(s_in)
            stream.wait_event(landed[buf])
            ys = {n_: layer.methods[n_].apply(None, dev_x2[buf][MODULES[n_][0]]) for n_ in names}
            consumed[buf].record(stream)              # one event a step: none between launches (they overlap)
            with torch.cuda.stream(s_out):
                s_out.wait_event(consumed[buf])
                for n_, y in ys.items():
                    host_y[n_].copy_(y, non_blocking=True)
                    y.record_stream(s_out)

    run(max(3, warmup))
    torch.cuda.synchronize(device)
    a, b = _events()
    a.record(stream)
    s_in.wait_stream(stream)
    run(steps)
    stream.wait_stream(s_out)
    stream.wait_stream(s_in)
    b.record(stream)
    torch.cuda.synchronize(device)
    ms = a.elapsed_time(b)
    return {"value": T * steps / (ms / 1e3), "unit": UNIT, "tokens": T, "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
            "how": "Compact.apply per module; pinned-host inputs copied in and every output copied back each step, on "
                   "input / output streams overlapping the kernels (double-buffered inputs)"}


def _clone_shard(sc):
    """The same shard with its own copy of the weight bytes (another address range), sharing everything else."""
    import copy
    other = copy.copy(sc)
    if sc.local is not None:
        tiles = copy.copy(sc.local.tiles)
        for name in ("data", "words", "seg"):
            if hasattr(tiles, name) and torch.is_tensor(getattr(tiles, name)):
                setattr(tiles, name, getattr(tiles, name).clone())
        other.local = copy.copy(sc.local)
        other.local.tiles = tiles
    return other


def run_sharded(args, layer, rank, world, device, peaks):
    """The cfg2 layer row-sharded over `world` GPUs (shard.ShardedCompact: each rank whole 128-row tiles of every
    module and the full x). Headline: the all-gather fused into the GEMM (each rank's bitmask-layout GEMM stores its
    rows of y into every rank's y over NVLink, one bounded peer barrier a step). Beside it: the same split with the
    GEMM writing its slot and one NCCL all-gather a module."""
    import hashlib
    import torch.distributed as dist
    from p2pllm_b200 import shard
    stream = torch.cuda.current_stream(device)
    names = list(MODULES)
    blocks = {m: [("compact", *layer.selected[n], layer.proj[n].cols) for n in MODULES[m][1]] for m in names}
    peers = shard.PeerGroup(None, device)
    push = None if args.push == "auto" else args.push == "on"
    sharded = {m: shard.ShardedCompact(blocks[m], fused=True, peers=peers, layout=args.layout, push=push)
               for m in names}
    for m in names:
        sharded[m].prepare(args.tokens, torch.bfloat16, device)
    xs = {m: layer.inputs[MODULES[m][0]] for m in names}

    # In-run parity: every module's y against the unsharded module on rank 0 (rel-L2 <= 1e-2: the shards may split
    # their columns differently, so sums can differ in the last bf16 bit), and the same bits on every rank.
    checks, ok = {}, True
    for m in names:
        y = sharded[m].apply(None, xs[m])
        digest = hashlib.sha256(y.cpu().view(torch.int16).numpy().tobytes()).digest()[:8]
        mine = torch.tensor([int.from_bytes(digest, "little", signed=True)], dtype=torch.int64, device=device)
        every = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(every, mine)
        same = all(int(e.item()) == int(mine.item()) for e in every)
        rel = 0.0
        if rank == 0:
            want = layer.methods[m].apply(None, xs[m]).double()
            rel = float((y.double() - want).norm() / want.norm())
        flag = torch.tensor([1 if (same and rel <= 1e-2) else 0], device=device)
        dist.broadcast(flag, 0)
        checks[m] = {"rel_l2_vs_one_gpu": rel, "same_bits_on_every_rank": same}
        ok = ok and bool(flag.item())
    peers.status()
    if not ok:
        if rank == 0:
            print(json.dumps({"metric": METRIC, "error": "row-sharded parity check failed", "checks": checks}),
                  flush=True)
        raise SystemExit(3)

    # A rank's shard of the weights is smaller than L2 from 4 GPUs on: each rank cycles through `copies` clones of its
    # shards' weight bytes, more than twice L2 in all, so every step streams its weights from HBM, and the K steps are
    # timed as one region (the launches keep their overlap, the peer barriers keep the ranks in step).
    shard_bytes = sum(sharded[m].local.nbytes() for m in names if sharded[m].local is not None)
    copies = max(1, -(-2 * L2_BYTES // max(shard_bytes, 1)))
    rotation = [sharded] + [{m: _clone_shard(sharded[m]) for m in names} for _ in range(copies - 1)]
    turn = [0]

    def step():
        mods = rotation[turn[0] % copies]
        turn[0] += 1
        for m in names:
            mods[m].apply_fused(xs[m], sync=False)
        peers.barrier()

    def kernels_only():
        mods = rotation[turn[0] % copies]
        turn[0] += 1
        for m in names:
            mods[m].apply_fused(xs[m], sync=False)

    for _ in range(max(args.warmup, copies)):
        step()
    torch.cuda.synchronize(device)
    dist.barrier()
    clocks = ClockSampler(device.index)
    with clocks:
        local_ms = _region_ms(step, args.steps, stream)
    dist.barrier()
    total_ms = max_over_ranks(local_ms, world, device)
    kern_ms = max_over_ranks(_region_ms(kernels_only, args.steps, stream), world, device)
    torch.cuda.synchronize(device)
    dist.barrier()
    peers.barrier()
    peers.status()
    ms_per_step = total_ms / args.steps
    value = args.tokens * args.steps / (total_ms / 1e3)

    # the NCCL path: the rank's GEMM writes its slot, one all-gather a module
    nccl = {m: shard.ShardedCompact(blocks[m], fused=False) for m in names}
    parts = {m: torch.empty(args.tokens, nccl[m].width, dtype=torch.bfloat16, device=device) for m in names}
    nccl_rotation = [nccl] + [{m: _clone_shard(nccl[m]) for m in names} for _ in range(copies - 1)]

    def nccl_step():
        mods = nccl_rotation[turn[0] % copies]
        turn[0] += 1
        for m in names:
            mods[m].gather(mods[m].local_part(xs[m], parts[m]))

    def nccl_gathers():
        for m in names:
            nccl[m].gather(parts[m])

    for _ in range(max(3, copies)):
        nccl_step()
    torch.cuda.synchronize(device)
    dist.barrier()
    nccl_ms = max_over_ranks(_region_ms(nccl_step, args.steps, stream), world, device)
    dist.barrier()
    gath_ms = max_over_ranks(_region_ms(nccl_gathers, args.steps, stream), world, device)
    dist.barrier()
    del nccl, parts, nccl_rotation

    # independent replicas (each rank the whole layer on its own tokens): the weak-scaling figure, kept beside
    for _ in range(3):
        layer.step()
    torch.cuda.synchronize(device)
    dist.barrier()
    rep_ms = max_over_ranks(_region_ms(layer.step, args.steps, stream), world, device)

    # e2e: the step's inputs sit in pinned host memory; each rank copies in its T/N rows of every input (input stream,
    # double-buffered) and one NCCL all-gather a module assembles x on every rank; every rank runs its shards, storing
    # into every rank's y; each rank copies its own columns of y back on an output stream while the next step
    # computes, so the host links of all ranks carry the copies. y of step k sits in the symmetric buffer k % 2 that
    # step k + 2 overwrites on every rank, so each rank enters step k + 1's peer barrier only once its copy-out of step
    # k has finished.
    chunk = -(-args.tokens // world)
    host_x = {}
    for m in names:
        padded = torch.zeros(chunk * world, xs[m].shape[1], dtype=torch.bfloat16)
        padded[:args.tokens] = xs[m].cpu()
        host_x[m] = padded[rank * chunk:(rank + 1) * chunk].contiguous().pin_memory()
    host_y = {m: torch.empty(args.tokens, sharded[m].mine, dtype=torch.bfloat16).pin_memory() for m in names}
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    stage = [{m: torch.empty(chunk, xs[m].shape[1], dtype=torch.bfloat16, device=device) for m in names}
             for _ in range(2)]
    full = [{m: torch.empty(chunk * world, xs[m].shape[1], dtype=torch.bfloat16, device=device) for m in names}
            for _ in range(2)]
    landed, consumed, copied = ([torch.cuda.Event() for _ in range(2)] for _ in range(3))
    for ev in consumed + copied:
        ev.record(stream)

    def e2e_run(n):
        for k in range(n):
            buf = k % 2
            with torch.cuda.stream(s_in):
                s_in.wait_event(consumed[buf])
                for m in names:
                    stage[buf][m].copy_(host_x[m], non_blocking=True)
                landed[buf].record(s_in)
            stream.wait_event(landed[buf])
            for m in names:
                dist.all_gather_into_tensor(full[buf][m], stage[buf][m])
            mods = rotation[k % copies]
            # The y buffers of this parity were last read by this rank's copy-out of step k - 2 (its own columns,
            # which only its own GEMM writes; peers push their columns), so the GEMMs wait for that copy alone and
            # the copy-out of step k - 1 overlaps them.
            stream.wait_event(copied[buf])
            ys = {}
            for m in names:
                mods[m]._turn = buf                    # y buffer by step parity, whichever weight copy runs
                ys[m] = mods[m].apply_fused(full[buf][m][:args.tokens], sync=False)
            consumed[buf].record(stream)
            peers.barrier()
            done = torch.cuda.Event()
            done.record(stream)
            with torch.cuda.stream(s_out):
                s_out.wait_event(done)
                for m in names:
                    a_, b_ = sharded[m].ranges[rank]
                    host_y[m].copy_(ys[m][:, a_:b_], non_blocking=True)
                copied[buf].record(s_out)

    e2e_run(max(3, copies))
    torch.cuda.synchronize(device)
    dist.barrier()
    a, b = _events()
    a.record(stream)
    s_in.wait_stream(stream)
    e2e_run(args.steps)
    stream.wait_stream(s_out)
    b.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = max_over_ranks(a.elapsed_time(b), world, device)
    peers.status()
    h2d = sum(chunk * world * t.shape[1] * 2 for t in xs.values())
    d2h = sum(args.tokens * sharded[m].rows * 2 for m in names)

    local_bytes = sum(sharded[m].local.nbytes() for m in names if sharded[m].local is not None) + \
        sum(args.tokens * (layer.cols(m) + sharded[m].mine) * 2 for m in names)
    achieved = local_bytes / (kern_ms / args.steps / 1e3) / 1e9
    if rank == 0:
        out = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,0.02) weights, lognormal-scaled N(0,1) activations; no checkpoint or dataset)",
            "config": {"workload": "cfg2 Llama-3-8B replica layer (q,k,v,o keep 33; gate,up,down keep 36), "
                                   f"T={args.tokens}", "tokens": args.tokens,
                       "layout": sharded[names[0]].local.tiles.layout,
                       "parallelism": f"row-sharded over {world} GPUs (whole 128-row tiles of every module a rank, "
                                      "full x); " + ("each rank's rows pushed to every peer's y by one kernel after "
                                                     "its GEMM" if sharded[names[0]].push else
                                                     "y gathered in the GEMM's epilogue by peer stores") +
                                      " over NVLink, one bounded peer barrier a step",
                       "l2": "inputs larger than L2: each rank cycles through %d copies of its %.0f MB of shard "
                             "weights (%.0f MB) vs %d MB L2" % (copies, shard_bytes / 1e6, copies * shard_bytes / 1e6,
                                                                L2_BYTES >> 20)},
            "parity": {"passed": True, "checks": checks},
            "breakdown_us_per_step": {"gemms_and_gather": kern_ms / args.steps * 1e3,
                                      "barrier_and_skew": (total_ms - kern_ms) / args.steps * 1e3,
                                      "step": ms_per_step * 1e3},
            "nccl_path": {"ms_per_step": nccl_ms / args.steps, "all_gathers_us": gath_ms / args.steps * 1e3,
                          "tokens_per_s": args.tokens * args.steps / (nccl_ms / 1e3),
                          "how": "the rank's GEMM writes its slot, one NCCL all_gather_into_tensor a module, then the "
                                 "slots laid side by side"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / peaks["hbm_gbs"], "traffic": None, "peak_source": peaks["source"],
                         "kernel": "the rank's fused GEMMs (bytes of its shards and x, y once, over their time)"},
            "replicas": {"value": args.tokens * world * args.steps / (rep_ms / 1e3), "unit": UNIT, "scaling": "weak",
                         "how": "each rank the whole layer on its own tokens, no data-path collective"},
            "e2e": {"value": args.tokens * args.steps / (e2e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "how": "each rank copies its T/N rows of the pinned-host inputs in (input stream), an NCCL "
                           "all-gather a module assembles x, every rank its fused shards + a peer barrier, each rank "
                           "copies its own columns of y back to pinned host memory on an output stream overlapping "
                           "the next step",
                    "d2h_mb_per_step": d2h / 1e6},
            "gpu_launches": args.steps * (len(names) + 1) * world,
            "clocks": clocks.summary(),
        }
        print(json.dumps(out), flush=True)


CFG5_DENSE_LAYER_BYTES = sum(p.rows * p.cols * 2 for p in workloads.QWEN25_32B)


def _bcast_from(v, src: int, world: int, device):
    """A float from rank src on every rank."""
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([float(v)], dtype=torch.float64, device=device)
    dist.broadcast(t, src)
    return float(t.item())


def _cfg5_down_sharded(args, rank, world, device, stream) -> dict:
    """The replica's 5120 x 27648 down projection (keep 40) row-sharded over the ranks, y gathered in the GEMM's
    epilogue by peer stores (shard.ShardedCompact): microseconds a call at the pass's T, against the same module on one
    GPU (rel-L2, rank 0) and the same bits on every rank."""
    import hashlib
    import torch.distributed as dist
    from p2pllm_b200 import compact, shard, wanda
    T = args.pass_tokens
    w = workloads.cfg5_weights(1, device)["down"]
    norms = workloads.cfg5_norms(1, device)["down"]
    values, idx = wanda.select(w, 40, norms)
    del w
    blocks = [("compact", values, idx, 27648)]
    x = workloads.activations(27648, T, 77, device)
    if world == 1:
        whole = compact.Compact(blocks)
        us = _region_ms(lambda: whole.apply(None, x), args.steps, stream) / args.steps * 1e3
        return {"us_per_call": us, "ranks": 1, "layout": whole.tiles.layout, "weights_mb": whole.nbytes() / 1e6}
    peers = shard.PeerGroup(None, device)
    sc = shard.ShardedCompact(blocks, fused=True, peers=peers, layout=args.layout)
    sc.prepare(T, torch.bfloat16, device)
    y = sc.apply(None, x).clone()
    digest = int.from_bytes(hashlib.sha256(y.cpu().view(torch.int16).numpy().tobytes()).digest()[:7], "little")
    every = [torch.zeros(1, dtype=torch.int64, device=device) for _ in range(world)]
    dist.all_gather(every, torch.tensor([digest], dtype=torch.int64, device=device))
    same = all(int(e.item()) == digest for e in every)
    rel = 0.0
    if rank == 0:
        want = compact.Compact(blocks).apply(None, x).double()
        rel = float((y.double() - want).norm() / want.norm())
    copies = max(1, -(-2 * L2_BYTES // max(sc.local.nbytes(), 1)))
    rotation = [sc] + [_clone_shard(sc) for _ in range(copies - 1)]
    turn = [0]

    def call():
        rotation[turn[0] % copies].apply_fused(x, sync=False)
        turn[0] += 1
        peers.barrier()

    for _ in range(max(3, copies)):
        call()
    torch.cuda.synchronize(device)
    dist.barrier()
    ms = max_over_ranks(_region_ms(call, args.steps, stream), world, device)
    peers.status()
    return {"us_per_call": ms / args.steps * 1e3, "ranks": world, "layout": sc.local.tiles.layout, "rows_per_rank": sc.mine,
            "shard_mb": sc.local.nbytes() / 1e6, "rel_l2_vs_one_gpu": _bcast_from(rel, 0, world, device),
            "same_bits_on_every_rank": same, "l2": f"{copies} copies of each rank's shard in turn",
            "how": "each rank its 128-row tiles of the module, y stored into every rank's y by the GEMM's epilogue, "
                   "one peer barrier a call"}


def run_cfg5(args, rank, world, device, peaks):
    """Config 5: the 64-layer Qwen2.5-32B-shaped model (workloads.DecoderBlock, random bf16
    weights) as 32 pair-steps, each with the keep-40 replica of its first layer, placed contiguously over `world` GPUs
    (plan.place). Each rank's share of a pass is one CUDA graph (plan.GraphedPass); the hidden state crosses each GPU
    boundary through the peer-memory hop with the step's group combine computed in the send (plan.PeerHop). Passes of
    T tokens are pipelined: rank r works on pass p while rank r + 1 works on pass p - 1. Beside it: one pass alone
    (latency), the hop's one-way time (peer memory and NCCL), and the row-sharded down projection."""
    import hashlib
    import torch.distributed as dist
    from p2pllm_b200 import plan
    T, H = args.pass_tokens, 5120
    stream = torch.cuda.current_stream(device)
    s = plan.steps(workloads.CFG5_GROUPS, workloads.CFG5_LAYERS)
    stages = plan.place(s, world)
    t0 = time.time()
    hop = plan.PeerHop(T, H, device=device) if world > 1 else None
    runner = plan.PlanRunner(s, stages, rank, None, None, hop)
    exact_ids, rep_ids = runner.layers_needed()
    exact = {i: workloads.cfg5_exact(i, device) for i in exact_ids}
    reps, rep_bytes = {}, 0
    for i in rep_ids:
        reps[i], nb = workloads.cfg5_replica(i, device, layout=args.layout)
        rep_bytes += nb
    runner.layer, runner.replica = exact.__getitem__, reps.__getitem__
    torch.cuda.synchronize(device)
    build_s = time.time() - t0
    like = torch.zeros(T, H, dtype=torch.bfloat16, device=device)
    inputs = [workloads.cfg5_input(p, T, device) for p in range(4)]
    last = world - 1

    # parity: pass 0 eager through the peer hop, and through the NCCL hop: the same bits on the last rank
    out0 = runner.pass_(0, inputs[0] if rank == 0 else None, like=like)
    same_nccl = True
    if world > 1:
        nccl_runner = plan.PlanRunner(s, stages, rank, exact.__getitem__, reps.__getitem__, plan.NcclHop())
        out_n = nccl_runner.pass_(0, inputs[0] if rank == 0 else None, like=like)
        nccl_runner.hop.finish()
        torch.cuda.synchronize(device)
        if rank == last:
            same_nccl = bool(torch.equal(out0, out_n))
        hop.status()
    digest = 0
    if rank == last:
        digest = int.from_bytes(hashlib.sha256(out0.cpu().view(torch.int16).numpy().tobytes()).digest()[:6], "little")
    digest = int(_bcast_from(digest, last, world, device))
    same_nccl = bool(_bcast_from(1.0 if same_nccl else 0.0, last, world, device))

    graphed = plan.GraphedPass(runner, like, next_pass=1)
    if rank == 0:
        graphed.h_in.copy_(inputs[0])
    graphed.run()                                      # pass 1 on pass 0's input: the graph gives the eager bits
    torch.cuda.synchronize(device)
    same_graph = bool(torch.equal(graphed.h_out, out0)) if rank == last else True
    same_graph = bool(_bcast_from(1.0 if same_graph else 0.0, last, world, device))
    done = [2]

    def one_pass():
        if rank == 0:
            graphed.h_in.copy_(inputs[done[0] % 4])
        graphed.run()
        done[0] += 1

    for _ in range(args.warmup):
        one_pass()
    torch.cuda.synchronize(device)
    barrier(world)
    # timed: K pipelined passes
    clocks = ClockSampler(device.index)
    with clocks:
        ms = max_over_ranks(_region_ms(one_pass, args.steps, stream), world, device)
    if hop is not None:
        hop.status()
    # one pass alone: the pipeline empty before and after it
    torch.cuda.synchronize(device)
    barrier(world)
    latency_ms = max_over_ranks(_region_ms(one_pass, 1, stream), world, device)

    # e2e: pinned-host inputs into rank 0, the pass's output back to pinned host memory on the last rank
    host_in = [t.cpu().pin_memory() for t in inputs]
    host_out = torch.empty(T, H, dtype=torch.bfloat16).pin_memory()

    def e2e_pass():
        if rank == 0:
            graphed.h_in.copy_(host_in[done[0] % 4], non_blocking=True)
        graphed.run()
        if rank == last:
            host_out.copy_(graphed.h_out, non_blocking=True)
        done[0] += 1

    for _ in range(3):
        e2e_pass()
    torch.cuda.synchronize(device)
    barrier(world)
    e2e_ms = max_over_ranks(_region_ms(e2e_pass, args.steps, stream), world, device)
    if hop is not None:
        hop.status()

    # the hop alone: ping-pong of a [T, 5120] bf16 hidden state between ranks 0 and 1, one-way time
    hop_us = {}
    if world > 1:
        ping = plan.PeerHop(T, H, device=device)
        buf = torch.zeros_like(like)
        x = inputs[0]
        k = [0]

        def peer_rt():
            if rank == 0:
                ping.send(plan.PART_SUM, [x], None, None, [1], k[0])
                ping.recv([1], k[0], like, out=buf)
            elif rank == 1:
                ping.recv([0], k[0], like, out=buf)
                ping.send(plan.PART_SUM, [buf], None, None, [0], k[0])
            k[0] += 1

        def nccl_rt():
            if rank == 0:
                dist.send(x, 1)
                dist.recv(buf, 1)
            elif rank == 1:
                dist.recv(buf, 0)
                dist.send(buf, 0)

        for fn, name in ((peer_rt, "peer_memory"), (nccl_rt, "nccl")):
            for _ in range(20):
                fn()
            torch.cuda.synchronize(device)
            barrier(world)
            rt_ms = _region_ms(fn, 200, stream) if rank < 2 else 0.0
            hop_us[name] = _bcast_from(rt_ms / 200 / 2 * 1e3, 0, world, device)
        ping.status()

    down = _cfg5_down_sharded(args, rank, world, device, stream)

    # bytes a pass reads on each rank: its dense layers' weights, its replicas' weights (activations are < 0.1%)
    my_bytes = len(exact_ids) * CFG5_DENSE_LAYER_BYTES + rep_bytes
    stage_bytes = max_over_ranks(float(my_bytes), world, device)
    per_gpu_gbs = stage_bytes * args.steps / (ms / 1e3) / 1e9
    st = stages[rank]
    n_steps = st.last - st.first + 1
    mine = n_steps * 4 + n_steps - (1 if runner.dsts else 0) + (1 if runner.dsts else 0) + (1 if runner.srcs else 0) \
        + (1 if (runner.srcs or runner.dsts) else 0)
    launches = mine
    if world > 1:
        t = torch.tensor([mine], dtype=torch.int64, device=device)
        dist.all_reduce(t)
        launches = int(t.item())
    if rank == 0:
        out = {
            "metric": "config-5 layer-parallel plan tokens/s (Qwen2.5-32B shapes, 64 layers as 32 pair-steps with "
                      f"keep-40 replicas, T={T})",
            "value": T * args.steps / (ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,0.02) bf16 weights; replicas selected with lognormal channel norms; "
                    "RMS-normalised N(0,1) pass inputs; no checkpoint)",
            "config": {"workload": f"cfg5 Qwen2.5-32B-shaped plan, T={T}", "layers": 64, "steps_per_gpu": n_steps,
                       "placement": "contiguous runs of whole pair-steps, one run a GPU",
                       "layer": "DecoderBlock: RMSNorm, qkv, causal attention of the pass's tokens (GQA 40/8, no KV "
                                "cache, no rotary), o, RMSNorm, SiLU(gate)*up, down; dense layers on cuBLAS, replicas "
                                "on the compact GEMM",
                       "step": "K passes pipelined over the GPUs, each rank's share of a pass one CUDA graph replay",
                       "l2": "inputs larger than L2: each rank reads %.1f GB of weights a pass" % (my_bytes / 1e9)},
            "parity": {"output_sha256_48": "%012x" % digest, "peer_hop_vs_nccl_hop_same_bits": same_nccl,
                       "graphed_vs_eager_same_bits": same_graph,
                       "how": "pass 0 through the plan with the peer-memory hop and with the NCCL hop; the hash is "
                              "the same at every GPU count when the plan is exact"},
            "latency_ms_one_pass": latency_ms,
            "hop_us_one_way": hop_us or None,
            "hop_bytes": T * H * 2,
            "down_row_sharded": down,
            "roofline": {"bound": "hbm", "achieved": per_gpu_gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": per_gpu_gbs / peaks["hbm_gbs"], "traffic": None, "peak_source": peaks["source"],
                         "kernel": "the slowest rank's stage: dense-layer and replica weight bytes a pass over the "
                                   "pipelined time a pass"},
            "e2e": {"value": T * args.steps / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": T * H * 2,
                    "d2h_bytes_per_step": T * H * 2,
                    "how": "rank 0 copies each pass's input from pinned host memory, the last rank copies the output "
                           "back, inside the timed region"},
            "gpu_launches": launches * args.steps,
            "build_s": build_s,
            "clocks": clocks.summary(),
        }
        print(json.dumps(out), flush=True)


def _timed_us(fn, reps: int) -> float:
    """Median CUDA-event time of fn over reps calls, each queued behind a spin (device time, not launch cost)."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    out = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(HEAD_START_CYCLES // 10)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        out.append(a.elapsed_time(b) * 1e3)
    return statistics.median(out)


def run_extra(args):
    """The extra workloads, one JSON line each (one GPU; not the headline)."""
    from p2pllm_b200 import compact, kernels, replica, wanda
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    peak = measured_peaks()
    reps = max(10, min(args.steps, 50))
    line = {"workload": args.workload, "n_gpus": 1, "higher_is_better": True, "data": "synthetic (seeded)",
            "peak_hbm_gbs": peak["hbm_gbs"], "peak_source": peak["source"]}
    if args.workload == "cfg1":
        # fp32 W [2048, 2048] keep 40, calibration 128 x 512 tokens, a 17-token forward (CUDA-core row kernel)
        cfg = workloads.config1(seed=0)
        sums = torch.zeros(cfg.w.shape[1], dtype=torch.float64, device=device)
        for chunk in cfg.calib_chunks(device):
            kernels.sumsq_cols(chunk, sums)
        w = cfg.w.to(device)
        values, idx = wanda.select(w, cfg.keep, wanda.channel_norms(sums, w))
        method = compact.Compact([("compact", values, idx, w.shape[1])])
        x = cfg.x.to(device)
        us = _timed_us(lambda: method.apply(None, x), reps)
        alg = values.numel() * (4 + 2) + 2 * x.numel() * 4
        line.update(metric="config-1 projection tokens/s (fp32, 2048 x 2048, keep 40, T=17)", value=17 / us * 1e6,
                    unit="tokens/s", us_per_pass=us, algorithmic_bytes=alg, hbm_gbs=alg / us / 1e3,
                    frac=alg / us / 1e3 / peak["hbm_gbs"], dtype="f32", kernel="spmm_rows (layout rows)")
    elif args.workload == "cfg3":
        # A Llama-shaped residual MLP block (hidden 4096, intermediate 14336): l(x) = x + down(silu(gate x) * up x).
        # The group: the dense block l0 (torch GEMMs, not timed) and the keep-40 replica of the next block; timed:
        # the replica's compact GEMMs (gate and up in one launch with SiLU * up in its epilogue) and the group combine
        # h' = l0(h) + dtype(l1'(h) - h).
        H, I = 4096, 14336
        g = torch.Generator(device=device).manual_seed(3)
        mods = {}
        for name, rows, cols in (("gate_up", 2 * I, H), ("down", H, I)):
            w = (torch.randn(rows, cols, generator=g, device=device) * 0.02).bfloat16()
            norms = torch.rand(cols, generator=g, device=device) + 0.1
            values, idx = wanda.select(w, 40, norms)
            if name == "gate_up":
                gt = compact.GatedTiles([("compact", values[:I], idx[:I], cols), ("compact", values[I:], idx[I:], cols)])
                mods[name] = (gt, values.numel() * 4)
            else:
                mods[name] = (compact.Compact([("compact", values, idx, cols)]), values.numel() * 4)
            del w
        per_t = {}
        for T in (1, 8, 32, 64):
            h = torch.randn(T, H, generator=g, device=device)
            h = (h / h.pow(2).mean(-1, keepdim=True).sqrt()).bfloat16()          # RMS-normalised rows
            l0 = torch.randn(T, H, generator=g, device=device).bfloat16()        # the dense member's output

            def step():
                a = mods["gate_up"][0](h)
                l1 = h + mods["down"][0].apply(None, a)
                return replica.combine([l0, l1], h, h)

            us = _timed_us(step, reps)
            alg = mods["gate_up"][1] + mods["down"][1] + T * (H * 2 + I * 2 + I * 2 + H * 2) + 4 * T * H * 2
            per_t[T] = {"us": us, "tokens_per_s": T / us * 1e6, "hbm_gbs": alg / us / 1e3,
                        "frac": alg / us / 1e3 / peak["hbm_gbs"]}
        line.update(metric="config-3 replica member + combine tokens/s (keep 40 MLP block, hidden 4096)",
                    value=per_t[64]["tokens_per_s"], unit="tokens/s", per_tokens=per_t, dtype="bf16",
                    note="synthetic residual-MLP block stands in for a decoder layer (no KV cache here)")
    elif args.workload == "cfg4":
        # Routed experts: hidden 2048, 128 experts, top-8 of N(0,1) router logits, intermediate 768, keep 30, 272
        # tokens; one pass of moe.GroupedMoE (route, gather, gate/up launch with SiLU * up in its epilogue, down
        # launch, weighted combine), and the same pass with SiLU * up between the launches
        from types import SimpleNamespace as NS
        from p2pllm_b200 import moe
        E, R, H, T, K = 128, 768, 2048, 272, 8
        g = torch.Generator(device=device).manual_seed(4)
        blocks = {}
        for name, rows, cols in (("w13_weight", 2 * R, H), ("w2_weight", H, R)):
            w = (torch.randn(E, rows, cols, generator=g, device=device) * 0.05).bfloat16()
            norms = torch.rand(E, cols, generator=g, device=device) + 0.1
            sel = [wanda.select(w[e], 30, norms[e]) for e in range(E)]
            values, idx = torch.stack([s_[0] for s_ in sel]), torch.stack([s_[1] for s_ in sel])
            if name == "w13_weight":
                blocks[name] = [("compact", values[:, :R], idx[:, :R], cols), ("compact", values[:, R:], idx[:, R:], cols)]
            else:
                blocks[name] = [("compact", values, idx, cols)]
            del w
        fused = moe.GroupedMoE(None, blocks)
        unfused = moe.GroupedMoE(None, blocks)
        unfused.w13 = moe.ExpertTiles(blocks["w13_weight"])
        wts, ids = torch.topk(torch.softmax(torch.randn(T, E, generator=g, device=device), -1), K)
        d = NS(hidden_states=torch.randn(T, H, generator=g, device=device).bfloat16(),
               topk_output=NS(topk_ids=ids, topk_weights=wts))
        us = _timed_us(lambda: fused.apply(None, d), reps)
        us_unfused = _timed_us(lambda: unfused.apply(None, d), reps)
        used = int(torch.unique(ids).numel())
        alg = sum(b[1].numel() * 4 for bl in blocks.values() for b in bl) * used // E + T * H * 2 * 2
        line.update(metric="config-4 routed-expert pass tokens/s (128 experts, top-8, keep 30, T=272)",
                    value=T / us * 1e6, unit="tokens/s", us_per_pass=us, us_per_pass_silu_between_launches=us_unfused,
                    experts_reached=used, algorithmic_bytes=alg, hbm_gbs=alg / us / 1e3,
                    frac=alg / us / 1e3 / peak["hbm_gbs"], dtype="bf16",
                    kernel="moe.GroupedMoE: p2p_moe_route, p2p_spmm_tc_grouped_gated, p2p_spmm_tc_grouped, "
                           "p2p_moe_combine")
    elif args.workload == "module":
        # one module of the cfg2 layer, --steps launches at --tokens tokens (each behind a spin), for profiling
        from p2pllm_b200 import compact as cp
        layer = ReplicaLayer(seed=0, tokens=args.tokens, calib_tokens=args.calib_tokens, device=device)
        names = MODULES[args.module][1]
        blocks = [("compact", *layer.selected[n], layer.proj[n].cols) for n in names]
        tiles = cp.Tiles(blocks, layout=args.layout)
        x = layer.inputs[MODULES[args.module][0]]
        us = _timed_us(lambda: tiles(x), max(3, args.steps))
        alg = layer.algorithmic_bytes(args.module, args.tokens)
        fmt = layer.mask_format_bytes(args.module) + args.tokens * (layer.cols(args.module) + layer.rows(args.module)) * 2
        line.update(metric=f"{args.module} launch us (cfg2 layer, T={args.tokens}, layout {tiles.layout})", value=us,
                    unit="us", higher_is_better=False, layout=tiles.layout, tokens=args.tokens,
                    bytes_read_and_written=tiles.nbytes() + args.tokens * (layer.cols(args.module)
                                                                           + layer.rows(args.module)) * 2,
                    hbm_gbs=(tiles.nbytes() + args.tokens * (layer.cols(args.module) + layer.rows(args.module)) * 2)
                    / us / 1e3, index_format_bytes=alg, mask_format_bytes=fmt, dtype="bf16")
    else:
        # a Qwen2.5-32B replica layer (keep 40 everywhere), T = 17
        layer = ReplicaLayer(seed=0, tokens=17, calib_tokens=args.calib_tokens, device=device,
                             projections=workloads.QWEN25_32B)
        us = _timed_us(layer.step, reps)
        alg = sum(layer.algorithmic_bytes(n, 17) for n in MODULES)
        line.update(metric="config-5 replica layer tokens/s (Qwen2.5-32B shapes, keep 40, T=17)", value=17 / us * 1e6,
                    unit="tokens/s", us_per_pass=us, algorithmic_bytes=alg, hbm_gbs=alg / us / 1e3,
                    frac=alg / us / 1e3 / peak["hbm_gbs"], dtype="bf16")
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    rank, world, local = dist_env()
    if args.workload == "cfg5" and not args.cfg5_single_layer and args.impl == "b200":
        if world > 1:
            import datetime
            import torch.distributed as dist
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", local))
        try:
            device = torch.device("cuda", local)
            torch.cuda.set_device(device)
            run_cfg5(args, rank, world, device, measured_peaks())
        finally:
            if world > 1:
                import torch.distributed as dist
                dist.destroy_process_group()
        return
    if args.workload != "cfg2":
        if rank == 0:
            run_extra(args)
        return
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    try:
        run_b200(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
