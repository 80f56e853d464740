"""A layer-parallel plan over the GPUs of one node: which rank runs which of a plan's steps, and the hidden-state hop
between them over NVLink, with a member's part and the receiver's sum computed in the hop's own kernels.

    steps       p2p/route.py:46-53     the plan's steps in order: its groups, and every other layer alone
    place       p2p/route.py:56-86     each rank's share: a run of whole steps, or one member of a spread step
    sources     p2p/route.py:89-96     the ranks a rank receives a pass's input from, in member order
    targets     p2p/route.py:99-110    the ranks a rank sends its output to
    PeerHop     p2p/route.py:800-810 (_send_piece), 825-831 (_summed), 1254-1274 (_member): one kernel a side
                (p2p_hop_send / p2p_hop_recv) over an inbox in symmetric memory
    NcclHop     the same hop as the reference runs it: the part and the sum as kernels of their own, NCCL isend/irecv
    PlanRunner  p2p/route.py:1208-1274 with p2p/replica.py:70-85: one rank's share of a pass

A step of n > 1 layers is a replica group: members 0..n-2 read the step's input h, the last reads h~ = replica(h),
the pruned copy of layer n-2, and the next step reads h' = combine(...) (p2p/replica.py:81-85). A rank that runs whole
steps combines locally, except on its last step, whose combine goes straight into the hop to the next ranks; a
member of a spread step sends its part -- l_0(h) for the first, dtype(l_k(x) - x) for the others -- and the next
step's ranks add the parts in fp32 in member order.

The SGLang pipeline around it (the head rank, request framing, KV-cache updates, streaming) is not part of this
package: a pass here is a [T, hidden] hidden state in and out.
"""
from __future__ import annotations

import ctypes
from typing import Callable, NamedTuple

import torch
import torch.distributed as dist

from . import _lib, kernels

PART_SUM, PART_DIFF, PART_COMBINE = 0, 1, 2


def steps(groups: list, num_layers: int) -> list:
    """The plan's steps in order: each group (a list of neighbouring layers) and every other layer alone."""
    starts = {g[0]: list(g) for g in groups}
    out, i = [], 0
    while i < num_layers:
        step = starts.get(i, [i])
        out.append(step)
        i = step[-1] + 1
    return out


class Stage(NamedTuple):
    """One rank's share of a plan: steps first..last (indices into steps()), whole, or member `member` of step first
    (a spread step, first == last)."""
    first: int
    last: int
    member: "int | None" = None


def _split(n: int, parts: int) -> list:
    """n items cut into `parts` runs as evenly as possible, the longer runs first: [(start, stop), ...]."""
    base, extra = divmod(n, parts)
    out, at = [], 0
    for k in range(parts):
        size = base + (1 if k < extra else 0)
        out.append((at, at + size))
        at += size
    return out


def place(plan_steps: list, world: int, spread=()) -> list:
    """The stages of `world` ranks in pipeline order (rank i runs stages[i]). Each step in `spread` (indices into
    plan_steps; groups of two or more layers, not the last step) takes one rank per member; the other steps run whole,
    cut into contiguous runs: every run of steps between spread steps gets ranks in proportion to its length (at least
    one each), and its steps are split evenly over them. Raises ValueError if the ranks do not fit the plan."""
    n = len(plan_steps)
    spread = sorted(set(spread))
    for j in spread:
        if not 0 <= j < n - 1:
            raise ValueError(f"step {j}: only steps before the last can be spread (the last rank ends the pass)")
        if len(plan_steps[j]) < 2:
            raise ValueError(f"step {j} is a single layer: nothing to spread")
    segments, at = [], 0
    for j in spread + [n]:
        if j > at:
            segments.append((at, j))
        if j < n:
            segments.append(("spread", j))
        at = j + 1
    runs = [s for s in segments if s[0] != "spread"]
    free = world - sum(len(plan_steps[j]) for _, j in (s for s in segments if s[0] == "spread"))
    if free < len(runs) or free > sum(b - a for a, b in runs):
        raise ValueError(f"{world} ranks for {len(runs)} runs of whole steps ({sum(b - a for a, b in runs)} steps) "
                         f"and {len(spread)} spread steps")
    share = {s: 1 for s in runs}
    for _ in range(free - len(runs)):
        s = max((s for s in runs if share[s] < s[1] - s[0]), key=lambda s: (s[1] - s[0]) / share[s])
        share[s] += 1
    stages = []
    for s in segments:
        if s[0] == "spread":
            stages += [Stage(s[1], s[1], k) for k in range(len(plan_steps[s[1]]))]
        else:
            stages += [Stage(s[0] + a, s[0] + b - 1) for a, b in _split(s[1] - s[0], share[s])]
    return stages


def _of_step(stages: list, j: int) -> list:
    return [i for i, s in enumerate(stages) if s.first <= j <= s.last]


def sources(stages: list, i: int) -> list:
    """The ranks that rank i receives its pass input from, in member order ([] for the first step: the pass's input)."""
    first = stages[i].first
    return _of_step(stages, first - 1) if first else []


def targets(stages: list, i: int) -> list:
    """The ranks that rank i sends its output to ([] for the last step: the pass's output)."""
    return _of_step(stages, stages[i].last + 1)


# ---- the hop ---------------------------------------------------------------------------------------------------------

class KernelOps:
    """The elementwise steps of a pass, as this package's CUDA kernels."""
    combine = staticmethod(kernels.combine)
    member_part = staticmethod(kernels.member_part)
    summed = staticmethod(kernels.sum_parts)


def _part(ops, mode: int, parts: list, h, h_copy):
    if mode == PART_SUM:
        return parts[0] if len(parts) == 1 else ops.summed(parts)
    if mode == PART_DIFF:
        return ops.member_part(parts[0], h)
    return ops.combine(parts, h, h_copy)


class NcclHop:
    """The hop as the reference runs it: the part made by a kernel of its own, one isend per destination, one irecv
    per source, then the sum (p2p/route.py:800-810, 825-831). ops: the elementwise steps (KernelOps by default)."""

    def __init__(self, group=None, ops=KernelOps):
        self.group, self.ops = group, ops
        self._pending: list = []

    def send(self, mode: int, parts: list, h, h_copy, dsts: list, p: int) -> None:
        part = _part(self.ops, mode, parts, h, h_copy).contiguous()
        works = [dist.isend(part, d, group=self.group) for d in dsts]
        self._pending.append((works, part))
        while len(self._pending) > 2:                  # the part stays alive until its sends are done
            for w in self._pending.pop(0)[0]:
                w.wait()

    def recv(self, srcs: list, p: int, like: torch.Tensor) -> torch.Tensor:
        bufs = [torch.empty_like(like) for _ in srcs]
        for w in [dist.irecv(b, s, group=self.group) for b, s in zip(bufs, srcs)]:
            w.wait()
        return bufs[0] if len(bufs) == 1 else self.ops.summed(bufs)

    def finish(self) -> None:
        for works, _ in self._pending:
            for w in works:
                w.wait()
        self._pending = []


class PeerHop:
    """The hop over NVLink peer memory: every rank an inbox in symmetric memory (ring slots per sender) that peers
    store into. send() computes the part and stores it into every destination's inbox in one kernel
    (p2p_hop_send); recv() waits for the parts and adds them in fp32 in member order in one kernel (p2p_hop_recv).
    Waits are bounded (wait_us); status() raises if one gave up. Created by all ranks of the group together."""

    def __init__(self, tokens: int, hidden: int, dtype=torch.bfloat16, ring: int = 2, group=None, device=None,
                 wait_us: int = 5_000_000):
        from .shard import _symmetric
        self.group = group
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.cap, self.hidden, self.dtype, self.ring, self.wait_us = tokens * hidden, hidden, dtype, ring, wait_us
        size = _lib.load().p2p_hop_inbox_bytes(self.world, self.cap, _lib.DTYPES[dtype], ring)
        if not size:
            raise _lib.P2PError(f"no inbox for {self.world} ranks, {self.cap} elements, ring {ring}")
        self.inbox, self.ptrs = _symmetric((size,), torch.uint8, self.device, group)
        self.inbox.zero_()
        torch.cuda.synchronize(self.device)
        dist.barrier(group)                            # every inbox is zero before the first hop

    @staticmethod
    def _ranks(rs: list):
        return (ctypes.c_int * len(rs))(*rs)

    @staticmethod
    def _pass(p) -> tuple:
        """(pass number, device address of the pass counter or None): p is an int or a counter tensor (int32 [1])."""
        if torch.is_tensor(p):
            return 0, p.data_ptr()
        return p & 0xffffffff, None

    def send(self, mode: int, parts: list, h, h_copy, dsts: list, p) -> None:
        ref = parts[0]
        parts = [t.contiguous() for t in parts]
        n, at = self._pass(p)
        _lib.call("p2p_hop_send", mode, kernels._ptr_array(parts), len(parts), _lib.ptr(h), _lib.ptr(h_copy),
                  _lib.dtype_code(ref), ref.numel(), self.ptrs, self.world, self.rank, self._ranks(dsts), len(dsts),
                  n, at, self.ring, self.cap, self.wait_us, _lib.stream_of(ref))

    def recv(self, srcs: list, p, like: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        out = torch.empty_like(like) if out is None else out
        n, at = self._pass(p)
        _lib.call("p2p_hop_recv", self.ptrs, self.world, self.rank, self._ranks(srcs), len(srcs), n, at, self.ring,
                  self.cap, _lib.dtype_code(out), out.numel(), _lib.ptr(out), self.wait_us, _lib.stream_of(out))
        return out

    @staticmethod
    def advance(counter: torch.Tensor) -> None:
        """The pass counter a graphed pass reads moves on by one (on the current stream)."""
        _lib.call("p2p_hop_advance", counter.data_ptr(), counter.numel(), _lib.stream_of(counter))

    def status(self) -> None:
        """Raises if a hop wait gave up since the last call. Syncs."""
        _lib.call("p2p_hop_status", 1, torch.cuda.current_stream(self.device).cuda_stream)

    def finish(self) -> None:
        pass


class _NoHop:
    """Stands in for the hop while a stage's kernels are run once before capture: receives zeros, sends nothing."""

    def recv(self, srcs, p, like, out=None):
        return torch.zeros_like(like)

    def send(self, *args) -> None:
        pass


# ---- one rank's share of a pass --------------------------------------------------------------------------------------

class PlanRunner:
    """Rank `rank`'s share of a plan: layer(i) -> the callable of layer i (h -> its output, residual included) and
    replica(i) -> the pruned copy of layer i, for the layers this rank's stage needs. pass_(p, h) runs pass p: receives
    the input from the previous step's ranks (or takes h on the first stage), runs the stage, sends its output or part
    to the next step's ranks, and returns the output on the last stage (None elsewhere). Every rank runs the same passes
    in the same order (p = 0, 1, 2, ...)."""

    def __init__(self, plan_steps: list, stages: list, rank: int, layer: Callable, replica: Callable, hop,
                 ops=KernelOps):
        self.steps, self.stages, self.rank = plan_steps, stages, rank
        self.stage = stages[rank]
        self.layer, self.replica, self.hop, self.ops = layer, replica, hop, ops
        self.srcs, self.dsts = sources(stages, rank), targets(stages, rank)

    def layers_needed(self) -> tuple:
        """(layer ids run exactly, layer ids run as replicas) on this rank."""
        s = self.stage
        if s.member is not None:
            g = self.steps[s.first]
            if s.member == len(g) - 1:
                return [g[-1]], [g[-2]]
            return [g[s.member]], []
        exact, copies = [], []
        for j in range(s.first, s.last + 1):
            exact += self.steps[j]
            if len(self.steps[j]) > 1:
                copies.append(self.steps[j][-2])
        return exact, copies

    def _members(self, g: list, h):
        """(the members' outputs, h~) of a group on input h."""
        ys = [self.layer(i)(h) for i in g[:-1]]
        h_copy = self.replica(g[-2])(h)
        ys.append(self.layer(g[-1])(h_copy))
        return ys, h_copy

    def pass_(self, p: int, h: torch.Tensor | None = None, like: torch.Tensor | None = None):
        s = self.stage
        if self.srcs:
            h = self.hop.recv(self.srcs, p, like if like is not None else h)
        if s.member is not None:
            g = self.steps[s.first]
            if s.member < len(g) - 1:
                y = self.layer(g[s.member])(h)
                mode, parts, x = (PART_SUM, [y], None) if s.member == 0 else (PART_DIFF, [y], h)
            else:
                x = self.replica(g[-2])(h)
                mode, parts = PART_DIFF, [self.layer(g[-1])(x)]
            self.hop.send(mode, parts, x, None, self.dsts, p)
            return None
        for j in range(s.first, s.last + 1):
            g = self.steps[j]
            boundary = j == s.last and self.dsts
            if len(g) == 1:
                y = self.layer(g[0])(h)
                if boundary:
                    self.hop.send(PART_SUM, [y], None, None, self.dsts, p)
                    return None
                h = y
                continue
            ys, h_copy = self._members(g, h)
            if boundary:
                self.hop.send(PART_COMBINE, ys, h, h_copy, self.dsts, p)
                return None
            h = self.ops.combine(ys, h, h_copy)
        return h


class GraphedPass:
    """A rank's share of a pass as one CUDA graph: receive (or read h_in on the first stage), the stage's layers,
    replicas and combines, the hop's send, and the step of the device pass counter the hops read -- one replay per
    pass, so the host's cost is one launch however many kernels the stage runs. The first stage copies each pass's
    input into h_in before run(); the last stage reads the pass's output from h_out after it (valid until the next
    run()). next_pass: the number of passes the ranks have run before (the counter's start). PeerHop only."""

    def __init__(self, runner: PlanRunner, like: torch.Tensor, next_pass: int = 0):
        self.runner = runner
        self.h_in = torch.zeros_like(like)
        self.counter = torch.full((1,), next_pass, dtype=torch.int32, device=like.device)
        hop = runner.hop
        runner.hop = _NoHop()
        try:                                    # every kernel's first launch (module loads, library handles) off-graph
            runner.pass_(0, self.h_in, like=self.h_in)
        finally:
            runner.hop = hop
        torch.cuda.synchronize(like.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=torch.cuda.Stream(like.device)):
            self.h_out = runner.pass_(self.counter, self.h_in, like=self.h_in)
            if hop is not None and (runner.srcs or runner.dsts):
                hop.advance(self.counter)

    def run(self) -> None:
        self.graph.replay()
