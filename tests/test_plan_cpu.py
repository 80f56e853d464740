"""The layer-parallel plan's host logic on CPU: the placement of a plan's steps over ranks (plan.place / sources /
targets, p2p/route.py:46-110) and a pass through the plan on gloo ranks in child processes, with the hop over
gloo isend/irecv (plan.NcclHop) and the elementwise steps from the oracle: the last rank's output is bit-identical
to the same plan run whole in one process, for contiguous runs and for a spread step whose members sit on ranks of
their own."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from p2pllm_b200 import plan
from p2pllm_b200.workloads import CFG5_GROUPS, CFG5_LAYERS


def test_steps_are_groups_and_single_layers():
    assert plan.steps([[1, 2], [4, 5, 6]], 8) == [[0], [1, 2], [3], [4, 5, 6], [7]]
    assert plan.steps(CFG5_GROUPS, CFG5_LAYERS) == CFG5_GROUPS


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_cfg5_contiguous_placement(world):
    s = plan.steps(CFG5_GROUPS, CFG5_LAYERS)
    stages = plan.place(s, world)
    per = 32 // world
    assert stages == [plan.Stage(r * per, (r + 1) * per - 1) for r in range(world)]
    for r in range(world):
        assert plan.sources(stages, r) == ([r - 1] if r else [])
        assert plan.targets(stages, r) == ([r + 1] if r < world - 1 else [])


def test_uneven_runs_take_the_extra_steps_first():
    stages = plan.place(plan.steps([], 7), 3)
    assert [(st.first, st.last) for st in stages] == [(0, 2), (3, 4), (5, 6)]


def test_spread_step_takes_a_rank_per_member():
    s = plan.steps([[0, 1], [2, 3, 4], [5, 6]], 9)          # [[0,1],[2,3,4],[5,6],[7],[8]]
    stages = plan.place(s, 6, spread=[1])
    assert stages[0] == plan.Stage(0, 0)
    assert stages[1:4] == [plan.Stage(1, 1, k) for k in range(3)]
    assert [(st.first, st.last, st.member) for st in stages[4:]] == [(2, 3, None), (4, 4, None)]
    assert plan.targets(stages, 0) == [1, 2, 3]               # every member gets the step's input
    assert plan.sources(stages, 4) == [1, 2, 3]               # the next rank adds the parts in member order
    assert all(plan.targets(stages, r) == [4] for r in (1, 2, 3))
    assert plan.sources(stages, 5) == [4] and plan.targets(stages, 5) == []


def test_every_send_has_its_receive():
    s = plan.steps([[0, 1], [2, 3], [4, 5], [6, 7]], 10)
    for world, spread in ((3, []), (5, [1]), (7, [0, 2]), (6, [])):
        stages = plan.place(s, world, spread)
        assert len(stages) == world
        sends = {(r, d) for r in range(world) for d in plan.targets(stages, r)}
        recvs = {(src, r) for r in range(world) for src in plan.sources(stages, r)}
        assert sends == recvs
        covered = sorted(j for st in stages for j in range(st.first, st.last + 1) if st.member in (None, 0))
        assert covered == list(range(len(s)))


def test_placements_that_do_not_fit_are_refused():
    s = plan.steps(CFG5_GROUPS, CFG5_LAYERS)
    with pytest.raises(ValueError):
        plan.place(s, 33)                                    # more ranks than steps
    with pytest.raises(ValueError):
        plan.place(s, 2, spread=[31])                         # the last step ends the pass
    with pytest.raises(ValueError):
        plan.place(plan.steps([], 4), 2, spread=[0])           # a single layer has no members to spread
    with pytest.raises(ValueError):
        plan.place(s, 2, spread=[3, 10])                       # 4 member ranks + 3 runs > 2 ranks


# ---- a pass through the plan over gloo ranks ---------------------------------------------------------------------------

HIDDEN, TOKENS, LAYERS = 16, 3, 8
GROUPS = [[0, 1], [2, 3], [4, 5], [6, 7]]


def _weights(i: int, pruned: bool) -> torch.Tensor:
    g = torch.Generator().manual_seed(100 + i)
    w = torch.randn(HIDDEN, HIDDEN, generator=g) * 0.3
    if pruned:
        w = w * (torch.rand(HIDDEN, HIDDEN, generator=g) < 0.5)
    return w


def _layer(i: int):
    w = _weights(i, False)
    return lambda h: h + torch.tanh(h @ w)


def _replica(i: int):
    w = _weights(i, True)
    return lambda h: h + torch.tanh(h @ w)


class _OracleOps:
    """The pass's elementwise steps from the oracle (fp32 on the CPU)."""
    import oracle as _o

    @classmethod
    def combine(cls, parts, h, h_copy):
        return torch.from_numpy(cls._o.combine([p.numpy() for p in parts], h.numpy(), h_copy.numpy(), "f32"))

    @classmethod
    def member_part(cls, y, x):
        return torch.from_numpy(cls._o.member_part(y.numpy(), x.numpy(), "f32"))

    @classmethod
    def summed(cls, parts):
        return torch.from_numpy(cls._o.summed([p.numpy() for p in parts], "f32"))


def _input(p: int) -> torch.Tensor:
    return torch.randn(TOKENS, HIDDEN, generator=torch.Generator().manual_seed(7 + p))


def _whole(p: int) -> torch.Tensor:
    s = plan.steps(GROUPS, LAYERS)
    runner = plan.PlanRunner(s, plan.place(s, 1), 0, _layer, _replica, None, ops=_OracleOps)
    return runner.pass_(p, _input(p))


def _pipeline(rank, world, spread):
    s = plan.steps(GROUPS, LAYERS)
    stages = plan.place(s, world, spread)
    hop = plan.NcclHop(ops=_OracleOps)
    runner = plan.PlanRunner(s, stages, rank, _layer, _replica, hop, ops=_OracleOps)
    outs = [runner.pass_(p, _input(p) if rank == 0 else None, like=_input(p)) for p in range(3)]
    hop.finish()
    return [None if o is None else o.numpy() for o in outs]


def _contiguous(rank, world):
    return _pipeline(rank, world, [])


def _spread(rank, world):
    return _pipeline(rank, world, [1])


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(rank, world, port, fn, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        q.put((rank, fn(rank, world)))
    finally:
        dist.destroy_process_group()


def _spawn(fn, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, world, port, fn, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return out


@pytest.mark.parametrize("fn,world", [(_contiguous, 2), (_contiguous, 4), (_spread, 4)],
                         ids=["contiguous-2", "contiguous-4", "spread-step-1-over-2-ranks"])
def test_pass_through_the_plan_is_the_whole_plan(fn, world):
    out = _spawn(fn, world)
    for p in range(3):
        assert np.array_equal(out[world - 1][p], _whole(p).numpy())
        assert all(out[r][p] is None for r in range(world - 1))
