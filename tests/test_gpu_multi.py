"""The multi-GPU paths on GPUs: a row-sharded compact module (shard.ShardedCompact, an NCCL all-gather of y) against
the single-GPU Compact; the spread-step hop (route.send_piece / recv_parts over NCCL, summed by the GPU kernel in
member order) against the oracle's sum; a layer-parallel plan placed over the ranks (plan.PlanRunner with the
peer-memory hop, eager and graphed, and with the NCCL hop) against the same plan on one GPU. One rank per GPU in child
processes; the two-rank cases need two GPUs and are skipped on one (the world-size-1 cases always run)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _module(seed=0, rows=(1024, 256, 256), cols=2048, keep=33):
    from p2pllm_b200 import wanda
    g = torch.Generator(device="cuda").manual_seed(seed)
    norms = torch.rand(cols, generator=g, device="cuda") + 0.1
    blocks = []
    for r in rows:
        w = (torch.randn(r, cols, generator=g, device="cuda") * 0.02).bfloat16()
        v, i = wanda.select(w, keep, norms)
        blocks.append(("compact", v, i, cols))
    x = torch.randn(17, cols, generator=g, device="cuda").bfloat16()
    return blocks, x


def _sharded(rank, world, fused=None, layout=None, push=None):
    """(rel-L2 of the sharded y against the whole module's, y's shape, a hash of y's bits). The shards may split their
    columns differently from the whole module, so sums can differ in the last bf16 bit."""
    import hashlib
    from p2pllm_b200 import compact, shard
    blocks, x = _module()
    sc = shard.ShardedCompact(blocks, fused=fused, layout=layout, push=push)
    y = sc.apply(None, x)
    y2 = sc.apply(None, x * 2)                          # the other of the two buffers (fused), then the first again
    y3 = sc.apply(None, x)
    want = compact.Compact(blocks).apply(None, x).double()
    rel = float((y3.double() - want).norm() / want.norm())
    rel2 = float((y2.double() - 2 * want).norm() / (2 * want).norm())
    if sc.peers is not None:
        sc.peers.status()
    return max(rel, rel2), tuple(y3.shape), hashlib.sha256(y3.cpu().view(torch.int16).numpy().tobytes()).hexdigest()


def _sharded_nccl(rank, world):
    return _sharded(rank, world, fused=False)


def _sharded_mask(rank, world):
    return _sharded(rank, world, layout="mask")


def _sharded_push(rank, world):
    return _sharded(rank, world, push=True)


def _barrier_gives_up(rank, world):
    """Rank 1 enters a peer barrier that rank 0 never joins: its wait runs out after 20 ms, the status names rank 0,
    and a barrier both ranks then join completes."""
    from p2pllm_b200 import shard
    from p2pllm_b200._lib import P2PError
    peers = shard.PeerGroup()
    failed = False
    if rank == 1:
        peers.barrier(timeout_us=20_000)
        torch.cuda.synchronize()
        try:
            peers.status()
        except P2PError as e:
            failed = "rank 0" in str(e)
    dist.barrier()                                       # the host learns of it; both ranks move on together
    peers.epoch = 1
    peers.barrier()
    torch.cuda.synchronize()
    peers.status()
    return failed if rank == 1 else True


def _hop(rank, world):
    from p2pllm_b200 import route
    import oracle
    g = torch.Generator(device="cuda").manual_seed(rank)
    piece = torch.randn(17, 4096, generator=g, device="cuda").bfloat16()
    peers = [r for r in range(world) if r != rank]
    others = route.exchange(piece, peers, peers)
    parts = [piece if r == rank else others.pop(0) for r in range(world)]
    got = route.summed(parts)
    bits = lambda t: t.cpu().view(torch.int16).numpy().view(np.uint16)
    want = oracle.summed([bits(p) for p in parts], "bf16")
    return bool(np.array_equal(bits(got), want))


def _plan_layers(hidden=512):
    """Small GPU layers for a plan of 4 pair-steps: layer i is h + tanh(h W_i^T) (dense bf16), its replica the same with
    W_i pruned to keep 40 by the package's selection and run by the compact GEMM."""
    import torch.nn.functional as F
    from p2pllm_b200 import compact, wanda
    exact, reps = {}, {}
    for i in range(8):
        g = torch.Generator(device="cuda").manual_seed(300 + i)
        w = (torch.randn(hidden, hidden, generator=g, device="cuda") * 0.05).bfloat16()
        norms = torch.rand(hidden, generator=g, device="cuda") + 0.1
        c = compact.Compact([("compact", *wanda.select(w, 40, norms), hidden)])
        exact[i] = (lambda w: lambda h: h + torch.tanh(F.linear(h, w)))(w)
        reps[i] = (lambda c: lambda h: h + torch.tanh(c.apply(None, h)))(c)
    return exact, reps


def _plan_over_gpus(rank, world):
    """A pass through a 4-step plan placed over the ranks, the hop over peer memory (eager, then as a CUDA graph a
    pass) and over NCCL: (the last rank's outputs equal the whole plan run on that GPU alone, bit for bit)."""
    from p2pllm_b200 import plan
    exact, reps = _plan_layers()
    s = plan.steps([[0, 1], [2, 3], [4, 5], [6, 7]], 8)
    stages = plan.place(s, world)
    inputs = [torch.randn(17, 512, generator=torch.Generator(device="cuda").manual_seed(50 + p),
                          device="cuda").bfloat16() for p in range(6)]
    hop = plan.PeerHop(17, 512)
    runner = plan.PlanRunner(s, stages, rank, exact.__getitem__, reps.__getitem__, hop)
    outs = [runner.pass_(p, inputs[p] if rank == 0 else None, like=inputs[0]) for p in range(2)]
    graphed = plan.GraphedPass(runner, inputs[0], next_pass=2)
    for p in range(2, 6):
        if rank == 0:
            graphed.h_in.copy_(inputs[p])
        graphed.run()
        outs.append(graphed.h_out.clone() if rank == world - 1 else None)
    hop.status()
    nccl = plan.PlanRunner(s, stages, rank, exact.__getitem__, reps.__getitem__, plan.NcclHop())
    outs.append(nccl.pass_(0, inputs[0] if rank == 0 else None, like=inputs[0]))
    nccl.hop.finish()
    torch.cuda.synchronize()
    if rank != world - 1:
        return all(o is None for o in outs)
    whole = plan.PlanRunner(s, plan.place(s, 1), 0, exact.__getitem__, reps.__getitem__, None)
    want = [whole.pass_(p, inputs[p]) for p in range(6)] + [whole.pass_(0, inputs[0])]
    return all(torch.equal(o, w) for o, w in zip(outs, want))


def _hop_gives_up(rank, world):
    """Rank 1 waits 20 ms for a part that rank 0 never sends: the status names rank 0; after the hosts agree, a pass
    sent and received goes through."""
    from p2pllm_b200 import plan
    from p2pllm_b200._lib import P2PError
    hop = plan.PeerHop(4, 256, wait_us=20_000)
    x = torch.full((4, 256), float(rank + 1), device="cuda").bfloat16()
    failed = True
    if rank == 1:
        hop.recv([0], 0, x)
        torch.cuda.synchronize()
        try:
            hop.status()
            failed = False
        except P2PError as e:
            failed = "rank 0" in str(e)
    dist.barrier()
    hop.wait_us = 5_000_000
    if rank == 0:
        hop.send(plan.PART_SUM, [x], None, None, [1], 0)
        ok = True
    else:
        ok = bool(torch.equal(hop.recv([0], 0, x), torch.ones_like(x)))
    torch.cuda.synchronize()
    hop.status()
    return failed and ok


def _run(rank, world, port, fn, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
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
    out = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return out


def test_sharded_module_on_one_gpu_is_the_module():
    rel, shape, _ = _sharded(0, 1)
    assert rel == 0.0 and shape == (17, 1536)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("fn", [_sharded, _sharded_mask, _sharded_push, _sharded_nccl],
                         ids=["fused_peer_stores_tc", "fused_peer_stores_mask", "push_kernel", "nccl_all_gather"])
def test_sharded_module_over_two_gpus(fn):
    out = _spawn(fn, 2)
    for rank in range(2):
        rel, shape, _ = out[rank]
        assert shape == (17, 1536) and rel <= 1e-3
    assert out[0][2] == out[1][2]                       # the same y on every rank


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_barrier_gives_up_on_a_rank_that_never_comes():
    out = _spawn(_barrier_gives_up, 2)
    assert out[1] is True and out[0] is True


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_hop_over_nccl_sums_in_member_order():
    out = _spawn(_hop, 2)
    assert out[0] and out[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_plan_over_two_gpus_is_the_plan_on_one():
    out = _spawn(_plan_over_gpus, 2)
    assert out[0] and out[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_hop_wait_gives_up_on_a_part_that_never_comes():
    out = _spawn(_hop_gives_up, 2)
    assert out[0] and out[1]


def test_plan_graphed_on_one_gpu_is_the_eager_plan():
    """World 1: the whole plan on this GPU, eager and as a CUDA graph, the same bits."""
    from p2pllm_b200 import plan
    exact, reps = _plan_layers()
    s = plan.steps([[0, 1], [2, 3], [4, 5], [6, 7]], 8)
    runner = plan.PlanRunner(s, plan.place(s, 1), 0, exact.__getitem__, reps.__getitem__, None)
    x = torch.randn(17, 512, generator=torch.Generator(device="cuda").manual_seed(1), device="cuda").bfloat16()
    want = runner.pass_(0, x)
    graphed = plan.GraphedPass(runner, x)
    graphed.h_in.copy_(x)
    graphed.run()
    assert torch.equal(graphed.h_out, want)
