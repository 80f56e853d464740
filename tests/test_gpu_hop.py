"""The step hop's kernels (p2p_hop_send / p2p_hop_recv) on one GPU against the oracle, bit for bit: the sender's part
(a member's output, a member's difference, or the whole group combine) and the receiver's fp32 sum in member order.

On one GPU the ranks of the hop are stand-ins: every "rank" addresses the same inbox, and the sends run before the
receive in stream order, so no wait depends on a later launch. The give-up case waits for a pass that nothing sends,
with a 20 ms limit, and checks the error status."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from p2pllm_b200 import _lib, kernels
from p2pllm_b200._lib import P2PError

pytestmark = pytest.mark.gpu

DT = {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}
SUM, DIFF, COMBINE = 0, 1, 2


def _bits(t: torch.Tensor) -> np.ndarray:
    a = t.cpu()
    if a.dtype == torch.float32:
        return a.numpy()
    return a.view(torch.int16).numpy().view(np.uint16)


class _Hop:
    """n_ranks stand-in ranks over one inbox on this GPU."""

    def __init__(self, n_ranks: int, cap: int, dtype, ring: int = 2):
        self.n, self.cap, self.ring, self.dtype = n_ranks, cap, ring, dtype
        size = _lib.load().p2p_hop_inbox_bytes(n_ranks, cap, _lib.DTYPES[dtype], ring)
        assert size > 0
        self.inbox = torch.zeros(size, dtype=torch.uint8, device="cuda")
        self.ptrs = (ctypes.c_void_p * n_ranks)(*([self.inbox.data_ptr()] * n_ranks))

    def send(self, me, mode, parts, h=None, hc=None, dsts=(0,), p=0, counter=None):
        ref = parts[0]
        _lib.call("p2p_hop_send", mode, kernels._ptr_array(parts), len(parts), _lib.ptr(h), _lib.ptr(hc),
                  _lib.dtype_code(ref), ref.numel(), self.ptrs, self.n, me, (ctypes.c_int * len(dsts))(*dsts),
                  len(dsts), p, None if counter is None else counter.data_ptr(), self.ring, self.cap, 1_000_000,
                  _lib.stream_of(ref))

    def recv(self, me, srcs, like, p=0, wait_us=1_000_000, counter=None):
        out = torch.empty_like(like)
        _lib.call("p2p_hop_recv", self.ptrs, self.n, me, (ctypes.c_int * len(srcs))(*srcs), len(srcs), p,
                  None if counter is None else counter.data_ptr(), self.ring, self.cap, _lib.dtype_code(out),
                  out.numel(), _lib.ptr(out), wait_us, _lib.stream_of(out))
        return out


def _rand(shape, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(*shape, generator=g, device="cuda").to(dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_spread_step_parts_summed_in_member_order(dtype):
    """Three members on ranks 0, 1, 2 send l_0(h), dtype(l_1(h) - h), dtype(l_2(h~) - h~) to rank 3, which adds them:
    the oracle's sum of the oracle's parts, and the oracle's whole-group combine."""
    T, H = 17, 5120
    h, hc = _rand((T, H), dtype, 1), _rand((T, H), dtype, 2)
    ys = [_rand((T, H), dtype, 10 + k) for k in range(3)]
    hop = _Hop(4, T * H, dtype)
    hop.send(0, SUM, [ys[0]], dsts=[3])
    hop.send(1, DIFF, [ys[1]], h=h, dsts=[3])
    hop.send(2, DIFF, [ys[2]], h=hc, dsts=[3])
    got = hop.recv(3, [0, 1, 2], h)
    torch.cuda.synchronize()
    d = DT[dtype]
    parts = [_bits(ys[0]), oracle.member_part(_bits(ys[1]), _bits(h), d), oracle.member_part(_bits(ys[2]), _bits(hc), d)]
    assert np.array_equal(_bits(got), oracle.summed(parts, d))
    assert np.array_equal(_bits(got), oracle.combine([_bits(y) for y in ys], _bits(h), _bits(hc), d))


@pytest.mark.parametrize("members", [2, 3, 5])
def test_combine_sent_whole_to_two_ranks(members):
    """A rank whose run of steps ends at a boundary sends the group combine itself, to both ranks of the next step."""
    T, H, dtype = 9, 1024, torch.bfloat16
    h, hc = _rand((T, H), dtype, 3), _rand((T, H), dtype, 4)
    ys = [_rand((T, H), dtype, 20 + k) for k in range(members)]
    hop = _Hop(3, T * H, dtype)
    hop.send(0, COMBINE, ys, h=h, hc=hc, dsts=[1, 2])
    a = hop.recv(1, [0], h)
    b = hop.recv(2, [0], h)
    want = oracle.combine([_bits(y) for y in ys], _bits(h), _bits(hc), "bf16")
    assert np.array_equal(_bits(a), want) and np.array_equal(_bits(b), want)
    assert np.array_equal(_bits(kernels.combine(ys, h, hc)), want)


def test_ring_slots_over_many_passes_and_a_device_pass_counter():
    """Passes 0..6 through a ring of 2 slots, alternately numbered by the host and read from a device counter that
    p2p_hop_advance moves on; every pass arrives whole."""
    T, H, dtype = 17, 5120, torch.bfloat16
    hop = _Hop(2, T * H, dtype)
    counter = torch.zeros(1, dtype=torch.int32, device="cuda")
    for p in range(7):
        y = _rand((T, H), dtype, 100 + p)
        if p % 2:
            hop.send(0, SUM, [y], dsts=[1], counter=counter)
            got = hop.recv(1, [0], y, counter=counter)
        else:
            hop.send(0, SUM, [y], dsts=[1], p=p)
            got = hop.recv(1, [0], y, p=p)
        _lib.call("p2p_hop_advance", counter.data_ptr(), 1, _lib.stream_of(counter))
        assert torch.equal(got, y), p
    assert int(counter.item()) == 7
    _lib.call("p2p_hop_status", 1, _lib.stream_of(counter))


def test_a_wait_for_a_part_that_never_comes_gives_up():
    """Rank 1 waits for pass 0 from rank 0, which sends nothing: the wait ends after 20 ms, the status names rank 0,
    and a hop sent afterwards goes through."""
    T, H, dtype = 4, 256, torch.bfloat16
    hop = _Hop(2, T * H, dtype)
    like = _rand((T, H), dtype, 5)
    hop.recv(1, [0], like, p=0, wait_us=20_000)
    torch.cuda.synchronize()
    with pytest.raises(P2PError, match="rank 0"):
        _lib.call("p2p_hop_status", 1, _lib.stream_of(like))
    _lib.call("p2p_hop_status", 1, _lib.stream_of(like))      # reset: clear now
    hop.send(0, SUM, [like], dsts=[1], p=0)
    assert torch.equal(hop.recv(1, [0], like, p=0), like)


def test_bad_arguments_are_refused_before_any_launch():
    T, H, dtype = 4, 256, torch.bfloat16
    hop = _Hop(2, T * H, dtype)
    x = _rand((T, H), dtype, 6)
    big = _rand((T + 1, H), dtype, 7)
    with pytest.raises(P2PError, match="slots hold"):
        hop.send(0, SUM, [big], dsts=[1])
    with pytest.raises(P2PError, match="listed twice"):
        hop.send(0, SUM, [x], dsts=[1, 1])
    with pytest.raises(P2PError, match="rank 2 of 2"):
        hop.recv(1, [2], x)
    with pytest.raises(P2PError, match="mode"):
        hop.send(0, 7, [x], dsts=[1])
    with pytest.raises(P2PError, match="difference"):
        hop.send(0, DIFF, [x], dsts=[1])
