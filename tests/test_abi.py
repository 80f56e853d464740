"""The C ABI without a GPU: the library loads, exports every function include/p2p_b200.h declares, and rejects bad
arguments with a status and a message before touching the device."""
import ctypes
import os
import re

import pytest

from p2pllm_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "p2p_b200.h")


def declared() -> set:
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    return set(re.findall(r"\b(p2p_[a-z0-9_]+)\s*\(", text))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(_lib.LIB_PATH):
        from p2pllm_b200 import build
        build.build()
    return _lib.load()


def test_every_declared_symbol_is_exported(lib):
    names = declared()
    assert len(names) >= 15
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_every_declared_symbol_has_a_binding():
    assert declared() <= set(_lib.SIGNATURES)


def test_abi_version(lib):
    assert lib.p2p_abi_version() == 1


def test_bad_arguments_give_a_status_and_a_message(lib):
    st = lib.p2p_spmm_rows(None, 0, 4, 8, 8, None, 0, 2, None, 4, None)
    assert st == -1 and b"row blocks" in lib.p2p_last_error()
    st = lib.p2p_wanda_select(None, 0, 4, 8, 8, None, 0, 9, None, None, 2, 9, None, 0, None, 0, None, 0, None)
    assert st == -1 and b"k=9" in lib.p2p_last_error()
    st = lib.p2p_combine(None, 1, None, None, None, 0, 4, None)
    assert st == -1 and b"at least 2" in lib.p2p_last_error()
    st = lib.p2p_wanda_select(None, 0, 4, 60000, 60000, None, 0, 9, None, None, 4, 9, None, 0, None, 0, None, 0, None)
    assert st == -2 and b"at most" in lib.p2p_last_error()


def test_empty_work_is_a_no_op(lib):
    assert lib.p2p_sumsq_cols(None, 0, 0, 16, 16, None, None, 0, None) == 0
    assert lib.p2p_member_part(None, None, None, 0, 0, None) == 0


def test_workspace_query_is_host_only(lib):
    assert lib.p2p_sumsq_workspace(0, 10, 0) == 0
    assert lib.p2p_sumsq_workspace(262144, 4096, 0) > 0
    assert lib.p2p_sumsq_workspace(100, 4096, 9) == 0


def test_persistent_runs_workspace_is_sized_on_the_host(lib):
    """The tensor-core GEMM's workspace for a module of more row tiles than SMs at up to 128 tokens (one CTA an SM,
    contiguous runs of units): the ticket region, then two fp32 partial tiles [tokens][128] a run. Without a GPU the
    query assumes the B200's 148 SMs. A run takes at most 256 units, so very wide modules get more runs than SMs."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("with a GPU the query uses that device's SM count")
    tickets = 16384 * 4
    runs = lambda g, t: tickets + g * 2 * t * 128 * 4
    assert lib.p2p_spmm_tc_workspace(149 * 128, 1024, 17) == runs(148, 17)
    assert lib.p2p_spmm_tc_workspace(19000, 1024, 100) == runs(148, 100)
    assert lib.p2p_spmm_tc_workspace(19000, 1024, 128) == runs(148, 128)
    assert lib.p2p_spmm_tc_workspace(149 * 128, 65536, 17) == runs(-(-149 * 1024 // 256), 17)
    assert lib.p2p_spmm_tc_workspace(148 * 128, 64, 17) == 0           # row tiles <= SMs: one CTA a row tile
    assert lib.p2p_spmm_tc_workspace(19000, 1024, 0) == 0


def test_cpu_tensors_are_refused():
    import torch
    from p2pllm_b200 import P2PError, kernels
    with pytest.raises(P2PError, match="CUDA"):
        kernels.combine([torch.zeros(4), torch.zeros(4)], torch.zeros(4), torch.zeros(4))


def test_grouped_launch_refuses_more_column_tiles_than_a_cta_stages(lib):
    """An item of a grouped launch takes whole rows in one CTA, which stages at most 256 column tiles' offsets and
    headers in shared memory: 16,384 + 64 columns are refused before any launch (no device memory is touched; the
    pointers are placeholders with the alignment the earlier checks ask for)."""
    fake = ctypes.c_void_p(256)
    cols = 16384 + 64
    st = lib.p2p_spmm_tc_grouped(fake, 0, 16, cols, cols, fake, fake, 1, 128, 1, 16, fake, 1, 16, fake, 128, None)
    assert st == -1 and b"at most 16384" in lib.p2p_last_error()


def test_withhold_test_entry_checks_its_limits(lib):
    fake = ctypes.c_void_p(256)
    st = lib.p2p_spmm_tc_withhold(fake, 0, 16, 64, 64, fake, fake, 128, 16, fake, 128, None, 0, 0, 10, None)
    assert st == -1 and b"1 ms to 2 s" in lib.p2p_last_error()
    st = lib.p2p_spmm_tc_withhold(fake, 0, 600, 64, 64, fake, fake, 128, 16, fake, 128, None, 0, 0, 5000, None)
    assert st == -1 and b"one launch" in lib.p2p_last_error()


def test_torch_ops_load_and_propagate_shapes_on_meta_tensors(lib):
    """The entry points as torch custom operators (p2p_b200::*, over the same C ABI): they register with the dispatcher
    and their Meta kernels give the output shapes without touching a device."""
    import torch
    from p2pllm_b200 import build
    build.build_ops()
    ops = _lib.ops()
    meta = lambda *shape, dtype=torch.bfloat16: torch.empty(*shape, device="meta", dtype=dtype)
    y = ops.spmm_tc(meta(17, 4096), meta(1000, dtype=torch.int32), meta(513, dtype=torch.int64), 6144, 4096, 600)
    assert y.shape == (17, 6144) and y.device.type == "meta" and y.dtype == torch.bfloat16
    y = ops.spmm_mask(meta(272, 4096), meta(1000, dtype=torch.uint8), meta(513, dtype=torch.int64), 1024, 4096)
    assert y.shape == (272, 1024)
    h = meta(8, 96)
    assert ops.combine([h, h, h], h, h).shape == (8, 96) and ops.sum_parts([h, h]).shape == (8, 96)
    names = {"spmm_tc", "spmm_tc_into", "spmm_mask", "spmm_mask_into", "sumsq_cols", "combine", "sum_parts",
             "zero_workspaces"}
    assert all(hasattr(ops, n) for n in names)
    ops.zero_workspaces(0)                              # no workspace cached on this host: nothing to zero


def test_a_give_up_zeroes_the_gemm_workspaces_of_its_device_again():
    """After a pipeline wait gave up, a launch may have left ticket counters of its workspace taken; the status check
    zeroes the cached workspaces of that purpose on that device (every stream), and no others."""
    import torch
    from p2pllm_b200 import kernels
    keys = [("cpu", None, "spmm_tc", 1), ("cpu", None, "spmm_tc", 2), ("cpu", None, "spmm_mask", 1),
            ("cpu", 3, "spmm_tc", 1)]
    saved = dict(kernels._workspaces)
    try:
        for k in keys:
            kernels._workspaces[k] = torch.full((64,), 7, dtype=torch.uint8)
        assert kernels._rezero_workspaces(torch.device("cpu"), "spmm_tc") == 2
        assert [int(kernels._workspaces[k].sum()) for k in keys] == [0, 0, 7 * 64, 7 * 64]
    finally:
        kernels._workspaces.clear()
        kernels._workspaces.update(saved)


def _ptrs(*vals):
    return (ctypes.c_void_p * len(vals))(*vals)


def _ints(*vals):
    return (ctypes.c_int * len(vals))(*vals)


def test_hop_inbox_size_is_host_only(lib):
    """Counters (256 bytes) and n_ranks x ring slots, each part's 32-bit words stored with a 32-bit flag (twice the
    bytes), rounded to 256; arguments out of range give 0."""
    assert lib.p2p_hop_inbox_bytes(2, 17 * 5120, 0, 2) == 256 + 2 * 2 * (17 * 5120 * 2 * 2)
    assert lib.p2p_hop_inbox_bytes(8, 100, 2, 1) == 256 + 8 * ((100 * 4 * 2 + 255) // 256 * 256)
    assert lib.p2p_hop_inbox_bytes(9, 100, 0, 2) == 0
    assert lib.p2p_hop_inbox_bytes(2, 100, 0, 0) == 0


@pytest.mark.parametrize("call,needle", [
    (lambda lib: lib.p2p_hop_send(0, _ptrs(65536), 1, None, None, 0, 64, _ptrs(4096, 8192), 2, 0, _ints(1, 1), 2, 0,
                                  None, 2, 64, 1000000, None), b"listed twice"),
    (lambda lib: lib.p2p_hop_send(0, _ptrs(65536), 1, None, None, 0, 65, _ptrs(4096, 8192), 2, 0, _ints(1), 1, 0,
                                  None, 2, 128, 1000000, None), b"multiple of 16 bytes"),
    (lambda lib: lib.p2p_hop_send(0, _ptrs(65536), 1, None, None, 0, 64, _ptrs(4100, 8192), 2, 0, _ints(1), 1, 0,
                                  None, 2, 64, 1000000, None), b"256-byte aligned"),
    (lambda lib: lib.p2p_hop_send(5, _ptrs(65536), 1, None, None, 0, 64, _ptrs(4096, 8192), 2, 0, _ints(1), 1, 0,
                                  None, 2, 64, 1000000, None), b"mode"),
    (lambda lib: lib.p2p_hop_recv(_ptrs(4096, 8192), 2, 1, _ints(2), 1, 0, None, 2, 64, 0, 64, _ptrs(65536)[0], 1000000,
                                  None), b"rank 2 of 2"),
    (lambda lib: lib.p2p_hop_recv(_ptrs(4096, 8192), 2, 1, _ints(0), 1, 0, None, 2, 64, 0, 128, 65536, 1000000, None),
     b"slots hold"),
    (lambda lib: lib.p2p_hop_recv(_ptrs(4096, 8192), 2, 1, _ints(0), 1, 0, None, 2, 64, 0, 64, 65536, 10, None),
     b"time limit"),
    (lambda lib: lib.p2p_peer_push(65536, _ptrs(4096), 1, 17, 3, 8, 64, 0, None), b"16-byte aligned"),
    (lambda lib: lib.p2p_peer_push(65536, _ptrs(4096), 8, 17, 0, 8, 64, 0, None), b"peers"),
    (lambda lib: lib.p2p_spmm_tc_gated(65536, 0, 17, 64, 64, 65536, 65536, 200, 64, 65536, 100, None, 0, None),
     b"not whole row tiles"),
    (lambda lib: lib.p2p_spmm_tc_peers(65536, 0, 17, 64, 64, 65536, 65536, 128, 64, _ptrs(4096), 1, 64, 128, None, 0,
                                       None), b"do not fit"),
], ids=["hop-dup-dst", "hop-size", "hop-inbox-align", "hop-mode", "hop-src-rank", "hop-capacity", "hop-limit",
        "push-align", "push-peers", "gated-rows", "peers-columns"])
def test_multi_gpu_entries_refuse_bad_arguments(lib, call, needle):
    assert call(lib) != 0
    assert needle in lib.p2p_last_error(), lib.p2p_last_error()
