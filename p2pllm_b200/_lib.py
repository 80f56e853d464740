"""ctypes binding of libp2p_b200.so (include/p2p_b200.h). There is no fallback: if the library is missing or the
tensors are not on a CUDA device, the call raises."""
from __future__ import annotations

import ctypes
import os
import threading

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libp2p_b200.so")

BF16, F16, F32 = 0, 1, 2
DTYPES = {torch.bfloat16: BF16, torch.float16: F16, torch.float32: F32}
IDX_BYTES = {torch.int16: 2, torch.int32: 4}


class P2PError(RuntimeError):
    """A p2p_b200 entry point returned an error status."""


class RowBlock(ctypes.Structure):
    _fields_ = [("vals", ctypes.c_void_p), ("idx", ctypes.c_void_p), ("row0", ctypes.c_int64),
                ("rows", ctypes.c_int64), ("k", ctypes.c_int64), ("ld", ctypes.c_int64)]


_i64, _int, _vp, _sz = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t
SIGNATURES = {
    "p2p_last_error": ([], ctypes.c_char_p),
    "p2p_abi_version": ([], _int),
    "p2p_sumsq_workspace": ([_i64, _i64, _int], _sz),
    "p2p_sumsq_cols": ([_vp, _int, _i64, _i64, _i64, _vp, _vp, _sz, _vp], _int),
    "p2p_sumsq_cols_noalloc": ([_vp, _int, _i64, _i64, _i64, _vp, _vp], _int),
    "p2p_expert_sumsq": ([_vp, _int, _i64, _i64, _i64, _vp, _vp, _i64, _i64, _vp, _vp], _int),
    "p2p_channel_norms": ([_vp, _i64, _i64, _int, _vp, _vp], _int),
    "p2p_wanda_select": ([_vp, _int, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _int, _i64, _vp, _i64, _vp, _i64,
                          _vp, _i64, _vp], _int),
    "p2p_words_to_idx": ([_vp, _i64, _i64, _i64, _i64, _vp, _int, _i64, _vp], _int),
    "p2p_pack_mask": ([_vp, _int, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _vp, _i64, _vp], _int),
    "p2p_unpack": ([_vp, _int, _i64, _i64, _i64, _vp, _i64, _vp, _int, _i64, _i64, _vp, _i64, _vp], _int),
    "p2p_check_idx": ([_vp, _int, _i64, _i64, _i64, _i64, _vp], _int),
    "p2p_spmm_rows": ([_vp, _int, _i64, _i64, _i64, ctypes.POINTER(RowBlock), _int, _int, _vp, _i64, _vp], _int),
    "p2p_tiles_workspace": ([ctypes.POINTER(RowBlock), _int, _i64], _sz),
    "p2p_tiles_plan": ([ctypes.POINTER(RowBlock), _int, _int, _i64, _vp, ctypes.POINTER(_i64), _vp, _sz, _vp], _int),
    "p2p_tiles_fill": ([ctypes.POINTER(RowBlock), _int, _int, _i64, _int, _vp, _vp, _i64, _vp, _sz, _vp], _int),
    "p2p_mask_workspace": ([ctypes.POINTER(RowBlock), _int, _i64], _sz),
    "p2p_mask_plan": ([ctypes.POINTER(RowBlock), _int, _int, _i64, _vp, ctypes.POINTER(_i64), _vp, _sz, _vp], _int),
    "p2p_mask_fill": ([ctypes.POINTER(RowBlock), _int, _int, _i64, _int, _vp, _vp, _i64, _vp], _int),
    "p2p_spmm_mask_workspace": ([_i64, _i64, _i64], _sz),
    "p2p_spmm_mask": ([_vp, _int, _i64, _i64, _i64, _vp, _vp, _i64, _vp, _i64, _vp, _sz, _vp], _int),
    "p2p_spmm_mask_status": ([_int, _vp], _int),
    "p2p_spmm_mask_peers": ([_vp, _int, _i64, _i64, _i64, _vp, _vp, _i64, ctypes.POINTER(_vp), _int, _i64, _i64, _vp,
                             _sz, _vp], _int),
    "p2p_peer_barrier": ([ctypes.POINTER(_vp), _int, _int, ctypes.c_uint32, _i64, _vp], _int),
    "p2p_peer_status": ([_int, _vp], _int),
    "p2p_peer_push": ([_vp, ctypes.POINTER(_vp), _int, _i64, _i64, _i64, _i64, _int, _vp], _int),
    "p2p_hop_inbox_bytes": ([_int, _i64, _int, _int], _sz),
    "p2p_hop_send": ([_int, ctypes.POINTER(_vp), _int, _vp, _vp, _int, _i64, ctypes.POINTER(_vp), _int, _int,
                      ctypes.POINTER(_int), _int, ctypes.c_uint32, _vp, _int, _i64, _i64, _vp], _int),
    "p2p_hop_recv": ([ctypes.POINTER(_vp), _int, _int, ctypes.POINTER(_int), _int, ctypes.c_uint32, _vp, _int, _i64,
                      _int, _i64, _vp, _i64, _vp], _int),
    "p2p_hop_advance": ([_vp, _int, _vp], _int),
    "p2p_hop_status": ([_int, _vp], _int),
    "p2p_spmm_tc_workspace": ([_i64, _i64, _i64], _sz),
    "p2p_spmm_tc": ([_vp, _int, _i64, _i64, _i64, _vp, _vp, _i64, _i64, _vp, _i64, _vp, _sz, _vp], _int),
    "p2p_spmm_tc_grouped": ([_vp, _int, _i64, _i64, _i64, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64,
                             _vp], _int),
    "p2p_spmm_tc_status": ([_int, _vp], _int),
    "p2p_spmm_tc_peers": ([_vp, _int, _i64, _i64, _i64, _vp, _vp, _i64, _i64, ctypes.POINTER(_vp), _int, _i64, _i64, _vp,
                           _sz, _vp], _int),
    "p2p_spmm_tc_gated": ([_vp, _int, _i64, _i64, _i64, _vp, _vp, _i64, _i64, _vp, _i64, _vp, _sz, _vp], _int),
    "p2p_spmm_tc_grouped_gated": ([_vp, _int, _i64, _i64, _i64, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _i64, _i64,
                                   _vp, _i64, _vp], _int),
    "p2p_spmm_tc_grouped_gated_sums": ([_vp, _int, _i64, _i64, _i64, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _i64,
                                        _i64, _vp, _i64, _vp], _int),
    "p2p_spmm_tc_withhold": ([_vp, _int, _i64, _i64, _i64, _vp, _vp, _i64, _i64, _vp, _i64, _vp, _sz, _i64, _i64,
                              _vp], _int),
    "p2p_moe_route": ([_vp, _i64, _int, _vp, _vp, _vp, _vp, _i64, _vp, _vp], _int),
    "p2p_moe_combine": ([_vp, _int, _i64, _vp, _vp, _i64, _int, _i64, _vp, _i64, _vp], _int),
    "p2p_combine": ([ctypes.POINTER(_vp), _int, _vp, _vp, _vp, _int, _i64, _vp], _int),
    "p2p_sum_parts": ([ctypes.POINTER(_vp), _int, _vp, _int, _i64, _vp], _int),
    "p2p_member_part": ([_vp, _vp, _vp, _int, _i64, _vp], _int),
}

OPS_PATH = os.path.join(HERE, "libp2p_torch_ops.so")

_lib = None
_ops = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """The loaded library, with every signature of the header bound. Raises if it was never built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise P2PError(f"{LIB_PATH} is missing: build it with `python -m p2pllm_b200.build` "
                                   "(the replica path has no CPU fallback)")
                lib = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_GLOBAL)    # the torch ops resolve its symbols
                for name, (args, res) in SIGNATURES.items():
                    fn = getattr(lib, name)
                    fn.argtypes, fn.restype = args, res
                _lib = lib
    return _lib


def ops():
    """torch.ops.p2p_b200: the entry points as torch custom operators (libp2p_torch_ops.so over the C ABI). Raises if
    either library was never built."""
    global _ops
    if _ops is None:
        load()
        with _lock:
            if _ops is None:
                if not os.path.exists(OPS_PATH):
                    raise P2PError(f"{OPS_PATH} is missing: build it with `python -m p2pllm_b200.build`")
                torch.ops.load_library(OPS_PATH)
                _ops = torch.ops.p2p_b200
    return _ops


def call(name: str, *args) -> None:
    """Calls entry point `name`; raises P2PError with the library's message on a non-zero status."""
    lib = load()
    status = getattr(lib, name)(*args)
    if status != 0:
        raise P2PError(f"{name}: {lib.p2p_last_error().decode()} (status {status})")


def stream_of(t: torch.Tensor) -> int:
    """The current CUDA stream of t's device, as the void* the C ABI takes."""
    return torch.cuda.current_stream(t.device).cuda_stream


def dtype_code(t: torch.Tensor) -> int:
    try:
        return DTYPES[t.dtype]
    except KeyError:
        raise P2PError(f"dtype {t.dtype}: bfloat16, float16 or float32") from None


def require_cuda(*ts) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise P2PError("the replica path runs on CUDA tensors only (no CPU fallback)")


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def idx_dtype(cols: int) -> torch.dtype:
    """Column indices are int16 while they fit (cols <= 32767), else int32."""
    return torch.int16 if cols <= 32767 else torch.int32
