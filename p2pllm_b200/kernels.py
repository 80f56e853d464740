"""Tensor-level wrappers of the C ABI: shape and device checks, outputs allocated with torch, launches on the current
stream of the inputs' device. Each function names the reference interface it serves."""
from __future__ import annotations

import ctypes
import os

import torch

from . import _lib
from ._lib import P2PError, call, dtype_code, ptr, require_cuda, stream_of

_workspaces: dict = {}
# P2P_CHECK_WAITS=1: after every tensor-core GEMM launch, read back whether a pipeline wait gave up (and raise if one
# did). It synchronizes the stream each time, so it is for debugging, not for serving.
CHECK_WAITS = os.environ.get("P2P_CHECK_WAITS", "0") not in ("", "0")


def _workspace(device: torch.device, nbytes: int, purpose: str = "sumsq") -> torch.Tensor:
    """A zeroed scratch buffer of at least nbytes per device, purpose and stream (the kernels leave it zeroed again;
    launches on one stream run in order, so they can share it, while launches on two streams may overlap and must
    not)."""
    key = (device.type, device.index, purpose, torch.cuda.current_stream(device).cuda_stream)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws


def _rezero_workspaces(dev: torch.device, purpose: str) -> int:
    """Zeroes every cached workspace of `purpose` on `dev` (all streams), and the torch operators' own workspaces
    there; returns how many of this module's it zeroed."""
    n = 0
    for (kind, index, what, _), ws in _workspaces.items():
        if kind == dev.type and index == dev.index and what == purpose:
            ws.zero_()
            n += 1
    if dev.type == "cuda" and _lib._ops is not None:
        _lib._ops.zero_workspaces(dev.index)
    return n


def _rows2d(x: torch.Tensor) -> torch.Tensor:
    x = x.reshape(-1, x.shape[-1])
    if x.stride(-1) != 1:
        x = x.contiguous()
    return x


def sumsq_cols(x: torch.Tensor, sums: torch.Tensor) -> torch.Tensor:
    """sums += x.float().pow(2).sum(0).double() over x [..., cols] (p2p/wanda.py:37-40). sums: float64 [cols]."""
    require_cuda(x, sums)
    if sums.dtype != torch.float64 or sums.numel() != x.shape[-1] or not sums.is_contiguous():
        raise P2PError("sums must be a contiguous float64 vector of x's columns")
    _lib.ops().sumsq_cols(x, sums)
    return sums


def expert_sumsq(x: torch.Tensor, ids: torch.Tensor, into: torch.Tensor) -> torch.Tensor:
    """into[e] += fp32 sum of x[t]^2 over the tokens routed to e, each once (the `into` half of p2p/wanda.py:10-20).
    ids: [tokens, topk] expert ids (negative = none)."""
    require_cuda(x, ids, into)
    x = _rows2d(x)
    n_exp = into.shape[0]
    if into.dtype != torch.float64 or into.shape[-1] != x.shape[1] or not into.is_contiguous():
        raise P2PError("into must be contiguous float64 [experts, cols]")
    topk = ids.shape[-1]
    flat = ids.reshape(-1).to(torch.int64)
    flat = torch.where((flat >= 0) & (flat < n_exp), flat, torch.full_like(flat, n_exp))
    # (token, slot) pairs grouped by expert, tokens ascending inside an expert: a stable sort of the expert ids.
    order = torch.sort(flat, stable=True).indices
    counts = torch.bincount(flat, minlength=n_exp + 1)[:n_exp]
    seg = torch.zeros(n_exp + 1, dtype=torch.int64, device=x.device)
    seg[1:] = counts.cumsum(0)
    call("p2p_expert_sumsq", ptr(x), dtype_code(x), x.shape[0], x.shape[1], x.stride(0), ptr(order), ptr(seg), topk,
         n_exp, ptr(into), stream_of(x))
    return into


def channel_norms(sums: torch.Tensor) -> torch.Tensor:
    """sums.sqrt().float(); for [experts, cols] sums a row of zeros gives ones, shaped [experts, 1, cols]
    (p2p/wanda.py:63-73)."""
    require_cuda(sums)
    sums = sums.to(torch.float64).contiguous()
    experts = sums.dim() == 2
    groups = sums.shape[0] if experts else 1
    norms = torch.empty(sums.shape, dtype=torch.float32, device=sums.device)
    call("p2p_channel_norms", ptr(sums), groups, sums.shape[-1], int(experts), ptr(norms), stream_of(sums))
    return norms[:, None, :] if experts else norms


def wanda_select(w: torch.Tensor, norms: torch.Tensor, k: int, *, values: bool = True, idx: bool = True,
                 words: bool = False, mask: bool = False, pruned: bool = False, idx_dtype=None) -> dict:
    """Per-row top-k of |w| * norms, ties to the lower column (p2p/wanda.py:76-87 + p2p/compact.py:36-45).
    w: [rows, cols] or [experts, rows, cols] with norms [experts, 1, cols]. Returns the requested outputs among
    values [.., k], idx [.., k] (int16 while cols <= 32767), words [.., ceil(cols/32)] int32, mask (bool) and pruned."""
    require_cuda(w, norms)
    lead, cols = w.shape[:-1], w.shape[-1]
    w2 = w.reshape(-1, cols)
    if w2.stride(-1) != 1:
        w2 = w2.contiguous()
    rows = w2.shape[0]
    norms = norms.to(torch.float32).contiguous()
    if norms.numel() == cols:
        group_rows = 0
    elif w.dim() == 3 and norms.numel() == w.shape[0] * cols:
        group_rows = w.shape[1]
    else:
        raise P2PError(f"norms of {tuple(norms.shape)} do not fit w of {tuple(w.shape)}")
    dev = w.device
    idt = idx_dtype or _lib.idx_dtype(cols)
    out = {}
    v = torch.empty(rows, k, dtype=w.dtype, device=dev) if values else None
    ix = torch.empty(rows, k, dtype=idt, device=dev) if idx else None
    wd = torch.empty(rows, (cols + 31) // 32, dtype=torch.int32, device=dev) if words else None
    m = torch.empty(rows, cols, dtype=torch.bool, device=dev) if mask else None
    p = torch.empty(rows, cols, dtype=w.dtype, device=dev) if pruned else None
    call("p2p_wanda_select", ptr(w2), dtype_code(w2), rows, cols, w2.stride(0), ptr(norms), group_rows, k,
         ptr(v), ptr(ix), _lib.IDX_BYTES[idt], k, ptr(wd), 0 if wd is None else wd.shape[1],
         ptr(m), cols, ptr(p), cols, stream_of(w2))
    for name, t in (("values", v), ("idx", ix), ("words", wd), ("mask", m), ("pruned", p)):
        if t is not None:
            out[name] = t.view(*lead, *t.shape[1:])
    return out


def words_to_idx(words: torch.Tensor, cols: int, k: int, idx_dtype=None) -> torch.Tensor:
    """Column indices [rows, k] of the reference's mask words (p2p/compact.py:36-45); raises if a row keeps another
    number of columns."""
    require_cuda(words)
    words = words.reshape(-1, words.shape[-1]).contiguous()
    idt = idx_dtype or _lib.idx_dtype(cols)
    idx = torch.empty(words.shape[0], k, dtype=idt, device=words.device)
    call("p2p_words_to_idx", ptr(words), words.shape[0], cols, words.stride(0), k, ptr(idx), _lib.IDX_BYTES[idt], k,
         stream_of(words))
    return idx


def pack_mask(w: torch.Tensor, mask: torch.Tensor):
    """(values [rows, k], words) from w and a bool mask that keeps the same k in every row (p2p/compact.py:36-45)."""
    require_cuda(w, mask)
    rows, cols = w.shape
    w = w.contiguous()
    m = mask.contiguous().view(torch.uint8)
    k = int(mask[0].sum()) if rows else 0
    values = torch.empty(rows, k, dtype=w.dtype, device=w.device)
    words = torch.empty(rows, (cols + 31) // 32, dtype=torch.int32, device=w.device)
    try:
        call("p2p_pack_mask", ptr(w), dtype_code(w), rows, cols, w.stride(0), ptr(m), m.stride(0), k, ptr(values),
             k, ptr(words), words.shape[1], stream_of(w))
    except P2PError as e:
        raise AssertionError("every row must keep the same number of weights") from e
    return values, words


def unpack(values: torch.Tensor, cols: int, words: torch.Tensor | None = None,
           idx: torch.Tensor | None = None) -> torch.Tensor:
    """Dense [rows, cols] from values [rows, k] and mask words or column indices (p2p/compact.py:48-85)."""
    require_cuda(values, words, idx)
    rows, k = values.shape
    values = values.contiguous()
    dense = torch.empty(rows, cols, dtype=values.dtype, device=values.device)
    if words is not None:
        words = words.contiguous()
        call("p2p_unpack", ptr(values), dtype_code(values), rows, k, values.stride(0), ptr(words), words.stride(0),
             None, 0, 0, cols, ptr(dense), cols, stream_of(values))
    else:
        idx = idx.contiguous()
        call("p2p_unpack", ptr(values), dtype_code(values), rows, k, values.stride(0), None, 0, ptr(idx),
             _lib.IDX_BYTES[idx.dtype], idx.stride(0), cols, ptr(dense), cols, stream_of(values))
    return dense


def check_idx(idx: torch.Tensor, cols: int) -> None:
    """Raises unless every column index lies in [0, cols)."""
    require_cuda(idx)
    idx = idx.reshape(-1, idx.shape[-1]).contiguous()
    call("p2p_check_idx", ptr(idx), _lib.IDX_BYTES[idx.dtype], idx.shape[0], idx.shape[1], idx.stride(0), cols,
         stream_of(idx))


def _out(out: torch.Tensor | None, shape: tuple, like: torch.Tensor, whole: bool = False) -> torch.Tensor:
    """A caller's output tensor, checked (shape, dtype, device, unit column stride; `whole`: contiguous), or a new one."""
    if out is None:
        return torch.empty(shape, dtype=like.dtype, device=like.device)
    require_cuda(out)
    if tuple(out.shape) != tuple(shape) or out.dtype != like.dtype or out.device != like.device:
        raise P2PError(f"out of {tuple(out.shape)} {out.dtype} on {out.device}, wanted {tuple(shape)} {like.dtype} "
                       f"on {like.device}")
    if (whole and not out.is_contiguous()) or (out.dim() and out.stride(-1) != 1 and out.numel()):
        raise P2PError(f"out of strides {out.stride()} is not laid out as the kernel writes it")
    return out


def spmm_rows(x: torch.Tensor, blocks: list, cols: int, out_rows: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """y [tokens, out_rows] = x [tokens, cols] times row blocks (CUDA cores). blocks: (row0, values, idx | None) with
    values [rows, k] (k == cols when idx is None: a dense block). Replaces p2p/compact.cu:265-278 for row layouts."""
    require_cuda(x)
    if x.dim() != 2 or x.shape[1] != cols:
        raise P2PError(f"x of {tuple(x.shape)} does not have {cols} columns")
    if x.stride(1) != 1:
        x = x.contiguous()
    out = _out(out, (x.shape[0], out_rows), x)
    table = (_lib.RowBlock * len(blocks))()
    idx_bytes = 2
    for i, (row0, v, ix) in enumerate(blocks):
        if v.dtype != x.dtype:
            raise P2PError(f"values {v.dtype} differ from x {x.dtype}")
        if ix is not None:
            idx_bytes = _lib.IDX_BYTES[ix.dtype]
        table[i] = _lib.RowBlock(v.data_ptr(), None if ix is None else ix.data_ptr(), row0, v.shape[0], v.shape[1],
                                 v.stride(0))
    kinds = {_lib.IDX_BYTES[ix.dtype] for _, _, ix in blocks if ix is not None}
    if len(kinds) > 1:
        raise P2PError("all row blocks of a module use one index type")
    call("p2p_spmm_rows", ptr(x), dtype_code(x), x.shape[0], cols, x.stride(0), table, len(blocks), idx_bytes,
         ptr(out), out.stride(0), stream_of(x))
    return out


def _row_table(blocks: list):
    table = (_lib.RowBlock * len(blocks))()
    idx_bytes = 2
    for i, (row0, v, ix) in enumerate(blocks):
        if ix is not None:
            idx_bytes = _lib.IDX_BYTES[ix.dtype]
        table[i] = _lib.RowBlock(v.data_ptr(), None if ix is None else ix.data_ptr(), row0, v.shape[0], v.shape[1],
                                 v.stride(0))
    return table, idx_bytes


def tiles_build(blocks: list, cols: int) -> tuple:
    """The tensor-core layout (words uint32, seg int64, largest segment in words) of a module's row blocks
    [(row0, values, idx | None)], bf16 or f16 values, ascending column indices. Load time; syncs."""
    dev = blocks[0][1].device
    table, idx_bytes = _row_table(blocks)
    lib = _lib.load()
    need = lib.p2p_tiles_workspace(table, len(blocks), cols)
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=dev)
    rows = max(r0 + v.shape[0] for r0, v, _ in blocks)
    n_seg = -(-rows // 128) * -(-cols // 64)
    seg = torch.empty(n_seg + 1, dtype=torch.int64, device=dev)
    total = ctypes.c_int64(0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    call("p2p_tiles_plan", table, len(blocks), idx_bytes, cols, ptr(seg), ctypes.byref(total), ptr(ws), ws.numel(),
         stream)
    words = torch.empty(max(total.value, 4), dtype=torch.int32, device=dev)
    call("p2p_tiles_fill", table, len(blocks), idx_bytes, cols, dtype_code(blocks[0][1]), ptr(seg), ptr(words),
         total.value, ptr(ws), ws.numel(), stream)
    seg_cap = int((seg[1:] - seg[:-1]).max().item()) if n_seg else 0
    return words, seg, seg_cap


def mask_build(blocks: list, cols: int) -> tuple:
    """The bitmask layout (data uint8, seg int64 byte offsets) of a module's row blocks [(row0, values, idx | None)],
    bf16 or f16 values, ascending column indices. Load time; syncs."""
    dev = blocks[0][1].device
    table, idx_bytes = _row_table(blocks)
    lib = _lib.load()
    need = lib.p2p_mask_workspace(table, len(blocks), cols)
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=dev)
    rows = max(r0 + v.shape[0] for r0, v, _ in blocks)
    n_seg = -(-rows // 128) * -(-cols // 64)
    seg = torch.empty(n_seg + 1, dtype=torch.int64, device=dev)
    total = ctypes.c_int64(0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    call("p2p_mask_plan", table, len(blocks), idx_bytes, cols, ptr(seg), ctypes.byref(total), ptr(ws), ws.numel(),
         stream)
    data = torch.empty(max(total.value, 16), dtype=torch.uint8, device=dev)
    call("p2p_mask_fill", table, len(blocks), idx_bytes, cols, dtype_code(blocks[0][1]), ptr(seg), ptr(data),
         total.value, stream)
    return data, seg


def spmm_mask(x: torch.Tensor, data: torch.Tensor, seg: torch.Tensor, rows: int, cols: int,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """y [tokens, rows] = x [tokens, cols] times a module in the bitmask layout (tcgen05, weights in TMEM), through the
    torch operator p2p_b200::spmm_mask."""
    require_cuda(x)
    if x.dim() != 2 or x.shape[1] != cols:
        raise P2PError(f"x of {tuple(x.shape)} does not have {cols} columns")
    if out is None:
        out = _lib.ops().spmm_mask(x, data, seg, rows, cols)
    else:
        _lib.ops().spmm_mask_into(x, data, seg, rows, cols, _out(out, (x.shape[0], rows), x))
    if CHECK_WAITS:
        spmm_mask_status(x.device)
    return out


def spmm_mask_peers(x: torch.Tensor, data: torch.Tensor, seg: torch.Tensor, rows: int, cols: int, ys, n_ys: int,
                    y_col0: int, ldy: int) -> None:
    """This rank's rows of y = x times a module in the bitmask layout, stored at columns y_col0.. of each of the n_ys
    y buffers (a ctypes array of device pointers: every rank's y, peers' through peer memory)."""
    require_cuda(x)
    if x.dim() != 2 or x.shape[1] != cols:
        raise P2PError(f"x of {tuple(x.shape)} does not have {cols} columns")
    if x.stride(1) != 1 or x.stride(0) % 8 or x.data_ptr() % 16:
        x = x.contiguous()
    lib = _lib.load()
    need = lib.p2p_spmm_mask_workspace(rows, cols, x.shape[0])
    ws = _workspace(x.device, need, "spmm_mask") if need else None
    call("p2p_spmm_mask_peers", ptr(x), dtype_code(x), x.shape[0], cols, x.stride(0), ptr(data), ptr(seg), rows, ys,
         n_ys, y_col0, ldy, ptr(ws), 0 if ws is None else ws.numel(), stream_of(x))
    if CHECK_WAITS:
        spmm_mask_status(x.device)


def spmm_mask_status(device=None, reset: bool = True) -> None:
    """Raises if a bitmask-layout GEMM launch gave up waiting on its pipeline since the last reset. Syncs. As with
    spmm_tc_status, the device's bitmask-GEMM workspaces are zeroed again before raising."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    try:
        call("p2p_spmm_mask_status", int(reset), torch.cuda.current_stream(dev).cuda_stream)
    except P2PError:
        torch.cuda.synchronize(dev)
        _rezero_workspaces(dev, "spmm_mask")
        torch.cuda.synchronize(dev)
        raise


def spmm_tc(x: torch.Tensor, words: torch.Tensor, seg: torch.Tensor, rows: int, cols: int, seg_cap: int,
            out: torch.Tensor | None = None) -> torch.Tensor:
    """y [tokens, rows] = x [tokens, cols] times a module in the tensor-core layout (tcgen05, bf16/f16), through the
    torch operator p2p_b200::spmm_tc."""
    require_cuda(x)
    if x.dim() != 2 or x.shape[1] != cols:
        raise P2PError(f"x of {tuple(x.shape)} does not have {cols} columns")
    if out is None:
        out = _lib.ops().spmm_tc(x, words, seg, rows, cols, seg_cap)
    else:
        _lib.ops().spmm_tc_into(x, words, seg, rows, cols, seg_cap, _out(out, (x.shape[0], rows), x))
    if CHECK_WAITS:
        spmm_tc_status(x.device)
    return out


def spmm_tc_peers(x: torch.Tensor, words: torch.Tensor, seg: torch.Tensor, rows: int, cols: int, seg_cap: int, ys,
                  n_ys: int, y_col0: int, ldy: int) -> None:
    """This rank's rows of y = x times a module in the tensor-core layout, stored at columns y_col0.. of each of the
    n_ys y buffers (a ctypes array of device pointers: every rank's y, peers' through peer memory)."""
    require_cuda(x)
    if x.dim() != 2 or x.shape[1] != cols:
        raise P2PError(f"x of {tuple(x.shape)} does not have {cols} columns")
    if x.stride(1) != 1 or x.stride(0) % 8 or x.data_ptr() % 16:
        x = x.contiguous()
    lib = _lib.load()
    need = lib.p2p_spmm_tc_workspace(rows, cols, x.shape[0])
    ws = _workspace(x.device, need, "spmm_tc") if need else None
    call("p2p_spmm_tc_peers", ptr(x), dtype_code(x), x.shape[0], cols, x.stride(0), ptr(words), ptr(seg), rows,
         seg_cap, ys, n_ys, y_col0, ldy, ptr(ws), 0 if ws is None else ws.numel(), stream_of(x))
    if CHECK_WAITS:
        spmm_tc_status(x.device)


def spmm_tc_gated(x: torch.Tensor, words: torch.Tensor, seg: torch.Tensor, layout_rows: int, cols: int, seg_cap: int,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """h [tokens, layout_rows / 2] = dtype(silu(g) * u) of a gate + up module in the interleaved tensor-core layout
    (compact.gate_up_rows), the gate applied in the GEMM's epilogue (p2p_spmm_tc_gated)."""
    require_cuda(x)
    if x.dim() != 2 or x.shape[1] != cols:
        raise P2PError(f"x of {tuple(x.shape)} does not have {cols} columns")
    if x.stride(1) != 1 or x.stride(0) % 8 or x.data_ptr() % 16:
        x = x.contiguous()
    out = _out(out, (x.shape[0], layout_rows // 2), x)
    lib = _lib.load()
    need = lib.p2p_spmm_tc_workspace(layout_rows, cols, x.shape[0])
    ws = _workspace(x.device, need, "spmm_tc") if need else None
    call("p2p_spmm_tc_gated", ptr(x), dtype_code(x), x.shape[0], cols, x.stride(0), ptr(words), ptr(seg), layout_rows,
         seg_cap, ptr(out), out.stride(0), ptr(ws), 0 if ws is None else ws.numel(), stream_of(x))
    if CHECK_WAITS:
        spmm_tc_status(x.device)
    return out


def spmm_tc_withhold(x: torch.Tensor, words: torch.Tensor, seg: torch.Tensor, rows: int, cols: int, seg_cap: int,
                     hold_tile: int, wait_us: int) -> torch.Tensor:
    """A launch of the tensor-core GEMM in which every CTA withholds its x tile number hold_tile, so the pipeline's
    bounded waits run out after wait_us: the give-up path under test. y is undefined; spmm_tc_status reports it."""
    require_cuda(x)
    x = x.contiguous()
    out = torch.zeros(x.shape[0], rows, dtype=x.dtype, device=x.device)
    lib = _lib.load()
    need = lib.p2p_spmm_tc_workspace(rows, cols, x.shape[0])
    ws = _workspace(x.device, need, "spmm_tc") if need else None
    call("p2p_spmm_tc_withhold", ptr(x), dtype_code(x), x.shape[0], cols, x.stride(0), ptr(words), ptr(seg), rows,
         seg_cap, ptr(out), out.stride(0), ptr(ws), 0 if ws is None else ws.numel(), hold_tile, wait_us, stream_of(x))
    return out


def spmm_tc_status(device=None, reset: bool = True) -> None:
    """Raises if a tensor-core GEMM launch gave up waiting on its pipeline since the last reset. Syncs. A launch that
    gave up may leave ticket counters of its workspace taken (a run that stopped before the last one of its row tile
    came), so before raising, the device's tensor-core workspaces are zeroed again: the next launch finds them as a
    fresh one would."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    try:
        call("p2p_spmm_tc_status", int(reset), torch.cuda.current_stream(dev).cuda_stream)
    except P2PError:
        torch.cuda.synchronize(dev)                   # launches on other streams may share none of them any more
        _rezero_workspaces(dev, "spmm_tc")
        torch.cuda.synchronize(dev)
        raise


def _ptr_array(ts) -> ctypes.Array:
    arr = (ctypes.c_void_p * len(ts))()
    for i, t in enumerate(ts):
        arr[i] = t.data_ptr()
    return arr


def _same(ts, ref: torch.Tensor) -> list:
    out = []
    for t in ts:
        require_cuda(t)
        if t.shape != ref.shape or t.dtype != ref.dtype:
            raise P2PError(f"part of {tuple(t.shape)} {t.dtype} differs from {tuple(ref.shape)} {ref.dtype}")
        out.append(t.contiguous())
    return out


def combine(parts: list, h: torch.Tensor, h_copy: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """h' = l_0(h) + sum_mid dtype(l_k(h) - h) + dtype(l_last(h~) - h~), fp32 sums (p2p/replica.py:81-85), through
    the torch operator p2p_b200::combine."""
    parts = _same(parts, h)
    h, h_copy = _same([h, h_copy], h)
    if out is None:
        return _lib.ops().combine(parts, h, h_copy)
    out = _out(out, tuple(h.shape), h, whole=True)
    call("p2p_combine", _ptr_array(parts), len(parts), ptr(h), ptr(h_copy), ptr(out), dtype_code(h), h.numel(),
         stream_of(h))
    return out


def sum_parts(parts: list, out: torch.Tensor | None = None) -> torch.Tensor:
    """dtype(sum of the parts in fp32, member order) (p2p/route.py:825-831), through the torch operator
    p2p_b200::sum_parts."""
    parts = _same(parts, parts[0])
    if out is None:
        return _lib.ops().sum_parts(parts)
    out = _out(out, tuple(parts[0].shape), parts[0], whole=True)
    call("p2p_sum_parts", _ptr_array(parts), len(parts), ptr(out), dtype_code(out), out.numel(), stream_of(out))
    return out


def member_part(y: torch.Tensor, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """dtype(float(y) - float(x)) (p2p/route.py:1268-1274)."""
    y, x = _same([y, x], y)
    out = _out(out, tuple(y.shape), y, whole=True)
    call("p2p_member_part", ptr(y), ptr(x), ptr(out), dtype_code(y), y.numel(), stream_of(y))
    return out
