"""Test infrastructure, not product: the reference's GPU kernel (p2p/compact.cu, built by oracle/build_ref.py) driven
the way the reference drives it, so it can be checked and timed beside this library's kernel on the same weights.

The reference kernel reads a module in its own layout, built on the host side by p2p.compact.Tiles
(p2p/compact.py:113-202), which cannot be imported on a machine without the reference tree. This file restates that
layout in torch:

  - the module's rows are cut into tiles of RT = 32 * WARPS rows, its columns into chunks of KCOLS;
  - within a (tile, chunk) each warp's 32 rows are held as 8 x 8 pieces, ordered by step of 16 columns, 16-row half,
    8-column half, 8-row half (the order of an m16n8k16 A fragment), p2p/compact.py:162;
  - a piece is a 64-bit mask (bit r * 8 + c) and its kept values in row-major order (p2p/compact.py:163-165);
  - woff[i] is where the values of (tile, chunk, warp) number i start (the exclusive scan of their counts), and vcap is
    the largest count of a (tile, chunk) rounded up to 8 past 7 extra (p2p/compact.py:167-173);
  - the values get 8 zero elements of tail padding, because the kernel reads 16 bytes at a time (p2p/compact.py:167).

The split choice restates Tiles._tune (p2p/compact.py:176-193): for 8, 16, 32 and 64 tokens, each candidate split
(1, 2, 3, 4, 6, 8, 12, 16, those with 2 * split <= chunks) is timed over 5 launches after one, and the fastest kept.
A pass cuts the tokens into launches of 64 (p2p/compact.py:195-201). Tests pin this restatement against layouts the
reference's own Tiles produced (tests/golden/tiles_cases.npz).
"""
from __future__ import annotations

import torch

RT, KCOLS, WARPS = 128, 64, 4            # compact.cu's defaults: P2P_WARPS 4, P2P_KCOLS 64


def words_of(idx: torch.Tensor, cols: int) -> torch.Tensor:
    """The reference's mask words of column indices [rows, k] (p2p/compact.py:36-45: bit c % 32 of word c // 32,
    int32 two's complement), built with torch on idx's device."""
    n_words = -(-cols // 32)
    mask = torch.zeros(idx.shape[0], n_words * 32, dtype=torch.int64, device=idx.device)
    mask.scatter_(1, idx.long(), 1)
    w = (mask.view(idx.shape[0], n_words, 32) << torch.arange(32, device=idx.device)).sum(-1)
    return torch.where(w >= 2 ** 31, w - 2 ** 32, w).to(torch.int32)


def _dense_and_kept(blocks: list, cols: int, dtype, device):
    """The module as one dense matrix and its kept mask, from the reference's block list (p2p/compact.py:127-128):
    ("dense", W) keeps every weight; ("sparse", values [rows, k] in column order, words int32 [rows, ceil(C/32)], C)."""
    dense, kept = [], []
    for b in blocks:
        if b[0] == "dense":
            w = b[1].to(device)
            dense.append(w)
            kept.append(torch.ones(w.shape, dtype=torch.bool, device=device))
            continue
        values, words = b[1].to(device), b[2].to(device)
        bit = torch.arange(32, device=device, dtype=torch.int32)
        m = ((words.unsqueeze(-1) >> bit) & 1).bool().reshape(words.shape[0], -1)[:, :cols]
        d = torch.zeros(m.shape, dtype=dtype, device=device)
        d[m] = values.reshape(-1)                # row by row, columns ascending: the values' own order
        dense.append(d)
        kept.append(m)
    return torch.cat(dense), torch.cat(kept)


def layout(blocks: list, device=None) -> dict:
    """The reference kernel's arrays for a module: vals, masks (int64), woff (int64), vcap, tiles, chunks, rows,
    cols."""
    first = blocks[0]
    cols = first[3] if first[0] == "sparse" else first[1].shape[1]
    dtype = first[1].dtype
    device = device or first[1].device
    dense, kept = _dense_and_kept(blocks, cols, dtype, device)
    rows = dense.shape[0]
    tiles, chunks = -(-rows // RT), -(-cols // KCOLS)
    pad_r, pad_c = tiles * RT - rows, chunks * KCOLS - cols
    dense = torch.nn.functional.pad(dense, (0, pad_c, 0, pad_r))
    kept = torch.nn.functional.pad(kept, (0, pad_c, 0, pad_r))

    def order(m):
        # rows: (tile, warp, 16-row half, 8-row half, row); columns: (chunk, 16-column step, 8-column half, column)
        v = m.reshape(tiles, WARPS, 2, 2, 8, chunks, KCOLS // 16, 2, 8)
        # -> (tile, chunk, warp, step, 16-row half, 8-column half, 8-row half, row, column)
        return v.permute(0, 5, 1, 6, 2, 7, 3, 4, 8).contiguous()

    k = order(kept)
    vals = order(dense)[k]
    bits = k.reshape(-1, 64).to(torch.int64) << torch.arange(64, device=device, dtype=torch.int64)
    masks = bits.sum(-1)                         # distinct bits: the sum is the OR (bit 63 wraps to the sign)
    counts = k.reshape(tiles, chunks, WARPS, -1).sum(-1).reshape(-1)
    woff = torch.zeros(counts.numel() + 1, dtype=torch.int64, device=device)
    woff[1:] = counts.cumsum(0)
    per_chunk = int(counts.reshape(-1, WARPS).sum(-1).max()) if counts.numel() else 0
    vcap = -(-(per_chunk + 7) // 8) * 8
    vals = torch.cat([vals, torch.zeros(8, dtype=dtype, device=device)])
    return {"vals": vals, "masks": masks, "woff": woff, "vcap": vcap, "tiles": tiles, "chunks": chunks, "rows": rows,
            "cols": cols}


class RefTiles:
    """A module in the reference kernel's layout, with the reference's per-token-count split choice."""

    def __init__(self, blocks: list, ext, tune: bool = True):
        self.ext = ext
        lay = layout(blocks)
        self.vals, self.masks, self.woff = lay["vals"], lay["masks"], lay["woff"]
        self.vcap, self.rows, self.cols, self.chunks = lay["vcap"], lay["rows"], lay["cols"], lay["chunks"]
        self._splits = self._tune() if tune else {8: 1, 16: 1, 32: 1, 64: 1}

    def _launch(self, x, splits):
        return self.ext.spmm(x, self.vals, self.woff, self.masks, self.rows, self.cols, self.vcap, splits)

    def _tune(self) -> dict:
        best = {}
        candidates = [c for c in (1, 2, 3, 4, 6, 8, 12, 16) if c == 1 or c * 2 <= self.chunks]
        for n in (8, 16, 32, 64):
            x = torch.randn(n, self.cols, device=self.vals.device, dtype=self.vals.dtype)
            times = {}
            for c in candidates:
                self._launch(x, c)
                start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record()
                for _ in range(5):
                    self._launch(x, c)
                end.record()
                end.synchronize()
                times[c] = start.elapsed_time(end)
            best[n] = min(times, key=times.get)
        return best

    def splits(self, tokens: int) -> int:
        return self._splits[8 if tokens <= 8 else 16 if tokens <= 16 else 32 if tokens <= 32 else 64]

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        x = x.contiguous()
        if x.data_ptr() % 16:
            x = x.clone()
        out = [self._launch(x[i:i + 64], self.splits(x.shape[0] - i)) for i in range(0, max(x.shape[0], 1), 64)]
        return out[0] if len(out) == 1 else torch.cat(out)
