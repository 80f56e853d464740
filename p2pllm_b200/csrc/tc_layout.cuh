// The tiled layout of a compact module for the tensor-core GEMM, shared by the builder (tiles.cu) and the GEMM
// (spmm_tc.cu).
//
// A module's rows are cut into row tiles of 128 and its columns into column tiles of 64. Each (row tile, column
// tile) pair is a segment: the kept weights that fall in it, one 32-bit word each,
//     bits 31..16  the value (bf16 or f16 bits)
//     bits 15..14  0
//     bit  13      pad flag (1: a filler word, ignored)
//     bits 12..6   row within the row tile (0..127)
//     bits  5..0   column within the column tile (0..63)
// in row order, then column order. A segment starts on a 16-byte boundary (its word count is padded to a multiple
// of 4 with filler words), and seg[rt * n_ct + ct] holds its first word; seg[n_seg] the total. Per kept weight this is
// the 2 bytes of the value plus 2 bytes of (row, column), the same 4 bytes as values + int16 column indices.
#pragma once
#include <stdint.h>

namespace p2p {
namespace tc {

constexpr int kTileRows = 128;
constexpr int kTileCols = 64;
constexpr uint32_t kPadWord = 1u << 13;

__host__ __device__ __forceinline__ uint32_t pack_word(uint16_t value_bits, int row_local, int col_local) {
    return ((uint32_t)value_bits << 16) | ((uint32_t)row_local << 6) | (uint32_t)col_local;
}

}  // namespace tc
}  // namespace p2p
