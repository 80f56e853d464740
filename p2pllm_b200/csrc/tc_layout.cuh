// The tiled layout of a compact module for the tensor-core GEMM, shared by the builder (tiles.cu) and the GEMM
// (spmm_tc.cu).
//
// A module's rows are cut into row tiles of 128 and its columns into column tiles of 64. Each (row tile, column
// tile) pair is a segment holding the kept weights that fall in it:
//
//   words 0..7    header: 16 uint16 (two a word, low half first); header[j] = entries in the segment's rows
//                 0 .. 8j + 7, so 32-row slice s (the rows one GEMM warp expands) owns entries
//                 [header[4s-1], header[4s+3]) (header[-1] = 0) and header[15] is the segment's entry count
//   words 8..     one word per kept weight, slice after slice. Within a slice the order is free (every word
//                 carries its place); the builder fills the GEMM warp's store rounds (tiles.cu, bank_order_kernel)
//                 so that the entries one store writes fall in as few passes of shared-memory banks as the slice
//                 allows, round by round. Each word:
//                   bits 31..16  the value (bf16 or f16 bits)
//                   bits 13..0   the byte offset of that weight in the 128 x 64 tile as the tensor cores read it:
//                                row * 128 + ((2 * column) ^ ((row % 8) << 4)), the 128-byte swizzle (always even)
//                 then filler words (value 0, offset 16384: past the tile) up to a multiple of 4 words; they lie
//                 outside every slice, and the GEMM never stores them
//
// A segment starts on a 16-byte boundary and seg[rt * n_ct + ct] holds its first word; seg[n_seg] the total. Per
// kept weight this is the 2 bytes of the value plus 2 bytes of position, the same 4 bytes as values + int16 column
// indices, plus 32 bytes of header per segment (0.3% at keep 36).
#pragma once
#include <stdint.h>

namespace p2p {
namespace tc {

constexpr int kTileRows = 128;
constexpr int kTileCols = 64;
constexpr int kHeaderWords = 8;
constexpr int kGroupRows = 8;
constexpr int kSliceRows = 32;                       // rows of a tile one GEMM expander warp writes
constexpr int kSliceChunks = 8;                      // 16-byte loads a GEMM lane holds for its slice (then one word)
constexpr uint32_t kFillWord = 16384u;

__host__ __device__ __forceinline__ uint32_t swizzled_offset(int row_local, int col_local) {
    return (uint32_t)row_local * 128u + (((uint32_t)col_local * 2u) ^ (((uint32_t)row_local & 7u) << 4));
}

__host__ __device__ __forceinline__ uint32_t pack_word(uint16_t value_bits, int row_local, int col_local) {
    return ((uint32_t)value_bits << 16) | swizzled_offset(row_local, col_local);
}

}  // namespace tc
}  // namespace p2p
