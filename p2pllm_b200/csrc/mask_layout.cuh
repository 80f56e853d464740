// The bitmask layout of a compact module for the tensor-core GEMM of spmm_mask.cu, shared by its builder (tiles.cu)
// and the GEMM. It stores what the reference stores (p2p/compact.py:36-45) -- the kept values, 2 bytes each, and one
// bit per weight -- plus a 16-bit offset per 32 bits of mask: 1.6x fewer bytes than values + int16 indices at keep
// 33-36.
//
// Rows are cut into row tiles of 128 and columns into column tiles of 64, as in tc_layout.cuh. Each (row tile, column
// tile) pair is a segment, 16-byte aligned, seg[rt * n_ct + ct] holding its first byte and seg[n_seg] the total:
//
//   bytes 0..15       header: 8 uint16, count[b] = the segment's values in 16-row blocks 0..b (count[7]: all)
//   bytes 16..1551    8 blocks of 192 bytes:
//                       lo[16]   uint32: bits 0..31 of each piece's mask (the piece's rows 0..3)
//                       hi[16]   uint32: bits 32..63 (rows 4..7)
//                       olo[16]  uint16: where the values of each piece's bits 0..31 start, in bytes from the
//                                segment's first value
//                       ohi[16]  uint16: where those of bits 32..63 start, likewise
//   bytes 1552..      values: block by block, piece by piece, each piece's in its bits' order; then zero bytes up to
//                     the next 16-byte boundary
//
// A block is 16 rows x 64 columns, held as the 16 pieces that the registers of one tcgen05.st.16x256b.x4 store hold:
// piece p = 4 rep + 2 h + j covers rows 8 h + g (g = 0..7) of the block and columns 16 rep + 4 u + 2 j + e (u = 0..3,
// e = 0..1) of the tile; bit 8 g + 2 u + e of its 64-bit mask is that weight. Lane 4 g + u of the warp that builds the
// block owns bits 8 g + 2 u and + 1 of every piece -- the two halves of its register p -- so it reads only one mask
// word per piece (lo for g < 4, hi otherwise) and one start offset, and finds its values with one popcount. A piece's
// values, at most 64, lie within 128 bytes: the 32 lanes' reads of a piece never clash on a shared-memory bank.
#pragma once
#include <stdint.h>

namespace p2p {
namespace mk {

constexpr int kTileRows = 128;
constexpr int kTileCols = 64;
constexpr int kBlockRows = 16;
constexpr int kBlocks = kTileRows / kBlockRows;          // 8
constexpr int kPieces = 16;                              // a block's pieces
constexpr int kHeaderBytes = 16;
constexpr int kBlockBytes = 192;                         // lo, hi, olo, ohi of one block
constexpr int kHiAt = 64, kOloAt = 128, kOhiAt = 160;    // within a block's 192 bytes
constexpr int kValuesAt = kHeaderBytes + kBlocks * kBlockBytes;      // 1552
constexpr int kMaxSegBytes = kValuesAt + kTileRows * kTileCols * 2;  // 17,936 (a multiple of 16)

// The row (within its block) and column (within its tile) of bit `bit` of piece p.
__host__ __device__ __forceinline__ int piece_row(int p, int bit) { return 8 * ((p >> 1) & 1) + (bit >> 3); }
__host__ __device__ __forceinline__ int piece_col(int p, int bit) {
    return 16 * (p >> 2) + 4 * ((bit >> 1) & 3) + 2 * (p & 1) + (bit & 1);
}

__host__ __device__ __forceinline__ int64_t segment_bytes(int64_t values) {
    return (kValuesAt + 2 * values + 15) / 16 * 16;
}

}  // namespace mk
}  // namespace p2p
