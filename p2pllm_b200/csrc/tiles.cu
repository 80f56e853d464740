// Builds the tiled layout of tc_layout.cuh from a module's row blocks (values + ascending column indices, or dense
// rows). The B200 counterpart of p2p/compact.py:124-166 (Tiles.__init__, which re-tiles a module into 8 x 8 pieces):
// run once when a replica is loaded.
//
//   p2p_tiles_plan: per (row, column tile) counts -> per segment prefix of rows -> padded segment sizes -> seg[]
//   p2p_tiles_fill: every kept weight to seg[segment] + (rows above it in the segment) + (its rank in its row's part)
//
// It also builds the bitmask layout of mask_layout.cuh (the reference's storage, p2p/compact.py:36-45, re-tiled for
// spmm_mask.cu), one CTA a segment:
//   p2p_mask_plan: each segment's kept weights -> its byte size -> seg[]
//   p2p_mask_fill: the segment's 128 x 64 tile in shared memory -> piece masks, their counts and offsets -> header,
//                  masks and values
#include "common.cuh"
#include "mask_layout.cuh"
#include "tc_layout.cuh"

namespace p2p {
namespace {

constexpr int kMaxBlocks = 8;
constexpr int kBuildBlock = 256;
constexpr int64_t kMaxColTiles = 4096;   // columns up to 262,144

struct Blocks {
    p2p_row_block b[kMaxBlocks];
    int n;
};

struct Shape {
    int64_t rows, cols, row_tiles, col_tiles, n_seg;
};

Shape shape_of(const p2p_row_block* blocks, int n, int64_t cols) {
    Shape s;
    s.rows = 0;
    for (int i = 0; i < n; ++i) s.rows = s.rows > blocks[i].row0 + blocks[i].rows ? s.rows : blocks[i].row0 + blocks[i].rows;
    s.cols = cols;
    s.row_tiles = (s.rows + tc::kTileRows - 1) / tc::kTileRows;
    s.col_tiles = (cols + tc::kTileCols - 1) / tc::kTileCols;
    s.n_seg = s.row_tiles * s.col_tiles;
    return s;
}

// The block holding output row `row`, or -1.
__device__ __forceinline__ int block_of(const Blocks& bl, int64_t row) {
    for (int i = 0; i < bl.n; ++i)
        if (row >= bl.b[i].row0 && row < bl.b[i].row0 + bl.b[i].rows) return i;
    return -1;
}

template <typename I>
__device__ __forceinline__ int col_at(const p2p_row_block& b, int64_t lr, int64_t j) {
    return b.idx ? (int)reinterpret_cast<const I*>(b.idx)[lr * b.ld + j] : (int)j;
}

// cnt[row, ct] = kept weights of `row` in column tile ct.
template <typename I>
__global__ void __launch_bounds__(kBuildBlock) count_kernel(Blocks bl, int64_t rows, int n_ct, int* __restrict__ cnt) {
    extern __shared__ int hist[];
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        for (int c = threadIdx.x; c < n_ct; c += kBuildBlock) hist[c] = 0;
        __syncthreads();
        const int bi = block_of(bl, row);
        if (bi >= 0) {
            const p2p_row_block& b = bl.b[bi];
            const int64_t lr = row - b.row0;
            for (int64_t j = threadIdx.x; j < b.k; j += kBuildBlock) atomicAdd(&hist[col_at<I>(b, lr, j) >> 6], 1);
        }
        __syncthreads();
        for (int c = threadIdx.x; c < n_ct; c += kBuildBlock) cnt[row * n_ct + c] = hist[c];
        __syncthreads();
    }
}

// Within each segment, cnt[row, ct] becomes the entries of the rows above `row`; segraw = the segment's entries,
// segcnt = its words (header + entries padded to a multiple of 4).
__global__ void __launch_bounds__(kBuildBlock) prefix_kernel(int64_t rows, int n_ct, int* __restrict__ cnt,
                                                              int64_t* __restrict__ segcnt, int* __restrict__ segraw) {
    const int64_t rt = blockIdx.x;
    for (int ct = threadIdx.x; ct < n_ct; ct += kBuildBlock) {
        int64_t run = 0;
        for (int rl = 0; rl < tc::kTileRows; ++rl) {
            const int64_t row = rt * tc::kTileRows + rl;
            if (row >= rows) break;
            const int c = cnt[row * n_ct + ct];
            cnt[row * n_ct + ct] = (int)run;
            run += c;
        }
        segraw[rt * n_ct + ct] = (int)run;
        segcnt[rt * n_ct + ct] = tc::kHeaderWords + ((run + 3) & ~(int64_t)3);
    }
}

// Each segment's header: the entries of its 8-row groups, cumulative.
__global__ void header_kernel(int64_t rows, int n_ct, int64_t n_seg, const int* __restrict__ cnt,
                              const int* __restrict__ segraw, const int64_t* __restrict__ seg,
                              uint32_t* __restrict__ words) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n_seg; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t rt = i / n_ct, ct = i % n_ct;
        uint32_t h[16];
        for (int j = 0; j < 16; ++j) {
            const int64_t next = rt * tc::kTileRows + (int64_t)tc::kGroupRows * (j + 1);   // first row past group j
            h[j] = (j < 15 && next < rows) ? (uint32_t)cnt[next * n_ct + ct] : (uint32_t)segraw[i];
        }
        for (int m = 0; m < tc::kHeaderWords; ++m) words[seg[i] + m] = (h[2 * m] & 0xffffu) | (h[2 * m + 1] << 16);
    }
}

// seg[i] = sum of segcnt[< i], seg[n] = the total: one block, each thread a contiguous chunk.
__global__ void __launch_bounds__(1024) scan_kernel(const int64_t* __restrict__ segcnt, int64_t n,
                                                     int64_t* __restrict__ seg) {
    __shared__ int64_t part[1024];
    const int t = threadIdx.x;
    const int64_t chunk = (n + 1023) / 1024;
    const int64_t a = min(n, t * chunk), b = min(n, a + chunk);
    int64_t s = 0;
    for (int64_t i = a; i < b; ++i) s += segcnt[i];
    part[t] = s;
    __syncthreads();
    if (t == 0) {
        int64_t run = 0;
        for (int i = 0; i < 1024; ++i) {
            const int64_t v = part[i];
            part[i] = run;
            run += v;
        }
        seg[n] = run;
    }
    __syncthreads();
    int64_t run = part[t];
    for (int64_t i = a; i < b; ++i) {
        seg[i] = run;
        run += segcnt[i];
    }
}

__global__ void fill_pad_kernel(uint32_t* __restrict__ words, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        words[i] = tc::kFillWord;
}

__device__ int g_fill_errors;

template <typename I>
__global__ void __launch_bounds__(kBuildBlock) fill_kernel(Blocks bl, int64_t rows, int n_ct, const int* __restrict__ cnt,
                                                            const int64_t* __restrict__ seg, uint32_t* __restrict__ words,
                                                            int64_t n_words) {
    extern __shared__ int sm[];
    int* hist = sm;            // [n_ct]: this row's count per column tile
    int* first = sm + n_ct;    // [n_ct]: this row's first entry in each column tile
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const int bi = block_of(bl, row);
        if (bi < 0) continue;                                   // uniform over the block
        const p2p_row_block& b = bl.b[bi];
        const int64_t lr = row - b.row0;
        for (int c = threadIdx.x; c < n_ct; c += kBuildBlock) hist[c] = 0;
        __syncthreads();
        for (int64_t j = threadIdx.x; j < b.k; j += kBuildBlock) atomicAdd(&hist[col_at<I>(b, lr, j) >> 6], 1);
        __syncthreads();
        if (threadIdx.x == 0) {
            int run = 0;
            for (int c = 0; c < n_ct; ++c) {
                first[c] = run;
                run += hist[c];
            }
        }
        __syncthreads();
        const int64_t rt = row / tc::kTileRows;
        const int rl = (int)(row % tc::kTileRows);
        const uint16_t* vals = reinterpret_cast<const uint16_t*>(b.vals);
        for (int64_t j = threadIdx.x; j < b.k; j += kBuildBlock) {
            const int col = col_at<I>(b, lr, j);
            const int ct = col >> 6;
            const int64_t rank = j - first[ct];
            const int64_t pos = seg[rt * n_ct + ct] + tc::kHeaderWords + cnt[row * n_ct + ct] + rank;
            if (rank < 0 || rank >= hist[ct] || pos >= n_words) {   // indices not ascending: refuse, never write
                atomicAdd(&g_fill_errors, 1);
                continue;
            }
            words[pos] = tc::pack_word(vals[lr * b.ld + j], rl, col & 63);
        }
        __syncthreads();
    }
}

// Reorders the entries of every 32-row slice of every segment for the GEMM's stores (a slice: the rows one expander
// warp writes, tc::kSliceRows). The GEMM's warp loads its slice in 16-byte pieces from the 4-word boundary A at or
// below the slice's start: lane l's load c (c < tc::kSliceChunks) holds words A + 4 (l + 32 c) .. + 3, and store round
// 4 c + j writes word j of every lane's load c (rounds 0..31, the first 1024 words from A); past those, round 32 + m
// stores words A + 1024 + 32 m + l. A store takes one pass per entry on its busiest shared-memory bank (bits 2..6 of
// the entry's byte offset), so the entries of one round should differ in bank. Round by round, the places are filled
// greedily: the fewest entries of any one bank the remaining entries allow (every bank gives up to m - 1, the banks
// with the most left give the m-th ones), which also keeps the banks' counts level for the later rounds. (Dealing
// entries in (rank within bank, bank) order instead lets the rounds drift off the bank boundaries once banks run out,
// and costs about half again as many store passes at keep 36.) One warp a slice (32 rows x 64 columns: at most 64
// entries a bank, 2048 in all).
constexpr int kOrderWarps = 2;
constexpr int kSlices = tc::kTileRows / tc::kSliceRows;                // a segment's slices
constexpr int kSliceMax = tc::kSliceRows * tc::kTileCols;
constexpr int kRegWords = tc::kSliceChunks * 128;                        // words the lanes' 16-byte loads hold
constexpr int kRegRounds = tc::kSliceChunks * 4;
constexpr int kStoreRounds = kRegRounds + (kSliceMax + 3 - kRegWords + 31) / 32;   // rounds over the slice's words
static_assert(kSlices % kOrderWarps == 0, "a block takes whole segments' slices");

__device__ __forceinline__ int ceil_div4(int x) { return (x + 3) >> 2; }   // arithmetic shift: negative x too

__global__ void __launch_bounds__(kOrderWarps * 32) bank_order_kernel(const int64_t* __restrict__ seg, int64_t n_seg,
                                                                      uint32_t* __restrict__ words) {
    __shared__ uint32_t buf[kOrderWarps][kSliceMax];
    __shared__ uint32_t byrank[kOrderWarps][kSliceMax];        // the entries grouped by bank
    __shared__ uint8_t rk[kOrderWarps][kSliceMax];
    __shared__ int cnt[kOrderWarps][32];
    __shared__ int rpre[kOrderWarps][32];                       // where each bank's entries start in byrank
    __shared__ int llo[kOrderWarps][kStoreRounds + 1];          // a round's first lane in the slice
    __shared__ int rstart[kOrderWarps][kStoreRounds + 1];       // and its lanes in the slice
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const unsigned below = (1u << lane) - 1u;
    const int64_t n_work = n_seg * (kSlices / kOrderWarps);
    for (int64_t item = blockIdx.x; item < n_work; item += gridDim.x) {
        const int64_t sg = item / (kSlices / kOrderWarps);
        const int slice = (int)(item % (kSlices / kOrderWarps)) * kOrderWarps + w;
        const int64_t s0 = seg[sg];
        auto hdr = [&](int j) { return (int)((words[s0 + j / 2] >> (16 * (j & 1))) & 0xffffu); };
        constexpr int g8 = tc::kSliceRows / tc::kGroupRows;           // 8-row groups a slice
        const int lo = slice ? hdr(g8 * slice - 1) : 0, hi = hdr(g8 * slice + g8 - 1);
        const int n = hi - lo;
        const int64_t first = s0 + tc::kHeaderWords + lo;        // the slice's first word
        const int lo_rel = (int)(first & 3);                      // its place above the 4-word boundary A
        uint32_t* base = words + (first - lo_rel);                // A
        cnt[w][lane] = 0;
        __syncwarp();
        if (n > 0 && n <= kSliceMax) {
            // rank of every entry within its bank
            for (int j = 0; j < n; j += 32) {
                const int e = j + lane;
                const bool ok = e < n;
                const uint32_t v = ok ? base[lo_rel + e] : 0u;
                const int b = ok ? (int)((v >> 2) & 31u) : 32 + lane;   // lanes past the end: a bank of their own
                const unsigned peers = __match_any_sync(0xffffffffu, b);
                const int before = __popc(peers & below);
                if (ok) {
                    buf[w][e] = v;
                    rk[w][e] = (uint8_t)(cnt[w][b] + before);
                }
                __syncwarp();
                if (ok && before == 0) cnt[w][b] += __popc(peers);
                __syncwarp();
            }
            // the entries grouped by bank (lane b: bank b), each bank's in their current order
            const int cb = cnt[w][lane];
            int start = cb;
            for (int d = 1; d < 32; d <<= 1) {
                const int t = __shfl_up_sync(0xffffffffu, start, d);
                if (lane >= d) start += t;
            }
            start -= cb;
            rpre[w][lane] = start;
            __syncwarp();
            for (int e = lane; e < n; e += 32) {
                const uint32_t v = buf[w][e];
                byrank[w][rpre[w][(v >> 2) & 31u] + rk[w][e]] = v;
            }
            // the store rounds: the lanes [llo, lhi) of round R that fall in the slice
            if (lane == 0) {
                for (int R = 0; R < kStoreRounds; ++R) {
                    int lo_l, hi_l;
                    if (R < kRegRounds) {
                        const int c = R >> 2, j = R & 3;
                        lo_l = max(0, ceil_div4(lo_rel - 128 * c - j));
                        hi_l = min(32, ceil_div4(lo_rel + n - 128 * c - j));
                    } else {
                        const int b0 = kRegWords + 32 * (R - kRegRounds);
                        lo_l = max(0, lo_rel - b0);
                        hi_l = min(32, lo_rel + n - b0);
                    }
                    llo[w][R] = lo_l;
                    rstart[w][R] = hi_l > lo_l ? hi_l - lo_l : 0;   // the round's entries
                }
            }
            __syncwarp();
            // Round by round, the fewest entries of any one bank: with cap places, the smallest m with
            // sum_b min(rem_b, m) >= cap; every bank gives min(rem_b, m - 1), and the banks with the most left give
            // the m-th entries still needed (ties to the lower bank), which keeps the counts level for later rounds.
            int rem = cb, taken = 0;
            for (int R = 0; R < kStoreRounds; ++R) {
                const int cap = rstart[w][R];
                if (cap == 0) continue;
                int m = 1;
                while (__reduce_add_sync(0xffffffffu, min(rem, m)) < cap) ++m;
                const int base_take = min(rem, m - 1);
                const int extra = cap - __reduce_add_sync(0xffffffffu, base_take);
                const bool cand = rem >= m;
                int rank = 0;
                for (int o = 0; o < 32; ++o) {
                    const int ro = __shfl_sync(0xffffffffu, rem, o);
                    const bool co = __shfl_sync(0xffffffffu, cand ? 1 : 0, o) != 0;
                    rank += (co && (ro > rem || (ro == rem && o < lane))) ? 1 : 0;
                }
                const int take = base_take + ((cand && rank < extra) ? 1 : 0);
                int off = take;
                for (int d = 1; d < 32; d <<= 1) {
                    const int t = __shfl_up_sync(0xffffffffu, off, d);
                    if (lane >= d) off += t;
                }
                off -= take;
                for (int q = 0; q < take; ++q) {
                    const int l = llo[w][R] + off + q;                    // the round's lane, hence its word
                    const int pr = R < kRegRounds ? 128 * (R >> 2) + 4 * l + (R & 3)
                                                  : kRegWords + 32 * (R - kRegRounds) + l;
                    base[pr] = byrank[w][start + taken + q];
                }
                rem -= take;
                taken += take;
            }
        }
        __syncwarp();
    }
}

// ---- the bitmask layout (mask_layout.cuh) ---------------------------------------------------------------------------

// [lo, hi): row lr's entries of block b in columns [c0, c0 + 64), by binary search of its ascending indices.
template <typename I>
__device__ __forceinline__ void row_range(const p2p_row_block& b, int64_t lr, int c0, int64_t& lo, int64_t& hi) {
    if (!b.idx) {
        lo = c0;
        hi = c0 + mk::kTileCols < b.k ? c0 + mk::kTileCols : b.k;
        return;
    }
    const I* ix = reinterpret_cast<const I*>(b.idx) + lr * b.ld;
    auto lower = [&](int v) {
        int64_t a = 0, z = b.k;
        while (a < z) {
            const int64_t m = (a + z) >> 1;
            if ((int)ix[m] < v) a = m + 1; else z = m;
        }
        return a;
    };
    lo = lower(c0);
    hi = lower(c0 + mk::kTileCols);
}

// segbytes[segment] = the segment's size in bytes (one CTA of 128 threads a segment, a thread a row).
template <typename I>
__global__ void __launch_bounds__(mk::kTileRows) mask_count_kernel(Blocks bl, int64_t rows, int n_ct, int64_t n_seg,
                                                                    int64_t* __restrict__ segbytes) {
    __shared__ int total;
    for (int64_t sg = blockIdx.x; sg < n_seg; sg += gridDim.x) {
        if (threadIdx.x == 0) total = 0;
        __syncthreads();
        const int64_t row = (sg / n_ct) * mk::kTileRows + threadIdx.x;
        const int c0 = (int)(sg % n_ct) * mk::kTileCols;
        const int bi = row < rows ? block_of(bl, row) : -1;
        if (bi >= 0) {
            int64_t lo, hi;
            row_range<I>(bl.b[bi], row - bl.b[bi].row0, c0, lo, hi);
            if (hi > lo) atomicAdd(&total, (int)(hi - lo));
        }
        __syncthreads();
        if (threadIdx.x == 0) segbytes[sg] = mk::segment_bytes(total);
        __syncthreads();
    }
}

// Writes every segment: its tile gathered into shared memory (values and keep bits by row), then thread t builds
// piece t % 16 of block t / 16 (its mask, its count), the counts are scanned in piece order, and each thread writes its
// piece's mask words, the start offsets of its two halves and its values. Indices out of ascending order within a tile, or past the columns, are counted as errors.
template <typename I>
__global__ void __launch_bounds__(mk::kTileRows) mask_fill_kernel(Blocks bl, int64_t rows, int64_t cols, int n_ct,
                                                                   int64_t n_seg, const int64_t* __restrict__ seg,
                                                                   uint8_t* __restrict__ data, int64_t n_bytes) {
    __shared__ uint16_t tile[mk::kTileRows][mk::kTileCols];
    __shared__ uint32_t keep[mk::kTileRows][2];
    __shared__ int off[mk::kTileRows + 1];
    const int t = threadIdx.x;
    for (int64_t sg = blockIdx.x; sg < n_seg; sg += gridDim.x) {
        const int64_t row = (sg / n_ct) * mk::kTileRows + t;
        const int c0 = (int)(sg % n_ct) * mk::kTileCols;
        uint32_t k0 = 0, k1 = 0;
        const int bi = row < rows ? block_of(bl, row) : -1;
        if (bi >= 0) {
            const p2p_row_block& b = bl.b[bi];
            const int64_t lr = row - b.row0;
            int64_t lo, hi;
            row_range<I>(b, lr, c0, lo, hi);
            const uint16_t* vals = reinterpret_cast<const uint16_t*>(b.vals) + lr * b.ld;
            int prev = -1;
            for (int64_t j = lo; j < hi; ++j) {
                const int c = b.idx ? (int)reinterpret_cast<const I*>(b.idx)[lr * b.ld + j] : (int)j;
                if (c <= prev || c < c0 || c >= c0 + mk::kTileCols || c >= cols) {
                    atomicAdd(&g_fill_errors, 1);
                    continue;
                }
                prev = c;
                tile[t][c - c0] = vals[j];
                if (c - c0 < 32) k0 |= 1u << (c - c0); else k1 |= 1u << (c - c0 - 32);
            }
        }
        keep[t][0] = k0;
        keep[t][1] = k1;
        __syncthreads();
        const int blk = t >> 4, p = t & 15;
        uint32_t m[2] = {0u, 0u};
        for (int bit = 0; bit < 64; ++bit) {
            const int r = blk * mk::kBlockRows + mk::piece_row(p, bit), c = mk::piece_col(p, bit);
            if ((keep[r][c >> 5] >> (c & 31)) & 1u) m[bit >> 5] |= 1u << (bit & 31);
        }
        const int n = __popc(m[0]) + __popc(m[1]);
        off[t + 1] = n;
        __syncthreads();
        if (t == 0) {
            off[0] = 0;
            for (int q = 1; q <= mk::kTileRows; ++q) off[q] += off[q - 1];
        }
        __syncthreads();
        const int64_t base = seg[sg];
        const int64_t end = mk::segment_bytes(off[mk::kTileRows]);
        if (base + end <= n_bytes && seg[sg + 1] - base == end) {
            uint8_t* d = data + base;
            if (t < mk::kBlocks) reinterpret_cast<uint16_t*>(d)[t] = (uint16_t)off[16 * (t + 1)];
            uint8_t* bd = d + mk::kHeaderBytes + blk * mk::kBlockBytes;
            reinterpret_cast<uint32_t*>(bd)[p] = m[0];
            reinterpret_cast<uint32_t*>(bd + mk::kHiAt)[p] = m[1];
            reinterpret_cast<uint16_t*>(bd + mk::kOloAt)[p] = (uint16_t)(2 * off[t]);
            reinterpret_cast<uint16_t*>(bd + mk::kOhiAt)[p] = (uint16_t)(2 * (off[t] + __popc(m[0])));
            uint16_t* v = reinterpret_cast<uint16_t*>(d + mk::kValuesAt) + off[t];
            for (int bit = 0; bit < 64; ++bit)
                if ((m[bit >> 5] >> (bit & 31)) & 1u)
                    *v++ = tile[blk * mk::kBlockRows + mk::piece_row(p, bit)][mk::piece_col(p, bit)];
            for (int64_t z = mk::kValuesAt + 2 * (int64_t)off[mk::kTileRows] + t; z < end; z += mk::kTileRows) d[z] = 0;
        } else if (t == 0) {
            atomicAdd(&g_fill_errors, 1);                       // seg[] does not fit this module: write nothing
        }
        __syncthreads();
    }
}

int check_blocks(const p2p_row_block* blocks, int nblocks, int idx_bytes, int64_t cols, Blocks& bl, const char* who) {
    if (!blocks || nblocks < 1 || nblocks > kMaxBlocks) return fail(P2P_EINVAL, "%s: 1 to %d row blocks", who, kMaxBlocks);
    if (idx_bytes != 2 && idx_bytes != 4) return fail(P2P_EINVAL, "%s: idx_bytes %d", who, idx_bytes);
    if (cols < 1 || (cols + 63) / 64 > kMaxColTiles) return fail(P2P_EUNSUPPORTED, "%s: %lld columns", who, (long long)cols);
    bl.n = nblocks;
    for (int i = 0; i < nblocks; ++i) {
        const p2p_row_block& b = blocks[i];
        if (b.rows < 0 || b.row0 < 0 || b.k < 0 || (b.rows > 0 && !b.vals) || (b.rows > 0 && b.k > 0 && b.ld < b.k))
            return fail(P2P_EINVAL, "%s: block %d", who, i);
        if (!b.idx && b.k != cols) return fail(P2P_EINVAL, "%s: dense block %d needs k == cols", who, i);
        bl.b[i] = b;
    }
    return P2P_OK;
}

}  // namespace
}  // namespace p2p

using namespace p2p;

extern "C" size_t p2p_tiles_workspace(const p2p_row_block* blocks, int nblocks, int64_t cols) {
    if (!blocks || nblocks < 1 || cols < 1) return 0;
    const Shape s = shape_of(blocks, nblocks, cols);
    const size_t cnt_bytes = (size_t)s.row_tiles * tc::kTileRows * s.col_tiles * sizeof(int);
    return (cnt_bytes + 255) / 256 * 256 + (size_t)s.n_seg * (sizeof(int64_t) + sizeof(int)) + 256;
}

namespace {
// Scratch of the builder: cnt [row_tiles * 128, col_tiles] int, segcnt [n_seg] int64, segraw [n_seg] int.
struct BuildScratch {
    int* cnt;
    int64_t* segcnt;
    int* segraw;
};
BuildScratch scratch_of(void* workspace, const Shape& s) {
    BuildScratch b;
    const size_t cnt_bytes = (size_t)s.row_tiles * tc::kTileRows * s.col_tiles * sizeof(int);
    char* w = reinterpret_cast<char*>(workspace);
    b.cnt = reinterpret_cast<int*>(w);
    b.segcnt = reinterpret_cast<int64_t*>(w + (cnt_bytes + 255) / 256 * 256);
    b.segraw = reinterpret_cast<int*>(b.segcnt + s.n_seg);
    return b;
}
}  // namespace

extern "C" int p2p_tiles_plan(const p2p_row_block* blocks, int nblocks, int idx_bytes, int64_t cols, int64_t* seg,
                              int64_t* total_words, void* workspace, size_t workspace_bytes, void* stream) {
    Blocks bl;
    if (int e = check_blocks(blocks, nblocks, idx_bytes, cols, bl, "p2p_tiles_plan")) return e;
    P2P_REQUIRE(seg && total_words && workspace, "p2p_tiles_plan: null seg, total or workspace");
    const Shape s = shape_of(blocks, nblocks, cols);
    P2P_REQUIRE(workspace_bytes >= p2p_tiles_workspace(blocks, nblocks, cols), "p2p_tiles_plan: workspace too small");
    cudaStream_t st = as_stream(stream);
    const BuildScratch sc = scratch_of(workspace, s);
    int* cnt = sc.cnt;
    int64_t* segcnt = sc.segcnt;
    const size_t cnt_bytes = (size_t)s.row_tiles * tc::kTileRows * s.col_tiles * sizeof(int);
    if (cudaMemsetAsync(cnt, 0, cnt_bytes, st) != cudaSuccess) return launch_status("p2p_tiles_plan memset");
    const int smem = (int)(s.col_tiles * sizeof(int));
    const int grid = (int)(s.rows < sm_count() * 8 ? s.rows : sm_count() * 8);
    if (s.rows > 0) {
        if (idx_bytes == 2) {
            if (int e = allow_smem((const void*)count_kernel<int16_t>, smem, "p2p_tiles_plan")) return e;
            count_kernel<int16_t><<<grid, kBuildBlock, smem, st>>>(bl, s.rows, (int)s.col_tiles, cnt);
        } else {
            if (int e = allow_smem((const void*)count_kernel<int32_t>, smem, "p2p_tiles_plan")) return e;
            count_kernel<int32_t><<<grid, kBuildBlock, smem, st>>>(bl, s.rows, (int)s.col_tiles, cnt);
        }
        prefix_kernel<<<(unsigned)s.row_tiles, kBuildBlock, 0, st>>>(s.rows, (int)s.col_tiles, cnt, segcnt, sc.segraw);
    }
    scan_kernel<<<1, 1024, 0, st>>>(segcnt, s.n_seg, seg);
    if (int e = launch_status("p2p_tiles_plan")) return e;
    if (cudaMemcpyAsync(total_words, seg + s.n_seg, sizeof(int64_t), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return launch_status("p2p_tiles_plan read-back");
    return P2P_OK;
}

extern "C" int p2p_tiles_fill(const p2p_row_block* blocks, int nblocks, int idx_bytes, int64_t cols, int dtype,
                              const int64_t* seg, uint32_t* words, int64_t n_words, void* workspace,
                              size_t workspace_bytes, void* stream) {
    Blocks bl;
    if (int e = check_blocks(blocks, nblocks, idx_bytes, cols, bl, "p2p_tiles_fill")) return e;
    if (dtype != P2P_BF16 && dtype != P2P_F16)
        return fail(P2P_EUNSUPPORTED, "p2p_tiles_fill: the tensor-core layout holds bf16 or f16 values");
    P2P_REQUIRE(seg && words && workspace, "p2p_tiles_fill: null pointer");
    P2P_REQUIRE(workspace_bytes >= p2p_tiles_workspace(blocks, nblocks, cols), "p2p_tiles_fill: workspace too small");
    const Shape s = shape_of(blocks, nblocks, cols);
    cudaStream_t st = as_stream(stream);
    const BuildScratch sc = scratch_of(workspace, s);
    const int* cnt = sc.cnt;
    const int zero = 0;
    if (cudaMemcpyToSymbolAsync(g_fill_errors, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return launch_status("p2p_tiles_fill reset");
    if (n_words > 0) fill_pad_kernel<<<sm_count() * 4, 256, 0, st>>>(words, n_words);
    if (s.n_seg > 0)
        header_kernel<<<(unsigned)((s.n_seg + 255) / 256), 256, 0, st>>>(s.rows, (int)s.col_tiles, s.n_seg, cnt,
                                                                          sc.segraw, seg, words);
    const int smem = (int)(2 * s.col_tiles * sizeof(int));
    const int grid = (int)(s.rows < sm_count() * 8 ? s.rows : sm_count() * 8);
    if (s.rows > 0) {
        if (idx_bytes == 2) {
            if (int e = allow_smem((const void*)fill_kernel<int16_t>, smem, "p2p_tiles_fill")) return e;
            fill_kernel<int16_t><<<grid, kBuildBlock, smem, st>>>(bl, s.rows, (int)s.col_tiles, cnt, seg, words, n_words);
        } else {
            if (int e = allow_smem((const void*)fill_kernel<int32_t>, smem, "p2p_tiles_fill")) return e;
            fill_kernel<int32_t><<<grid, kBuildBlock, smem, st>>>(bl, s.rows, (int)s.col_tiles, cnt, seg, words, n_words);
        }
    }
    if (s.n_seg > 0) {
        const int64_t items = s.n_seg * (kSlices / kOrderWarps);
        bank_order_kernel<<<(unsigned)(items < sm_count() * 8 ? items : sm_count() * 8), kOrderWarps * 32, 0, st>>>(
            seg, s.n_seg, words);
    }
    if (int e = launch_status("p2p_tiles_fill")) return e;
    int bad = 0;
    if (cudaMemcpyFromSymbolAsync(&bad, g_fill_errors, sizeof(int), 0, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return launch_status("p2p_tiles_fill read-back");
    if (bad) return fail(P2P_EDATA, "p2p_tiles_fill: %d column indices out of ascending order", bad);
    return P2P_OK;
}

extern "C" size_t p2p_mask_workspace(const p2p_row_block* blocks, int nblocks, int64_t cols) {
    if (!blocks || nblocks < 1 || cols < 1) return 0;
    const Shape s = shape_of(blocks, nblocks, cols);
    return (size_t)s.n_seg * sizeof(int64_t) + 256;
}

extern "C" int p2p_mask_plan(const p2p_row_block* blocks, int nblocks, int idx_bytes, int64_t cols, int64_t* seg,
                             int64_t* total_bytes, void* workspace, size_t workspace_bytes, void* stream) {
    Blocks bl;
    if (int e = check_blocks(blocks, nblocks, idx_bytes, cols, bl, "p2p_mask_plan")) return e;
    P2P_REQUIRE(seg && total_bytes && workspace, "p2p_mask_plan: null seg, total or workspace");
    P2P_REQUIRE(workspace_bytes >= p2p_mask_workspace(blocks, nblocks, cols), "p2p_mask_plan: workspace too small");
    const Shape s = shape_of(blocks, nblocks, cols);
    cudaStream_t st = as_stream(stream);
    int64_t* segbytes = reinterpret_cast<int64_t*>(workspace);
    const int grid = (int)(s.n_seg < sm_count() * 16 ? s.n_seg : sm_count() * 16);
    if (s.n_seg > 0) {
        if (idx_bytes == 2)
            mask_count_kernel<int16_t><<<grid, mk::kTileRows, 0, st>>>(bl, s.rows, (int)s.col_tiles, s.n_seg, segbytes);
        else
            mask_count_kernel<int32_t><<<grid, mk::kTileRows, 0, st>>>(bl, s.rows, (int)s.col_tiles, s.n_seg, segbytes);
    }
    scan_kernel<<<1, 1024, 0, st>>>(segbytes, s.n_seg, seg);
    if (int e = launch_status("p2p_mask_plan")) return e;
    if (cudaMemcpyAsync(total_bytes, seg + s.n_seg, sizeof(int64_t), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return launch_status("p2p_mask_plan read-back");
    return P2P_OK;
}

extern "C" int p2p_mask_fill(const p2p_row_block* blocks, int nblocks, int idx_bytes, int64_t cols, int dtype,
                             const int64_t* seg, void* data, int64_t n_bytes, void* stream) {
    Blocks bl;
    if (int e = check_blocks(blocks, nblocks, idx_bytes, cols, bl, "p2p_mask_fill")) return e;
    if (dtype != P2P_BF16 && dtype != P2P_F16)
        return fail(P2P_EUNSUPPORTED, "p2p_mask_fill: the bitmask layout holds bf16 or f16 values");
    P2P_REQUIRE(seg && data && n_bytes >= 0, "p2p_mask_fill: null pointer");
    P2P_REQUIRE(aligned16(data), "p2p_mask_fill: data must start on a 16-byte boundary");
    const Shape s = shape_of(blocks, nblocks, cols);
    cudaStream_t st = as_stream(stream);
    const int zero = 0;
    if (cudaMemcpyToSymbolAsync(g_fill_errors, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return launch_status("p2p_mask_fill reset");
    const int grid = (int)(s.n_seg < sm_count() * 16 ? s.n_seg : sm_count() * 16);
    if (s.n_seg > 0) {
        if (idx_bytes == 2)
            mask_fill_kernel<int16_t><<<grid, mk::kTileRows, 0, st>>>(bl, s.rows, cols, (int)s.col_tiles, s.n_seg, seg,
                                                                       reinterpret_cast<uint8_t*>(data), n_bytes);
        else
            mask_fill_kernel<int32_t><<<grid, mk::kTileRows, 0, st>>>(bl, s.rows, cols, (int)s.col_tiles, s.n_seg, seg,
                                                                       reinterpret_cast<uint8_t*>(data), n_bytes);
    }
    if (int e = launch_status("p2p_mask_fill")) return e;
    int bad = 0;
    if (cudaMemcpyFromSymbolAsync(&bad, g_fill_errors, sizeof(int), 0, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return launch_status("p2p_mask_fill read-back");
    if (bad) return fail(P2P_EDATA, "p2p_mask_fill: %d column indices out of ascending order or range", bad);
    return P2P_OK;
}
