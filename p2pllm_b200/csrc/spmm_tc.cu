// (2b) Compact sparse GEMM on the 5th-generation tensor cores: y[t, r] = sum_j v[r, j] * x[t, idx[r, j]] for bf16/f16
// weights in the tiled layout of tc_layout.cuh.
//
// Replaces p2p/compact.cu:82-278 (spmm_kernel + sum_parts + spmm), which rebuilds 8 x 8 pieces from bit masks into
// mma.sync fragments and re-reads every weight once per 64 tokens. Here a CTA owns one 128-row tile and a range of
// 64-column tiles (split-K), and every token of the pass at once (up to 512 in TMEM):
//
//   warp 16 (producer)  per column tile: TMA of the x tile [tokens x 64] (128-byte swizzle) into the x ring, one
//                       producer lane per ring slot.
//   warps 0-15 (expand) four groups of 4 warps take column tiles in turn. Each warp zeroes its 32 rows of a
//                       128 x 64 bf16 tile in the A ring (in a persistent run, warp 19 zeroes the slot instead) and
//                       writes its slice of the segment's words at the swizzled byte offsets they carry, with no
//                       barrier between warps. The words come straight from HBM into registers (coalesced, 16 bytes a
//                       lane), never through shared memory.
//   warp 19 (zero)      persistent runs only (one CTA an SM over a contiguous run of (row tile, column tile) units):
//                       a bulk copy of a zero tile into each A slot once the MMAs have read its previous tile.
//   warps 17-18 (MMA)   one elected thread each issues tcgen05.mma (M = 128, N = tokens rounded to 16, K = 16 a step)
//                       with fp32 accumulators in TMEM (alternate tiles, or halves of N past 256 tokens);
//                       tcgen05.commit frees the rings' slots.
//   warps 0-15 (epilogue) tcgen05.ld D out of TMEM, round, and write y[t, row] (through shared memory and TMA stores
//                       when unsplit), or reduce the column splits: in a thread-block cluster over DSMEM, or through
//                       fp32 partials and a ticket per row tile; both add in split order, so results do not depend on
//                       scheduling.
//
// Every mbarrier wait is bounded (about 2 s of %globaltimer): past it the kernel records where it gave up, the waits of
// the same launch give up at once, no role issues further TMA loads or MMAs, and the CTA drains what it had issued
// (the x loads landed, the MMAs completed) before it frees TMEM and exits, so a broken pipeline ends the kernel with
// an error status (p2p_spmm_tc_status) instead of hanging the GPU or leaving copies in flight.
#include <cuda.h>

#include <atomic>
#include <map>
#include <mutex>
#include <type_traits>
#include <utility>

#include "common.cuh"
#include "sm100.cuh"
#include "tc_layout.cuh"
#include "tma_host.cuh"

namespace p2p {
namespace {

using namespace sm100;

constexpr int kGroupWarps = tc::kTileRows / tc::kSliceRows;        // warps expanding one tile (a slice each)
constexpr int kGroups = 4;                                         // groups taking column tiles in turn
constexpr int kWarpRows = tc::kTileRows / kGroupWarps;             // a warp's rows of a tile
constexpr int kExpWarps = kGroupWarps * kGroups;
constexpr int kProducerWarp = kExpWarps;
constexpr int kMmaWarp = kExpWarps + 1;                           // and kMmaWarp + 1: two MMA issuers
constexpr int kTcThreads = kExpWarps * 32 + 96;
constexpr int kZeroWarp = kExpWarps + 3;                           // runs: zero copies into the A slots
constexpr int kRunThreads = kTcThreads + 32;
constexpr int kATileBytes = tc::kTileRows * tc::kTileCols * 2;   // 16 KiB
constexpr int kASlotBytes = kATileBytes;                           // 1 KiB aligned, as the 128-byte swizzle needs
constexpr int kMaxASlots = 12;                                     // A tiles in flight (even: the groups alternate)
constexpr int kMaxXSlots = 4;                                      // x tiles in flight
constexpr int kChunks = tc::kSliceChunks;                          // 16-byte loads a lane holds for one tile
constexpr int kL2Ahead = 8;                                        // tiles between a segment's L2 prefetch and its loads
constexpr uint32_t kOffsetMask = 0x3FFEu;                         // an even byte offset inside the 16 KiB tile
constexpr int kMaxTilesPerCta = 256;                               // segment offsets and headers staged in smem
// Dynamic shared memory: the 227 KiB a block may hold, less the static offsets and headers and a few scalars.
constexpr int kSmemLimit =
    227 * 1024 - (int)sizeof(int64_t) * (kMaxTilesPerCta + 1) - tc::kHeaderWords * 4 * kMaxTilesPerCta - 256;
constexpr uint64_t kWaitNs = 2000000000ull;
// The workspace: a fixed region of per-row-tile ticket counters, then the fp32 partials; no call's partials can
// overlap another call's counters, whatever the shapes.
constexpr int64_t kMaxRowTiles = 16384;
constexpr size_t kTicketRegion = kMaxRowTiles * sizeof(unsigned);

__device__ int g_tc_error;            // site of the first wait that gave up since the last reset (0: none)
__device__ unsigned g_tc_failed_seq;  // sequence number of the last launch in which a wait gave up
__device__ __align__(128) uint4 g_zero_tile[kATileBytes / 16];   // zeros, bulk-copied into a run's A slots

struct TcParams {
    const uint32_t* words;            // the module's packed words
    const int64_t* seg;               // [row_tiles * col_tiles + 1]
    int rows, col_tiles, tokens, n_total, box_rows, n_boxes, tmem_cols;
    int acc_stride;                   // TMEM columns between the two issuers' accumulators (n_total <= 256), else 0
    int a_slots, x_slots, b_bytes, kt_per_split, n_split;
    void* y;
    int64_t ldy;
    float* partial;                   // [n_split, tokens, rows_pad] when n_split > 1
    unsigned* tickets;                // [row_tiles]
    int64_t rows_pad;
    // Grouped launches (routed experts): CTA (x, y) takes row tile x of item y, an item being {expert, first row of
    // its tokens in x and y, tokens (at most 256), 0}; expert e's rows start at row tile e * item_row_tiles of the
    // stacked layout; rows = an expert's rows. Null for a plain launch.
    const int4* items;
    int item_row_tiles;
    int64_t item_bound_tiles, item_bound_rows;   // grouped: the layout's row tiles and x's rows (items past them skip)
    // Split columns reduced inside a thread-block cluster (the splits of a row tile, cluster dims 1 x n_split): each
    // CTA leaves its fp32 partial tile [tokens][128] in its own shared memory (the rings, free by then) and adds its
    // share of the tile's rows over DSMEM, split by split. 0: partials through the global workspace and a ticket.
    int cluster;
    // Unsplit plain launches: y leaves through shared memory and TMA stores (tmap_y: y [tokens, rows], boxes of 128
    // rows x box_rows tokens), instead of one 2-byte store per value.
    int y_tma;
    uint64_t wait_ns;                 // how long a pipeline wait may take before the launch gives up
    unsigned seq;                     // this launch's sequence number (nonzero), naming it in g_tc_failed_seq
    int hold_tile;                    // a test's withheld x tile (each CTA's tile of that index is never loaded), or -1
    // Gated (SiLU-and-multiply) output: the module's rows are interleaved gate / up, 64 of each a row tile (tile k:
    // gate rows 64k..64k+63, then the up rows of the same units), and y [tokens, rows / 2] takes
    // dtype(silu(gate) * up) of the two rounded outputs, column 64k + j. The accumulators meet in shared memory (or
    // the cluster's, or the partials) before the product; y never leaves through TMA.
    // gated == 2 (grouped launches only): no y; per item and unit j, sums[item, 64k + j] = the fp32 sum over the
    // item's tokens of (silu(g) * u)^2, g and u the unrounded fp32 accumulators (the gated half of expert calibration).
    int gated;
    float* sums;
    int64_t ld_sums;
    // Row sharding with the all-gather fused in: n_ys > 0 sends every value of y to each ys[k] (every rank's y, peers'
    // through peer memory) at column y_col0 + row, instead of y. Plain stores only (no TMA); vec4: 8-byte stores of 4
    // values are aligned.
    void* ys[8];
    int n_ys, vec4;                   // vec4: 8-byte stores of 4 values of y (or of every ys[k]) are aligned
    int64_t y_col0;
    int stage_peers;                  // unsplit: the tile staged in shared memory, then 16-byte stores to every ys[k]
    // Persistent runs (the kRuns instantiation; plain launches only): the module's n_units (row tile, column tile)
    // units in row-major order are cut into gridDim.x contiguous runs, CTA b taking [b U / G, (b + 1) U / G). A run
    // walks its row tiles in turn, row tile k of the run accumulating in TMEM set k % acc_sets; a row tile the run
    // holds whole goes to y, its first and last, when other runs share them, leave fp32 partials (run_partial
    // [G][2][tokens][128]: 0 = the run's first row tile, 1 = its last), and the last run of a row tile to leave its
    // partial (a ticket a row tile) adds them all in run order.
    int64_t n_units;
    float* run_partial;
    int acc_sets;
};

// The run holding unit u of a persistent launch (runs b hold [b U / G, (b + 1) U / G)).
__device__ __forceinline__ int64_t run_of(int64_t u, int64_t U, int64_t G) { return ((u + 1) * G - 1) / U; }

// Four values of y row `yrow` from module row c0 on (rows past the module are not written): to y, or to every ys[k].
template <typename T, bool kPeers>
__device__ __forceinline__ void put4(const TcParams& p, int64_t yrow, int64_t c0, const float (&v)[4]) {
    if constexpr (!kPeers) {
        T* yt = reinterpret_cast<T*>(p.y) + yrow * p.ldy;
        if (p.vec4 && c0 + 3 < p.rows) {
            uint2 raw;
            T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
            for (int c = 0; c < 4; ++c) e[c] = from_f32<T>(v[c]);
            *reinterpret_cast<uint2*>(yt + c0) = raw;
            return;
        }
#pragma unroll
        for (int c = 0; c < 4; ++c)
            if (c0 + c < p.rows) yt[c0 + c] = from_f32<T>(v[c]);
        return;
    }
    const int64_t at = yrow * p.ldy + p.y_col0 + c0;
    if (p.vec4 && c0 + 3 < p.rows) {
        uint2 raw;
        T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
        for (int c = 0; c < 4; ++c) e[c] = from_f32<T>(v[c]);
        for (int k = 0; k < p.n_ys; ++k) *reinterpret_cast<uint2*>(reinterpret_cast<T*>(p.ys[k]) + at) = raw;
        return;
    }
    for (int k = 0; k < p.n_ys; ++k) {
        T* yt = reinterpret_cast<T*>(p.ys[k]) + at;
#pragma unroll
        for (int c = 0; c < 4; ++c)
            if (c0 + c < p.rows) yt[c] = from_f32<T>(v[c]);
    }
}

// y[t, c] of a gated launch from one unit of 4 gate sums g and the 4 up sums u of the same units (fp32): each output
// rounded as the unfused path rounds it -- the projection's outputs to the model dtype, then SiLU(gate) * up in fp32.
template <typename T>
__device__ __forceinline__ void store_gated(T* yt, int64_t c0, int64_t limit, float4 g, float4 u) {
    const float gv[4] = {g.x, g.y, g.z, g.w}, uv[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        if (c0 + c >= limit) break;
        const float gr = to_f32(from_f32<T>(gv[c])), ur = to_f32(from_f32<T>(uv[c]));
        yt[c0 + c] = from_f32<T>(gr / (1.0f + expf(-gr)) * ur);
    }
}

// A warp's share of one segment's words: the entries of its 32 rows (8-row groups 4 wg .. 4 wg + 3), [lo, hi) in
// words from the CTA's first segment, from the segment's header (cumulative counts of its 8-row groups).
__device__ __forceinline__ void warp_piece(const int64_t* offs, const uint16_t* hdr, int i, int wg, int& lo, int& hi) {
    const uint16_t* h = hdr + i * 2 * tc::kHeaderWords;
    const int s0 = (int)(offs[i] - offs[0]) + tc::kHeaderWords;
    constexpr int g8 = kWarpRows / 8;                              // 8-row groups a warp
    lo = s0 + (wg ? h[g8 * wg - 1] : 0);
    hi = s0 + h[g8 * wg + g8 - 1];
}

__device__ __forceinline__ uint32_t ldg_stream(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.b32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

__device__ __forceinline__ uint4 ldg_stream4(const uint32_t* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// A warp's slice [lo, hi) in 16-byte loads from its 4-word-aligned base A = lo & ~3: load c of lane l holds words
// A + 4 (l + 32 c) .. + 3 (coalesced, and inside the segment, which ends on a 16-byte boundary). Words outside the
// slice are masked when stored; loads wholly past the slice are skipped.
__device__ __forceinline__ void load_piece(const uint32_t* words, int lo, int hi, int lane, uint4 (&buf)[kChunks]) {
    const int a0 = lo & ~3;
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
        const int a = a0 + 4 * (lane + 32 * c);
        buf[c] = a < hi ? ldg_stream4(words + a) : make_uint4(tc::kFillWord, tc::kFillWord, tc::kFillWord, tc::kFillWord);
    }
}

// A hint: bring `bytes` (a multiple of 16, 16-byte aligned) of global memory into L2, with no completion to wait on.
__device__ __forceinline__ void l2_prefetch(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}


// kL2: the launch prefetches segments into L2 ahead of the register loads (few tokens; see the expanders).
// kPeers: y goes to every ys[k] (row sharding with the all-gather fused in) instead of y.
// kRuns: a persistent run of units across row tiles (see TcParams::n_units) instead of one row tile's column range.
template <typename T, bool kL2, bool kPeers, bool kRuns = false>
__global__ void __launch_bounds__(kRuns ? kRunThreads : kTcThreads, 1)
    spmm_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_y, TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint32_t s_tmem;
    __shared__ int s_last;
    __shared__ int64_t s_offs[kMaxTilesPerCta + 1];                // this CTA's segment offsets
    __shared__ uint32_t s_hdr[kMaxTilesPerCta * tc::kHeaderWords];   // and their headers
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* gbase = smem_raw + (base - raw);
    // Two rings: A tiles (tile i in slot i % SA) and x tiles (tile i in slot i % SX), sized apart so that large x
    // tiles (many tokens) do not take the A tiles' depth.
    const int SA = p.a_slots, SX = p.x_slots;
    const uint32_t a_ring = base;                                  // SA slots of kASlotBytes
    const uint32_t x_ring = a_ring + SA * kASlotBytes;             // SX slots of b_bytes
    const uint32_t bars = x_ring + SX * p.b_bytes;
    // fulla(s): the A tile expanded (4 warps arrive); fullx(s): the x tile landed (the producer's arrive with the TMA
    // transaction count); emptya / emptyx: consumed (MMA commits).
    auto fulla = [&](int s) { return bars + 8u * s; };
    auto emptya = [&](int s) { return bars + 8u * (kMaxASlots + s); };
    auto fullx = [&](int s) { return bars + 8u * (2 * kMaxASlots + s); };
    auto emptyx = [&](int s) { return bars + 8u * (2 * kMaxASlots + kMaxXSlots + s); };
    const uint32_t done = bars + 8u * (2 * kMaxASlots + 2 * kMaxXSlots);
    // Runs: accfull(s) -- a row tile's MMAs into accumulator set s complete (both issuers commit); accempty(s) -- the set
    // read out (the 16 expander warps arrive); partdone / tickdone -- a shared row tile's partial written (16 warps) /
    // its ticket taken (thread 0); zeroed(s) -- A slot s holds zeros for its next tile (the zero warp's bulk copy).
    auto accfull = [&](int st) { return done + 8u * (1 + st); };
    auto accempty = [&](int st) { return done + 8u * (3 + st); };
    const uint32_t partdone = done + 40u, tickdone = done + 48u;
    auto zeroed = [&](int st) { return done + 56u + 8u * st; };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const WaitCtl wc{&g_tc_error, &g_tc_failed_seq, p.wait_ns, p.seq};
    // This CTA's row tile, column split, tokens, and where its rows start in x and y (a plain launch: every token,
    // row tile blockIdx.x of the module; a grouped one: its item's tokens, row tile blockIdx.x of its expert).
    int rt, split, tokens, n_total;
    int64_t xrow0 = 0, col0;
    if (p.items) {
        const int4 it = p.items[blockIdx.y];
        rt = it.x * p.item_row_tiles + (int)blockIdx.x;
        split = 0;
        xrow0 = it.y;
        tokens = it.z;
        n_total = (tokens + 15) / 16 * 16;
        col0 = (int64_t)blockIdx.x * tc::kTileRows;
        if (tokens <= 0 || n_total > p.n_total || it.x < 0 || rt >= p.item_bound_tiles || xrow0 < 0 ||
            xrow0 + tokens > p.item_bound_rows)
            return;                                                 // uniform over the CTA, before any barrier
    } else {
        rt = blockIdx.x;
        split = blockIdx.y;
        tokens = p.tokens;
        n_total = p.n_total;
        col0 = (int64_t)rt * tc::kTileRows;
    }
    // This CTA's units [u0, u1) of the module's row-major (row tile, column tile) units: one row tile's column tiles
    // kt0 .. kt0 + nk - 1, or (a run) units that may span row tiles r0 .. r0 + n_rows - 1.
    const int64_t C = p.col_tiles;
    int kt0, nk, n_rows = 1;
    int64_t u0, u1, r0 = rt;
    if constexpr (kRuns) {
        u0 = (int64_t)blockIdx.x * p.n_units / gridDim.x;
        u1 = ((int64_t)blockIdx.x + 1) * p.n_units / gridDim.x;
        nk = (int)(u1 - u0);
        r0 = u0 / C;
        n_rows = nk > 0 ? (int)((u1 - 1) / C - r0 + 1) : 0;
        kt0 = (int)(u0 - r0 * C);
        rt = (int)r0;
        col0 = r0 * tc::kTileRows;
    } else {
        kt0 = split * p.kt_per_split;
        nk = min(p.col_tiles, kt0 + p.kt_per_split) - kt0;
        u0 = (int64_t)rt * C + kt0;
        u1 = u0 + nk;
    }
    const int64_t seg0 = u0;
    for (int j = threadIdx.x; j <= nk; j += blockDim.x) s_offs[j] = p.seg[seg0 + j];
    if constexpr (kRuns) {
        // a run's many segments: their offsets first, then every header load from them at once
        __syncthreads();
        for (int j = threadIdx.x; j < nk * tc::kHeaderWords; j += blockDim.x)
            s_hdr[j] = __ldg(p.words + s_offs[j / tc::kHeaderWords] + j % tc::kHeaderWords);
    } else {
        for (int j = threadIdx.x; j < nk * tc::kHeaderWords; j += blockDim.x)
            s_hdr[j] = __ldg(p.words + p.seg[seg0 + j / tc::kHeaderWords] + j % tc::kHeaderWords);
    }

    if (threadIdx.x == 0) {
        const uint32_t consumers = p.acc_stride ? 1u : 2u;        // issuers that commit a tile's slots
        for (int s = 0; s < SA; ++s) {
            mbar_init(fulla(s), kGroupWarps);
            mbar_init(emptya(s), consumers);
        }
        for (int s = 0; s < SX; ++s) {
            mbar_init(fullx(s), 1);
            mbar_init(emptyx(s), consumers);
        }
        mbar_init(done, 2);
        if constexpr (kRuns) {
            for (int st = 0; st < 2; ++st) {
                mbar_init(accfull(st), 2);
                mbar_init(accempty(st), kExpWarps);
            }
            mbar_init(partdone, kExpWarps);
            mbar_init(tickdone, 1);
            for (int st = 0; st < SA; ++st) mbar_init(zeroed(st), 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == kProducerWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(p.tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    // Every CTA of this grid is resident: the next kernel in the stream may start launching on SMs as they free up.
    if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (warp == kProducerWarp) {
        // The x tiles (the B operand), one producer lane per slot so the slots' waits and TMA issues run side by side.
        if (lane == 0) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_x)) : "memory");
        // Launched as a programmatic dependent of the stream's previous kernel, this CTA may start while that kernel
        // still runs: everything before the first x load (barriers, TMEM, segment offsets, the weights streaming in,
        // expansion of the first tiles) overlaps its tail. x may be that kernel's output, so its loads wait here for
        // it to complete; every global write of this kernel comes after an MMA, hence after this wait.
        asm volatile("griddepcontrol.wait;" ::: "memory");
        if (lane < SX) {
            const int s = lane;
            uint32_t ph = 0;
            int uses = 0;                                           // loads issued into slot s
            int col = kt0 + lane;                                   // the x tile's column tile (runs wrap at C)
            if constexpr (kRuns) col = (int)(col % C);
            for (int i = lane; i < nk; i += SX) {
                if (i >= SX) {
                    if (!mbar_wait(emptyx(s), ph, 1, wc)) break;
                    ph ^= 1u;
                }
                if (i == p.hold_tile) break;                        // a test withholds this load
                mbar_expect_tx(fullx(s), (uint32_t)p.b_bytes);
                for (int b = 0; b < p.n_boxes; ++b)
                    tma_load_2d(x_ring + s * p.b_bytes + b * p.box_rows * 128, &tmap_x, col * tc::kTileCols,
                                (int)xrow0 + b * p.box_rows, fullx(s));
                ++uses;
                col += SX;
                if constexpr (kRuns) {
                    while (col >= C) col -= (int)C;
                }
            }
            // The slot's last load must have landed before the CTA exits (the TMA unit writes its shared memory): on
            // a normal run the MMA consumed it long ago; after a give-up this waits for the copy itself.
            if (uses) mbar_drain(fullx(s), (uint32_t)((uses - 1) & 1), 7, wc);
        }
        __syncwarp();
    } else if (warp == kMmaWarp || warp == kMmaWarp + 1) {
        // Two MMA issuers: one thread's tcgen05.mma stream runs one instruction at a time (about 63 ns each, whatever
        // N up to 256), while two threads' streams overlap. With N <= 256 issuer j takes the tiles of expander group j
        // into its own accumulator (the epilogue adds the two); with N > 256 both take every tile, issuer 0 the first
        // n0 token columns and issuer 1 the rest, into one accumulator.
        const int j = warp - kMmaWarp;
        if (lane == 0) {
            const bool by_tile = p.acc_stride != 0;
            const int n0 = by_tile ? n_total : (n_total / 2 + 15) / 16 * 16;
            const int n_mine = by_tile ? n_total : (j ? n_total - n0 : n0);
            const uint32_t id = idesc_f16<T>(n_mine);
            const uint32_t d = tmem + (by_tile ? (uint32_t)(j * p.acc_stride) : (uint32_t)(j * n0));
            const uint64_t a0 = sw128_desc(a_ring);
            const uint64_t b0 = sw128_desc(x_ring) + (by_tile ? 0u : (uint64_t)((j * n0 * 128) >> 4));
            const int step = by_tile ? 2 : 1;
            int sa = by_tile ? j : 0, sx = sa;
            uint32_t pha = 0, phx = 0, acc = 0;
            if constexpr (kRuns) {
                // Row tile by row tile: row tile k into accumulator set k % acc_sets, once the expanders have read that
                // set's previous row tile out; each row tile ends with a commit to its set's accfull.
                const int SC = p.acc_sets;
                const uint32_t set_cols = by_tile ? 2u * (uint32_t)p.acc_stride : 0u;
                int i = by_tile ? j : 0;
                bool ok = true;
                for (int k = 0; k < n_rows && ok; ++k) {
                    const int ub = (int)(min(u1, (r0 + k + 1) * C) - u0);
                    const int st = k % SC;
                    if (k >= SC) {
                        if (!(ok = mbar_wait(accempty(st), (uint32_t)((k / SC - 1) & 1), 8, wc))) break;
                        tc_fence_after();
                    }
                    const uint32_t dk = d + (uint32_t)st * set_cols;
                    acc = 0u;
                    for (; i < ub; i += step) {
                        if (!(ok = mbar_wait(fulla(sa), pha, 2, wc))) break;
                        if (!(ok = mbar_wait(fullx(sx), phx, 3, wc))) break;
                        tc_fence_after();
                        const uint64_t a_desc = a0 + (uint64_t)((sa * kASlotBytes) >> 4);
                        const uint64_t b_desc = b0 + (uint64_t)((sx * p.b_bytes) >> 4);
#pragma unroll
                        for (int kk = 0; kk < tc::kTileCols / 16; ++kk)
                            umma_f16(dk, a_desc + 2 * kk, b_desc + 2 * kk, id, acc | kk);
                        acc = 1u;
                        umma_commit(emptya(sa));
                        umma_commit(emptyx(sx));
                        advance(sa, pha, step, SA);
                        advance(sx, phx, step, SX);
                    }
                    if (ok) umma_commit(accfull(st));   // this row tile's MMAs of this issuer, once complete
                }
                umma_commit(done);
            }
            for (int i = by_tile ? j : 0; !kRuns && i < nk; i += step) {
                if (!mbar_wait(fulla(sa), pha, 2, wc)) break;     // no MMA on a tile not there
                if (!mbar_wait(fullx(sx), phx, 3, wc)) break;
                tc_fence_after();
                const uint64_t a_desc = a0 + (uint64_t)((sa * kASlotBytes) >> 4);
                const uint64_t b_desc = b0 + (uint64_t)((sx * p.b_bytes) >> 4);
#pragma unroll
                for (int k = 0; k < tc::kTileCols / 16; ++k)
                    umma_f16(d, a_desc + 2 * k, b_desc + 2 * k, id, acc | k);     // +32 bytes a K step of 16
                acc = 1u;
                umma_commit(emptya(sa));                // frees the A tile and the x tile (with the other issuer)
                umma_commit(emptyx(sx));
                advance(sa, pha, step, SA);
                advance(sx, phx, step, SX);
            }
            if (!kRuns) umma_commit(done);              // arrives once every MMA this thread issued completed
        }
        __syncwarp();
    } else if (kRuns && warp == kZeroWarp) {
        // A run's A slots are zeroed by bulk copies from a zero tile in L2, tile after tile, each once the MMAs have
        // read the slot's previous tile; the expanders wait for the copy instead of storing zeros themselves, which
        // takes the zero stores (a quarter of the expanders' shared-memory stores at 17 tokens) off their path.
        if (lane == 0) {
            int issued = 0;
            for (int i = 0; i < nk; ++i) {
                const int st = i % SA, u = i / SA;
                if (u > 0 && !mbar_wait(emptya(st), (uint32_t)((u - 1) & 1), 12, wc)) break;
                mbar_expect_tx(zeroed(st), (uint32_t)kATileBytes);
                bulk_load(a_ring + (uint32_t)(st * kASlotBytes), g_zero_tile, (uint32_t)kATileBytes, zeroed(st));
                issued = i + 1;
            }
            // every copy has landed before the CTA exits (after a give-up too)
            for (int st = 0; st < SA && st < issued; ++st)
                mbar_drain(zeroed(st), (uint32_t)(((issued - 1 - st) / SA) & 1), 13, wc);
        }
        __syncwarp();
    } else {
        // Expanders: group `grp` builds the dense 128 x 64 tiles of every fourth column tile in shared memory. Warp wg
        // owns rows 32 wg .. 32 wg + 31 of the tile: it zeroes them and writes their entries at the offsets the words
        // carry, apart from the other warps (no barrier between them), then arrives on the slot's barrier. The words
        // come straight from HBM (or L2, see below) into registers in 16-byte loads, never through shared memory.
        const int grp = warp / kGroupWarps, wg = warp % kGroupWarps;
        const uint16_t* hdr = reinterpret_cast<const uint16_t*>(s_hdr);
        int s = grp % SA;
        uint32_t ph = 0;
        const uint32_t* wbase = p.words + s_offs[0];        // 16-byte aligned: segments start on 4-word boundaries
        uint4 b0[kChunks];
        int l0 = 0, h0 = 0;
        // With few tokens (the loads, not the tensor cores or the x tiles, set the pace), each group also pulls its tile
        // kL2Ahead tiles past the one it loads into L2 (one bulk prefetch a segment), so the register loads, a few
        // tiles later, wait on L2 rather than HBM. (Measured on gate_up, 2 x 14336 x 4096: 6% faster at 17 tokens,
        // 2% slower at 272, where the x tiles and the MMAs already share the L2 traffic.)
        auto prefetch = [&](int j) {
            if (kL2 && wg == 0 && lane == 0 && j < nk)
                l2_prefetch(p.words + s_offs[j], (uint32_t)(4 * (s_offs[j + 1] - s_offs[j])));
        };
        for (int j = grp; j < kL2Ahead + 2 * kGroups && j < nk; j += kGroups) prefetch(j);
        auto fetch = [&](int i, uint4 (&b)[kChunks], int& lo, int& hi) {
            if (i < nk) {
                warp_piece(s_offs, hdr, i, wg, lo, hi);
                load_piece(wbase, lo, hi, lane, b);
                prefetch(i + kL2Ahead + 2 * kGroups);
            }
        };
        // Zeroing a slot's rows: with three or more slots a group, the group's next slot is zeroed while this tile is
        // scattered (its last use is two tiles back, long consumed), which takes the zeroing off the warp's chain of
        // waits; with two, the slot is zeroed just before its own scatter. (A run's slots are zeroed by the zero warp.)
        const bool zero_ahead = !kRuns && SA / kGroups >= 3;
        auto zero_rows = [&](int slot) {
            uint4* rows16 = reinterpret_cast<uint4*>(gbase + (size_t)slot * kASlotBytes + wg * kWarpRows * 128);
#pragma unroll
            for (int z = 0; z < kWarpRows / 4; ++z) rows16[lane + 32 * z] = make_uint4(0, 0, 0, 0);
        };
        if (zero_ahead && grp < nk) {
            zero_rows(s);                               // the group's first slot: no earlier use to wait for
            __syncwarp();
        }
        // false: a wait gave up, and the warp stops expanding (no further tiles for the MMAs to read)
        auto expand = [&](int i, const uint4 (&cur)[kChunks], int lo, int hi) -> bool {
            if (kRuns) {
                const int ok = mbar_wait(zeroed(s), ph, 5, wc);              // every lane sees the zeros landed
                if (!__all_sync(0xffffffffu, ok)) return false;
            } else if (zero_ahead) {
                int sn = s + kGroups;
                uint32_t pn = ph;
                if (sn >= SA) {
                    sn -= SA;
                    pn ^= 1u;
                }
                if (i + kGroups < nk) {
                    int ok = 1;
                    if (lane == 0 && i + kGroups >= SA) ok = mbar_wait(emptya(sn), pn ^ 1u, 5, wc);
                    if (!__shfl_sync(0xffffffffu, ok, 0)) return false;
                    zero_rows(sn);                      // ordered before its scatter by this tile's fence + sync
                }
            } else {
                int ok = 1;
                if (lane == 0 && i >= SA) ok = mbar_wait(emptya(s), ph ^ 1u, 5, wc);
                if (!__shfl_sync(0xffffffffu, ok, 0)) return false;
                zero_rows(s);
                __syncwarp();                                                // the warp's rows zeroed
            }
            const uint32_t a_s = a_ring + s * kASlotBytes;
            const int a0 = lo & ~3;
            const int lo_rel = lo - a0, hi_rel = hi - a0;
#pragma unroll
            for (int c = 0; c < kChunks; ++c) {
                if (128 * c >= hi_rel) break;                                 // the rest of the loads are filler
                const uint32_t wv[4] = {cur[c].x, cur[c].y, cur[c].z, cur[c].w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int pr = 4 * (lane + 32 * c) + j;
                    if (pr >= lo_rel && pr < hi_rel) sts_u16(a_s + (wv[j] & kOffsetMask), wv[j] >> 16);
                }
            }
            for (int e = a0 + 128 * kChunks + lane; e < hi; e += 32) {          // slices longer than the registers
                const uint32_t w = ldg_stream(wbase + e);
                sts_u16(a_s + (w & kOffsetMask), w >> 16);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(fulla(s));
            advance(s, ph, kGroups, SA);
            return true;
        };
        constexpr int G = kGroups;
        // Each tile's words are loaded just before they are written: a warp's loads are complete by the fence and
        // arrive that end its tile, so the tiles whose words are in flight at once are one a group. Four groups of 4
        // warps (32 rows a warp) measured 5.5% faster at 17 tokens and 7.7% at 272 on the bench layer than two groups
        // of 8; loading a group's next tile ahead into more register buffers measured slower.
        if constexpr (kRuns) {
            // A run. Row tile k of the run is read out of TMEM set k % SC by every expander warp (lane quarter warp %
            // 4, every fourth 16-column chunk) -- to y when the run holds the whole row tile, else to this run's fp32
            // partial, the last of the row tile's runs adding all partials in run order. A warp reads a row tile out
            // only when it must: before expanding a tile whose slot is freed by MMAs that wait for that read-out (so
            // the ring is full of later row tiles' tiles meanwhile; with two sets that is two row tiles on), and at
            // the end. (Reading out as soon as a warp is a few tiles into the next row tile stalled every warp on the
            // MMAs at once.) Every wait is bounded; a warp whose wait gave up expands no further tile but keeps to
            // the same barrier sequence.
            const int quarter = warp & 3, cgroup = warp >> 2;
            const int row_local = quarter * 32 + lane;
            const bool by_tile = p.acc_stride != 0;
            const int SC = p.acc_sets;
            const uint32_t set_cols = by_tile ? 2u * (uint32_t)p.acc_stride : 0u;
            const int64_t RG = gridDim.x, U = p.n_units;
            int n_shared = 0;                                       // shared row tiles read out so far
            auto epilogue = [&](int k) {
                const int ia = (int)(max(u0, (r0 + k) * C) - u0), ib = (int)(min(u1, (r0 + k + 1) * C) - u0);
                const int st = k % SC;
                int ok = 1;
                if (lane == 0) ok = mbar_wait(accfull(st), (uint32_t)((k / SC) & 1), 9, wc);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                tc_fence_after();
                const int64_t r = r0 + k;
                const bool whole = u0 + ia == r * C && u0 + ib == (r + 1) * C;
                const int64_t row = r * tc::kTileRows + row_local;
                const bool row_ok = row < p.rows;
                const int j_first = by_tile ? (ia & 1) : 0;             // issuer j took the run's tiles i = j mod 2
                const bool both = by_tile && ib - ia >= 2;
                const uint32_t tset = tmem + (uint32_t)st * set_cols + ((uint32_t)(quarter * 32) << 16);
                float* part = p.run_partial + ((int64_t)blockIdx.x * 2 + (k == 0 ? 0 : 1)) * tokens * tc::kTileRows +
                              row_local;
                for (int c = cgroup; ok && c < n_total / 16; c += kExpWarps / 4) {
                    float v[16];
                    const uint32_t ta = tset + (uint32_t)(c * 16);
                    tmem_ld16(ta + (uint32_t)(j_first * p.acc_stride), v);
                    if (both) {
                        float w2[16];
                        tmem_ld16(ta + (uint32_t)((j_first ^ 1) * p.acc_stride), w2);
#pragma unroll
                        for (int q = 0; q < 16; ++q) v[q] += w2[q];
                    }
                    const int t0 = c * 16, jn = min(16, tokens - t0);
                    if (whole) {
                        if (row_ok) {
                            T* dst = reinterpret_cast<T*>(p.y) + (xrow0 + t0) * p.ldy + row;
                            const int64_t ld = p.ldy;
#pragma unroll
                            for (int jj = 0; jj < 16; ++jj)
                                if (jj < jn) dst[jj * ld] = from_f32<T>(v[jj]);
                        }
                    } else {
                        float* dst = part + t0 * tc::kTileRows;
#pragma unroll
                        for (int jj = 0; jj < 16; ++jj)
                            if (jj < jn) dst[jj * tc::kTileRows] = v[jj];
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(accempty(st));              // the set may take its next row tile
                if (whole) return;
                // A shared row tile: once the 16 warps have written the partial, thread 0 takes the row tile's ticket;
                // the last run to take it adds every run's partial, run by run.
                __threadfence();
                __syncwarp();
                if (lane == 0) mbar_arrive(partdone);
                const uint32_t par = (uint32_t)(n_shared & 1);
                ++n_shared;
                const int64_t b_first = run_of(r * C, U, RG), b_last = run_of((r + 1) * C - 1, U, RG);
                if (threadIdx.x == 0) {
                    s_last = mbar_wait(partdone, par, 10, wc) &&
                             atomicAdd(&p.tickets[r], 1u) == (unsigned)(b_last - b_first);
                    mbar_arrive(tickdone);
                }
                int ok2 = 1;
                if (lane == 0) ok2 = mbar_wait(tickdone, par, 11, wc);
                if (!__shfl_sync(0xffffffffu, ok2, 0) || !s_last) return;
                __threadfence();
                // Units of (token, 4 rows), eight a thread at a time with every load of a run's partial in flight
                // together (one unit at a time, the L2 latency made this 17 us at 272 tokens); runs added in order.
                constexpr int kU = 8, kThr = kExpWarps * 32;
                const int nu = tokens * (tc::kTileRows / 4);
                for (int ub0 = threadIdx.x; ub0 < nu; ub0 += kThr * kU) {
                    float4 a[kU];
#pragma unroll
                    for (int q = 0; q < kU; ++q) a[q] = make_float4(0.f, 0.f, 0.f, 0.f);
                    for (int64_t b = b_first; b <= b_last; ++b) {
                        const int wb = (b * U / RG) / C == r ? 0 : 1;      // r is run b's first row tile, or its last
                        const float* base = p.run_partial + (b * 2 + wb) * tokens * tc::kTileRows;
                        float4 pv[kU];
#pragma unroll
                        for (int q = 0; q < kU; ++q) {
                            const int u = ub0 + q * kThr;
                            pv[q] = u < nu ? __ldcg(reinterpret_cast<const float4*>(base + (u >> 5) * tc::kTileRows +
                                                                                    (u & 31) * 4))
                                           : make_float4(0.f, 0.f, 0.f, 0.f);
                        }
#pragma unroll
                        for (int q = 0; q < kU; ++q) {
                            a[q].x += pv[q].x; a[q].y += pv[q].y; a[q].z += pv[q].z; a[q].w += pv[q].w;
                        }
                    }
#pragma unroll
                    for (int q = 0; q < kU; ++q) {
                        const int u = ub0 + q * kThr;
                        if (u >= nu) break;
                        const float vv[4] = {a[q].x, a[q].y, a[q].z, a[q].w};
                        put4<T, false>(p, xrow0 + (u >> 5), r * tc::kTileRows + (u & 31) * 4, vv);
                    }
                }
                if (threadIdx.x == 0) p.tickets[r] = 0u;                  // zero again for the next call
            };
            bool live = true;
            int k_epi = 0;
            // The tile whose MMAs expand(i) waits for, i - SA (the zero warp copies zeros into a slot, in tile order, once
            // the MMAs have read the slot's previous tile), and its row tile in the run, kept by increments (no division
            // on the warp's per-tile path).
            int dep = grp - SA, dep_row = 0;
            int dep_row_end = (int)(min(u1, (r0 + 1) * C) - u0);      // local end of row tile dep_row
            for (int i = grp;; i += G, dep += G) {
                int need = n_rows;                                      // row tiles to have read out first
                if (live && i < nk) {
                    while (dep >= dep_row_end) {
                        ++dep_row;
                        dep_row_end += (int)C;
                    }
                    need = dep >= 0 ? dep_row - SC + 1 : 0;
                }
                while (k_epi < need) epilogue(k_epi++);
                if (!live || i >= nk) break;
                fetch(i, b0, l0, h0);
                live = expand(i, b0, l0, h0);
            }
            while (k_epi < n_rows) epilogue(k_epi++);
            if (lane == 0) mbar_drain(done, 0, 6, wc);                 // no MMA may still write TMEM
            __syncwarp();
        } else {
        for (int i = grp; i < nk; i += G) {
            fetch(i, b0, l0, h0);
            if (!expand(i, b0, l0, h0)) break;
        }

        // Epilogue: D[row, token] out of TMEM, once every MMA of both issuers has completed (also after a give-up:
        // TMEM is freed below, and no MMA may still write it). Warp w reads lanes 32 (w % 4) .. + 31, every other
        // 16-column chunk.
        if (lane == 0) mbar_drain(done, 0, 6, wc);
        __syncwarp();
        tc_fence_after();
        const int quarter = warp & 3, cgroup = warp >> 2;          // 4 column groups of the 16 expander warps
        const int row_local = quarter * 32 + lane;
        const int64_t row = col0 + row_local;                       // y's column: the module's (or expert's) row
        const bool row_ok = row < p.rows;
        const bool two = p.acc_stride != 0 && nk > 1;                // issuer 1 took tiles: add its accumulator
        // Where the tile goes, decided once per CTA, with no test left inside the value loop (the chain of tests per
        // value it replaces took about 170 cycles a value: 5-9 us a CTA at 272 tokens): 0 = fp32 [token][128 rows] in the freed rings (gated, or column splits
        // added in the cluster), 1 = the dtype the same way (TMA stores of y, or peer stores), 2 = y directly,
        // 3 = the fp32 partials of the workspace.
        const int mode = ((p.gated && p.n_split == 1) || (p.n_split > 1 && p.cluster)) ? 0
                         : (p.y_tma || (kPeers && p.stage_peers))                    ? 1
                         : p.n_split == 1                                            ? 2
                                                                                     : 3;
        float* const tile_f = reinterpret_cast<float*>(gbase) + row_local;        // [t * 128] of this lane's row
        T* const tile_t = reinterpret_cast<T*>(gbase) + row_local;
        for (int c = cgroup; c < n_total / 16; c += kExpWarps / 4) {
            float v[16];
            const uint32_t ta = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(c * 16);
            tmem_ld16(ta, v);
            if (two) {
                float u[16];
                tmem_ld16(ta + (uint32_t)p.acc_stride, u);
#pragma unroll
                for (int q = 0; q < 16; ++q) v[q] += u[q];
            }
            const int t0 = c * 16, jn = min(16, tokens - t0);            // this chunk's tokens
            if (mode == 0) {
                float* d = tile_f + t0 * tc::kTileRows;
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    if (j < jn) d[j * tc::kTileRows] = v[j];
            } else if (mode == 1) {
                T* d = tile_t + t0 * tc::kTileRows;
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    if (j < jn) d[j * tc::kTileRows] = from_f32<T>(v[j]);
            } else if (mode == 2) {
                if (row_ok) {
                    if constexpr (!kPeers) {
                        T* d = reinterpret_cast<T*>(p.y) + (xrow0 + t0) * p.ldy + row;
                        const int64_t ld = p.ldy;
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            if (j < jn) d[j * ld] = from_f32<T>(v[j]);
                    } else {
                        for (int j = 0; j < jn; ++j) {
                            const int64_t at = (xrow0 + t0 + j) * p.ldy + p.y_col0 + row;
                            for (int k = 0; k < p.n_ys; ++k) reinterpret_cast<T*>(p.ys[k])[at] = from_f32<T>(v[j]);
                        }
                    }
                }
            } else if (row_ok) {
                float* d = p.partial + ((int64_t)split * p.tokens + t0) * p.rows_pad + row;
                const int64_t ld = p.rows_pad;
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    if (j < jn) d[j * ld] = v[j];
            }
        }
        if (p.y_tma) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // the staged tile, for the TMA
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kProducerWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(p.tmem_cols) : "memory");
    }
    if constexpr (kRuns) return;
    if (p.gated == 2) {
        // Column sums of squares of the gated activations: thread (unit j, token group tg) adds tokens tg, tg + 8,
        // ... in fp32; then the 8 groups are added in order (the result does not depend on scheduling).
        const float* acc = reinterpret_cast<const float*>(gbase);
        float* red = reinterpret_cast<float*>(gbase) + (size_t)p.n_total * tc::kTileRows;
        for (int q = threadIdx.x; q < 64 * 8; q += kTcThreads) {
            const int j = q & 63, tg = q >> 6;
            float sum = 0.f;
            for (int t = tg; t < tokens; t += 8) {
                const float g = acc[t * tc::kTileRows + j], u = acc[t * tc::kTileRows + 64 + j];
                const float a = g / (1.0f + expf(-g)) * u;
                sum = fmaf(a, a, sum);
            }
            red[tg * 64 + j] = sum;
        }
        __syncthreads();
        if (threadIdx.x < 64) {
            float sum = 0.f;
#pragma unroll
            for (int tg = 0; tg < 8; ++tg) sum += red[tg * 64 + threadIdx.x];
            p.sums[(int64_t)blockIdx.y * p.ld_sums + (col0 >> 1) + threadIdx.x] = sum;
        }
        return;
    }
    if (p.gated && p.n_split == 1) {
        // The tile's accumulators are in shared memory ([token][128 rows], fp32): gate unit r and up unit r sit 64
        // rows apart; every thread takes (token, 4 units) pieces.
        const float* acc = reinterpret_cast<const float*>(gbase);
        T* y = reinterpret_cast<T*>(p.y);
        const int64_t c_base = (col0 >> 1), limit = p.rows >> 1;
        for (int u = threadIdx.x; u < tokens * 16; u += kTcThreads) {
            const int t = u >> 4, r4 = (u & 15) * 4;
            const float4 g = *reinterpret_cast<const float4*>(acc + t * tc::kTileRows + r4);
            const float4 up = *reinterpret_cast<const float4*>(acc + t * tc::kTileRows + 64 + r4);
            store_gated<T>(y + (xrow0 + t) * p.ldy, c_base + r4, limit, g, up);
        }
        return;
    }
    if constexpr (kPeers) {
        if (p.stage_peers) {
            // The tile staged as [token][128 rows]: each token's 256 bytes go to every rank's y in 16-byte stores
            // (16 threads a token), the last tile's rows past the module one value at a time.
            const T* tile = reinterpret_cast<const T*>(gbase);
            for (int q = threadIdx.x; q < tokens * 16; q += kTcThreads) {
                const int t = q >> 4, c8 = (q & 15) * 8;
                const int64_t at = (xrow0 + t) * p.ldy + p.y_col0 + col0 + c8;
                if (col0 + c8 + 8 <= p.rows) {
                    const uint4 raw = *reinterpret_cast<const uint4*>(tile + t * tc::kTileRows + c8);
                    for (int k = 0; k < p.n_ys; ++k) *reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.ys[k]) + at) = raw;
                } else {
                    for (int e = 0; e < 8 && col0 + c8 + e < p.rows; ++e)
                        for (int k = 0; k < p.n_ys; ++k)
                            reinterpret_cast<T*>(p.ys[k])[at + e] = tile[t * tc::kTileRows + c8 + e];
                }
            }
            return;
        }
    }
    if (p.y_tma) {
        // The tile of y staged as [token][128 rows] in shared memory goes out in one TMA store a box (rows past the
        // module and tokens past the pass lie outside the map and are not written).
        if (threadIdx.x == 0) {
            for (int b = 0; b < p.n_boxes; ++b)
                tma_store_2d(&tmap_y, smem_u32(gbase) + (uint32_t)(b * p.box_rows * tc::kTileRows * 2), (int)col0,
                             b * p.box_rows);
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
            asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        }
        return;
    }
    if (p.n_split == 1) return;

    if (p.cluster) {
        // Every split's partial tile is in its CTA's shared memory; CTA `split` of the cluster adds up its share of the
        // tile's (token, 4-row) units, split by split, and writes y. The second barrier keeps each CTA's shared memory
        // alive until every CTA of the cluster has read it.
        cluster_sync_all();
        const int ns = p.n_split;
        const uint32_t part = smem_u32(gbase);
        if (p.gated) {
            // units of 4 gate rows, each with the 4 up rows 64 below
            const int64_t n4 = (int64_t)tokens * 16;
            const int64_t u_begin = n4 * split / ns, u_end = n4 * (split + 1) / ns;
            for (int64_t u = u_begin + threadIdx.x; u < u_end; u += kTcThreads) {
                const int t = (int)(u / 16), r4 = (int)(u % 16) * 4;
                const uint32_t off = part + (uint32_t)(t * tc::kTileRows + r4) * 4u;
                float4 g = make_float4(0.f, 0.f, 0.f, 0.f), up = g;
                for (int sp = 0; sp < ns; ++sp) {
                    const float4 a = ld_cluster_f4(cluster_addr(off, sp));
                    const float4 b = ld_cluster_f4(cluster_addr(off + 256u, sp));
                    g.x += a.x; g.y += a.y; g.z += a.z; g.w += a.w;
                    up.x += b.x; up.y += b.y; up.z += b.z; up.w += b.w;
                }
                store_gated<T>(reinterpret_cast<T*>(p.y) + (xrow0 + t) * p.ldy, (col0 >> 1) + r4, p.rows >> 1, g, up);
            }
            cluster_sync_all();
            return;
        }
        // Units of (token, 4 rows); each thread takes two at a time, every split's loads of both in flight together
        // (a remote load's latency, not the bytes, set the pace of one unit at a time); the sums still run split by
        // split, in order.
        const int n4 = tokens * (tc::kTileRows / 4);
        const int u_begin = (int)((int64_t)n4 * split / ns), u_end = (int)((int64_t)n4 * (split + 1) / ns);
        for (int u = u_begin + (int)threadIdx.x; u < u_end; u += 2 * kTcThreads) {
            const int ub = u + kTcThreads < u_end ? u + kTcThreads : u;             // the second unit (or again u)
            const uint32_t off_a = part + (uint32_t)((u >> 5) * tc::kTileRows + (u & 31) * 4) * 4u;
            const uint32_t off_b = part + (uint32_t)((ub >> 5) * tc::kTileRows + (ub & 31) * 4) * 4u;
            float4 pa[8], pb[8];
#pragma unroll
            for (int sp = 0; sp < 8; ++sp)
                if (sp < ns) {
                    pa[sp] = ld_cluster_f4(cluster_addr(off_a, sp));
                    pb[sp] = ld_cluster_f4(cluster_addr(off_b, sp));
                }
            float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
#pragma unroll
            for (int sp = 0; sp < 8; ++sp)
                if (sp < ns) {
                    a.x += pa[sp].x; a.y += pa[sp].y; a.z += pa[sp].z; a.w += pa[sp].w;
                    b.x += pb[sp].x; b.y += pb[sp].y; b.z += pb[sp].z; b.w += pb[sp].w;
                }
            const float va[4] = {a.x, a.y, a.z, a.w};
            put4<T, kPeers>(p, xrow0 + (u >> 5), col0 + (u & 31) * 4, va);
            if (ub != u) {
                const float vb[4] = {b.x, b.y, b.z, b.w};
                put4<T, kPeers>(p, xrow0 + (ub >> 5), col0 + (ub & 31) * 4, vb);
            }
        }
        cluster_sync_all();
        return;
    }

    // Split columns: the last CTA of this row tile adds the partials in split order.
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(&p.tickets[rt], 1u) == (unsigned)(p.n_split - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (p.gated) {
        // units of 4 gate rows with their 4 up rows, the splits added in order
        const int64_t n4 = (int64_t)p.tokens * 16;
        const int64_t col = (int64_t)rt * tc::kTileRows;
        const int64_t split_stride = (int64_t)p.tokens * p.rows_pad;
        for (int64_t u = threadIdx.x; u < n4; u += kTcThreads) {
            const int64_t t = u / 16, off = t * p.rows_pad + col + (u % 16) * 4;
            float4 g = make_float4(0.f, 0.f, 0.f, 0.f), up = g;
            for (int sp = 0; sp < p.n_split; ++sp) {
                const float4 a = __ldcg(reinterpret_cast<const float4*>(p.partial + sp * split_stride + off));
                const float4 b = __ldcg(reinterpret_cast<const float4*>(p.partial + sp * split_stride + off + 64));
                g.x += a.x; g.y += a.y; g.z += a.z; g.w += a.w;
                up.x += b.x; up.y += b.y; up.z += b.z; up.w += b.w;
            }
            store_gated<T>(reinterpret_cast<T*>(p.y) + t * p.ldy, (col >> 1) + (u % 16) * 4, p.rows >> 1, g, up);
        }
        if (threadIdx.x == 0) p.tickets[rt] = 0u;
        return;
    }
    // Four rows a unit (16-byte loads), kUnits units a thread at a time, every split's loads of a pair of splits in
    // flight together; the sums still run split by split, so the result does not depend on who added them.
    constexpr int kUnits = 8;
    const int64_t n4 = (int64_t)p.tokens * (tc::kTileRows / 4);
    const int64_t col = (int64_t)rt * tc::kTileRows;
    for (int64_t u0 = threadIdx.x; u0 < n4; u0 += (int64_t)kTcThreads * kUnits) {
        float4 acc[kUnits];
        int64_t off[kUnits];                                        // unit q's place in one split's partials
#pragma unroll
        for (int q = 0; q < kUnits; ++q) {
            const int64_t u = u0 + (int64_t)q * kTcThreads;
            const int64_t uc = u < n4 ? u : 0;
            off[q] = (uc / 32) * p.rows_pad + col + (uc % 32) * 4;
            acc[q] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        const int64_t split_stride = (int64_t)p.tokens * p.rows_pad;
        int sp = 0;
        for (; sp + 1 < p.n_split; sp += 2) {
            float4 a[kUnits], b[kUnits];
#pragma unroll
            for (int q = 0; q < kUnits; ++q) {
                a[q] = __ldcg(reinterpret_cast<const float4*>(p.partial + sp * split_stride + off[q]));
                b[q] = __ldcg(reinterpret_cast<const float4*>(p.partial + (sp + 1) * split_stride + off[q]));
            }
#pragma unroll
            for (int q = 0; q < kUnits; ++q) {
                acc[q].x += a[q].x; acc[q].y += a[q].y; acc[q].z += a[q].z; acc[q].w += a[q].w;
                acc[q].x += b[q].x; acc[q].y += b[q].y; acc[q].z += b[q].z; acc[q].w += b[q].w;
            }
        }
        if (sp < p.n_split) {
#pragma unroll
            for (int q = 0; q < kUnits; ++q) {
                const float4 a = __ldcg(reinterpret_cast<const float4*>(p.partial + sp * split_stride + off[q]));
                acc[q].x += a.x; acc[q].y += a.y; acc[q].z += a.z; acc[q].w += a.w;
            }
        }
#pragma unroll
        for (int q = 0; q < kUnits; ++q) {
            const int64_t u = u0 + (int64_t)q * kTcThreads;
            if (u >= n4) break;
            const int64_t t = u / 32, row = col + (u % 32) * 4;
            const float v[4] = {acc[q].x, acc[q].y, acc[q].z, acc[q].w};
            put4<T, kPeers>(p, t, row, v);
        }
    }
    if (threadIdx.x == 0) p.tickets[rt] = 0u;            // the workspace is zeroed again for the next call
}

struct TcPlan {
    int n_total, box_rows, n_boxes, tmem_cols, acc_stride, a_slots, x_slots, b_bytes, n_split, kt_per_split, smem;
};

// Token-dependent part of a launch plan: MMA N, x boxes, TMEM columns, ring depths, shared memory. Fails when the
// tokens do not fit shared memory.
int plan_tokens(int tn, TcPlan& pl) {
    // + done, the runs' six barriers and their zeroed(s) per A slot
    const int fixed = 1024 + 8 * (3 * kMaxASlots + 2 * kMaxXSlots + 7) + 64;
    pl.n_total = (tn + 15) / 16 * 16;
    pl.n_boxes = pl.n_total <= 256 ? 1 : 2;
    pl.box_rows = pl.n_total / pl.n_boxes;
    // N <= 256: an accumulator per issuer, side by side; N > 256: one, the issuers splitting its columns.
    const int acc_cols = pow2_at_least(pl.n_total);
    pl.acc_stride = pl.n_total <= 256 ? acc_cols : 0;
    pl.tmem_cols = pl.n_total <= 256 ? 2 * acc_cols : acc_cols;
    pl.b_bytes = pl.n_total * 128;
    // Ring depths: x slots first, then as many A slots as the rest holds (even, at most kMaxASlots): the
    // expanders' latency needs the A depth. When the issuers split the tiles (N <= 256) the x slots are even, so
    // every use of a slot belongs to the same issuer -- a parity wait cannot then pass on another issuer's
    // earlier, unfinished use. When both issuers take every tile, three large x slots are enough.
    const int step_x = pl.acc_stride ? 2 : 1;
    pl.x_slots = (pl.b_bytes <= 4096 || pl.acc_stride) ? 4 : 3;
    while (pl.x_slots - step_x >= 2 && kSmemLimit - fixed - pl.x_slots * pl.b_bytes < kGroups * kASlotBytes)
        pl.x_slots -= step_x;
    pl.a_slots = (kSmemLimit - fixed - pl.x_slots * pl.b_bytes) / kASlotBytes;
    if (pl.a_slots > kMaxASlots) pl.a_slots = kMaxASlots;
    pl.a_slots &= ~1;
    // Each expander group needs a slot of its own (a group's tile i takes slot i % SA, advancing kGroups a tile).
    if (pl.a_slots < kGroups) return fail(P2P_EUNSUPPORTED, "p2p_spmm_tc: %d tokens exceed shared memory", tn);
    pl.smem = fixed + pl.a_slots * kASlotBytes + pl.x_slots * pl.b_bytes;
    return P2P_OK;
}

template <typename T>
int launch_tc(const CUtensorMap& map, const CUtensorMap& ymap, const TcParams& prm, dim3 grid, int smem,
              cudaStream_t st) {
    // Few tokens: the variant that prefetches the segments into L2.
    const bool l2 = prm.n_total <= 64;
    auto kernel = spmm_tc_kernel<T, false, false>;
    if (prm.n_ys) kernel = l2 ? spmm_tc_kernel<T, true, true> : spmm_tc_kernel<T, false, true>;
    else if (prm.run_partial) kernel = l2 ? spmm_tc_kernel<T, true, false, true> : spmm_tc_kernel<T, false, false, true>;
    else if (l2) kernel = spmm_tc_kernel<T, true, false>;
    if (int e = allow_smem((const void*)kernel, smem, "p2p_spmm_tc")) return e;
    // A programmatic dependent of the stream's previous kernel (the kernel waits for it before loading x), and with
    // split columns reduced in clusters, the n_split CTAs of a row tile as one cluster (grid.y == n_split).
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = grid.y;
    attr[1].val.clusterDim.z = 1;
    cfg.gridDim = grid;
    cfg.blockDim = dim3(prm.run_partial ? kRunThreads : kTcThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = prm.cluster ? 2 : 1;
    if (cudaLaunchKernelEx(&cfg, kernel, map, ymap, prm) != cudaSuccess) return launch_status("p2p_spmm_tc");
    return launch_status("p2p_spmm_tc");
}

// Whether a launch's column splits are added inside clusters: 2 to 8 splits, the fp32 partial tile
// [tokens (rounded to 16)][128] fits the rings it replaces, and the device holds the launch's clusters in as few waves
// as the plain grid takes (a cluster of whole-SM CTAs must fit one GPC, so fewer clusters than SMs / n_split may be
// resident at once).
int max_clusters(const TcPlan& pl, int n_split);

bool cluster_reduce(const TcPlan& pl, int n_split, int64_t row_tiles) {
    if (n_split < 2 || n_split > 8) return false;
    if ((int64_t)pl.n_total * tc::kTileRows * 4 > (int64_t)pl.a_slots * kASlotBytes + (int64_t)pl.x_slots * pl.b_bytes)
        return false;
    const int resident = max_clusters(pl, n_split);
    if (resident <= 0) return false;
    const int64_t sms = sm_count();
    const int64_t plain_waves = (row_tiles * n_split + sms - 1) / sms;
    const int64_t cluster_waves = (row_tiles + resident - 1) / resident;
    return cluster_waves <= plain_waves;
}

// Clusters of n_split CTAs (this plan's shared memory) the device can run at once (cached per device and shape).
int max_clusters(const TcPlan& pl, int n_split) {
    static std::mutex mu;
    static std::map<std::pair<int, int>, int> known;         // (n_split, device) x smem -> clusters at once
    std::lock_guard<std::mutex> lock(mu);
    int dev = 0;
    cudaGetDevice(&dev);
    const auto key = std::make_pair(n_split * 64 + dev, pl.smem);
    auto it = known.find(key);
    if (it != known.end()) return it->second;
    int clusters = 0;
    const void* variants[8] = {
        (const void*)spmm_tc_kernel<__nv_bfloat16, false, false>, (const void*)spmm_tc_kernel<__nv_bfloat16, true, false>,
        (const void*)spmm_tc_kernel<__half, false, false>,        (const void*)spmm_tc_kernel<__half, true, false>,
        (const void*)spmm_tc_kernel<__nv_bfloat16, false, true>,  (const void*)spmm_tc_kernel<__nv_bfloat16, true, true>,
        (const void*)spmm_tc_kernel<__half, false, true>,         (const void*)spmm_tc_kernel<__half, true, true>};
    bool allowed = true;
    for (const void* k : variants) allowed = allowed && allow_smem(k, pl.smem, "p2p_spmm_tc") == P2P_OK;
    if (allowed) {
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 1;
        attr[0].val.clusterDim.y = n_split;
        attr[0].val.clusterDim.z = 1;
        cfg.gridDim = dim3(1, n_split);
        cfg.blockDim = dim3(kTcThreads);
        cfg.dynamicSmemBytes = pl.smem;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&clusters, spmm_tc_kernel<__nv_bfloat16, false, false>, &cfg) != cudaSuccess)
            clusters = 0;
        cudaGetLastError();                                  // a refusal here only means: use the workspace path
    }
    known[key] = clusters;
    return clusters;
}

// Columns split so that the row tiles fill the SMs: the fewest waves of CTAs a column tile's work, plus the cost of
// writing and re-reading fp32 partials (one KiB a token a row tile, against ~12 KiB a column tile of weights).
int choose_split(int64_t row_tiles, int col_tiles, int tokens, int sms) {
    int best = 1;
    double best_cost = 1e30;
    const int max_split = col_tiles < 32 ? col_tiles : 32;
    for (int s = 1; s <= max_split; ++s) {
        const int per = (col_tiles + s - 1) / s;
        if ((s - 1) * per >= col_tiles) continue;                     // an empty split
        const double waves = (double)((row_tiles * s + sms - 1) / sms);
        double cost = waves * (per + 10.0);         // + a CTA's fixed cost (fill, TMEM, epilogue): ~10 tiles' time
        if (s > 1) cost += (double)s * tokens * row_tiles / 12.0 / sms;
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = s;
        }
    }
    return best;
}

// A nonzero sequence number for each launch, so that a give-up in one launch cuts short only that launch's waits.
unsigned next_seq() {
    static std::atomic<unsigned> counter{0};
    unsigned v = ++counter;
    while (v == 0) v = ++counter;
    return v;
}

// The column split of one launch: (splits, column tiles a split), at most kMaxTilesPerCta tiles a CTA.
void plan_split(int64_t row_tiles, int col_tiles, int tokens, int sms, int* n_split, int* per) {
    int s = choose_split(row_tiles, col_tiles, tokens, sms);
    int k = (col_tiles + s - 1) / s;
    if (k > kMaxTilesPerCta) k = kMaxTilesPerCta;
    *per = k;
    *n_split = (col_tiles + k - 1) / k;
}

// Persistent runs (see TcParams::n_units): one CTA an SM, each a run of about units / SMs units (more CTAs only when
// a run would pass kMaxTilesPerCta), every SM busy to the end, instead of one CTA a row tile, which leaves a partial
// last wave when there are more row tiles than SMs. Taken for such modules when a row tile's accumulators fit TMEM
// twice (at most 128 tokens: the next row tile accumulates while the last is read out). Measured on the bench layer at
// 17 tokens: gate_up (224 row tiles, two waves on 148 SMs, the second half empty) 69.4 -> 63.9 us. Not taken: at 272
// tokens (one accumulator set, the MMAs waiting on each read-out) runs made the layer step slower, and modules of
// fewer row tiles than SMs were slower in runs than in their column splits. Returns the grid, 0 for no runs.
int64_t run_grid(int64_t row_tiles, int col_tiles, int tokens, int sms) {
    const int n = (tokens + 15) / 16 * 16;
    if (n > 128 || row_tiles <= sms) return 0;
    const int64_t U = row_tiles * col_tiles;
    int64_t g = sms;
    if ((U + g - 1) / g > kMaxTilesPerCta) g = (U + kMaxTilesPerCta - 1) / kMaxTilesPerCta;
    return g;
}

size_t run_workspace(int64_t grid, int tokens) {
    return kTicketRegion + (size_t)grid * 2 * tokens * tc::kTileRows * sizeof(float);
}

}  // namespace
}  // namespace p2p

using namespace p2p;

extern "C" size_t p2p_spmm_tc_workspace(int64_t rows, int64_t cols, int64_t tokens) {
    if (rows <= 0 || cols <= 0 || tokens <= 0) return 0;
    const int64_t row_tiles = (rows + tc::kTileRows - 1) / tc::kTileRows;
    const int col_tiles = (int)((cols + tc::kTileCols - 1) / tc::kTileCols);
    size_t need = 0;
    // Every token count a launch may take (512 a launch).
    const int chunks[2] = {(int)(tokens < 512 ? tokens : 512), (int)(tokens % 512)};
    for (int t : chunks) {
        if (t <= 0) continue;
        if (const int64_t g = run_grid(row_tiles, col_tiles, t, sm_count())) {
            const size_t w = run_workspace(g, t);
            need = need > w ? need : w;
            continue;
        }
        int n = 1, per = col_tiles;
        plan_split(row_tiles, col_tiles, t, sm_count(), &n, &per);
        if (n == 1) continue;
        TcPlan pl;
        if (plan_tokens(t, pl) == P2P_OK && cluster_reduce(pl, n, row_tiles)) continue;   // partials stay in smem
        const size_t w = kTicketRegion + (size_t)n * t * row_tiles * tc::kTileRows * sizeof(float);
        need = need > w ? need : w;
    }
    return need;
}

namespace {
// p2p_spmm_tc, with the wait limit and withheld tile of p2p_spmm_tc_withhold (hold_tile < 0: none).
int spmm_tc_impl(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ldx, const uint32_t* words,
                 const int64_t* seg, int64_t rows, int64_t seg_cap_words, void* y, int64_t ldy, void* workspace,
                 size_t workspace_bytes, void* stream, int hold_tile, uint64_t wait_ns, int gated,
                 void* const* ys = nullptr, int n_ys = 0, int64_t y_col0 = 0) {
    P2P_REQUIRE(tokens >= 0 && rows >= 0 && cols >= 1, "p2p_spmm_tc: bad shape");
    P2P_REQUIRE(!gated || rows % tc::kTileRows == 0, "p2p_spmm_tc_gated: %lld interleaved rows, not whole row tiles",
                (long long)rows);
    if (tokens == 0 || rows == 0) return P2P_OK;
    if (dtype != P2P_BF16 && dtype != P2P_F16)
        return fail(P2P_EUNSUPPORTED, "p2p_spmm_tc: bf16 or f16 (fp32 weights take p2p_spmm_rows)");
    P2P_REQUIRE(x && words && seg && (y || n_ys > 0), "p2p_spmm_tc: null pointer");
    P2P_REQUIRE(n_ys >= 0 && n_ys <= 8 && !(n_ys && gated), "p2p_spmm_tc_peers: 1 to 8 y buffers, not gated");
    for (int k = 0; k < n_ys; ++k) P2P_REQUIRE(ys[k], "p2p_spmm_tc_peers: y buffer %d is null", k);
    P2P_REQUIRE(n_ys == 0 || (y_col0 >= 0 && y_col0 + rows <= ldy),
                "p2p_spmm_tc_peers: columns %lld.. of %lld rows do not fit ldy %lld", (long long)y_col0,
                (long long)rows, (long long)ldy);
    P2P_REQUIRE(aligned16(words), "p2p_spmm_tc: words must start on a 16-byte boundary");
    P2P_REQUIRE(cols % 8 == 0 && ldx % 8 == 0 && ldx >= cols && aligned16(x),
                "p2p_spmm_tc: x needs 16-byte aligned rows (cols and ldx multiples of 8)");
    P2P_REQUIRE(ldy >= (gated ? rows / 2 : rows), "p2p_spmm_tc: ldy %lld below y's width", (long long)ldy);
    P2P_REQUIRE(seg_cap_words >= 0 && seg_cap_words % 4 == 0 &&
                    seg_cap_words <= tc::kHeaderWords + tc::kTileRows * tc::kTileCols + 4,
                "p2p_spmm_tc: segment capacity %lld words", (long long)seg_cap_words);
    P2P_REQUIRE(rows <= 0x7fffffff && cols <= 0x7fffffff, "p2p_spmm_tc: too large");
    cudaStream_t st = as_stream(stream);
    const int sms = sm_count();
    const int64_t row_tiles = (rows + tc::kTileRows - 1) / tc::kTileRows;
    const int col_tiles = (int)((cols + tc::kTileCols - 1) / tc::kTileCols);
    const int elem = 2;

    for (int64_t t0 = 0; t0 < tokens; t0 += 512) {             // at most 512 tokens (TMEM columns) a launch
        const int tn = (int)(tokens - t0 < 512 ? tokens - t0 : 512);
        TcPlan pl;
        if (int e = plan_tokens(tn, pl)) return e;
        plan_split(row_tiles, col_tiles, tn, sms, &pl.n_split, &pl.kt_per_split);
        const int64_t run_g = (!gated && n_ys == 0) ? run_grid(row_tiles, col_tiles, tn, sms) : 0;
        int acc_sets = 1;
        if (run_g) {
            pl.n_split = 1;
            pl.kt_per_split = col_tiles;
            // two accumulator sets (a row tile accumulates while the last one is read out); n_total <= 128 here
            acc_sets = 2;
            pl.tmem_cols = 4 * pl.acc_stride;
        }

        TcParams prm;
        prm.n_units = row_tiles * col_tiles;
        prm.run_partial = nullptr;
        prm.acc_sets = acc_sets;
        prm.words = words;
        prm.seg = seg;
        prm.rows = (int)rows;
        prm.col_tiles = col_tiles;
        prm.tokens = tn;
        prm.n_total = pl.n_total;
        prm.box_rows = pl.box_rows;
        prm.n_boxes = pl.n_boxes;
        prm.tmem_cols = pl.tmem_cols;
        prm.acc_stride = pl.acc_stride;
        prm.a_slots = pl.a_slots;
        prm.x_slots = pl.x_slots;
        prm.b_bytes = pl.b_bytes;
        prm.kt_per_split = pl.kt_per_split;
        prm.n_split = pl.n_split;
        prm.y = y ? reinterpret_cast<char*>(y) + t0 * ldy * elem : nullptr;
        prm.ldy = ldy;
        prm.rows_pad = row_tiles * tc::kTileRows;
        prm.partial = nullptr;
        prm.tickets = nullptr;
        prm.cluster = !run_g && cluster_reduce(pl, pl.n_split, row_tiles) ? 1 : 0;
        if (run_g) {
            const size_t need = run_workspace(run_g, tn);
            P2P_REQUIRE(workspace && workspace_bytes >= need, "p2p_spmm_tc: workspace of %zu bytes, %zu needed",
                        workspace_bytes, need);
            if (row_tiles > kMaxRowTiles) return fail(P2P_EUNSUPPORTED, "p2p_spmm_tc: %lld rows is too many", (long long)rows);
            prm.tickets = reinterpret_cast<unsigned*>(workspace);
            prm.run_partial = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + kTicketRegion);
        }
        if (pl.n_split > 1 && !prm.cluster) {
            const size_t need = kTicketRegion + (size_t)pl.n_split * tn * prm.rows_pad * sizeof(float);
            P2P_REQUIRE(workspace && workspace_bytes >= need, "p2p_spmm_tc: workspace of %zu bytes, %zu needed",
                        workspace_bytes, need);
            if (row_tiles > kMaxRowTiles) return fail(P2P_EUNSUPPORTED, "p2p_spmm_tc: %lld rows is too many", (long long)rows);
            prm.tickets = reinterpret_cast<unsigned*>(workspace);
            prm.partial = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + kTicketRegion);
        }

        prm.items = nullptr;
        prm.item_bound_tiles = prm.item_bound_rows = 0;
        prm.item_row_tiles = 0;
        prm.wait_ns = wait_ns;
        prm.seq = next_seq();
        prm.hold_tile = hold_tile;
        prm.gated = gated;
        prm.sums = nullptr;
        prm.ld_sums = 0;
        prm.n_ys = n_ys;
        prm.y_col0 = y_col0;
        prm.vec4 = ldy % 4 == 0 && y_col0 % 4 == 0;
        bool al16 = ldy % 8 == 0 && y_col0 % 8 == 0;
        for (int k = 0; k < 8; ++k) {
            prm.ys[k] = k < n_ys ? reinterpret_cast<char*>(ys[k]) + t0 * ldy * elem : nullptr;
            if (k < n_ys && (reinterpret_cast<uintptr_t>(ys[k]) & 7)) prm.vec4 = 0;
            if (k == 0 && n_ys == 0 && (reinterpret_cast<uintptr_t>(prm.y) & 7)) prm.vec4 = 0;
            if (k < n_ys && (reinterpret_cast<uintptr_t>(ys[k]) & 15)) al16 = false;
        }
        prm.stage_peers = n_ys > 0 && pl.n_split == 1 && al16 &&
                          (int64_t)pl.n_total * tc::kTileRows * 2 <= (int64_t)pl.a_slots * kASlotBytes;
        if (gated && pl.n_split == 1 &&
            (int64_t)pl.n_total * tc::kTileRows * 4 > (int64_t)pl.a_slots * kASlotBytes + (int64_t)pl.x_slots * pl.b_bytes)
            return fail(P2P_EUNSUPPORTED, "p2p_spmm_tc_gated: %d tokens do not fit the staged tile", tn);
        CUtensorMap map, ymap;
        const void* xt = reinterpret_cast<const char*>(x) + t0 * ldx * elem;
        if (int e = encode_x_map(&map, xt, dtype, tn, cols, ldx, pl.box_rows)) return e;
        // y through TMA stores when unsplit and aligned (rows of y start on 16 bytes); the staged tile is
        // n_total x 128 x 2 bytes of the rings
        prm.y_tma = !run_g && !gated && n_ys == 0 && pl.n_split == 1 && ldy % 8 == 0 && aligned16(prm.y) &&
                    (int64_t)pl.n_total * tc::kTileRows * 2 <= (int64_t)pl.a_slots * kASlotBytes;
        ymap = map;
        if (prm.y_tma && encode_y_map(&ymap, prm.y, dtype, tn, rows, ldy, pl.box_rows) != P2P_OK) prm.y_tma = 0;
        const dim3 grid(run_g ? (unsigned)run_g : (unsigned)row_tiles, (unsigned)pl.n_split);
        if (int e = dtype == P2P_BF16 ? launch_tc<__nv_bfloat16>(map, ymap, prm, grid, pl.smem, st)
                                      : launch_tc<__half>(map, ymap, prm, grid, pl.smem, st))
            return e;
    }
    return P2P_OK;
}
}  // namespace

extern "C" int p2p_spmm_tc(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ldx, const uint32_t* words,
                           const int64_t* seg, int64_t rows, int64_t seg_cap_words, void* y, int64_t ldy,
                           void* workspace, size_t workspace_bytes, void* stream) {
    return spmm_tc_impl(x, dtype, tokens, cols, ldx, words, seg, rows, seg_cap_words, y, ldy, workspace,
                        workspace_bytes, stream, -1, kWaitNs, 0);
}

extern "C" int p2p_spmm_tc_peers(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ldx,
                                 const uint32_t* words, const int64_t* seg, int64_t rows, int64_t seg_cap_words,
                                 void* const* ys, int n_ys, int64_t y_col0, int64_t ldy, void* workspace,
                                 size_t workspace_bytes, void* stream) {
    P2P_REQUIRE(ys && n_ys >= 1, "p2p_spmm_tc_peers: no y buffers");
    return spmm_tc_impl(x, dtype, tokens, cols, ldx, words, seg, rows, seg_cap_words, nullptr, ldy, workspace,
                        workspace_bytes, stream, -1, kWaitNs, 0, ys, n_ys, y_col0);
}

extern "C" int p2p_spmm_tc_gated(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ldx,
                                 const uint32_t* words, const int64_t* seg, int64_t rows, int64_t seg_cap_words,
                                 void* y, int64_t ldy, void* workspace, size_t workspace_bytes, void* stream) {
    return spmm_tc_impl(x, dtype, tokens, cols, ldx, words, seg, rows, seg_cap_words, y, ldy, workspace,
                        workspace_bytes, stream, -1, kWaitNs, 1);
}

extern "C" int p2p_spmm_tc_withhold(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ldx,
                                    const uint32_t* words, const int64_t* seg, int64_t rows, int64_t seg_cap_words,
                                    void* y, int64_t ldy, void* workspace, size_t workspace_bytes, int64_t hold_tile,
                                    int64_t wait_us, void* stream) {
    P2P_REQUIRE(hold_tile >= 0 && hold_tile < 4096, "p2p_spmm_tc_withhold: tile %lld", (long long)hold_tile);
    P2P_REQUIRE(wait_us >= 1000 && wait_us <= 2000000, "p2p_spmm_tc_withhold: a limit of 1 ms to 2 s (%lld us)",
                (long long)wait_us);
    P2P_REQUIRE(tokens <= 512, "p2p_spmm_tc_withhold: one launch (at most 512 tokens)");
    return spmm_tc_impl(x, dtype, tokens, cols, ldx, words, seg, rows, seg_cap_words, y, ldy, workspace,
                        workspace_bytes, stream, (int)hold_tile, (uint64_t)wait_us * 1000ull, 0);
}

namespace {
int grouped_impl(const void* x, int dtype, int64_t x_rows, int64_t cols, int64_t ldx, const uint32_t* words,
                 const int64_t* seg, int64_t layout_row_tiles, int64_t rows, int64_t item_row_tiles,
                 int64_t seg_cap_words, const int32_t* items, int64_t n_items, int64_t max_tokens, void* y,
                 int64_t ldy, void* stream, int gated, float* sums = nullptr, int64_t ld_sums = 0) {
    P2P_REQUIRE(x_rows >= 0 && rows >= 1 && cols >= 1 && n_items >= 0, "p2p_spmm_tc_grouped: bad shape");
    if (n_items == 0 || x_rows == 0) return P2P_OK;
    if (dtype != P2P_BF16 && dtype != P2P_F16) return fail(P2P_EUNSUPPORTED, "p2p_spmm_tc_grouped: bf16 or f16");
    P2P_REQUIRE(x && words && seg && items && (y || gated == 2) && (sums || gated != 2),
                "p2p_spmm_tc_grouped: null pointer");
    P2P_REQUIRE(aligned16(words) && aligned16(items), "p2p_spmm_tc_grouped: words and items need 16-byte alignment");
    P2P_REQUIRE(cols % 8 == 0 && ldx % 8 == 0 && ldx >= cols && aligned16(x),
                "p2p_spmm_tc_grouped: x needs 16-byte aligned rows (cols and ldx multiples of 8)");
    P2P_REQUIRE(ldy >= (gated ? rows / 2 : rows), "p2p_spmm_tc_grouped: ldy %lld below y's width", (long long)ldy);
    P2P_REQUIRE(!gated || rows % tc::kTileRows == 0,
                "p2p_spmm_tc_grouped_gated: %lld interleaved rows an expert, not whole row tiles", (long long)rows);
    P2P_REQUIRE(item_row_tiles == (rows + tc::kTileRows - 1) / tc::kTileRows,
                "p2p_spmm_tc_grouped: %lld row tiles an item for %lld rows", (long long)item_row_tiles, (long long)rows);
    P2P_REQUIRE(max_tokens >= 1 && max_tokens <= 256, "p2p_spmm_tc_grouped: items of 1 to 256 tokens (%lld)",
                (long long)max_tokens);
    P2P_REQUIRE(seg_cap_words >= 0 && seg_cap_words % 4 == 0 &&
                    seg_cap_words <= tc::kHeaderWords + tc::kTileRows * tc::kTileCols + 4,
                "p2p_spmm_tc_grouped: segment capacity %lld words", (long long)seg_cap_words);
    P2P_REQUIRE(x_rows <= 0x7fffffff && n_items <= 65535, "p2p_spmm_tc_grouped: too large");
    const int col_tiles = (int)((cols + tc::kTileCols - 1) / tc::kTileCols);
    // An item takes whole rows in one CTA, which stages the offsets and headers of all its column tiles.
    P2P_REQUIRE(col_tiles <= kMaxTilesPerCta, "p2p_spmm_tc_grouped: %lld columns; at most %d (%d column tiles a CTA)",
                (long long)cols, kMaxTilesPerCta * tc::kTileCols, kMaxTilesPerCta);
    cudaStream_t st = as_stream(stream);
    TcPlan pl;
    if (int e = plan_tokens((int)max_tokens, pl)) return e;
    TcParams prm;
    prm.words = words;
    prm.seg = seg;
    prm.rows = (int)rows;
    prm.col_tiles = col_tiles;
    prm.tokens = (int)max_tokens;
    prm.n_total = pl.n_total;
    prm.box_rows = pl.box_rows;
    prm.n_boxes = pl.n_boxes;
    prm.tmem_cols = pl.tmem_cols;
    prm.acc_stride = pl.acc_stride;
    prm.a_slots = pl.a_slots;
    prm.x_slots = pl.x_slots;
    prm.b_bytes = pl.b_bytes;
    prm.kt_per_split = col_tiles;                             // whole rows: items already spread the work
    prm.n_split = 1;
    prm.y = y;
    prm.ldy = ldy;
    prm.rows_pad = 0;
    prm.partial = nullptr;
    prm.tickets = nullptr;
    prm.items = reinterpret_cast<const int4*>(items);
    prm.item_bound_tiles = layout_row_tiles;
    prm.item_bound_rows = x_rows;
    prm.item_row_tiles = (int)item_row_tiles;
    prm.y_tma = 0;
    prm.cluster = 0;
    prm.wait_ns = kWaitNs;
    prm.seq = next_seq();
    prm.hold_tile = -1;
    prm.gated = gated;
    prm.sums = sums;
    prm.ld_sums = ld_sums;
    prm.n_ys = 0;
    prm.vec4 = 0;
    prm.y_col0 = 0;
    prm.stage_peers = 0;
    prm.n_units = 0;
    prm.run_partial = nullptr;
    prm.acc_sets = 1;
    for (int k = 0; k < 8; ++k) prm.ys[k] = nullptr;
    if (gated && (int64_t)pl.n_total * tc::kTileRows * 4 + (gated == 2 ? 64 * 8 * 4 : 0) >
                     (int64_t)pl.a_slots * kASlotBytes + (int64_t)pl.x_slots * pl.b_bytes)
        return fail(P2P_EUNSUPPORTED, "p2p_spmm_tc_grouped_gated: %lld tokens an item do not fit the staged tile",
                    (long long)max_tokens);
    CUtensorMap map;
    if (int e = encode_x_map(&map, x, dtype, x_rows, cols, ldx, pl.box_rows)) return e;
    const dim3 grid((unsigned)item_row_tiles, (unsigned)n_items);
    return dtype == P2P_BF16 ? launch_tc<__nv_bfloat16>(map, map, prm, grid, pl.smem, st)
                             : launch_tc<__half>(map, map, prm, grid, pl.smem, st);
}
}  // namespace

extern "C" int p2p_spmm_tc_grouped(const void* x, int dtype, int64_t x_rows, int64_t cols, int64_t ldx,
                                   const uint32_t* words, const int64_t* seg, int64_t layout_row_tiles,
                                   int64_t rows, int64_t item_row_tiles, int64_t seg_cap_words, const int32_t* items,
                                   int64_t n_items, int64_t max_tokens, void* y, int64_t ldy, void* stream) {
    return grouped_impl(x, dtype, x_rows, cols, ldx, words, seg, layout_row_tiles, rows, item_row_tiles,
                        seg_cap_words, items, n_items, max_tokens, y, ldy, stream, 0);
}

extern "C" int p2p_spmm_tc_grouped_gated(const void* x, int dtype, int64_t x_rows, int64_t cols, int64_t ldx,
                                         const uint32_t* words, const int64_t* seg, int64_t layout_row_tiles,
                                         int64_t rows, int64_t item_row_tiles, int64_t seg_cap_words,
                                         const int32_t* items, int64_t n_items, int64_t max_tokens, void* y,
                                         int64_t ldy, void* stream) {
    return grouped_impl(x, dtype, x_rows, cols, ldx, words, seg, layout_row_tiles, rows, item_row_tiles,
                        seg_cap_words, items, n_items, max_tokens, y, ldy, stream, 1);
}

extern "C" int p2p_spmm_tc_grouped_gated_sums(const void* x, int dtype, int64_t x_rows, int64_t cols, int64_t ldx,
                                              const uint32_t* words, const int64_t* seg, int64_t layout_row_tiles,
                                              int64_t rows, int64_t item_row_tiles, int64_t seg_cap_words,
                                              const int32_t* items, int64_t n_items, int64_t max_tokens, float* sums,
                                              int64_t ld_sums, void* stream) {
    P2P_REQUIRE(ld_sums >= rows / 2, "p2p_spmm_tc_grouped_gated_sums: ld_sums %lld below %lld", (long long)ld_sums,
                (long long)(rows / 2));
    return grouped_impl(x, dtype, x_rows, cols, ldx, words, seg, layout_row_tiles, rows, item_row_tiles,
                        seg_cap_words, items, n_items, max_tokens, nullptr, rows / 2, stream, 2, sums, ld_sums);
}

extern "C" int p2p_spmm_tc_status(int reset, void* stream) {
    cudaStream_t st = as_stream(stream);
    int v = 0;
    if (cudaMemcpyFromSymbolAsync(&v, g_tc_error, sizeof(int), 0, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return fail(P2P_ECUDA, "p2p_spmm_tc_status: %s", cudaGetErrorString(cudaGetLastError()));
    if (reset && v) {
        const int zero = 0;
        cudaMemcpyToSymbolAsync(g_tc_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
        cudaStreamSynchronize(st);
    }
    if (v) return fail(P2P_ECUDA, "p2p_spmm_tc: a pipeline wait timed out (site %d)", v);
    return P2P_OK;
}
