// (2c) The compact sparse GEMM on the bitmask layout of mask_layout.cuh: y[t, r] = sum_c W[r, c] x[t, c] for bf16 /
// f16 weights stored as the reference stores them (the kept values, 2 bytes each, plus one bit a weight), on tcgen05
// tensor cores with the weight tiles in tensor memory.
//
// Replaces p2p/compact.cu:82-278 (spmm_kernel, sum_parts, spmm), whose warps build mma.sync fragments from 8 x 8 mask
// pieces and re-read every weight once per 64 tokens. Here the module's (128-row tile, 64-column tile) units, in row
// order, are split into one contiguous run per CTA, one CTA per SM (a persistent grid: no partial waves, and the
// pipeline fills once per CTA, not once per row tile), with every token of the launch (up to 288) at once:
//
//   warp 17 (segments)  one thread streams the run's segments (header, masks, offsets, values: ~7 KB a tile at keep
//                       33-36; the run is one contiguous range of the layout) into a byte ring in shared memory with
//                       bulk copies, up to 16 segments ahead: the bytes in flight that keep HBM busy, no registers held.
//   warp 16 (x)         TMA of each unit's x tile [tokens x 64] (128-byte swizzle) into the x ring, one lane a slot.
//   warps 0-15 (build)  two groups of 8 warps take alternate units. Warp w builds 16-row block 2 (w % 4) + (w % 8) / 4
//                       of its group's tile (the block's rows are TMEM lanes warp w may write): each lane turns its two
//                       bits of each of the block's 16 pieces, with the piece's values read from the ring, into a
//                       register of two bf16 weights, and one tcgen05.st.16x256b.x4 writes the block into the tile's A
//                       slot in tensor memory. A piece's values lie within 128 bytes, so a warp's reads never clash on
//                       a bank; there is no zeroing pass, no scattered store and no A tile in shared memory.
//   warps 18-19 (MMA)   one elected thread each issues tcgen05.mma kind::f16 with A from tensor memory (M = 128,
//                       K = 16 a step) and B = the x tile (N = tokens rounded to 16), fp32 accumulators in TMEM: with
//                       N <= 128 the issuers take alternate units into accumulators of their own (two MMA streams run
//                       side by side), above that both take every unit, each half of N. A row tile's accumulators are
//                       double-buffered when they fit (N <= 64), so the next row tile starts while the last drains.
//   warps 20-23 (epilogue) per finished row tile: tcgen05.ld D, round and write y; a row tile shared with the
//                       neighbouring CTAs' runs leaves an fp32 partial instead, and the last of its CTAs to finish (a
//                       ticket per row tile) adds the partials in CTA order -- column order -- and writes y, so results
//                       do not depend on scheduling.
//
// Every wait is bounded (2 s of %globaltimer): a launch that gives up records where, issues no further copies or MMAs,
// drains what it issued and exits (p2p_spmm_mask_status reads the site).
#include <atomic>
#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"
#include "mask_layout.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

namespace p2p {
namespace {

using namespace sm100;

constexpr int kGroupWarps = 8;                         // warps building one tile (a 16-row block each)
constexpr int kGroups = 2;                             // groups taking alternate units
constexpr int kBuildWarps = kGroupWarps * kGroups;
constexpr int kXWarp = kBuildWarps;                    // 16: x tiles (and the TMEM allocation)
constexpr int kSegWarp = kBuildWarps + 1;              // 17: segments
constexpr int kMmaWarp = kBuildWarps + 2;              // 18 and 19: MMA issuers
constexpr int kEpiWarp = kBuildWarps + 4;              // 20..23: epilogue (warp % 4 = its TMEM lane quarter)
constexpr int kThreads = (kBuildWarps + 8) * 32;       // 768
constexpr int kTickets = 16;                           // segments in flight
constexpr int kMaxXSlots = 4;
constexpr int kMaxASlots = 12;                         // A tiles in tensor memory
constexpr int kMaxAccSlots = 2;                        // row-tile accumulator sets
constexpr int kACols = 32;                             // TMEM columns of one A tile (128 x 64 16-bit weights)
constexpr int kTmemCols = 512;
constexpr int kMaxN = 288;                             // tokens a launch (accumulator + A slots fit 512 columns)
constexpr int kMaxUnits = 256;                         // units a CTA (segment offsets staged in shared memory)
constexpr int kRingPad = 64;                           // slack past the ring: reads of a piece may run 2 bytes past it
constexpr int kSmemLimit = 227 * 1024 - (int)sizeof(int64_t) * (kMaxUnits + 1) - 8 * kTickets - 128;
constexpr uint64_t kWaitNs = 2000000000ull;
constexpr int64_t kMaxRowTiles = 16384;
constexpr int kMaxPeers = 8;                           // y buffers a launch writes (the ranks of one node)
constexpr size_t kTicketRegion = kMaxRowTiles * sizeof(unsigned);

__device__ int g_mask_error;            // site of the first wait that gave up since the last reset (0: none)
__device__ unsigned g_mask_failed_seq;  // sequence number of the last launch in which a wait gave up

struct MaskParams {
    const uint8_t* data;              // the module's segments
    const int64_t* seg;               // [row_tiles * col_tiles + 1] byte offsets
    int rows, col_tiles, tokens, n_total, box_rows, n_boxes;
    int by_tile;                      // 1: issuer j takes units j, j + 2, .. into its own accumulator (N <= 128)
    int acc_cols;                     // TMEM columns of one issuer's accumulator (by_tile), else N
    int acc_slots;                    // accumulator sets (row tiles in flight): 2 when they fit, else 1
    int a_col0;                       // first TMEM column of the A slots
    int a_slots, x_slots, b_bytes, ring_bytes;
    int64_t units;                    // row tiles x column tiles
    int ctas;                         // the grid
    // How the units are cut into runs. splits == 0 (persistent): CTA b takes units [units b / ctas, units (b + 1) /
    // ctas), whatever row tiles they span. splits = s >= 1 (aligned): CTA b takes the (b % s)-th run of per_split
    // column tiles of row tile b / s; with cluster, the s CTAs of a row tile form a thread-block cluster and add their
    // partial tiles over DSMEM.
    int splits, per_split, cluster;
    // y [tokens, ldy]: every value of row r goes to column y_col0 + r of each of the n_ys buffers -- this rank's y and,
    // when the module is row-sharded over a node's GPUs, every peer's (stores over NVLink: the gather fused into the
    // GEMM's epilogue).
    void* ys[kMaxPeers];
    int n_ys;
    int64_t y_col0;
    int64_t ldy;
    float* partial;                   // [ctas][2][tokens][128]: each CTA's first and last row tile, when shared
    unsigned* tickets;                // [row tiles], zero between calls
    uint64_t wait_ns;
    unsigned seq;
};

// y[t, row] = v in each of the launch's y buffers.
template <typename T>
__device__ __forceinline__ void store_y(const MaskParams& p, int64_t t, int64_t row, float v) {
    const T val = from_f32<T>(v);
    const int64_t at = t * p.ldy + p.y_col0 + row;
    for (int k = 0; k < p.n_ys; ++k) reinterpret_cast<T*>(p.ys[k])[at] = val;
}

// 1 in every thread of the 4 epilogue warps if `ok` holds in all 128 of them (barrier 1), else 0.
__device__ __forceinline__ int epilogue_all(int ok) {
    int r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.s32 p, %1, 0;\n\t"
        "bar.red.and.pred q, 1, 128, p;\n\t"
        "selp.s32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(ok)
        : "memory");
    return r;
}

// The first unit of CTA b's run, and one past its last.
__device__ __forceinline__ int64_t run_start(const MaskParams& p, int64_t b) {
    if (p.splits == 0) return p.units * b / p.ctas;
    const int64_t rt = b / p.splits, sp = b % p.splits;
    return rt * p.col_tiles + min((int64_t)p.col_tiles, sp * p.per_split);
}
__device__ __forceinline__ int64_t run_end(const MaskParams& p, int64_t b) {
    if (p.splits == 0) return p.units * (b + 1) / p.ctas;
    const int64_t rt = b / p.splits, sp = b % p.splits;
    return rt * p.col_tiles + min((int64_t)p.col_tiles, (sp + 1) * p.per_split);
}

// The CTA whose run holds unit u.
__device__ __forceinline__ int64_t run_of(const MaskParams& p, int64_t u) {
    if (p.splits == 0) return ((u + 1) * p.ctas + p.units - 1) / p.units - 1;
    return (u / p.col_tiles) * p.splits + (u % p.col_tiles) / p.per_split;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    spmm_mask_kernel(const __grid_constant__ CUtensorMap tmap_x, MaskParams p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint32_t s_tmem;
    __shared__ int s_last;
    __shared__ int64_t s_offs[kMaxUnits + 1];                       // this CTA's segment offsets (bytes)
    __shared__ uint32_t s_ring_off[kTickets];                       // where segment i sits in the ring (ticket i % 16)
    __shared__ uint32_t s_span[kTickets];                           // and the ring bytes it holds (with wrap waste)
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* gbase = smem_raw + (base - raw);
    const int SX = p.x_slots, SA = p.a_slots, SC = p.acc_slots;
    const uint32_t x_ring = base;                                   // SX slots of b_bytes (1024-aligned)
    const uint32_t ring = x_ring + SX * p.b_bytes;                  // the segment ring
    const uint32_t bars = ring + p.ring_bytes + kRingPad;
    // xfull / xempty: an x tile landed / consumed; sfull / sempty: a segment landed / read by its 8 builder warps;
    // afull / aempty: an A tile written to TMEM by its 8 warps / consumed by the MMAs; accfull / accempty: a row
    // tile's accumulators complete (both issuers) / read out by the 4 epilogue warps; done: every MMA completed.
    auto xfull = [&](int s) { return bars + 8u * s; };
    auto xempty = [&](int s) { return bars + 8u * (kMaxXSlots + s); };
    auto sfull = [&](int s) { return bars + 8u * (2 * kMaxXSlots + s); };
    auto sempty = [&](int s) { return bars + 8u * (2 * kMaxXSlots + kTickets + s); };
    auto afull = [&](int s) { return bars + 8u * (2 * kMaxXSlots + 2 * kTickets + s); };
    auto aempty = [&](int s) { return bars + 8u * (2 * kMaxXSlots + 2 * kTickets + kMaxASlots + s); };
    auto accfull = [&](int s) { return bars + 8u * (2 * kMaxXSlots + 2 * kTickets + 2 * kMaxASlots + s); };
    auto accempty = [&](int s) {
        return bars + 8u * (2 * kMaxXSlots + 2 * kTickets + 2 * kMaxASlots + kMaxAccSlots + s);
    };
    const uint32_t done = bars + 8u * (2 * kMaxXSlots + 2 * kTickets + 2 * kMaxASlots + 2 * kMaxAccSlots);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const WaitCtl wc{&g_mask_error, &g_mask_failed_seq, p.wait_ns, p.seq};
    const int C = p.col_tiles;
    const int64_t u0 = run_start(p, blockIdx.x), u1 = run_end(p, blockIdx.x);
    const int nk = (int)(u1 - u0);                                  // this CTA's units
    const int64_t r0 = u0 / C;                                      // its first row tile
    const int n_rows = nk > 0 ? (int)((u1 - 1) / C - r0 + 1) : 0;   // and how many it touches
    const int tokens = p.tokens, n_total = p.n_total;
    for (int j = threadIdx.x; j <= nk; j += blockDim.x) s_offs[j] = p.seg[u0 + j];

    if (threadIdx.x == 0) {
        const uint32_t consumers = p.by_tile ? 1u : 2u;              // issuers that commit a unit's slots
        for (int s = 0; s < SX; ++s) {
            mbar_init(xfull(s), 1);
            mbar_init(xempty(s), consumers);
        }
        for (int s = 0; s < kTickets; ++s) {
            mbar_init(sfull(s), 1);
            mbar_init(sempty(s), kGroupWarps);
        }
        for (int s = 0; s < SA; ++s) {
            mbar_init(afull(s), kGroupWarps);
            mbar_init(aempty(s), consumers);
        }
        for (int s = 0; s < SC; ++s) {
            mbar_init(accfull(s), 2);
            mbar_init(accempty(s), 4);
        }
        mbar_init(done, 2);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == kXWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // TMEM column of issuer j's accumulator in set s (by_tile: one each; else one, issuer j owning a half of N).
    auto acc_col = [&](int s, int j) {
        return p.by_tile ? (uint32_t)((2 * s + j) * p.acc_cols) : (uint32_t)(s * p.acc_cols);
    };

    if (warp == kSegWarp) {
        // The run's segments, in order, into the byte ring: segment i takes ticket i % 16 and the next free bytes
        // (wrapping to the ring's start when it would not fit before its end). Before reusing bytes or a ticket the
        // thread waits for the oldest segments in flight to be read.
        if (lane == 0) {
            const uint32_t R = (uint32_t)p.ring_bytes;
            uint32_t head = 0, used = 0;
            int tail = 0, issued = 0;
            bool ok = true;
            for (int i = 0; i < nk && ok; ++i) {
                const uint32_t size = (uint32_t)(s_offs[i + 1] - s_offs[i]);
                bool wrap;
                uint32_t waste;
                for (;;) {
                    if (tail == i) {                        // nothing in flight: the whole ring is free
                        head = 0;
                        used = 0;
                    }
                    wrap = head + size > R;                 // (head may sit exactly at R: a wrap with no waste)
                    waste = wrap ? R - head : 0u;
                    if (used + waste + size <= R && i - tail < kTickets) break;
                    ok = mbar_wait(sempty(tail % kTickets), (uint32_t)((tail / kTickets) & 1), 1, wc);
                    if (!ok) break;
                    used -= s_span[tail % kTickets];
                    ++tail;
                }
                if (!ok) break;
                if (wrap) head = 0;
                if (head + size > R || size > (uint32_t)mk::kMaxSegBytes || (size & 15u)) {
                    give_up(10, wc);                        // a layout that does not fit: stop, never copy past the ring
                    break;
                }
                s_span[i % kTickets] = size + waste;
                s_ring_off[i % kTickets] = head;
                used += size + waste;
                mbar_expect_tx(sfull(i % kTickets), size);
                bulk_load(ring + head, p.data + s_offs[i], size, sfull(i % kTickets));
                head += size;
                issued = i + 1;
            }
            // Every segment issued and not yet read must have landed before the CTA may exit.
            for (int j = tail; j < issued; ++j)
                mbar_drain(sfull(j % kTickets), (uint32_t)((j / kTickets) & 1), 7, wc);
        }
        __syncwarp();
    } else if (warp == kXWarp) {
        if (lane == 0) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_x)) : "memory");
        // A programmatic dependent of the stream's previous kernel: x may be its output, so the x loads wait for it
        // (everything else -- barriers, TMEM, the weights streaming in, the first tiles built -- overlaps its tail).
        asm volatile("griddepcontrol.wait;" ::: "memory");
        if (lane < SX) {
            const int s = lane;
            uint32_t ph = 0;
            int uses = 0;
            for (int i = lane; i < nk; i += SX) {
                if (i >= SX) {
                    if (!mbar_wait(xempty(s), ph, 2, wc)) break;
                    ph ^= 1u;
                }
                const int c = (int)((u0 + i) % C);
                mbar_expect_tx(xfull(s), (uint32_t)p.b_bytes);
                for (int b = 0; b < p.n_boxes; ++b)
                    tma_load_2d(x_ring + s * p.b_bytes + b * p.box_rows * 128, &tmap_x, c * mk::kTileCols,
                                b * p.box_rows, xfull(s));
                ++uses;
            }
            if (uses) mbar_drain(xfull(s), (uint32_t)((uses - 1) & 1), 8, wc);
        }
        __syncwarp();
    } else if (warp == kMmaWarp || warp == kMmaWarp + 1) {
        const int j = warp - kMmaWarp;
        if (lane == 0) {
            const bool by_tile = p.by_tile != 0;
            const int n0 = by_tile ? n_total : (n_total / 2 + 15) / 16 * 16;
            const int n_mine = by_tile ? n_total : (j ? n_total - n0 : n0);
            const uint32_t id = idesc_f16<T>(n_mine);
            const uint64_t b0 = sw128_desc(x_ring) + (by_tile ? 0u : (uint64_t)((j * n0 * 128) >> 4));
            const int step = by_tile ? 2 : 1;
            int i = by_tile ? j : 0;                               // this issuer's next unit (local)
            int sa = i % SA, sx = i % SX;
            uint32_t pha = 0, phx = 0;
            bool ok = true;
            for (int k = 0; k < n_rows && ok; ++k) {
                // Row tile r0 + k: its units [ua, ub) of the run, into accumulator set k % SC once the epilogue has
                // read that set's previous row tile out.
                const int ub = (int)(min(u1, (r0 + k + 1) * C) - u0);
                const int sc = k % SC;
                if (k >= SC && !(ok = mbar_wait(accempty(sc), (uint32_t)(((k / SC) - 1) & 1), 11, wc))) break;
                tc_fence_after();
                const uint32_t d = tmem + acc_col(sc, j) + (by_tile ? 0u : (uint32_t)(j * n0));
                uint32_t acc = 0;
                for (; i < ub; i += step) {
                    if (!(ok = mbar_wait(afull(sa), pha, 3, wc))) break;       // no MMA on a tile not there
                    if (!(ok = mbar_wait(xfull(sx), phx, 4, wc))) break;
                    tc_fence_after();
                    const uint32_t a = tmem + (uint32_t)(p.a_col0 + sa * kACols);
                    const uint64_t bd = b0 + (uint64_t)((sx * p.b_bytes) >> 4);
#pragma unroll
                    for (int kk = 0; kk < mk::kTileCols / 16; ++kk)
                        umma_f16_ts(d, a + 8u * kk, bd + 2 * kk, id, acc | kk);    // K = 16: 8 TMEM columns
                    acc = 1u;
                    umma_commit(aempty(sa));
                    umma_commit(xempty(sx));
                    advance(sa, pha, step, SA);
                    advance(sx, phx, step, SX);
                }
                if (ok) umma_commit(accfull(sc));           // the row tile's MMAs of this issuer, once complete
            }
            umma_commit(done);                              // arrives once every MMA this thread issued completed
        }
        __syncwarp();
    } else if (warp >= kEpiWarp) {
        // Epilogue of persistent runs: row tile after row tile, D out of TMEM (lanes 32 e .. + 31: rows 32 e + lane
        // of the tile), overlapping the next row tile's MMAs. (Aligned runs hold one row tile: all warps drain it at
        // the end, below.)
        const int e = warp & 3;
        const int row_local = 32 * e + lane;
        for (int k = 0; k < (p.splits == 0 ? n_rows : 0); ++k) {
            const int64_t r = r0 + k;
            const int sc = k % SC;
            const int ok = lane == 0 ? mbar_wait(accfull(sc), (uint32_t)((k / SC) & 1), 12, wc) : 1;
            if (!epilogue_all(ok)) break;                           // the four warps stop together
            tc_fence_after();
            const int64_t ua = max(u0, r * C), ub = min(u1, (r + 1) * C);
            const bool whole = ua == r * C && ub == (r + 1) * C;   // no other CTA holds units of this row tile
            // by_tile: the issuer of the row tile's first unit, and the other too when it holds two or more.
            const int j_first = p.by_tile ? (int)((ua - u0) & 1) : 0;
            const bool both = p.by_tile && ub - ua >= 2;
            const int which = k == 0 ? 0 : 1;                    // a shared row tile is this run's first or last
            const int64_t row = r * mk::kTileRows + row_local;
            float* part = p.partial + ((int64_t)blockIdx.x * 2 + which) * tokens * mk::kTileRows;
            for (int c = 0; c < n_total / 16; ++c) {
                float v[16];
                const uint32_t ta = tmem + ((uint32_t)(32 * e) << 16) + (uint32_t)(c * 16);
                tmem_ld16(ta + acc_col(sc, j_first), v);
                if (both) {
                    float w2[16];
                    tmem_ld16(ta + acc_col(sc, j_first ^ 1), w2);
#pragma unroll
                    for (int q = 0; q < 16; ++q) v[q] += w2[q];
                }
#pragma unroll
                for (int q = 0; q < 16; ++q) {
                    const int t = c * 16 + q;
                    if (t < tokens) {
                        if (whole) {
                            if (row < p.rows) store_y<T>(p, t, row, v[q]);
                        } else if (p.cluster) {
                            reinterpret_cast<float*>(gbase)[t * mk::kTileRows + row_local] = v[q];   // rings free
                        } else {
                            part[t * mk::kTileRows + row_local] = v[q];
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(accempty(sc));               // the set may take the next row tile
            if (!whole && !p.cluster) {
                // The last CTA of the row tile to leave its partial adds them all, CTA by CTA: at once (persistent
                // runs, small partials) or, for aligned runs (one row tile a CTA), after the pipeline has drained,
                // with all of the CTA's threads.
                __threadfence();
                asm volatile("bar.sync 1, 128;" ::: "memory");
                if (e == 0 && lane == 0) {
                    const int64_t b_first = run_of(p, r * C);
                    const int64_t b_last = run_of(p, (r + 1) * C - 1);
                    s_last = atomicAdd(&p.tickets[r], 1u) == (unsigned)(b_last - b_first);
                }
                asm volatile("bar.sync 1, 128;" ::: "memory");
                if (s_last && p.splits == 0) {
                    __threadfence();
                    const int64_t b_first = run_of(p, r * C);
                    const int64_t b_last = run_of(p, (r + 1) * C - 1);
                    // Contributor b's partial of this row tile: its run's last row tile for b_first (unless the run
                    // starts in it), its first for the others. Units of (token, 4 rows), float4 loads, four
                    // contributors' loads in flight at a time; the sums still go contributor by contributor.
                    const int wb_first = run_start(p, b_first) / C == r ? 0 : 1;
                    auto part_of = [&](int64_t b) {
                        return p.partial + (b * 2 + (b == b_first ? wb_first : 0)) * tokens * mk::kTileRows;
                    };
                    const int et = 32 * e + lane;                        // 0..127
                    for (int u = et; u < tokens * 32; u += 128) {
                        const int t = u >> 5, r4 = (u & 31) * 4;
                        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                        for (int64_t b = b_first; b <= b_last; b += 4) {
                            float4 v[4];
#pragma unroll
                            for (int q = 0; q < 4; ++q)
                                if (b + q <= b_last)
                                    v[q] = __ldcg(reinterpret_cast<const float4*>(part_of(b + q) + t * mk::kTileRows + r4));
#pragma unroll
                            for (int q = 0; q < 4; ++q)
                                if (b + q <= b_last) {
                                    acc.x += v[q].x; acc.y += v[q].y; acc.z += v[q].z; acc.w += v[q].w;
                                }
                        }
                        const int64_t row4 = r * mk::kTileRows + r4;
                        const float vv[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
                        for (int c = 0; c < 4; ++c)
                            if (row4 + c < p.rows) store_y<T>(p, t, row4 + c, vv[c]);
                    }
                    if (e == 0 && lane == 0) p.tickets[r] = 0u;     // zero again for the next call
                }
                asm volatile("bar.sync 1, 128;" ::: "memory");
            }
        }
    } else {
        // Builders: warp w of group grp writes block blk (rows 16 blk .. + 15) of each of the group's tiles.
        const int grp = warp / kGroupWarps, wb = warp % kGroupWarps;
        const int blk = 2 * (wb & 3) + (wb >> 2);                 // (w % 4) == blk / 2: the lanes this warp may write
        const int g = lane >> 2;
        const uint32_t q = 8u * (g & 3) + 2u * (lane & 3);        // this lane's first bit in its 32-bit mask word
        const uint32_t below = (1u << q) - 1u;
        // Rows 0..3 of a piece (g < 4) read the lo words and offsets, rows 4..7 the hi ones.
        const uint32_t words_at = (uint32_t)(mk::kHeaderBytes + mk::kBlockBytes * blk + (g >= 4 ? mk::kHiAt : 0));
        const uint32_t offs_at = (uint32_t)(mk::kHeaderBytes + mk::kBlockBytes * blk + (g >= 4 ? mk::kOhiAt : mk::kOloAt));
        const uint32_t t_lanes = (uint32_t)(16 * blk) << 16;
        int ticket = grp, sa = grp % SA;
        uint32_t tph = 0, aph = 0;
        for (int i = grp; i < nk; i += kGroups) {
            // Every lane observes the segment's barrier (the bulk copy's bytes are then visible to its reads); lane 0
            // also waits until the MMAs are done with the A slot.
            int ok = mbar_wait(sfull(ticket), tph, 5, wc);
            if (ok && lane == 0 && i >= SA) ok = mbar_wait(aempty(sa), aph ^ 1u, 6, wc);
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();                                           // TMEM stores after the MMAs' reads
            const uint32_t segp = ring + s_ring_off[ticket];
            const uint32_t vals = segp + (uint32_t)mk::kValuesAt;
            uint32_t w[16], o[8];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint4 v = lds_v4(segp + words_at + 16u * k);    // two addresses a warp: broadcasts
                w[4 * k] = v.x; w[4 * k + 1] = v.y; w[4 * k + 2] = v.z; w[4 * k + 3] = v.w;
            }
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const uint4 v = lds_v4(segp + offs_at + 16u * k);
                o[4 * k] = v.x; o[4 * k + 1] = v.y; o[4 * k + 2] = v.z; o[4 * k + 3] = v.w;
            }
            uint32_t r[16];
#pragma unroll
            for (int pp = 0; pp < 16; ++pp) {
                const uint32_t start = (pp & 1) ? (o[pp >> 1] >> 16) : (o[pp >> 1] & 0xffffu);   // bytes
                const uint32_t a0 = vals + start + 2u * __popc(w[pp] & below);   // this lane's first value
                const uint32_t x = w[pp] >> q;
                const uint32_t b0 = x & 1u;                             // its two weights kept? (bits 0, 1 of x)
                const uint32_t va = lds_u16(a0);
                const uint32_t vn = lds_u16(a0 + 2u * b0);              // the next value if the first is kept
                r[pp] = va * b0 + vn * ((x & 2u) << 15);                // (va if kept) | (vn if kept) << 16
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(sempty(ticket));                 // this warp is done with the segment
            tmem_st_16x256b_x4(tmem + t_lanes + (uint32_t)(p.a_col0 + sa * kACols), r);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(afull(sa));
            advance(ticket, tph, kGroups, kTickets);
            advance(sa, aph, kGroups, SA);
        }

    }

    tc_fence_before();
    __syncthreads();
    const bool aligned = p.splits > 0 && nk > 0;
    const int64_t rt = r0;
    const int split = p.splits > 0 ? (int)(blockIdx.x % p.splits) : 0;
    const int ns = p.splits;
    if (aligned) {
        // The run's one row tile, drained by every warp once both issuers' MMAs completed: warp w reads TMEM lanes
        // 32 (w % 4) .. + 31 and every sixth 16-column chunk from chunk w / 4.
        const int ok = lane == 0 ? mbar_wait(accfull(0), 0, 12, wc) : 1;
        __syncwarp();
        tc_fence_after();
        const int quarter = warp & 3, gid = warp >> 2, n_gid = kThreads / 128;
        const int row_local = quarter * 32 + lane;
        const int64_t row = rt * mk::kTileRows + row_local;
        const bool both = p.by_tile && nk >= 2;
        float* part = p.partial + (int64_t)blockIdx.x * 2 * tokens * mk::kTileRows;
        for (int c = gid; c < n_total / 16 && __shfl_sync(0xffffffffu, ok, 0); c += n_gid) {
            float v[16];
            const uint32_t ta = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(c * 16);
            tmem_ld16(ta + acc_col(0, 0), v);
            if (both) {
                float w2[16];
                tmem_ld16(ta + acc_col(0, 1), w2);
#pragma unroll
                for (int q = 0; q < 16; ++q) v[q] += w2[q];
            }
#pragma unroll
            for (int q = 0; q < 16; ++q) {
                const int t = c * 16 + q;
                if (t < tokens) {
                    if (ns == 1) {
                        if (row < p.rows) store_y<T>(p, t, row, v[q]);
                    } else if (p.cluster) {
                        reinterpret_cast<float*>(gbase)[t * mk::kTileRows + row_local] = v[q];   // rings free
                    } else {
                        part[t * mk::kTileRows + row_local] = v[q];
                    }
                }
            }
        }
        tc_fence_before();
        if (ns > 1 && !p.cluster) __threadfence();
        __syncthreads();
    }
    if (warp == kXWarp) {
        if (lane == 0) mbar_drain(done, 0, 9, wc);                  // no MMA may still write TMEM
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
    if (!aligned || ns <= 1) return;
    if (p.cluster) {
        // Every split's partial tile is in its CTA's shared memory; CTA `split` of the cluster adds up its share of the
        // tile's (token, 4-row) units, split by split, and writes y. The second barrier keeps each CTA's shared memory
        // alive until every CTA of the cluster has read it.
        cluster_sync_all();
        const int64_t n4 = (int64_t)tokens * (mk::kTileRows / 4);
        const int64_t u_begin = n4 * split / ns, u_end = n4 * (split + 1) / ns;
        const uint32_t partial = smem_u32(gbase);
        for (int64_t u = u_begin + threadIdx.x; u < u_end; u += kThreads) {
            const int t = (int)(u / 32), r4 = (int)(u % 32) * 4;
            const uint32_t off = partial + (uint32_t)(t * mk::kTileRows + r4) * 4u;
            float4 parts[8];
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int sp = 0; sp < 8; ++sp)
                if (sp < ns) parts[sp] = ld_cluster_f4(cluster_addr(off, sp));
#pragma unroll
            for (int sp = 0; sp < 8; ++sp)
                if (sp < ns) {
                    acc.x += parts[sp].x; acc.y += parts[sp].y; acc.z += parts[sp].z; acc.w += parts[sp].w;
                }
            const int64_t row = rt * mk::kTileRows + r4;
            const float v[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
            for (int c = 0; c < 4; ++c)
                if (row + c < p.rows) store_y<T>(p, t, row + c, v[c]);
        }
        cluster_sync_all();
        return;
    }
    // Splits meeting in the workspace: the last of the row tile's CTAs to finish adds the partials of all ns splits,
    // split by split, every thread on (token, 4-row) units, a pair of splits' loads in flight at a time.
    if (threadIdx.x == 0) s_last = atomicAdd(&p.tickets[rt], 1u) == (unsigned)(ns - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const int64_t b0 = rt * ns;
    const int64_t n4 = (int64_t)tokens * (mk::kTileRows / 4);
    const int64_t stride = (int64_t)2 * tokens * mk::kTileRows;
    for (int64_t u = threadIdx.x; u < n4; u += kThreads) {
        const int t = (int)(u / 32), r4 = (int)(u % 32) * 4;
        const float* base_p = p.partial + b0 * stride + (int64_t)t * mk::kTileRows + r4;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        int sp = 0;
        for (; sp + 1 < ns; sp += 2) {
            const float4 a = __ldcg(reinterpret_cast<const float4*>(base_p + sp * stride));
            const float4 b = __ldcg(reinterpret_cast<const float4*>(base_p + (sp + 1) * stride));
            acc.x += a.x; acc.y += a.y; acc.z += a.z; acc.w += a.w;
            acc.x += b.x; acc.y += b.y; acc.z += b.z; acc.w += b.w;
        }
        if (sp < ns) {
            const float4 a = __ldcg(reinterpret_cast<const float4*>(base_p + sp * stride));
            acc.x += a.x; acc.y += a.y; acc.z += a.z; acc.w += a.w;
        }
        const int64_t row = rt * mk::kTileRows + r4;
        const float v[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
        for (int c = 0; c < 4; ++c)
            if (row + c < p.rows) store_y<T>(p, t, row + c, v[c]);
    }
    if (threadIdx.x == 0) p.tickets[rt] = 0u;             // zero again for the next call
}

struct MaskPlan {
    int n_total, box_rows, n_boxes, by_tile, acc_cols, acc_slots, a_col0, a_slots, x_slots, b_bytes, ring_bytes, smem;
};

// Token-dependent part of a launch plan: MMA N, accumulators and A slots in TMEM, x boxes, the rings.
int plan_tokens(int tn, MaskPlan& pl) {
    if (tn < 1 || tn > kMaxN) return fail(P2P_EINVAL, "p2p_spmm_mask: %d tokens in one launch", tn);
    const int bar_bytes = 8 * (2 * kMaxXSlots + 2 * kTickets + 2 * kMaxASlots + 2 * kMaxAccSlots + 1);
    const int fixed = 1024 + kRingPad + bar_bytes + 16;
    pl.n_total = (tn + 15) / 16 * 16;
    pl.n_boxes = pl.n_total <= 256 ? 1 : 2;
    pl.box_rows = pl.n_total / pl.n_boxes;
    pl.by_tile = pl.n_total <= 128;
    pl.acc_cols = pl.by_tile ? pow2_at_least(pl.n_total) : pl.n_total;
    pl.acc_slots = pl.n_total <= 64 ? 2 : 1;
    const int acc_total = pl.acc_slots * (pl.by_tile ? 2 : 1) * pl.acc_cols;
    pl.a_col0 = (acc_total + kACols - 1) / kACols * kACols;
    pl.a_slots = (kTmemCols - pl.a_col0) / kACols;
    if (pl.a_slots > kMaxASlots) pl.a_slots = kMaxASlots;
    if (pl.by_tile) pl.a_slots &= ~1;                 // even: each issuer's units keep to its own slots
    pl.b_bytes = pl.n_total * 128;
    // Four x slots (even when the issuers split the units), three only when four would leave the segment ring under
    // two of the largest segments.
    pl.x_slots = 4;
    if (!pl.by_tile && kSmemLimit - fixed - 4 * pl.b_bytes < 2 * mk::kMaxSegBytes) pl.x_slots = 3;
    pl.ring_bytes = (kSmemLimit - fixed - pl.x_slots * pl.b_bytes) / 16 * 16;
    if (pl.a_slots < 2 || pl.ring_bytes < mk::kMaxSegBytes)
        return fail(P2P_EUNSUPPORTED, "p2p_spmm_mask: %d tokens do not fit one launch", tn);
    pl.smem = fixed + pl.x_slots * pl.b_bytes + pl.ring_bytes;
    return P2P_OK;
}

// The persistent grid: one CTA an SM, more only when a run would pass kMaxUnits units.
int grid_of(int64_t units) {
    int64_t g = sm_count();
    if (g > units) g = units;
    const int64_t need = (units + kMaxUnits - 1) / kMaxUnits;
    if (g < need) g = need;
    return (int)(g < 1 ? 1 : g);
}

// Aligned runs: columns split so that the row tiles fill the SMs -- the fewest waves of CTAs a column tile's work,
// plus a CTA's fixed cost (fill, TMEM, the epilogue: about 10 tiles' time) and the cost of adding partial tiles.
void plan_split(int64_t row_tiles, int col_tiles, int tokens, int sms, int* n_split, int* per) {
    int best = 1;
    double best_cost = 1e30;
    const int max_split = col_tiles < 32 ? col_tiles : 32;
    for (int s = 1; s <= max_split; ++s) {
        const int k = (col_tiles + s - 1) / s;
        if ((s - 1) * k >= col_tiles) continue;
        const double waves = (double)((row_tiles * s + sms - 1) / sms);
        double cost = waves * (k + 10.0);
        if (s > 1) cost += (double)s * tokens * row_tiles / 12.0 / sms;
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = s;
        }
    }
    int k = (col_tiles + best - 1) / best;
    if (k > kMaxUnits) k = kMaxUnits;
    *per = k;
    *n_split = (col_tiles + k - 1) / k;
}

// Clusters of n CTAs of this shared-memory size the device holds at once (cached per device and shape).
int max_clusters(int smem, int n) {
    static std::mutex mu;
    static std::map<std::pair<int, int>, int> known;
    std::lock_guard<std::mutex> lock(mu);
    int dev = 0;
    cudaGetDevice(&dev);
    const auto key = std::make_pair(n * 64 + dev, smem);
    auto it = known.find(key);
    if (it != known.end()) return it->second;
    int clusters = 0;
    if (allow_smem((const void*)spmm_mask_kernel<__nv_bfloat16>, smem, "p2p_spmm_mask") == P2P_OK &&
        allow_smem((const void*)spmm_mask_kernel<__half>, smem, "p2p_spmm_mask") == P2P_OK) {
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = n;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.gridDim = dim3(n);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&clusters, spmm_mask_kernel<__nv_bfloat16>, &cfg) != cudaSuccess)
            clusters = 0;
        cudaGetLastError();                               // a refusal only means: no cluster reduction
    }
    known[key] = clusters;
    return clusters;
}

// The runs of one launch: persistent (splits = 0) for few tokens on modules with at least half an SM's worth of row
// tiles each, where partial tiles are small and whole waves matter; otherwise aligned runs, reduced in clusters when
// 2..8 splits' partial tiles fit the rings and the clusters fit the waves the plain grid takes.
void plan_runs(int64_t row_tiles, int col_tiles, int tokens, const MaskPlan& pl, int* splits, int* per, int* cluster,
               int* ctas) {
    const int sms = sm_count();
    *cluster = 0;
    if (tokens <= 64 && row_tiles * 2 >= sms) {
        *splits = 0;
        *per = 0;
        *ctas = grid_of(row_tiles * col_tiles);
        return;
    }
    plan_split(row_tiles, col_tiles, tokens, sms, splits, per);
    *ctas = (int)(row_tiles * *splits);
    if (*splits >= 2 && *splits <= 8 &&
        (int64_t)pl.n_total * mk::kTileRows * 4 <= (int64_t)pl.x_slots * pl.b_bytes + pl.ring_bytes) {
        const int resident = max_clusters(pl.smem, *splits);
        if (resident > 0) {
            const int64_t plain_waves = (row_tiles * *splits + sms - 1) / sms;
            const int64_t cluster_waves = (row_tiles + resident - 1) / resident;
            *cluster = cluster_waves <= plain_waves ? 1 : 0;
        }
    }
}

unsigned next_seq() {
    static std::atomic<unsigned> counter{0};
    unsigned v = ++counter;
    while (v == 0) v = ++counter;
    return v;
}

// The launches of one call: tokens in chunks of at most kMaxN, as even as they divide.
int chunk_tokens(int64_t tokens) {
    const int64_t n = (tokens + kMaxN - 1) / kMaxN;
    return (int)((tokens + n - 1) / n);
}

template <typename T>
int launch_mask(const CUtensorMap& map, const MaskParams& prm, int smem, cudaStream_t st) {
    auto kernel = spmm_mask_kernel<T>;
    if (int e = allow_smem((const void*)kernel, smem, "p2p_spmm_mask")) return e;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;           // the splits of a row tile as one cluster
    attr[1].val.clusterDim.x = prm.splits;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.gridDim = dim3((unsigned)prm.ctas);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = prm.cluster ? 2 : 1;
    cudaLaunchKernelEx(&cfg, kernel, map, prm);
    return launch_status("p2p_spmm_mask");
}

}  // namespace
}  // namespace p2p

using namespace p2p;

extern "C" size_t p2p_spmm_mask_workspace(int64_t rows, int64_t cols, int64_t tokens) {
    if (rows <= 0 || cols <= 0 || tokens <= 0) return 0;
    const int64_t row_tiles = (rows + mk::kTileRows - 1) / mk::kTileRows;
    const int col_tiles = (int)((cols + mk::kTileCols - 1) / mk::kTileCols);
    const int chunk = chunk_tokens(tokens);
    const int sizes[2] = {(int)(tokens < chunk ? tokens : chunk), (int)(tokens % chunk)};
    size_t need = kTicketRegion;
    for (int t : sizes) {
        MaskPlan pl;
        if (t <= 0 || plan_tokens(t, pl) != P2P_OK) continue;
        int splits, per, cluster, ctas;
        plan_runs(row_tiles, col_tiles, t, pl, &splits, &per, &cluster, &ctas);
        const size_t w = kTicketRegion + (size_t)ctas * 2 * t * mk::kTileRows * sizeof(float);
        need = need > w ? need : w;
    }
    return need;
}

namespace {
int spmm_mask_impl(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ldx, const void* data,
                   const int64_t* seg, int64_t rows, void* const* ys, int n_ys, int64_t y_col0, int64_t ldy,
                   void* workspace, size_t workspace_bytes, void* stream) {
    P2P_REQUIRE(tokens >= 0 && rows >= 0 && cols >= 1, "p2p_spmm_mask: bad shape");
    if (tokens == 0 || rows == 0) return P2P_OK;
    if (dtype != P2P_BF16 && dtype != P2P_F16) return fail(P2P_EUNSUPPORTED, "p2p_spmm_mask: bf16 or f16");
    P2P_REQUIRE(x && data && seg && ys && n_ys >= 1 && n_ys <= kMaxPeers, "p2p_spmm_mask: null pointer or %d outputs",
                n_ys);
    for (int k = 0; k < n_ys; ++k) P2P_REQUIRE(ys[k], "p2p_spmm_mask: null output %d", k);
    P2P_REQUIRE(aligned16(data), "p2p_spmm_mask: the layout must start on a 16-byte boundary");
    P2P_REQUIRE(cols % 8 == 0 && ldx % 8 == 0 && ldx >= cols && aligned16(x),
                "p2p_spmm_mask: x needs 16-byte aligned rows (cols and ldx multiples of 8)");
    P2P_REQUIRE(y_col0 >= 0 && ldy >= y_col0 + rows, "p2p_spmm_mask: ldy %lld below columns %lld + %lld",
                (long long)ldy, (long long)y_col0, (long long)rows);
    P2P_REQUIRE(rows <= 0x7fffffff && cols <= 0x7fffffff, "p2p_spmm_mask: too large");
    const int64_t row_tiles = (rows + mk::kTileRows - 1) / mk::kTileRows;
    const int col_tiles = (int)((cols + mk::kTileCols - 1) / mk::kTileCols);
    if (row_tiles > kMaxRowTiles) return fail(P2P_EUNSUPPORTED, "p2p_spmm_mask: %lld rows", (long long)rows);
    P2P_REQUIRE(workspace && workspace_bytes >= p2p_spmm_mask_workspace(rows, cols, tokens),
                "p2p_spmm_mask: workspace of %zu bytes, %zu needed", workspace_bytes,
                p2p_spmm_mask_workspace(rows, cols, tokens));
    cudaStream_t st = as_stream(stream);
    const int chunk = chunk_tokens(tokens);
    for (int64_t t0 = 0; t0 < tokens; t0 += chunk) {
        const int tn = (int)(tokens - t0 < chunk ? tokens - t0 : chunk);
        MaskPlan pl;
        if (int e = plan_tokens(tn, pl)) return e;
        MaskParams prm;
        prm.data = reinterpret_cast<const uint8_t*>(data);
        prm.seg = seg;
        prm.rows = (int)rows;
        prm.col_tiles = col_tiles;
        prm.tokens = tn;
        prm.n_total = pl.n_total;
        prm.box_rows = pl.box_rows;
        prm.n_boxes = pl.n_boxes;
        prm.by_tile = pl.by_tile;
        prm.acc_cols = pl.acc_cols;
        prm.acc_slots = pl.acc_slots;
        prm.a_col0 = pl.a_col0;
        prm.a_slots = pl.a_slots;
        prm.x_slots = pl.x_slots;
        prm.b_bytes = pl.b_bytes;
        prm.ring_bytes = pl.ring_bytes;
        prm.units = row_tiles * col_tiles;
        plan_runs(row_tiles, col_tiles, tn, pl, &prm.splits, &prm.per_split, &prm.cluster, &prm.ctas);
        for (int k = 0; k < kMaxPeers; ++k)
            prm.ys[k] = k < n_ys ? reinterpret_cast<char*>(ys[k]) + t0 * ldy * 2 : nullptr;
        prm.n_ys = n_ys;
        prm.y_col0 = y_col0;
        prm.ldy = ldy;
        prm.tickets = reinterpret_cast<unsigned*>(workspace);
        prm.partial = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + kTicketRegion);
        prm.wait_ns = kWaitNs;
        prm.seq = next_seq();
        CUtensorMap map;
        const void* xt = reinterpret_cast<const char*>(x) + t0 * ldx * 2;
        if (int e = encode_x_map(&map, xt, dtype, tn, cols, ldx, pl.box_rows)) return e;
        if (int e = dtype == P2P_BF16 ? launch_mask<__nv_bfloat16>(map, prm, pl.smem, st)
                                      : launch_mask<__half>(map, prm, pl.smem, st))
            return e;
    }
    return P2P_OK;
}
}  // namespace

extern "C" int p2p_spmm_mask(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ldx, const void* data,
                             const int64_t* seg, int64_t rows, void* y, int64_t ldy, void* workspace,
                             size_t workspace_bytes, void* stream) {
    void* ys[1] = {y};
    return spmm_mask_impl(x, dtype, tokens, cols, ldx, data, seg, rows, ys, 1, 0, ldy, workspace, workspace_bytes,
                          stream);
}

extern "C" int p2p_spmm_mask_peers(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ldx,
                                   const void* data, const int64_t* seg, int64_t rows, void* const* ys, int n_ys,
                                   int64_t y_col0, int64_t ldy, void* workspace, size_t workspace_bytes,
                                   void* stream) {
    return spmm_mask_impl(x, dtype, tokens, cols, ldx, data, seg, rows, ys, n_ys, y_col0, ldy, workspace,
                          workspace_bytes, stream);
}

extern "C" int p2p_spmm_mask_status(int reset, void* stream) {
    cudaStream_t st = as_stream(stream);
    int v = 0;
    if (cudaMemcpyFromSymbolAsync(&v, g_mask_error, sizeof(int), 0, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return fail(P2P_ECUDA, "p2p_spmm_mask_status: %s", cudaGetErrorString(cudaGetLastError()));
    if (reset && v) {
        const int zero = 0;
        cudaMemcpyToSymbolAsync(g_mask_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
        cudaStreamSynchronize(st);
    }
    if (v) return fail(P2P_ECUDA, "p2p_spmm_mask: a pipeline wait timed out (site %d)", v);
    return P2P_OK;
}
