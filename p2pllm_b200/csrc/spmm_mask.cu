// (2c) The compact sparse GEMM on the bitmask layout of mask_layout.cuh: y[t, r] = sum_c W[r, c] x[t, c] for bf16 /
// f16 weights stored as the reference stores them (the kept values, 2 bytes each, plus one bit a weight), on tcgen05
// tensor cores with the weight tile in tensor memory.
//
// Replaces p2p/compact.cu:82-278 (spmm_kernel, sum_parts, spmm), whose warps build mma.sync fragments from 8 x 8 mask
// pieces and re-read every weight once per 64 tokens. Here a CTA owns one 128-row tile and a range of 64-column tiles
// (split-K), and every token of the launch (up to 288) at once:
//
//   warp 17 (segments)  one thread streams the CTA's segments (header, masks, values: ~6.5 KB a tile at keep 33-36)
//                       into a byte ring in shared memory with bulk copies, up to 16 segments ahead: the bytes in
//                       flight that keep HBM busy, with no registers held for them.
//   warp 16 (x)         TMA of the x tile [tokens x 64] (128-byte swizzle) into the x ring, one lane a slot.
//   warps 0-15 (build)  two groups of 8 warps take alternate tiles. Warp w builds 16-row block 2 (w % 4) + (w % 8) / 4
//                       of its group's tile (the block's rows are TMEM lanes warp w may write): each lane turns its two
//                       bits of each of the block's 16 pieces, with the piece's values read from the ring, into a
//                       register of two bf16 weights, and one tcgen05.st.16x256b.x4 writes the block into the tile's A
//                       slot in tensor memory. A piece's values lie within 128 bytes, so a warp's reads never clash on
//                       a bank; there is no zeroing pass, no scattered store and no A tile in shared memory.
//   warps 18-19 (MMA)   one elected thread each issues tcgen05.mma kind::f16 with A from tensor memory (M = 128,
//                       K = 16 a step) and B = the x tile (N = tokens rounded to 16), fp32 accumulators in TMEM: with
//                       N <= 128 the issuers take alternate tiles into accumulators of their own (two MMA streams run
//                       side by side), above that both take every tile, each half of N.
//   warps 0-15 (epilogue) tcgen05.ld D, round, and write y: directly, through TMA stores, or reducing the column
//                       splits in a thread-block cluster over DSMEM or through fp32 partials and a ticket per row tile
//                       (split order either way, so results do not depend on scheduling).
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
constexpr int kGroups = 2;                             // groups taking alternate tiles
constexpr int kBuildWarps = kGroupWarps * kGroups;
constexpr int kXWarp = kBuildWarps;                    // 16: x tiles
constexpr int kSegWarp = kBuildWarps + 1;              // 17: segments
constexpr int kMmaWarp = kBuildWarps + 2;              // 18 and 19: MMA issuers
constexpr int kThreads = (kBuildWarps + 4) * 32;       // 640
constexpr int kTickets = 16;                           // segments in flight
constexpr int kMaxXSlots = 4;
constexpr int kMaxASlots = 14;                         // A tiles in tensor memory
constexpr int kACols = 32;                             // TMEM columns of one A tile (128 x 64 16-bit weights)
constexpr int kTmemCols = 512;
constexpr int kMaxN = 288;                             // tokens a launch (accumulator + A slots fit 512 columns)
constexpr int kMaxTilesPerCta = 256;
constexpr int kRingPad = 64;                           // slack past the ring: reads of a piece may run 2 bytes past it
constexpr int kSmemLimit = 227 * 1024 - (int)sizeof(int64_t) * (kMaxTilesPerCta + 1) - 8 * kTickets - 64;
constexpr uint64_t kWaitNs = 2000000000ull;
constexpr int64_t kMaxRowTiles = 16384;
constexpr size_t kTicketRegion = kMaxRowTiles * sizeof(unsigned);

__device__ int g_mask_error;            // site of the first wait that gave up since the last reset (0: none)
__device__ unsigned g_mask_failed_seq;  // sequence number of the last launch in which a wait gave up

struct MaskParams {
    const uint8_t* data;              // the module's segments
    const int64_t* seg;               // [row_tiles * col_tiles + 1] byte offsets
    int rows, col_tiles, tokens, n_total, box_rows, n_boxes;
    int by_tile;                      // 1: issuer j takes tiles j, j + 2, .. into its own accumulator (N <= 128)
    int acc_stride;                   // TMEM columns between the two accumulators (by_tile)
    int a_col0;                       // first TMEM column of the A slots
    int a_slots, x_slots, b_bytes, ring_bytes, kt_per_split, n_split;
    void* y;
    int64_t ldy;
    float* partial;                   // [n_split, tokens, rows_pad] when the splits meet in the workspace
    unsigned* tickets;                // [row_tiles]
    int64_t rows_pad;
    int cluster;                      // the splits of a row tile run as one cluster and add over DSMEM
    int y_tma;                        // unsplit: y leaves through shared memory and TMA stores
    uint64_t wait_ns;
    unsigned seq;
};

__device__ __forceinline__ uint32_t bfe_s(uint32_t v, uint32_t pos) {       // bit pos of v as 0 or 0xffffffff
    uint32_t r;
    asm("bfe.s32 %0, %1, %2, 1;" : "=r"(r) : "r"(v), "r"(pos));
    return r;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    spmm_mask_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_y,
                     MaskParams p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint32_t s_tmem;
    __shared__ int s_last;
    __shared__ int64_t s_offs[kMaxTilesPerCta + 1];                // this CTA's segment offsets (bytes)
    __shared__ uint32_t s_ring_off[kTickets];                       // where segment i sits in the ring (ticket i % 16)
    __shared__ uint32_t s_span[kTickets];                           // and the ring bytes it holds (with wrap waste)
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* gbase = smem_raw + (base - raw);
    const int SX = p.x_slots, SA = p.a_slots;
    const uint32_t x_ring = base;                                   // SX slots of b_bytes (1024-aligned)
    const uint32_t ring = x_ring + SX * p.b_bytes;                  // the segment ring
    const uint32_t bars = ring + p.ring_bytes + kRingPad;
    // xfull / xempty: an x tile landed / consumed; sfull / sempty: a segment landed / read by its 8 builder warps;
    // afull / aempty: an A tile written to TMEM by its 8 warps / consumed by the MMAs.
    auto xfull = [&](int s) { return bars + 8u * s; };
    auto xempty = [&](int s) { return bars + 8u * (kMaxXSlots + s); };
    auto sfull = [&](int s) { return bars + 8u * (2 * kMaxXSlots + s); };
    auto sempty = [&](int s) { return bars + 8u * (2 * kMaxXSlots + kTickets + s); };
    auto afull = [&](int s) { return bars + 8u * (2 * kMaxXSlots + 2 * kTickets + s); };
    auto aempty = [&](int s) { return bars + 8u * (2 * kMaxXSlots + 2 * kTickets + kMaxASlots + s); };
    const uint32_t done = bars + 8u * (2 * kMaxXSlots + 2 * kTickets + 2 * kMaxASlots);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const WaitCtl wc{&g_mask_error, &g_mask_failed_seq, p.wait_ns, p.seq};
    const int rt = blockIdx.x, split = blockIdx.y;
    const int tokens = p.tokens, n_total = p.n_total;
    const int64_t col0 = (int64_t)rt * mk::kTileRows;               // y's first column: the tile's first row
    const int kt0 = split * p.kt_per_split;
    const int kt1 = min(p.col_tiles, kt0 + p.kt_per_split);
    const int nk = kt1 - kt0;
    const int64_t seg0 = (int64_t)rt * p.col_tiles + kt0;
    for (int j = threadIdx.x; j <= nk; j += blockDim.x) s_offs[j] = p.seg[seg0 + j];

    if (threadIdx.x == 0) {
        const uint32_t consumers = p.by_tile ? 1u : 2u;              // issuers that commit a tile's slots
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

    if (warp == kSegWarp) {
        // The segments, in order, into the byte ring: segment i takes ticket i % 16 and the next free bytes (wrapping
        // to the ring's start when it would not fit before its end). Before reusing bytes or a ticket the thread waits
        // for the oldest segments in flight to be read.
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
                mbar_expect_tx(xfull(s), (uint32_t)p.b_bytes);
                for (int b = 0; b < p.n_boxes; ++b)
                    tma_load_2d(x_ring + s * p.b_bytes + b * p.box_rows * 128, &tmap_x, (kt0 + i) * mk::kTileCols,
                                b * p.box_rows, xfull(s));
                ++uses;
            }
            if (uses) mbar_drain(xfull(s), (uint32_t)((uses - 1) & 1), 8, wc);
        }
        __syncwarp();
    } else if (warp >= kMmaWarp) {
        const int j = warp - kMmaWarp;
        if (lane == 0) {
            const bool by_tile = p.by_tile != 0;
            const int n0 = by_tile ? n_total : (n_total / 2 + 15) / 16 * 16;
            const int n_mine = by_tile ? n_total : (j ? n_total - n0 : n0);
            const uint32_t id = idesc_f16<T>(n_mine);
            const uint32_t d = tmem + (by_tile ? (uint32_t)(j * p.acc_stride) : (uint32_t)(j * n0));
            const uint64_t b0 = sw128_desc(x_ring) + (by_tile ? 0u : (uint64_t)((j * n0 * 128) >> 4));
            const int step = by_tile ? 2 : 1;
            int sa = by_tile ? j : 0, sx = sa;
            uint32_t pha = 0, phx = 0, acc = 0;
            for (int i = by_tile ? j : 0; i < nk; i += step) {
                if (!mbar_wait(afull(sa), pha, 3, wc)) break;
                if (!mbar_wait(xfull(sx), phx, 4, wc)) break;
                tc_fence_after();
                const uint32_t a = tmem + (uint32_t)(p.a_col0 + sa * kACols);
                const uint64_t bd = b0 + (uint64_t)((sx * p.b_bytes) >> 4);
#pragma unroll
                for (int k = 0; k < mk::kTileCols / 16; ++k)
                    umma_f16_ts(d, a + 8u * k, bd + 2 * k, id, acc | k);    // K = 16: 8 TMEM columns, 32 bytes of x
                acc = 1u;
                umma_commit(aempty(sa));
                umma_commit(xempty(sx));
                advance(sa, pha, step, SA);
                advance(sx, phx, step, SX);
            }
            umma_commit(done);                  // arrives once every MMA this thread issued completed
        }
        __syncwarp();
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

        // Epilogue: D[row, token] out of TMEM once every MMA of both issuers has completed (also after a give-up: TMEM
        // is freed below, and no MMA may still write it). Warp w reads lanes 32 (w % 4) .. + 31, every fourth
        // 16-column chunk.
        if (lane == 0) mbar_drain(done, 0, 9, wc);
        __syncwarp();
        tc_fence_after();
        const int quarter = warp & 3, cgroup = warp >> 2;
        const int row_local = quarter * 32 + lane;
        const int64_t row = col0 + row_local;
        const bool row_ok = row < p.rows;
        const bool two = p.by_tile && nk > 1;                         // issuer 1 took tiles: add its accumulator
        for (int c = cgroup; c < n_total / 16; c += kBuildWarps / 4) {
            float v[16];
            const uint32_t ta = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(c * 16);
            tmem_ld16(ta, v);
            if (two) {
                float u[16];
                tmem_ld16(ta + (uint32_t)p.acc_stride, u);
#pragma unroll
                for (int k = 0; k < 16; ++k) v[k] += u[k];
            }
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                const int t = c * 16 + k;
                if (t < tokens) {
                    if (p.y_tma) {
                        reinterpret_cast<T*>(gbase)[t * mk::kTileRows + row_local] = from_f32<T>(v[k]);  // rings free
                    } else if (p.n_split == 1) {
                        if (row_ok) reinterpret_cast<T*>(p.y)[t * p.ldy + row] = from_f32<T>(v[k]);
                    } else if (p.cluster) {
                        reinterpret_cast<float*>(gbase)[t * mk::kTileRows + row_local] = v[k];
                    } else if (row_ok) {
                        p.partial[((int64_t)split * p.tokens + t) * p.rows_pad + row] = v[k];
                    }
                }
            }
        }
        if (p.y_tma) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kXWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
    if (p.y_tma) {
        if (threadIdx.x == 0) {
            for (int b = 0; b < p.n_boxes; ++b)
                tma_store_2d(&tmap_y, smem_u32(gbase) + (uint32_t)(b * p.box_rows * mk::kTileRows * 2), (int)col0,
                             b * p.box_rows);
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
            asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        }
        return;
    }
    if (p.n_split == 1) return;

    if (p.cluster) {
        // Every split's partial tile is in its CTA's shared memory; CTA `split` adds its share of the tile's (token,
        // 4-row) units, split by split, and writes y. The second barrier keeps each CTA's shared memory alive until
        // every CTA of the cluster has read it.
        cluster_sync_all();
        const int ns = p.n_split;
        const int64_t n4 = (int64_t)tokens * (mk::kTileRows / 4);
        const int64_t u_begin = n4 * split / ns, u_end = n4 * (split + 1) / ns;
        const uint32_t part = smem_u32(gbase);
        for (int64_t u = u_begin + threadIdx.x; u < u_end; u += kThreads) {
            const int t = (int)(u / 32), r4 = (int)(u % 32) * 4;
            const uint32_t off = part + (uint32_t)(t * mk::kTileRows + r4) * 4u;
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
            const int64_t row = col0 + r4;
            T* yt = reinterpret_cast<T*>(p.y) + t * p.ldy;
            const float v[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
            for (int c = 0; c < 4; ++c)
                if (row + c < p.rows) yt[row + c] = from_f32<T>(v[c]);
        }
        cluster_sync_all();
        return;
    }

    // Split columns through the workspace: the last CTA of this row tile adds the partials in split order.
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(&p.tickets[rt], 1u) == (unsigned)(p.n_split - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const int64_t n4 = (int64_t)p.tokens * (mk::kTileRows / 4);
    const int64_t split_stride = (int64_t)p.tokens * p.rows_pad;
    for (int64_t u = threadIdx.x; u < n4; u += kThreads) {
        const int64_t t = u / 32, row = col0 + (u % 32) * 4;
        const int64_t off = t * p.rows_pad + row;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int sp = 0; sp < p.n_split; ++sp) {
            const float4 a = __ldcg(reinterpret_cast<const float4*>(p.partial + sp * split_stride + off));
            acc.x += a.x; acc.y += a.y; acc.z += a.z; acc.w += a.w;
        }
        T* yt = reinterpret_cast<T*>(p.y) + t * p.ldy;
        const float v[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
        for (int c = 0; c < 4; ++c)
            if (row + c < p.rows) yt[row + c] = from_f32<T>(v[c]);
    }
    if (threadIdx.x == 0) p.tickets[rt] = 0u;            // zeroed again for the next call
}

struct MaskPlan {
    int n_total, box_rows, n_boxes, by_tile, acc_stride, a_col0, a_slots, x_slots, b_bytes, ring_bytes, smem;
    int n_split, kt_per_split;
};

// Token-dependent part of a launch plan: MMA N, accumulators and A slots in TMEM, x boxes, the rings.
int plan_tokens(int tn, MaskPlan& pl) {
    if (tn < 1 || tn > kMaxN) return fail(P2P_EINVAL, "p2p_spmm_mask: %d tokens in one launch", tn);
    const int bar_bytes = 8 * (2 * kMaxXSlots + 2 * kTickets + 2 * kMaxASlots + 1);
    const int fixed = 1024 + kRingPad + bar_bytes + 16;
    pl.n_total = (tn + 15) / 16 * 16;
    pl.n_boxes = pl.n_total <= 256 ? 1 : 2;
    pl.box_rows = pl.n_total / pl.n_boxes;
    pl.by_tile = pl.n_total <= 128;
    const int acc_cols = pl.by_tile ? pow2_at_least(pl.n_total) : pl.n_total;
    pl.acc_stride = pl.by_tile ? acc_cols : 0;
    pl.a_col0 = pl.by_tile ? 2 * acc_cols : (pl.n_total + kACols - 1) / kACols * kACols;
    pl.a_slots = (kTmemCols - pl.a_col0) / kACols;
    if (pl.a_slots > kMaxASlots) pl.a_slots = kMaxASlots;
    if (pl.by_tile) pl.a_slots &= ~1;                 // even: each issuer's tiles keep to its own slots
    pl.b_bytes = pl.n_total * 128;
    pl.x_slots = (pl.by_tile || pl.b_bytes <= 8192) ? 4 : 3;
    pl.ring_bytes = (kSmemLimit - fixed - pl.x_slots * pl.b_bytes) / 16 * 16;
    if (pl.a_slots < 2 || pl.ring_bytes < mk::kMaxSegBytes)
        return fail(P2P_EUNSUPPORTED, "p2p_spmm_mask: %d tokens do not fit one launch", tn);
    pl.smem = fixed + pl.x_slots * pl.b_bytes + pl.ring_bytes;
    return P2P_OK;
}

// Columns split so that the row tiles fill the SMs: the fewest waves of CTAs a column tile's work, plus a CTA's fixed
// cost (fill and drain, TMEM, the epilogue: about 10 tiles' time) and the cost of writing and re-reading fp32 partials.
void plan_split(int64_t row_tiles, int col_tiles, int tokens, int sms, int* n_split, int* per) {
    int best = 1;
    double best_cost = 1e30;
    const int max_split = col_tiles < 32 ? col_tiles : 32;
    for (int s = 1; s <= max_split; ++s) {
        const int k = (col_tiles + s - 1) / s;
        if ((s - 1) * k >= col_tiles) continue;
        const double waves = (double)((row_tiles * s + sms - 1) / sms);
        double cost = waves * (k + 10.0);
        if (s > 1) cost += (double)s * tokens * row_tiles / 8.0 / sms;
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = s;
        }
    }
    int k = (col_tiles + best - 1) / best;
    if (k > kMaxTilesPerCta) k = kMaxTilesPerCta;
    *per = k;
    *n_split = (col_tiles + k - 1) / k;
}

// Clusters of n_split CTAs of this plan's shared memory that the device holds at once (cached per device and shape).
int max_clusters(const MaskPlan& pl, int n_split) {
    static std::mutex mu;
    static std::map<std::pair<int, int>, int> known;
    std::lock_guard<std::mutex> lock(mu);
    int dev = 0;
    cudaGetDevice(&dev);
    const auto key = std::make_pair(n_split * 64 + dev, pl.smem);
    auto it = known.find(key);
    if (it != known.end()) return it->second;
    int clusters = 0;
    if (allow_smem((const void*)spmm_mask_kernel<__nv_bfloat16>, pl.smem, "p2p_spmm_mask") == P2P_OK &&
        allow_smem((const void*)spmm_mask_kernel<__half>, pl.smem, "p2p_spmm_mask") == P2P_OK) {
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 1;
        attr[0].val.clusterDim.y = n_split;
        attr[0].val.clusterDim.z = 1;
        cfg.gridDim = dim3(1, n_split);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = pl.smem;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&clusters, spmm_mask_kernel<__nv_bfloat16>, &cfg) != cudaSuccess)
            clusters = 0;
        cudaGetLastError();                               // a refusal only means: use the workspace path
    }
    known[key] = clusters;
    return clusters;
}

// Whether the column splits of a launch are added inside clusters: 2 to 8 splits, the fp32 partial tile fits the
// rings, and the device holds the launch's clusters in as few waves as the plain grid takes.
bool cluster_reduce(const MaskPlan& pl, int n_split, int64_t row_tiles) {
    if (n_split < 2 || n_split > 8) return false;
    if ((int64_t)pl.n_total * mk::kTileRows * 4 > (int64_t)pl.x_slots * pl.b_bytes + pl.ring_bytes) return false;
    const int resident = max_clusters(pl, n_split);
    if (resident <= 0) return false;
    const int64_t sms = sm_count();
    const int64_t plain_waves = (row_tiles * n_split + sms - 1) / sms;
    const int64_t cluster_waves = (row_tiles + resident - 1) / resident;
    return cluster_waves <= plain_waves;
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
int launch_mask(const CUtensorMap& map, const CUtensorMap& ymap, const MaskParams& prm, dim3 grid, int smem,
                cudaStream_t st) {
    auto kernel = spmm_mask_kernel<T>;
    if (int e = allow_smem((const void*)kernel, smem, "p2p_spmm_mask")) return e;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = grid.y;
    attr[1].val.clusterDim.z = 1;
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = prm.cluster ? 2 : 1;
    cudaLaunchKernelEx(&cfg, kernel, map, ymap, prm);
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
    size_t need = 0;
    for (int t : sizes) {
        if (t <= 0) continue;
        int n = 1, per = col_tiles;
        plan_split(row_tiles, col_tiles, t, sm_count(), &n, &per);
        if (n == 1) continue;
        MaskPlan pl;
        if (plan_tokens(t, pl) == P2P_OK && cluster_reduce(pl, n, row_tiles)) continue;
        const size_t w = kTicketRegion + (size_t)n * t * row_tiles * mk::kTileRows * sizeof(float);
        need = need > w ? need : w;
    }
    return need;
}

extern "C" int p2p_spmm_mask(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ldx, const void* data,
                             const int64_t* seg, int64_t rows, void* y, int64_t ldy, void* workspace,
                             size_t workspace_bytes, void* stream) {
    P2P_REQUIRE(tokens >= 0 && rows >= 0 && cols >= 1, "p2p_spmm_mask: bad shape");
    if (tokens == 0 || rows == 0) return P2P_OK;
    if (dtype != P2P_BF16 && dtype != P2P_F16) return fail(P2P_EUNSUPPORTED, "p2p_spmm_mask: bf16 or f16");
    P2P_REQUIRE(x && data && seg && y, "p2p_spmm_mask: null pointer");
    P2P_REQUIRE(aligned16(data), "p2p_spmm_mask: the layout must start on a 16-byte boundary");
    P2P_REQUIRE(cols % 8 == 0 && ldx % 8 == 0 && ldx >= cols && aligned16(x),
                "p2p_spmm_mask: x needs 16-byte aligned rows (cols and ldx multiples of 8)");
    P2P_REQUIRE(ldy >= rows, "p2p_spmm_mask: ldy %lld below rows %lld", (long long)ldy, (long long)rows);
    P2P_REQUIRE(rows <= 0x7fffffff && cols <= 0x7fffffff, "p2p_spmm_mask: too large");
    cudaStream_t st = as_stream(stream);
    const int sms = sm_count();
    const int64_t row_tiles = (rows + mk::kTileRows - 1) / mk::kTileRows;
    const int col_tiles = (int)((cols + mk::kTileCols - 1) / mk::kTileCols);
    const int chunk = chunk_tokens(tokens);
    for (int64_t t0 = 0; t0 < tokens; t0 += chunk) {
        const int tn = (int)(tokens - t0 < chunk ? tokens - t0 : chunk);
        MaskPlan pl;
        if (int e = plan_tokens(tn, pl)) return e;
        plan_split(row_tiles, col_tiles, tn, sms, &pl.n_split, &pl.kt_per_split);
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
        prm.acc_stride = pl.acc_stride;
        prm.a_col0 = pl.a_col0;
        prm.a_slots = pl.a_slots;
        prm.x_slots = pl.x_slots;
        prm.b_bytes = pl.b_bytes;
        prm.ring_bytes = pl.ring_bytes;
        prm.kt_per_split = pl.kt_per_split;
        prm.n_split = pl.n_split;
        prm.y = reinterpret_cast<char*>(y) + t0 * ldy * 2;
        prm.ldy = ldy;
        prm.rows_pad = row_tiles * mk::kTileRows;
        prm.partial = nullptr;
        prm.tickets = nullptr;
        prm.cluster = cluster_reduce(pl, pl.n_split, row_tiles) ? 1 : 0;
        if (pl.n_split > 1 && !prm.cluster) {
            const size_t need = kTicketRegion + (size_t)pl.n_split * tn * prm.rows_pad * sizeof(float);
            P2P_REQUIRE(workspace && workspace_bytes >= need, "p2p_spmm_mask: workspace of %zu bytes, %zu needed",
                        workspace_bytes, need);
            if (row_tiles > kMaxRowTiles) return fail(P2P_EUNSUPPORTED, "p2p_spmm_mask: %lld rows", (long long)rows);
            prm.tickets = reinterpret_cast<unsigned*>(workspace);
            prm.partial = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + kTicketRegion);
        }
        prm.wait_ns = kWaitNs;
        prm.seq = next_seq();
        CUtensorMap map, ymap;
        const void* xt = reinterpret_cast<const char*>(x) + t0 * ldx * 2;
        if (int e = encode_x_map(&map, xt, dtype, tn, cols, ldx, pl.box_rows)) return e;
        prm.y_tma = pl.n_split == 1 && ldy % 8 == 0 && aligned16(prm.y) &&
                    (int64_t)pl.n_total * mk::kTileRows * 2 <= (int64_t)pl.x_slots * pl.b_bytes + pl.ring_bytes;
        ymap = map;
        if (prm.y_tma && encode_y_map(&ymap, prm.y, dtype, tn, rows, ldy, pl.box_rows) != P2P_OK) prm.y_tma = 0;
        const dim3 grid((unsigned)row_tiles, (unsigned)pl.n_split);
        if (int e = dtype == P2P_BF16 ? launch_mask<__nv_bfloat16>(map, ymap, prm, grid, pl.smem, st)
                                      : launch_mask<__half>(map, ymap, prm, grid, pl.smem, st))
            return e;
    }
    return P2P_OK;
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
