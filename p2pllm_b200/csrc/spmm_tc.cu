// (2b) Compact sparse GEMM on the 5th-generation tensor cores: y[t, r] = sum_j v[r, j] * x[t, idx[r, j]] for bf16/f16
// weights in the tiled layout of tc_layout.cuh.
//
// Replaces p2p/compact.cu:82-278 (spmm_kernel + sum_parts + spmm), which rebuilds 8 x 8 pieces from bit masks into
// mma.sync fragments and re-reads every weight once per 64 tokens. Here a CTA owns one 128-row tile and a range of
// 64-column tiles (split-K), and every token of the pass at once (up to 512 in TMEM):
//
//   warp 8  (producer)  per column tile: TMA of the x tile [tokens x 64] (128-byte swizzle) into ring 1, and a bulk
//                       copy of the segment's packed words from HBM into ring 1 beside it; one mbarrier, tx-counted.
//   warps 0-7 (expand)  zero a 128 x 64 bf16 tile in ring 2 and scatter the segment's words into it at their swizzled
//                       (row, column) places: the dense A operand, built in shared memory, never in HBM.
//   warp 9  (MMA)       one elected thread issues tcgen05.mma (M = 128, N = tokens rounded to 16, K = 16 a step)
//                       with the accumulator D[128 x N] fp32 in TMEM; tcgen05.commit frees both rings' slots.
//   warps 0-7 (epilogue) tcgen05.ld D out of TMEM, round, and write y[t, row] (coalesced along rows), or write fp32
//                       partials when the columns are split; the last CTA of a row tile adds the partials in split
//                       order (a ticket per row tile), so results do not depend on scheduling.
//
// Every mbarrier wait is bounded (about 2 s of %globaltimer): past it the kernel records where it gave up in *err and
// runs on, so a broken pipeline ends the kernel with an error status instead of hanging the GPU.
#include <cuda.h>

#include <type_traits>

#include "common.cuh"
#include "tc_layout.cuh"

namespace p2p {
namespace {

constexpr int kExpWarps = 8;
constexpr int kExpThreads = kExpWarps * 32;
constexpr int kProducerWarp = kExpWarps;
constexpr int kMmaWarp = kExpWarps + 1;
constexpr int kTcThreads = kExpThreads + 64;
constexpr int kATileBytes = tc::kTileRows * tc::kTileCols * 2;   // 16 KiB
constexpr int kS2 = 2;                                             // A tiles in flight
constexpr int kMaxS1 = 8;
constexpr int kSmemLimit = 227 * 1024 - 1024;          // dynamic shared memory, leaving room for the static
constexpr uint64_t kWaitNs = 2000000000ull;

__device__ int g_tc_error;            // first failed wait of the last launches (0: none); read back by the host

struct TcParams {
    const uint32_t* words;            // the module's packed words
    const int64_t* seg;               // [row_tiles * col_tiles + 1]
    int rows, col_tiles, tokens, n_total, box_rows, n_boxes, tmem_cols;
    int s1, b_bytes, seg_cap, kt_per_split, n_split;
    void* y;
    int64_t ldy;
    float* partial;                   // [n_split, tokens, rows_pad] when n_split > 1
    unsigned* tickets;                // [row_tiles]
    int64_t rows_pad;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase of parity `parity`; after kWaitNs (or at once, once another wait has failed) records `where`.
__device__ __forceinline__ void mbar_wait(uint32_t bar, uint32_t parity, int where) {
    if (mbar_try(bar, parity)) return;
    const uint64_t t0 = now_ns();
    while (!mbar_try(bar, parity)) {
        if (*(volatile int*)&g_tc_error != 0 || now_ns() - t0 > kWaitNs) {
            atomicCAS(&g_tc_error, 0, where);
            return;
        }
    }
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
                 : "memory");
}

// Shared-memory matrix descriptor of a K-major tile in the 128-byte swizzle layout: rows of 128 bytes, 8-row atoms of
// 1024 bytes (stride byte offset), version 1, swizzle mode 2 (128B).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor of kind::f16: D fp32, A and B bf16 (or both f16), both K-major, M = 128, N.
template <typename T> __device__ __forceinline__ uint32_t idesc_f16(int n) {
    constexpr uint32_t ab = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
    return (1u << 4) | (ab << 7) | (ab << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
        "[%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

template <typename T>
__global__ void __launch_bounds__(kTcThreads, 1) spmm_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint32_t s_tmem;
    __shared__ int s_last;
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* gbase = smem_raw + (base - raw);
    const int S1 = p.s1;
    const uint32_t a_ring = base;
    const uint32_t b_ring = a_ring + kS2 * kATileBytes;
    const uint32_t seg_ring = b_ring + S1 * p.b_bytes;
    const uint32_t bars = seg_ring + S1 * p.seg_cap;
    auto full1 = [&](int s) { return bars + 8u * s; };
    auto empty1 = [&](int s) { return bars + 8u * (kMaxS1 + s); };
    auto full2 = [&](int s) { return bars + 8u * (2 * kMaxS1 + s); };
    auto empty2 = [&](int s) { return bars + 8u * (2 * kMaxS1 + kS2 + s); };
    const uint32_t done = bars + 8u * (2 * kMaxS1 + 2 * kS2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rt = blockIdx.x, split = blockIdx.y;
    const int kt0 = split * p.kt_per_split;
    const int kt1 = min(p.col_tiles, kt0 + p.kt_per_split);
    const int nk = kt1 - kt0;
    const int64_t seg0 = (int64_t)rt * p.col_tiles + kt0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S1; ++s) {
            mbar_init(full1(s), 1);
            mbar_init(empty1(s), 1);
        }
        for (int s = 0; s < kS2; ++s) {
            mbar_init(full2(s), kExpWarps);
            mbar_init(empty2(s), 1);
        }
        mbar_init(done, 1);
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

    if (warp == kProducerWarp) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_x)) : "memory");
            for (int i = 0; i < nk; ++i) {
                const int s = i % S1;
                if (i >= S1) mbar_wait(empty1(s), ((i / S1) - 1) & 1, 1);
                const int64_t w0 = p.seg[seg0 + i], w1 = p.seg[seg0 + i + 1];
                const uint32_t seg_bytes = (uint32_t)((w1 - w0) * 4);
                mbar_expect_tx(full1(s), (uint32_t)p.b_bytes + seg_bytes);
                for (int b = 0; b < p.n_boxes; ++b)
                    tma_load_2d(b_ring + s * p.b_bytes + b * p.box_rows * 128, &tmap_x, (kt0 + i) * tc::kTileCols,
                                b * p.box_rows, full1(s));
                if (seg_bytes) bulk_load(seg_ring + s * p.seg_cap, p.words + w0, seg_bytes, full1(s));
            }
        }
        __syncwarp();
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            const uint32_t id0 = idesc_f16<T>(p.n_total <= 256 ? p.n_total : 256);
            const uint32_t id1 = idesc_f16<T>(p.n_total > 256 ? p.n_total - 256 : 16);
            for (int i = 0; i < nk; ++i) {
                const int s1 = i % S1, s2 = i % kS2;
                mbar_wait(full2(s2), (i / kS2) & 1, 2);
                mbar_wait(full1(s1), (i / S1) & 1, 3);
                tc_fence_after();
                const uint64_t a_desc = sw128_desc(a_ring + s2 * kATileBytes);
                const uint64_t b_desc = sw128_desc(b_ring + s1 * p.b_bytes);
#pragma unroll
                for (int k = 0; k < tc::kTileCols / 16; ++k) {
                    const uint32_t acc = (i > 0 || k > 0) ? 1u : 0u;
                    umma_f16(tmem, a_desc + 2 * k, b_desc + 2 * k, id0, acc);     // +32 bytes a K step of 16
                    if (p.n_total > 256)
                        umma_f16(tmem + 256, a_desc + 2 * k, b_desc + (uint64_t)((256 * 128) >> 4) + 2 * k, id1, acc);
                }
                umma_commit(empty2(s2));
                umma_commit(empty1(s1));
            }
            umma_commit(done);
        }
        __syncwarp();
    } else {
        // Expanders: the dense 128 x 64 tile of each column tile, built in shared memory.
        const int tid = threadIdx.x;
        for (int i = 0; i < nk; ++i) {
            const int s1 = i % S1, s2 = i % kS2;
            mbar_wait(full1(s1), (i / S1) & 1, 4);
            if (i >= kS2) mbar_wait(empty2(s2), ((i / kS2) - 1) & 1, 5);
            uint4* a = reinterpret_cast<uint4*>(gbase + (size_t)s2 * kATileBytes);
#pragma unroll
            for (int j = tid; j < kATileBytes / 16; j += kExpThreads) a[j] = make_uint4(0, 0, 0, 0);
            asm volatile("bar.sync 1, %0;" ::"n"(kExpThreads) : "memory");
            const int64_t w0 = p.seg[seg0 + i], w1 = p.seg[seg0 + i + 1];
            const int nq = (int)((w1 - w0) >> 2);
            const uint4* sg = reinterpret_cast<const uint4*>(gbase + (seg_ring - base) + (size_t)s1 * p.seg_cap);
            const uint32_t a_s = a_ring + s2 * kATileBytes;
            for (int q = tid; q < nq; q += kExpThreads) {
                const uint4 v = sg[q];
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    if (w[e] & tc::kPadWord) continue;
                    const uint32_t r = (w[e] >> 6) & 127u, c = w[e] & 63u;
                    const uint32_t off = r * 128u + ((c * 2u) ^ ((r & 7u) << 4));
                    asm volatile("st.shared.u16 [%0], %1;" ::"r"(a_s + off), "h"((unsigned short)(w[e] >> 16)) : "memory");
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(full2(s2));
        }

        // Epilogue: D[row, token] out of TMEM. Warp w reads lanes 32 (w % 4) .. + 31, every other 16-column chunk.
        mbar_wait(done, 0, 6);
        tc_fence_after();
        const int quarter = warp & 3, half = warp >> 2;
        const int row_local = quarter * 32 + lane;
        const int64_t row = (int64_t)rt * tc::kTileRows + row_local;
        const bool row_ok = row < p.rows;
        for (int c = half; c < p.n_total / 16; c += 2) {
            float v[16];
            tmem_ld16(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(c * 16), v);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int t = c * 16 + j;
                if (t < p.tokens && row_ok) {
                    if (p.n_split == 1)
                        reinterpret_cast<T*>(p.y)[(int64_t)t * p.ldy + row] = from_f32<T>(v[j]);
                    else
                        p.partial[((int64_t)split * p.tokens + t) * p.rows_pad + row] = v[j];
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kProducerWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(p.tmem_cols) : "memory");
    }
    if (p.n_split == 1) return;

    // Split columns: the last CTA of this row tile adds the partials in split order.
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(&p.tickets[rt], 1u) == (unsigned)(p.n_split - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const int64_t n = (int64_t)p.tokens * tc::kTileRows;
    for (int64_t i = threadIdx.x; i < n; i += kTcThreads) {
        const int t = (int)(i / tc::kTileRows);
        const int64_t row = (int64_t)rt * tc::kTileRows + (i % tc::kTileRows);
        if (row >= p.rows) continue;
        float s = 0.f;
        for (int sp = 0; sp < p.n_split; ++sp) s += __ldcg(p.partial + ((int64_t)sp * p.tokens + t) * p.rows_pad + row);
        reinterpret_cast<T*>(p.y)[(int64_t)t * p.ldy + row] = from_f32<T>(s);
    }
    if (threadIdx.x == 0) p.tickets[rt] = 0u;            // the workspace is zeroed again for the next call
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
    return fn;
}

struct TcPlan {
    int n_total, box_rows, n_boxes, tmem_cols, s1, b_bytes, seg_cap, n_split, kt_per_split, smem;
};

int pow2_at_least(int v) {
    int p = 32;
    while (p < v) p <<= 1;
    return p;
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
        double cost = waves * (per + 3.0);                            // + pipeline fill and epilogue
        if (s > 1) cost += (double)s * tokens * row_tiles / 12.0 / sms;
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = s;
        }
    }
    return best;
}

}  // namespace
}  // namespace p2p

using namespace p2p;

extern "C" size_t p2p_spmm_tc_workspace(int64_t rows, int64_t cols, int64_t tokens) {
    if (rows <= 0 || cols <= 0 || tokens <= 0) return 0;
    const int64_t row_tiles = (rows + tc::kTileRows - 1) / tc::kTileRows;
    const int col_tiles = (int)((cols + tc::kTileCols - 1) / tc::kTileCols);
    size_t need = 0;
    const int chunks[2] = {(int)(tokens < 512 ? tokens : 512), (int)(tokens % 512)};
    for (int t : chunks) {
        if (t <= 0) continue;
        const int s = choose_split(row_tiles, col_tiles, t, sm_count());
        const int per = (col_tiles + s - 1) / s, n = (col_tiles + per - 1) / per;
        if (n == 1) continue;
        const size_t w = ((size_t)row_tiles * sizeof(unsigned) + 255) / 256 * 256 +
                         (size_t)n * t * row_tiles * tc::kTileRows * sizeof(float);
        need = need > w ? need : w;
    }
    return need;
}

extern "C" int p2p_spmm_tc(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ldx, const uint32_t* words,
                           const int64_t* seg, int64_t rows, int64_t seg_cap_words, void* y, int64_t ldy,
                           void* workspace, size_t workspace_bytes, void* stream) {
    P2P_REQUIRE(tokens >= 0 && rows >= 0 && cols >= 1, "p2p_spmm_tc: bad shape");
    if (tokens == 0 || rows == 0) return P2P_OK;
    if (dtype != P2P_BF16 && dtype != P2P_F16)
        return fail(P2P_EUNSUPPORTED, "p2p_spmm_tc: bf16 or f16 (fp32 weights take p2p_spmm_rows)");
    P2P_REQUIRE(x && words && seg && y, "p2p_spmm_tc: null pointer");
    P2P_REQUIRE(cols % 8 == 0 && ldx % 8 == 0 && ldx >= cols && aligned16(x),
                "p2p_spmm_tc: x needs 16-byte aligned rows (cols and ldx multiples of 8)");
    P2P_REQUIRE(ldy >= rows, "p2p_spmm_tc: ldy %lld below rows %lld", (long long)ldy, (long long)rows);
    P2P_REQUIRE(seg_cap_words >= 0 && seg_cap_words % 4 == 0 && seg_cap_words <= tc::kTileRows * tc::kTileCols + 4,
                "p2p_spmm_tc: segment capacity %lld words", (long long)seg_cap_words);
    P2P_REQUIRE(rows <= 0x7fffffff && cols <= 0x7fffffff, "p2p_spmm_tc: too large");
    EncodeTiledFn encode = encode_fn();
    if (!encode) return fail(P2P_ECUDA, "p2p_spmm_tc: cuTensorMapEncodeTiled unavailable");
    cudaStream_t st = as_stream(stream);
    const int sms = sm_count();
    const int64_t row_tiles = (rows + tc::kTileRows - 1) / tc::kTileRows;
    const int col_tiles = (int)((cols + tc::kTileCols - 1) / tc::kTileCols);
    const int elem = 2;

    for (int64_t t0 = 0; t0 < tokens; t0 += 512) {             // at most 512 tokens (TMEM columns) a launch
        const int tn = (int)(tokens - t0 < 512 ? tokens - t0 : 512);
        TcPlan pl;
        pl.n_total = (tn + 15) / 16 * 16;
        pl.n_boxes = pl.n_total <= 256 ? 1 : 2;
        pl.box_rows = pl.n_total / pl.n_boxes;
        pl.tmem_cols = pow2_at_least(pl.n_total);
        pl.b_bytes = pl.n_total * 128;
        pl.seg_cap = (int)((seg_cap_words * 4 + 127) / 128 * 128);
        if (pl.seg_cap == 0) pl.seg_cap = 128;
        const int fixed = 1024 + kS2 * kATileBytes + 8 * (2 * kMaxS1 + 2 * kS2 + 1) + 64;
        pl.s1 = (kSmemLimit - fixed) / (pl.b_bytes + pl.seg_cap);
        if (pl.s1 > kMaxS1) pl.s1 = kMaxS1;
        if (pl.s1 < 2) return fail(P2P_EUNSUPPORTED, "p2p_spmm_tc: %d tokens and %d-byte segments exceed shared memory",
                                   tn, pl.seg_cap);
        pl.smem = fixed + pl.s1 * (pl.b_bytes + pl.seg_cap);
        pl.n_split = choose_split(row_tiles, col_tiles, tn, sms);
        pl.kt_per_split = (col_tiles + pl.n_split - 1) / pl.n_split;
        pl.n_split = (col_tiles + pl.kt_per_split - 1) / pl.kt_per_split;

        TcParams prm;
        prm.words = words;
        prm.seg = seg;
        prm.rows = (int)rows;
        prm.col_tiles = col_tiles;
        prm.tokens = tn;
        prm.n_total = pl.n_total;
        prm.box_rows = pl.box_rows;
        prm.n_boxes = pl.n_boxes;
        prm.tmem_cols = pl.tmem_cols;
        prm.s1 = pl.s1;
        prm.b_bytes = pl.b_bytes;
        prm.seg_cap = pl.seg_cap;
        prm.kt_per_split = pl.kt_per_split;
        prm.n_split = pl.n_split;
        prm.y = reinterpret_cast<char*>(y) + t0 * ldy * elem;
        prm.ldy = ldy;
        prm.rows_pad = row_tiles * tc::kTileRows;
        prm.partial = nullptr;
        prm.tickets = nullptr;
        if (pl.n_split > 1) {
            const size_t need = ((size_t)row_tiles * sizeof(unsigned) + 255) / 256 * 256 +
                                (size_t)pl.n_split * tn * prm.rows_pad * sizeof(float);
            P2P_REQUIRE(workspace && workspace_bytes >= need, "p2p_spmm_tc: workspace of %zu bytes, %zu needed",
                        workspace_bytes, need);
            prm.tickets = reinterpret_cast<unsigned*>(workspace);
            const size_t tb = ((size_t)row_tiles * sizeof(unsigned) + 255) / 256 * 256;
            prm.partial = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + tb);
        }

        CUtensorMap map;
        const cuuint64_t gdim[2] = {(cuuint64_t)cols, (cuuint64_t)tn};
        const cuuint64_t gstride[1] = {(cuuint64_t)(ldx * elem)};
        const cuuint32_t box[2] = {(cuuint32_t)tc::kTileCols, (cuuint32_t)pl.box_rows};
        const cuuint32_t estride[2] = {1, 1};
        const void* xt = reinterpret_cast<const char*>(x) + t0 * ldx * elem;
        CUresult r = encode(&map, dtype == P2P_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                            const_cast<void*>(xt), gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return fail(P2P_ECUDA, "p2p_spmm_tc: tensor map encode failed (%d)", (int)r);

        const dim3 grid((unsigned)row_tiles, (unsigned)pl.n_split);
        if (dtype == P2P_BF16) {
            if (int e = allow_smem((const void*)spmm_tc_kernel<__nv_bfloat16>, pl.smem, "p2p_spmm_tc")) return e;
            spmm_tc_kernel<__nv_bfloat16><<<grid, kTcThreads, pl.smem, st>>>(map, prm);
        } else {
            if (int e = allow_smem((const void*)spmm_tc_kernel<__half>, pl.smem, "p2p_spmm_tc")) return e;
            spmm_tc_kernel<__half><<<grid, kTcThreads, pl.smem, st>>>(map, prm);
        }
        if (int e = launch_status("p2p_spmm_tc")) return e;
    }
    return P2P_OK;
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
