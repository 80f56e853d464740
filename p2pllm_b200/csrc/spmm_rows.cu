// (2a) Compact sparse GEMM on CUDA cores, straight from the row layout: y[t, r] = sum_j vals[r, j] * x[t, idx[r, j]].
//
// Replaces p2p/compact.cu:265-278 (spmm) for weights held as values + column indices (p2p/compact.py:192-199 calls it
// per chunk of tokens). This is the fp32 path and the general one (any dtype, any token count); bf16/f16 modules run
// the tensor-core kernel of spmm_tc.cu instead.
//
// A block stages TT tokens of x in shared memory column by column (xs[c * TT + t]), so one 16-byte shared load
// fetches a kept weight's column for all TT tokens. Each warp walks one row at a time: lanes read the row's values
// and column indices with 16-byte loads (rows need not start on a 16-byte boundary: the loads start at the aligned
// element below and mask the strays), gather the columns and accumulate TT sums in fp32, then combine the lanes with
// shuffles. Blocks of the same rows but different token tiles are adjacent in launch order, so a row's weights come
// from HBM once and from L2 for the other tiles.
//
// Few tokens (a draft pass of 16 + 1): one block per SM stages ALL of x at once, column-major (each kept weight's
// column for every token is a few 16-byte shared loads), while its warps prefetch their first rows' weights into L2;
// then every warp of the grid takes whole rows in turn (dealt across the blocks first, so all SMs share the gathers,
// which bind: random columns make them bank-conflicted), each lane keeping a chunk of the row's loads in flight. x is
// read from L2 once per SM instead of once per (token tile, row group) block. (Staging x row-major by bulk copies
// was measured slower: a column then costs one shared load a token, with bank conflicts.)
#include "common.cuh"

namespace p2p {
namespace {

constexpr int kRowsBlock = 256;
constexpr int kRowsWarps = kRowsBlock / 32;
constexpr int kMaxBlocks = 8;
constexpr int kSmemCap = 200 * 1024;
constexpr int kSmemPreferred = 72 * 1024;

struct BlockTable {
    p2p_row_block b[kMaxBlocks];
    int64_t start[kMaxBlocks + 1];   // first row of each block in the concatenated row order
    int n;
};

template <typename T, int TT>
struct alignas(sizeof(T) * TT >= 16 ? 16 : sizeof(T) * TT) XCol {   // TT tokens of one column in shared memory
    T v[TT];
};

template <typename T, int TT>
__device__ __forceinline__ void gather(const T* xs, int c, float (&out)[TT]) {
    const T* p = xs + (size_t)c * TT;
    if constexpr (sizeof(T) == 4) {
        if constexpr (TT % 4 == 0) {
#pragma unroll
            for (int q = 0; q < TT / 4; ++q) {
                const float4 v = reinterpret_cast<const float4*>(p)[q];
                out[4 * q] = v.x; out[4 * q + 1] = v.y; out[4 * q + 2] = v.z; out[4 * q + 3] = v.w;
            }
        } else if constexpr (TT == 2) {
            const float2 v = *reinterpret_cast<const float2*>(p);
            out[0] = v.x; out[1] = v.y;
        } else {
            out[0] = p[0];
        }
    } else {
        if constexpr (TT % 8 == 0) {
#pragma unroll
            for (int q = 0; q < TT / 8; ++q) {
                const uint4 v = reinterpret_cast<const uint4*>(p)[q];
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float2 f = unpack2<T>(w[i]);
                    out[8 * q + 2 * i] = f.x; out[8 * q + 2 * i + 1] = f.y;
                }
            }
        } else if constexpr (TT == 4) {
            const uint2 v = *reinterpret_cast<const uint2*>(p);
            const float2 a = unpack2<T>(v.x), b = unpack2<T>(v.y);
            out[0] = a.x; out[1] = a.y; out[2] = b.x; out[3] = b.y;
        } else if constexpr (TT == 2) {
            const float2 a = unpack2<T>(*reinterpret_cast<const uint32_t*>(p));
            out[0] = a.x; out[1] = a.y;
        } else {
            out[0] = to_f32(p[0]);
        }
    }
}

// One value as fp32 through the read-only path.
__device__ __forceinline__ float ldg_f32(const float* p) { return __ldg(p); }
__device__ __forceinline__ float ldg_f32(const __nv_bfloat16* p) {
    return __uint_as_float((uint32_t)__ldg(reinterpret_cast<const unsigned short*>(p)) << 16);
}
__device__ __forceinline__ float ldg_f32(const __half* p) {
    return __half2float(__ushort_as_half(__ldg(reinterpret_cast<const unsigned short*>(p))));
}

// VEC values and VEC column indices of one 16-byte-aligned step of a row.
template <typename T, typename I, int VEC>
__device__ __forceinline__ void load_step(const T* v, const I* ix, int64_t e, float (&fv)[VEC], int (&ci)[VEC]) {
    if constexpr (sizeof(T) == 4) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(v + e));
        fv[0] = a.x; fv[1] = a.y; fv[2] = a.z; fv[3] = a.w;
    } else {
        const uint4 a = __ldg(reinterpret_cast<const uint4*>(v + e));
        const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = unpack2<T>(w[i]);
            fv[2 * i] = f.x; fv[2 * i + 1] = f.y;
        }
    }
    if (ix == nullptr) {
#pragma unroll
        for (int i = 0; i < VEC; ++i) ci[i] = i;
        return;
    }
    if constexpr (sizeof(I) * VEC == 16) {
        const uint4 a = __ldg(reinterpret_cast<const uint4*>(ix + e));
        const I* q = reinterpret_cast<const I*>(&a);
#pragma unroll
        for (int i = 0; i < VEC; ++i) ci[i] = (int)q[i];
    } else if constexpr (sizeof(I) * VEC == 32) {
        const uint4 a = __ldg(reinterpret_cast<const uint4*>(ix + e));
        const uint4 b = __ldg(reinterpret_cast<const uint4*>(ix + e) + 1);
        const I* qa = reinterpret_cast<const I*>(&a);
        const I* qb = reinterpret_cast<const I*>(&b);
#pragma unroll
        for (int i = 0; i < VEC / 2; ++i) { ci[i] = (int)qa[i]; ci[VEC / 2 + i] = (int)qb[i]; }
    } else {   // 8 bytes: four int16
        const uint2 a = __ldg(reinterpret_cast<const uint2*>(ix + e));
        const I* q = reinterpret_cast<const I*>(&a);
#pragma unroll
        for (int i = 0; i < VEC; ++i) ci[i] = (int)q[i];
    }
}

template <typename T, typename I, int TT>
__global__ void __launch_bounds__(kRowsBlock) spmm_rows_kernel(const T* __restrict__ x, int64_t tokens, int cols,
                                                                int64_t ldx, BlockTable bt, int64_t total_rows,
                                                                int64_t rows_per_group, T* __restrict__ y,
                                                                int64_t ldy) {
    constexpr int VEC = 16 / sizeof(T);
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T* xs = reinterpret_cast<T*>(smem_raw);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t t0 = (int64_t)blockIdx.x * TT;

    // Stage TT tokens, one column a thread: TT 2-byte (or 4-byte) loads, one vector store.
    for (int c = tid; c < cols; c += kRowsBlock) {
        XCol<T, TT> col;
#pragma unroll
        for (int t = 0; t < TT; ++t) col.v[t] = (t0 + t < tokens) ? x[(t0 + t) * ldx + c] : from_f32<T>(0.f);
        reinterpret_cast<XCol<T, TT>*>(xs)[c] = col;
    }
    __syncthreads();

    const int64_t r_begin = (int64_t)blockIdx.y * rows_per_group;
    const int64_t r_end = min(total_rows, r_begin + rows_per_group);
    const unsigned cmax = (unsigned)(cols - 1);
    for (int64_t r = r_begin + warp; r < r_end; r += kRowsWarps) {
        int b = 0;
        while (b + 1 < bt.n && r >= bt.start[b + 1]) ++b;
        const p2p_row_block& blk = bt.b[b];
        const int64_t lr = r - bt.start[b];
        const T* v = reinterpret_cast<const T*>(blk.vals);
        const I* ix = reinterpret_cast<const I*>(blk.idx);
        const int64_t base = lr * blk.ld, end = base + blk.k;

        float acc[TT];
#pragma unroll
        for (int t = 0; t < TT; ++t) acc[t] = 0.f;
        for (int64_t e = (base & ~(int64_t)(VEC - 1)) + lane * VEC; e < end; e += 32 * VEC) {
            float fv[VEC];
            int ci[VEC];
            load_step<T, I, VEC>(v, ix, e, fv, ci);
            if (ix == nullptr) {
#pragma unroll
                for (int i = 0; i < VEC; ++i) ci[i] += (int)(e - base);   // a dense block: column = position in its row
            }
            const bool whole = e >= base && e + VEC <= end;
#pragma unroll
            for (int i = 0; i < VEC; ++i) {
                if (!whole && (e + i < base || e + i >= end)) continue;
                float xv[TT];
                gather<T, TT>(xs, (int)min((unsigned)ci[i], cmax), xv);
#pragma unroll
                for (int t = 0; t < TT; ++t) acc[t] = fmaf(fv[i], xv[t], acc[t]);
            }
        }
#pragma unroll
        for (int t = 0; t < TT; ++t) {
#pragma unroll
            for (int d = 16; d > 0; d >>= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], d);
        }
        float mine = 0.f;
#pragma unroll
        for (int t = 0; t < TT; ++t)
            if (lane == t) mine = acc[t];
        if (lane < TT && t0 + lane < tokens) y[(t0 + lane) * ldy + blk.row0 + lr] = from_f32<T>(mine);
    }
}

constexpr int kStagedBlock = 512;
constexpr int kStagedWarps = kStagedBlock / 32;
constexpr int kStagedMaxTokens = 32;
constexpr int kStagedSmem = 200 * 1024;

// Token tiles of the staged kernel: fp32 columns in multiples of 4 tokens (16-byte loads), 2-byte ones of 8.
template <typename T> constexpr int staged_step() { return sizeof(T) == 4 ? 4 : 8; }
template <typename T> int staged_tt(int64_t tokens) {
    const int q = staged_step<T>();
    return (int)((tokens + q - 1) / q * q);
}

// y rows of the grid's warps; x [tokens <= TT, cols] staged column-major in shared memory (xs[c * TT + t], zeros past
// the tokens), so a kept weight's column for every token is TT / VEC 16-byte shared loads.
template <typename T, typename I, int TT>
__global__ void __launch_bounds__(kStagedBlock, 1) spmm_rows_staged_kernel(const T* __restrict__ x, int tokens,
                                                                           int cols, int64_t ldx, BlockTable bt,
                                                                           int64_t total_rows, T* __restrict__ y,
                                                                           int64_t ldy) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T* xs = reinterpret_cast<T*>(smem_raw);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // rows dealt across the blocks first (row r to block r % grid), so every SM's shared memory takes an equal share
    // of the gathers even when the rows do not fill every block's warps
    const int64_t gw = (int64_t)warp * gridDim.x + blockIdx.x;
    const int64_t stride = (int64_t)gridDim.x * kStagedWarps;
    // the first row of this warp, into L2 (a 128-byte line a lane), while x is staged
    if (gw < total_rows) {
        int bi = 0;
        while (bi + 1 < bt.n && gw >= bt.start[bi + 1]) ++bi;
        const p2p_row_block& blk = bt.b[bi];
        const int64_t base = (gw - bt.start[bi]) * blk.ld;
        const char* v = reinterpret_cast<const char*>(blk.vals) + base * sizeof(T);
        for (int64_t off = (int64_t)lane * 128; off < blk.k * (int64_t)sizeof(T); off += 32 * 128)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(v + off));
        if (blk.idx) {
            const char* ix = reinterpret_cast<const char*>(blk.idx) + base * sizeof(I);
            for (int64_t off = (int64_t)lane * 128; off < blk.k * (int64_t)sizeof(I); off += 32 * 128)
                asm volatile("prefetch.global.L2 [%0];" ::"l"(ix + off));
        }
    }
    // stage: one column a thread (a warp reads 32 consecutive columns of a token row), one vector store; two columns
    // a thread at a time, so that all their loads are in flight together
    for (int c = tid; c < cols; c += 2 * kStagedBlock) {
        const int c2 = c + kStagedBlock;
        XCol<T, TT> col, col2;
#pragma unroll
        for (int t = 0; t < TT; ++t) {
            col.v[t] = t < tokens ? x[t * ldx + c] : from_f32<T>(0.f);
            col2.v[t] = (t < tokens && c2 < cols) ? x[t * ldx + c2] : from_f32<T>(0.f);
        }
        reinterpret_cast<XCol<T, TT>*>(xs)[c] = col;
        if (c2 < cols) reinterpret_cast<XCol<T, TT>*>(xs)[c2] = col2;
    }
    __syncthreads();

    const unsigned cmax = (unsigned)(cols - 1);
    for (int64_t r = gw; r < total_rows; r += stride) {
        int bi = 0;
        while (bi + 1 < bt.n && r >= bt.start[bi + 1]) ++bi;
        const p2p_row_block& blk = bt.b[bi];
        const int64_t lr = r - bt.start[bi];
        const T* v = reinterpret_cast<const T*>(blk.vals);
        const I* ix = reinterpret_cast<const I*>(blk.idx);
        const int64_t base = lr * blk.ld, end = base + blk.k;
        float acc[TT];
#pragma unroll
        for (int t = 0; t < TT; ++t) acc[t] = 0.f;
        // Lane l takes the row's entries l, l + 32, ...: one gather instruction then reads 32 consecutive kept columns,
        // which fall on all eight 16-byte bank groups of the staged columns. (Four consecutive entries a lane, as
        // 16-byte loads, put neighbouring lanes k / keep columns apart -- 10 at keep 40 -- which with 80-byte columns
        // lands on four of the eight groups: twice the wavefronts a gather.) kPer entries a lane in flight at once.
        constexpr int kPer = TT >= 32 ? 8 : TT >= 16 ? 16 : 32;
        for (int64_t e0 = base + lane; e0 < end; e0 += (int64_t)kPer * 32) {
            float fv[kPer];
            int ci[kPer];
#pragma unroll
            for (int j = 0; j < kPer; ++j) {
                const int64_t e = e0 + (int64_t)j * 32;
                if (e < end) {
                    fv[j] = ldg_f32(v + e);
                    ci[j] = ix ? (int)__ldg(ix + e) : (int)(e - base);
                }
            }
#pragma unroll
            for (int j = 0; j < kPer; ++j) {
                if (e0 + (int64_t)j * 32 >= end) break;
                float xv[TT];
                gather<T, TT>(xs, (int)min((unsigned)ci[j], cmax), xv);
#pragma unroll
                for (int t = 0; t < TT; ++t) acc[t] = fmaf(fv[j], xv[t], acc[t]);
            }
        }
#pragma unroll
        for (int t = 0; t < TT; ++t) {
#pragma unroll
            for (int d = 16; d > 0; d >>= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], d);
        }
        float mine = 0.f;
#pragma unroll
        for (int t = 0; t < TT; ++t)
            if (lane == t) mine = acc[t];
        if (lane < tokens) y[(int64_t)lane * ldy + blk.row0 + lr] = from_f32<T>(mine);
    }
}

// The staged kernel takes the launch when all tokens (padded to its token step) fit one block's shared memory.
template <typename T>
bool staged_fits(int64_t tokens, int64_t cols) {
    return tokens >= 1 && tokens <= kStagedMaxTokens && cols * staged_tt<T>(tokens) * (int64_t)sizeof(T) <= kStagedSmem;
}

template <typename T, typename I, int TT>
int launch_staged(const void* x, int64_t tokens, int64_t cols, int64_t ldx, const BlockTable& bt, int64_t total_rows,
                  void* y, int64_t ldy, cudaStream_t s) {
    auto kern = spmm_rows_staged_kernel<T, I, TT>;
    const int smem = (int)(cols * TT * sizeof(T));
    if (int e = allow_smem((const void*)kern, kStagedSmem, "p2p_spmm_rows")) return e;
    const int grid = (int)(total_rows < sm_count() ? total_rows : sm_count());   // a block an SM, a row at least
    kern<<<grid, kStagedBlock, smem, s>>>(reinterpret_cast<const T*>(x), (int)tokens, (int)cols, ldx, bt, total_rows,
                                          reinterpret_cast<T*>(y), ldy);
    return launch_status("p2p_spmm_rows");
}

template <typename T, typename I>
int dispatch_staged(const void* x, int64_t tokens, int64_t cols, int64_t ldx, const BlockTable& bt, int64_t total_rows,
                    void* y, int64_t ldy, cudaStream_t s) {
    switch (staged_tt<T>(tokens)) {
        case 4: if constexpr (sizeof(T) == 4) return launch_staged<T, I, 4>(x, tokens, cols, ldx, bt, total_rows, y, ldy, s);
                break;
        case 8: return launch_staged<T, I, 8>(x, tokens, cols, ldx, bt, total_rows, y, ldy, s);
        case 12: if constexpr (sizeof(T) == 4) return launch_staged<T, I, 12>(x, tokens, cols, ldx, bt, total_rows, y, ldy, s);
                 break;
        case 16: return launch_staged<T, I, 16>(x, tokens, cols, ldx, bt, total_rows, y, ldy, s);
        case 20: if constexpr (sizeof(T) == 4) return launch_staged<T, I, 20>(x, tokens, cols, ldx, bt, total_rows, y, ldy, s);
                 break;
        case 24: return launch_staged<T, I, 24>(x, tokens, cols, ldx, bt, total_rows, y, ldy, s);
        case 28: if constexpr (sizeof(T) == 4) return launch_staged<T, I, 28>(x, tokens, cols, ldx, bt, total_rows, y, ldy, s);
                 break;
        case 32: return launch_staged<T, I, 32>(x, tokens, cols, ldx, bt, total_rows, y, ldy, s);
        default: break;
    }
    return fail(P2P_EINVAL, "p2p_spmm_rows: no staged tile for %lld tokens", (long long)tokens);
}

template <typename T, typename I, int TT>
int launch_rows(const void* x, int64_t tokens, int64_t cols, int64_t ldx, const BlockTable& bt, int64_t total_rows,
                void* y, int64_t ldy, cudaStream_t s) {
    auto kern = spmm_rows_kernel<T, I, TT>;
    const int smem = (int)(cols * TT * sizeof(T));
    if (int e = allow_smem((const void*)kern, smem, "p2p_spmm_rows")) return e;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kRowsBlock, smem) != cudaSuccess || per_sm < 1)
        per_sm = 1;
    const int64_t tiles = (tokens + TT - 1) / TT;
    int64_t groups = ((int64_t)sm_count() * per_sm * 2 + tiles - 1) / tiles;      // two waves of blocks in all
    const int64_t max_groups = (total_rows + kRowsWarps - 1) / kRowsWarps;
    groups = groups < max_groups ? groups : max_groups;
    groups = groups < 1 ? 1 : groups;
    const int64_t rows_per_group = (total_rows + groups - 1) / groups;
    groups = (total_rows + rows_per_group - 1) / rows_per_group;
    if (tiles > 0x7fffffff || groups > 65535) return fail(P2P_EUNSUPPORTED, "p2p_spmm_rows: grid too large");
    kern<<<dim3((unsigned)tiles, (unsigned)groups), kRowsBlock, smem, s>>>(
        reinterpret_cast<const T*>(x), tokens, (int)cols, ldx, bt, total_rows, rows_per_group, reinterpret_cast<T*>(y),
        ldy);
    return launch_status("p2p_spmm_rows");
}

// The widest token tile whose staged x fits: at most the token count rounded up to a power of two and 16, preferring
// a tile that leaves room for three blocks an SM.
template <typename T> int pick_tt(int64_t tokens, int64_t cols) {
    int cap = 1;
    while (cap < tokens && cap < 16) cap <<= 1;
    for (int tt = cap; tt >= 1; tt >>= 1)
        if (cols * tt * (int64_t)sizeof(T) <= kSmemPreferred) return tt;
    return cols * (int64_t)sizeof(T) <= kSmemCap ? 1 : 0;
}

template <typename T, typename I>
int dispatch_tt(const void* x, int64_t tokens, int64_t cols, int64_t ldx, const BlockTable& bt, int64_t total_rows,
                void* y, int64_t ldy, cudaStream_t s) {
    switch (pick_tt<T>(tokens, cols)) {
        case 16: return launch_rows<T, I, 16>(x, tokens, cols, ldx, bt, total_rows, y, ldy, s);
        case 8: return launch_rows<T, I, 8>(x, tokens, cols, ldx, bt, total_rows, y, ldy, s);
        case 4: return launch_rows<T, I, 4>(x, tokens, cols, ldx, bt, total_rows, y, ldy, s);
        case 2: return launch_rows<T, I, 2>(x, tokens, cols, ldx, bt, total_rows, y, ldy, s);
        case 1: return launch_rows<T, I, 1>(x, tokens, cols, ldx, bt, total_rows, y, ldy, s);
        default:
            return fail(P2P_EUNSUPPORTED, "p2p_spmm_rows: %lld columns of %d bytes exceed %d KiB of shared memory",
                        (long long)cols, (int)sizeof(T), kSmemCap / 1024);
    }
}

}  // namespace
}  // namespace p2p

using namespace p2p;

extern "C" int p2p_spmm_rows(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ldx,
                             const p2p_row_block* blocks, int nblocks, int idx_bytes, void* y, int64_t ldy,
                             void* stream) {
    P2P_REQUIRE(tokens >= 0 && cols >= 1, "p2p_spmm_rows: shape [%lld, %lld]", (long long)tokens, (long long)cols);
    P2P_REQUIRE(nblocks >= 1 && nblocks <= kMaxBlocks && blocks, "p2p_spmm_rows: 1 to %d row blocks", kMaxBlocks);
    P2P_REQUIRE(idx_bytes == 2 || idx_bytes == 4, "p2p_spmm_rows: idx_bytes %d", idx_bytes);
    P2P_REQUIRE(cols <= 0x7fffffff, "p2p_spmm_rows: too many columns");
    if (!dtype_ok(dtype)) return fail(P2P_EUNSUPPORTED, "p2p_spmm_rows: dtype %d", dtype);
    BlockTable bt;
    bt.n = nblocks;
    int64_t total = 0;
    int64_t out_rows = 0;
    for (int i = 0; i < nblocks; ++i) {
        const p2p_row_block& b = blocks[i];
        P2P_REQUIRE(b.rows >= 0 && b.k >= 0 && b.row0 >= 0, "p2p_spmm_rows: block %d has a negative size", i);
        P2P_REQUIRE(b.rows == 0 || (b.vals && (b.k == 0 || b.ld >= b.k)), "p2p_spmm_rows: block %d values", i);
        P2P_REQUIRE(b.idx || b.k == cols, "p2p_spmm_rows: dense block %d needs k == cols", i);
        P2P_REQUIRE(b.rows == 0 || (aligned16(b.vals) && (!b.idx || aligned16(b.idx))),
                    "p2p_spmm_rows: block %d values and indices must start on a 16-byte boundary", i);
        bt.b[i] = b;
        bt.start[i] = total;
        total += b.rows;
        out_rows = out_rows > b.row0 + b.rows ? out_rows : b.row0 + b.rows;
    }
    bt.start[nblocks] = total;
    if (tokens == 0 || total == 0) return P2P_OK;
    P2P_REQUIRE(x && y, "p2p_spmm_rows: null x or y");
    P2P_REQUIRE(ldx >= cols && ldy >= out_rows, "p2p_spmm_rows: strides ldx=%lld ldy=%lld too small", (long long)ldx,
                (long long)ldy);
    cudaStream_t s = as_stream(stream);
    P2P_DISPATCH(dtype, {
        if (staged_fits<scalar_t>(tokens, cols)) {
            if (idx_bytes == 2) return dispatch_staged<scalar_t, int16_t>(x, tokens, cols, ldx, bt, total, y, ldy, s);
            return dispatch_staged<scalar_t, int32_t>(x, tokens, cols, ldx, bt, total, y, ldy, s);
        }
        if (idx_bytes == 2) return dispatch_tt<scalar_t, int16_t>(x, tokens, cols, ldx, bt, total, y, ldy, s);
        return dispatch_tt<scalar_t, int32_t>(x, tokens, cols, ldx, bt, total, y, ldy, s);
    });
    return P2P_OK;
}
