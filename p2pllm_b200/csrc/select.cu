// (1b) Wanda selection and the compact formats.
//
// p2p_wanda_select replaces p2p/wanda.py:76-87 (prune: score = |w|.float() * norms, k = max(1, round(keep/100 * cols)),
// top-k per row -> mask) fused with p2p/compact.py:36-45 (pack: kept values in column order + int32 mask words). One
// block per row (grid-strided): the row's scores go to shared memory as order-preserving 32-bit keys, a 4-digit MSB
// radix select (8 bits a digit, per-warp histograms fed by match_any-aggregated atomics) finds the k-th largest key,
// and a block scan in column order keeps every key above it plus the first (lowest-column) `need` keys equal to it.
// Ties therefore go to the lower column, deterministically. The reference's torch.topk leaves tie order unspecified;
// everywhere the k-th and (k+1)-th scores differ both choose the same set.
//
// p2p_words_to_idx / p2p_pack_mask / p2p_unpack convert between the reference's mask words, uint8 masks, values +
// column indices and dense rows, one block per row with the same column-order block scan.
#include "common.cuh"

namespace p2p {
namespace {

constexpr int kSelBlock = 256;
constexpr int kSelWarps = kSelBlock / 32;
constexpr int64_t kMaxSelCols = 52000;

__device__ int g_bad_rows;   // rows that broke a format rule in the last checking call (read back by the host)

__device__ __forceinline__ int padded(int c) { return c + (c >> 5); }   // one spare word per 32: fewer bank clashes

// An order-preserving key of a float: larger floats give larger keys; -0 counts as +0.
__device__ __forceinline__ uint32_t key_of(float s) {
    if (s == 0.f) s = 0.f;
    const uint32_t b = __float_as_uint(s);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Exclusive scan of (a, b) over the block in thread order; returns the block totals through `tot`.
__device__ __forceinline__ int2 block_scan2(int a, int b, int2* warp_tot, int2& tot) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int ia = a, ib = b;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int va = __shfl_up_sync(0xffffffffu, ia, d), vb = __shfl_up_sync(0xffffffffu, ib, d);
        if (lane >= d) { ia += va; ib += vb; }
    }
    if (lane == 31) warp_tot[warp] = make_int2(ia, ib);
    __syncthreads();
    int ba = 0, bb = 0, ta = 0, tb = 0;
#pragma unroll
    for (int w = 0; w < kSelWarps; ++w) {
        const int2 v = warp_tot[w];
        if (w < warp) { ba += v.x; bb += v.y; }
        ta += v.x;
        tb += v.y;
    }
    __syncthreads();
    tot = make_int2(ta, tb);
    return make_int2(ba + ia - a, bb + ib - b);
}

template <typename I> __device__ __forceinline__ void put_idx(void* idx, int64_t at, int c) {
    reinterpret_cast<I*>(idx)[at] = (I)c;
}

template <typename T, typename I>
__global__ void __launch_bounds__(kSelBlock) select_kernel(const T* __restrict__ w, int64_t rows, int cols, int64_t ldw,
                                                            const float* __restrict__ norms, int64_t norm_group_rows,
                                                            int k, T* __restrict__ vals, I* __restrict__ idx,
                                                            int64_t ldo, int32_t* __restrict__ words, int64_t ldwords,
                                                            uint8_t* __restrict__ mask, int64_t ldm,
                                                            T* __restrict__ pruned, int64_t ldp) {
    extern __shared__ uint32_t smem[];
    uint32_t* keys = smem;                                   // [padded(cols) + 1]
    uint32_t* hist = keys + padded(cols) + 1;                 // [kSelWarps][256]
    __shared__ int2 warp_tot[kSelWarps];
    __shared__ uint32_t s_digit, s_above;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int n_words = (cols + 31) >> 5;
    const int wpt = (n_words + kSelBlock - 1) / kSelBlock;   // mask words a thread owns in the column-order passes
    const int w_begin = min(n_words, tid * wpt), w_end = min(n_words, w_begin + wpt);
    const int c_begin = w_begin * 32, c_end = min(cols, w_end * 32);

    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const T* wr = w + r * ldw;
        const float* nr = norms + (norm_group_rows > 0 ? (r / norm_group_rows) * (int64_t)cols : 0);
        for (int c = tid; c < cols; c += kSelBlock) keys[padded(c)] = key_of(fabsf(to_f32(wr[c])) * nr[c]);

        // Radix select of the k-th largest key, most significant digit first.
        uint32_t prefix = 0, pmask = 0;
        int remaining = k;
#pragma unroll 1
        for (int shift = 24; shift >= 0; shift -= 8) {
            for (int i = tid; i < kSelWarps * 256; i += kSelBlock) hist[i] = 0;
            __syncthreads();
            for (int c = tid; c < cols; c += kSelBlock) {
                const uint32_t key = keys[padded(c)];
                if ((key & pmask) == prefix) {
                    const uint32_t d = (key >> shift) & 255u;
                    const unsigned peers = __match_any_sync(__activemask(), d);
                    if (lane == __ffs(peers) - 1) atomicAdd(&hist[warp * 256 + d], (uint32_t)__popc(peers));
                }
            }
            __syncthreads();
            if (warp == 0) {
                // Lane l holds bins 255 - 8l - i (i = 0..7): a prefix over lanes counts the keys in higher bins.
                uint32_t cnt[8], sum = 0;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int b = 255 - 8 * lane - i;
                    uint32_t v = 0;
#pragma unroll
                    for (int q = 0; q < kSelWarps; ++q) v += hist[q * 256 + b];
                    cnt[i] = v;
                    sum += v;
                }
                uint32_t incl = sum;
#pragma unroll
                for (int d = 1; d < 32; d <<= 1) {
                    const uint32_t v = __shfl_up_sync(0xffffffffu, incl, d);
                    if (lane >= d) incl += v;
                }
                uint32_t run = incl - sum;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    if (run < (uint32_t)remaining && run + cnt[i] >= (uint32_t)remaining) {
                        s_digit = 255 - 8 * lane - i;
                        s_above = run;
                    }
                    run += cnt[i];
                }
            }
            __syncthreads();
            prefix |= s_digit << shift;
            pmask |= 255u << shift;
            remaining -= (int)s_above;
            __syncthreads();
        }
        const uint32_t kth = prefix;
        const int need = remaining;            // keys equal to kth that are kept: the lowest columns first

        int gt = 0, eq = 0;
        for (int c = c_begin; c < c_end; ++c) {
            const uint32_t key = keys[padded(c)];
            gt += key > kth;
            eq += key == kth;
        }
        int2 tot;
        const int2 before = block_scan2(eq, 0, warp_tot, tot);
        const int eq_before = before.x;
        const int kept = gt + max(0, min(eq, need - eq_before));
        const int2 pos2 = block_scan2(kept, 0, warp_tot, tot);
        int64_t pos = pos2.x;
        int er = eq_before;
        for (int wi = w_begin; wi < w_end; ++wi) {
            uint32_t bits = 0;
            const int cw = wi * 32;
            for (int b = 0; b < 32 && cw + b < cols; ++b) {
                const int c = cw + b;
                const uint32_t key = keys[padded(c)];
                bool keep = key > kth;
                if (key == kth) {
                    keep = er < need;
                    ++er;
                }
                const T v = wr[c];
                if (keep) {
                    bits |= 1u << b;
                    if (vals) vals[r * ldo + pos] = v;
                    if (idx) idx[r * ldo + pos] = (I)c;
                    ++pos;
                }
                if (mask) mask[r * ldm + c] = keep ? 1 : 0;
                if (pruned) pruned[r * ldp + c] = keep ? v : from_f32<T>(to_f32(v) * 0.0f);
            }
            if (words) words[r * ldwords + wi] = (int32_t)bits;
        }
        __syncthreads();
    }
}

// ---- mask words -> column indices ----------------------------------------------------------------------------------

template <typename I>
__global__ void __launch_bounds__(kSelBlock) words_to_idx_kernel(const int32_t* __restrict__ words, int64_t rows,
                                                                  int cols, int64_t ldwords, int k, I* __restrict__ idx,
                                                                  int64_t ldi) {
    __shared__ int2 warp_tot[kSelWarps];
    const int tid = threadIdx.x;
    const int n_words = (cols + 31) >> 5;
    const int wpt = (n_words + kSelBlock - 1) / kSelBlock;
    const int w_begin = min(n_words, tid * wpt), w_end = min(n_words, w_begin + wpt);
    const uint32_t tail = (cols & 31) ? ((1u << (cols & 31)) - 1u) : 0xffffffffu;
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const int32_t* wr = words + r * ldwords;
        int cnt = 0, stray = 0;
        for (int wi = w_begin; wi < w_end; ++wi) {
            uint32_t b = (uint32_t)wr[wi];
            if (wi == n_words - 1) {
                stray += __popc(b & ~tail);
                b &= tail;
            }
            cnt += __popc(b);
        }
        int2 tot;
        const int2 before = block_scan2(cnt, stray, warp_tot, tot);
        if (tot.x != k || tot.y != 0) {
            if (tid == 0) atomicAdd(&g_bad_rows, 1);
            continue;
        }
        int64_t pos = before.x;
        for (int wi = w_begin; wi < w_end; ++wi) {
            uint32_t b = (uint32_t)wr[wi];
            if (wi == n_words - 1) b &= tail;
            while (b) {
                const int bit = __ffs(b) - 1;
                b &= b - 1;
                idx[r * ldi + pos++] = (I)(wi * 32 + bit);
            }
        }
    }
}

// ---- uint8 mask -> values + words ----------------------------------------------------------------------------------

template <typename T>
__global__ void __launch_bounds__(kSelBlock) pack_mask_kernel(const T* __restrict__ w, int64_t rows, int cols,
                                                               int64_t ldw, const uint8_t* __restrict__ mask,
                                                               int64_t ldm, int k, T* __restrict__ vals, int64_t ldo,
                                                               int32_t* __restrict__ words, int64_t ldwords) {
    __shared__ int2 warp_tot[kSelWarps];
    const int tid = threadIdx.x;
    const int n_words = (cols + 31) >> 5;
    const int wpt = (n_words + kSelBlock - 1) / kSelBlock;
    const int w_begin = min(n_words, tid * wpt), w_end = min(n_words, w_begin + wpt);
    const int c_begin = w_begin * 32, c_end = min(cols, w_end * 32);
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const uint8_t* mr = mask + r * ldm;
        int cnt = 0;
        for (int c = c_begin; c < c_end; ++c) cnt += mr[c] != 0;
        int2 tot;
        const int2 before = block_scan2(cnt, 0, warp_tot, tot);
        if (tot.x != k) {
            if (tid == 0) atomicAdd(&g_bad_rows, 1);
            continue;
        }
        int64_t pos = before.x;
        for (int wi = w_begin; wi < w_end; ++wi) {
            uint32_t bits = 0;
            for (int b = 0; b < 32 && wi * 32 + b < cols; ++b) {
                const int c = wi * 32 + b;
                if (mr[c]) {
                    bits |= 1u << b;
                    if (vals) vals[r * ldo + pos] = w[r * ldw + c];
                    ++pos;
                }
            }
            if (words) words[r * ldwords + wi] = (int32_t)bits;
        }
    }
}

// ---- values + (words | idx) -> dense -------------------------------------------------------------------------------

template <typename T, typename I>
__global__ void __launch_bounds__(kSelBlock) unpack_kernel(const T* __restrict__ vals, int64_t rows, int k, int64_t ldv,
                                                            const int32_t* __restrict__ words, int64_t ldwords,
                                                            const I* __restrict__ idx, int64_t ldi, int cols,
                                                            T* __restrict__ dense, int64_t ldd) {
    __shared__ int2 warp_tot[kSelWarps];
    const int tid = threadIdx.x;
    const int n_words = (cols + 31) >> 5;
    const int wpt = (n_words + kSelBlock - 1) / kSelBlock;
    const int w_begin = min(n_words, tid * wpt), w_end = min(n_words, w_begin + wpt);
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        T* dr = dense + r * ldd;
        const T* vr = vals + r * ldv;
        if (words) {
            const int32_t* wr = words + r * ldwords;
            int cnt = 0;
            for (int wi = w_begin; wi < w_end; ++wi) cnt += __popc((uint32_t)wr[wi]);
            int2 tot;
            int64_t pos = block_scan2(cnt, 0, warp_tot, tot).x;
            for (int wi = w_begin; wi < w_end; ++wi) {
                const uint32_t b = (uint32_t)wr[wi];
                for (int q = 0; q < 32 && wi * 32 + q < cols; ++q) {
                    const bool on = (b >> q) & 1u;
                    dr[wi * 32 + q] = (on && pos < k) ? vr[pos] : from_f32<T>(0.f);
                    pos += on;
                }
            }
        } else {
            for (int c = tid; c < cols; c += kSelBlock) dr[c] = from_f32<T>(0.f);
            __syncthreads();
            const I* ir = idx + r * ldi;
            for (int j = tid; j < k; j += kSelBlock) {
                const int c = (int)ir[j];
                if (c >= 0 && c < cols) dr[c] = vr[j];
            }
            __syncthreads();
        }
    }
}

// ---- column indices in range and strictly ascending in each row ----------------------------------------------------

template <typename I>
__global__ void check_idx_kernel(const I* __restrict__ idx, int64_t rows, int64_t k, int64_t ldi, int64_t cols) {
    int bad = 0;
    const int64_t n = rows * k;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / k, j = i - r * k;
        const int64_t c = (int64_t)idx[r * ldi + j];
        bad |= (c < 0 || c >= cols);
        if (j > 0) bad |= (int64_t)idx[r * ldi + j - 1] >= c;
    }
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicAdd(&g_bad_rows, 1);
}

int grid_rows(int64_t rows) {
    const int64_t cap = (int64_t)sm_count() * 8;
    return (int)(rows < cap ? rows : cap);
}

int reset_status(cudaStream_t s) {
    const int zero = 0;
    if (cudaMemcpyToSymbolAsync(g_bad_rows, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s) != cudaSuccess)
        return fail(P2P_ECUDA, "status reset failed");
    return P2P_OK;
}

int read_status(cudaStream_t s, int* bad) {
    if (cudaMemcpyFromSymbolAsync(bad, g_bad_rows, sizeof(int), 0, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return fail(P2P_ECUDA, "status read-back failed: %s", cudaGetErrorString(cudaGetLastError()));
    return P2P_OK;
}

}  // namespace
}  // namespace p2p

using namespace p2p;

extern "C" int p2p_wanda_select(const void* w, int dtype, int64_t rows, int64_t cols, int64_t ldw, const float* norms,
                                int64_t norm_group_rows, int64_t k, void* vals, void* idx, int idx_bytes, int64_t ldo,
                                int32_t* words, int64_t ldwords, uint8_t* mask, int64_t ldm, void* pruned, int64_t ldp,
                                void* stream) {
    P2P_REQUIRE(rows >= 0 && cols >= 1, "p2p_wanda_select: shape [%lld, %lld]", (long long)rows, (long long)cols);
    if (cols > kMaxSelCols)
        return fail(P2P_EUNSUPPORTED, "p2p_wanda_select: %lld columns; at most %lld", (long long)cols,
                    (long long)kMaxSelCols);
    P2P_REQUIRE(k >= 1 && k <= cols, "p2p_wanda_select: k=%lld outside [1, %lld]", (long long)k, (long long)cols);
    if (rows == 0) return P2P_OK;
    P2P_REQUIRE(w && norms && ldw >= cols, "p2p_wanda_select: null w/norms or row stride below the columns");
    P2P_REQUIRE(!(vals || idx) || ldo >= k, "p2p_wanda_select: output stride %lld below k=%lld", (long long)ldo,
                (long long)k);
    P2P_REQUIRE(!idx || idx_bytes == 4 || (idx_bytes == 2 && cols <= 32767),
                "p2p_wanda_select: idx_bytes %d for %lld columns (int16 holds up to 32767)", idx_bytes,
                (long long)cols);
    P2P_REQUIRE(!words || ldwords >= (cols + 31) / 32, "p2p_wanda_select: words stride too small");
    P2P_REQUIRE(!mask || ldm >= cols, "p2p_wanda_select: mask stride too small");
    P2P_REQUIRE(!pruned || ldp >= cols, "p2p_wanda_select: pruned stride too small");
    P2P_REQUIRE(norm_group_rows >= 0, "p2p_wanda_select: negative norm_group_rows");
    const int c = (int)cols;
    const int smem = (int)((c + (c >> 5) + 1 + kSelWarps * 256) * sizeof(uint32_t));
    const int grid = grid_rows(rows);
    P2P_DISPATCH(dtype, {
        const scalar_t* wp = reinterpret_cast<const scalar_t*>(w);
        scalar_t* vp = reinterpret_cast<scalar_t*>(vals);
        scalar_t* pp = reinterpret_cast<scalar_t*>(pruned);
        if (idx_bytes == 2 || !idx) {
            auto kern = select_kernel<scalar_t, int16_t>;
            if (int e = allow_smem((const void*)kern, smem, "p2p_wanda_select")) return e;
            kern<<<grid, kSelBlock, smem, as_stream(stream)>>>(wp, rows, c, ldw, norms, norm_group_rows, (int)k, vp,
                                                               reinterpret_cast<int16_t*>(idx), ldo, words, ldwords,
                                                               mask, ldm, pp, ldp);
        } else {
            auto kern = select_kernel<scalar_t, int32_t>;
            if (int e = allow_smem((const void*)kern, smem, "p2p_wanda_select")) return e;
            kern<<<grid, kSelBlock, smem, as_stream(stream)>>>(wp, rows, c, ldw, norms, norm_group_rows, (int)k, vp,
                                                               reinterpret_cast<int32_t*>(idx), ldo, words, ldwords,
                                                               mask, ldm, pp, ldp);
        }
    });
    return launch_status("p2p_wanda_select");
}

extern "C" int p2p_words_to_idx(const int32_t* words, int64_t rows, int64_t cols, int64_t ldwords, int64_t k, void* idx,
                                int idx_bytes, int64_t ldi, void* stream) {
    P2P_REQUIRE(rows >= 0 && cols >= 1 && k >= 1 && k <= cols, "p2p_words_to_idx: bad shape");
    if (rows == 0) return P2P_OK;
    P2P_REQUIRE(words && idx && ldwords >= (cols + 31) / 32 && ldi >= k, "p2p_words_to_idx: null pointer or stride");
    P2P_REQUIRE(idx_bytes == 4 || (idx_bytes == 2 && cols <= 32767), "p2p_words_to_idx: idx_bytes %d", idx_bytes);
    P2P_REQUIRE(cols <= 0x7fffffff, "p2p_words_to_idx: too many columns");
    cudaStream_t s = as_stream(stream);
    if (int e = reset_status(s)) return e;
    if (idx_bytes == 2)
        words_to_idx_kernel<int16_t><<<grid_rows(rows), kSelBlock, 0, s>>>(words, rows, (int)cols, ldwords, (int)k,
                                                                           reinterpret_cast<int16_t*>(idx), ldi);
    else
        words_to_idx_kernel<int32_t><<<grid_rows(rows), kSelBlock, 0, s>>>(words, rows, (int)cols, ldwords, (int)k,
                                                                           reinterpret_cast<int32_t*>(idx), ldi);
    if (int e = launch_status("p2p_words_to_idx")) return e;
    int bad = 0;
    if (int e = read_status(s, &bad)) return e;
    if (bad) return fail(P2P_EDATA, "p2p_words_to_idx: %d rows do not keep exactly k=%lld columns below %lld", bad,
                         (long long)k, (long long)cols);
    return P2P_OK;
}

extern "C" int p2p_pack_mask(const void* w, int dtype, int64_t rows, int64_t cols, int64_t ldw, const uint8_t* mask,
                             int64_t ldm, int64_t k, void* vals, int64_t ldo, int32_t* words, int64_t ldwords,
                             void* stream) {
    P2P_REQUIRE(rows >= 0 && cols >= 1 && k >= 0 && k <= cols, "p2p_pack_mask: bad shape");
    if (rows == 0) return P2P_OK;
    P2P_REQUIRE(w && mask && ldw >= cols && ldm >= cols, "p2p_pack_mask: null pointer or stride");
    P2P_REQUIRE(!vals || ldo >= k, "p2p_pack_mask: values stride");
    P2P_REQUIRE(!words || ldwords >= (cols + 31) / 32, "p2p_pack_mask: words stride");
    P2P_REQUIRE(cols <= 0x7fffffff, "p2p_pack_mask: too many columns");
    cudaStream_t s = as_stream(stream);
    if (int e = reset_status(s)) return e;
    P2P_DISPATCH(dtype, {
        pack_mask_kernel<scalar_t><<<grid_rows(rows), kSelBlock, 0, s>>>(
            reinterpret_cast<const scalar_t*>(w), rows, (int)cols, ldw, mask, ldm, (int)k,
            reinterpret_cast<scalar_t*>(vals), ldo, words, ldwords);
    });
    if (int e = launch_status("p2p_pack_mask")) return e;
    int bad = 0;
    if (int e = read_status(s, &bad)) return e;
    if (bad) return fail(P2P_EDATA, "p2p_pack_mask: %d rows do not keep exactly k=%lld weights", bad, (long long)k);
    return P2P_OK;
}

extern "C" int p2p_unpack(const void* vals, int dtype, int64_t rows, int64_t k, int64_t ldv, const int32_t* words,
                          int64_t ldwords, const void* idx, int idx_bytes, int64_t ldi, int64_t cols, void* dense,
                          int64_t ldd, void* stream) {
    P2P_REQUIRE(rows >= 0 && cols >= 0 && k >= 0, "p2p_unpack: bad shape");
    if (rows == 0 || cols == 0) return P2P_OK;
    P2P_REQUIRE(dense && ldd >= cols, "p2p_unpack: null output or stride");
    P2P_REQUIRE(words || idx, "p2p_unpack: needs mask words or column indices");
    P2P_REQUIRE(k == 0 || (vals && ldv >= k), "p2p_unpack: values");
    P2P_REQUIRE(!words || ldwords >= (cols + 31) / 32, "p2p_unpack: words stride");
    P2P_REQUIRE(words || idx_bytes == 2 || idx_bytes == 4, "p2p_unpack: idx_bytes %d", idx_bytes);
    P2P_REQUIRE(cols <= 0x7fffffff && k <= 0x7fffffff, "p2p_unpack: too large");
    cudaStream_t s = as_stream(stream);
    P2P_DISPATCH(dtype, {
        const scalar_t* vp = reinterpret_cast<const scalar_t*>(vals);
        scalar_t* dp = reinterpret_cast<scalar_t*>(dense);
        if (words || idx_bytes == 2)
            unpack_kernel<scalar_t, int16_t><<<grid_rows(rows), kSelBlock, 0, s>>>(
                vp, rows, (int)k, ldv, words, ldwords, reinterpret_cast<const int16_t*>(idx), ldi, (int)cols, dp, ldd);
        else
            unpack_kernel<scalar_t, int32_t><<<grid_rows(rows), kSelBlock, 0, s>>>(
                vp, rows, (int)k, ldv, words, ldwords, reinterpret_cast<const int32_t*>(idx), ldi, (int)cols, dp, ldd);
    });
    return launch_status("p2p_unpack");
}

extern "C" int p2p_check_idx(const void* idx, int idx_bytes, int64_t rows, int64_t k, int64_t ldi, int64_t cols,
                             void* stream) {
    P2P_REQUIRE(rows >= 0 && k >= 0 && cols >= 1, "p2p_check_idx: bad shape");
    if (rows == 0 || k == 0) return P2P_OK;
    P2P_REQUIRE(idx && ldi >= k && (idx_bytes == 2 || idx_bytes == 4), "p2p_check_idx: bad arguments");
    cudaStream_t s = as_stream(stream);
    if (int e = reset_status(s)) return e;
    const int grid = sm_count() * 4;
    if (idx_bytes == 2)
        check_idx_kernel<int16_t><<<grid, 256, 0, s>>>(reinterpret_cast<const int16_t*>(idx), rows, k, ldi, cols);
    else
        check_idx_kernel<int32_t><<<grid, 256, 0, s>>>(reinterpret_cast<const int32_t*>(idx), rows, k, ldi, cols);
    if (int e = launch_status("p2p_check_idx")) return e;
    int bad = 0;
    if (int e = read_status(s, &bad)) return e;
    if (bad) return fail(P2P_EDATA, "p2p_check_idx: column indices outside [0, %lld) or not ascending", (long long)cols);
    return P2P_OK;
}
