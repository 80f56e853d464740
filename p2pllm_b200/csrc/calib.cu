// (1a) Wanda calibration: per-input-channel sums of squares, the reduction behind p2p/wanda.py:37-40
// (Calibration._linear: x.float().pow(2).sum(0).double(), accumulated by _add at wanda.py:34-35) and the `into` half of
// p2p/wanda.py:10-20 (expert_inputs).
//
// HBM-bound: every element of x is read once with 16-byte loads. A block owns a strip of 32 * VEC columns and a slab
// of rows; each thread squares in fp32, adds 16 rows at a time in fp32 and folds them into fp64. The slabs of a strip
// meet in the workspace: each writes its fp64 partial there, and the last slab to finish (a ticket counter per strip)
// adds the partials in slab order, rounds the column total to fp32 as the reference's fp32 sum does, and adds it to
// the caller's fp64 sums. The result therefore does not depend on which block finishes first.
#include "common.cuh"

namespace p2p {
namespace {

constexpr int kBlock = 256;              // 8 warps
constexpr int kWarps = kBlock / 32;
constexpr int kFold = 16;                // rows added in fp32 before folding into fp64
constexpr int kTargetBlocks = 148 * 8;   // enough blocks to keep every SM's loads in flight
constexpr int kMaxSlabs = 512;

template <typename T> struct Vec { static constexpr int n = 16 / sizeof(T); };

// Squares of VEC consecutive elements at p (16-byte aligned when VEC > 1), in fp32.
template <typename T, int VEC>
__device__ __forceinline__ void load_squares(const T* p, float (&sq)[VEC]) {
    if constexpr (VEC == 1) {
        const float v = to_f32(p[0]);
        sq[0] = v * v;
    } else {
        const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
        if constexpr (sizeof(T) == 4) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float v = __uint_as_float(w[i]);
                sq[i] = v * v;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 v = unpack2<T>(w[i]);
                sq[2 * i] = v.x * v.x;
                sq[2 * i + 1] = v.y * v.y;
            }
        }
    }
}

template <typename T, int VEC>
__global__ void __launch_bounds__(kBlock) sumsq_kernel(const T* __restrict__ x, int64_t tokens, int64_t cols, int64_t ldx,
                                                        int64_t rows_per_slab, double* __restrict__ sums,
                                                        double* __restrict__ partial, unsigned* __restrict__ tickets) {
    __shared__ double red[kWarps][32 * VEC];
    __shared__ bool last;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int strip = blockIdx.x, slab = blockIdx.y, nslabs = gridDim.y;
    const int64_t c0 = (int64_t)strip * 32 * VEC + lane * VEC;
    const bool active = c0 < cols;
    const int64_t r_begin = (int64_t)slab * rows_per_slab;
    const int64_t r_end = min(tokens, r_begin + rows_per_slab);

    double acc[VEC];
#pragma unroll
    for (int i = 0; i < VEC; ++i) acc[i] = 0.0;
    if (active) {
        int64_t r = r_begin + warp;
        while (r < r_end) {
            float part[VEC];
#pragma unroll
            for (int i = 0; i < VEC; ++i) part[i] = 0.f;
#pragma unroll 4
            for (int f = 0; f < kFold && r < r_end; ++f, r += kWarps) {
                float sq[VEC];
                load_squares<T, VEC>(x + r * ldx + c0, sq);
#pragma unroll
                for (int i = 0; i < VEC; ++i) part[i] += sq[i];
            }
#pragma unroll
            for (int i = 0; i < VEC; ++i) acc[i] += (double)part[i];
        }
    }
#pragma unroll
    for (int i = 0; i < VEC; ++i) red[warp][lane * VEC + i] = acc[i];
    __syncthreads();

    // Column c of the strip: the slab's total over its warps, in warp order.
    const int t = threadIdx.x;
    for (int j = t; j < 32 * VEC; j += kBlock) {
        const int64_t c = (int64_t)strip * 32 * VEC + j;
        double total = 0.0;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) total += red[w][j];
        if (c >= cols) continue;
        if (nslabs == 1) {
            sums[c] += (double)(float)total;
        } else {
            partial[(int64_t)slab * cols + c] = total;
        }
    }
    if (nslabs == 1) return;
    __threadfence();
    __syncthreads();
    if (t == 0) last = atomicAdd(&tickets[strip], 1u) == (unsigned)(nslabs - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int j = t; j < 32 * VEC; j += kBlock) {
        const int64_t c = (int64_t)strip * 32 * VEC + j;
        if (c >= cols) continue;
        double total = 0.0;
        for (int s = 0; s < nslabs; ++s) total += __ldcg(partial + (int64_t)s * cols + c);
        sums[c] += (double)(float)total;
    }
    if (t == 0) tickets[strip] = 0u;       // the workspace is zeroed again for the next call
}

struct SumsqShape {
    int vec;
    int64_t strips, slabs, rows_per_slab;
};

SumsqShape sumsq_shape(int64_t tokens, int64_t cols, int vec) {
    SumsqShape s;
    s.vec = vec;
    s.strips = (cols + 32 * vec - 1) / (32 * vec);
    int64_t slabs = (kTargetBlocks + s.strips - 1) / s.strips;
    const int64_t by_rows = (tokens + 63) / 64;      // at least 64 rows a slab
    slabs = slabs < by_rows ? slabs : by_rows;
    slabs = slabs < kMaxSlabs ? slabs : kMaxSlabs;
    slabs = slabs < 1 ? 1 : slabs;
    s.rows_per_slab = (tokens + slabs - 1) / slabs;
    if (s.rows_per_slab < 1) s.rows_per_slab = 1;
    s.slabs = (tokens + s.rows_per_slab - 1) / s.rows_per_slab;
    if (s.slabs < 1) s.slabs = 1;
    return s;
}

// The workspace: a fixed region of ticket counters (so that no call's partials ever overlap another call's
// counters, whatever the shapes) and the fp64 partials after it.
constexpr int64_t kMaxStrips = 16384;
constexpr size_t kTicketRegion = kMaxStrips * sizeof(unsigned);

size_t workspace_for(const SumsqShape& s, int64_t cols) {
    if (s.slabs <= 1) return 0;
    return kTicketRegion + (size_t)s.slabs * cols * sizeof(double);
}

// The vectorised kernel needs 16-byte aligned rows; anything else takes the one-element-a-thread variant.
int pick_vec(const void* x, int dtype, int64_t cols, int64_t ldx) {
    const int vec = 16 / dtype_size(dtype);
    if (x && (reinterpret_cast<uintptr_t>(x) & 15u)) return 1;
    if (cols % vec || ldx % vec) return 1;
    return vec;
}

// ---- per-expert sums: one block per (strip, expert) over the expert's routed tokens ------------------------------

template <typename T, int VEC>
__global__ void __launch_bounds__(kBlock) expert_sumsq_kernel(const T* __restrict__ x, int64_t cols, int64_t ldx,
                                                               const int64_t* __restrict__ order,
                                                               const int64_t* __restrict__ seg, int64_t topk,
                                                               double* __restrict__ into) {
    __shared__ double red[kWarps][32 * VEC];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int strip = blockIdx.x;
    const int64_t e = blockIdx.y;
    const int64_t c0 = (int64_t)strip * 32 * VEC + lane * VEC;
    const int64_t i0 = seg[e], i1 = seg[e + 1];
    double acc[VEC];
#pragma unroll
    for (int i = 0; i < VEC; ++i) acc[i] = 0.0;
    if (c0 < cols) {
        int64_t i = i0 + warp;
        while (i < i1) {
            float part[VEC];
#pragma unroll
            for (int q = 0; q < VEC; ++q) part[q] = 0.f;
            for (int f = 0; f < kFold && i < i1; ++f, i += kWarps) {
                const int64_t tok = order[i] / topk;
                if (i > i0 && order[i - 1] / topk == tok) continue;   // the token routed twice to e counts once
                float sq[VEC];
                load_squares<T, VEC>(x + tok * ldx + c0, sq);
#pragma unroll
                for (int q = 0; q < VEC; ++q) part[q] += sq[q];
            }
#pragma unroll
            for (int q = 0; q < VEC; ++q) acc[q] += (double)part[q];
        }
    }
#pragma unroll
    for (int q = 0; q < VEC; ++q) red[warp][lane * VEC + q] = acc[q];
    __syncthreads();
    for (int j = threadIdx.x; j < 32 * VEC; j += kBlock) {
        const int64_t c = (int64_t)strip * 32 * VEC + j;
        if (c >= cols) continue;
        double total = 0.0;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) total += red[w][j];
        into[e * cols + c] += (double)(float)total;
    }
}

// ---- channel norms -----------------------------------------------------------------------------------------------

__global__ void __launch_bounds__(kBlock) norms_kernel(const double* __restrict__ sums, int64_t cols, int experts,
                                                        float* __restrict__ norms) {
    __shared__ float wsum[kWarps];
    __shared__ bool zero;
    const int64_t g = blockIdx.x;
    const double* s = sums + g * cols;
    float* n = norms + g * cols;
    float local = 0.f;
    for (int64_t c = threadIdx.x; c < cols; c += kBlock) {
        const float v = (float)sqrt(s[c]);
        n[c] = v;
        local += v;
    }
    if (!experts) return;
    // An expert whose norms add up to zero (no token reached it) keeps its weights by size alone: norms of one.
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) local += __shfl_xor_sync(0xffffffffu, local, d);
    if ((threadIdx.x & 31) == 0) wsum[threadIdx.x >> 5] = local;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int w = 0; w < kWarps; ++w) t += wsum[w];
        zero = !(t > 0.f);
    }
    __syncthreads();
    if (zero)
        for (int64_t c = threadIdx.x; c < cols; c += kBlock) n[c] = 1.0f;
}

}  // namespace

// ---- the reduction with its scratch inside the library ----------------------------------------------------------
//
// Some callers cannot allocate device memory: the calibration hook runs inside an SGLang forward pass, after SGLang
// has reserved its static share of the GPU for weights and the KV pool, where an extra allocation can fail or
// fragment what is left. For them the scratch lives in this fixed array: 4 MiB of fp64 partials plus 4 KiB of ticket
// counters, enough for up to 16,384 columns. Every GPU that loads the library holds one copy until the process exits.
constexpr int64_t kNoAllocMaxCols = 16384;
constexpr size_t kNoAllocTicketBytes = 4096;                      // 1024 strips' counters (16,384 columns need 512)
constexpr size_t kNoAllocPartialBytes = 4u << 20;
static __device__ __align__(256) unsigned char g_sumsq_scratch[kNoAllocTicketBytes + kNoAllocPartialBytes];

namespace {
// The device address of g_sumsq_scratch in the current device's context (the host-side name of a __device__ array is
// only a stand-in, not an address a kernel may use). Looked up on every call: once the module is loaded the lookup
// is cheap, and a cached address would go stale if the context were torn down and created again.
int scratch_address(void** out) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_sumsq_scratch);
    if (e != cudaSuccess || !ptr)
        return fail(P2P_ECUDA, "p2p_sumsq_cols_noalloc: scratch address lookup failed: %s", cudaGetErrorString(e));
    *out = ptr;
    return P2P_OK;
}
}  // namespace

}  // namespace p2p

using namespace p2p;

extern "C" int p2p_sumsq_cols_noalloc(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ldx,
                                      double* sums, void* stream) {
    P2P_REQUIRE(tokens >= 0 && cols >= 0, "p2p_sumsq_cols_noalloc: negative shape [%lld, %lld]", (long long)tokens,
                (long long)cols);
    if (tokens == 0 || cols == 0) return P2P_OK;
    P2P_REQUIRE(x && sums, "p2p_sumsq_cols_noalloc: null x or sums");
    P2P_REQUIRE(ldx >= cols, "p2p_sumsq_cols_noalloc: row stride %lld below %lld columns", (long long)ldx,
                (long long)cols);
    if (!dtype_ok(dtype)) return fail(P2P_EUNSUPPORTED, "p2p_sumsq_cols_noalloc: dtype %d", dtype);
    if (cols > kNoAllocMaxCols)
        return fail(P2P_EUNSUPPORTED, "p2p_sumsq_cols_noalloc: %lld columns; its built-in scratch holds at most %lld "
                    "(use p2p_sumsq_cols with a workspace)", (long long)cols, (long long)kNoAllocMaxCols);
    const int vec = pick_vec(x, dtype, cols, ldx);
    SumsqShape s = sumsq_shape(tokens, cols, vec);
    // Fewer, taller slabs when the usual split would not fit the fixed scratch.
    const int64_t max_slabs = (int64_t)(kNoAllocPartialBytes / ((size_t)cols * sizeof(double)));
    if (s.slabs > max_slabs) {
        s.rows_per_slab = (tokens + max_slabs - 1) / max_slabs;
        s.slabs = (tokens + s.rows_per_slab - 1) / s.rows_per_slab;
    }
    void* scratch = nullptr;
    if (int e = scratch_address(&scratch)) return e;
    unsigned* tickets = reinterpret_cast<unsigned*>(scratch);
    double* partial = reinterpret_cast<double*>(reinterpret_cast<char*>(scratch) + kNoAllocTicketBytes);
    cudaStream_t st = as_stream(stream);
    // The array keeps whatever the last call left: the counters must start at zero.
    if (s.slabs > 1 && cudaMemsetAsync(tickets, 0, (size_t)s.strips * sizeof(unsigned), st) != cudaSuccess)
        return launch_status("p2p_sumsq_cols_noalloc: clearing the counters");
    const dim3 grid((unsigned)s.strips, (unsigned)s.slabs);
    P2P_DISPATCH(dtype, {
        const scalar_t* xp = reinterpret_cast<const scalar_t*>(x);
        if (vec == 1)
            sumsq_kernel<scalar_t, 1><<<grid, kBlock, 0, st>>>(xp, tokens, cols, ldx, s.rows_per_slab, sums, partial,
                                                               tickets);
        else
            sumsq_kernel<scalar_t, Vec<scalar_t>::n><<<grid, kBlock, 0, st>>>(xp, tokens, cols, ldx, s.rows_per_slab,
                                                                              sums, partial, tickets);
    });
    return launch_status("p2p_sumsq_cols_noalloc");
}

extern "C" size_t p2p_sumsq_workspace(int64_t tokens, int64_t cols, int dtype) {
    if (tokens <= 0 || cols <= 0 || !dtype_ok(dtype)) return 0;
    // The workspace is sized for the widest vector the shape allows; a narrower variant needs no more.
    const int vec = 16 / dtype_size(dtype);
    const SumsqShape a = sumsq_shape(tokens, cols, vec), b = sumsq_shape(tokens, cols, 1);
    const size_t wa = workspace_for(a, cols), wb = workspace_for(b, cols);
    return wa > wb ? wa : wb;
}

extern "C" int p2p_sumsq_cols(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ldx, double* sums,
                              void* workspace, size_t workspace_bytes, void* stream) {
    P2P_REQUIRE(tokens >= 0 && cols >= 0, "p2p_sumsq_cols: negative shape [%lld, %lld]", (long long)tokens,
                (long long)cols);
    if (tokens == 0 || cols == 0) return P2P_OK;
    P2P_REQUIRE(x && sums, "p2p_sumsq_cols: null x or sums");
    P2P_REQUIRE(ldx >= cols, "p2p_sumsq_cols: row stride %lld below %lld columns", (long long)ldx, (long long)cols);
    if (!dtype_ok(dtype)) return fail(P2P_EUNSUPPORTED, "p2p_sumsq_cols: dtype %d", dtype);
    const int vec = pick_vec(x, dtype, cols, ldx);
    const SumsqShape s = sumsq_shape(tokens, cols, vec);
    const size_t need = workspace_for(s, cols);
    P2P_REQUIRE(workspace_bytes >= need && (need == 0 || workspace),
                "p2p_sumsq_cols: workspace of %zu bytes, %zu needed", workspace_bytes, need);
    if (s.strips > kMaxStrips)
        return fail(P2P_EUNSUPPORTED, "p2p_sumsq_cols: %lld columns is too many", (long long)cols);
    unsigned* tickets = reinterpret_cast<unsigned*>(workspace);
    double* partial = need ? reinterpret_cast<double*>(reinterpret_cast<char*>(workspace) + kTicketRegion) : nullptr;
    const dim3 grid((unsigned)s.strips, (unsigned)s.slabs);
    P2P_DISPATCH(dtype, {
        const scalar_t* xp = reinterpret_cast<const scalar_t*>(x);
        if (vec == 1)
            sumsq_kernel<scalar_t, 1><<<grid, kBlock, 0, as_stream(stream)>>>(xp, tokens, cols, ldx, s.rows_per_slab,
                                                                             sums, partial, tickets);
        else
            sumsq_kernel<scalar_t, Vec<scalar_t>::n><<<grid, kBlock, 0, as_stream(stream)>>>(
                xp, tokens, cols, ldx, s.rows_per_slab, sums, partial, tickets);
    });
    return launch_status("p2p_sumsq_cols");
}

extern "C" int p2p_expert_sumsq(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ldx,
                                const int64_t* order, const int64_t* seg, int64_t topk, int64_t n_experts,
                                double* into, void* stream) {
    P2P_REQUIRE(tokens >= 0 && cols >= 0 && topk >= 1 && n_experts >= 1, "p2p_expert_sumsq: bad shape");
    if (tokens == 0 || cols == 0) return P2P_OK;
    P2P_REQUIRE(x && order && seg && into, "p2p_expert_sumsq: null pointer");
    P2P_REQUIRE(ldx >= cols, "p2p_expert_sumsq: row stride below the columns");
    P2P_REQUIRE(n_experts <= 65535, "p2p_expert_sumsq: at most 65535 experts");
    if (!dtype_ok(dtype)) return fail(P2P_EUNSUPPORTED, "p2p_expert_sumsq: dtype %d", dtype);
    const int vec = pick_vec(x, dtype, cols, ldx);
    const int64_t strips = (cols + 32 * vec - 1) / (32 * vec);
    const dim3 grid((unsigned)strips, (unsigned)n_experts);
    P2P_DISPATCH(dtype, {
        const scalar_t* xp = reinterpret_cast<const scalar_t*>(x);
        if (vec == 1)
            expert_sumsq_kernel<scalar_t, 1><<<grid, kBlock, 0, as_stream(stream)>>>(xp, cols, ldx, order, seg, topk,
                                                                                    into);
        else
            expert_sumsq_kernel<scalar_t, Vec<scalar_t>::n><<<grid, kBlock, 0, as_stream(stream)>>>(
                xp, cols, ldx, order, seg, topk, into);
    });
    return launch_status("p2p_expert_sumsq");
}

extern "C" int p2p_channel_norms(const double* sums, int64_t groups, int64_t cols, int experts, float* norms,
                                 void* stream) {
    P2P_REQUIRE(groups >= 0 && cols >= 0, "p2p_channel_norms: negative shape");
    if (groups == 0 || cols == 0) return P2P_OK;
    P2P_REQUIRE(sums && norms, "p2p_channel_norms: null pointer");
    P2P_REQUIRE(groups <= 0x7fffffff, "p2p_channel_norms: too many groups");
    norms_kernel<<<(unsigned)groups, kBlock, 0, as_stream(stream)>>>(sums, cols, experts, norms);
    return launch_status("p2p_channel_norms");
}
