// Routed experts, the steps around the grouped GEMM (p2p_spmm_tc_grouped): who goes to which expert, and the
// weighted sum of each token's expert outputs. Replaces the torch plumbing of CompactMoE-style routing
// (p2p/compact.py:241-256 leaves it to SGLang's fused MoE): one launch each, no host round trip but the final count.
//
//   p2p_moe_route    the (token, slot) pairs with an expert, sorted by expert and, within an expert, by pair index
//                    (stable): order[p] = pair, where[pair] = p (or -1), counts, and the grouped GEMM's items of at
//                    most 256 tokens {expert, first row, tokens, 0}; meta = {pairs, items, most tokens in an item}
//   p2p_moe_combine  out[t] = dtype(sum over slots j in order of float(w[t, j]) * float(y[where[t K + j]]))
#include "common.cuh"

namespace p2p {
namespace {

constexpr int kRouteThreads = 1024;
constexpr int kItemTokens = 256;
constexpr int kMaxExperts = 8192;

// One CTA: counts by shared atomics (order-free), an exclusive scan over experts, then a stable placement by one warp
// that walks the pairs 32 at a time (lanes with the same expert take consecutive places in lane order).
__global__ void __launch_bounds__(kRouteThreads) route_kernel(const int64_t* __restrict__ ids, int64_t n_pairs,
                                                              int experts, int64_t* __restrict__ order,
                                                              int64_t* __restrict__ where, int32_t* __restrict__ counts,
                                                              int32_t* __restrict__ items, int64_t max_items,
                                                              int64_t* __restrict__ meta) {
    extern __shared__ int sm[];
    int* cnt = sm;                     // [experts]
    int* start = sm + experts;         // [experts + 1]: exclusive scan of cnt
    int* nitem = start + experts + 1;  // [experts + 1]: exclusive scan of items an expert needs
    for (int e = threadIdx.x; e < experts; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int64_t i = threadIdx.x; i < n_pairs; i += blockDim.x) {
        const int64_t e = ids[i];
        if (e >= 0 && e < experts) atomicAdd(&cnt[e], 1);
        where[i] = -1;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int run = 0, runi = 0;
        for (int e = 0; e < experts; ++e) {
            start[e] = run;
            nitem[e] = runi;
            run += cnt[e];
            runi += (cnt[e] + kItemTokens - 1) / kItemTokens;
        }
        start[experts] = run;
        nitem[experts] = runi;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < experts; e += blockDim.x) counts[e] = cnt[e];
    // items, and the largest
    int most = 0;
    for (int e = threadIdx.x; e < experts; e += blockDim.x) {
        int k = nitem[e];
        for (int s = 0; s < cnt[e]; s += kItemTokens, ++k) {
            const int n = cnt[e] - s < kItemTokens ? cnt[e] - s : kItemTokens;
            most = n > most ? n : most;
            if (k < max_items) {
                items[4 * k + 0] = e;
                items[4 * k + 1] = start[e] + s;
                items[4 * k + 2] = n;
                items[4 * k + 3] = 0;
            }
        }
    }
    __syncthreads();
    // stable placement: warp 0, 32 pairs a step; cnt[] is reused as each expert's next free place
    for (int e = threadIdx.x; e < experts; e += blockDim.x) cnt[e] = start[e];
    __syncthreads();
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        const unsigned below = (1u << lane) - 1u;
        for (int64_t i0 = 0; i0 < n_pairs; i0 += 32) {
            const int64_t i = i0 + lane;
            const int64_t e64 = i < n_pairs ? ids[i] : -1;
            const bool ok = e64 >= 0 && e64 < experts;
            const int e = ok ? (int)e64 : experts + lane;         // a key of its own when not routed
            const unsigned peers = __match_any_sync(0xffffffffu, e);
            const int before = __popc(peers & below);
            int base = 0;
            if (ok) base = cnt[e];
            __syncwarp();
            if (ok) {
                const int p = base + before;
                order[p] = i;
                where[i] = p;
                if (before == 0) cnt[e] = base + __popc(peers);
            }
            __syncwarp();
        }
    }
    // the largest item, across the block
    __shared__ int s_most;
    if (threadIdx.x == 0) s_most = 0;
    __syncthreads();
    atomicMax(&s_most, most);
    __syncthreads();
    if (threadIdx.x == 0) {
        meta[0] = start[experts];
        meta[1] = nitem[experts];
        meta[2] = s_most;
    }
}

template <typename T>
__global__ void moe_combine_kernel(const T* __restrict__ y, int64_t ldy, const int64_t* __restrict__ where,
                                   const float* __restrict__ w, int64_t tokens, int k, int64_t hidden,
                                   T* __restrict__ out, int64_t ldo) {
    const int64_t n = tokens * hidden;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = i / hidden, c = i % hidden;
        float acc = 0.f;
        for (int j = 0; j < k; ++j) {
            const int64_t p = where[t * k + j];
            if (p >= 0) acc += w[t * k + j] * to_f32(y[p * ldy + c]);
        }
        out[t * ldo + c] = from_f32<T>(acc);
    }
}

}  // namespace
}  // namespace p2p

using namespace p2p;

extern "C" int p2p_moe_route(const int64_t* ids, int64_t n_pairs, int experts, int64_t* order, int64_t* where,
                             int32_t* counts, int32_t* items, int64_t max_items, int64_t* meta, void* stream) {
    P2P_REQUIRE(n_pairs >= 0 && experts >= 1 && experts <= kMaxExperts, "p2p_moe_route: %lld pairs, %d experts",
                (long long)n_pairs, experts);
    P2P_REQUIRE(ids && order && where && counts && items && meta, "p2p_moe_route: null pointer");
    P2P_REQUIRE(max_items >= (n_pairs + kItemTokens - 1) / kItemTokens + experts,
                "p2p_moe_route: room for %lld items, up to %lld needed", (long long)max_items,
                (long long)((n_pairs + kItemTokens - 1) / kItemTokens + experts));
    const int smem = (int)((3 * (size_t)experts + 2) * sizeof(int));
    if (int e = allow_smem((const void*)route_kernel, smem, "p2p_moe_route")) return e;
    route_kernel<<<1, kRouteThreads, smem, as_stream(stream)>>>(ids, n_pairs, experts, order, where, counts, items,
                                                                max_items, meta);
    return launch_status("p2p_moe_route");
}

extern "C" int p2p_moe_combine(const void* y, int dtype, int64_t ldy, const int64_t* where, const float* weights,
                               int64_t tokens, int k, int64_t hidden, void* out, int64_t ldo, void* stream) {
    P2P_REQUIRE(tokens >= 0 && k >= 1 && hidden >= 1 && ldy >= hidden && ldo >= hidden, "p2p_moe_combine: bad shape");
    if (tokens == 0) return P2P_OK;
    P2P_REQUIRE(y && where && weights && out, "p2p_moe_combine: null pointer");
    const int64_t n = tokens * hidden;
    const int grid = (int)((n + 255) / 256 < sm_count() * 8 ? (n + 255) / 256 : sm_count() * 8);
    cudaStream_t st = as_stream(stream);
    if (dtype == P2P_BF16)
        moe_combine_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(y), ldy, where,
                                                                 weights, tokens, k, hidden,
                                                                 reinterpret_cast<__nv_bfloat16*>(out), ldo);
    else if (dtype == P2P_F16)
        moe_combine_kernel<__half><<<grid, 256, 0, st>>>(reinterpret_cast<const __half*>(y), ldy, where, weights, tokens,
                                                         k, hidden, reinterpret_cast<__half*>(out), ldo);
    else
        return fail(P2P_EUNSUPPORTED, "p2p_moe_combine: bf16 or f16");
    return launch_status("p2p_moe_combine");
}
