// (3) The group-combine epilogue of a replica group and the spread-step parts, one pass over all members' outputs.
//
//   combine      p2p/replica.py:81-85   total = float(l_0(h)); total += dtype(float(l_k(h)) - float(h)) for the middle
//                                       members; total += dtype(float(l_last(h~)) - float(h~)); out = dtype(total)
//   sum_parts    p2p/route.py:825-831   out = dtype(sum of float(parts) in member order)
//   member_part  p2p/route.py:1268-1274 part = dtype(float(y) - float(x))
//
// The reference runs these as 2n separate ATen elementwise ops, each re-reading h; here one kernel reads every
// member's output once, 16 bytes a thread, and keeps the fp32 running sum in registers. Rounding follows the reference
// step for step: each difference is rounded to the model dtype before it is added in fp32.
#include "common.cuh"

namespace p2p {
namespace {

constexpr int kMaxParts = 16;
constexpr int kCombBlock = 256;

struct Parts {
    const void* p[kMaxParts];
    int n;
};

enum Mode { kReplica = 0, kSum = 1, kDiff = 2 };

template <typename T> __device__ __forceinline__ float rnd(float v) { return to_f32(from_f32<T>(v)); }

template <typename T, int VEC> struct Pack {
    T v[VEC];
};

template <typename T, int VEC>
__device__ __forceinline__ void load_vec(const void* base, int64_t i, float (&out)[VEC]) {
    const T* p = reinterpret_cast<const T*>(base) + i;
    if constexpr (VEC == 1) {
        out[0] = to_f32(p[0]);
    } else {
        const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
        const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
        for (int q = 0; q < VEC; ++q) out[q] = to_f32(e[q]);
    }
}

template <typename T, int VEC>
__device__ __forceinline__ void store_vec(void* base, int64_t i, const float (&v)[VEC]) {
    T* p = reinterpret_cast<T*>(base) + i;
    if constexpr (VEC == 1) {
        p[0] = from_f32<T>(v[0]);
    } else {
        uint4 raw;
        T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
        for (int q = 0; q < VEC; ++q) e[q] = from_f32<T>(v[q]);
        *reinterpret_cast<uint4*>(p) = raw;
    }
}

template <typename T, int VEC, int MODE>
__global__ void __launch_bounds__(kCombBlock) combine_kernel(Parts parts, const void* __restrict__ h,
                                                              const void* __restrict__ hc, void* __restrict__ out,
                                                              int64_t n_vec, int64_t offset) {
    for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < n_vec; v += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = offset + v * VEC;
        float total[VEC], a[VEC];
        load_vec<T, VEC>(parts.p[0], i, total);
        if constexpr (MODE == kDiff) {
            load_vec<T, VEC>(h, i, a);
#pragma unroll
            for (int q = 0; q < VEC; ++q) total[q] = total[q] - a[q];
        } else if constexpr (MODE == kSum) {
            for (int k = 1; k < parts.n; ++k) {
                load_vec<T, VEC>(parts.p[k], i, a);
#pragma unroll
                for (int q = 0; q < VEC; ++q) total[q] += a[q];
            }
        } else {
            float hv[VEC];
            if (parts.n > 2) load_vec<T, VEC>(h, i, hv);
            for (int k = 1; k < parts.n - 1; ++k) {
                load_vec<T, VEC>(parts.p[k], i, a);
#pragma unroll
                for (int q = 0; q < VEC; ++q) total[q] += rnd<T>(a[q] - hv[q]);
            }
            float cv[VEC];
            load_vec<T, VEC>(parts.p[parts.n - 1], i, a);
            load_vec<T, VEC>(hc, i, cv);
#pragma unroll
            for (int q = 0; q < VEC; ++q) total[q] += rnd<T>(a[q] - cv[q]);
        }
        store_vec<T, VEC>(out, i, total);
    }
}

template <typename T, int MODE>
int launch_combine(const Parts& parts, const void* h, const void* hc, void* out, int64_t n, cudaStream_t s) {
    constexpr int VEC = 16 / sizeof(T);
    bool vec_ok = aligned16(out) && (!h || aligned16(h)) && (!hc || aligned16(hc));
    for (int k = 0; k < parts.n; ++k) vec_ok = vec_ok && aligned16(parts.p[k]);
    const int64_t n_vec = vec_ok ? n / VEC : 0;
    const int64_t tail = n - n_vec * VEC;
    const int64_t cap = (int64_t)sm_count() * 8;
    if (n_vec) {
        const int64_t blocks = (n_vec + kCombBlock - 1) / kCombBlock;
        combine_kernel<T, VEC, MODE><<<(unsigned)(blocks < cap ? blocks : cap), kCombBlock, 0, s>>>(parts, h, hc, out,
                                                                                                    n_vec, 0);
    }
    if (tail) {
        const int64_t blocks = (tail + kCombBlock - 1) / kCombBlock;
        combine_kernel<T, 1, MODE><<<(unsigned)(blocks < cap ? blocks : cap), kCombBlock, 0, s>>>(parts, h, hc, out,
                                                                                                  tail, n_vec * VEC);
    }
    return launch_status("p2p combine");
}

int fill_parts(Parts& p, const void* const* parts, int n) {
    if (!parts || n < 1 || n > kMaxParts) return fail(P2P_EINVAL, "1 to %d parts", kMaxParts);
    p.n = n;
    for (int k = 0; k < n; ++k) {
        if (!parts[k]) return fail(P2P_EINVAL, "part %d is null", k);
        p.p[k] = parts[k];
    }
    return P2P_OK;
}

}  // namespace
}  // namespace p2p

using namespace p2p;

extern "C" int p2p_combine(const void* const* parts, int n, const void* h, const void* h_copy, void* out, int dtype,
                           int64_t n_elem, void* stream) {
    P2P_REQUIRE(n >= 2, "p2p_combine: a group has at least 2 members, got %d", n);
    P2P_REQUIRE(n_elem >= 0, "p2p_combine: negative size");
    if (n_elem == 0) return P2P_OK;
    Parts p;
    if (int e = fill_parts(p, parts, n)) return e;
    P2P_REQUIRE(out && h_copy && (n == 2 || h), "p2p_combine: null h, h_copy or out");
    P2P_DISPATCH(dtype, { return launch_combine<scalar_t, kReplica>(p, h, h_copy, out, n_elem, as_stream(stream)); });
    return P2P_OK;
}

extern "C" int p2p_sum_parts(const void* const* parts, int n, void* out, int dtype, int64_t n_elem, void* stream) {
    P2P_REQUIRE(n_elem >= 0, "p2p_sum_parts: negative size");
    if (n_elem == 0) return P2P_OK;
    Parts p;
    if (int e = fill_parts(p, parts, n)) return e;
    P2P_REQUIRE(out, "p2p_sum_parts: null out");
    P2P_DISPATCH(dtype, { return launch_combine<scalar_t, kSum>(p, nullptr, nullptr, out, n_elem, as_stream(stream)); });
    return P2P_OK;
}

extern "C" int p2p_member_part(const void* y, const void* x, void* out, int dtype, int64_t n_elem, void* stream) {
    P2P_REQUIRE(n_elem >= 0, "p2p_member_part: negative size");
    if (n_elem == 0) return P2P_OK;
    P2P_REQUIRE(y && x && out, "p2p_member_part: null pointer");
    Parts p;
    p.n = 1;
    p.p[0] = y;
    P2P_DISPATCH(dtype, { return launch_combine<scalar_t, kDiff>(p, x, nullptr, out, n_elem, as_stream(stream)); });
    return P2P_OK;
}
