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
#include "elementwise.cuh"

namespace p2p {
namespace {

constexpr int kCombBlock = 256;

template <typename T, int VEC, int MODE>
__global__ void __launch_bounds__(kCombBlock) combine_kernel(Parts parts, const void* __restrict__ h,
                                                              const void* __restrict__ hc, void* __restrict__ out,
                                                              int64_t n_vec, int64_t offset) {
    for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < n_vec; v += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = offset + v * VEC;
        float total[VEC];
        member_value<T, VEC, MODE>(parts, h, hc, i, total);
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
