// The elementwise pieces of the group combine, the spread-step parts and the hop: one member value per element,
// computed in fp32 from every operand, rounded the way p2p/replica.py:81-85 and p2p/route.py:825-831 round.
#pragma once

#include "common.cuh"

namespace p2p {

constexpr int kMaxParts = 16;

struct Parts {
    const void* p[kMaxParts];
    int n;
};

// kReplica: float(p0) + sum over middle members of dtype(float(pk) - float(h)) + dtype(float(p_last) - float(hc))
// kSum:     float(p0) + float(p1) + ... in member order
// kDiff:    float(p0) - float(h)                                (a member's part before its rounding)
enum Mode { kReplica = 0, kSum = 1, kDiff = 2 };

template <typename T> __device__ __forceinline__ float rnd(float v) { return to_f32(from_f32<T>(v)); }

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

template <typename T, int VEC> __device__ __forceinline__ uint4 pack_vec(const float (&v)[VEC]) {
    static_assert(VEC * sizeof(T) == 16, "16-byte vectors");
    uint4 raw;
    T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int q = 0; q < VEC; ++q) e[q] = from_f32<T>(v[q]);
    return raw;
}

template <typename T, int VEC>
__device__ __forceinline__ void store_vec(void* base, int64_t i, const float (&v)[VEC]) {
    T* p = reinterpret_cast<T*>(base) + i;
    if constexpr (VEC == 1) {
        p[0] = from_f32<T>(v[0]);
    } else {
        *reinterpret_cast<uint4*>(p) = pack_vec<T, VEC>(v);
    }
}

// The fp32 value of elements [i, i + VEC) under MODE (before the final rounding to T).
template <typename T, int VEC, int MODE>
__device__ __forceinline__ void member_value(const Parts& parts, const void* h, const void* hc, int64_t i,
                                             float (&total)[VEC]) {
    float a[VEC];
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
}

// Copies `n` part pointers into p (1..kMaxParts, none null); P2P_EINVAL otherwise.
inline int fill_parts(Parts& p, const void* const* parts, int n) {
    if (!parts || n < 1 || n > kMaxParts) return fail(P2P_EINVAL, "1 to %d parts", kMaxParts);
    p.n = n;
    for (int k = 0; k < n; ++k) {
        if (!parts[k]) return fail(P2P_EINVAL, "part %d is null", k);
        p.p[k] = parts[k];
    }
    return P2P_OK;
}

}  // namespace p2p
