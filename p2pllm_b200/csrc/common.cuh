// Shared helpers of the p2p_b200 kernels: dtype traits, conversions, error reporting.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/p2p_b200.h"

namespace p2p {

// Records a printf-style message as this host thread's last error and returns `code`.
int fail(int code, const char* fmt, ...);
// P2P_OK if the last launch succeeded, else P2P_ECUDA with the CUDA error named after `what`.
int launch_status(const char* what);
// Opts a kernel into `bytes` of dynamic shared memory (once per kernel and size class); P2P_ECUDA on failure.
int allow_smem(const void* kernel, int bytes, const char* what);
// The number of SMs of the current device (cached per device).
int sm_count();

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline int dtype_size(int dtype) { return dtype == P2P_F32 ? 4 : 2; }
inline bool dtype_ok(int dtype) { return dtype == P2P_BF16 || dtype == P2P_F16 || dtype == P2P_F32; }

template <typename T> struct Elem;
template <> struct Elem<__nv_bfloat16> {
    static __device__ __forceinline__ float f32(__nv_bfloat16 v) { return __bfloat162float(v); }
    static __device__ __forceinline__ __nv_bfloat16 from(float v) { return __float2bfloat16_rn(v); }
};
template <> struct Elem<__half> {
    static __device__ __forceinline__ float f32(__half v) { return __half2float(v); }
    static __device__ __forceinline__ __half from(float v) { return __float2half_rn(v); }
};
template <> struct Elem<float> {
    static __device__ __forceinline__ float f32(float v) { return v; }
    static __device__ __forceinline__ float from(float v) { return v; }
};

template <typename T> __device__ __forceinline__ float to_f32(T v) { return Elem<T>::f32(v); }
template <typename T> __device__ __forceinline__ T from_f32(float v) { return Elem<T>::from(v); }

// Two bf16 / f16 packed in a 32-bit word, as fp32 (low half first).
template <typename T> __device__ __forceinline__ float2 unpack2(uint32_t w);
template <> __device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t w) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <> __device__ __forceinline__ float2 unpack2<__half>(uint32_t w) {
    __half2 h = *reinterpret_cast<__half2*>(&w);
    return __half22float2(h);
}

__host__ __device__ __forceinline__ bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace p2p

// Dispatch on the element type: runs `body` with `scalar_t` bound to the C++ type of `dtype`.
#define P2P_DISPATCH(dtype, ...)                                   \
    switch (dtype) {                                               \
        case P2P_BF16: { using scalar_t = __nv_bfloat16; __VA_ARGS__; break; } \
        case P2P_F16: { using scalar_t = __half; __VA_ARGS__; break; }         \
        case P2P_F32: { using scalar_t = float; __VA_ARGS__; break; }          \
        default: return p2p::fail(P2P_EUNSUPPORTED, "dtype %d: bf16 (0), f16 (1) or f32 (2)", (int)(dtype)); \
    }

#define P2P_REQUIRE(cond, ...) \
    do { if (!(cond)) return p2p::fail(P2P_EINVAL, __VA_ARGS__); } while (0)
