// Host-side pieces of the sm_100a GEMMs (spmm_tc.cu, spmm_mask.cu): TMA descriptors of x and y, and small helpers.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "tc_layout.cuh"

namespace p2p {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
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

inline int pow2_at_least(int v) {
    int p = 32;
    while (p < v) p <<= 1;
    return p;
}

// The TMA map of x [rows, cols] (row stride ldx elements): boxes of 64 columns x box_rows rows, 128-byte swizzle.
inline int encode_x_map(CUtensorMap* map, const void* x, int dtype, int64_t rows, int64_t cols, int64_t ldx, int box_rows) {
    EncodeTiledFn encode = encode_fn();
    if (!encode) return fail(P2P_ECUDA, "cuTensorMapEncodeTiled unavailable");
    const cuuint64_t gdim[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t gstride[1] = {(cuuint64_t)(ldx * 2)};
    const cuuint32_t box[2] = {(cuuint32_t)tc::kTileCols, (cuuint32_t)box_rows};
    const cuuint32_t estride[2] = {1, 1};
    CUresult r = encode(map, dtype == P2P_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                        const_cast<void*>(x), gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(P2P_ECUDA, "x tensor map encode failed (%d)", (int)r);
    return P2P_OK;
}

// The TMA map of y [tokens, rows] (row stride ldy elements) for the epilogue's stores: boxes of 128 rows x box_rows
// tokens, no swizzle.
inline int encode_y_map(CUtensorMap* map, void* y, int dtype, int64_t tokens, int64_t rows, int64_t ldy, int box_rows) {
    EncodeTiledFn encode = encode_fn();
    if (!encode) return fail(P2P_ECUDA, "cuTensorMapEncodeTiled unavailable");
    const cuuint64_t gdim[2] = {(cuuint64_t)rows, (cuuint64_t)tokens};
    const cuuint64_t gstride[1] = {(cuuint64_t)(ldy * 2)};
    const cuuint32_t box[2] = {(cuuint32_t)tc::kTileRows, (cuuint32_t)box_rows};
    const cuuint32_t estride[2] = {1, 1};
    CUresult r = encode(map, dtype == P2P_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, y,
                        gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(P2P_ECUDA, "y tensor map encode failed (%d)", (int)r);
    return P2P_OK;
}


}  // namespace p2p
