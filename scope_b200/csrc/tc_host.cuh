// Host helpers of the tensor-core kernels: TMA tensor maps for the bf16
// operand tiles (cuTensorMapEncodeTiled, fetched through the runtime so the
// library needs no link-time libcuda dependency).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace scope {
namespace tchost {

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(f);
    }
    return fn;
}

inline CUtensorMapSwizzle swizzle_for(int row_bytes) {
    return row_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                            : (row_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
}

// [H][T][inner] bf16 tensor with element strides (sh, st), box (box_inner, 128, 1)
inline bool map3d(CUtensorMap *m, const void *base, int inner, int T, int H, int64_t st, int64_t sh, int box_inner) {
    cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)T, (cuuint64_t)H};
    cuuint64_t strides[2] = {(cuuint64_t)(st * 2), (cuuint64_t)(sh * 2)};
    cuuint32_t box[3] = {(cuuint32_t)box_inner, 128u, 1u};
    cuuint32_t es[3] = {1, 1, 1};
    return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides, box, es,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_for(box_inner * 2), CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
// [T][inner] bf16, box (box_inner, 128)
inline bool map2d(CUtensorMap *m, const void *base, int inner, int T, int box_inner) {
    cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)T};
    cuuint64_t strides[1] = {(cuuint64_t)inner * 2};
    cuuint32_t box[2] = {(cuuint32_t)box_inner, 128u};
    cuuint32_t es[2] = {1, 1};
    return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_for(box_inner * 2), CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [rows][inner] fp32 with 64-byte swizzle, box (16, box_rows): the target of
// tensor reduce-adds from 64-byte-swizzled shared-memory boxes
inline bool map2d_f32_sw64(CUtensorMap *m, const void *base, int inner, int64_t rows, int box_rows) {
    cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)inner * 4};
    cuuint32_t box[2] = {16u, (cuuint32_t)box_rows};
    cuuint32_t es[2] = {1, 1};
    return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void *>(base), dims, strides, box, es,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace tchost
}  // namespace scope
