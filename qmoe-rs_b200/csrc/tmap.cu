// tmap.cu -- host-side TMA tensor-map encoding through the driver entry point
// (the library links the static CUDA runtime, not libcuda, so the driver's
// cuTensorMapEncodeTiled is fetched at run time).
#include <cudaTypedefs.h>

#include <mutex>

#include "kernels.h"

namespace qmoe {
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

}  // namespace

bool make_tmap_u8(CUtensorMap *tm, const void *base, uint64_t row_bytes, uint64_t rows,
                  uint32_t box_bytes, uint32_t box_rows, int swizzle) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {row_bytes, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_bytes, box_rows};
    const cuuint32_t elem[2] = {1, 1};
    CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides,
                    box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    static_cast<CUtensorMapSwizzle>(swizzle), CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool make_tmap_u8_3d(CUtensorMap *tm, const void *base, uint64_t d0, uint64_t d1, uint64_t d2,
                     uint64_t stride1, uint64_t stride2, uint32_t b0, uint32_t b1, uint32_t b2,
                     int swizzle) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[3] = {d0, d1, d2};
    const cuuint64_t strides[2] = {stride1, stride2};
    const cuuint32_t box[3] = {b0, b1, b2};
    const cuuint32_t elem[3] = {1, 1, 1};
    CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides,
                    box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    static_cast<CUtensorMapSwizzle>(swizzle), CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool make_tmap_u8_4d(CUtensorMap *tm, const void *base, const uint64_t (&dims)[4],
                     const uint64_t (&strides)[3], const uint32_t (&box)[4], int swizzle) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t d[4] = {dims[0], dims[1], dims[2], dims[3]};
    const cuuint64_t st[3] = {strides[0], strides[1], strides[2]};
    const cuuint32_t b[4] = {box[0], box[1], box[2], box[3]};
    const cuuint32_t elem[4] = {1, 1, 1, 1};
    CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void *>(base), d, st, b, elem,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, static_cast<CUtensorMapSwizzle>(swizzle),
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool make_tmap_bf16(CUtensorMap *tm, const void *base, uint64_t cols, uint64_t rows,
                    uint64_t row_stride, uint32_t box_cols, uint32_t box_rows, int swizzle) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {row_stride};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t elem[2] = {1, 1};
    CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims,
                    strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    static_cast<CUtensorMapSwizzle>(swizzle), CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace qmoe
