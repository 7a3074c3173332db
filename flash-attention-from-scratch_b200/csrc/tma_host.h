#pragma once
// Host-side TMA tensor-map encoding for [heads][rows][head_dim] fp16 / bf16 tensors.
// cuTensorMapEncodeTiled is fetched through the runtime's driver entry point, so the library
// does not link libcuda directly.

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <mutex>

namespace fa_sm100 {

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000,
                                             cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        }
    });
    return fn;
}

// 3-D map over a contiguous [heads][rows][head_dim] fp16 (bf16: bfloat16) tensor: dims
// (innermost first) {head_dim, rows, heads}, box {64, box_rows, 1}, 128-byte swizzle, zero fill
// out of bounds. Out-of-range rows of a head are zero-filled on load and dropped on store, per
// head.
inline CUresult encode_bhnd_map(CUtensorMap* map, const void* base, int heads, int rows,
                                int head_dim, int box_rows, bool bf16 = false) {
    auto fn = tensor_map_encoder();
    if (fn == nullptr) {
        return CUDA_ERROR_NOT_SUPPORTED;
    }
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(head_dim), static_cast<cuuint64_t>(rows),
                                static_cast<cuuint64_t>(heads)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(head_dim) * 2,
                                   static_cast<cuuint64_t>(rows) * head_dim * 2};
    const cuuint32_t box[3] = {64, static_cast<cuuint32_t>(box_rows), 1};
    const cuuint32_t elem_strides[3] = {1, 1, 1};
    const CUtensorMapDataType type = bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    return fn(map, type, 3, const_cast<void*>(base), dims, strides, box, elem_strides,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

// 3-D map over a contiguous [dim2][dim1][dim0] tensor of bytes (e4m3 elements): box {box0,
// box1, 1}, 128-byte swizzle (box0 = 128), zero fill out of bounds. dim0 must be a multiple of
// 16 (the row stride is dim0 bytes).
inline CUresult encode_u8_map(CUtensorMap* map, const void* base, int dim0, int dim1, int dim2, int box0,
                              int box1) {
    auto fn = tensor_map_encoder();
    if (fn == nullptr) {
        return CUDA_ERROR_NOT_SUPPORTED;
    }
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(dim0), static_cast<cuuint64_t>(dim1),
                                static_cast<cuuint64_t>(dim2)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(dim0),
                                   static_cast<cuuint64_t>(dim1) * static_cast<cuuint64_t>(dim0)};
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(box0), static_cast<cuuint32_t>(box1), 1};
    const cuuint32_t elem_strides[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, elem_strides,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

}  // namespace fa_sm100
