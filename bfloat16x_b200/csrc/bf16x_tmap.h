// bf16x_tmap.h -- host-side creation of TMA tensor maps.
//
// cuTensorMapEncodeTiled is a driver-API entry point; it is fetched through
// the runtime (cudaGetDriverEntryPoint) so the library needs no link against
// libcuda.  Encoding is a host-only operation (no device work).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

namespace bf16x {

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// Rank-n tiled map without interleave, zero fill out of bounds.  dims/box
// innermost first; strides (bytes) for dims 1..rank-1.
inline bool encode_tiled(CUtensorMap *map, CUtensorMapDataType dt, int rank, const void *base,
                         const cuuint64_t *dims, const cuuint64_t *strides, const cuuint32_t *box,
                         CUtensorMapL2promotion l2 = CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE) {
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn) return false;
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    return fn(map, dt, (cuuint32_t)rank, const_cast<void *>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, l2, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The resident layout [rows][chunks][3 lines of 128 bytes] (row pitch
// row_bytes) as a rank-4 map of u32 with the 128-byte swizzle: a box of
// `box_rows` rows x one chunk lands as 3 * box_rows swizzled 128-byte lines.
inline bool encode_resident_map(CUtensorMap *map, const void *layout, int64_t rows, int64_t nch,
                                int64_t row_bytes, int box_rows) {
    const cuuint64_t dims[4] = {32u, 3u, (cuuint64_t)nch, (cuuint64_t)rows};
    const cuuint64_t strides[3] = {128u, 384u, (cuuint64_t)row_bytes};
    const cuuint32_t box[4] = {32u, 3u, 1u, (cuuint32_t)box_rows};
    return encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, layout, dims, strides, box,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace bf16x
