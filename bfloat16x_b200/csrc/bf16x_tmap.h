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

// Rank-n tiled map without swizzle or interleave, zero fill out of bounds.
// dims/box innermost first; strides (bytes) for dims 1..rank-1.
inline bool encode_tiled(CUtensorMap *map, CUtensorMapDataType dt, int rank, const void *base,
                         const cuuint64_t *dims, const cuuint64_t *strides, const cuuint32_t *box,
                         CUtensorMapL2promotion l2 = CU_TENSOR_MAP_L2_PROMOTION_L2_256B) {
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn) return false;
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    return fn(map, dt, (cuuint32_t)rank, const_cast<void *>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, l2,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace bf16x
