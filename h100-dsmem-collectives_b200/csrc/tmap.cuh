// tmap.cuh -- host-side tiled tensor maps (TMA descriptors) for the sm_100a kernels.
//
// cuTensorMapEncodeTiled is reached through the CUDA runtime's driver entry point, so the library does
// not link against the driver library. The maps are passed to kernels inside __grid_constant__ argument
// structs; the kernels issue cp.async.bulk.tensor loads without multicast.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

namespace dsb_tmap {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

// Encode a tiled map of `rank` dimensions (dims[0] innermost, contiguous); strides[i] is the byte stride of
// dimension i + 1. Elements outside the tensor read as zero. False if the encoder is unavailable or
// rejects the shape.
inline bool encode(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* base, const cuuint64_t* dims,
                   const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapSwizzle swizzle) {
    const EncodeTiledFn enc = encode_fn();
    if (enc == nullptr) return false;
    const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    return enc(m, dt, (cuuint32_t)rank, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace dsb_tmap
