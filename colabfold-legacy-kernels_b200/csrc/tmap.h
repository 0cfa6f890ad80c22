// Host side of TMA: tensor-map encoding through the driver entry point (no link to libcuda).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace cflk {

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (fn == nullptr) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        }
    }
    return fn;
}

// The swizzle mode TMA must use so that a box row of `row_bytes` lands in the layout the MMA
// descriptors expect (32, 64 or 128-byte swizzle atoms).
inline CUtensorMapSwizzle swizzle_for_row(int row_bytes) {
    return row_bytes >= 128 ? CU_TENSOR_MAP_SWIZZLE_128B
           : row_bytes >= 64 ? CU_TENSOR_MAP_SWIZZLE_64B
           : row_bytes >= 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                             : CU_TENSOR_MAP_SWIZZLE_NONE;
}

// A tiled map of rank 1..5. dims and box run innermost first; strides (in elements) are those of
// dims 1..rank-1. Elements outside dims read as zero. Returns false when the driver rejects it.
inline bool encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, int rank,
                         const void* base, const uint64_t* dims, const uint64_t* strides,
                         const uint32_t* box, CUtensorMapSwizzle swizzle) {
    auto fn = tensor_map_encoder();
    if (fn == nullptr) {
        return false;
    }
    cuuint64_t gdim[5], gstride[4];
    cuuint32_t bdim[5], estride[5];
    for (int i = 0; i < rank; ++i) {
        gdim[i] = dims[i];
        bdim[i] = box[i];
        estride[i] = 1;
        if (i > 0) {
            gstride[i - 1] = strides[i - 1] * (uint64_t)elem_bytes;
        }
    }
    const CUresult r = fn(map, dtype, (cuuint32_t)rank, const_cast<void*>(base), gdim, gstride,
                          bdim, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace cflk
