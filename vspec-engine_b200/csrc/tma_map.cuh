// tma_map.cuh -- host-side helper that encodes a 2-D TMA tensor map over a
// row-major byte matrix (packed weight rows), through the driver entry point
// the runtime exposes (no link-time dependency on a particular libcuda).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace vb200 {

static inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
    return fn;
}

// Tiles of box_rows rows x box_bytes bytes of a [rows][row_bytes] uint8 matrix.
// Rows past the end read as zero.
static inline int make_row_tile_map(CUtensorMap* map, const uint8_t* base, int rows, int row_bytes, int box_bytes,
                                    int box_rows, CUtensorMapSwizzle swizzle) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc) { set_error("cuTensorMapEncodeTiled unavailable"); return VSPEC_B200_ERR_CUDA; }
    cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    cuuint32_t box[2] = {(cuuint32_t)box_bytes, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) { set_error("cuTensorMapEncodeTiled failed (%d)", (int)r); return VSPEC_B200_ERR_CUDA; }
    return VSPEC_B200_OK;
}

}  // namespace vb200
