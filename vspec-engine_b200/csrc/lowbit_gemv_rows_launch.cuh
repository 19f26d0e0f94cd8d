// lowbit_gemv_rows_launch.cuh -- launch templates of the row-sliced GEMV,
// included by the per-bit-width translation units lowbit_gemv_rows_b*.cu.
#pragma once

#include "lowbit_gemv_rows.cuh"

namespace vb200 {

template <int BITS, int NT, bool UNS, int EPI, bool SZ16, int NB>
static cudaError_t launch_rows_k(const CUtensorMap& wm, const CUtensorMap& sm, const CUtensorMap& zm,
                                 const GemvParams& p, const RowsGeom& geo, size_t smem, cudaStream_t st, bool pdl) {
    auto kern = lowbit_gemv_rows_kernel<BITS, NT, UNS, EPI, SZ16, NB>;
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kRowsSmemMax);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        if (e != cudaSuccess) return e;
        configured[dev] = 1;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(geo.ctas);
    cfg.blockDim = dim3(kRowsThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, wm, sm, zm, p, geo);
}

template <int BITS, int NT, bool UNS, int EPI, bool SZ16>
static cudaError_t launch_rows_nb(const CUtensorMap& wm, const CUtensorMap& sm, const CUtensorMap& zm,
                                  const GemvParams& p, const RowsGeom& geo, size_t smem, cudaStream_t st, bool pdl) {
    switch (geo.br / 16) {
        case 1: return launch_rows_k<BITS, NT, UNS, EPI, SZ16, 1>(wm, sm, zm, p, geo, smem, st, pdl);
        case 2: return launch_rows_k<BITS, NT, UNS, EPI, SZ16, 2>(wm, sm, zm, p, geo, smem, st, pdl);
        case 3: return launch_rows_k<BITS, NT, UNS, EPI, SZ16, 3>(wm, sm, zm, p, geo, smem, st, pdl);
        case 4: return launch_rows_k<BITS, NT, UNS, EPI, SZ16, 4>(wm, sm, zm, p, geo, smem, st, pdl);
        case 5: return launch_rows_k<BITS, NT, UNS, EPI, SZ16, 5>(wm, sm, zm, p, geo, smem, st, pdl);
        default: return launch_rows_k<BITS, NT, UNS, EPI, SZ16, 6>(wm, sm, zm, p, geo, smem, st, pdl);
    }
}

template <int BITS, int NT, bool UNS, int EPI>
static cudaError_t launch_rows_sz(const CUtensorMap& wm, const CUtensorMap& sm, const CUtensorMap& zm,
                                  const GemvParams& p, const RowsGeom& geo, size_t smem, cudaStream_t st, bool pdl) {
    if (p.flags & VSPEC_B200_F_SZ_F16) return launch_rows_nb<BITS, NT, UNS, EPI, true>(wm, sm, zm, p, geo, smem, st, pdl);
    return launch_rows_nb<BITS, NT, UNS, EPI, false>(wm, sm, zm, p, geo, smem, st, pdl);
}

template <int BITS, int NT>
static cudaError_t launch_rows_nt(const CUtensorMap& wm, const CUtensorMap& sm, const CUtensorMap& zm,
                                  const GemvParams& p, const RowsGeom& geo, size_t smem, bool uns, bool swiglu,
                                  cudaStream_t st, bool pdl) {
    if (uns) return swiglu ? launch_rows_sz<BITS, NT, true, kEpiSwiGLU>(wm, sm, zm, p, geo, smem, st, pdl)
                           : launch_rows_sz<BITS, NT, true, kEpiPlain>(wm, sm, zm, p, geo, smem, st, pdl);
    return swiglu ? launch_rows_sz<BITS, NT, false, kEpiSwiGLU>(wm, sm, zm, p, geo, smem, st, pdl)
                  : launch_rows_sz<BITS, NT, false, kEpiPlain>(wm, sm, zm, p, geo, smem, st, pdl);
}

template <int BITS>
cudaError_t rows_launch_bits(const CUtensorMap& wm, const CUtensorMap& sm, const CUtensorMap& zm,
                             const GemvParams& p, const RowsGeom& geo, size_t smem, bool uns, bool swiglu,
                             cudaStream_t st, bool pdl) {
    if (rows_nt(p.m) == 1) return launch_rows_nt<BITS, 1>(wm, sm, zm, p, geo, smem, uns, swiglu, st, pdl);
    return launch_rows_nt<BITS, 2>(wm, sm, zm, p, geo, smem, uns, swiglu, st, pdl);
}

template <int BITS>
int rows_timeout_bits(int* out) {
    int v = 0, zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_rows_timeout, sizeof(int));
    if (e != cudaSuccess) return cuda_status(e, "read row-sliced GEMV timeout flag");
    e = cudaMemcpyToSymbol(g_rows_timeout, &zero, sizeof(int));
    if (e != cudaSuccess) return cuda_status(e, "clear row-sliced GEMV timeout flag");
    *out = v;
    return VSPEC_B200_OK;
}

}  // namespace vb200
