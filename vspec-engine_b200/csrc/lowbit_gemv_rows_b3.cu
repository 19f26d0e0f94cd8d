// lowbit_gemv_rows_b3.cu -- the int3 instantiations of the row-sliced GEMV
// (lowbit_gemv_rows.cuh); one file per bit width so they compile in parallel.
#include "lowbit_gemv_rows_launch.cuh"

namespace vb200 {
template cudaError_t rows_launch_bits<3>(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                                         const GemvParams&, const RowsGeom&, size_t, bool, bool, cudaStream_t, bool);
template int rows_timeout_bits<3>(int*);
}  // namespace vb200
