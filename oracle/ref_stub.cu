// Link stub (oracle only) for the reference planner build: rocblas_gemm_ex is never reached by
// emugemm_plan / emugemm_model_*; if anything calls it, it reports not_implemented.
#include "rocblas/rocblas.h"

extern "C" rocblas_status rocblas_gemm_ex(rocblas_handle, rocblas_operation, rocblas_operation, rocblas_int,
                                          rocblas_int, rocblas_int, const void*, const void*, rocblas_datatype,
                                          rocblas_int, const void*, rocblas_datatype, rocblas_int, const void*,
                                          const void*, rocblas_datatype, rocblas_int, void*, rocblas_datatype,
                                          rocblas_int, rocblas_datatype, rocblas_gemm_algo, int32_t, uint32_t) {
    return rocblas_status_not_implemented;
}
