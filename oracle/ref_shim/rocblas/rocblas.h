/* Build shim (oracle only): declarations of the rocBLAS names used by emugemm-cdna's src/emugemm.cpp.
 * rocblas_gemm_ex is a stub that returns rocblas_status_not_implemented (oracle/ref_stub.cu); the planner
 * and model functions of the reference never reach it. */
#pragma once
#include <stdint.h>

typedef int32_t rocblas_int;
typedef struct _rocblas_handle* rocblas_handle;

typedef enum {
    rocblas_status_success = 0,
    rocblas_status_invalid_handle = 1,
    rocblas_status_not_implemented = 2,
    rocblas_status_invalid_pointer = 3,
    rocblas_status_invalid_size = 4,
    rocblas_status_memory_error = 5,
    rocblas_status_internal_error = 6
} rocblas_status;

typedef enum { rocblas_operation_none = 111, rocblas_operation_transpose = 112 } rocblas_operation;
typedef enum {
    rocblas_datatype_f16_r = 150,
    rocblas_datatype_f32_r = 151,
    rocblas_datatype_f64_r = 152,
    rocblas_datatype_bf16_r = 168
} rocblas_datatype;
typedef enum { rocblas_gemm_algo_standard = 0, rocblas_gemm_algo_solution_index = 2 } rocblas_gemm_algo;

#ifdef __cplusplus
extern "C" {
#endif
rocblas_status rocblas_gemm_ex(rocblas_handle handle, rocblas_operation transA, rocblas_operation transB,
                               rocblas_int m, rocblas_int n, rocblas_int k, const void* alpha, const void* a,
                               rocblas_datatype a_type, rocblas_int lda, const void* b, rocblas_datatype b_type,
                               rocblas_int ldb, const void* beta, const void* c, rocblas_datatype c_type,
                               rocblas_int ldc, void* d, rocblas_datatype d_type, rocblas_int ldd,
                               rocblas_datatype compute_type, rocblas_gemm_algo algo, int32_t solution_index,
                               uint32_t flags);
#ifdef __cplusplus
}
#endif
