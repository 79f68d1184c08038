/* Build shim (test only): lets emugemm-cdna's own harnesses bench/emugemm_test.cpp and bench/emu_adversarial.cpp
 * compile UNCHANGED against this library's include/emugemm.h, force-included ahead of them (nvcc -include).
 *
 *   - EMUGEMM_ROCBLAS_COMPAT gives the two vendor type names of the reference API (rocblas_handle,
 *     rocblas_status) as typedefs of the library's handle and status types;
 *   - the HIP runtime names the harnesses use map onto the CUDA runtime;
 *   - rocblas_create_handle creates an emugemm handle (what the harnesses then pass to emugemm_sgemm);
 *   - rocblas_gemm_ex, which the harnesses call only for their own FP64 ground truth and their native FP32
 *     comparison, runs cuBLAS's GemmEx with the same column-major arguments (FP64 compute for f64 operands,
 *     plain FP32 compute, no TF32, for f32 operands), on the default stream like the handle.
 * Nothing here is linked into libemugemm.so.
 */
#pragma once

#define EMUGEMM_ROCBLAS_COMPAT 1
#include "emugemm.h"

#include <cublas_v2.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

/* ---- HIP runtime ---- */
typedef cudaError_t hipError_t;
typedef cudaEvent_t hipEvent_t;
#define hipSuccess cudaSuccess
#define hipMalloc cudaMalloc
#define hipFree cudaFree
#define hipMemcpy cudaMemcpy
#define hipMemset cudaMemset
#define hipMemcpyHostToDevice cudaMemcpyHostToDevice
#define hipMemcpyDeviceToHost cudaMemcpyDeviceToHost
#define hipDeviceSynchronize cudaDeviceSynchronize
#define hipGetErrorString cudaGetErrorString
#define hipEventCreate cudaEventCreate
#define hipEventRecord cudaEventRecord
#define hipEventSynchronize cudaEventSynchronize
#define hipEventElapsedTime cudaEventElapsedTime

/* ---- rocBLAS names used by the harnesses ---- */
typedef int32_t rocblas_int;
typedef enum { rocblas_operation_none = 111, rocblas_operation_transpose = 112 } rocblas_operation;
typedef enum {
    rocblas_datatype_f16_r = 150,
    rocblas_datatype_f32_r = 151,
    rocblas_datatype_f64_r = 152,
    rocblas_datatype_bf16_r = 168
} rocblas_datatype;
typedef enum { rocblas_gemm_algo_standard = 0, rocblas_gemm_algo_solution_index = 2 } rocblas_gemm_algo;
typedef enum { rocblas_pointer_mode_host = 0, rocblas_pointer_mode_device = 1 } rocblas_pointer_mode;
#define rocblas_status_success EMUGEMM_STATUS_SUCCESS
#define rocblas_status_not_implemented EMUGEMM_STATUS_NOT_IMPLEMENTED
#define rocblas_status_internal_error EMUGEMM_STATUS_INTERNAL_ERROR

static inline rocblas_status rocblas_create_handle(rocblas_handle* h) { return emugemm_create_handle(h); }
static inline rocblas_status rocblas_destroy_handle(rocblas_handle h) { return emugemm_destroy_handle(h); }
static inline rocblas_status rocblas_set_pointer_mode(rocblas_handle, rocblas_pointer_mode) {
    return rocblas_status_success;   /* scalars are host values, as in the harnesses */
}

static inline cublasHandle_t harness_cublas(void) {
    static cublasHandle_t cb = NULL;
    if (!cb && cublasCreate(&cb) != CUBLAS_STATUS_SUCCESS) {
        fprintf(stderr, "harness shim: cublasCreate failed\n");
        cb = NULL;
    }
    return cb;
}

static inline cudaDataType_t harness_type(rocblas_datatype t) {
    switch (t) {
        case rocblas_datatype_f16_r: return CUDA_R_16F;
        case rocblas_datatype_bf16_r: return CUDA_R_16BF;
        case rocblas_datatype_f64_r: return CUDA_R_64F;
        default: return CUDA_R_32F;
    }
}

/* D = alpha * op(A) op(B) + beta * C, column-major; the harnesses always pass C == D (ldc == ldd). */
static inline rocblas_status rocblas_gemm_ex(rocblas_handle, rocblas_operation transA, rocblas_operation transB,
                                             rocblas_int m, rocblas_int n, rocblas_int k, const void* alpha,
                                             const void* a, rocblas_datatype a_type, rocblas_int lda, const void* b,
                                             rocblas_datatype b_type, rocblas_int ldb, const void* beta, const void* c,
                                             rocblas_datatype c_type, rocblas_int ldc, void* d,
                                             rocblas_datatype d_type, rocblas_int ldd, rocblas_datatype compute_type,
                                             rocblas_gemm_algo, int32_t, uint32_t) {
    cublasHandle_t cb = harness_cublas();
    if (!cb || c != d || ldc != ldd || c_type != d_type) return rocblas_status_not_implemented;
    const cublasComputeType_t ct =
        compute_type == rocblas_datatype_f64_r ? CUBLAS_COMPUTE_64F : CUBLAS_COMPUTE_32F;
    const cublasStatus_t s = cublasGemmEx(
        cb, transA == rocblas_operation_transpose ? CUBLAS_OP_T : CUBLAS_OP_N,
        transB == rocblas_operation_transpose ? CUBLAS_OP_T : CUBLAS_OP_N, m, n, k, alpha, a, harness_type(a_type), lda,
        b, harness_type(b_type), ldb, beta, d, harness_type(d_type), ldd, ct, CUBLAS_GEMM_DEFAULT);
    return s == CUBLAS_STATUS_SUCCESS ? rocblas_status_success : rocblas_status_internal_error;
}
