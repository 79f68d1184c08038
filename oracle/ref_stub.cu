// Link stub and test-only launchers (oracle only) for the reference build of emugemm-cdna's src/emugemm.cpp.
//
// rocblas_gemm_ex is never reached by emugemm_plan / emugemm_model_*; if anything calls it, it reports
// not_implemented.
//
// emuref_split_bf16 / emuref_split_f16 launch the reference's OWN split kernels k_split_bf and k_split_f16
// (src/emugemm.cpp:143-148), which that file defines with external linkage and this library compiles from the
// reference source unchanged, with the same 256-thread grid as the reference's executor (src/emugemm.cpp:332-333,
// 346-347). A GPU test compares their output bit for bit with the library's emugemm_split_bf16 / _f16. The HIP types
// map to CUDA's (ref_shim/hip/hip_bf16.h, -D_Float16=__half): both convert float with round-to-nearest-even.
#include "rocblas/rocblas.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <stddef.h>

extern "C" rocblas_status rocblas_gemm_ex(rocblas_handle, rocblas_operation, rocblas_operation, rocblas_int,
                                          rocblas_int, rocblas_int, const void*, const void*, rocblas_datatype,
                                          rocblas_int, const void*, rocblas_datatype, rocblas_int, const void*,
                                          const void*, rocblas_datatype, rocblas_int, void*, rocblas_datatype,
                                          rocblas_int, rocblas_datatype, rocblas_gemm_algo, int32_t, uint32_t) {
    return rocblas_status_not_implemented;
}

// defined in src/emugemm.cpp (same library)
__global__ void k_split_bf(const float* X, __nv_bfloat16* S0, __nv_bfloat16* S1, size_t n);
__global__ void k_split_f16(const float* X, __half* H, __half* L, size_t n);

// Device pointers; synchronous. Returns a cudaError_t (0 = success).
extern "C" int emuref_split_bf16(const float* X, size_t n, void* hi, void* lo) {
    if (n == 0) return 0;
    const int tpb = 256;
    k_split_bf<<<(unsigned)((n + tpb - 1) / tpb), tpb>>>(X, static_cast<__nv_bfloat16*>(hi),
                                                          static_cast<__nv_bfloat16*>(lo), n);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    return (int)e;
}

extern "C" int emuref_split_f16(const float* X, size_t n, void* hi, void* lo) {
    if (n == 0) return 0;
    const int tpb = 256;
    k_split_f16<<<(unsigned)((n + tpb - 1) / tpb), tpb>>>(X, static_cast<__half*>(hi), static_cast<__half*>(lo), n);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    return (int)e;
}
