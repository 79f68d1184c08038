/* Build shim (oracle only): maps the few HIP runtime names that emugemm-cdna's src/emugemm.cpp uses onto
 * the CUDA runtime, so that its host planner and model functions compile unmodified. The GPU paths of that
 * file are never called through this shim. The device arch string reported to the reference's
 * emugemm_init comes from the EMUREF_ARCH environment variable (default "gfx90a"). */
#pragma once
#include <cuda_runtime.h>
#include <stdlib.h>
#include <string.h>

typedef cudaError_t hipError_t;
#define hipSuccess cudaSuccess
#define hipMalloc cudaMalloc
#define hipFree cudaFree
#define hipMemcpy cudaMemcpy
#define hipMemset cudaMemset
#define hipMemcpyHostToDevice cudaMemcpyHostToDevice
#define hipMemcpyDeviceToHost cudaMemcpyDeviceToHost

typedef struct { char gcnArchName[256]; } hipDeviceProp_t;

static inline hipError_t hipGetDeviceProperties(hipDeviceProp_t* p, int dev) {
    (void)dev;
    const char* a = getenv("EMUREF_ARCH");
    strncpy(p->gcnArchName, a ? a : "gfx90a", sizeof(p->gcnArchName) - 1);
    p->gcnArchName[sizeof(p->gcnArchName) - 1] = 0;
    return cudaSuccess;
}
