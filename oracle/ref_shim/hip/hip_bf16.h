/* Build shim (oracle only): the bf16 type name of HIP mapped to CUDA's (both convert from float with
 * round-to-nearest-even). */
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
typedef __nv_bfloat16 __hip_bfloat16;
