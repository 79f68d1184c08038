// k_split.cu - memory-bound kernels around the tensor-core GEMM: the hi/lo slice split (element-wise
// debug form and the K-major pre-split that feeds TMA), the absmax scan, and the per-row / per-column
// power-of-two exponents of the scaled fp16 split.
//
// Split rule (emugemm-cdna src/emugemm.cpp:143-148), kept bit for bit:
//   bf16:  hi = RNE_bf16(x),  lo = RNE_bf16(x - float(hi))          (the subtraction is exact in FP32)
//   fp16:  hi = RNE_f16(x),   lo = RNE_f16((x - float(hi)) * 2048)
// The scaled fp16 split applies the same rule to x * 2^-e, with e chosen per row of A / column of B.
#include "emugemm_internal.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace emu {
namespace {

__device__ __forceinline__ void split_bf16(float x, uint16_t& hi, uint16_t& lo) {
    __nv_bfloat16 h = __float2bfloat16_rn(x);
    __nv_bfloat16 l = __float2bfloat16_rn(x - __bfloat162float(h));
    hi = __bfloat16_as_ushort(h);
    lo = __bfloat16_as_ushort(l);
}

__device__ __forceinline__ void split_f16(float x, uint16_t& hi, uint16_t& lo) {
    __half h = __float2half_rn(x);
    __half l = __float2half_rn((x - __half2float(h)) * 2048.0f);
    hi = __half_as_ushort(h);
    lo = __half_as_ushort(l);
}

// x * 2^-e rounded once (exact unless the result leaves the normal range). When 2^-e is itself a normal float this is
// one multiply by it, which gives the same correctly rounded result as ldexpf(x, -e) without its range handling (the
// split ran at 0.29 ms at 8192^2 with ldexpf on every element); other e take ldexpf.
__device__ __forceinline__ float scale_pow2(float x, int e) {
    if (e >= -127 && e <= 126) return x * __int_as_float((127 - e) << 23);
    return ldexpf(x, -e);
}

__global__ void k_split_bf16_elem(const float* __restrict__ X, size_t n, uint16_t* __restrict__ hi,
                                  uint16_t* __restrict__ lo) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    size_t stride = (size_t)gridDim.x * blockDim.x;
    for (; i < n; i += stride) {
        uint16_t h, l;
        split_bf16(X[i], h, l);
        hi[i] = h;
        lo[i] = l;
    }
}

__global__ void k_split_f16_elem(const float* __restrict__ X, size_t n, uint16_t* __restrict__ hi,
                                 uint16_t* __restrict__ lo) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    size_t stride = (size_t)gridDim.x * blockDim.x;
    for (; i < n; i += stride) {
        uint16_t h, l;
        split_f16(X[i], h, l);
        hi[i] = h;
        lo[i] = l;
    }
}

// max |x| over a rows x cols matrix with leading dimension ld. Non-negative floats order like their bit
// patterns as signed ints, so the cross-block combine is an integer atomicMax (order independent).
__global__ void k_absmax(const float* __restrict__ X, long rows, long cols, long ld, float* out) {
    float m = 0.f;
    const size_t n = (size_t)rows * cols;
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    size_t stride = (size_t)gridDim.x * blockDim.x;
    if (ld == cols) {
        for (; i < n; i += stride) m = fmaxf(m, fabsf(X[i]));
    } else {
        for (; i < n; i += stride) {
            size_t r = i / cols, c = i - r * cols;
            m = fmaxf(m, fabsf(X[r * ld + c]));
        }
    }
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    __shared__ float warp_max[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) warp_max[warp] = m;
    __syncthreads();
    if (warp == 0) {
        m = (lane < (int)(blockDim.x >> 5)) ? warp_max[lane] : 0.f;
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) atomicMax(reinterpret_cast<int*>(out), __float_as_int(m));
    }
}

// e with max * 2^-e < 2^15: frexp gives max = f * 2^q, f in [0.5,1), so e = q - 15.
__device__ __forceinline__ int exponent_for_max(float mx) {
    if (!(mx > 0.f) || isinf(mx)) return 0;
    int q;
    frexpf(mx, &q);
    return q - 15;
}

// Row maxima of A over a segment of K per blockIdx.y: one warp per (row, segment), 16-byte loads when the row and
// the segment start are aligned, combined across segments with integer atomicMax on the (non-negative) float bits.
// Segments keep the whole GPU busy when A has few rows and long ones (M = 256, K = 262144).
__global__ void k_row_max(const float* __restrict__ A, int M, long K, long lda, long k_per_seg,
                          unsigned* __restrict__ rowmax_bits) {
    const int warps = blockDim.x >> 5;
    const int row = blockIdx.x * warps + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= M) return;
    const long k0 = (long)blockIdx.y * k_per_seg;
    const long k1 = min(K, k0 + k_per_seg);
    const float* a = A + (size_t)row * lda;
    float m = 0.f;
    long k = k0;
    if ((((uintptr_t)(a + k0)) & 15) == 0) {
        const float4* a4 = reinterpret_cast<const float4*>(a + k0);
        const long n4 = (k1 - k0) >> 2;
        for (long i = lane; i < n4; i += 32) {
            const float4 v = __ldg(a4 + i);
            m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
        k = k0 + 4 * n4;
    }
    for (long kk = k + lane; kk < k1; kk += 32) m = fmaxf(m, fabsf(a[kk]));
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) atomicMax(rowmax_bits + row, __float_as_uint(m));
}

// In place: the max bits of each row become the row's exponent.
__global__ void k_row_exponents(int* __restrict__ e, int M) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r < M) e[r] = exponent_for_max(__uint_as_float((unsigned)e[r]));
}

// Column maxima of B (K x N) over a slice of K per blockIdx.y, combined with integer atomicMax.
__global__ void k_col_max(const float* __restrict__ B, long K, int N, long ldb, long k_per_slice,
                          unsigned* __restrict__ colmax_bits) {
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= N) return;
    const long k0 = (long)blockIdx.y * k_per_slice;
    const long k1 = min(K, k0 + k_per_slice);
    float m = 0.f;
    for (long k = k0; k < k1; ++k) m = fmaxf(m, fabsf(B[(size_t)k * ldb + n]));
    atomicMax(colmax_bits + n, __float_as_uint(m));
}

__global__ void k_col_exponents(const unsigned* __restrict__ colmax_bits, int N, int* __restrict__ e_out) {
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    if (n < N) e_out[n] = exponent_for_max(__uint_as_float(colmax_bits[n]));
}

// A (M x K, lda) -> hi/lo slices, K-major in K panels ([Kp / KP][Mp][KP]), zero padded. One thread per
// (row, 8 consecutive k); item g writes values 8g .. 8g+7 of the slice, so the stores are contiguous.
template <int KIND>
__global__ void k_split_rows(const float* __restrict__ A, int M, long K, long lda, int Mp, long Kp, long KP,
                             const int* __restrict__ row_exp, uint16_t* __restrict__ hi,
                             uint16_t* __restrict__ lo) {
    const long groups_per_row = KP / 8;
    const size_t per_panel = (size_t)Mp * groups_per_row;
    const size_t total = per_panel * (size_t)(Kp / KP);
    const bool vec = ((lda & 3) == 0) && ((reinterpret_cast<uintptr_t>(A) & 15) == 0);
    for (size_t g = (size_t)blockIdx.x * blockDim.x + threadIdx.x; g < total;
         g += (size_t)gridDim.x * blockDim.x) {
        const size_t panel = g / per_panel;
        const size_t rem = g - panel * per_panel;
        const int m = (int)(rem / groups_per_row);
        const long k0 = (long)panel * KP + (long)(rem - (size_t)m * groups_per_row) * 8;
        float x[8];
        if (m < M && vec && k0 + 8 <= K) {
            const float4* p = reinterpret_cast<const float4*>(A + (size_t)m * lda + k0);
            float4 u = __ldg(p), v = __ldg(p + 1);
            x[0] = u.x; x[1] = u.y; x[2] = u.z; x[3] = u.w;
            x[4] = v.x; x[5] = v.y; x[6] = v.z; x[7] = v.w;
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j)
                x[j] = (m < M && k0 + j < K) ? __ldg(A + (size_t)m * lda + k0 + j) : 0.f;
        }
        int e = 0;
        if (KIND == 1 && m < M) e = row_exp[m];
        uint32_t h4[4], l4[4];
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
            uint16_t h0, l0, h1, l1;
            if (KIND == 0) {
                split_bf16(x[j], h0, l0);
                split_bf16(x[j + 1], h1, l1);
            } else {
                split_f16(scale_pow2(x[j], e), h0, l0);
                split_f16(scale_pow2(x[j + 1], e), h1, l1);
            }
            h4[j / 2] = (uint32_t)h0 | ((uint32_t)h1 << 16);
            l4[j / 2] = (uint32_t)l0 | ((uint32_t)l1 << 16);
        }
        const size_t o = g * 8;
        *reinterpret_cast<uint4*>(hi + o) = make_uint4(h4[0], h4[1], h4[2], h4[3]);
        *reinterpret_cast<uint4*>(lo + o) = make_uint4(l4[0], l4[1], l4[2], l4[3]);
    }
}

// B (K x N, ldb) -> transposed hi/lo slices, K-major in K panels ([Kp / KP][Np][KP]), zero padded. 64 x 64
// tiles through shared memory: coalesced reads along n, coalesced 16-byte writes along k. blockIdx.y strides
// over the k-tiles, so any K fits the grid's y limit.
template <int KIND>
__global__ void __launch_bounds__(256) k_split_cols(const float* __restrict__ B, long K, int N, long ldb,
                                                    int Np, long Kp, long KP, const int* __restrict__ col_exp,
                                                    uint16_t* __restrict__ hi, uint16_t* __restrict__ lo) {
    __shared__ float t[64][65];
    const int n0 = blockIdx.x * 64;
    const int tx = threadIdx.x & 63, ty = threadIdx.x >> 6;   // 64 x 4
    for (long kt = blockIdx.y; kt < Kp / 64; kt += gridDim.y) {
        const long k0 = kt * 64;
        const long panel = k0 / KP;
        uint16_t* const hi_p = hi + (size_t)panel * Np * KP + (k0 - panel * KP);
        uint16_t* const lo_p = lo + (size_t)panel * Np * KP + (k0 - panel * KP);
        // all 16 loads of a thread are issued before any is stored, so 16 are in flight at once
        float v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const long k = k0 + ty + 4 * i;
            const int n = n0 + tx;
            v[i] = (k < K && n < N) ? __ldg(B + (size_t)k * ldb + n) : 0.f;
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) t[ty + 4 * i][tx] = v[i];
        __syncthreads();
        // 64 columns x 8 groups of 8 k = 512 items, 2 per thread. Eight consecutive lanes take the eight k-groups
        // of one output row, so each warp store fills four whole 128-byte lines.
        for (int item = threadIdx.x; item < 512; item += 256) {
            const int kg = item & 7, nn = item >> 3;
            const int n = n0 + nn;
            if (n >= Np) continue;
            int e = 0;
            if (KIND == 1 && n < N) e = col_exp[n];
            uint32_t h4[4], l4[4];
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
                const float x0 = t[kg * 8 + j][nn], x1 = t[kg * 8 + j + 1][nn];
                uint16_t h0, l0, h1, l1;
                if (KIND == 0) {
                    split_bf16(x0, h0, l0);
                    split_bf16(x1, h1, l1);
                } else {
                    split_f16(scale_pow2(x0, e), h0, l0);
                    split_f16(scale_pow2(x1, e), h1, l1);
                }
                h4[j / 2] = (uint32_t)h0 | ((uint32_t)h1 << 16);
                l4[j / 2] = (uint32_t)l0 | ((uint32_t)l1 << 16);
            }
            const size_t o = (size_t)n * KP + kg * 8;
            *reinterpret_cast<uint4*>(hi_p + o) = make_uint4(h4[0], h4[1], h4[2], h4[3]);
            *reinterpret_cast<uint4*>(lo_p + o) = make_uint4(l4[0], l4[1], l4[2], l4[3]);
        }
        __syncthreads();   // the tile is rewritten by the next k-tile
    }
}

int grid_for(size_t n, int threads, int cap = 148 * 16) {
    size_t g = (n + threads - 1) / threads;
    if (g > (size_t)cap) g = cap;
    if (g < 1) g = 1;
    return (int)g;
}

}  // namespace

int launch_split_bf16(const float* X, size_t n, uint16_t* hi, uint16_t* lo, void* stream) {
    if (n == 0) return 0;
    k_split_bf16_elem<<<grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(X, n, hi, lo);
    count_launch();
    return (int)cudaGetLastError();
}

int launch_split_f16(const float* X, size_t n, uint16_t* hi, uint16_t* lo, void* stream) {
    if (n == 0) return 0;
    k_split_f16_elem<<<grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(X, n, hi, lo);
    count_launch();
    return (int)cudaGetLastError();
}

int launch_absmax(const float* X, long rows, long cols, long ld, float* out, void* stream) {
    cudaStream_t s = (cudaStream_t)stream;
    cudaError_t e = cudaMemsetAsync(out, 0, sizeof(float), s);
    if (e != cudaSuccess) return (int)e;
    size_t n = (size_t)rows * cols;
    if (n == 0) return 0;
    k_absmax<<<grid_for(n, 512, 148 * 8), 512, 0, s>>>(X, rows, cols, ld, out);
    count_launch();
    return (int)cudaGetLastError();
}

int launch_row_exponents(const float* A, int M, long K, long lda, int* e_out, void* stream) {
    if (M == 0) return 0;
    cudaStream_t s = (cudaStream_t)stream;
    cudaError_t e = cudaMemsetAsync(e_out, 0, sizeof(int) * (size_t)M, s);
    if (e != cudaSuccess) return (int)e;
    const int warps = 8;
    const long bx = (M + warps - 1) / warps;
    // about 8 blocks per SM, segments of at least 4096 values of K, starting on multiples of 4
    long segs = (148 * 8 + bx - 1) / bx;
    const long max_segs = (K + 4095) / 4096;
    if (segs > max_segs) segs = max_segs;
    if (segs < 1) segs = 1;
    long kps = (K + segs - 1) / segs;
    kps = (kps + 3) / 4 * 4;
    segs = (K + kps - 1) / kps;
    if (segs < 1) segs = 1;
    k_row_max<<<dim3((unsigned)bx, (unsigned)segs), warps * 32, 0, s>>>(A, M, K, lda, kps,
                                                                         reinterpret_cast<unsigned*>(e_out));
    k_row_exponents<<<(M + 255) / 256, 256, 0, s>>>(e_out, M);
    count_launch(2);
    return (int)cudaGetLastError();
}

int launch_col_exponents(const float* B, long K, int N, long ldb, int* e_out, unsigned* scratch, void* stream) {
    if (N == 0) return 0;
    cudaStream_t s = (cudaStream_t)stream;
    cudaError_t e = cudaMemsetAsync(scratch, 0, sizeof(unsigned) * (size_t)N, s);
    if (e != cudaSuccess) return (int)e;
    const int bx = (N + 255) / 256;
    long slices = (148 * 8 + bx - 1) / bx;
    if (slices < 1) slices = 1;
    if (slices > K) slices = K > 0 ? K : 1;
    long kps = (K + slices - 1) / slices;
    if (kps < 1) kps = 1;
    slices = (K + kps - 1) / kps;
    if (slices < 1) slices = 1;
    k_col_max<<<dim3(bx, (unsigned)slices), 256, 0, s>>>(B, K, N, ldb, kps, scratch);
    k_col_exponents<<<bx, 256, 0, s>>>(scratch, N, e_out);
    count_launch(2);
    return (int)cudaGetLastError();
}

int launch_split_rows(const float* A, int M, long K, long lda, int Mp, long Kp, long KP, int kind,
                      const int* row_exp, uint16_t* hi, uint16_t* lo, void* stream) {
    size_t total = (size_t)Mp * (Kp / 8);
    if (total == 0) return 0;
    if (KP <= 0 || KP % 64 || Kp % KP) return (int)cudaErrorInvalidValue;
    int g = grid_for(total, 256, 148 * 32);
    if (kind == 0)
        k_split_rows<0><<<g, 256, 0, (cudaStream_t)stream>>>(A, M, K, lda, Mp, Kp, KP, row_exp, hi, lo);
    else
        k_split_rows<1><<<g, 256, 0, (cudaStream_t)stream>>>(A, M, K, lda, Mp, Kp, KP, row_exp, hi, lo);
    count_launch();
    return (int)cudaGetLastError();
}

int launch_split_cols(const float* B, long K, int N, long ldb, int Np, long Kp, long KP, int kind,
                      const int* col_exp, uint16_t* hi, uint16_t* lo, void* stream) {
    if (Np == 0 || Kp == 0) return 0;
    if (KP <= 0 || KP % 64 || Kp % KP) return (int)cudaErrorInvalidValue;
    const long ktiles = Kp / 64;
    dim3 grid((unsigned)((Np + 63) / 64), (unsigned)(ktiles < 65535 ? ktiles : 65535));
    if (kind == 0)
        k_split_cols<0><<<grid, 256, 0, (cudaStream_t)stream>>>(B, K, N, ldb, Np, Kp, KP, col_exp, hi, lo);
    else
        k_split_cols<1><<<grid, 256, 0, (cudaStream_t)stream>>>(B, K, N, ldb, Np, Kp, KP, col_exp, hi, lo);
    count_launch();
    return (int)cudaGetLastError();
}

}  // namespace emu
