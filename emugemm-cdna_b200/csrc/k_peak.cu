// k_peak.cu - peak rates of the B200's arithmetic pipes and of HBM, measured with one instrument: the B200
// counterpart of emugemm-cdna bench/mfma_peak2.cpp:1-142. That probe times one matrix-core instruction per
// precision in a register loop, all kernels interleaved round-robin with the median of the repetitions, so that
// clock drift hits every kernel alike, and prints the ratios the emulation's economics rest on (bf16:fp32 = R,
// so a 3-product scheme is capped at R/3 of native FP32).
//
// Here the instruments are:
//   tcgen05 MMA  kind::f16 (bf16 and fp16 inputs) and kind::tf32, 128x256 tiles, FP32 accumulators in TMEM,
//                one CTA per SM issuing back-to-back MMAs on operand tiles resident in shared memory;
//   FFMA / DFMA  independent FMA chains in registers (FP32 SIMT is the native-FP32 denominator on B200: there
//                is no FP32-input tensor-core instruction, only TF32);
//   HBM          a device-to-device copy, read + written bytes.
// No global memory is touched by the MMA and FMA loops, so they measure the pipes alone.
#include "emugemm_internal.h"
#include "device_utils.cuh"

#include <algorithm>
#include <cuda_runtime.h>
#include <vector>

namespace emu {
namespace {

using namespace dev;

constexpr int kMmaThreads = 128;
constexpr int kTileA = 128 * 128, kTileB = 256 * 128;   // bytes: 128 / 256 rows of one 128-byte swizzle row
// Dynamic shared memory per CTA: the two tiles plus alignment slack, padded to more than half of the SM's
// 228 KB so that no SM holds two CTAs (each allocates all 512 TMEM columns; a second CTA would wait in
// tcgen05.alloc for the first to finish and serialise).
constexpr int kMmaSmem = 120 * 1024;
static_assert(kTileA + kTileB + 1024 <= kMmaSmem, "tiles fit");
constexpr int kMmaPerCta = 16384;

__device__ __forceinline__ unsigned mix(unsigned h) {
    h ^= h >> 16;
    h *= 0x7feb352du;
    h ^= h >> 15;
    h *= 0x846ca68bu;
    h ^= h >> 16;
    return h;
}

// 16-bit operand value of magnitude in [2^-4, 2^-3) with a hashed sign and mantissa (finite, no subnormals), or
// an FP32 bit pattern of the same range for tf32.
__device__ __forceinline__ uint32_t operand_bits(unsigned h, int kind) {
    if (kind == 2) return (h & 0x80000000u) | 0x3d800000u | (h & 0x007fffffu);
    auto half = [&](unsigned x) -> uint32_t {
        return kind == 0 ? ((x & 0x8000u) | 0x3d80u | (x & 0x7fu))       // bf16
                         : ((x & 0x8000u) | 0x2c00u | (x & 0x3ffu));     // fp16
    };
    return half(h & 0xffffu) | (half(h >> 16) << 16);
}

__device__ __forceinline__ void mma_tf32_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    uint32_t m0 = 0, m1 = 0, m2 = 0, m3 = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(m0), "r"(m1), "r"(m2), "r"(m3));
}

// KIND: 0 bf16, 1 fp16 (kind::f16, K = 16 per MMA), 2 tf32 (kind::tf32, K = 8 per MMA). Each MMA reads one
// 32-byte K step of the 128-byte rows (A: 128 rows, B: 256 rows) and accumulates into one of two 128x256 FP32
// accumulators (TMEM columns 0-255 and 256-511).
template <int KIND>
__global__ void __launch_bounds__(kMmaThreads, 1) k_peak_mma(int n_mma, unsigned seed, unsigned* err) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t done;
    __shared__ uint32_t tmem_base;
    __shared__ int abort_flag;
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint32_t* words = reinterpret_cast<uint32_t*>(base);
    for (int i = threadIdx.x; i < (kTileA + kTileB) / 4; i += kMmaThreads)
        words[i] = operand_bits(mix((unsigned)i ^ seed), KIND);
    fence_proxy_async_smem();   // the tensor core reads shared memory through the async proxy
    const int warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        mbar_init(&done, 1);
        fence_mbar_init();
        abort_flag = 0;
    }
    if (warp == 0) {
        tmem_alloc(&tmem_base, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = tmem_base;
    if (threadIdx.x == 0) {
        constexpr uint32_t idesc = KIND == 2 ? ((1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(256 >> 3) << 17) |
                                                ((uint32_t)(128 >> 4) << 24))
                                             : idesc_f16(128, 256, KIND == 0);
        const uint64_t a0 = sdesc_kmajor(smem_u32(base), 128);
        const uint64_t b0 = sdesc_kmajor(smem_u32(base + kTileA), 128);
        for (int i = 0; i < n_mma; ++i) {
            const uint64_t adv = (uint64_t)((i & 3) * 32) >> 4;   // 32 bytes along K per MMA, 4 per row
            const uint32_t d = tm + (uint32_t)(i & 1) * 256u;
            if (KIND == 2)
                mma_tf32_ss(d, a0 + adv, b0 + adv, idesc, i >= 2 ? 1u : 0u);
            else
                mma_f16_ss(d, a0 + adv, b0 + adv, idesc, i >= 2 ? 1u : 0u);
        }
        mma_commit(&done);
    }
    __syncwarp();
    if (!mbar_wait(&done, 0, &abort_flag, err, kErrTimeoutMma)) {
        // unwinding: give the MMAs in flight a further bounded wait before the columns are released
        const uint32_t a = smem_u32(&done);
        const unsigned long long t0 = globaltimer();
        while (!mbar_try_wait(a, 0) && globaltimer() - t0 < kWaitLimitNs) {
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tm, 512);
}

constexpr int kFmaChains = 16;

// FP32 / FP64 FMA chains: acc = acc * a + b, 16 independent chains per thread; the sums are stored so that no
// chain is dead code. a and b come from memory (not foldable).
template <typename T>
__global__ void __launch_bounds__(256) k_peak_fma(const T* __restrict__ ab, int loops, T* __restrict__ out) {
    const T a = ab[0], b = ab[1];
    T acc[kFmaChains];
#pragma unroll
    for (int i = 0; i < kFmaChains; ++i) acc[i] = (T)(threadIdx.x & 7) * (T)0.125 + (T)i;
#pragma unroll 4
    for (int l = 0; l < loops; ++l) {
#pragma unroll
        for (int i = 0; i < kFmaChains; ++i) acc[i] = fma(acc[i], a, b);
    }
    T s = 0;
#pragma unroll
    for (int i = 0; i < kFmaChains; ++i) s += acc[i];
    out[(size_t)blockIdx.x * blockDim.x + threadIdx.x] = s;
}

// Streaming copy, four 16-byte loads in flight per thread before their stores.
__global__ void k_peak_copy(const float4* __restrict__ src, float4* __restrict__ dst, size_t n4) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (; i + 3 * stride < n4; i += 4 * stride) {
        const float4 v0 = __ldcs(src + i), v1 = __ldcs(src + i + stride), v2 = __ldcs(src + i + 2 * stride),
                     v3 = __ldcs(src + i + 3 * stride);
        __stcs(dst + i, v0);
        __stcs(dst + i + stride, v1);
        __stcs(dst + i + 2 * stride, v2);
        __stcs(dst + i + 3 * stride, v3);
    }
    for (; i < n4; i += stride) __stcs(dst + i, __ldcs(src + i));
}

__global__ void k_fill_src(float4* p, size_t n4) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const float v = (float)(i & 1023u);
        p[i] = make_float4(v, v + 1.f, v + 2.f, v + 3.f);
    }
}

__global__ void k_fill_ab(float* f, double* d) {
    f[0] = 0.9999999f;
    f[1] = 1.0e-7f;
    d[0] = 0.9999999999;
    d[1] = 1.0e-10;
}

}  // namespace

// Runs every instrument `reps` times, interleaved round-robin after one warm-up launch each, and stores the
// median rates: rates[0..2] tensor-core TFLOP/s (bf16, fp16, tf32), [3] FFMA TFLOP/s, [4] DFMA TFLOP/s,
// [5] copy GB/s (bytes read + written). Returns a cudaError_t, or -1 when a tensor-core wait timed out.
int run_peak_probe(int reps, int num_sms, unsigned* err_dev, const unsigned* err_host, void* stream,
                   double* rates) {
    cudaStream_t st = (cudaStream_t)stream;
    constexpr int kKinds = 6;
    const size_t copy_bytes = (size_t)1 << 30;   // 1 GiB read, 1 GiB written
    const int fma_blocks = num_sms * 8, fma_threads = 256;
    const int ffma_loops = 4096, dfma_loops = 1024;
    void *src = nullptr, *dst = nullptr, *sink = nullptr, *abf = nullptr, *abd = nullptr;
    cudaEvent_t ev[2] = {nullptr, nullptr};
    std::vector<std::vector<float>> ms(kKinds);
    int rc = 0;
    auto fail = [&](cudaError_t e) {
        if (e != cudaSuccess && rc == 0) rc = (int)e;
        return rc != 0;
    };
    if (fail(cudaMalloc(&src, copy_bytes)) || fail(cudaMalloc(&dst, copy_bytes)) ||
        fail(cudaMalloc(&sink, (size_t)fma_blocks * fma_threads * sizeof(double))) ||
        fail(cudaMalloc(&abf, 2 * sizeof(float))) || fail(cudaMalloc(&abd, 2 * sizeof(double))) ||
        fail(cudaEventCreate(&ev[0])) || fail(cudaEventCreate(&ev[1])) ||
        fail(cudaFuncSetAttribute(k_peak_mma<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMmaSmem)) ||
        fail(cudaFuncSetAttribute(k_peak_mma<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMmaSmem)) ||
        fail(cudaFuncSetAttribute(k_peak_mma<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMmaSmem))) {
    } else {
        k_fill_src<<<num_sms * 8, 256, 0, st>>>((float4*)src, copy_bytes / 16);
        k_fill_ab<<<1, 1, 0, st>>>((float*)abf, (double*)abd);
        auto launch = [&](int k) {
            switch (k) {
                case 0: k_peak_mma<0><<<num_sms, kMmaThreads, kMmaSmem, st>>>(kMmaPerCta, 0x1234u, err_dev); break;
                case 1: k_peak_mma<1><<<num_sms, kMmaThreads, kMmaSmem, st>>>(kMmaPerCta, 0x1234u, err_dev); break;
                case 2: k_peak_mma<2><<<num_sms, kMmaThreads, kMmaSmem, st>>>(kMmaPerCta, 0x1234u, err_dev); break;
                case 3:
                    k_peak_fma<float><<<fma_blocks, fma_threads, 0, st>>>((const float*)abf, ffma_loops, (float*)sink);
                    break;
                case 4:
                    k_peak_fma<double><<<fma_blocks, fma_threads, 0, st>>>((const double*)abd, dfma_loops,
                                                                           (double*)sink);
                    break;
                case 5:
                    k_peak_copy<<<num_sms * 8, 256, 0, st>>>((const float4*)src, (float4*)dst, copy_bytes / 16);
                    break;
            }
        };
        for (int k = 0; k < kKinds; ++k) launch(k);
        count_launch(kKinds + 2);
        if (!fail(cudaStreamSynchronize(st))) {
            for (int r = 0; r < reps && rc == 0; ++r)
                for (int k = 0; k < kKinds && rc == 0; ++k) {
                    cudaEventRecord(ev[0], st);
                    launch(k);
                    cudaEventRecord(ev[1], st);
                    count_launch(1);
                    if (fail(cudaEventSynchronize(ev[1]))) break;
                    float t = 0.f;
                    cudaEventElapsedTime(&t, ev[0], ev[1]);
                    ms[k].push_back(t);
                }
        }
        if (rc == 0) rc = (int)cudaGetLastError();
    }
    if (rc == 0 && *reinterpret_cast<const volatile unsigned*>(err_host) != 0) rc = -1;
    if (rc == 0) {
        const double mma_flop = 2.0 * 128 * 256 * (double)kMmaPerCta * num_sms;
        const double work[kKinds] = {
            mma_flop * 16, mma_flop * 16, mma_flop * 8,
            2.0 * kFmaChains * (double)ffma_loops * fma_blocks * fma_threads,
            2.0 * kFmaChains * (double)dfma_loops * fma_blocks * fma_threads,
            2.0 * (double)copy_bytes};
        for (int k = 0; k < kKinds; ++k) {
            std::vector<float> v = ms[k];
            std::sort(v.begin(), v.end());
            const double med = v.empty() ? 0.0 : v[v.size() / 2];
            rates[k] = med > 0 ? work[k] / (med * 1e-3) / (k == 5 ? 1e9 : 1e12) : 0.0;
        }
    }
    for (void* p : {src, dst, sink, abf, abd})
        if (p) cudaFree(p);
    for (cudaEvent_t e : ev)
        if (e) cudaEventDestroy(e);
    return rc;
}

}  // namespace emu
