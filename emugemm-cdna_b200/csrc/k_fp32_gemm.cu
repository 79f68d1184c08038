// k_fp32_gemm.cu - FP32 SIMT GEMM with K-chunks summed in FP64: the NATIVE_FP32 (c = 1) and FP32_CHUNKED
// schemes of emugemm (emugemm-cdna src/emugemm.cpp:313-330).
//
// The reference runs one rocBLAS SGEMM per chunk into an FP32 buffer and adds it into an FP64 buffer with
// a separate kernel (k_accum_f64, src/emugemm.cpp:149-154). Here one kernel does both: every output
// element is a single sequential FP32 FMA chain over the chunk's K range (k ascending), and the chunk
// partial is folded into an FP64 sum kept in a workspace tile owned by the same thread. Chunk c covers
// [c*kc, min(K, (c+1)*kc)) with kc = ceil(K/chunks), exactly the reference's chunk boundaries.
//
// When there are too few output tiles to fill the GPU, the chunks are divided into G contiguous groups
// (grid.z); group g writes its FP64 sum to partial plane g and a reduce kernel adds the planes in order
// g = 0..G-1 and rounds once to FP32. With this fixed order the result is deterministic and a CPU oracle
// that performs the same FMA chains and FP64 additions reproduces it bit for bit.
#include "emugemm_internal.h"

#include <cuda_runtime.h>

namespace emu {
namespace {

constexpr int kThr = 256;

struct Params {
    const float* A; long lda;
    const float* B; long ldb;
    float* C; long ldc;
    double* C64; long ldc64;
    double* W;          // G planes of M x N (ld N), used when G > 1
    int M, N; long K;
    long kc;            // chunk length
    int ce;             // non-empty chunks
    int cpg;            // chunks per group
    int G;
};

// kBKf: values of K per shared-memory stage (16; a 64-deep stage for the 32 tile measured slower: its
// unrolled k-loop ran at 64 registers with spills).
template <int BM, int BN, int TM, int TN, bool VEC, int kBKf>
__global__ void __launch_bounds__(kThr) k_fp32_gemm(Params p) {
    __shared__ __align__(16) float As[2][kBKf][BM];
    __shared__ __align__(16) float Bs[2][kBKf][BN];
    constexpr int HM = TM / 2, HN = TN / 2;
    constexpr int A_F4 = BM * kBKf / 4, B_F4 = BN * kBKf / 4;   // float4s per k-block tile
    constexpr int A_VEC = (A_F4 + kThr - 1) / kThr;             // float4 per thread (the last may be idle)
    constexpr int B_VEC = (B_F4 + kThr - 1) / kThr;
    constexpr int A_SC = (BM * kBKf + kThr - 1) / kThr;         // scalars per thread
    constexpr int B_SC = (BN * kBKf + kThr - 1) / kThr;
    static_assert(16 * TM == BM && 16 * TN == BN, "tile shape");

    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int g = blockIdx.z;
    const int c_first = g * p.cpg;
    const int c_last = min(p.ce, c_first + p.cpg);   // exclusive

    float acc[TM][TN];
    double* Wg = p.W ? p.W + (size_t)g * p.M * p.N : nullptr;

    float ra[VEC ? A_VEC * 4 : A_SC];
    float rb[VEC ? B_VEC * 4 : B_SC];

    auto load_global = [&](long kb, long kend) {
        if (VEC) {
#pragma unroll
            for (int j = 0; j < A_VEC; ++j) {
                const int f = tid + j * kThr;
                const int row = f / (kBKf / 4), kq = f % (kBKf / 4);
                const int m = m0 + row;
                const long k = kb + kq * 4;
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (f < A_F4 && m < p.M && k < kend)
                    v = __ldg(reinterpret_cast<const float4*>(p.A + (size_t)m * p.lda + k));
                ra[4 * j] = v.x; ra[4 * j + 1] = v.y; ra[4 * j + 2] = v.z; ra[4 * j + 3] = v.w;
            }
#pragma unroll
            for (int j = 0; j < B_VEC; ++j) {
                const int f = tid + j * kThr;
                const int kk = f / (BN / 4), nq = f % (BN / 4);
                const long k = kb + kk;
                const int n = n0 + nq * 4;
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (f < B_F4 && k < kend && n < p.N)
                    v = __ldg(reinterpret_cast<const float4*>(p.B + (size_t)k * p.ldb + n));
                rb[4 * j] = v.x; rb[4 * j + 1] = v.y; rb[4 * j + 2] = v.z; rb[4 * j + 3] = v.w;
            }
        } else {
#pragma unroll
            for (int j = 0; j < A_SC; ++j) {
                const int f = tid + j * kThr;
                const int row = f / kBKf, kk = f % kBKf;
                const int m = m0 + row;
                const long k = kb + kk;
                ra[j] = (f < BM * kBKf && m < p.M && k < kend) ? __ldg(p.A + (size_t)m * p.lda + k) : 0.f;
            }
#pragma unroll
            for (int j = 0; j < B_SC; ++j) {
                const int f = tid + j * kThr;
                const int kk = f / BN, nn = f % BN;
                const long k = kb + kk;
                const int n = n0 + nn;
                rb[j] = (f < BN * kBKf && k < kend && n < p.N) ? __ldg(p.B + (size_t)k * p.ldb + n) : 0.f;
            }
        }
    };
    auto store_smem = [&](int buf) {
        if (VEC) {
#pragma unroll
            for (int j = 0; j < A_VEC; ++j) {
                const int f = tid + j * kThr;
                const int row = f / (kBKf / 4), kq = f % (kBKf / 4);
                if (f >= A_F4) continue;
#pragma unroll
                for (int e = 0; e < 4; ++e) As[buf][kq * 4 + e][row] = ra[4 * j + e];
            }
#pragma unroll
            for (int j = 0; j < B_VEC; ++j) {
                const int f = tid + j * kThr;
                const int kk = f / (BN / 4), nq = f % (BN / 4);
                if (f >= B_F4) continue;
                *reinterpret_cast<float4*>(&Bs[buf][kk][nq * 4]) =
                    make_float4(rb[4 * j], rb[4 * j + 1], rb[4 * j + 2], rb[4 * j + 3]);
            }
        } else {
#pragma unroll
            for (int j = 0; j < A_SC; ++j) {
                const int f = tid + j * kThr;
                if (f >= BM * kBKf) continue;
                As[buf][f % kBKf][f / kBKf] = ra[j];
            }
#pragma unroll
            for (int j = 0; j < B_SC; ++j) {
                const int f = tid + j * kThr;
                if (f >= BN * kBKf) continue;
                Bs[buf][f / BN][f % BN] = rb[j];
            }
        }
    };

    for (int ci = c_first; ci < c_last; ++ci) {
        const long kbeg = (long)ci * p.kc;
        const long kend = min(p.K, kbeg + p.kc);
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
            for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

        const long nkb = (kend - kbeg + kBKf - 1) / kBKf;
        load_global(kbeg, kend);
        store_smem(0);
        __syncthreads();
        for (long kt = 0; kt < nkb; ++kt) {
            const int cur = (int)(kt & 1);
            if (kt + 1 < nkb) load_global(kbeg + (kt + 1) * kBKf, kend);
#pragma unroll
            for (int k = 0; k < kBKf; ++k) {
                float a[TM], b[TN];
#pragma unroll
                for (int i = 0; i < HM; ++i) {
                    a[i] = As[cur][k][ty * HM + i];
                    a[HM + i] = As[cur][k][BM / 2 + ty * HM + i];
                }
#pragma unroll
                for (int j = 0; j < HN; ++j) {
                    b[j] = Bs[cur][k][tx * HN + j];
                    b[HN + j] = Bs[cur][k][BN / 2 + tx * HN + j];
                }
#pragma unroll
                for (int i = 0; i < TM; ++i)
#pragma unroll
                    for (int j = 0; j < TN; ++j) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
            }
            if (kt + 1 < nkb) store_smem(cur ^ 1);
            __syncthreads();
        }

        // Fold this chunk's FP32 partials into the FP64 sum of the group.
        const bool first = (ci == c_first), last = (ci == c_last - 1);
#pragma unroll
        for (int i = 0; i < TM; ++i) {
            const int m = m0 + (i < HM ? ty * HM + i : BM / 2 + ty * HM + (i - HM));
            if (m >= p.M) continue;
#pragma unroll
            for (int j = 0; j < TN; ++j) {
                const int n = n0 + (j < HN ? tx * HN + j : BN / 2 + tx * HN + (j - HN));
                if (n >= p.N) continue;
                const size_t wi = (size_t)m * p.N + n;
                double s = first ? (double)acc[i][j] : Wg[wi] + (double)acc[i][j];
                if (last && p.G == 1) {
                    if (p.C64) p.C64[(size_t)m * p.ldc64 + n] = s;
                    else p.C[(size_t)m * p.ldc + n] = (float)s;
                } else {
                    Wg[wi] = s;
                }
            }
        }
    }
}

// 32 x 32 and 64 x 64 tiles (2 x 2 / 4 x 4 chains per thread) with the operands streamed through a cp.async ring,
// for products with few output tiles (C3: M = N = 256) and mid-size ones. (At the 128 tile the register-staged
// k_fp32_gemm stays: the ring version measured 41.8 against 44.5 TFLOP/s at 8192^3.) A register-staged k-block of prefetch left
// the global-load latency exposed on every k-block when a thread has few FMAs per loaded value; the ring keeps
// STAGES - 1 k-blocks of 16 in flight. Shared tiles keep the global layouts (A [m][k], B [k][n]): per four k a
// thread reads its TM rows of A as float4 along k and, per k, its TM columns of B as one vector, then runs the
// same chains (k ascending per element) with the same FP64 folds as k_fp32_gemm. Needs the VEC conditions
// (16-byte aligned rows, K, N and the chunk length multiples of 4), so no 16-byte copy straddles a bound.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc, bool valid) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
    const int n = valid ? 16 : 0;   // 0 source bytes: the 16 destination bytes are zero-filled
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(gsrc), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int BM, int STAGES>
__global__ void __launch_bounds__(kThr) k_fp32_gemm_cp(Params p) {
    constexpr int TM = BM / 16;                          // chains per thread along m and along n
    constexpr int A_CH = BM * 4, CH = 8 * BM;            // 16-byte copies: A (BM rows x 4), A + B
    constexpr int CPT = CH / kThr;                       // copies per thread per k-block
    static_assert(CH % kThr == 0 && (TM == 2 || TM == 4 || TM == 8), "tile shape");
    __shared__ __align__(16) float As[STAGES][BM][16];   // [m][k]
    __shared__ __align__(16) float Bs[STAGES][16][BM];   // [k][n]
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BM;
    const int g = blockIdx.z;
    const int c_first = g * p.cpg;
    const int c_last = min(p.ce, c_first + p.cpg);
    double* Wg = p.W ? p.W + (size_t)g * p.M * p.N : nullptr;

    for (int ci = c_first; ci < c_last; ++ci) {
        const long kbeg = (long)ci * p.kc;
        const long kend = min(p.K, kbeg + p.kc);
        const long nkb = (kend - kbeg + 15) / 16;
        auto issue = [&](long kt) {
            const int st = (int)(kt % STAGES);
            const long k = kbeg + kt * 16;
#pragma unroll
            for (int c = 0; c < CPT; ++c) {
                const int f = tid + c * kThr;
                if (f < A_CH) {
                    const int r = f >> 2, q = f & 3;
                    const int m = m0 + r;
                    const long kk = k + q * 4;
                    const bool v = m < p.M && kk < kend;
                    cp_async16(&As[st][r][q * 4], v ? (const void*)(p.A + (size_t)m * p.lda + kk) : (const void*)p.A,
                               v);
                } else {
                    const int f2 = f - A_CH;
                    const int kr = f2 / (BM / 4), q = f2 % (BM / 4);
                    const long kk = k + kr;
                    const int n = n0 + q * 4;
                    const bool v = kk < kend && n < p.N;
                    cp_async16(&Bs[st][kr][q * 4], v ? (const void*)(p.B + (size_t)kk * p.ldb + n) : (const void*)p.B,
                               v);
                }
            }
        };
        float acc[TM][TM];
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
            for (int j = 0; j < TM; ++j) acc[i][j] = 0.f;
        for (int kt = 0; kt < STAGES - 1; ++kt) {
            if (kt < nkb) issue(kt);
            cp_async_commit();
        }
        for (long kt = 0; kt < nkb; ++kt) {
            if (kt + STAGES - 1 < nkb) issue(kt + STAGES - 1);
            cp_async_commit();
            cp_async_wait<STAGES - 1>();   // k-block kt has landed (this thread's copies)
            __syncthreads();               // ... and every thread's
            const int st = (int)(kt % STAGES);
#pragma unroll
            for (int k4 = 0; k4 < 4; ++k4) {
                float4 a[TM];
#pragma unroll
                for (int i = 0; i < TM; ++i) a[i] = *reinterpret_cast<const float4*>(&As[st][ty * TM + i][k4 * 4]);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    float b[TM];
                    if (TM == 2) {
                        const float2 v = *reinterpret_cast<const float2*>(&Bs[st][k4 * 4 + kk][tx * TM]);
                        b[0] = v.x; b[1] = v.y;
                    } else {
#pragma unroll
                        for (int h = 0; h < TM / 4; ++h) {
                            const float4 v = *reinterpret_cast<const float4*>(&Bs[st][k4 * 4 + kk][tx * TM + 4 * h]);
                            b[4 * h] = v.x; b[4 * h + 1] = v.y; b[4 * h + 2] = v.z; b[4 * h + 3] = v.w;
                        }
                    }
#pragma unroll
                    for (int i = 0; i < TM; ++i) {
                        const float av = kk == 0 ? a[i].x : kk == 1 ? a[i].y : kk == 2 ? a[i].z : a[i].w;
#pragma unroll
                        for (int j = 0; j < TM; ++j) acc[i][j] = __fmaf_rn(av, b[j], acc[i][j]);
                    }
                }
            }
            __syncthreads();               // stage st is refilled by a later iteration
        }
        cp_async_wait<0>();
        // fold this chunk's FP32 partials into the FP64 sum of the group (as in k_fp32_gemm)
        const bool first = (ci == c_first), last = (ci == c_last - 1);
#pragma unroll
        for (int i = 0; i < TM; ++i) {
            const int m = m0 + ty * TM + i;
            if (m >= p.M) continue;
#pragma unroll
            for (int j = 0; j < TM; ++j) {
                const int n = n0 + tx * TM + j;
                if (n >= p.N) continue;
                const size_t wi = (size_t)m * p.N + n;
                const double s = first ? (double)acc[i][j] : Wg[wi] + (double)acc[i][j];
                if (last && p.G == 1) {
                    if (p.C64) p.C64[(size_t)m * p.ldc64 + n] = s;
                    else p.C[(size_t)m * p.ldc + n] = (float)s;
                } else {
                    Wg[wi] = s;
                }
            }
        }
    }
}

// 16 x 32 tiles for products whose output has too few elements to give every SM a 32 x 32 tile (C3: M = N = 256,
// 65536 chains, c = 1). 128 threads, each running a 2 x 2 block of chains, so the CTA grid covers 128 SMs (the 32
// tile: 64) with one warp per SM sub-partition.
//
// What bounds every FP32 SIMT tile here is shared-memory delivery, not the FMA pipe: an SM serves one 128-byte
// wavefront per clock (one float per lane of a warp) while it can issue four FFMA warp-instructions, and a thread
// with a TM x TN block of chains needs TM + TN floats per k for TM * TN FMAs. The FMA pipe can therefore be at most
// TM * TN / (TM + TN) / 4 busy: 0.25 for 2 x 2, 0.5 for 4 x 4, 1 for 8 x 8 (ncu: the 1 x 4 form of this kernel
// ran with the L1/shared pipe 97 % busy and the FMA pipe at 24 %). Few output elements force small blocks.
//
// Per four k a thread reads each of its two rows of A as one float4 along k (rows padded by 4 floats) and, per k,
// its two columns of B as one float2: 16 wavefronts per 16 FMAs per warp. The stage is 64 deep. Same chains (k
// ascending per element), same FP64 folds and the same VEC conditions as k_fp32_gemm_cp.
template <int STAGES>
__global__ void __launch_bounds__(128) k_fp32_narrow(Params p) {
    constexpr int BK = 64, BKP = BK + 4, TR = 16, TC = 32;
    constexpr int A_CH = TR * BK / 4, CH = A_CH + BK * TC / 4, CPT = CH / 128;
    static_assert(CH % 128 == 0, "copies per thread");
    extern __shared__ __align__(16) float narrow_smem[];
    auto As = reinterpret_cast<float (*)[TR][BKP]>(narrow_smem);                       // [stage][m][k], rows padded
    auto Bs = reinterpret_cast<float (*)[BK][TC]>(narrow_smem + STAGES * TR * BKP);    // [stage][k][n]
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;               // rows 2*ty, 2*ty+1; columns 2*tx, 2*tx+1
    const int m0 = blockIdx.y * TR, n0 = blockIdx.x * TC;
    const int g = blockIdx.z;
    const int c_first = g * p.cpg;
    const int c_last = min(p.ce, c_first + p.cpg);
    double* Wg = p.W ? p.W + (size_t)g * p.M * p.N : nullptr;

    for (int ci = c_first; ci < c_last; ++ci) {
        const long kbeg = (long)ci * p.kc;
        const long kend = min(p.K, kbeg + p.kc);
        const long nkb = (kend - kbeg + BK - 1) / BK;
        auto issue = [&](long kt) {
            const int st = (int)(kt % STAGES);
            const long k = kbeg + kt * BK;
#pragma unroll
            for (int c = 0; c < CPT; ++c) {
                const int f = tid + c * 128;
                if (f < A_CH) {
                    const int r = f / (BK / 4), q = f % (BK / 4);
                    const int m = m0 + r;
                    const long kk = k + q * 4;
                    const bool v = m < p.M && kk < kend;
                    cp_async16(&As[st][r][q * 4], v ? (const void*)(p.A + (size_t)m * p.lda + kk) : (const void*)p.A,
                               v);
                } else {
                    const int f2 = f - A_CH;
                    const int kr = f2 / (TC / 4), q = f2 % (TC / 4);
                    const long kk = k + kr;
                    const int n = n0 + q * 4;
                    const bool v = kk < kend && n < p.N;
                    cp_async16(&Bs[st][kr][q * 4], v ? (const void*)(p.B + (size_t)kk * p.ldb + n) : (const void*)p.B,
                               v);
                }
            }
        };
        float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
        for (int kt = 0; kt < STAGES - 1; ++kt) {
            if (kt < nkb) issue(kt);
            cp_async_commit();
        }
        for (long kt = 0; kt < nkb; ++kt) {
            if (kt + STAGES - 1 < nkb) issue(kt + STAGES - 1);
            cp_async_commit();
            cp_async_wait<STAGES - 1>();
            __syncthreads();
            const int st = (int)(kt % STAGES);
#pragma unroll
            for (int k4 = 0; k4 < BK / 4; ++k4) {
                const float4 a0 = *reinterpret_cast<const float4*>(&As[st][2 * ty][k4 * 4]);
                const float4 a1 = *reinterpret_cast<const float4*>(&As[st][2 * ty + 1][k4 * 4]);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const float2 b = *reinterpret_cast<const float2*>(&Bs[st][k4 * 4 + kk][tx * 2]);
                    const float x0 = kk == 0 ? a0.x : kk == 1 ? a0.y : kk == 2 ? a0.z : a0.w;
                    const float x1 = kk == 0 ? a1.x : kk == 1 ? a1.y : kk == 2 ? a1.z : a1.w;
                    acc[0][0] = __fmaf_rn(x0, b.x, acc[0][0]);
                    acc[0][1] = __fmaf_rn(x0, b.y, acc[0][1]);
                    acc[1][0] = __fmaf_rn(x1, b.x, acc[1][0]);
                    acc[1][1] = __fmaf_rn(x1, b.y, acc[1][1]);
                }
            }
            __syncthreads();
        }
        cp_async_wait<0>();
        const bool first = (ci == c_first), last = (ci == c_last - 1);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int m = m0 + 2 * ty + i;
            if (m >= p.M) continue;
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int n = n0 + tx * 2 + j;
                if (n >= p.N) continue;
                const size_t wi = (size_t)m * p.N + n;
                const double s = first ? (double)acc[i][j] : Wg[wi] + (double)acc[i][j];
                if (last && p.G == 1) {
                    if (p.C64) p.C64[(size_t)m * p.ldc64 + n] = s;
                    else p.C[(size_t)m * p.ldc + n] = (float)s;
                } else {
                    Wg[wi] = s;
                }
            }
        }
    }
}

__global__ void k_reduce_f64(const double* __restrict__ P, int G, int M, int N, long ldp_plane, float* C,
                             long ldc, double* C64, long ldc64) {
    const size_t total = (size_t)M * N;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        // planes in order g = 0 .. G-1; eight loads are issued before their adds, so the loads overlap while the
        // additions keep their order
        double s = P[i];
        int g = 1;
        for (; g + 8 <= G; g += 8) {
            double v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = __ldg(P + (size_t)(g + u) * ldp_plane + i);
#pragma unroll
            for (int u = 0; u < 8; ++u) s += v[u];
        }
        for (; g < G; ++g) s += P[(size_t)g * ldp_plane + i];
        const size_t m = i / N, n = i - m * N;
        if (C64) C64[m * ldc64 + n] = s;
        else C[m * ldc + n] = (float)s;
    }
}

struct Shape {
    int bm;
    long kc;
    int ce, cpg, G;
    int tiles;
};

// Chunk groups for `tiles` output tiles: enough CTAs for `per_sm` per SM (two 8-warp CTAs, or four 4-warp CTAs of
// the narrow kernel), at most one group per chunk.
static int groups_for(int ce, long tiles, int sms, int per_sm = 2) {
    if (ce <= 1) return 1;
    long want = ((long)per_sm * sms + tiles - 1) / tiles;
    if (want < 1) want = 1;
    return (int)(want < ce ? want : ce);
}

// Tile edge: 128 when its tiles fill at least half the SMs (in the B200 tile table 128 won 83 of 87 FP32 shapes,
// by 30-50 % at 1024 x 2048 where its 128 tiles cover 86 % of the SMs); else 64 when its tiles x chunk groups fill
// the SMs; else 32 (2 x 2 chains per thread) when those fill the SMs; else the 16 x 32 tiles of k_fp32_narrow, so
// that a product with few output tiles and few chunks (M = N = 256, c = 1) spreads its FMA chains over more SMs.
// No chain changes with the tile.
// The 16-byte copies of the cp.async kernels need 16-byte aligned rows and K, N and the chunk length multiples of 4.
static bool vec_ok(const Fp32GemmArgs& a, long kc) {
    return (a.lda % 4 == 0) && (a.ldb % 4 == 0) && (a.N % 4 == 0) && (a.K % 4 == 0) && (kc % 4 == 0) &&
           ((reinterpret_cast<uintptr_t>(a.A) & 15) == 0) && ((reinterpret_cast<uintptr_t>(a.B) & 15) == 0);
}

// Tile codes: 128, 64, 32 (square tiles) and 16 (16 x 32 tiles of k_fp32_narrow).
static long tiles_of(const Fp32GemmArgs& a, int bm) {
    const int bn = bm == 16 ? 32 : bm;
    return (long)((a.M + bm - 1) / bm) * ((a.N + bn - 1) / bn);
}

Shape shape_of(const Fp32GemmArgs& a) {
    Shape s;
    const int sms = a.num_sms > 0 ? a.num_sms : 148;
    const int c = a.chunks < 1 ? 1 : a.chunks;
    s.kc = (a.K + c - 1) / c;
    if (s.kc < 1) s.kc = 1;
    s.ce = (int)((a.K + s.kc - 1) / s.kc);
    if (s.ce < 1) s.ce = 1;
    if (a.bm) s.bm = a.bm;
    else if (2 * tiles_of(a, 128) >= sms) s.bm = 128;
    else if (tiles_of(a, 64) * groups_for(s.ce, tiles_of(a, 64), sms) >= sms) s.bm = 64;
    else if (tiles_of(a, 32) * groups_for(s.ce, tiles_of(a, 32), sms) >= sms) s.bm = 32;
    else s.bm = 16;
    if (s.bm == 16 && !vec_ok(a, s.kc)) s.bm = 32;   // the narrow kernel exists only in the cp.async form
    s.tiles = (int)tiles_of(a, s.bm);
    const int G = groups_for(s.ce, s.tiles, sms, s.bm == 16 ? 4 : 2);
    s.cpg = (s.ce + G - 1) / G;
    s.G = (s.ce + s.cpg - 1) / s.cpg;
    return s;
}

template <int BM, int TM, bool VEC>
void launch_cfg(const Params& p, dim3 grid, cudaStream_t st) {
    k_fp32_gemm<BM, BM, TM, TM, VEC, 16><<<grid, kThr, 0, st>>>(p);
}

}  // namespace

int fp32_gemm_groups(const Fp32GemmArgs& a) { return shape_of(a).G; }

size_t fp32_gemm_ws_bytes(const Fp32GemmArgs& a) {
    Shape s = shape_of(a);
    if (s.G <= 1) {
        // A single group still needs the FP64 running sum when it has more than one chunk.
        return s.ce > 1 ? (size_t)a.M * a.N * sizeof(double) : 0;
    }
    return (size_t)s.G * a.M * a.N * sizeof(double);
}

int launch_fp32_gemm(const Fp32GemmArgs& a, void* stream) {
    if (a.M <= 0 || a.N <= 0 || a.K <= 0) return 0;
    Shape s = shape_of(a);
    Params p;
    p.A = a.A; p.lda = a.lda;
    p.B = a.B; p.ldb = a.ldb;
    p.C = a.C; p.ldc = a.ldc;
    p.C64 = a.C64; p.ldc64 = a.ldc64;
    p.W = a.ws64;
    p.M = a.M; p.N = a.N; p.K = a.K;
    p.kc = s.kc; p.ce = s.ce; p.cpg = s.cpg; p.G = s.G;
    if ((s.G > 1 || s.ce > 1) && !a.ws64) return (int)cudaErrorInvalidValue;
    const bool vec = vec_ok(a, s.kc);
    cudaStream_t st = (cudaStream_t)stream;
    const int bn = s.bm == 16 ? 32 : s.bm;
    dim3 grid((unsigned)((a.N + bn - 1) / bn), (unsigned)((a.M + s.bm - 1) / s.bm), (unsigned)s.G);
    if (s.bm == 128) {
        if (vec) launch_cfg<128, 8, true>(p, grid, st);
        else launch_cfg<128, 8, false>(p, grid, st);
    } else if (s.bm == 64) {
        if (vec) k_fp32_gemm_cp<64, 5><<<grid, kThr, 0, st>>>(p);
        else launch_cfg<64, 4, false>(p, grid, st);
    } else if (s.bm == 32) {
        if (vec) k_fp32_gemm_cp<32, 8><<<grid, kThr, 0, st>>>(p);
        else launch_cfg<32, 2, false>(p, grid, st);
    } else if (s.bm == 16) {
        constexpr int kNarrowStages = 4;   // 50 KB: four CTAs per SM
        const int smem = kNarrowStages * (16 * 68 + 64 * 32) * (int)sizeof(float);
        cudaError_t e = cudaFuncSetAttribute(k_fp32_narrow<kNarrowStages>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             smem);
        if (e != cudaSuccess) return (int)e;
        k_fp32_narrow<kNarrowStages><<<grid, 128, smem, st>>>(p);
    } else {
        return (int)cudaErrorInvalidValue;
    }
    count_launch();
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return (int)e;
    if (s.G > 1) return launch_reduce_f64(a.ws64, s.G, a.M, a.N, (long)a.M * a.N, a.C, a.ldc, a.C64, a.ldc64, stream);
    return 0;
}

int launch_reduce_f64(const double* P, int G, int M, int N, long ldp, float* C, long ldc, double* C64, long ldc64,
                      void* stream) {
    const size_t total = (size_t)M * N;
    if (total == 0) return 0;
    size_t blocks = (total + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    k_reduce_f64<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(P, G, M, N, ldp, C, ldc, C64, ldc64);
    count_launch();
    return (int)cudaGetLastError();
}

}  // namespace emu
