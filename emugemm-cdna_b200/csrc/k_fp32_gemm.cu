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
#include "device_utils.cuh"
#include "emugemm_internal.h"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <type_traits>

namespace emu {

bool tc_get_encode(PFN_cuTensorMapEncodeTiled_v12000* out);

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
    unsigned* err;      // the handle's error word (bounded waits of k_fp32_pipe)
    int stall;          // test hook (k_fp32_pipe): after k-block 0 lands every thread waits 1 ms on a barrier nothing arrives on
};

// The register-staged kernel, for operands the 16-byte copies of the other kernels cannot take (rows not 16-byte
// aligned, or K, N or the chunk length not a multiple of 4): scalar global loads staged through registers into
// double-buffered shared memory. kBKf: values of K per shared-memory stage (16; a 64-deep stage for the 32 tile
// measured slower: its unrolled k-loop ran at 64 registers with spills).
template <int BM, int BN, int TM, int TN, int kBKf>
__global__ void __launch_bounds__(kThr) k_fp32_gemm(Params p) {
    __shared__ __align__(16) float As[2][kBKf][BM];
    __shared__ __align__(16) float Bs[2][kBKf][BN];
    constexpr int HM = TM / 2, HN = TN / 2;
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

    float ra[A_SC];
    float rb[B_SC];

    auto load_global = [&](long kb, long kend) {
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
    };
    auto store_smem = [&](int buf) {
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
// for products with few output tiles (C3: M = N = 256) and mid-size ones. (At the 128 tile a ring of this kind measured
// 41.8 against 44.5 TFLOP/s for k_fp32_gemm at 8192^3; the TMA-fed k_fp32_pipe replaced both there, 51.4.) A
// register-staged k-block of prefetch left
// the global-load latency exposed on every k-block when a thread has few FMAs per loaded value; the ring keeps
// STAGES - 1 k-blocks of 16 in flight. Shared tiles keep the global layouts (A [m][k], B [k][n]): per four k a
// thread reads its TM rows of A as float4 along k and, per k, its TM columns of B as one vector, then runs the
// same chains (k ascending per element) with the same FP64 folds as k_fp32_gemm. Needs the vec_ok conditions
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

// Register-pipelined chains for products with few chains per SM sub-partition (C3: M = N = 256 holds 65536 chains,
// one warp of 2 x 2 chains per sub-partition of 128 SMs). BM x BN tile, TM x TN chains per thread, (BM/TM) x (BN/TN)
// threads, a STAGES-deep ring of 64-deep k-blocks. Two loaders, two kernels with the same k-loop:
// - k_fp32_pipe (32 x 64 tiles with 4 x 4 chains; 128 x 128 tiles with 8 x 8): TMA. One thread issues a k-block (two
//   32-deep boxes of A's rows with the 128-byte swizzle, one 64-row box of B) completing on the stage's mbarrier. It
//   runs the c = 4 and c = 16 products at 28.9 and 34.4 TFLOP/s against 17.5 and 29.4 for the 32 and 64 square tiles
//   (cp.async rings), and NATIVE 8192^3 at 51.4 against 44.5 for the register-staged 128 tile.
// - k_fp32_pipe_cp (16 x 32 tiles, 2 x 2 chains): per-thread 16-byte cp.async copies whose source pointers are set
//   once per chunk, A's rows padded to 68 floats. Its warp has the least slack (four chains per thread): the c = 1
//   product runs at 14.1 TFLOP/s; the TMA form of the same tile ran at 12.2, and the earlier cp.async kernel with two
//   barriers per k-block and per-copy index arithmetic at 12.5.
//
// With one warp per sub-partition nothing hides a shared-memory load's latency but the warp's own independent
// work, so the fragments of four k (TM float4 of A along k, four TN-vectors of B) are loaded PF steps ahead of the
// FMAs that use them, in PF + 1 register sets. One barrier per k-block: a thread loads the first fragments of the
// next k-block right after it, while it still multiplies the last PF steps of the current one, and the copies issued
// at the top of the next iteration refill the stage every thread finished reading before that barrier.
//
// Warp layout: 4 rows of threads x 8 columns, so a warp reads 4 distinct rows of A (rows i*TY + ty interleaved; the
// swizzle or the padding puts their 16-byte pieces in distinct bank groups) and, per k and load instruction, 8
// contiguous TN-vectors of B: one wavefront per load instruction. TMA fills with zeros only outside the matrices, so
// the last k-block of a chunk that ends inside K holds the next chunk's values past the chunk end: that block runs a
// copy of the unrolled loop that stops at the chunk end (chunk lengths are multiples of 4; full k-blocks carry no
// per-step test; cp.async fills past the chunk end with zeros). Same chains (k ascending per element), same FP64 folds
// and the same vec_ok conditions as k_fp32_gemm_cp.
struct PipeMaps {
    CUtensorMap a;   // A: x = k, y = row; box 32 x BM, 128-byte swizzle
    CUtensorMap b;   // B: x = column, y = k; box BN x 64
};

template <int BM, int BN>
constexpr int pipe_smem_bytes(int stages) {   // alignment slack, A and B stages, mbarriers
    return 1024 + stages * (BM * 64 + 64 * BN) * 4 + (stages + 1) * 8;
}

template <int BM, int BN, int TM, int TN, int STAGES, int PF>
__global__ void __launch_bounds__((BM / TM) * (BN / TN)) k_fp32_pipe(const __grid_constant__ PipeMaps maps,
                                                                      Params p) {
    constexpr int BK = 64, STEPS = BK / 4, NF = PF + 1;
    constexpr int TX = BN / TN, TY = BM / TM;
    constexpr int A_STAGE = BM * BK, B_STAGE = BK * BN;   // floats
    constexpr uint32_t STAGE_BYTES = (A_STAGE + B_STAGE) * 4;
    static_assert(TX % 8 == 0 && TY % 8 == 0 && (TN == 2 || TN == 4 || TN == 8), "warp layout");
    constexpr int CW = TN == 8 ? BN / 2 : 4;   // TN = 8: a thread's columns come in two groups of four, BN/2 apart
    // TN = 8 (8 x 8 chains): B is read at its use, not PF steps ahead (four k of B would be 32 more registers per
    // fragment set); then the last PF steps of a k-block still read its B after the barrier, so a stage is refilled
    // one k-block later (LA k-blocks in flight instead of STAGES - 1).
    constexpr bool BJIT = TN == 8;
    constexpr int LA = BJIT ? STAGES - 2 : STAGES - 1;
    static_assert(LA >= 1, "k-blocks in flight");
    static_assert(PF >= 1 && STEPS % NF == 0 && STAGES >= 2, "fragment ring");
    static_assert(BM % 8 == 0 && BM <= 256 && BN * 4 % 16 == 0 && BN <= 256, "TMA boxes");
    extern __shared__ __align__(16) unsigned char pipe_raw[];
    const uint32_t raw = dev::smem_u32(pipe_raw);
    float* const base = reinterpret_cast<float*>(pipe_raw + (((raw + 1023u) & ~1023u) - raw));   // 1024-aligned
    float* const As = base;                                // [stage][half][BM][32], swizzled 128-byte rows
    float* const Bs = base + STAGES * A_STAGE;             // [stage][64][BN]
    uint64_t* const full = reinterpret_cast<uint64_t*>(Bs + STAGES * B_STAGE);
    __shared__ int abort_flag;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int tx = (warp % (TX / 8)) * 8 + (lane & 7);     // columns tx*TN .. tx*TN + TN-1
    const int ty = (warp / (TX / 8)) * 4 + (lane >> 3);    // rows ty, ty + TY, ..., ty + (TM-1)*TY
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int g = blockIdx.z;
    const int c_first = g * p.cpg;
    const int c_last = min(p.ce, c_first + p.cpg);
    double* Wg = p.W ? p.W + (size_t)g * p.M * p.N : nullptr;
    uint64_t* const never = full + STAGES;   // the test hook's barrier: nothing arrives on it
    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) dev::mbar_init(&full[s], 1);
        dev::mbar_init(never, 1);
        abort_flag = 0;
        dev::fence_mbar_init();
        dev::prefetch_tmap(&maps.a);
        dev::prefetch_tmap(&maps.b);
    }
    __syncthreads();

    struct Frag {
        float4 a[TM];
        float b[BJIT ? 1 : 4][TN];
    };
    // Step s of a k-block covers k = 4s .. 4s+3: A half s / 8, 16-byte piece s % 8 of each 128-byte row, stored at
    // piece (s % 8) ^ (row % 8). A thread's rows i*TY + ty all have row % 8 = ty % 8 (TY is a multiple of 8), so the
    // eight offsets are set once.
    int aoff[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) aoff[c] = ty * 32 + ((c ^ (ty & 7)) << 2);
    auto load_frag = [&](Frag& f, int st, int s) {
        const float* a_row = As + st * A_STAGE + (s >> 3) * (BM * 32) + aoff[s & 7];
#pragma unroll
        for (int i = 0; i < TM; ++i) f.a[i] = *reinterpret_cast<const float4*>(a_row + i * TY * 32);
        const float* b_st = Bs + st * B_STAGE;
#pragma unroll
        for (int kk = 0; kk < (BJIT ? 0 : 4); ++kk) {
            if (TN == 2) {
                const float2 v = *reinterpret_cast<const float2*>(b_st + (s * 4 + kk) * BN + tx * 2);
                f.b[kk][0] = v.x; f.b[kk][1] = v.y;
            } else {
#pragma unroll
                for (int h = 0; h < TN / 4; ++h) {
                    const float4 v = *reinterpret_cast<const float4*>(b_st + (s * 4 + kk) * BN + h * CW + tx * 4);
                    f.b[kk][4 * h] = v.x; f.b[kk][4 * h + 1] = v.y; f.b[kk][4 * h + 2] = v.z; f.b[kk][4 * h + 3] = v.w;
                }
            }
        }
    };
    long ring = 0;   // ring index of the current chunk's k-block 0 (k-blocks run through the stages in order)
    bool ok = true;  // false after a wait gave up: the kernel runs on over whatever the ring holds, and reports
    long issued = 0;  // thread 0: k-blocks issued (none after one of its own waits gave up)

    for (int ci = c_first; ci < c_last; ++ci) {
        const long kbeg = (long)ci * p.kc;
        const long kend = min(p.K, kbeg + p.kc);
        const long nkb = (kend - kbeg + BK - 1) / BK;
        auto issue_block = [&](long kt) {   // by thread 0, k-blocks in order
            if (tid == 0 && ok) {   // thread 0 waited for every earlier k-block of this stage itself
                const long q = ring + kt;
                issued = q + 1;
                const int st = (int)(q % STAGES);
                const int k = (int)(kbeg + kt * BK);
                dev::mbar_arrive_expect_tx(&full[st], STAGE_BYTES);
                dev::tma_load_2d(As + st * A_STAGE, &maps.a, &full[st], k, m0);
                dev::tma_load_2d(As + st * A_STAGE + BM * 32, &maps.a, &full[st], k + 32, m0);
                dev::tma_load_2d(Bs + st * B_STAGE, &maps.b, &full[st], n0, k);
            }
        };
        auto wait_block = [&](long kt) {   // by every thread: k-block kt has landed
            const long q = ring + kt;
            if (!dev::mbar_wait(&full[q % STAGES], (uint32_t)((q / STAGES) & 1), &abort_flag, p.err, kErrTimeoutFp32))
                ok = false;
        };
        float acc[TM][TN];
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
            for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;
        for (int kt = 0; kt < LA && kt < nkb; ++kt) issue_block(kt);
        wait_block(0);
        // test hook: with the first k-blocks issued, every thread gives up a 1 ms wait on a barrier nothing arrives on
        if (p.stall && ring == 0 && !dev::mbar_wait_for(never, 0, &abort_flag, p.err, kErrTimeoutFp32, 1000000ull))
            ok = false;
        Frag fr[NF];
#pragma unroll
        for (int s = 0; s < PF; ++s) load_frag(fr[s], (int)(ring % STAGES), s);
        for (long kt = 0; kt < nkb; ++kt) {
            const int st = (int)((ring + kt) % STAGES);
            const bool more = kt + 1 < nkb;
            // refills the stage of k-block kt + LA - STAGES (kt - 1, or kt - 2 when B is read at its use): every thread
            // issued its last read of it before the previous barrier
            if (kt + LA < nkb) issue_block(kt + LA);
            const long left = kend - (kbeg + kt * BK);
            // one k-block; GUARD: the chunk ends inside it and only its first vs steps run (a separate copy of the
            // unrolled loop, so full k-blocks carry no per-step test)
            auto run_block = [&](auto guard, int vs) {
                constexpr bool GUARD = decltype(guard)::value;
#pragma unroll
                for (int s = 0; s < STEPS; ++s) {
                    const int ls = s + PF;   // the step whose fragments are loaded now
                    if (ls < STEPS) {
                        load_frag(fr[ls % NF], st, ls);
                    } else {
                        if (ls == STEPS) {
                            if (more) wait_block(kt + 1);
                            __syncthreads();
                        }
                        if (more) load_frag(fr[ls % NF], (int)((ring + kt + 1) % STAGES), ls - STEPS);
                    }
                    if (!GUARD || s < vs) {
                        const Frag& f = fr[s % NF];
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk) {
                            float bj[TN];
#pragma unroll
                            for (int j = 0; j < TN; ++j) bj[j] = BJIT ? 0.f : f.b[BJIT ? 0 : kk][j];
                            if (BJIT) {
                                const float* b_row = Bs + st * B_STAGE + (s * 4 + kk) * BN + tx * 4;
#pragma unroll
                                for (int h = 0; h < TN / 4; ++h) {
                                    const float4 v = *reinterpret_cast<const float4*>(b_row + h * CW);
                                    bj[4 * h] = v.x; bj[4 * h + 1] = v.y; bj[4 * h + 2] = v.z; bj[4 * h + 3] = v.w;
                                }
                            }
#pragma unroll
                            for (int i = 0; i < TM; ++i) {
                                const float av = kk == 0 ? f.a[i].x : kk == 1 ? f.a[i].y : kk == 2 ? f.a[i].z : f.a[i].w;
#pragma unroll
                                for (int j = 0; j < TN; ++j) acc[i][j] = __fmaf_rn(av, bj[j], acc[i][j]);
                            }
                        }
                    }
                }
            };
            if (left >= BK) run_block(std::false_type{}, STEPS);
            else run_block(std::true_type{}, (int)(left >> 2));   // chunk lengths are multiples of 4
        }
        ring += nkb;
        const bool first = (ci == c_first), last = (ci == c_last - 1);
#pragma unroll
        for (int i = 0; i < TM; ++i) {
            const int m = m0 + i * TY + ty;
            if (m >= p.M) continue;
#pragma unroll
            for (int j = 0; j < TN; ++j) {
                const int n = n0 + (TN == 2 ? tx * 2 + j : (j / 4) * CW + tx * 4 + (j % 4));
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
    // After a wait gave up, no k-block is issued any more, and the loads still in flight land before the CTA's shared
    // memory is released: thread 0 waits (bounded, ignoring the abort flag) for the last k-block issued into each
    // stage.
    if (!ok && tid == 0) {
        int no_abort = 0;
        for (long q = issued > STAGES ? issued - STAGES : 0; q < issued; ++q)
            dev::mbar_wait(&full[q % STAGES], (uint32_t)((q / STAGES) & 1), &no_abort, nullptr, 0);
    }
}

template <int BM, int BN, int TM, int TN, int STAGES, int PF>
__global__ void __launch_bounds__((BM / TM) * (BN / TN)) k_fp32_pipe_cp(Params p) {
    constexpr int BK = 64, BKP = BK + 4, STEPS = BK / 4, NF = PF + 1;
    constexpr int TX = BN / TN, TY = BM / TM, NT = TX * TY;
    constexpr int A_CH = BM * BK / 4, CH = A_CH + BK * BN / 4, CPT = CH / NT, CA = A_CH / NT;
    static_assert(A_CH % NT == 0 && CH % NT == 0, "whole 16-byte copies of A and of B per thread");
    static_assert(TX % 8 == 0 && TY % 4 == 0 && (TN == 2 || TN == 4), "warp layout");
    static_assert(PF >= 1 && STEPS % NF == 0 && STAGES >= 2, "fragment ring");
    extern __shared__ __align__(16) float pipe_cp_smem[];
    auto As = reinterpret_cast<float (*)[BM][BKP]>(pipe_cp_smem);                       // [stage][m][k], rows padded
    auto Bs = reinterpret_cast<float (*)[BK][BN]>(pipe_cp_smem + STAGES * BM * BKP);   // [stage][k][n]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int tx = (warp % (TX / 8)) * 8 + (lane & 7);     // columns tx*TN .. tx*TN + TN-1
    const int ty = (warp / (TX / 8)) * 4 + (lane >> 3);    // rows ty, ty + TY, ..., ty + (TM-1)*TY
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int g = blockIdx.z;
    const int c_first = g * p.cpg;
    const int c_last = min(p.ce, c_first + p.cpg);
    double* Wg = p.W ? p.W + (size_t)g * p.M * p.N : nullptr;

    struct Frag {
        float4 a[TM];
        float b[4][TN];
    };
    auto load_frag = [&](Frag& f, int st, int s) {
#pragma unroll
        for (int i = 0; i < TM; ++i) f.a[i] = *reinterpret_cast<const float4*>(&As[st][i * TY + ty][s * 4]);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            if (TN == 2) {
                const float2 v = *reinterpret_cast<const float2*>(&Bs[st][s * 4 + kk][tx * 2]);
                f.b[kk][0] = v.x; f.b[kk][1] = v.y;
            } else {
                const float4 v = *reinterpret_cast<const float4*>(&Bs[st][s * 4 + kk][tx * 4]);
                f.b[kk][0] = v.x; f.b[kk][1] = v.y; f.b[kk][2] = v.z; f.b[kk][3] = v.w;
            }
        }
    };

    for (int ci = c_first; ci < c_last; ++ci) {
        const long kbeg = (long)ci * p.kc;
        const long kend = min(p.K, kbeg + p.kc);
        const long nkb = (kend - kbeg + BK - 1) / BK;
        // This thread's 16-byte copies of a k-block (the first CA of A, the rest of B): source pointers set once per
        // chunk and advanced by one k-block per issue, so a copy costs a compare and a pointer add, not the index
        // arithmetic (a thread here has only TM * TN FMAs per k to spread that over).
        const float* src[CPT];
        float* dst[CPT];
        int kofs[CPT];   // k of the copy's first element within its k-block
        bool inb[CPT];   // row of A / columns of B inside the product
#pragma unroll
        for (int c = 0; c < CPT; ++c) {
            const int f = tid + c * NT;
            if (c < CA) {
                const int r = f / (BK / 4), q = f % (BK / 4);
                inb[c] = m0 + r < p.M;
                kofs[c] = q * 4;
                src[c] = p.A + (size_t)(inb[c] ? m0 + r : 0) * p.lda + kbeg + q * 4;
                dst[c] = &As[0][r][q * 4];
            } else {
                const int f2 = f - A_CH;
                const int kr = f2 / (BN / 4), q = f2 % (BN / 4);
                inb[c] = n0 + q * 4 < p.N;
                kofs[c] = kr;
                src[c] = p.B + (size_t)(kbeg + kr) * p.ldb + (inb[c] ? n0 + q * 4 : 0);
                dst[c] = &Bs[0][kr][q * 4];
            }
        }
        const long b_step = (long)BK * p.ldb;
        auto issue = [&](long kt) {   // called for kt = 0, 1, 2, ... in order
            const int st = (int)(kt % STAGES);
            const long left = kend - (kbeg + kt * BK);   // K values left from this k-block's start
#pragma unroll
            for (int c = 0; c < CPT; ++c) {
                const bool v = inb[c] && kofs[c] < left;
                float* d = dst[c] + (c < CA ? st * (BM * BKP) : st * (BK * BN));
                cp_async16(d, v ? (const void*)src[c] : (const void*)p.A, v);
                src[c] += c < CA ? (long)BK : b_step;
            }
        };
        float acc[TM][TN];
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
            for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;
        for (int kt = 0; kt < STAGES - 1; ++kt) {
            if (kt < nkb) issue(kt);
            cp_async_commit();
        }
        cp_async_wait<STAGES - 2>();   // k-block 0 has landed (this thread's copies)
        __syncthreads();               // ... and every thread's
        Frag fr[NF];
#pragma unroll
        for (int s = 0; s < PF; ++s) load_frag(fr[s], 0, s);
        for (long kt = 0; kt < nkb; ++kt) {
            const int st = (int)(kt % STAGES);
            const bool more = kt + 1 < nkb;
            // refills stage (kt - 1) % STAGES: every thread issued its last read of it before the previous barrier
            if (kt + STAGES - 1 < nkb) issue(kt + STAGES - 1);
            cp_async_commit();
#pragma unroll
            for (int s = 0; s < STEPS; ++s) {
                const int ls = s + PF;   // the step whose fragments are loaded now
                if (ls < STEPS) {
                    load_frag(fr[ls % NF], st, ls);
                } else {
                    if (ls == STEPS) {
                        if (more) cp_async_wait<STAGES - 2>();   // k-block kt + 1 has landed
                        __syncthreads();
                    }
                    if (more) load_frag(fr[ls % NF], (int)((kt + 1) % STAGES), ls - STEPS);
                }
                const Frag& f = fr[s % NF];
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
                    for (int i = 0; i < TM; ++i) {
                        const float av = kk == 0 ? f.a[i].x : kk == 1 ? f.a[i].y : kk == 2 ? f.a[i].z : f.a[i].w;
#pragma unroll
                        for (int j = 0; j < TN; ++j) acc[i][j] = __fmaf_rn(av, f.b[kk][j], acc[i][j]);
                    }
                }
            }
        }
        cp_async_wait<0>();   // only empty groups remain; the next chunk's prologue refills stages 0 .. STAGES-2
        const bool first = (ci == c_first), last = (ci == c_last - 1);
#pragma unroll
        for (int i = 0; i < TM; ++i) {
            const int m = m0 + i * TY + ty;
            if (m >= p.M) continue;
#pragma unroll
            for (int j = 0; j < TN; ++j) {
                const int n = n0 + tx * TN + j;
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
// the 16 x 32 tiles), at most one group per chunk.
static int groups_for(int ce, long tiles, int sms, int per_sm = 2) {
    if (ce <= 1) return 1;
    long want = ((long)per_sm * sms + tiles - 1) / tiles;
    if (want < 1) want = 1;
    return (int)(want < ce ? want : ce);
}

// Tile: 128 when its tiles fill at least half the SMs (in the B200 tile table 128 won 83 of 87 FP32 shapes, by
// 30-50 % at 1024 x 2048 where its 128 tiles cover 86 % of the SMs); else the 32 x 64 tiles of k_fp32_pipe when their
// tiles x chunk groups give between half a CTA and two CTAs per SM (one wave); else 64 when its tiles x chunk groups
// fill the SMs; else 32 (2 x 2 chains per thread) when those fill the SMs; else the 16 x 32 tiles of k_fp32_pipe, so
// that a product with few output tiles and few chunks (M = N = 256, c = 1) spreads its FMA chains over more SMs.
// No chain changes with the tile.
// The 16-byte copies of the cp.async kernels need 16-byte aligned rows and K, N and the chunk length multiples of 4.
// (TMA coordinates are 32-bit: K below 2^31 - 64.)
static bool vec_ok(const Fp32GemmArgs& a, long kc) {
    return (a.lda % 4 == 0) && (a.ldb % 4 == 0) && (a.N % 4 == 0) && (a.K % 4 == 0) && (kc % 4 == 0) &&
           a.K < (1L << 31) - 64 &&
           ((reinterpret_cast<uintptr_t>(a.A) & 15) == 0) && ((reinterpret_cast<uintptr_t>(a.B) & 15) == 0);
}

// Tile codes: 128, 64, 32 (square tiles), 16 (16 x 32, k_fp32_pipe_cp) and 3264 (32 x 64, k_fp32_pipe).
static void tile_dims(int code, int& bm, int& bn) {
    if (code == 16) { bm = 16; bn = 32; }
    else if (code == 3264) { bm = 32; bn = 64; }
    else { bm = code; bn = code; }
}
static int per_sm_of(int code) { return code == 16 ? 4 : 2; }   // CTAs resident per SM, for the chunk groups
static long tiles_of(const Fp32GemmArgs& a, int code) {
    int bm, bn;
    tile_dims(code, bm, bn);
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
    const long t3264 = tiles_of(a, 3264);
    const int g3264 = groups_for(s.ce, t3264, sms), cpg3264 = (s.ce + g3264 - 1) / g3264;
    const long ctas3264 = t3264 * ((s.ce + cpg3264 - 1) / cpg3264);   // groups after rounding to whole chunks
    if (a.bm) s.bm = a.bm;
    else if (2 * tiles_of(a, 128) >= sms) s.bm = 128;
    else if (2 * ctas3264 >= sms && ctas3264 <= 2L * sms) s.bm = 3264;
    else if (tiles_of(a, 64) * groups_for(s.ce, tiles_of(a, 64), sms) >= sms) s.bm = 64;
    else if (tiles_of(a, 32) * groups_for(s.ce, tiles_of(a, 32), sms) >= sms) s.bm = 32;
    else s.bm = 16;
    // k_fp32_pipe_cp and k_fp32_pipe need 16-byte aligned rows and chunks, and k_fp32_pipe TMA
    if ((s.bm == 16 || s.bm == 3264) && !vec_ok(a, s.kc)) s.bm = 32;
    if (s.bm == 3264) {
        PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
        if (!tc_get_encode(&enc)) s.bm = 32;
    }
    s.tiles = (int)tiles_of(a, s.bm);
    const int G = groups_for(s.ce, s.tiles, sms, per_sm_of(s.bm));
    s.cpg = (s.ce + G - 1) / G;
    s.G = (s.ce + s.cpg - 1) / s.cpg;
    return s;
}

template <int BM, int TM>
void launch_cfg(const Params& p, dim3 grid, cudaStream_t st) {
    k_fp32_gemm<BM, BM, TM, TM, 16><<<grid, kThr, 0, st>>>(p);
}

// A: x = k (32-deep boxes, 128-byte swizzle), y = row; B: x = column, y = k (64-deep boxes). Needs the vec_ok conditions
// (16-byte aligned operands, leading dimensions multiples of 4), which shape_of checks before choosing these tiles.
template <int BM, int BN, int TM, int TN, int STAGES, int PF>
cudaError_t launch_pipe(const Fp32GemmArgs& a, const Params& p, dim3 grid, cudaStream_t st) {
    PipeMaps maps;
    PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
    if (!tc_get_encode(&enc)) return cudaErrorNotSupported;
    {
        cuuint64_t dims[2] = {(cuuint64_t)a.K, (cuuint64_t)a.M};
        cuuint64_t strides[1] = {(cuuint64_t)a.lda * 4};
        cuuint32_t box[2] = {32, (cuuint32_t)BM};
        cuuint32_t estr[2] = {1, 1};
        if (enc(&maps.a, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(a.A), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    {
        cuuint64_t dims[2] = {(cuuint64_t)a.N, (cuuint64_t)a.K};
        cuuint64_t strides[1] = {(cuuint64_t)a.ldb * 4};
        cuuint32_t box[2] = {(cuuint32_t)BN, 64};
        cuuint32_t estr[2] = {1, 1};
        if (enc(&maps.b, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(a.B), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    const int smem = pipe_smem_bytes<BM, BN>(STAGES);
    auto kern = k_fp32_pipe<BM, BN, TM, TN, STAGES, PF>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    Params q = p;
    q.stall = take_test_stall() ? 1 : 0;
    kern<<<grid, (BM / TM) * (BN / TN), smem, st>>>(maps, q);
    return cudaSuccess;
}

template <int BM, int BN, int TM, int TN, int STAGES, int PF>
cudaError_t launch_pipe_cp(const Params& p, dim3 grid, cudaStream_t st) {
    const int smem = STAGES * (BM * 68 + 64 * BN) * (int)sizeof(float);
    auto kern = k_fp32_pipe_cp<BM, BN, TM, TN, STAGES, PF>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    kern<<<grid, (BM / TM) * (BN / TN), smem, st>>>(p);
    return cudaSuccess;
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
    p.err = a.err;
    p.stall = 0;
    if ((s.G > 1 || s.ce > 1) && !a.ws64) return (int)cudaErrorInvalidValue;
    const bool vec = vec_ok(a, s.kc);
    cudaStream_t st = (cudaStream_t)stream;
    int bm, bn;
    tile_dims(s.bm, bm, bn);
    dim3 grid((unsigned)((a.N + bn - 1) / bn), (unsigned)((a.M + bm - 1) / bm), (unsigned)s.G);
    if (s.bm == 128) {
        // 16-byte aligned operands: the TMA-fed k_fp32_pipe with 8 x 8 chains per thread (NATIVE 8192^3 at 51.4
        // TFLOP/s against 44.5 for the register-staged k_fp32_gemm, and ahead at 1024^3 to 4096^3 as well); else, or
        // without TMA, k_fp32_gemm. Same chains either way.
        PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
        if (vec && tc_get_encode(&enc)) {
            cudaError_t e = launch_pipe<128, 128, 8, 8, 3, 1>(a, p, grid, st);
            if (e != cudaSuccess) return (int)e;
        } else {
            launch_cfg<128, 8>(p, grid, st);
        }
    } else if (s.bm == 64) {
        if (vec) k_fp32_gemm_cp<64, 5><<<grid, kThr, 0, st>>>(p);
        else launch_cfg<64, 4>(p, grid, st);
    } else if (s.bm == 32) {
        if (vec) k_fp32_gemm_cp<32, 8><<<grid, kThr, 0, st>>>(p);
        else launch_cfg<32, 2>(p, grid, st);
    } else if (s.bm == 16) {
        cudaError_t e = launch_pipe_cp<16, 32, 2, 2, 4, 3>(p, grid, st);
        if (e != cudaSuccess) return (int)e;
    } else if (s.bm == 3264) {
        cudaError_t e = launch_pipe<32, 64, 4, 4, 4, 1>(a, p, grid, st);
        if (e != cudaSuccess) return (int)e;
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
