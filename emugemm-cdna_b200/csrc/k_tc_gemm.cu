// k_tc_gemm.cu - the 3-product emulated-FP32 GEMM on the sm_100a tensor cores.
//
// C = A_hi*B_hi + A_lo*B_hi + A_hi*B_lo, the three slice products of the bf16x3 / fp16x3 schemes
// (emugemm-cdna src/emugemm.cpp:331-356, where they are three rocBLAS calls with beta=1). Here the three
// products of every k-step are issued back to back as tcgen05.mma into one TMEM accumulator (bf16x3) or
// into two (fp16x3: hi*hi and the two cross products, which carry the lo slice's 2^11 factor), so C is
// written once.
//
// Promotion. The tensor-core FP32 accumulator truncates its partial sums (measured on B200: the error of
// an accumulation grows linearly in K with a systematic bias toward zero, about 4e-6 relative at
// K = 4096), which would exceed the bf16x3 floor by K ~ 4000. So a TMEM accumulator only ever sums one
// chunk of kChunkKB k-blocks (128 values of K); the epilogue warps drain every chunk into FP32 registers
// with round-to-nearest adds while the MMAs of the next chunk run into the other TMEM buffer. Measured at
// 8192^3 on N(0,1) data: chunks of 64/128/256/512 values of K give bf16x3 errors 4.43/4.44/4.50/4.72e-6
// (the representation floor of the split is 4.4355e-6) for kernel times 2.44/2.34/2.30/2.25 ms.
//
// Operands are pre-split 16-bit slices in HBM, K-major (A: Mp x Kp, B transposed: Np x Kp), loaded by
// TMA with the 128-byte swizzle straight into the UMMA canonical layout.
//
// Warp roles (320 threads, one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer (one elected thread)
//   warp 1      TMEM allocator and MMA issuer (one elected thread)
//   warps 2..9  promotion/epilogue: warp w drains TMEM lanes 32*(w%4).. and half (w-2)/4 of the columns,
//               keeps the running FP32 sums of its 32 rows x BN/2 columns in registers, stores C
// TMEM holds two accumulator buffers (512 columns) that alternate chunk by chunk. Every wait is bounded;
// on a timeout the kernel records it in the error word, drains its copies and MMAs in flight, frees TMEM
// and returns.
#include "device_utils.cuh"
#include "emugemm_internal.h"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>

namespace emu {
namespace {

using namespace dev;

constexpr int kBM = 128;
#ifndef EMUGEMM_TC_BK
#define EMUGEMM_TC_BK 64
#endif
constexpr int kBK = EMUGEMM_TC_BK;   // k-block: 64 (rows of 128 B, 128-byte swizzle) or 32 (64-byte swizzle)
constexpr int kSwizzleBytes = kBK * 2;
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
#ifndef EMUGEMM_CHUNK_K
#define EMUGEMM_CHUNK_K 128
#endif
constexpr int kChunkKB = EMUGEMM_CHUNK_K / kBK;   // k-blocks accumulated in TMEM before promotion
constexpr int kGroupM = 16;          // tile raster: groups of 16 row blocks sweep all column blocks

template <bool FP16>
struct Cfg {
    static constexpr int BN = FP16 ? 128 : 256;
    static constexpr int A_BYTES = kBM * kBK * 2;
    static constexpr int B_BYTES = BN * kBK * 2;
    static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
    static constexpr int STAGES = (196608 / STAGE_BYTES) < 6 ? (196608 / STAGE_BYTES) : 6;
    static constexpr int ACC_COLS = FP16 ? 2 * BN : BN;    // TMEM columns per accumulator buffer
    static constexpr int HALF = BN / 2;                     // columns per epilogue thread
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*control*/;
    static constexpr uint32_t IDESC = idesc_f16(kBM, BN, !FP16);
    // fp16: A_hi x [B_hi | B_lo] as one MMA of twice the width (the two B slices are adjacent in the stage and the
    // two accumulators adjacent in TMEM), so A_hi is read from shared memory once per k16 step instead of twice
    static constexpr uint32_t IDESC2 = idesc_f16(kBM, 2 * BN, !FP16);
};

struct Ctl {
    uint64_t full[8];
    uint64_t empty[8];
    uint64_t tmem_full[2];
    uint64_t tmem_empty[2];
    uint64_t drain;
    uint64_t never;            // nothing arrives on it: the target of the test stall below
    uint32_t tmem_base;
    int abort;
};

struct KParams {
    int M, N, num_m, num_n, nk;
    int kpb;   // k-blocks per K panel of the slices
    float* C; long ldc;
    double* C64; long ldc64;
    const int* row_exp; const int* col_exp;
    unsigned* err;
    int stall_chunk;   // test hook: the MMA issuer waits on `never` before this chunk (-1: never)
};

// Limit of the test stall's wait: short, so a test of failure reporting takes about a millisecond.
constexpr unsigned long long kStallLimitNs = 1000000ull;

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& mb, int& nb) {
    const int per_group = kGroupM * num_n;
    const int g = t / per_group;
    const int first_m = g * kGroupM;
    const int gm = min(num_m - first_m, kGroupM);
    const int r = t - g * per_group;
    mb = first_m + r % gm;
    nb = r / gm;
}

// Bounded wait used while unwinding: ignores the abort flag, shorter limit.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    unsigned long long t0 = globaltimer();
    while (!mbar_try_wait(a, parity)) {
        if (globaltimer() - t0 > 200000000ull) return;
    }
}

template <bool FP16>
__global__ void __launch_bounds__(kThreads, 1)
    k_tc_gemm(const __grid_constant__ CUtensorMap tm_ahi, const __grid_constant__ CUtensorMap tm_alo,
              const __grid_constant__ CUtensorMap tm_bhi, const __grid_constant__ CUtensorMap tm_blo, KParams p) {
    using C_ = Cfg<FP16>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Ctl* ctl = reinterpret_cast<Ctl*>(smem + C_::STAGES * C_::STAGE_BYTES);
    volatile int* abort = &ctl->abort;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int num_tiles = p.num_m * p.num_n;
    const int nchunks = (p.nk + kChunkKB - 1) / kChunkKB;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C_::STAGES; ++s) {
            mbar_init(&ctl->full[s], 1);
            mbar_init(&ctl->empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&ctl->tmem_full[b], 1);
            mbar_init(&ctl->tmem_empty[b], 32 * kEpiWarps);
        }
        mbar_init(&ctl->drain, 1);
        mbar_init(&ctl->never, 1);
        ctl->abort = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tm_ahi);
        prefetch_tmap(&tm_alo);
        prefetch_tmap(&tm_bhi);
        prefetch_tmap(&tm_blo);
    }
    if (warp == 1) {
        tmem_alloc(&ctl->tmem_base, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = ctl->tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            long it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                int mb, nb;
                tile_coords(t, p.num_m, p.num_n, mb, nb);
                for (int kb = 0; kb < p.nk; ++kb, ++it) {
                    const int s = (int)(it % C_::STAGES);
                    const uint32_t ph = (uint32_t)((it / C_::STAGES) & 1);
                    if (!mbar_wait(&ctl->empty[s], ph ^ 1u, abort, p.err, kErrTimeoutProducer)) { ok = false; break; }
                    uint8_t* st = smem + s * C_::STAGE_BYTES;
                    mbar_arrive_expect_tx(&ctl->full[s], C_::STAGE_BYTES);
                    const int kz = kb / p.kpb, kx = (kb - kz * p.kpb) * kBK;
                    tma_load_3d(st, &tm_ahi, &ctl->full[s], kx, mb * kBM, kz);
                    tma_load_3d(st + C_::A_BYTES, &tm_alo, &ctl->full[s], kx, mb * kBM, kz);
                    tma_load_3d(st + 2 * C_::A_BYTES, &tm_bhi, &ctl->full[s], kx, nb * C_::BN, kz);
                    tma_load_3d(st + 2 * C_::A_BYTES + C_::B_BYTES, &tm_blo, &ctl->full[s], kx, nb * C_::BN, kz);
                }
            }
            if (!ok) {
                // Let the loads already issued land before the CTA can exit.
                const long first = it > C_::STAGES ? it - C_::STAGES : 0;
                for (long j = first; j < it; ++j)
                    drain_wait(&ctl->full[j % C_::STAGES], (uint32_t)((j / C_::STAGES) & 1));
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer: one TMEM buffer per chunk of kChunkKB k-blocks ----------------
            long it = 0, ch = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                for (int kb0 = 0; kb0 < p.nk && ok; kb0 += kChunkKB, ++ch) {
                    const int b = (int)(ch & 1);
                    const uint32_t bph = (uint32_t)((ch >> 1) & 1);
                    // test hook: a wait that must run out, with MMAs of earlier chunks and loads of later stages in
                    // flight; the kernel then unwinds exactly as after any timed-out wait
                    if (ch == (long)p.stall_chunk &&
                        !mbar_wait_for(&ctl->never, 0, abort, p.err, kErrTimeoutMma, kStallLimitNs)) {
                        ok = false;
                        break;
                    }
                    if (!mbar_wait(&ctl->tmem_empty[b], bph ^ 1u, abort, p.err, kErrTimeoutMma)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t d_main = tmem_base + (uint32_t)(b * C_::ACC_COLS);
                    const uint32_t d_cross = FP16 ? d_main + (uint32_t)C_::BN : d_main;
                    const int kb1 = min(p.nk, kb0 + kChunkKB);
                    for (int kb = kb0; kb < kb1; ++kb, ++it) {
                        const int s = (int)(it % C_::STAGES);
                        const uint32_t ph = (uint32_t)((it / C_::STAGES) & 1);
                        if (!mbar_wait(&ctl->full[s], ph, abort, p.err, kErrTimeoutMma)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t st = smem_u32(smem + s * C_::STAGE_BYTES);
                        const uint64_t a_hi = sdesc_kmajor(st, kSwizzleBytes);
                        const uint64_t a_lo = sdesc_kmajor(st + C_::A_BYTES, kSwizzleBytes);
                        const uint64_t b_hi = sdesc_kmajor(st + 2 * C_::A_BYTES, kSwizzleBytes);
                        const uint64_t b_lo = sdesc_kmajor(st + 2 * C_::A_BYTES + C_::B_BYTES, kSwizzleBytes);
#pragma unroll
                        for (int ks = 0; ks < kBK / 16; ++ks) {
                            const uint64_t adv = (uint64_t)(ks * 32) >> 4;   // 16 elements = 32 bytes along K
                            const uint32_t acc = (kb != kb0 || ks != 0) ? 1u : 0u;
                            if (FP16) {
                                // columns [main, main+BN) += hi*hi, [main+BN, main+2BN) = cross += hi*lo; then lo*hi
                                mma_f16_ss(d_main, a_hi + adv, b_hi + adv, C_::IDESC2, acc);
                                mma_f16_ss(d_cross, a_lo + adv, b_hi + adv, C_::IDESC, 1u);
                            } else {
                                mma_f16_ss(d_cross, a_lo + adv, b_hi + adv, C_::IDESC, acc);
                                mma_f16_ss(d_cross, a_hi + adv, b_lo + adv, C_::IDESC, 1u);
                                mma_f16_ss(d_main, a_hi + adv, b_hi + adv, C_::IDESC, 1u);
                            }
                        }
                        mma_commit(&ctl->empty[s]);
                    }
                    if (!ok) break;
                    mma_commit(&ctl->tmem_full[b]);
                }
            }
            if (!ok) {
                mma_commit(&ctl->drain);
                drain_wait(&ctl->drain, 0);
            }
        }
    } else {
        // ---------------- promotion + epilogue (warps 2..9) ----------------
        const int sp = warp & 3;                       // TMEM sub-partition this warp may access
        const int half = (warp - 2) >> 2;              // column half of the tile
        const int row_in_tile = sp * 32 + lane;
        const int col0 = half * C_::HALF;
        const uint32_t lane_off = (uint32_t)(sp * 32) << 16;
        long ch = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
            int mb, nb;
            tile_coords(t, p.num_m, p.num_n, mb, nb);
            float sum[C_::HALF];
#pragma unroll
            for (int j = 0; j < C_::HALF; ++j) sum[j] = 0.f;
            for (int c = 0; c < nchunks; ++c, ++ch) {
                const int b = (int)(ch & 1);
                const uint32_t bph = (uint32_t)((ch >> 1) & 1);
                bool ready = mbar_wait(&ctl->tmem_full[b], bph, abort, p.err, kErrTimeoutEpilogue);
                if (!__all_sync(0xffffffffu, ready)) { ok = false; break; }   // tcgen05.ld needs the whole warp
                tc_fence_after();
                const uint32_t tb = tmem_base + lane_off + (uint32_t)(b * C_::ACC_COLS + col0);
#pragma unroll
                for (int q = 0; q < C_::HALF / 16; ++q) {
                    uint32_t r[16];
                    tmem_ld_32x32b_x16(tb + (uint32_t)(q * 16), r);
                    if (FP16) {
                        uint32_t x[16];
                        tmem_ld_32x32b_x16(tb + (uint32_t)(C_::BN + q * 16), x);
                        tmem_ld_wait();
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const float v = __uint_as_float(r[j]) + __uint_as_float(x[j]) * (1.0f / 2048.0f);
                            sum[q * 16 + j] += v;
                        }
                    } else {
                        tmem_ld_wait();
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const float v = __uint_as_float(r[j]);
                            sum[q * 16 + j] += v;
                        }
                    }
                }
                tc_fence_before();
                mbar_arrive(&ctl->tmem_empty[b]);
            }
            if (!ok) break;
            const int m = mb * kBM + row_in_tile;
            if (m < p.M) {
                const int n0 = nb * C_::BN + col0;
                if (FP16) {
                    const int e_row = p.row_exp[m];
#pragma unroll
                    for (int j = 0; j < C_::HALF; ++j) {
                        const int n = n0 + j;
                        if (n < p.N) sum[j] = ldexpf(sum[j], e_row + p.col_exp[n]);
                    }
                }
                if (p.C64) {
                    double* crow = p.C64 + (size_t)m * p.ldc64;
#pragma unroll
                    for (int j = 0; j < C_::HALF; ++j)
                        if (n0 + j < p.N) crow[n0 + j] = (double)sum[j];
                } else {
                    float* crow = p.C + (size_t)m * p.ldc;
                    const bool vec = (n0 + C_::HALF <= p.N) && ((p.ldc & 3) == 0) &&
                                     ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0);
                    if (vec) {
                        float4* c4 = reinterpret_cast<float4*>(crow + n0);
#pragma unroll
                        for (int j = 0; j < C_::HALF / 4; ++j)
                            c4[j] = make_float4(sum[4 * j], sum[4 * j + 1], sum[4 * j + 2], sum[4 * j + 3]);
                    } else {
#pragma unroll
                        for (int j = 0; j < C_::HALF; ++j)
                            if (n0 + j < p.N) crow[n0 + j] = sum[j];
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 512);
    }
}

// ---- host side: tensor maps ------------------------------------------------------------------------------
// Launches still to stall (emugemm_test_stall_next_launches).
std::atomic<int> g_stall_launches{0};

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

bool get_encode() {
    std::call_once(g_encode_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    return g_encode != nullptr;
}

// 16-bit slice of `rows` rows in K panels ([Kp / KP][rows][KP]), K-major; box = kBK (K) x box_rows x 1 panel,
// swizzled by the k-block's row width.
bool make_tmap(CUtensorMap* m, const uint16_t* base, long Kp, long KP, int rows, int box_rows) {
    cuuint64_t dims[3] = {(cuuint64_t)KP, (cuuint64_t)rows, (cuuint64_t)(Kp / KP)};
    cuuint64_t strides[2] = {(cuuint64_t)KP * 2, (cuuint64_t)rows * (cuuint64_t)KP * 2};
    cuuint32_t box[3] = {(cuuint32_t)kBK, (cuuint32_t)box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<uint16_t*>(base), dims, strides, box,
                          estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          kSwizzleBytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <bool FP16>
int launch_impl(const TcGemmArgs& a, void* stream) {
    using C_ = Cfg<FP16>;
    if (!get_encode()) return (int)cudaErrorNotSupported;
    if (a.Mp % kBM || a.Np % C_::BN || a.Kp % kBK || a.Kp <= 0 || a.KP <= 0 || a.KP % kBK || a.Kp % a.KP)
        return (int)cudaErrorInvalidValue;
    CUtensorMap tah, tal, tbh, tbl;
    if (!make_tmap(&tah, a.a_hi, a.Kp, a.KP, a.Mp, kBM) || !make_tmap(&tal, a.a_lo, a.Kp, a.KP, a.Mp, kBM) ||
        !make_tmap(&tbh, a.b_hi, a.Kp, a.KP, a.Np, C_::BN) || !make_tmap(&tbl, a.b_lo, a.Kp, a.KP, a.Np, C_::BN))
        return (int)cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(k_tc_gemm<FP16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C_::SMEM_BYTES);
    if (e != cudaSuccess) return (int)e;
    KParams p;
    p.M = a.M;
    p.N = a.N;
    p.num_m = a.Mp / kBM;
    p.num_n = a.Np / C_::BN;
    p.nk = (int)(a.Kp / kBK);
    p.kpb = (int)(a.KP / kBK);
    p.C = a.C;
    p.ldc = a.ldc;
    p.C64 = a.C64;
    p.ldc64 = a.ldc64;
    p.row_exp = a.row_exp;
    p.col_exp = a.col_exp;
    p.err = a.err;
    p.stall_chunk = take_test_stall() ? 1 : -1;
    const int tiles = p.num_m * p.num_n;
    int grid = a.num_sms > 0 ? a.num_sms : 148;
    if (grid > tiles) grid = tiles;
    k_tc_gemm<FP16><<<grid, kThreads, C_::SMEM_BYTES, (cudaStream_t)stream>>>(tah, tal, tbh, tbl, p);
    count_launch();
    return (int)cudaGetLastError();
}

}  // namespace

bool tc_get_encode(PFN_cuTensorMapEncodeTiled_v12000* out) {
    if (!get_encode()) return false;
    *out = g_encode;
    return true;
}

int tc_gemm_bn(int fp16) { return fp16 ? Cfg<true>::BN : Cfg<false>::BN; }

int launch_tc_gemm(const TcGemmArgs& a, void* stream) {
    return a.fp16 ? launch_impl<true>(a, stream) : launch_impl<false>(a, stream);
}

}  // namespace emu

namespace emu {
bool take_test_stall() {
    for (int n = g_stall_launches.load(); n > 0;)
        if (g_stall_launches.compare_exchange_weak(n, n - 1)) return true;
    return false;
}
}  // namespace emu

extern "C" void emugemm_test_stall_next_launches(int n) { emu::g_stall_launches.store(n < 0 ? 0 : n); }
