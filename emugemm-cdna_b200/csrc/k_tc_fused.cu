// k_tc_fused.cu - bf16x3 and fp16x3 emulated SGEMM with the hi/lo split fused into the GEMM (CTA pairs,
// cta_group::2).
//
// fp16x3 (FP16 = true): the converters split x * 2^-e (e: the row exponent of A's row, the column exponent of B's
// column, both from the exponent scans of k_split.cu) with the fp16 rule hi = RNE_f16(x'), lo = RNE_f16((x' - hi) *
// 2048), exactly as k_split.cu does; the MMAs of a 64-K chunk (two k-blocks, both stages held) run in the order of
// the fp16 pair kernel (k_tc_gemm2.cu): the cross products lo*hi and hi*lo of all four k16 steps, then the first
// hi*hi scaling the accumulator by 2^-11 on the way in, then the other hi*hi; the store undoes 2^(e_row + e_col).
// So its C is bit-identical to the pre-split fp16 pair kernel's, and the slices never exist in HBM.
//
// The pre-split path (k_split.cu + k_tc_gemm*.cu) writes the bf16 slices of A and B to HBM and reads them back.
// Here TMA loads the caller's FP32 tiles straight into a shared-memory staging ring, converter warps split them
// (hi = RNE_bf16(x), lo = RNE_bf16(x - hi): the rule of emugemm-cdna src/emugemm.cpp:143-145) into the UMMA
// K-major layout with the 64-byte swizzle (B is transposed on the way), and the pair's leader issues the three
// tcgen05 MMAs per k-step from those slices. The slices never exist in HBM.
//
// Per CTA (one of a pair sharing a 256 x 256 tile): 128 rows of A and 128 columns of B, k-blocks of 32.
//   fp32 ring  kF32Stages x (A 128x32 + B 32x128 FP32)        TMA -> converters
//   bf16 ring  kBfStages  x (A hi,lo 128x32 + B^T hi,lo 128x32) converters -> pair MMA
// Warps (EMUGEMM_FUSED_WARPS = 16, the default): warpgroup 0 = TMA producer, MMA issuer (leader) / TMEM
// allocator and two converter warps; warpgroups 1-2 = promotion + epilogue (as in k_tc_gemm2.cu); warpgroup 3 =
// four converter warps. The register file is rebalanced per warpgroup with setmaxnreg, executed by every warp of
// a warpgroup at the top of its branch: launch 512 threads x 128 = 65536 registers; epilogue warpgroups grow to
// 176, the others shrink to 80 (2*128*176 + 2*128*80 = 65536). EMUGEMM_FUSED_WARPS = 12: warps 2..9 epilogue,
// 10-11 converters, 168 registers each, no rebalancing.
// Signalling: fp32 ring local to each CTA; bf16 stages of both CTAs are announced on the leader's bf_full after a
// generic->async proxy fence: the leader's converter warps arrive locally (one arming 16 bytes per peer converter
// warp), the peer's each send a 16-byte cp.async.bulk that completes those bytes on the leader's barrier (a
// thread-issued remote arrive with release at cluster scope stalls its warp for ~1200 cycles). The leader's commits
// free the bf16 stages and publish TMEM chunks in both CTAs. All waits are bounded.
// K splits (few output tiles, long K): a work unit is a tile and a range of whole 128-K chunks, as in
// k_tc_gemm2.cu, with the same boundaries; each split writes an FP64 partial plane that the caller sums in order, so
// the two kernels stay bit-identical. Reading each FP32 operand element once, this kernel then needs no split pass.
#include "device_utils.cuh"
#include "emugemm_internal.h"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace emu {

bool tc_get_encode(PFN_cuTensorMapEncodeTiled_v12000* out);

namespace {

using namespace dev;

#ifndef EMUGEMM_FUSED_WARPS
#define EMUGEMM_FUSED_WARPS 16
#endif
constexpr int kWarps = EMUGEMM_FUSED_WARPS;
constexpr int kThreads = 32 * kWarps;
constexpr bool kRegSplit = (kWarps == 16);
constexpr int kEpiFirst = kRegSplit ? 4 : 2;        // first epilogue warp
constexpr int kEpiWarps = 8;
constexpr int kConvWarps = kWarps - 2 - kEpiWarps;  // 6 or 2
constexpr int kConvThreads = 32 * kConvWarps;
constexpr int kRegEpi = 176, kRegOther = 80;        // setmaxnreg targets (16 warps)
static_assert(!kRegSplit || 2 * 128 * kRegEpi + 2 * 128 * kRegOther == kThreads * 128, "register split");
constexpr int kBM = 128;                            // rows per CTA
constexpr int kBN = 256;                            // pair tile width
constexpr int kBNH = 128;                           // columns of B per CTA
constexpr int kBK = 32;                             // k-block (64-byte rows of bf16)
constexpr int kChunkKB = 128 / kBK;                 // promotion every 128 values of K
constexpr int kGroupM = 8;
constexpr int kF32Stages = 3;
// bf16 stages: 3 for bf16x3; 4 for fp16x3, whose MMA issuer holds the two stages of a 64-K chunk at once (with 3 the
// converters could run only one stage ahead of it)
constexpr int kBfStagesMax = 4;
template <bool FP16>
constexpr int bf_stages() { return FP16 ? 4 : 3; }
constexpr int kF32A = kBM * kBK * 4;                // 16 KB
constexpr int kF32B = kBK * kBNH * 4;               // 16 KB
constexpr int kF32Stage = kF32A + kF32B;
constexpr int kBfA = kBM * kBK * 2;                 // 8 KB per slice
constexpr int kBfB = kBNH * kBK * 2;
constexpr int kBfStage = 2 * kBfA + 2 * kBfB;       // 32 KB
static_assert(kBfA == kBfB, "each lo slice sits kBfA bytes after its hi slice");
constexpr int kAccCols = kBN;
constexpr int kHalf = kBN / 2;
template <bool FP16>
constexpr int smem_bytes() { return kF32Stages * kF32Stage + bf_stages<FP16>() * kBfStage + 1024 + 512; }
static_assert(smem_bytes<true>() <= 232448, "shared memory per CTA");
// k-blocks per accumulator: bf16x3 promotes every 128 values of K, fp16x3 every 64 (as the pair kernels do)
template <bool FP16>
constexpr int chunk_kb() { return FP16 ? 64 / kBK : kChunkKB; }

struct CtlF {
    uint64_t f32_full[kF32Stages];
    uint64_t f32_empty[kF32Stages];
    uint64_t bf_full[kBfStagesMax];  // leader: its converter warps arrive; the peer's deliver 16 bytes each
    uint64_t bf_empty[kBfStagesMax]; // both: leader's commit
    uint64_t tmem_full[2];
    uint64_t tmem_empty[2];
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
    alignas(16) uint32_t sig_src[4];              // source of the peer's 16-byte signals (contents unused)
    alignas(16) uint32_t sig_dst[kConvWarps][4];  // leader: landing slots, one per peer converter warp
};

struct KParamsF {
    int M, N, num_m2, num_n, nk;
    int splits, kps;   // K splits and k-blocks (of 32) per split; split boundaries fall on 128-K chunks
    float* C; long ldc;
    double* C64; long ldc64;
    double* part;      // splits > 1: FP64 partial planes [splits][M][N]
    unsigned* err;
    const int* row_exp; const int* col_exp;   // fp16x3: scale exponents of A's rows and B's columns
};

// Work unit u (tile x K split): the tile, the split and its k-block range [kb0, kb1).
__device__ __forceinline__ void unit_of_f(const KParamsF& p, int num_tiles, int u, int& tile, int& sp, int& kb0,
                                          int& kb1) {
    tile = u % num_tiles;
    sp = u / num_tiles;
    kb0 = sp * p.kps;
    kb1 = min(p.nk, kb0 + p.kps);
}

__device__ __forceinline__ void tile_coords_f(int t, int num_m2, int num_n, int& mb2, int& nb) {
    const int per_group = kGroupM * num_n;
    const int g = t / per_group;
    const int first_m = g * kGroupM;
    const int gm = min(num_m2 - first_m, kGroupM);
    const int r = t - g * per_group;
    mb2 = first_m + r % gm;
    nb = r / gm;
}

__device__ __forceinline__ void drain_wait_f(uint64_t* bar, uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    unsigned long long t0 = globaltimer();
    while (!mbar_try_wait(a, parity)) {
        if (globaltimer() - t0 > 200000000ull) return;
    }
}

__device__ __forceinline__ void abort_pair_f(CtlF* ctl, uint32_t peer) {
    ctl->abort = 1;
    st_shared_cluster_u32(mapa_shared(smem_u32(&ctl->abort), peer), 1u);
}

template <int N>
__device__ __forceinline__ void setmaxnreg_inc() {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void setmaxnreg_dec() {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// hi/lo bf16 slices of 8 consecutive values, packed 2 per 32-bit word (lower k in the low half).
__device__ __forceinline__ void split8(const float (&x)[8], uint4& hi, uint4& lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const __nv_bfloat162 hb = __floats2bfloat162_rn(x[2 * j], x[2 * j + 1]);
        const uint32_t hw = *reinterpret_cast<const uint32_t*>(&hb);
        const float h0 = __uint_as_float(hw << 16), h1 = __uint_as_float(hw & 0xffff0000u);
        const __nv_bfloat162 lb = __floats2bfloat162_rn(x[2 * j] - h0, x[2 * j + 1] - h1);
        h[j] = hw;
        l[j] = *reinterpret_cast<const uint32_t*>(&lb);
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// The same, fp16 slices of x' = x * 2^-e: hi = RNE_f16(x'), lo = RNE_f16((x' - hi) * 2048), the rule of the split
// pass. x * 2^-e is one multiply by the normal float 2^-e, which equals ldexpf(x, -e) (both one correctly rounded
// result); only an item whose 2^-e is not a normal float (a row or column of values below about 2^-112) takes ldexpf.
__device__ __forceinline__ void split8_f16_scaled(const float (&xs)[8], uint4& hi, uint4& lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const __half2 hh = __floats2half2_rn(xs[2 * j], xs[2 * j + 1]);   // low half: the lower k
        const float2 hf = __half22float2(hh);
        const __half2 ll = __floats2half2_rn((xs[2 * j] - hf.x) * 2048.0f, (xs[2 * j + 1] - hf.y) * 2048.0f);
        h[j] = *reinterpret_cast<const uint32_t*>(&hh);
        l[j] = *reinterpret_cast<const uint32_t*>(&ll);
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}
__device__ __forceinline__ void split8_f16(float (&x)[8], int e, uint4& hi, uint4& lo) {
    if (e >= -127 && e <= 126) {
        const float sc = __int_as_float((127 - e) << 23);
#pragma unroll
        for (int j = 0; j < 8; ++j) x[j] *= sc;
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) x[j] = ldexpf(x[j], -e);
    }
    split8_f16_scaled(x, hi, lo);
}

// x * 2^e rounded once to float, for the fp16x3 store of a row whose 2^e is not a normal float (as in k_tc_gemm2.cu)
__device__ __forceinline__ float scale_pow2_exact(float x, int e) {
    e = min(max(e, -1022), 1023);
    return __double2float_rn((double)x * __longlong_as_double((long long)(e + 1023) << 52));
}

// byte offset of 16-byte chunk `c` of row `r` in a K-major tile with 64-byte rows and the 64-byte swizzle
__device__ __forceinline__ uint32_t sw64(int r, int c) { return (uint32_t)(r * 64 + ((c ^ ((r >> 1) & 3)) << 4)); }

template <bool FP16>
__global__ void __launch_bounds__(kThreads, 1)
    k_tc_fused(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b, KParamsF p) {
    constexpr int kChunk = chunk_kb<FP16>();
    constexpr int kBfStages = bf_stages<FP16>();
    constexpr uint32_t kIdesc = idesc_f16(2 * kBM, kBN, !FP16);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* f32 = smem;
    uint8_t* bf = smem + kF32Stages * kF32Stage;
    CtlF* ctl = reinterpret_cast<CtlF*>(bf + kBfStages * kBfStage);
    volatile int* abort = &ctl->abort;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const uint32_t peer = rank ^ 1u;
    const bool leader = rank == 0;
    const int pair = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;
    const int num_tiles = p.num_m2 * p.num_n;
    const int num_units = num_tiles * p.splits;
    const bool is_epi = warp >= kEpiFirst && warp < kEpiFirst + kEpiWarps;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kF32Stages; ++s) {
            mbar_init(&ctl->f32_full[s], 1);
            mbar_init(&ctl->f32_empty[s], kConvWarps);
        }
        for (int s = 0; s < kBfStages; ++s) {
            mbar_init(&ctl->bf_full[s], kConvWarps);
            mbar_init(&ctl->bf_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&ctl->tmem_full[b], 1);
            mbar_init(&ctl->tmem_empty[b], 2 * kEpiWarps);
        }
        mbar_init(&ctl->drain, 1);
        ctl->abort = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tm_a);
        prefetch_tmap(&tm_b);
    }
    if (warp == 1) {
        tmem_alloc_pair(&ctl->tmem_base, 512);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem_base = ctl->tmem_base;

    if (!is_epi) {
        if (kRegSplit) setmaxnreg_dec<kRegOther>();
        if (warp == 0) {
            if (lane == 0) {
                // ---------------- TMA producer: FP32 tiles of this CTA's A rows and B columns ----------------
                long it = 0;
                bool ok = true;
                for (int u = pair; u < num_units && ok; u += num_pairs) {
                    int t, sp, kbb, kbe, mb2, nb;
                    unit_of_f(p, num_tiles, u, t, sp, kbb, kbe);
                    tile_coords_f(t, p.num_m2, p.num_n, mb2, nb);
                    const int a_row = mb2 * 2 * kBM + (int)rank * kBM;
                    const int b_col = nb * kBN + (int)rank * kBNH;
                    for (int kb = kbb; kb < kbe; ++kb, ++it) {
                        const int s = (int)(it % kF32Stages);
                        const uint32_t ph = (uint32_t)((it / kF32Stages) & 1);
                        if (!mbar_wait(&ctl->f32_empty[s], ph ^ 1u, abort, p.err, kErrTimeoutProducer)) { ok = false; break; }
                        uint8_t* st = f32 + s * kF32Stage;
                        mbar_arrive_expect_tx(&ctl->f32_full[s], kF32Stage);
                        tma_load_2d(st, &tm_a, &ctl->f32_full[s], kb * kBK, a_row);
                        tma_load_2d(st + kF32A, &tm_b, &ctl->f32_full[s], b_col, kb * kBK);
                    }
                }
                if (!ok) {
                    abort_pair_f(ctl, peer);
                    const long first = it > kF32Stages ? it - kF32Stages : 0;
                    for (long j = first; j < it; ++j)
                        drain_wait_f(&ctl->f32_full[j % kF32Stages], (uint32_t)((j / kF32Stages) & 1));
                }
            }
        } else if (warp == 1) {
            if (lane == 0 && leader) {
                // ---------------- leader: pair MMA issuer ----------------
                long it = 0, ch = 0;
                bool ok = true;
                for (int u = pair; u < num_units && ok; u += num_pairs) {
                    int t, sp, kbb, kbe;
                    unit_of_f(p, num_tiles, u, t, sp, kbb, kbe);
                    for (int kb0 = kbb; kb0 < kbe && ok; kb0 += kChunk, ++ch) {
                        const int b = (int)(ch & 1);
                        const uint32_t bph = (uint32_t)((ch >> 1) & 1);
                        if (!mbar_wait_cluster(&ctl->tmem_empty[b], bph ^ 1u, abort, p.err, kErrTimeoutMma)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t d = tmem_base + (uint32_t)(b * kAccCols);
                        const int kb1 = min(kbe, kb0 + kChunk);
                        if (FP16) {
                            // both k-blocks of the 64-K chunk: cross products of all k16 steps, then hi*hi, the
                            // first of which scales the accumulator by 2^-11 (the fp16 pair kernel's order)
                            uint32_t st[2] = {0u, 0u};
                            int s_of[2] = {0, 0};
                            const int nkb = kb1 - kb0;
                            for (int i = 0; i < nkb; ++i) {
                                const long itk = it + i;
                                s_of[i] = (int)(itk % kBfStages);
                                const uint32_t ph = (uint32_t)((itk / kBfStages) & 1);
                                if (!mbar_wait_cluster(&ctl->bf_full[s_of[i]], ph, abort, p.err, kErrTimeoutMma)) {
                                    ok = false;
                                    break;
                                }
                                st[i] = smem_u32(bf + s_of[i] * kBfStage);
                            }
                            if (!ok) break;
                            tc_fence_after();
#pragma unroll
                            for (int i = 0; i < 2; ++i) {
                                if (i >= nkb) break;
                                const uint64_t a_hi = sdesc_kmajor(st[i], 64), a_lo = sdesc_kmajor(st[i] + kBfA, 64);
                                const uint64_t b_hi = sdesc_kmajor(st[i] + 2 * kBfA, 64);
                                const uint64_t b_lo = sdesc_kmajor(st[i] + 2 * kBfA + kBfB, 64);
#pragma unroll
                                for (int ks = 0; ks < kBK / 16; ++ks) {
                                    const uint64_t adv = (uint64_t)(ks * 32) >> 4;
                                    mma_f16_ss_pair(d, a_lo + adv, b_hi + adv, kIdesc, (i != 0 || ks != 0) ? 1u : 0u);
                                    mma_f16_ss_pair(d, a_hi + adv, b_lo + adv, kIdesc, 1u);
                                }
                            }
#pragma unroll
                            for (int i = 0; i < 2; ++i) {
                                if (i >= nkb) break;
                                const uint64_t a_hi = sdesc_kmajor(st[i], 64);
                                const uint64_t b_hi = sdesc_kmajor(st[i] + 2 * kBfA, 64);
#pragma unroll
                                for (int ks = 0; ks < kBK / 16; ++ks) {
                                    const uint64_t adv = (uint64_t)(ks * 32) >> 4;
                                    if (i == 0 && ks == 0) mma_f16_ss_pair_scale11(d, a_hi, b_hi, kIdesc);
                                    else mma_f16_ss_pair(d, a_hi + adv, b_hi + adv, kIdesc, 1u);
                                }
                            }
                            for (int i = 0; i < nkb; ++i) mma_commit_pair_both(&ctl->bf_empty[s_of[i]], (uint16_t)0x3);
                            it += nkb;
                            mma_commit_pair_both(&ctl->tmem_full[b], (uint16_t)0x3);
                            continue;
                        }
                        for (int kb = kb0; kb < kb1; ++kb, ++it) {
                            const int s = (int)(it % kBfStages);
                            const uint32_t ph = (uint32_t)((it / kBfStages) & 1);
                            if (!mbar_wait_cluster(&ctl->bf_full[s], ph, abort, p.err, kErrTimeoutMma)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            const uint32_t st = smem_u32(bf + s * kBfStage);
                            const uint64_t a_hi = sdesc_kmajor(st, 64);
                            const uint64_t a_lo = sdesc_kmajor(st + kBfA, 64);
                            const uint64_t b_hi = sdesc_kmajor(st + 2 * kBfA, 64);
                            const uint64_t b_lo = sdesc_kmajor(st + 2 * kBfA + kBfB, 64);
#pragma unroll
                            for (int ks = 0; ks < kBK / 16; ++ks) {
                                const uint64_t adv = (uint64_t)(ks * 32) >> 4;
                                const uint32_t acc = (kb != kb0 || ks != 0) ? 1u : 0u;
                                mma_f16_ss_pair(d, a_lo + adv, b_hi + adv, kIdesc, acc);
                                mma_f16_ss_pair(d, a_hi + adv, b_lo + adv, kIdesc, 1u);
                                mma_f16_ss_pair(d, a_hi + adv, b_hi + adv, kIdesc, 1u);
                            }
                            mma_commit_pair_both(&ctl->bf_empty[s], (uint16_t)0x3);
                        }
                        if (!ok) break;
                        mma_commit_pair_both(&ctl->tmem_full[b], (uint16_t)0x3);
                    }
                }
                if (!ok) {
                    abort_pair_f(ctl, peer);
                    mma_commit_pair(&ctl->drain);
                    drain_wait_f(&ctl->drain, 0);
                }
            }
        } else {
            // ---------------- converters: FP32 stage -> bf16 hi/lo stage (both operands K-major) ----------------
            const int ct = (warp < kEpiFirst ? warp - 2 : warp - 2 - kEpiWarps) * 32 + lane;   // 0 .. kConvThreads-1
            const uint32_t lead_bf_full0 = mapa_shared(smem_u32(&ctl->bf_full[0]), 0);
            const int cw = ct >> 5;   // converter warp index
            const uint32_t lead_slot = mapa_shared(smem_u32(&ctl->sig_dst[cw][0]), 0);
            const uint32_t sig_src = smem_u32(&ctl->sig_src[0]);
            constexpr int kPer = (1024 + kConvThreads - 1) / kConvThreads;   // items per thread and k-block
            // items loaded before any is stored: 3 for bf16x3; 1 for fp16x3, whose split holds more registers per item
            // (fewer spills: the long-K fp16x3 GEMM 0.212 -> 0.206 ms)
            constexpr int kBatch = FP16 ? 1 : 3;
            long it = 0;
            bool ok = true;
            for (int u = pair; u < num_units && ok; u += num_pairs) {
                int t, sp, kbb, kbe, mb2, nb;
                unit_of_f(p, num_tiles, u, t, sp, kbb, kbe);
                tile_coords_f(t, p.num_m2, p.num_n, mb2, nb);
                const int a_row0 = mb2 * 2 * kBM + (int)rank * kBM;   // this CTA's first row of A
                const int b_col0 = nb * kBN + (int)rank * kBNH;       // and first column of B
                // fp16x3: a thread converts the same items (row or column, k-group) in every k-block of the unit, so
                // their scale exponents are loaded once per unit (a load per item and k-block stalled the converters)
                int exq[kPer];
#pragma unroll
                for (int i = 0; i < kPer; ++i) {
                    const int item = ct + i * kConvThreads;
                    int e = 0;
                    if (FP16 && item < 1024) {
                        if (item < 512) {
                            const int m = a_row0 + (item >> 2);
                            e = m < p.M ? __ldg(p.row_exp + m) : 0;
                        } else {
                            const int n = b_col0 + ((item - 512) & (kBNH - 1));
                            e = n < p.N ? __ldg(p.col_exp + n) : 0;
                        }
                    }
                    exq[i] = e;
                }
                for (int kb = kbb; kb < kbe; ++kb, ++it) {
                    const int s = (int)(it % kF32Stages);
                    const uint32_t ph = (uint32_t)((it / kF32Stages) & 1);
                    const int q = (int)(it % kBfStages);
                    const uint32_t qh = (uint32_t)((it / kBfStages) & 1);
                    bool ready = mbar_wait(&ctl->f32_full[s], ph, abort, p.err, kErrTimeoutConvert) &&
                                 mbar_wait_cluster(&ctl->bf_empty[q], qh ^ 1u, abort, p.err, kErrTimeoutConvert);
                    if (!__all_sync(0xffffffffu, ready)) { ok = false; break; }
                    const uint8_t* fa = f32 + s * kF32Stage;   // A: 128 rows x 32 floats, 128-byte swizzle
                    const float* fb = reinterpret_cast<const float*>(fa + kF32A);   // B: 32 rows x 128 floats
                    uint8_t* ob = bf + q * kBfStage;
                    // 1024 items of 8 values: A rows x 4 k-groups (0..511), then B columns x 4 k-groups
                    // (512..1023). A warp's 32 items are consecutive, so no warp mixes A and B; the 64-byte
                    // swizzle makes both store patterns (4 lanes per A row, one lane per B column) conflict-free.
#pragma unroll
                    for (int i0 = 0; i0 < kPer; i0 += kBatch) {
                        float x[kBatch][8];
                        uint32_t dst[kBatch];   // offset of the hi chunk in the stage; lo is kBfA further
                        int ex[kBatch];         // fp16x3: the item's scale exponent
#pragma unroll
                        for (int i = 0; i < kBatch; ++i) {
                            const int item = ct + (i0 + i) * kConvThreads;
                            if (i0 + i >= kPer || item >= 1024) continue;
                            if (item < 512) {
                                const int r = item >> 2, g = item & 3;
                                const uint8_t* row = fa + r * 128;
                                const float4 u = *reinterpret_cast<const float4*>(row + (((2 * g) ^ (r & 7)) << 4));
                                const float4 v = *reinterpret_cast<const float4*>(row + (((2 * g + 1) ^ (r & 7)) << 4));
                                x[i][0] = u.x; x[i][1] = u.y; x[i][2] = u.z; x[i][3] = u.w;
                                x[i][4] = v.x; x[i][5] = v.y; x[i][6] = v.z; x[i][7] = v.w;
                                dst[i] = sw64(r, g);
                                ex[i] = exq[i0 + i];
                            } else {
                                const int i2 = item - 512;
                                const int r = i2 & (kBNH - 1), g = i2 >> 7;   // column n of this CTA's B, k-group
#pragma unroll
                                for (int j = 0; j < 8; ++j) x[i][j] = fb[(8 * g + j) * kBNH + r];
                                dst[i] = (uint32_t)(2 * kBfA) + sw64(r, g);
                                ex[i] = exq[i0 + i];
                            }
                        }
#pragma unroll
                        for (int i = 0; i < kBatch; ++i) {
                            const int item = ct + (i0 + i) * kConvThreads;
                            if (i0 + i >= kPer || item >= 1024) continue;
                            uint4 hv, lv;
                            if (FP16) split8_f16(x[i], ex[i], hv, lv);
                            else split8(x[i], hv, lv);
                            *reinterpret_cast<uint4*>(ob + dst[i]) = hv;
                            *reinterpret_cast<uint4*>(ob + dst[i] + kBfA) = lv;
                        }
                    }
                    // each thread makes its slice writes visible to the tensor cores' async proxy; the warp
                    // barrier orders all lanes' writes before lane 0's signal to the leader
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        if (leader) {
                            if (cw == 0) mbar_arrive_expect_tx(&ctl->bf_full[q], 16 * kConvWarps);
                            else mbar_arrive(&ctl->bf_full[q]);
                        } else {
                            bulk_signal_cluster(lead_slot, sig_src, 16, lead_bf_full0 + (uint32_t)(q * sizeof(uint64_t)));
                        }
                        mbar_arrive(&ctl->f32_empty[s]);
                    }
                }
            }
            if (!ok && lane == 0) abort_pair_f(ctl, peer);
        }
    } else {
        if (kRegSplit) setmaxnreg_inc<kRegEpi>();
        // ---------------- promotion + epilogue ----------------
        const int sp = warp & 3;
        const int half = (warp - kEpiFirst) >> 2;
        const int row_in_tile = (int)rank * kBM + sp * 32 + lane;
        const int col0 = half * kHalf;
        const uint32_t lane_off = (uint32_t)(sp * 32) << 16;
        const uint32_t lead_te0 = mapa_shared(smem_u32(&ctl->tmem_empty[0]), 0);
        long ch = 0;
        bool ok = true;
        for (int u = pair; u < num_units && ok; u += num_pairs) {
            int t, sp, kbb, kbe, mb2, nb;
            unit_of_f(p, num_tiles, u, t, sp, kbb, kbe);
            tile_coords_f(t, p.num_m2, p.num_n, mb2, nb);
            const int nchunks = (kbe - kbb + kChunk - 1) / kChunk;
            float sum[kHalf];
#pragma unroll
            for (int j = 0; j < kHalf; ++j) sum[j] = 0.f;
            for (int c = 0; c < nchunks; ++c, ++ch) {
                const int b = (int)(ch & 1);
                const uint32_t bph = (uint32_t)((ch >> 1) & 1);
                bool ready = mbar_wait_cluster(&ctl->tmem_full[b], bph, abort, p.err, kErrTimeoutEpilogue);
                if (!__all_sync(0xffffffffu, ready)) { ok = false; break; }
                tc_fence_after();
                const uint32_t tb = tmem_base + lane_off + (uint32_t)(b * kAccCols + col0);
#pragma unroll
                for (int q = 0; q < kHalf / 16; ++q) {
                    uint32_t r[16];
                    tmem_ld_32x32b_x16(tb + (uint32_t)(q * 16), r);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 16; ++j) sum[q * 16 + j] += __uint_as_float(r[j]);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_remote(lead_te0 + (uint32_t)(b * sizeof(uint64_t)));
            }
            if (!ok) break;
            const int m = mb2 * 2 * kBM + row_in_tile;
            if (m < p.M) {
                const int n0 = nb * kBN + col0;
                auto store_row = [&](auto&& val) {
                    if (p.splits > 1) {
                        double* crow = p.part + ((size_t)sp * p.M + m) * p.N;
#pragma unroll
                        for (int j = 0; j < kHalf; ++j)
                            if (n0 + j < p.N) crow[n0 + j] = (double)val(j);
                    } else if (p.C64) {
                        double* crow = p.C64 + (size_t)m * p.ldc64;
#pragma unroll
                        for (int j = 0; j < kHalf; ++j)
                            if (n0 + j < p.N) crow[n0 + j] = (double)val(j);
                    } else {
                        float* crow = p.C + (size_t)m * p.ldc;
                        const bool vec = (n0 + kHalf <= p.N) && ((p.ldc & 3) == 0) &&
                                         ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0);
                        if (vec) {
                            float4* c4 = reinterpret_cast<float4*>(crow + n0);
#pragma unroll
                            for (int j = 0; j < kHalf / 4; ++j)
                                c4[j] = make_float4(val(4 * j), val(4 * j + 1), val(4 * j + 2), val(4 * j + 3));
                        } else {
#pragma unroll
                            for (int j = 0; j < kHalf; ++j)
                                if (n0 + j < p.N) crow[n0 + j] = val(j);
                        }
                    }
                };
                if (!FP16) {
                    store_row([&](int j) { return sum[j]; });
                } else {
                    // undo the split's 2^-(e_row + e_col): one exact multiply while 2^e is a normal float, the exact
                    // double form for a row where it is not (as the fp16 pair kernel stores); columns past N read
                    // exponent 0 and are not stored
                    const int e_row = p.row_exp[m];
                    const int* cexp = p.col_exp + n0;
                    bool normal = true;
                    store_row([&](int j) {
                        const int e = e_row + (n0 + j < p.N ? cexp[j] : 0);
                        const int ec = min(max(e, -126), 127);
                        normal = normal && (e == ec);
                        return sum[j] * __int_as_float((ec + 127) << 23);
                    });
                    if (!normal)
                        store_row([&](int j) { return scale_pow2_exact(sum[j], e_row + (n0 + j < p.N ? cexp[j] : 0)); });
                }
            }
        }
        if (!ok && lane == 0) abort_pair_f(ctl, peer);
    }

    tc_fence_before();
    cluster_sync_all();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, 512);
    }
}

}  // namespace

// A: M x K row-major FP32 (lda), B: K x N row-major FP32 (ldb); needs lda % 4 == ldb % 4 == 0 and 16-byte
// aligned A, B (TMA). Returns cudaErrorNotSupported when those do not hold, so the caller can pre-split instead.
int launch_tc_fused(const float* A, long lda, const float* B, long ldb, int M, int N, long K, float* C, long ldc,
                    double* C64, long ldc64, unsigned* err, int num_sms, void* stream, int splits,
                    double* part64, int fp16, const int* row_exp, const int* col_exp) {
    if (fp16 && (!row_exp || !col_exp)) return (int)cudaErrorInvalidValue;
    if ((lda & 3) || (ldb & 3) || (reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(B) & 15))
        return (int)cudaErrorNotSupported;
    PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
    if (!tc_get_encode(&enc)) return (int)cudaErrorNotSupported;
    CUtensorMap ta, tb;
    {
        cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
        cuuint64_t strides[1] = {(cuuint64_t)lda * 4};
        cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)kBM};
        cuuint32_t estr[2] = {1, 1};
        if (enc(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(A), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return (int)cudaErrorInvalidValue;
    }
    {
        cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)K};
        cuuint64_t strides[1] = {(cuuint64_t)ldb * 4};
        cuuint32_t box[2] = {(cuuint32_t)kBNH, (cuuint32_t)kBK};
        cuuint32_t estr[2] = {1, 1};
        if (enc(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(B), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return (int)cudaErrorInvalidValue;
    }
    auto kern = fp16 ? k_tc_fused<true> : k_tc_fused<false>;
    const int smem = fp16 ? smem_bytes<true>() : smem_bytes<false>();
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return (int)e;
    KParamsF p;
    p.M = M;
    p.N = N;
    p.num_m2 = (M + 2 * kBM - 1) / (2 * kBM);
    p.num_n = (N + kBN - 1) / kBN;
    p.nk = (int)((K + kBK - 1) / kBK);
    p.splits = splits > 1 ? splits : 1;
    p.kps = p.nk;
    if (p.splits > 1) {
        const int nck = (int)((K + 127) / 128);   // 128-K chunks of the true K, as in launch_tc_gemm_pair
        const int kpc = (nck + p.splits - 1) / p.splits;
        p.kps = kpc * kChunkKB;
        if (!part64 || (nck + kpc - 1) / kpc != p.splits) return (int)cudaErrorInvalidValue;
    }
    p.part = part64;
    p.C = C;
    p.ldc = ldc;
    p.C64 = C64;
    p.ldc64 = ldc64;
    p.err = err;
    p.row_exp = row_exp;
    p.col_exp = col_exp;
    const int tiles = p.num_m2 * p.num_n;

    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = (cudaStream_t)stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(2, 1, 1);
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
    if (e != cudaSuccess || clusters <= 0) {
        cudaGetLastError();
        clusters = (num_sms > 0 ? num_sms : 148) / 2;
    }
    if (num_sms > 0 && clusters > num_sms / 2) clusters = num_sms / 2;   // a caller that leaves SMs to other work
    if (clusters > tiles * p.splits) clusters = tiles * p.splits;
    cfg.gridDim = dim3(2 * clusters, 1, 1);
    e = cudaLaunchKernelEx(&cfg, kern, ta, tb, p);
    count_launch();
    if (e != cudaSuccess) return (int)e;
    return (int)cudaGetLastError();
}

}  // namespace emu
