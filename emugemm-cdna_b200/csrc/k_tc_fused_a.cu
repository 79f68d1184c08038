// k_tc_fused_a.cu - bf16x3 emulated SGEMM on CTA pairs with A split inside the kernel into tensor memory.
//
// A's hi/lo bf16 slices (hi = RNE_bf16(x), lo = RNE_bf16(x - hi): emugemm-cdna src/emugemm.cpp:143-145) never
// exist in HBM: TMA loads the caller's FP32 rows of A into shared memory, four converter warps split them and
// write the slices straight into TMEM with tcgen05.st, and the pair MMA reads A from TMEM. B's slices are split
// once per call by k_split_cols (transposed, K-major, in K panels) and loaded by TMA, because every row block of
// the output reads the same B; the split of A, which each column block would otherwise redo, is the one fused.
// Writing slices for the tensor cores from registers into shared memory needs a generic->async proxy fence per
// stage, which measured about as long as converting the stage (k_tc_fused.cu); tcgen05.st into TMEM needs only
// tcgen05.wait::st and a thread sync.
//
// Per CTA (one of a pair sharing a 256 x 224 tile): 128 rows of A, 112 rows of B^T, k-blocks of 32.
//   shared ring  kStages x (A FP32 128x32, 128-byte swizzle | B^T hi, lo 112x32 bf16, 64-byte swizzle)
//   TMEM (512 columns): two 224-column accumulators, two A stages of 32 columns (hi k0-15, hi k16-31, lo, lo).
//   A converter warp loads and splits its rows of the next k-block before it waits for a free A stage, so only the
//   TMEM stores and the hand-off stand between the MMAs of stage n and the refill of stage n + 2. (Stages of one
//   k16 step measured slower: the fixed cost of a hand-off, ~330 cycles, then paid twice per k-block.)
// The three products of a k16 step (lo*hi, hi*lo, hi*hi), the 128-long promotion chunks and the epilogue are
// those of k_tc_gemm2.cu, so C is bit-identical to the pre-split kernels'.
// A stage is handed to the leader's MMA warp by local arrives from the leader's converters and by 16-byte bulk
// copies (completing transaction bytes on the leader's barrier) from the peer's: a thread-issued remote arrive
// with release at cluster scope stalls its warp for ~1200 cycles, twice the MMA time of a k-block.
// Warps: warpgroup 0 = TMA producer, MMA issuer (leader) / TMEM allocator, converters for lane quadrants 2, 3;
// warpgroup 1 = converters for quadrants 0, 1 (warps 6, 7 idle); warpgroups 2-3 = promotion + epilogue. Registers
// per warpgroup with setmaxnreg: 80 / 80 / 176 / 176 (launch 512 x 128 = 65536). All waits are bounded.
#include "device_utils.cuh"
#include "emugemm_internal.h"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace emu {

bool tc_get_encode(PFN_cuTensorMapEncodeTiled_v12000* out);

namespace {

using namespace dev;

constexpr int kThreads = 512;
constexpr int kBM = 128;                            // rows per CTA
constexpr int kBN = 224;                            // pair tile width
constexpr int kBNH = kBN / 2;                       // B^T rows per CTA
constexpr int kHalf = kBN / 2;                      // columns per epilogue warp
constexpr int kBK = 32;                             // k-block
constexpr int kChunkKB = 128 / kBK;                 // promotion every 128 values of K
constexpr int kGroupM = 8;
constexpr int kStages = 6;
constexpr int kF32A = kBM * kBK * 4;                // 16 KB
constexpr int kBfB = kBNH * kBK * 2;                // 7 KB per slice
constexpr int kStage = kF32A + 2 * kBfB;            // 30 KB
constexpr int kSmemBytes = kStages * kStage + 1024 + 512;
constexpr uint32_t kIdesc = idesc_f16(2 * kBM, kBN, true);
constexpr uint32_t kAccCols = kBN;                  // accumulator b at columns [b*224, b*224+224)
constexpr uint32_t kACol0 = 2 * kBN;                // A stage sa at columns [448 + 32*sa, +32): hi 16, lo 16
constexpr int kAStages = 2;
constexpr int kRegEpi = 176, kRegOther = 80;
static_assert(2 * kBN + kAStages * 32 <= 512, "TMEM columns");
static_assert(2 * 128 * kRegEpi + 2 * 128 * kRegOther == kThreads * 128, "register split");
static_assert(kStage % 1024 == 0 && kF32A % 512 == 0 && kBfB % 512 == 0, "swizzle atom alignment");

struct CtlA {
    uint64_t full[kStages];      // each CTA: its own TMA loads of the stage
    uint64_t empty[kStages];     // both: leader's commit (the pair MMAs of the stage are done)
    uint64_t a_ready[kAStages];  // leader: its 4 converter warps arrive, one arming 64 bytes that the peer's 4
                                 // converter warps deliver by 16-byte bulk copies
    uint64_t a_empty[kAStages];  // both: leader's commit
    uint64_t tmem_full[2];
    uint64_t tmem_empty[2];
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
    alignas(16) uint32_t sig_src[4];       // source of the peer's 16-byte signals (contents unused)
    alignas(16) uint32_t sig_dst[4][4];    // leader: landing slots, one per peer converter warp
};

struct KParamsA {
    int M, N, num_m2, num_n, nk, kpb;
    float* C; long ldc;
    double* C64; long ldc64;
    unsigned* err;
};

__device__ __forceinline__ void tile_coords_a(int t, int num_m2, int num_n, int& mb2, int& nb) {
    const int per_group = kGroupM * num_n;
    const int g = t / per_group;
    const int first_m = g * kGroupM;
    const int gm = min(num_m2 - first_m, kGroupM);
    const int r = t - g * per_group;
    mb2 = first_m + r % gm;
    nb = r / gm;
}

__device__ __forceinline__ void drain_wait_a(uint64_t* bar, uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    unsigned long long t0 = globaltimer();
    while (!mbar_try_wait(a, parity)) {
        if (globaltimer() - t0 > 200000000ull) return;
    }
}

__device__ __forceinline__ void abort_pair_a(CtlA* ctl, uint32_t peer) {
    ctl->abort = 1;
    st_shared_cluster_u32(mapa_shared(smem_u32(&ctl->abort), peer), 1u);
}

template <int N>
__device__ __forceinline__ void setmaxnreg_inc_a() {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void setmaxnreg_dec_a() {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// hi/lo bf16 of 16 consecutive values, two per 32-bit word (lower k in the low half).
__device__ __forceinline__ void split16(const float (&x)[16], uint32_t (&hi)[8], uint32_t (&lo)[8]) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const __nv_bfloat162 hb = __floats2bfloat162_rn(x[2 * j], x[2 * j + 1]);
        const uint32_t hw = *reinterpret_cast<const uint32_t*>(&hb);
        const float h0 = __uint_as_float(hw << 16), h1 = __uint_as_float(hw & 0xffff0000u);
        const __nv_bfloat162 lb = __floats2bfloat162_rn(x[2 * j] - h0, x[2 * j + 1] - h1);
        hi[j] = hw;
        lo[j] = *reinterpret_cast<const uint32_t*>(&lb);
    }
}

__global__ void __launch_bounds__(kThreads, 1)
    k_tc_fused_a(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_bhi,
                 const __grid_constant__ CUtensorMap tm_blo, KParamsA p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    CtlA* ctl = reinterpret_cast<CtlA*>(smem + kStages * kStage);
    volatile int* abort = &ctl->abort;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const uint32_t peer = rank ^ 1u;
    const bool leader = rank == 0;
    const int pair = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;
    const int num_tiles = p.num_m2 * p.num_n;
    const int nchunks = (p.nk + kChunkKB - 1) / kChunkKB;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&ctl->full[s], 1);
            mbar_init(&ctl->empty[s], 1);
        }
        for (int a = 0; a < kAStages; ++a) {
            mbar_init(&ctl->a_ready[a], 4);
            mbar_init(&ctl->a_empty[a], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&ctl->tmem_full[b], 1);
            mbar_init(&ctl->tmem_empty[b], 2 * 8);
        }
        mbar_init(&ctl->drain, 1);
        ctl->abort = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tm_a);
        prefetch_tmap(&tm_bhi);
        prefetch_tmap(&tm_blo);
    }
    if (warp == 1) {
        tmem_alloc_pair(&ctl->tmem_base, 512);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem_base = ctl->tmem_base;

    if (warp < 8) {
        setmaxnreg_dec_a<kRegOther>();
        if (warp == 0) {
            if (lane == 0) {
                // ---------------- TMA producer: this CTA's FP32 rows of A and its rows of B^T's slices -------------
                long it = 0;
                bool ok = true;
                for (int t = pair; t < num_tiles && ok; t += num_pairs) {
                    int mb2, nb;
                    tile_coords_a(t, p.num_m2, p.num_n, mb2, nb);
                    const int a_row = mb2 * 2 * kBM + (int)rank * kBM;
                    const int b_row = nb * kBN + (int)rank * kBNH;
                    for (int kb = 0; kb < p.nk; ++kb, ++it) {
                        const int s = (int)(it % kStages);
                        const uint32_t ph = (uint32_t)((it / kStages) & 1);
                        if (!mbar_wait_cluster(&ctl->empty[s], ph ^ 1u, abort, p.err, kErrTimeoutProducer)) {
                            ok = false;
                            break;
                        }
                        uint8_t* st = smem + s * kStage;
                        mbar_arrive_expect_tx(&ctl->full[s], kStage);
                        const int kz = kb / p.kpb, kx = (kb - kz * p.kpb) * kBK;
                        tma_load_2d(st, &tm_a, &ctl->full[s], kb * kBK, a_row);
                        tma_load_3d(st + kF32A, &tm_bhi, &ctl->full[s], kx, b_row, kz);
                        tma_load_3d(st + kF32A + kBfB, &tm_blo, &ctl->full[s], kx, b_row, kz);
                    }
                }
                if (!ok) {
                    abort_pair_a(ctl, peer);
                    const long first = it > kStages ? it - kStages : 0;
                    for (long j = first; j < it; ++j)
                        drain_wait_a(&ctl->full[j % kStages], (uint32_t)((j / kStages) & 1));
                }
            }
        } else if (warp == 1) {
            if (lane == 0 && leader) {
                // ---------------- leader: pair MMA issuer, A from TMEM, B from shared memory ----------------
                long it = 0, ch = 0;
                bool ok = true;
                for (int t = pair; t < num_tiles && ok; t += num_pairs) {
                    for (int kb0 = 0; kb0 < p.nk && ok; kb0 += kChunkKB, ++ch) {
                        const int b = (int)(ch & 1);
                        const uint32_t bph = (uint32_t)((ch >> 1) & 1);
                        if (!mbar_wait_cluster(&ctl->tmem_empty[b], bph ^ 1u, abort, p.err, kErrTimeoutMma)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t d = tmem_base + (uint32_t)b * kAccCols;
                        const int kb1 = min(p.nk, kb0 + kChunkKB);
                        for (int kb = kb0; kb < kb1; ++kb, ++it) {
                            const int s = (int)(it % kStages);
                            const int sa = (int)(it % kAStages);
                            const uint32_t aph = (uint32_t)((it / kAStages) & 1);
                            if (!mbar_wait_cluster(&ctl->a_ready[sa], aph, abort, p.err, kErrTimeoutMma)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            const uint32_t st = smem_u32(smem + s * kStage);
                            const uint64_t b_hi = sdesc_kmajor(st + kF32A, 64);
                            const uint64_t b_lo = sdesc_kmajor(st + kF32A + kBfB, 64);
                            const uint32_t a_hi = tmem_base + kACol0 + 32u * (uint32_t)sa;
                            const uint32_t a_lo = a_hi + 16u;
#pragma unroll
                            for (int ks = 0; ks < kBK / 16; ++ks) {
                                const uint64_t adv = (uint64_t)(ks * 32) >> 4;
                                const uint32_t acc = (kb != kb0 || ks != 0) ? 1u : 0u;
                                mma_f16_ts_pair(d, a_lo + 8u * ks, b_hi + adv, kIdesc, acc);
                                mma_f16_ts_pair(d, a_hi + 8u * ks, b_lo + adv, kIdesc, 1u);
                                mma_f16_ts_pair(d, a_hi + 8u * ks, b_hi + adv, kIdesc, 1u);
                            }
                            mma_commit_pair_both(&ctl->a_empty[sa], (uint16_t)0x3);
                            mma_commit_pair_both(&ctl->empty[s], (uint16_t)0x3);
                        }
                        if (!ok) break;
                        mma_commit_pair_both(&ctl->tmem_full[b], (uint16_t)0x3);
                    }
                }
                if (!ok) {
                    abort_pair_a(ctl, peer);
                    mma_commit_pair(&ctl->drain);
                    drain_wait_a(&ctl->drain, 0);
                }
            }
        } else if (warp <= 5) {
            // ---------------- converters: FP32 row of A -> hi/lo bf16 columns of this CTA's TMEM ----------------
            // warp w owns TMEM lanes (rows) 32*(w%4) .. +31; lane = row within them.
            const int q = warp & 3;
            const int r = q * 32 + lane;
            const uint32_t lane_off = (uint32_t)(q * 32) << 16;
            const uint32_t lead_ready0 = mapa_shared(smem_u32(&ctl->a_ready[0]), 0);
            const uint32_t lead_slot = mapa_shared(smem_u32(&ctl->sig_dst[q][0]), 0);
            const uint32_t sig_src = smem_u32(&ctl->sig_src[0]);
            long it = 0;
            bool ok = true;
            for (int t = pair; t < num_tiles && ok; t += num_pairs) {
                for (int kb = 0; kb < p.nk && ok; ++kb, ++it) {
                    const int s = (int)(it % kStages);
                    const uint32_t ph = (uint32_t)((it / kStages) & 1);
                    bool ready = mbar_wait(&ctl->full[s], ph, abort, p.err, kErrTimeoutConvert);
                    if (!__all_sync(0xffffffffu, ready)) { ok = false; break; }
                    // row r of the FP32 tile: 128 bytes, 16-byte chunk c stored at chunk c ^ (r & 7)
                    const uint8_t* row = smem + s * kStage + r * 128;
                    // the stage's 32 columns for this row: hi k0-15, hi k16-31, lo k0-15, lo k16-31
                    uint32_t cols[32];
#pragma unroll
                    for (int h = 0; h < 2; ++h) {   // k 0-15, then k 16-31
                        float x[16];
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            const float4 v = *reinterpret_cast<const float4*>(row + (((4 * h + c) ^ (r & 7)) << 4));
                            x[4 * c] = v.x; x[4 * c + 1] = v.y; x[4 * c + 2] = v.z; x[4 * c + 3] = v.w;
                        }
                        uint32_t hi[8], lo[8];
                        split16(x, hi, lo);
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            cols[8 * h + j] = hi[j];
                            cols[16 + 8 * h + j] = lo[j];
                        }
                    }
                    const int sa = (int)(it % kAStages);
                    const uint32_t aph = (uint32_t)((it / kAStages) & 1);
                    ready = mbar_wait_cluster(&ctl->a_empty[sa], aph ^ 1u, abort, p.err, kErrTimeoutConvert);
                    if (!__all_sync(0xffffffffu, ready)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t ta = tmem_base + lane_off + kACol0 + 32u * (uint32_t)sa;
                    tmem_st_32x32b_x32(ta, cols);
                    tmem_st_wait();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        // This warp's rows of the A stage are in TMEM (wait::st returned). The leader's warps arrive
                        // locally, quadrant 0 arming the peer's 4 x 16 bytes; the peer's warps send them.
                        if (leader) {
                            if (q == 0) mbar_arrive_expect_tx(&ctl->a_ready[sa], 4 * 16);
                            else mbar_arrive(&ctl->a_ready[sa]);
                        } else {
                            bulk_signal_cluster(lead_slot, sig_src, 16, lead_ready0 + (uint32_t)(sa * sizeof(uint64_t)));
                        }
                    }
                }
            }
            if (!ok && lane == 0) abort_pair_a(ctl, peer);
        }
        // warps 6, 7: no role
    } else {
        setmaxnreg_inc_a<kRegEpi>();
        // ---------------- promotion + epilogue ----------------
        const int sp = warp & 3;
        const int half = (warp - 8) >> 2;
        const int row_in_tile = (int)rank * kBM + sp * 32 + lane;
        const int col0 = half * kHalf;
        const uint32_t lane_off = (uint32_t)(sp * 32) << 16;
        const uint32_t lead_te0 = mapa_shared(smem_u32(&ctl->tmem_empty[0]), 0);
        long ch = 0;
        bool ok = true;
        for (int t = pair; t < num_tiles && ok; t += num_pairs) {
            int mb2, nb;
            tile_coords_a(t, p.num_m2, p.num_n, mb2, nb);
            float sum[kHalf];
#pragma unroll
            for (int j = 0; j < kHalf; ++j) sum[j] = 0.f;
            for (int c = 0; c < nchunks; ++c, ++ch) {
                const int b = (int)(ch & 1);
                const uint32_t bph = (uint32_t)((ch >> 1) & 1);
                bool ready = mbar_wait_cluster(&ctl->tmem_full[b], bph, abort, p.err, kErrTimeoutEpilogue);
                if (!__all_sync(0xffffffffu, ready)) { ok = false; break; }
                tc_fence_after();
                const uint32_t tb = tmem_base + lane_off + (uint32_t)b * kAccCols + (uint32_t)col0;
#pragma unroll
                for (int q = 0; q < kHalf / 16; ++q) {
                    uint32_t v[16];
                    tmem_ld_32x32b_x16(tb + (uint32_t)(q * 16), v);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 16; ++j) sum[q * 16 + j] += __uint_as_float(v[j]);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_remote(lead_te0 + (uint32_t)(b * sizeof(uint64_t)));
            }
            if (!ok) break;
            const int m = mb2 * 2 * kBM + row_in_tile;
            if (m < p.M) {
                const int n0 = nb * kBN + col0;
                if (p.C64) {
                    double* crow = p.C64 + (size_t)m * p.ldc64;
#pragma unroll
                    for (int j = 0; j < kHalf; ++j)
                        if (n0 + j < p.N) crow[n0 + j] = (double)sum[j];
                } else {
                    float* crow = p.C + (size_t)m * p.ldc;
                    const bool vec = (n0 + kHalf <= p.N) && ((p.ldc & 3) == 0) &&
                                     ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0);
                    if (vec) {
                        float4* c4 = reinterpret_cast<float4*>(crow + n0);
#pragma unroll
                        for (int j = 0; j < kHalf / 4; ++j)
                            c4[j] = make_float4(sum[4 * j], sum[4 * j + 1], sum[4 * j + 2], sum[4 * j + 3]);
                    } else {
#pragma unroll
                        for (int j = 0; j < kHalf; ++j)
                            if (n0 + j < p.N) crow[n0 + j] = sum[j];
                    }
                }
            }
        }
        if (!ok && lane == 0) abort_pair_a(ctl, peer);
    }

    tc_fence_before();
    cluster_sync_all();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, 512);
    }
}

}  // namespace

int tc_fused_a_bn() { return kBN; }

// A: M x K row-major FP32 (lda % 4 == 0, 16-byte aligned, else cudaErrorNotSupported); b_hi, b_lo: B^T slices of
// Np rows (Np % 224 == 0) in K panels of KP (Kp % KP == 0, KP % 32 == 0), as written by launch_split_cols.
int launch_tc_fused_a(const float* A, long lda, const uint16_t* b_hi, const uint16_t* b_lo, int M, int N, int Np,
                      long K, long Kp, long KP, float* C, long ldc, double* C64, long ldc64, unsigned* err,
                      int num_sms, void* stream) {
    if ((lda & 3) || (reinterpret_cast<uintptr_t>(A) & 15)) return (int)cudaErrorNotSupported;
    if (Np % kBN || Kp % kBK || KP % kBK || Kp % KP || Kp <= 0 || K <= 0) return (int)cudaErrorInvalidValue;
    PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
    if (!tc_get_encode(&enc)) return (int)cudaErrorNotSupported;
    CUtensorMap ta, tbh, tbl;
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
    const uint16_t* bases[2] = {b_hi, b_lo};
    CUtensorMap* maps[2] = {&tbh, &tbl};
    for (int i = 0; i < 2; ++i) {
        cuuint64_t dims[3] = {(cuuint64_t)KP, (cuuint64_t)Np, (cuuint64_t)(Kp / KP)};
        cuuint64_t strides[2] = {(cuuint64_t)KP * 2, (cuuint64_t)Np * (cuuint64_t)KP * 2};
        cuuint32_t box[3] = {(cuuint32_t)kBK, (cuuint32_t)kBNH, 1};
        cuuint32_t estr[3] = {1, 1, 1};
        if (enc(maps[i], CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<uint16_t*>(bases[i]), dims, strides, box,
                estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return (int)cudaErrorInvalidValue;
    }
    cudaError_t e = cudaFuncSetAttribute(k_tc_fused_a, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return (int)e;
    KParamsA p;
    p.M = M;
    p.N = N;
    p.num_m2 = (M + 2 * kBM - 1) / (2 * kBM);
    p.num_n = Np / kBN;
    p.nk = (int)(Kp / kBK);
    p.kpb = (int)(KP / kBK);
    p.C = C;
    p.ldc = ldc;
    p.C64 = C64;
    p.ldc64 = ldc64;
    p.err = err;
    const int tiles = p.num_m2 * p.num_n;

    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = (cudaStream_t)stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(2, 1, 1);
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, k_tc_fused_a, &cfg);
    if (e != cudaSuccess || clusters <= 0) {
        cudaGetLastError();
        clusters = (num_sms > 0 ? num_sms : 148) / 2;
    }
    if (clusters > tiles) clusters = tiles;
    cfg.gridDim = dim3(2 * clusters, 1, 1);
    e = cudaLaunchKernelEx(&cfg, k_tc_fused_a, ta, tbh, tbl, p);
    count_launch();
    if (e != cudaSuccess) return (int)e;
    return (int)cudaGetLastError();
}

}  // namespace emu
