// k_tc_gemm2.cu - the 3-product emulated-FP32 GEMM on CTA pairs (tcgen05 cta_group::2).
//
// Same slices as k_tc_gemm.cu (see there), but two CTAs of a cluster share one 256 x 256 output tile: each CTA
// loads 128 rows of A and 128 rows of the transposed B into its own shared memory, the pair's leader issues
// tcgen05.mma.cta_group::2 (M = 256, N = 256), which reads the other halves from the peer, and each CTA's TMEM
// receives the accumulator of its own 128 rows. Per SM this halves the B operand's shared-memory and L2 traffic
// for the same tensor work.
//
// Promotion: each accumulator holds one chunk of K and is added into FP32 registers with round-to-nearest.
//   bf16x3: chunks of 128; per k16 step lo*hi, hi*lo, hi*hi into one accumulator (bit-identical to k_tc_gemm.cu).
//   fp16x3: chunks of 64 (one stage); the stage's cross products lo*hi and hi*lo (lo carries a factor 2048)
//   accumulate first, then the first hi*hi MMA scales the accumulator by 2^-11 on the way in (scale-input-d), then
//   the remaining hi*hi follow. One accumulator of 256 columns per buffer, as for bf16x3.
//
// K splits (few output tiles, long K; TcGemmArgs::splits > 1): a work unit is a tile and a range of whole 128-K
// chunks of the true K; units are dealt to the SM pairs like tiles, and each writes an FP64 partial plane that the
// caller sums in order.
//
// Cross-CTA signalling:
//   both CTAs' TMA loads of a stage complete on the LEADER's full barrier (TMA .cta_group::2 form, each
//   load writing only its own CTA), which the leader armed with the bytes of both halves;
//   the leader's commits after a stage / a chunk arrive on the empty / tmem_full barriers of BOTH CTAs
//   (tcgen05.commit to the CTA mask 0b11);
//   every epilogue warp of both CTAs arrives on the leader's tmem_empty once it has drained a chunk, with a
//   CTA-scope arrive (its TMEM reads have completed; a cluster-scope release stalled each warp for ~1000 cycles
//   per chunk, which at 64-K chunks made the epilogue the bottleneck).
// Every wait is bounded; a CTA that gives up raises the abort flag of both CTAs, unwinds, and both meet at a
// final cluster barrier before the pair's TMEM is freed.
#include "device_utils.cuh"
#include "emugemm_internal.h"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>

namespace emu {

bool tc_get_encode(PFN_cuTensorMapEncodeTiled_v12000* out);

namespace {

using namespace dev;

constexpr int kBM = 128;             // rows per CTA (the pair covers 256)
constexpr int kBK = 64;
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kGroupM = 8;           // pair tiles: groups of 8 row blocks of 256

template <bool FP16>
struct Cfg2 {
    static constexpr int BN = 256;                   // pair tile width
    static constexpr int BNH = BN / 2;               // rows of transposed B held by each CTA
    static constexpr int A_BYTES = kBM * kBK * 2;
    static constexpr int B_BYTES = BNH * kBK * 2;
    static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
    static constexpr int STAGES = (196608 / STAGE_BYTES) < 6 ? (196608 / STAGE_BYTES) : 6;
    static constexpr int ACC_COLS = BN;
    // k-blocks per accumulator: bf16x3 promotes every 128 values of K; fp16x3 every 64, one stage, because its
    // hi*hi product is added after the stage's cross products have been scaled by 2^-11 in the accumulator
    static constexpr int CHUNK_KB = FP16 ? 1 : 128 / kBK;
    static constexpr int HALF = BN / 2;              // columns per epilogue thread
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 512;
    static constexpr uint32_t IDESC = idesc_f16(2 * kBM, BN, !FP16);
};

struct Ctl2 {
    uint64_t full[8];
    uint64_t empty[8];
    uint64_t tmem_full[2];
    uint64_t tmem_empty[2];    // leader only: 8 local + 8 peer epilogue warps
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
};

struct KParams2 {
    int M, N, num_m2, num_n, nk;   // num_m2: row blocks of 256
    int kpb;                       // k-blocks per K panel of the slices
    int splits, kps;               // K splits and k-blocks per split (splits = 1: whole K per tile)
    float* C; long ldc;
    double* C64; long ldc64;
    double* part;                  // splits > 1: FP64 partial planes [splits][M][N]
    const int* row_exp; const int* col_exp;
    unsigned* err;
};

// Work unit u (tile x K split): the tile, the split and its k-block range [kb0, kb1).
__device__ __forceinline__ void unit_of(const KParams2& p, int num_tiles, int u, int& tile, int& sp, int& kb0,
                                        int& kb1) {
    tile = u % num_tiles;
    sp = u / num_tiles;
    kb0 = sp * p.kps;
    kb1 = min(p.nk, kb0 + p.kps);
}

__device__ __forceinline__ void tile_coords2(int t, int num_m2, int num_n, int& mb2, int& nb) {
    const int per_group = kGroupM * num_n;
    const int g = t / per_group;
    const int first_m = g * kGroupM;
    const int gm = min(num_m2 - first_m, kGroupM);
    const int r = t - g * per_group;
    mb2 = first_m + r % gm;
    nb = r / gm;
}

__device__ __forceinline__ void drain_wait2(uint64_t* bar, uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    unsigned long long t0 = globaltimer();
    while (!mbar_try_wait(a, parity)) {
        if (globaltimer() - t0 > 200000000ull) return;
    }
}

// x * 2^e rounded once to float, as ldexpf rounds it (subnormal and overflowing results included): the product with
// the power of two is exact in double (a 24-bit significand, |e| far inside the double exponent range), so the one
// rounding is the conversion. Used for the rare rows whose 2^e is not a normal float; a per-element branch to an
// ldexpf fallback in the 128-way unrolled store tail had cost about 17 us per tile (fp16x3 at 4096^3: 0.358 ms
// against 0.295 ms without the rescale).
__device__ __forceinline__ float scale_pow2(float x, int e) {
    e = min(max(e, -1022), 1023);   // beyond this every float result is 0 or inf already
    return __double2float_rn((double)x * __longlong_as_double((long long)(e + 1023) << 52));
}

// Raise the abort flag of both CTAs of the pair.
__device__ __forceinline__ void abort_pair(Ctl2* ctl, uint32_t peer) {
    ctl->abort = 1;
    st_shared_cluster_u32(mapa_shared(smem_u32(&ctl->abort), peer), 1u);
}

template <bool FP16>
__global__ void __launch_bounds__(kThreads, 1)
    k_tc_gemm_pair(const __grid_constant__ CUtensorMap tm_ahi, const __grid_constant__ CUtensorMap tm_alo,
                   const __grid_constant__ CUtensorMap tm_bhi, const __grid_constant__ CUtensorMap tm_blo,
                   KParams2 p) {
    using C_ = Cfg2<FP16>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Ctl2* ctl = reinterpret_cast<Ctl2*>(smem + C_::STAGES * C_::STAGE_BYTES);
    volatile int* abort = &ctl->abort;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const uint32_t peer = rank ^ 1u;
    const bool leader = rank == 0;
    const int pair = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;
    const int num_tiles = p.num_m2 * p.num_n;
    const int num_units = num_tiles * p.splits;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C_::STAGES; ++s) {
            mbar_init(&ctl->full[s], 1);
            mbar_init(&ctl->empty[s], 1);
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
        prefetch_tmap(&tm_ahi);
        prefetch_tmap(&tm_alo);
        prefetch_tmap(&tm_bhi);
        prefetch_tmap(&tm_blo);
    }
    if (warp == 1) {
        tmem_alloc_pair(&ctl->tmem_base, 512);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync_all();      // barriers of both CTAs initialised, TMEM of the pair allocated
    tc_fence_after();
    const uint32_t tmem_base = ctl->tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer: each CTA fills its own halves, completing on the leader ----------------
            long it = 0;
            bool ok = true;
            const uint32_t lead_full0 = mapa_shared(smem_u32(&ctl->full[0]), 0);
            for (int u = pair; u < num_units && ok; u += num_pairs) {
                int t, sp, kbb, kbe, mb2, nb;
                unit_of(p, num_tiles, u, t, sp, kbb, kbe);
                tile_coords2(t, p.num_m2, p.num_n, mb2, nb);
                const int a_row = mb2 * 2 * kBM + (int)rank * kBM;
                const int b_row = nb * C_::BN + (int)rank * C_::BNH;
                for (int kb = kbb; kb < kbe; ++kb, ++it) {
                    const int s = (int)(it % C_::STAGES);
                    const uint32_t ph = (uint32_t)((it / C_::STAGES) & 1);
                    // empty[s] of both CTAs is signalled by the leader's commit once the pair MMA read stage s
                    if (!mbar_wait_cluster(&ctl->empty[s], ph ^ 1u, abort, p.err, kErrTimeoutProducer)) {
                        ok = false;
                        break;
                    }
                    if (leader) mbar_arrive_expect_tx(&ctl->full[s], 2 * C_::STAGE_BYTES);
                    const uint32_t fb = lead_full0 + (uint32_t)(s * sizeof(uint64_t));
                    uint8_t* st = smem + s * C_::STAGE_BYTES;
                    const int kz = kb / p.kpb, kx = (kb - kz * p.kpb) * kBK;
                    tma_load_3d_pair(st, &tm_ahi, fb, kx, a_row, kz);
                    tma_load_3d_pair(st + C_::A_BYTES, &tm_alo, fb, kx, a_row, kz);
                    tma_load_3d_pair(st + 2 * C_::A_BYTES, &tm_bhi, fb, kx, b_row, kz);
                    tma_load_3d_pair(st + 2 * C_::A_BYTES + C_::B_BYTES, &tm_blo, fb, kx, b_row, kz);
                }
            }
            if (!ok) {
                abort_pair(ctl, peer);
                // the leader's full barriers count both CTAs' loads: let those in flight land
                if (leader) {
                    const long first = it > C_::STAGES ? it - C_::STAGES : 0;
                    for (long j = first; j < it; ++j)
                        drain_wait2(&ctl->full[j % C_::STAGES], (uint32_t)((j / C_::STAGES) & 1));
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            // ---------------- leader: pair MMA issuer ----------------
            long it = 0, ch = 0;
            bool ok = true;
            for (int u = pair; u < num_units && ok; u += num_pairs) {
                int t, sp, kbb, kbe;
                unit_of(p, num_tiles, u, t, sp, kbb, kbe);
                for (int kb0 = kbb; kb0 < kbe && ok; kb0 += C_::CHUNK_KB, ++ch) {
                    const int b = (int)(ch & 1);
                    const uint32_t bph = (uint32_t)((ch >> 1) & 1);
                    if (!mbar_wait_cluster(&ctl->tmem_empty[b], bph ^ 1u, abort, p.err, kErrTimeoutMma)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d = tmem_base + (uint32_t)(b * C_::ACC_COLS);
                    const int kb1 = min(kbe, kb0 + C_::CHUNK_KB);
                    for (int kb = kb0; kb < kb1; ++kb, ++it) {
                        const int s = (int)(it % C_::STAGES);
                        const uint32_t ph = (uint32_t)((it / C_::STAGES) & 1);
                        if (!mbar_wait_cluster(&ctl->full[s], ph, abort, p.err, kErrTimeoutMma)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t st = smem_u32(smem + s * C_::STAGE_BYTES);
                        const uint64_t a_hi = sdesc_kmajor(st, 128);
                        const uint64_t a_lo = sdesc_kmajor(st + C_::A_BYTES, 128);
                        const uint64_t b_hi = sdesc_kmajor(st + 2 * C_::A_BYTES, 128);
                        const uint64_t b_lo = sdesc_kmajor(st + 2 * C_::A_BYTES + C_::B_BYTES, 128);
                        if (FP16) {
                            // D = sum(lo*hi + hi*lo) over the stage, then D = hi*hi + D * 2^-11 (the cross slices
                            // carry the 2048 of lo), then the remaining hi*hi: one accumulator holds the 64-K chunk
#pragma unroll
                            for (int ks = 0; ks < kBK / 16; ++ks) {
                                const uint64_t adv = (uint64_t)(ks * 32) >> 4;
                                mma_f16_ss_pair(d, a_lo + adv, b_hi + adv, C_::IDESC, ks != 0 ? 1u : 0u);
                                mma_f16_ss_pair(d, a_hi + adv, b_lo + adv, C_::IDESC, 1u);
                            }
                            mma_f16_ss_pair_scale11(d, a_hi, b_hi, C_::IDESC);
#pragma unroll
                            for (int ks = 1; ks < kBK / 16; ++ks) {
                                const uint64_t adv = (uint64_t)(ks * 32) >> 4;
                                mma_f16_ss_pair(d, a_hi + adv, b_hi + adv, C_::IDESC, 1u);
                            }
                        } else {
#pragma unroll
                            for (int ks = 0; ks < kBK / 16; ++ks) {
                                const uint64_t adv = (uint64_t)(ks * 32) >> 4;
                                const uint32_t acc = (kb != kb0 || ks != 0) ? 1u : 0u;
                                mma_f16_ss_pair(d, a_lo + adv, b_hi + adv, C_::IDESC, acc);
                                mma_f16_ss_pair(d, a_hi + adv, b_lo + adv, C_::IDESC, 1u);
                                mma_f16_ss_pair(d, a_hi + adv, b_hi + adv, C_::IDESC, 1u);
                            }
                        }
                        mma_commit_pair_both(&ctl->empty[s], (uint16_t)0x3);
                    }
                    if (!ok) break;
                    mma_commit_pair_both(&ctl->tmem_full[b], (uint16_t)0x3);
                }
            }
            if (!ok) {
                abort_pair(ctl, peer);
                mma_commit_pair(&ctl->drain);
                drain_wait2(&ctl->drain, 0);
            }
        }
    } else {
        // ---------------- promotion + epilogue (warps 2..9 of each CTA) ----------------
        const int sp = warp & 3;
        const int half = (warp - 2) >> 2;
        const int row_in_tile = (int)rank * kBM + sp * 32 + lane;
        const int col0 = half * C_::HALF;
        const uint32_t lane_off = (uint32_t)(sp * 32) << 16;
        const uint32_t lead_te0 = mapa_shared(smem_u32(&ctl->tmem_empty[0]), 0);
        long ch = 0;
        bool ok = true;
        for (int u = pair; u < num_units && ok; u += num_pairs) {
            int t, sp, kbb, kbe, mb2, nb;
            unit_of(p, num_tiles, u, t, sp, kbb, kbe);
            tile_coords2(t, p.num_m2, p.num_n, mb2, nb);
            const int nchunks = (kbe - kbb + C_::CHUNK_KB - 1) / C_::CHUNK_KB;
            float sum[C_::HALF];
#pragma unroll
            for (int j = 0; j < C_::HALF; ++j) sum[j] = 0.f;
            for (int c = 0; c < nchunks; ++c, ++ch) {
                const int b = (int)(ch & 1);
                const uint32_t bph = (uint32_t)((ch >> 1) & 1);
                bool ready = mbar_wait_cluster(&ctl->tmem_full[b], bph, abort, p.err, kErrTimeoutEpilogue);
                if (!__all_sync(0xffffffffu, ready)) { ok = false; break; }
                tc_fence_after();
                const uint32_t tb = tmem_base + lane_off + (uint32_t)(b * C_::ACC_COLS + col0);
#pragma unroll
                for (int q = 0; q < C_::HALF / 16; ++q) {
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
                const int n0 = nb * C_::BN + col0;
                // fp16x3: undo the power-of-two row and column scaling of the split as each value is stored
                const int e_row = FP16 ? p.row_exp[m] : 0;
                const int* ce = p.col_exp + n0;
                auto store_row = [&](auto&& val) {
                    if (p.splits > 1) {
                        double* crow = p.part + ((size_t)sp * p.M + m) * p.N;
#pragma unroll
                        for (int j = 0; j < C_::HALF; ++j)
                            if (n0 + j < p.N) crow[n0 + j] = (double)val(j);
                    } else if (p.C64) {
                        double* crow = p.C64 + (size_t)m * p.ldc64;
#pragma unroll
                        for (int j = 0; j < C_::HALF; ++j)
                            if (n0 + j < p.N) crow[n0 + j] = (double)val(j);
                    } else {
                        float* crow = p.C + (size_t)m * p.ldc;
                        const bool vec = (n0 + C_::HALF <= p.N) && ((p.ldc & 3) == 0) &&
                                         ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0);
                        if (vec) {
                            float4* c4 = reinterpret_cast<float4*>(crow + n0);
#pragma unroll
                            for (int j = 0; j < C_::HALF / 4; ++j)
                                c4[j] = make_float4(val(4 * j), val(4 * j + 1), val(4 * j + 2), val(4 * j + 3));
                        } else {
#pragma unroll
                            for (int j = 0; j < C_::HALF; ++j)
                                if (n0 + j < p.N) crow[n0 + j] = val(j);
                        }
                    }
                };
                if (!FP16) {
                    store_row([&](int j) { return sum[j]; });
                } else {
                    // 2^e as a normal float: one exact multiply, correctly rounded like ldexpf. A row whose scale
                    // leaves that range anywhere (outputs near the ends of the FP32 range) is stored again with the
                    // exact double form; the common path stays short and branch-free.
                    bool normal = true;
                    store_row([&](int j) {
                        const int e = e_row + ce[j];
                        const int ec = min(max(e, -126), 127);
                        normal = normal && (e == ec);
                        return sum[j] * __int_as_float((ec + 127) << 23);
                    });
                    if (!normal) store_row([&](int j) { return scale_pow2(sum[j], e_row + ce[j]); });
                }
            }
        }
        if (!ok && lane == 0) abort_pair(ctl, peer);
    }

    tc_fence_before();
    cluster_sync_all();      // both CTAs finished: no remote arrival or MMA is still in flight
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, 512);
    }
}

// 16-bit slice in K panels ([Kp / KP][rows][KP]); box = kBK (K) x box_rows x 1 panel, 128-byte swizzle.
bool make_tmap2(PFN_cuTensorMapEncodeTiled_v12000 enc, CUtensorMap* m, const uint16_t* base, long Kp, long KP,
                int rows, int box_rows) {
    cuuint64_t dims[3] = {(cuuint64_t)KP, (cuuint64_t)rows, (cuuint64_t)(Kp / KP)};
    cuuint64_t strides[2] = {(cuuint64_t)KP * 2, (cuuint64_t)rows * (cuuint64_t)KP * 2};
    cuuint32_t box[3] = {(cuuint32_t)kBK, (cuuint32_t)box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<uint16_t*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool FP16>
int launch_pair_impl(const TcGemmArgs& a, void* stream) {
    using C_ = Cfg2<FP16>;
    PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
    if (!tc_get_encode(&enc)) return (int)cudaErrorNotSupported;
    if (a.Mp % (2 * kBM) || a.Np % C_::BN || a.Kp % kBK || a.Kp <= 0 || a.KP <= 0 || a.KP % kBK || a.Kp % a.KP)
        return (int)cudaErrorInvalidValue;
    CUtensorMap tah, tal, tbh, tbl;
    if (!make_tmap2(enc, &tah, a.a_hi, a.Kp, a.KP, a.Mp, kBM) || !make_tmap2(enc, &tal, a.a_lo, a.Kp, a.KP, a.Mp, kBM) ||
        !make_tmap2(enc, &tbh, a.b_hi, a.Kp, a.KP, a.Np, C_::BNH) ||
        !make_tmap2(enc, &tbl, a.b_lo, a.Kp, a.KP, a.Np, C_::BNH))
        return (int)cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(k_tc_gemm_pair<FP16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C_::SMEM_BYTES);
    if (e != cudaSuccess) return (int)e;
    KParams2 p;
    p.M = a.M;
    p.N = a.N;
    p.num_m2 = a.Mp / (2 * kBM);
    p.num_n = a.Np / C_::BN;
    p.nk = (int)(a.Kp / kBK);
    p.kpb = (int)(a.KP / kBK);
    p.splits = a.splits > 1 ? a.splits : 1;
    p.kps = p.nk;
    if (p.splits > 1) {
        // split boundaries on 128-K chunks of the true K (two k-blocks), so that every split starts a promotion
        // chunk and the fused kernel, whose k-blocks are 32 deep, splits at the same values of K; k-blocks past
        // the last split are zero padding of the K panels
        const long K = a.K > 0 ? a.K : a.Kp;
        const int nck = (int)((K + 127) / 128);
        const int kpc = (nck + p.splits - 1) / p.splits;
        p.kps = 2 * kpc;
        if (!a.part64 || (nck + kpc - 1) / kpc != p.splits) return (int)cudaErrorInvalidValue;
    }
    p.part = a.part64;
    p.C = a.C;
    p.ldc = a.ldc;
    p.C64 = a.C64;
    p.ldc64 = a.ldc64;
    p.row_exp = a.row_exp;
    p.col_exp = a.col_exp;
    p.err = a.err;
    const int tiles = p.num_m2 * p.num_n;

    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = C_::SMEM_BYTES;
    cfg.stream = (cudaStream_t)stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    cfg.gridDim = dim3(2, 1, 1);
    e = cudaOccupancyMaxActiveClusters(&clusters, k_tc_gemm_pair<FP16>, &cfg);
    if (e != cudaSuccess || clusters <= 0) {
        cudaGetLastError();
        clusters = (a.num_sms > 0 ? a.num_sms : 148) / 2;
    }
    if (a.num_sms > 0 && clusters > a.num_sms / 2) clusters = a.num_sms / 2;   // a caller that leaves SMs to other work
    if (clusters > tiles * p.splits) clusters = tiles * p.splits;
    cfg.gridDim = dim3(2 * clusters, 1, 1);
    e = cudaLaunchKernelEx(&cfg, k_tc_gemm_pair<FP16>, tah, tal, tbh, tbl, p);
    count_launch();
    if (e != cudaSuccess) return (int)e;
    return (int)cudaGetLastError();
}

}  // namespace

int tc_pair_bn(int fp16) { return fp16 ? Cfg2<true>::BN : Cfg2<false>::BN; }

int launch_tc_gemm_pair(const TcGemmArgs& a, void* stream) {
    return a.fp16 ? launch_pair_impl<true>(a, stream) : launch_pair_impl<false>(a, stream);
}

}  // namespace emu
