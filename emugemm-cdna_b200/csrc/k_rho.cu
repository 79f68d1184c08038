// k_rho.cu - Hutchinson estimate of the cancellation ratio rho = || |A||B| ||_F / ||AB||_F
// (emugemm-cdna src/emugemm.cpp:171-213, emugemm_estimate_rho).
//
// With a Rademacher probe matrix Omega (N x P, row-major, Omega[i] = +1 if bit 0 of hash(i ^ 0x5eed) is
// set, else -1, i = n*P + p; the hash of src/emugemm.cpp:173-176):
//     T1 = B*Omega, T2 = A*T1          den = sqrt(sum T2^2 / P)
//     U1 = |B|*Omega, U2 = |A|*U1      num = sqrt(sum U2^2 / P)        rho_hat = num / den
// The reference materialises |A| and |B| and calls four FP32 rocBLAS GEMMs. Here one "skinny" kernel
// reads each operand once and produces the signed and the absolute product together (|x| is applied on
// the fly), Omega is generated in the kernel, and the sums of squares are FP64 warp-shuffle reductions
// with a fixed combine order (deterministic).
#include "emugemm_internal.h"

#include <cuda_runtime.h>

namespace emu {
namespace {

constexpr int kRows = 128, kP = 64, kBJ = 32, kT = 256;
constexpr int kTM = 8, kTN = 4;      // rows x probe columns per thread (16 x 16 threads)
constexpr int kXs = kRows + 4;       // padded row of the transposed X tile (16-byte aligned reads)

__device__ __forceinline__ float rademacher(unsigned i) {
    unsigned h = i ^ 0x5eedu;
    h ^= h >> 16;
    h *= 0x7feb352du;
    h ^= h >> 15;
    h *= 0x846ca68bu;
    h ^= h >> 16;
    return (h & 1u) ? 1.f : -1.f;
}

// Ypart[s] (rows x P) = X[:, Js] * W[Js, :],  Yabs_part[s] = |X[:, Js]| * Wabs[Js, :].
// OMEGA: W = Wabs = Omega (generated; J = N). Otherwise W, Wabs are J x P row-major.
// Each thread owns 8 rows x 4 probe columns of both products (64 FMAs per j for three or four 16-byte shared
// loads). X arrives as float4 along j (8 lanes per row: 128-byte global reads) and is stored transposed into
// rows of kXs = 132 floats, read back as two float4 per thread. The transposed stores conflict 4 ways (bank
// (16*jq + 4*e + rr) mod 32), which is a quarter of the inner loop's shared-memory wavefronts per k-block; with
// the unpadded 64-row tile they conflicted 32 ways and cost more than the inner loop.
template <bool OMEGA>
__global__ void __launch_bounds__(kT, 2) k_skinny(const float* __restrict__ X, long ld, long rows, long J, int P,
                                                  const float* __restrict__ W, const float* __restrict__ Wabs,
                                                  long j_per_split, float* __restrict__ Ypart,
                                                  float* __restrict__ Yabs_part) {
    __shared__ __align__(16) float Xs[kBJ][kXs];
    __shared__ __align__(16) float Ws[kBJ][kP];
    __shared__ __align__(16) float Was[OMEGA ? 1 : kBJ][kP];
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const long r0 = (long)blockIdx.x * kRows;
    const int p0 = blockIdx.y * kP;
    const int s = blockIdx.z;
    const long j_begin = (long)s * j_per_split;
    const long j_end = min(J, j_begin + j_per_split);
    const bool vec = ((ld & 3) == 0) && ((reinterpret_cast<uintptr_t>(X) & 15) == 0);

    float acc[kTM][kTN] = {}, acca[kTM][kTN] = {};
    for (long jb = j_begin; jb < j_end; jb += kBJ) {
        // X tile: 128 rows x 32 j = 1024 float4, 4 per thread; lanes 8q..8q+7 read one row's 128 bytes
#pragma unroll
        for (int i = 0; i < kRows * kBJ / 4 / kT; ++i) {
            const int f = tid + i * kT;
            const int rr = f >> 3, jq = f & 7;
            const long r = r0 + rr, j = jb + 4 * jq;
            float v[4] = {0.f, 0.f, 0.f, 0.f};
            if (r < rows) {
                if (vec && j + 3 < j_end) {
                    const float4 t = __ldg(reinterpret_cast<const float4*>(X + (size_t)r * ld + j));
                    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
                } else {
#pragma unroll
                    for (int e = 0; e < 4; ++e) v[e] = (j + e < j_end) ? __ldg(X + (size_t)r * ld + j + e) : 0.f;
                }
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) Xs[4 * jq + e][rr] = v[e];
        }
        for (int f = tid; f < kBJ * kP; f += kT) {
            const int jj = f / kP, pp = f % kP;
            const long j = jb + jj;
            const int pc = p0 + pp;
            if (OMEGA) {
                Ws[jj][pp] = (j < j_end && pc < P) ? rademacher((unsigned)((size_t)j * P + pc)) : 0.f;
            } else {
                const bool in = j < j_end && pc < P;
                Ws[jj][pp] = in ? __ldg(W + (size_t)j * P + pc) : 0.f;
                Was[jj][pp] = in ? __ldg(Wabs + (size_t)j * P + pc) : 0.f;
            }
        }
        __syncthreads();
#pragma unroll 4
        for (int jj = 0; jj < kBJ; ++jj) {
            const float4 x0 = *reinterpret_cast<const float4*>(&Xs[jj][ty * kTM]);
            const float4 x1 = *reinterpret_cast<const float4*>(&Xs[jj][ty * kTM + 4]);
            const float4 wv = *reinterpret_cast<const float4*>(&Ws[jj][tx * kTN]);
            const float4 av = OMEGA ? wv : *reinterpret_cast<const float4*>(&Was[OMEGA ? 0 : jj][tx * kTN]);
            const float x[kTM] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
            const float w[kTN] = {wv.x, wv.y, wv.z, wv.w};
            const float a[kTN] = {av.x, av.y, av.z, av.w};
#pragma unroll
            for (int i = 0; i < kTM; ++i)
#pragma unroll
                for (int q = 0; q < kTN; ++q) {
                    acc[i][q] = __fmaf_rn(x[i], w[q], acc[i][q]);
                    acca[i][q] = __fmaf_rn(fabsf(x[i]), a[q], acca[i][q]);
                }
        }
        __syncthreads();
    }
    float* Y = Ypart + (size_t)s * rows * P;
    float* Ya = Yabs_part + (size_t)s * rows * P;
#pragma unroll
    for (int i = 0; i < kTM; ++i) {
        const long r = r0 + ty * kTM + i;
        if (r >= rows) continue;
#pragma unroll
        for (int q = 0; q < kTN; ++q) {
            const int pc = p0 + tx * kTN + q;
            if (pc >= P) continue;
            Y[(size_t)r * P + pc] = acc[i][q];
            Ya[(size_t)r * P + pc] = acca[i][q];
        }
    }
}

// The same products with the operands streamed through a kStagesR-deep cp.async ring (the kernel above loads
// each k-block's X tile synchronously, and its global-load latency showed as the main stall). The tiles keep the
// global layouts (X [r][j], W [j][p]); per four j a thread reads its 8 rows of X as float4 along j and, per j, its
// 4 probe columns of W (and Wabs) as a float4. Each output element still sums x[j] * w[j] for j ascending from
// the split's start, so the partials equal the kernel above's. Needs 16-byte aligned rows (ld, P multiples of 4)
// and J and the split length multiples of 16; W = Omega is precomputed (k_omega) for the first pass.
// (A 4-row x 8-column thread tile, which halves the |x| instructions per FMA, measured slower: 0.90 ms against
// 0.83 ms for the probe at 8192^3.)
constexpr int kStagesR = 3;
constexpr int kBJc = 16;

__device__ __forceinline__ void cp_async16_r(void* smem_dst, const void* gsrc, bool valid) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
    const int n = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(gsrc), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit_r() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_r() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__global__ void k_omega(int P, long J, float* __restrict__ Om) {
    const size_t n = (size_t)J * P;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        Om[i] = rademacher((unsigned)i);
}

template <bool SAME_W>   // SAME_W: Wabs == W (the Omega pass): one tile serves both products
__global__ void __launch_bounds__(kT, 2) k_skinny_cp(const float* __restrict__ X, long ld, long rows, long J, int P,
                                                     const float* __restrict__ W, const float* __restrict__ Wabs,
                                                     long j_per_split, float* __restrict__ Ypart,
                                                     float* __restrict__ Yabs_part) {
    __shared__ __align__(16) float Xs[kStagesR][kRows][kBJc];
    __shared__ __align__(16) float Ws[kStagesR][kBJc][kP];
    __shared__ __align__(16) float Was[SAME_W ? 1 : kStagesR][kBJc][kP];
    constexpr int X_CH = kRows * kBJc / 4, W_CH = kBJc * kP / 4;     // 16-byte copies per k-block
    constexpr int CH = X_CH + (SAME_W ? 1 : 2) * W_CH;
    static_assert(CH % kT == 0, "copies per thread");
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const long r0 = (long)blockIdx.x * kRows;
    const int p0 = blockIdx.y * kP;
    const int s = blockIdx.z;
    const long j_begin = (long)s * j_per_split;
    const long j_end = min(J, j_begin + j_per_split);
    const long nkb = j_end > j_begin ? (j_end - j_begin + kBJc - 1) / kBJc : 0;

    auto issue = [&](long kt) {
        const int st = (int)(kt % kStagesR);
        const long j0 = j_begin + kt * kBJc;
#pragma unroll
        for (int c = 0; c < CH / kT; ++c) {
            const int f = tid + c * kT;
            if (f < X_CH) {
                const int rr = f >> 2, q = f & 3;
                const long r = r0 + rr, j = j0 + 4 * q;
                const bool v = r < rows && j < j_end;
                cp_async16_r(&Xs[st][rr][4 * q], v ? (const void*)(X + (size_t)r * ld + j) : (const void*)X, v);
            } else {
                const int f2 = f - X_CH;
                const bool abs_tile = !SAME_W && f2 >= W_CH;
                const int f3 = abs_tile ? f2 - W_CH : f2;
                const int jj = f3 / (kP / 4), q = f3 % (kP / 4);
                const long j = j0 + jj;
                const int pc = p0 + 4 * q;
                const bool v = j < j_end && pc < P;
                const float* src = abs_tile ? Wabs : W;
                float* dst = abs_tile ? &Was[SAME_W ? 0 : st][jj][4 * q] : &Ws[st][jj][4 * q];
                cp_async16_r(dst, v ? (const void*)(src + (size_t)j * P + pc) : (const void*)src, v);
            }
        }
    };

    float acc[kTM][kTN] = {}, acca[kTM][kTN] = {};
    for (int kt = 0; kt < kStagesR - 1; ++kt) {
        if (kt < nkb) issue(kt);
        cp_async_commit_r();
    }
    for (long kt = 0; kt < nkb; ++kt) {
        if (kt + kStagesR - 1 < nkb) issue(kt + kStagesR - 1);
        cp_async_commit_r();
        cp_async_wait_r<kStagesR - 1>();
        __syncthreads();
        const int st = (int)(kt % kStagesR);
#pragma unroll
        for (int j4 = 0; j4 < kBJc / 4; ++j4) {
            float4 a[kTM];
#pragma unroll
            for (int i = 0; i < kTM; ++i) a[i] = *reinterpret_cast<const float4*>(&Xs[st][ty * kTM + i][4 * j4]);
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                const float4 wv = *reinterpret_cast<const float4*>(&Ws[st][4 * j4 + jj][tx * kTN]);
                const float4 av = SAME_W ? wv : *reinterpret_cast<const float4*>(&Was[SAME_W ? 0 : st][4 * j4 + jj][tx * kTN]);
                const float w[kTN] = {wv.x, wv.y, wv.z, wv.w};
                const float wa[kTN] = {av.x, av.y, av.z, av.w};
#pragma unroll
                for (int i = 0; i < kTM; ++i) {
                    const float x = jj == 0 ? a[i].x : jj == 1 ? a[i].y : jj == 2 ? a[i].z : a[i].w;
#pragma unroll
                    for (int q = 0; q < kTN; ++q) {
                        acc[i][q] = __fmaf_rn(x, w[q], acc[i][q]);
                        acca[i][q] = __fmaf_rn(fabsf(x), wa[q], acca[i][q]);
                    }
                }
            }
        }
        __syncthreads();
    }
    cp_async_wait_r<0>();
    float* Y = Ypart + (size_t)s * rows * P;
    float* Ya = Yabs_part + (size_t)s * rows * P;
#pragma unroll
    for (int i = 0; i < kTM; ++i) {
        const long r = r0 + ty * kTM + i;
        if (r >= rows) continue;
#pragma unroll
        for (int q = 0; q < kTN; ++q) {
            const int pc = p0 + tx * kTN + q;
            if (pc >= P) continue;
            Y[(size_t)r * P + pc] = acc[i][q];
            Ya[(size_t)r * P + pc] = acca[i][q];
        }
    }
}

// T = sum_s Ypart[s] (FP32, in order s = 0..S-1), for both the signed and the absolute product.
__global__ void k_combine(const float* __restrict__ Ypart, const float* __restrict__ Yabs_part, int S, size_t n,
                          float* __restrict__ T, float* __restrict__ Tabs) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        float y = Ypart[i], ya = Yabs_part[i];
        for (int s = 1; s < S; ++s) {
            y += Ypart[(size_t)s * n + i];
            ya += Yabs_part[(size_t)s * n + i];
        }
        T[i] = y;
        Tabs[i] = ya;
    }
}

// Same combine, then FP64 sums of squares per block (warp shuffles), written to part[block][2].
__global__ void k_combine_sq(const float* __restrict__ Ypart, const float* __restrict__ Yabs_part, int S, size_t n,
                             double* __restrict__ part) {
    double sq = 0.0, sqa = 0.0;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        float y = Ypart[i], ya = Yabs_part[i];
        for (int s = 1; s < S; ++s) {
            y += Ypart[(size_t)s * n + i];
            ya += Yabs_part[(size_t)s * n + i];
        }
        sq += (double)y * (double)y;
        sqa += (double)ya * (double)ya;
    }
    for (int o = 16; o > 0; o >>= 1) {
        sq += __shfl_xor_sync(0xffffffffu, sq, o);
        sqa += __shfl_xor_sync(0xffffffffu, sqa, o);
    }
    __shared__ double ws[2][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
        ws[0][warp] = sq;
        ws[1][warp] = sqa;
    }
    __syncthreads();
    if (warp == 0) {
        const int nw = blockDim.x >> 5;
        sq = lane < nw ? ws[0][lane] : 0.0;
        sqa = lane < nw ? ws[1][lane] : 0.0;
        for (int o = 16; o > 0; o >>= 1) {
            sq += __shfl_xor_sync(0xffffffffu, sq, o);
            sqa += __shfl_xor_sync(0xffffffffu, sqa, o);
        }
        if (lane == 0) {
            part[2 * blockIdx.x] = sq;
            part[2 * blockIdx.x + 1] = sqa;
        }
    }
}

// out2[0] = sum of |.| squares (numerator), out2[1] = sum of signed squares (denominator).
__global__ void k_final(const double* __restrict__ part, int nblocks, double* __restrict__ out2) {
    if (threadIdx.x == 0) {
        double sq = 0.0, sqa = 0.0;
        for (int b = 0; b < nblocks; ++b) {
            sq += part[2 * b];
            sqa += part[2 * b + 1];
        }
        out2[0] = sqa;
        out2[1] = sq;
    }
}

constexpr int kCombineBlocks = 296;

// Splits of J per (row block, probe block): the fewest whose blocks fill the 2 * sms resident slots to at least
// 90% over whole waves (the kernels are FFMA-bound, so a last wave that is mostly empty costs a full block time;
// 64 row blocks on 148 SMs take 9 splits, 97% of 2 waves, not 5, 54%), at most one per 256 j.
int splits_for(long rows, int P, long J, int sms) {
    const long blocks = ((rows + kRows - 1) / kRows) * ((P + kP - 1) / kP);
    const long slots = 2L * sms;
    long smax = (J + 255) / 256;
    if (smax < 1) smax = 1;
    long best = 1;
    double best_eff = 0.0;
    for (long s = 1; s <= smax; ++s) {
        const long n = blocks * s;
        const double eff = (double)n / (double)(((n + slots - 1) / slots) * slots);
        if (eff >= 0.9) return (int)s;
        if (eff > best_eff + 1e-9) { best_eff = eff; best = s; }
    }
    return (int)best;
}

long j_per(long J, int S) {
    long j = (J + S - 1) / S;
    return ((j + kBJ - 1) / kBJ) * kBJ;
}

struct RhoLayout {
    int S1, S2;
    size_t t1, t1a, y1, y1a, y2, y2a, part, omega, total;
};

RhoLayout layout(int M, int N, long K, int P, int sms) {
    RhoLayout L;
    L.S1 = splits_for(K, P, N, sms);
    L.S2 = splits_for(M, P, K, sms);
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t o = off; off += (bytes + 255) & ~size_t(255); return o; };
    L.t1 = take((size_t)K * P * 4);
    L.t1a = take((size_t)K * P * 4);
    L.y1 = take((size_t)L.S1 * K * P * 4);
    L.y1a = take((size_t)L.S1 * K * P * 4);
    L.y2 = take((size_t)L.S2 * M * P * 4);
    L.y2a = take((size_t)L.S2 * M * P * 4);
    L.part = take((size_t)kCombineBlocks * 2 * 8);
    L.omega = take((size_t)N * P * 4);
    L.total = off;
    return L;
}

}  // namespace

size_t rho_ws_bytes(int M, int N, long K, int P, int sms) { return layout(M, N, K, P, sms).total; }

int launch_rho(const float* A, long lda, const float* B, long ldb, int M, int N, long K, int P, void* ws, int sms,
               double* out2, void* stream) {
    cudaStream_t st = (cudaStream_t)stream;
    RhoLayout L = layout(M, N, K, P, sms);
    char* w = static_cast<char*>(ws);
    float* T1 = (float*)(w + L.t1);
    float* T1a = (float*)(w + L.t1a);
    float* Y1 = (float*)(w + L.y1);
    float* Y1a = (float*)(w + L.y1a);
    float* Y2 = (float*)(w + L.y2);
    float* Y2a = (float*)(w + L.y2a);
    double* part = (double*)(w + L.part);
    float* Om = (float*)(w + L.omega);
    unsigned launches = 0;
    // the cp.async ring needs 16-byte rows and j ranges in whole 16-wide blocks
    auto ring_ok = [&](const float* X, long ld, long J, int S) {
        return (ld & 3) == 0 && (reinterpret_cast<uintptr_t>(X) & 15) == 0 && (P & 3) == 0 && J % kBJc == 0 &&
               j_per(J, S) % kBJc == 0;
    };

    // T1 = B * Omega (rows = K, J = N).
    dim3 g1((unsigned)((K + kRows - 1) / kRows), (unsigned)((P + kP - 1) / kP), (unsigned)L.S1);
    if (ring_ok(B, ldb, N, L.S1)) {
        k_omega<<<148 * 4, 256, 0, st>>>(P, N, Om);
        k_skinny_cp<true><<<g1, kT, 0, st>>>(B, ldb, K, N, P, Om, Om, j_per(N, L.S1), Y1, Y1a);
        launches += 2;
    } else {
        k_skinny<true><<<g1, kT, 0, st>>>(B, ldb, K, N, P, nullptr, nullptr, j_per(N, L.S1), Y1, Y1a);
        launches += 1;
    }
    const size_t n1 = (size_t)K * P;
    k_combine<<<kCombineBlocks, 256, 0, st>>>(Y1, Y1a, L.S1, n1, T1, T1a);
    // T2 = A * T1 (rows = M, J = K); only its sums of squares are kept.
    dim3 g2((unsigned)((M + kRows - 1) / kRows), (unsigned)((P + kP - 1) / kP), (unsigned)L.S2);
    if (ring_ok(A, lda, K, L.S2))
        k_skinny_cp<false><<<g2, kT, 0, st>>>(A, lda, M, K, P, T1, T1a, j_per(K, L.S2), Y2, Y2a);
    else
        k_skinny<false><<<g2, kT, 0, st>>>(A, lda, M, K, P, T1, T1a, j_per(K, L.S2), Y2, Y2a);
    const size_t n2 = (size_t)M * P;
    k_combine_sq<<<kCombineBlocks, 256, 0, st>>>(Y2, Y2a, L.S2, n2, part);
    k_final<<<1, 32, 0, st>>>(part, kCombineBlocks, out2);
    count_launch(launches + 4);
    return (int)cudaGetLastError();
}

}  // namespace emu
