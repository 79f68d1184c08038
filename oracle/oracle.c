/* oracle.c - CPU restatement of the emugemm hot path, used ONLY as test infrastructure: by tests/, by
 * __graft_entry__.smoke() to check the device result, and by bench.py's cpu_baseline / reference leg. Nothing
 * in the library links or calls it.
 *
 * Each function restates the emugemm-cdna algorithm it checks (file:line in that project):
 *   orc_split_bf16 / orc_split_f16   src/emugemm.cpp:143-148   (bf16: RNE as in CUDA/HIP __float2bfloat16)
 *   orc_split_f16_scaled             the same fp16 rule applied to x * 2^-e (scaled fp16x3 of this library)
 *   orc_absmax                       src/emugemm.cpp:155-168
 *   orc_fp32_chunked                 src/emugemm.cpp:317-330: FP32 GEMM per K-chunk, chunk partials summed
 *                                    in FP64 in chunk order, one final rounding to FP32. Each output is a
 *                                    sequential fmaf chain over k, as in the library's SIMT kernel, so the
 *                                    result is bit-identical to it for the same group split.
 *   orc_slice_product                the bf16x3 / fp16x3 three-product sum, evaluated exactly in FP64
 *                                    from the slices (src/emugemm.cpp:331-356 without FP32 rounding)
 *   orc_gemm_f64                     FP64 ground truth (the reference's device DGEMM, bench/emugemm_test.cpp:85-88)
 *   orc_rho_hutchinson               src/emugemm.cpp:171-213 evaluated in FP64 (same Rademacher hash)
 *
 * Build: oracle/Makefile (gcc, OpenMP, -ffp-contract=off so that only explicit fmaf calls fuse).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

static inline uint32_t f2u(float x) { uint32_t u; memcpy(&u, &x, 4); return u; }
static inline float u2f(uint32_t u) { float x; memcpy(&x, &u, 4); return x; }

/* float -> bf16 bits, round to nearest even (NaN kept quiet). */
static inline uint16_t bf16_rne(float x) {
    uint32_t u = f2u(x);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    uint32_t bias = 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)((u + bias) >> 16);
}
static inline float bf16_to_f(uint16_t h) { return u2f((uint32_t)h << 16); }

static inline uint16_t f16_bits(_Float16 h) { uint16_t b; memcpy(&b, &h, 2); return b; }
static inline _Float16 f16_from_bits(uint16_t b) { _Float16 h; memcpy(&h, &b, 2); return h; }

/* src/emugemm.cpp:143-145 */
void orc_split_bf16(const float* x, long n, uint16_t* hi, uint16_t* lo) {
    for (long i = 0; i < n; ++i) {
        uint16_t h = bf16_rne(x[i]);
        hi[i] = h;
        lo[i] = bf16_rne(x[i] - bf16_to_f(h));
    }
}

/* src/emugemm.cpp:146-148 (gcc's float -> _Float16 conversion is round to nearest even). */
void orc_split_f16(const float* x, long n, uint16_t* hi, uint16_t* lo) {
    for (long i = 0; i < n; ++i) {
        _Float16 h = (_Float16)x[i];
        hi[i] = f16_bits(h);
        lo[i] = f16_bits((_Float16)((x[i] - (float)h) * 2048.0f));
    }
}

/* Exponent used by the scaled fp16 split: e with max * 2^-e < 2^15 (0 for zero / non-finite). */
int orc_exponent_for_max(float mx) {
    if (!(mx > 0.f) || isinf(mx)) return 0;
    int q;
    frexpf(mx, &q);
    return q - 15;
}

void orc_row_exponents(const float* A, int M, long K, long lda, int* e) {
    for (int m = 0; m < M; ++m) {
        float mx = 0.f;
        for (long k = 0; k < K; ++k) mx = fmaxf(mx, fabsf(A[(long)m * lda + k]));
        e[m] = orc_exponent_for_max(mx);
    }
}

void orc_col_exponents(const float* B, long K, int N, long ldb, int* e) {
    for (int n = 0; n < N; ++n) {
        float mx = 0.f;
        for (long k = 0; k < K; ++k) mx = fmaxf(mx, fabsf(B[k * ldb + n]));
        e[n] = orc_exponent_for_max(mx);
    }
}

/* fp16 split of x * 2^-e. */
void orc_split_f16_scaled(const float* x, long n, int e, uint16_t* hi, uint16_t* lo) {
    for (long i = 0; i < n; ++i) {
        float v = ldexpf(x[i], -e);
        _Float16 h = (_Float16)v;
        hi[i] = f16_bits(h);
        lo[i] = f16_bits((_Float16)((v - (float)h) * 2048.0f));
    }
}

/* src/emugemm.cpp:155-162 */
float orc_absmax(const float* x, long n) {
    float m = 0.f;
    for (long i = 0; i < n; ++i) m = fmaxf(m, fabsf(x[i]));
    return m;
}

/* FP64 ground truth: C = A * B (row-major, lda/ldb/ldc), blocked, OpenMP over rows. */
void orc_gemm_f64(const double* A, const double* B, double* C, int M, int N, long K, long lda, long ldb, long ldc) {
    const long KB = 256;
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; ++m) {
        double* c = C + (long)m * ldc;
        for (int n = 0; n < N; ++n) c[n] = 0.0;
        for (long k0 = 0; k0 < K; k0 += KB) {
            long k1 = k0 + KB < K ? k0 + KB : K;
            for (long k = k0; k < k1; ++k) {
                const double a = A[(long)m * lda + k];
                const double* b = B + k * ldb;
                for (int n = 0; n < N; ++n) c[n] += a * b[n];
            }
        }
    }
}

/* Same from FP32 inputs (converted on the fly). */
void orc_gemm_f32_in_f64(const float* A, const float* B, double* C, int M, int N, long K, long lda, long ldb,
                         long ldc) {
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; ++m) {
        double* c = C + (long)m * ldc;
        for (int n = 0; n < N; ++n) c[n] = 0.0;
        for (long k = 0; k < K; ++k) {
            const double a = (double)A[(long)m * lda + k];
            const float* b = B + k * ldb;
            for (int n = 0; n < N; ++n) c[n] += a * (double)b[n];
        }
    }
}

/* src/emugemm.cpp:317-330 with the library's summation order: chunk c covers
 * [c*kc, min(K,(c+1)*kc)), kc = ceil(K/chunks); within a chunk each output is one fmaf chain over k
 * ascending starting from +0; chunks are grouped `cpg` per group; a group's FP64 sum adds its chunk
 * partials in order starting from the first partial; group sums are added in group order. */
void orc_fp32_chunked(const float* A, const float* B, float* C, double* C64, int M, int N, long K, long lda,
                      long ldb, long ldc, int chunks, int cpg) {
    if (chunks < 1) chunks = 1;
    long kc = (K + chunks - 1) / chunks;
    if (kc < 1) kc = 1;
    const int ce = (int)((K + kc - 1) / kc);
    if (cpg < 1) cpg = ce;
    const int G = (ce + cpg - 1) / cpg;
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; ++m) {
        for (int n = 0; n < N; ++n) {
            double total = 0.0;
            for (int g = 0; g < G; ++g) {
                double gs = 0.0;
                const int c0 = g * cpg, c1 = (c0 + cpg < ce) ? c0 + cpg : ce;
                for (int c = c0; c < c1; ++c) {
                    const long k0 = (long)c * kc, k1 = (k0 + kc < K) ? k0 + kc : K;
                    float acc = 0.0f;
                    for (long k = k0; k < k1; ++k) acc = fmaf(A[(long)m * lda + k], B[k * ldb + n], acc);
                    gs = (c == c0) ? (double)acc : gs + (double)acc;
                }
                total = (g == 0) ? gs : total + gs;
            }
            if (C64) C64[(long)m * ldc + n] = total;
            if (C) C[(long)m * ldc + n] = (float)total;
        }
    }
}

/* Exact FP64 value of the three slice products from FP32 inputs.
 * kind 0: bf16x3  R = Ah*Bh + Al*Bh + Ah*Bl.
 * kind 1: scaled fp16x3  R = 2^(ea_m + eb_n) * (Ah*Bh + (Al*Bh + Ah*Bl) / 2048) with the slices of the
 *         scaled values (ea/eb from orc_row_exponents / orc_col_exponents).
 * kind 2: unscaled fp16x3 of the reference (ea = eb = 0). */
static void slice_pair(float x, int kind, int e, double* hi, double* lo) {
    uint16_t h, l;
    if (kind == 0) {
        orc_split_bf16(&x, 1, &h, &l);
        *hi = bf16_to_f(h);
        *lo = bf16_to_f(l);
    } else {
        orc_split_f16_scaled(&x, 1, e, &h, &l);
        *hi = (double)f16_from_bits(h);
        *lo = (double)f16_from_bits(l);
    }
}

void orc_slice_product(const float* A, const float* B, double* R, int M, int N, long K, long lda, long ldb,
                       int kind) {
    int* ea = (int*)__builtin_malloc(sizeof(int) * (size_t)(M > 0 ? M : 1));
    int* eb = (int*)__builtin_malloc(sizeof(int) * (size_t)(N > 0 ? N : 1));
    double* bh = (double*)__builtin_malloc(sizeof(double) * (size_t)K * N + 8);
    double* bl = (double*)__builtin_malloc(sizeof(double) * (size_t)K * N + 8);
    if (kind == 1) {
        orc_row_exponents(A, M, K, lda, ea);
        orc_col_exponents(B, K, N, ldb, eb);
    } else {
        for (int m = 0; m < M; ++m) ea[m] = 0;
        for (int n = 0; n < N; ++n) eb[n] = 0;
    }
#pragma omp parallel for schedule(static)
    for (long k = 0; k < K; ++k)
        for (int n = 0; n < N; ++n) slice_pair(B[k * ldb + n], kind, eb[n], &bh[k * N + n], &bl[k * N + n]);
#pragma omp parallel
    {
        double* hh = (double*)__builtin_malloc(sizeof(double) * (size_t)N + 8);
        double* cr = (double*)__builtin_malloc(sizeof(double) * (size_t)N + 8);
#pragma omp for schedule(static)
        for (int m = 0; m < M; ++m) {
            for (int n = 0; n < N; ++n) { hh[n] = 0.0; cr[n] = 0.0; }
            for (long k = 0; k < K; ++k) {
                double ahi, alo;
                slice_pair(A[(long)m * lda + k], kind, ea[m], &ahi, &alo);
                const double* bhk = bh + k * N;
                const double* blk = bl + k * N;
                for (int n = 0; n < N; ++n) {
                    hh[n] += ahi * bhk[n];
                    cr[n] += alo * bhk[n] + ahi * blk[n];
                }
            }
            for (int n = 0; n < N; ++n) {
                double v = (kind == 0) ? hh[n] + cr[n] : hh[n] + cr[n] / 2048.0;
                R[(long)m * N + n] = (kind == 1) ? ldexp(v, ea[m] + eb[n]) : v;
            }
        }
        __builtin_free(hh);
        __builtin_free(cr);
    }
    __builtin_free(ea);
    __builtin_free(eb);
    __builtin_free(bh);
    __builtin_free(bl);
}

/* Rademacher entry of src/emugemm.cpp:173-176: i = n*P + p, seed 0x5eed. */
static inline double rademacher(uint32_t i) {
    uint32_t h = i ^ 0x5eedu;
    h ^= h >> 16; h *= 0x7feb352du; h ^= h >> 15; h *= 0x846ca68bu; h ^= h >> 16;
    return (h & 1u) ? 1.0 : -1.0;
}

/* src/emugemm.cpp:185-213 in FP64: returns rho_hat, and the two sums of squares in out2
 * (out2[0] = sum (|A|(|B| Omega))^2, out2[1] = sum (A(B Omega))^2). */
double orc_rho_hutchinson(const float* A, const float* B, int M, int N, long K, long lda, long ldb, int P,
                          double* out2) {
    if (P <= 0) P = 64;
    double* T1 = (double*)__builtin_malloc(sizeof(double) * (size_t)K * P);
    double* U1 = (double*)__builtin_malloc(sizeof(double) * (size_t)K * P);
#pragma omp parallel for schedule(static)
    for (long k = 0; k < K; ++k) {
        for (int p = 0; p < P; ++p) { T1[k * P + p] = 0.0; U1[k * P + p] = 0.0; }
        for (int n = 0; n < N; ++n) {
            const double b = B[k * ldb + n];
            for (int p = 0; p < P; ++p) {
                const double w = rademacher((uint32_t)((size_t)n * P + p));
                T1[k * P + p] += b * w;
                U1[k * P + p] += fabs(b) * w;
            }
        }
    }
    double sq = 0.0, sqa = 0.0;
#pragma omp parallel for schedule(static) reduction(+ : sq, sqa)
    for (int m = 0; m < M; ++m) {
        for (int p = 0; p < P; ++p) {
            double t = 0.0, u = 0.0;
            for (long k = 0; k < K; ++k) {
                const double a = A[(long)m * lda + k];
                t += a * T1[k * P + p];
                u += fabs(a) * U1[k * P + p];
            }
            sq += t * t;
            sqa += u * u;
        }
    }
    __builtin_free(T1);
    __builtin_free(U1);
    if (out2) { out2[0] = sqa; out2[1] = sq; }
    if (!(sq > 0)) return -1.0;
    return sqrt(sqa / P) / sqrt(sq / P);
}

/* True rho = || |A||B| ||_F / ||AB||_F in FP64 (bench/rho_sweep.cpp:194-209). */
double orc_rho_true(const float* A, const float* B, int M, int N, long K, long lda, long ldb) {
    double num = 0.0, den = 0.0;
#pragma omp parallel for schedule(static) reduction(+ : num, den)
    for (int m = 0; m < M; ++m) {
        for (int n = 0; n < N; ++n) {
            double s = 0.0, sa = 0.0;
            for (long k = 0; k < K; ++k) {
                const double a = A[(long)m * lda + k], b = B[k * ldb + n];
                s += a * b;
                sa += fabs(a) * fabs(b);
            }
            num += sa * sa;
            den += s * s;
        }
    }
    return sqrt(num) / sqrt(den);
}

/* Normwise relative error ||C - R||_F / ||R||_F (bench/emugemm_test.cpp:96-99). */
double orc_rel_err(const float* C, const double* R, long n) {
    double num = 0.0, den = 0.0;
    for (long i = 0; i < n; ++i) {
        double d = (double)C[i] - R[i];
        num += d * d;
        den += R[i] * R[i];
    }
    return den > 0 ? sqrt(num / den) : (num > 0 ? INFINITY : 0.0);
}

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Threads of the calling thread's later parallel regions (a launcher such as torchrun sets OMP_NUM_THREADS=1 for
   every rank; the CPU baseline then asks for the cores it is allowed to run on). */
void orc_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
