// api.cpp - the emugemm C ABI: handles, workspace and the emugemm_sgemm executor
// (emugemm-cdna src/emugemm.cpp:75-87 workspace, :185-213 rho estimate, :285-358 executor).
//
// Every compute path runs CUDA kernels built for sm_100a; there is no CPU fallback. A handle refuses to
// be created on any device other than compute capability 10.0.
#include "emugemm_internal.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

namespace emu {

std::string live_arch_string();
void tune_clear();
int tc_gemm_bn(int fp16);
size_t rho_ws_bytes(int M, int N, long K, int P, int sms);
int launch_rho(const float* A, long lda, const float* B, long ldb, int M, int N, long K, int P, void* ws, int sms,
               double* out2, void* stream);

static std::atomic<unsigned long long> g_launches{0};
void count_launch(unsigned n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

emugemm_status_t from_cuda(int e) {
    if (e == 0) return EMUGEMM_STATUS_SUCCESS;
    if (e == (int)cudaErrorMemoryAllocation) return EMUGEMM_STATUS_MEMORY_ERROR;
    if (e == (int)cudaErrorInvalidValue) return EMUGEMM_STATUS_INVALID_VALUE;
    return EMUGEMM_STATUS_INTERNAL_ERROR;
}

// Grow-only workspace slot (src/emugemm.cpp:79-87, but per handle and with an optional cap).
void* ws_get(Handle* h, int slot, size_t bytes) {
    if (bytes == 0) bytes = 256;
    if (h->ws_size[slot] >= bytes) return h->ws[slot];
    size_t total = 0;
    for (int i = 0; i < kWsCount; ++i) total += (i == slot) ? 0 : h->ws_size[i];
    if (h->ws_limit && total + bytes > h->ws_limit) return nullptr;
    if (h->ws[slot]) {
        cudaStreamSynchronize((cudaStream_t)h->stream);
        cudaFree(h->ws[slot]);
    }
    h->ws[slot] = nullptr;
    h->ws_size[slot] = 0;
    if (cudaMalloc(&h->ws[slot], bytes) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    h->ws_size[slot] = bytes;
    return h->ws[slot];
}

DeviceGuard::DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) { ok = false; return; }
    if (prev != dev && cudaSetDevice(dev) != cudaSuccess) ok = false;
}
DeviceGuard::~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
}

static emugemm_status_t take_device_error(Handle* h) {
    unsigned e = *reinterpret_cast<volatile unsigned*>(h->err_host);
    if (e) {
        *reinterpret_cast<volatile unsigned*>(h->err_host) = 0;
        std::fprintf(stderr, "emugemm: a device-side wait timed out (flags 0x%x)\n", e);
        return EMUGEMM_STATUS_TIMEOUT;
    }
    return EMUGEMM_STATUS_SUCCESS;
}

emugemm_status_t sync_check(Handle* h) {
    cudaError_t e = cudaStreamSynchronize((cudaStream_t)h->stream);
    emugemm_status_t d = take_device_error(h);
    if (d != EMUGEMM_STATUS_SUCCESS) return d;
    return from_cuda((int)e);
}

// max|x| of a rows x cols matrix, read back to the host (synchronises the stream).
emugemm_status_t absmax(Handle* h, const float* X, long rows, long cols, long ld, float* out) {
    float* d = (float*)ws_get(h, kWsScalar, 64);
    if (!d) return EMUGEMM_STATUS_MEMORY_ERROR;
    int e;
    {
        ProfScope ps(h, kProfScan);
        e = launch_absmax(X, rows, cols, ld, d, h->stream);
    }
    if (e) return from_cuda(e);
    float v = 0.f;
    e = (int)cudaMemcpyAsync(&v, d, sizeof(float), cudaMemcpyDeviceToHost, (cudaStream_t)h->stream);
    if (e) return from_cuda(e);
    emugemm_status_t s = sync_check(h);
    if (s != EMUGEMM_STATUS_SUCCESS) return s;
    *out = v;
    return EMUGEMM_STATUS_SUCCESS;
}

// The two Hutchinson sums of the rho estimate (src/emugemm.cpp:185-213), read back to the host: v[0] = sum over
// probes of ||(|A|(|B| w))||^2, v[1] = sum of ||A(B w)||^2. Returns false on failure.
bool rho_sums(Handle* h, int M, int N, long K, const float* A, long lda, const float* B, long ldb, int P,
              double v[2]) {
    if (M <= 0 || N <= 0 || K <= 0) return false;
    void* ws = ws_get(h, kWsRhoT1, rho_ws_bytes(M, N, K, P, h->num_sms));
    double* out2 = (double*)ws_get(h, kWsRhoPart, 2 * sizeof(double));
    if (!ws || !out2) return false;
    {
        ProfScope ps(h, kProfRho);
        if (launch_rho(A, lda, B, ldb, M, N, K, P, ws, h->num_sms, out2, h->stream)) return false;
    }
    if (cudaMemcpyAsync(v, out2, 2 * sizeof(double), cudaMemcpyDeviceToHost, (cudaStream_t)h->stream) != cudaSuccess)
        return false;
    return sync_check(h) == EMUGEMM_STATUS_SUCCESS;
}

// src/emugemm.cpp:185-213. Returns < 0 on failure.
static double estimate_rho(Handle* h, int M, int N, long K, const float* A, long lda, const float* B, long ldb,
                           int P) {
    if (P <= 0) P = 64;
    double v[2] = {0, 0};
    if (!rho_sums(h, M, N, K, A, lda, B, ldb, P, v)) return -1.0;
    const double num = std::sqrt(v[0] / (double)P), den = std::sqrt(v[1] / (double)P);
    if (num < 0 || !(den > 0)) return -1.0;
    return num / den;
}

ProfScope::ProfScope(Handle* h_, int kind_) : h(h_), kind(kind_) {
    if (!h->profiling) return;
    if (h->prof_n == h->prof_cap) {
        int cap = h->prof_cap ? 2 * h->prof_cap : 64;
        ProfRec* p = new ProfRec[cap];
        for (int i = 0; i < h->prof_n; ++i) p[i] = h->prof[i];
        delete[] h->prof;
        h->prof = p;
        h->prof_cap = cap;
    }
    cudaEvent_t a, b;
    if (cudaEventCreate(&a) != cudaSuccess) return;
    if (cudaEventCreate(&b) != cudaSuccess) { cudaEventDestroy(a); return; }
    rec = &h->prof[h->prof_n++];
    rec->a = a;
    rec->b = b;
    rec->kind = kind;
    cudaEventRecord(a, (cudaStream_t)h->stream);
}

ProfScope::~ProfScope() {
    if (rec) cudaEventRecord((cudaEvent_t)rec->b, (cudaStream_t)h->stream);
}

static void prof_clear(Handle* h) {
    for (int i = 0; i < h->prof_n; ++i) {
        cudaEventDestroy((cudaEvent_t)h->prof[i].a);
        cudaEventDestroy((cudaEvent_t)h->prof[i].b);
    }
    h->prof_n = 0;
}

long round_up(long x, long m) { return (x + m - 1) / m * m; }

// Tensor-core kernel for a shape: 1 = single-CTA, 2 = CTA pair, 3 = CTA pair with the split fused in, 4 = CTA pair
// with A split into TMEM in the kernel (3 and 4: bf16x3). The handle's EMUGEMM_ATTR_TC_KERNEL (default: the
// environment variable EMUGEMM_TC_KERNEL, "single", "pair", "fused" or "fusea", read when the handle was created)
// wins, then the tile table's code, then the built-in choice, fitted to the B200 tile table (tiles_b200.csv):
//   bf16x3: CTA pairs when K > 1024 or their 256 x 256 tiles fill the SM pairs (pairs won every shape with K >= 4096
//   and the K = 1024 shapes with at least 128 tiles; with fewer, single-CTA or fused tiles won by up to 8 %); the
//   fused CTA-pair kernel instead when there are fewer than 16 tiles and K is split over the SM pairs;
//   fp16x3: with tiles that fill the SM pairs, pairs when K > 1024 or at least 512 tiles (else the 128 x 128
//   single-CTA tiles won, by up to 26 %); with fewer tiles, pairs when K >= 16384, long enough for the K splits; and,
//   as for bf16x3, the fused kernel below 16 tiles when K is split (256^2 x 262144: 69 -> 101 TFLOPS).
// EMUGEMM_LOG (set and not "0"): one stderr line per GEMM with the plan (scheme, chunks, predicted error, reason)
// and one per tensor-core launch with the kernel chosen. The reference's observable decision record is plan.reason;
// this makes it and the kernel choice visible without changing the API.
static bool log_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("EMUGEMM_LOG");
        return e && *e && std::strcmp(e, "0") != 0;
    }();
    return on;
}

static const char* scheme_name(emu_scheme_t s) {
    switch (s) {
        case EMU_SCHEME_AUTO: return "AUTO";
        case EMU_SCHEME_NATIVE_FP32: return "NATIVE_FP32";
        case EMU_SCHEME_FP32_CHUNKED: return "FP32_CHUNKED";
        case EMU_SCHEME_BF16X3: return "BF16X3";
        case EMU_SCHEME_FP16X3: return "FP16X3";
        case EMU_SCHEME_BF16X6: return "BF16X6";
        default: return "?";
    }
}

static void log_plan(const char* entry, int M, int N, long K, const emu_plan_t& p, const emu_hints_t& hn) {
    if (!log_enabled()) return;
    std::fprintf(stderr, "emugemm: %s M=%d N=%d K=%ld scheme=%s chunks=%d predicted_err=%.4e rho=%g reason=\"%s\"\n",
                 entry, M, N, K, scheme_name(p.chosen), p.chunks, p.predicted_err, (double)hn.rho,
                 p.reason ? p.reason : "");
}

// K splits of the CTA-pair kernels. When their 256 x 256 tiles cannot occupy the SM pairs (a few output tiles and a
// long K: M = N = 256, K = 262144 is one tile for 74 pairs), each tile's K range is split into ranges of whole 128-K
// chunks of the true K, at least 1024 values of K each, for at most one unit per SM pair; every split writes an FP64
// partial and the partials are summed in order (deterministic). Every split starts a promotion chunk, so the pre-split
// and the fused kernel split at the same values of K and stay bit-identical. The handle's EMUGEMM_ATTR_TC_SPLITK
// (`forced`, a count >= 1; 0 = choose) overrides the choice.
int tc_split_count(long Mp, long Np, long K, int num_sms, int forced) {
    const long nck = (K + 127) / 128, tiles = (Mp / 256) * (Np / 256), pairs = num_sms / 2;   // 128-K chunks
    long want = 1;
    if (forced > 0) want = forced;
    else if (tiles > 0 && tiles < pairs) want = std::min(pairs / tiles, nck / 8);
    if (want < 1) want = 1;
    if (want > nck) want = nck;
    const long kpc = (nck + want - 1) / want;
    return (int)((nck + kpc - 1) / kpc);   // every split non-empty
}

int tc_kernel_choice(Handle* h, int M, int N, long K, bool fp16) {
    if (h->pin_tc_code) return h->pin_tc_code;
    int code = h->tc_kernel;
    if (!code) code = lookup_tile(M, N, K, fp16 ? 2 : 1).tc_variant;
    if (!code) {
        const long pair_tiles = (round_up(M, 256) / 256) * (round_up(N, 256) / 256), pairs = h->num_sms / 2;
        if (!fp16) {
            code = (K > 1024 || pair_tiles >= pairs) ? 2 : 1;
            // few tiles and K split over the SM pairs: the GEMM reads each operand element once, so the split pass
            // (8 bytes moved per element) costs more than the GEMM; the fused kernel splits in shared memory
            // (256^2 x 262144: 106 -> 217 TFLOPS; at 16 tiles both kernels tie)
            if (code == 2 && pair_tiles < 16 &&
                tc_split_count(round_up(M, 256), round_up(N, 256), K, h->num_sms, h->tc_splitk) > 1)
                code = 3;
        }
        else {
            code = (pair_tiles >= pairs ? (K > 1024 || pair_tiles >= 512) : K >= 16384) ? 2 : 1;
            // few tiles and K split over the SM pairs: as for bf16x3, the split in shared memory saves the split pass
            if (code == 2 && pair_tiles < 16 &&
                tc_split_count(round_up(M, 256), round_up(N, 256), K, h->num_sms, h->tc_splitk) > 1)
                code = 3;
        }
    }
    if (fp16 && code == 4) code = 2;   // fp16x3 has no A-in-TMEM kernel
    if (log_enabled()) {
        static const char* names[] = {"?", "single", "pair", "fused", "fusea"};
        std::fprintf(stderr, "emugemm: tensor-core kernel=%s (%s) M=%d N=%d K=%ld\n", names[code], fp16 ? "fp16x3" : "bf16x3",
                     M, N, K);
    }
    return code;
}

// SMs the tensor-core kernels may spread over: all of them, unless a multi-GPU call leaves some to its collectives
// (the grid only; the K split count, and with it every bit of C, follows the whole GPU).
static int tc_grid_sms(const Handle* h) {
    return h->tc_grid_sms > 0 && h->tc_grid_sms < h->num_sms ? h->tc_grid_sms : h->num_sms;
}

// bf16x3 / fp16x3 through the tensor-core kernel over pre-split slices. With a_reused (hints->a_is_reused) and
// the same A (pointer, shape, leading dimension, scheme) as the split already held in the workspace, A is not
// split again: the caller has declared A unchanged since that call. With a_only, only A's slices (and its fp16
// row exponents) are made, for a caller that runs the GEMMs later with a_reused (B, C, N unused).
static emugemm_status_t run_tc(Handle* h, int M, int N, long K, const float* A, long lda, const float* B, long ldb,
                               float* C, long ldc, double* C64, long ldc64, bool fp16, bool a_reused,
                               bool a_only = false) {
    const int choice = tc_kernel_choice(h, M, N, K, fp16);
    if (a_only && (choice == 3 || choice == 4)) return EMUGEMM_STATUS_SUCCESS;   // these split A in the kernel
    if (choice == 3 && (lda & 3) == 0 && (ldb & 3) == 0 && (reinterpret_cast<uintptr_t>(A) & 15) == 0 &&
        (reinterpret_cast<uintptr_t>(B) & 15) == 0) {
        const int splits = h->pin_splits ? h->pin_splits
                                         : tc_split_count(round_up(M, 256), round_up(N, 256), K, h->num_sms, h->tc_splitk);
        double* part = nullptr;
        if (splits > 1) {
            part = (double*)ws_get(h, bank_slot(h, kWsSplitK), (size_t)splits * M * N * sizeof(double));
            if (!part) return EMUGEMM_STATUS_MEMORY_ERROR;
        }
        int* rexp = nullptr;
        int* cexp = nullptr;
        if (fp16) {
            // the scale exponents of the split, made by the same scans as on the pre-split path
            rexp = (int*)ws_get(h, kWsScaleA, (size_t)M * 4);
            cexp = (int*)ws_get(h, bank_slot(h, kWsScaleB), (size_t)N * 8);
            if (!rexp || !cexp) return EMUGEMM_STATUS_MEMORY_ERROR;
            h->a_key = Handle::ASplitKey();   // the row exponents are rewritten below
            ProfScope ps(h, kProfScan);
            int e = launch_row_exponents(A, M, K, lda, rexp, h->stream);
            if (!e) e = launch_col_exponents(B, K, N, ldb, cexp, reinterpret_cast<unsigned*>(cexp + N), h->stream);
            if (e) return from_cuda(e);
        }
        ProfScope ps(h, kProfTcGemm);
        const int e = launch_tc_fused(A, lda, B, ldb, M, N, K, C, ldc, C64, ldc64, h->err_dev, tc_grid_sms(h), h->stream,
                                      splits, part, fp16 ? 1 : 0, rexp, cexp);
        if (e != (int)cudaErrorNotSupported) {
            if (e || splits <= 1) return from_cuda(e);
            return from_cuda(launch_reduce_f64(part, splits, M, N, (long)M * N, C, ldc, C64, ldc64, h->stream));
        }
        // operands TMA cannot address (odd leading dimension or alignment): pre-split below
    }
    if (choice == 4 && (lda & 3) == 0 && (reinterpret_cast<uintptr_t>(A) & 15) == 0) {
        const long Np4 = round_up(N, tc_fused_a_bn()), Kp4 = slice_kp(K), KP4 = slice_panel(Kp4);
        if (Np4 > 0x7fffffffL) return EMUGEMM_STATUS_INVALID_SIZE;
        uint16_t* b0 = (uint16_t*)ws_get(h, bank_slot(h, kWsSplitB0), (size_t)Np4 * Kp4 * 2);
        uint16_t* b1 = (uint16_t*)ws_get(h, bank_slot(h, kWsSplitB1), (size_t)Np4 * Kp4 * 2);
        if (!b0 || !b1) return EMUGEMM_STATUS_MEMORY_ERROR;
        int e = 0;
        {
            ProfScope ps(h, kProfSplit);
            e = launch_split_cols(B, K, N, ldb, (int)Np4, Kp4, KP4, 0, nullptr, b0, b1, h->stream);
        }
        if (e) return from_cuda(e);
        ProfScope ps(h, kProfTcGemm);
        return from_cuda(launch_tc_fused_a(A, lda, b0, b1, M, N, (int)Np4, K, Kp4, KP4, C, ldc, C64, ldc64,
                                           h->err_dev, tc_grid_sms(h), h->stream));
    }
    const bool pair = choice >= 2;
    const int BN = pair ? tc_pair_bn(fp16 ? 1 : 0) : tc_gemm_bn(fp16 ? 1 : 0);
    const long Mp = round_up(M, pair ? 256 : 128), Np = round_up(N, BN), Kp = slice_kp(K), KP = slice_panel(Kp);
    if (Mp > 0x7fffffffL || Np > 0x7fffffffL || Kp > 0x7fffffffL) return EMUGEMM_STATUS_INVALID_SIZE;
    uint16_t* a0 = (uint16_t*)ws_get(h, kWsSplitA0, (size_t)Mp * Kp * 2);
    uint16_t* a1 = (uint16_t*)ws_get(h, kWsSplitA1, (size_t)Mp * Kp * 2);
    uint16_t* b0 = (uint16_t*)ws_get(h, bank_slot(h, kWsSplitB0), (size_t)Np * Kp * 2);
    uint16_t* b1 = (uint16_t*)ws_get(h, bank_slot(h, kWsSplitB1), (size_t)Np * Kp * 2);
    if (!a0 || !a1 || !b0 || !b1) return EMUGEMM_STATUS_MEMORY_ERROR;
    int* rexp = nullptr;
    int* cexp = nullptr;
    if (fp16) {
        rexp = (int*)ws_get(h, kWsScaleA, (size_t)M * 4);
        cexp = (int*)ws_get(h, bank_slot(h, kWsScaleB), (size_t)N * 8);
        if (!rexp || !cexp) return EMUGEMM_STATUS_MEMORY_ERROR;
    }
    const int kind = fp16 ? 1 : 0;
    Handle::ASplitKey key;
    key.A = A; key.M = M; key.K = K; key.lda = lda; key.kind = kind; key.Mp = Mp; key.Kp = Kp;
    key.ws0 = a0; key.ws1 = a1; key.rexp = rexp;
    const Handle::ASplitKey& k0 = h->a_key;
    const bool reuse = a_reused && k0.A == key.A && k0.M == key.M && k0.K == key.K && k0.lda == key.lda &&
                       k0.kind == key.kind && k0.Mp == key.Mp && k0.Kp == key.Kp && k0.ws0 == key.ws0 &&
                       k0.ws1 == key.ws1 && k0.rexp == key.rexp;
    int e = 0;
    if (fp16) {
        ProfScope ps(h, kProfScan);
        if (!reuse) e = launch_row_exponents(A, M, K, lda, rexp, h->stream);
        if (!e && !a_only)
            e = launch_col_exponents(B, K, N, ldb, cexp, reinterpret_cast<unsigned*>(cexp + N), h->stream);
        if (e) return from_cuda(e);
    }
    {
        ProfScope ps(h, kProfSplit);
        if (!reuse) {
            h->a_key = Handle::ASplitKey();   // invalid until the split below has been enqueued
            e = launch_split_rows(A, M, K, lda, (int)Mp, Kp, KP, kind, rexp, a0, a1, h->stream);
        }
        if (!e && !a_only) e = launch_split_cols(B, K, N, ldb, (int)Np, Kp, KP, kind, cexp, b0, b1, h->stream);
    }
    if (e) return from_cuda(e);
    h->a_key = key;
    if (a_only) {
        // size the FP64 planes of the K splits now, so that no later panel grows the workspace (a reallocation
        // synchronises the stream)
        const int sp = !pair ? 1 : h->pin_splits ? h->pin_splits : tc_split_count(Mp, Np, K, h->num_sms, h->tc_splitk);
        for (int b = 0; b < 2; ++b) {   // both banks, for panel GEMMs on two streams
            const int keep = h->bank;
            h->bank = b;
            const bool ok = ws_get(h, bank_slot(h, kWsSplitB0), (size_t)Np * Kp * 2) &&
                            ws_get(h, bank_slot(h, kWsSplitB1), (size_t)Np * Kp * 2) &&
                            (!fp16 || ws_get(h, bank_slot(h, kWsScaleB), (size_t)N * 8)) &&
                            (sp <= 1 || ws_get(h, bank_slot(h, kWsSplitK), (size_t)sp * M * N * sizeof(double)));
            h->bank = keep;
            if (!ok) return EMUGEMM_STATUS_MEMORY_ERROR;
        }
        return EMUGEMM_STATUS_SUCCESS;
    }
    TcGemmArgs t;
    t.a_hi = a0; t.a_lo = a1; t.b_hi = b0; t.b_lo = b1;
    t.M = M; t.N = N; t.Mp = (int)Mp; t.Np = (int)Np; t.Kp = Kp; t.KP = KP;
    t.C = C; t.ldc = ldc; t.C64 = C64; t.ldc64 = ldc64;
    t.fp16 = fp16 ? 1 : 0;
    t.row_exp = rexp; t.col_exp = cexp;
    t.err = h->err_dev;
    t.num_sms = tc_grid_sms(h);
    if (pair) {
        t.splits = h->pin_splits ? h->pin_splits : tc_split_count(Mp, Np, K, h->num_sms, h->tc_splitk);
        t.K = K;
        if (t.splits > 1) {
            t.part64 = (double*)ws_get(h, bank_slot(h, kWsSplitK), (size_t)t.splits * M * N * sizeof(double));
            if (!t.part64) return EMUGEMM_STATUS_MEMORY_ERROR;
        }
    }
    ProfScope ps(h, kProfTcGemm);
    e = pair ? launch_tc_gemm_pair(t, h->stream) : launch_tc_gemm(t, h->stream);
    if (e || t.splits <= 1) return from_cuda(e);
    return from_cuda(launch_reduce_f64(t.part64, t.splits, M, N, (long)M * N, C, ldc, C64, ldc64, h->stream));
}

// FP32 SIMT tile code for a shape: `forced` (the handle's EMUGEMM_ATTR_FP32_TILE, a code of fp32_tile_code_ok; 0 = choose) wins,
// then the tile table's code (looked up at the chunk length), else 0 (the built-in choice of launch_fp32_gemm).
static int fp32_tile_choice(int M, int N, long K, int chunks, int forced) {
    if (fp32_tile_code_ok(forced)) return forced;
    return lookup_tile(M, N, K / (chunks < 1 ? 1 : chunks), 0).fp32_bm;
}

// Defaults of the per-handle kernel choices, from the environment (read when a handle is created).
static int env_tc_kernel() {
    const char* v = std::getenv("EMUGEMM_TC_KERNEL");
    if (!v) return 0;
    if (std::strcmp(v, "single") == 0) return 1;
    if (std::strcmp(v, "pair") == 0) return 2;
    if (std::strcmp(v, "fused") == 0) return 3;
    if (std::strcmp(v, "fusea") == 0) return 4;
    return 0;
}
static int env_tc_splitk() {
    const char* v = std::getenv("EMUGEMM_TC_SPLITK");
    const long n = v ? std::atol(v) : 0;
    return n >= 1 && n <= (1L << 20) ? (int)n : 0;
}
static int env_fp32_tile() {
    const char* v = std::getenv("EMUGEMM_FP32_TILE");
    const int t = v ? std::atoi(v) : 0;
    return fp32_tile_code_ok(t) ? t : 0;
}

static emugemm_status_t run_fp32(Handle* h, int M, int N, long K, const float* A, long lda, const float* B, long ldb,
                                 float* C, long ldc, double* C64, long ldc64, int chunks) {
    Fp32GemmArgs f;
    f.A = A; f.lda = lda; f.B = B; f.ldb = ldb;
    f.C = C; f.ldc = ldc; f.C64 = C64; f.ldc64 = ldc64;
    f.M = M; f.N = N; f.K = K;
    f.chunks = chunks < 1 ? 1 : chunks;
    f.num_sms = h->num_sms;
    f.bm = fp32_tile_choice(M, N, K, f.chunks, h->fp32_tile);
    f.err = h->err_dev;
    f.ws64 = nullptr;
    size_t wsb = fp32_gemm_ws_bytes(f);
    if (wsb) {
        f.ws64 = (double*)ws_get(h, bank_slot(h, kWsF64Acc), wsb);
        if (!f.ws64) return EMUGEMM_STATUS_MEMORY_ERROR;
    }
    ProfScope ps(h, kProfFp32Gemm);
    return from_cuda(launch_fp32_gemm(f, h->stream));
}

// Zero an M x N output (K == 0).
static emugemm_status_t zero_out(Handle* h, int M, int N, float* C, long ldc, double* C64, long ldc64) {
    cudaError_t e;
    if (C64)
        e = cudaMemset2DAsync(C64, (size_t)ldc64 * 8, 0, (size_t)N * 8, (size_t)M, (cudaStream_t)h->stream);
    else
        e = cudaMemset2DAsync(C, (size_t)ldc * 4, 0, (size_t)N * 4, (size_t)M, (cudaStream_t)h->stream);
    return from_cuda((int)e);
}

emugemm_status_t dispatch(Handle* h, emu_scheme_t s, int chunks, int M, int N, long K, const float* A, long lda,
                          const float* B, long ldb, float* C, long ldc, double* C64, long ldc64, bool a_reused) {
    if (M == 0 || N == 0) return EMUGEMM_STATUS_SUCCESS;
    if (K == 0) return zero_out(h, M, N, C, ldc, C64, ldc64);
    switch (s) {
        case EMU_SCHEME_NATIVE_FP32: return run_fp32(h, M, N, K, A, lda, B, ldb, C, ldc, C64, ldc64, 1);
        case EMU_SCHEME_FP32_CHUNKED: return run_fp32(h, M, N, K, A, lda, B, ldb, C, ldc, C64, ldc64, chunks);
        // A forced BF16X6 runs the bf16x3 kernel, as the reference does (src/emugemm.cpp:331).
        case EMU_SCHEME_BF16X3:
        case EMU_SCHEME_BF16X6: return run_tc(h, M, N, K, A, lda, B, ldb, C, ldc, C64, ldc64, false, a_reused);
        case EMU_SCHEME_FP16X3: return run_tc(h, M, N, K, A, lda, B, ldb, C, ldc, C64, ldc64, true, a_reused);
        default: return EMUGEMM_STATUS_NOT_IMPLEMENTED;
    }
}

emugemm_status_t prepare_a(Handle* h, emu_scheme_t s, int M, int N, long K, const float* A, long lda) {
    if (M == 0 || N == 0 || K == 0) return EMUGEMM_STATUS_SUCCESS;
    switch (s) {
        case EMU_SCHEME_BF16X3:
        case EMU_SCHEME_BF16X6:
            return run_tc(h, M, N, K, A, lda, nullptr, N, nullptr, N, nullptr, 0, false, false, true);
        case EMU_SCHEME_FP16X3:
            return run_tc(h, M, N, K, A, lda, nullptr, N, nullptr, N, nullptr, 0, true, false, true);
        default: return EMUGEMM_STATUS_SUCCESS;   // the FP32 kernels read A as it is
    }
}

static bool is_sm100(int dev) {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return false;
    if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) return false;
    return major == 10 && minor == 0;
}

}  // namespace emu

using emu::Handle;

extern "C" {

emugemm_status_t emugemm_create_handle(emugemm_handle_t* out) {
    if (!out) return EMUGEMM_STATUS_INVALID_POINTER;
    *out = nullptr;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) { cudaGetLastError(); return EMUGEMM_STATUS_INTERNAL_ERROR; }
    if (!emu::is_sm100(dev)) return EMUGEMM_STATUS_ARCH_MISMATCH;
    Handle* h = new Handle();
    h->device = dev;
    h->tc_kernel = emu::env_tc_kernel();
    h->tc_splitk = emu::env_tc_splitk();
    h->fp32_tile = emu::env_fp32_tile();
    cudaDeviceGetAttribute(&h->num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (cudaHostAlloc((void**)&h->err_host, sizeof(unsigned), cudaHostAllocMapped) != cudaSuccess ||
        cudaHostGetDevicePointer((void**)&h->err_dev, h->err_host, 0) != cudaSuccess) {
        cudaGetLastError();
        if (h->err_host) cudaFreeHost(h->err_host);
        delete h;
        return EMUGEMM_STATUS_MEMORY_ERROR;
    }
    *h->err_host = 0;
    *out = reinterpret_cast<emugemm_handle_t>(h);
    return EMUGEMM_STATUS_SUCCESS;
}

emugemm_status_t emugemm_destroy_handle(emugemm_handle_t handle) {
    Handle* h = reinterpret_cast<Handle*>(handle);
    if (!h) return EMUGEMM_STATUS_INVALID_HANDLE;
    emu::DeviceGuard g(h->device);
    cudaStreamSynchronize((cudaStream_t)h->stream);
    for (void* ev : h->host_ev)
        if (ev) cudaEventDestroy((cudaEvent_t)ev);
    if (h->copy_in) cudaStreamDestroy((cudaStream_t)h->copy_in);
    if (h->copy_out) cudaStreamDestroy((cudaStream_t)h->copy_out);
    emu::multigpu_release(h);
    for (int i = 0; i < emu::kWsCount; ++i)
        if (h->ws[i]) cudaFree(h->ws[i]);
    emu::prof_clear(h);
    delete[] h->prof;
    if (h->err_host) cudaFreeHost(h->err_host);
    delete h;
    return EMUGEMM_STATUS_SUCCESS;
}

emugemm_status_t emugemm_set_stream(emugemm_handle_t handle, void* stream) {
    Handle* h = reinterpret_cast<Handle*>(handle);
    if (!h) return EMUGEMM_STATUS_INVALID_HANDLE;
    h->stream = stream;
    return EMUGEMM_STATUS_SUCCESS;
}

emugemm_status_t emugemm_set_workspace_limit(emugemm_handle_t handle, size_t bytes) {
    Handle* h = reinterpret_cast<Handle*>(handle);
    if (!h) return EMUGEMM_STATUS_INVALID_HANDLE;
    h->ws_limit = bytes;
    return EMUGEMM_STATUS_SUCCESS;
}

emugemm_status_t emugemm_set_attr(emugemm_handle_t handle, int attr, long value) {
    Handle* h = reinterpret_cast<Handle*>(handle);
    if (!h) return EMUGEMM_STATUS_INVALID_HANDLE;
    switch (attr) {
        case EMUGEMM_ATTR_TC_KERNEL:
            if (value < 0 || value > 4) return EMUGEMM_STATUS_INVALID_VALUE;
            h->tc_kernel = (int)value;
            return EMUGEMM_STATUS_SUCCESS;
        case EMUGEMM_ATTR_TC_SPLITK:
            if (value < 0 || value > (1L << 20)) return EMUGEMM_STATUS_INVALID_VALUE;
            h->tc_splitk = (int)value;
            return EMUGEMM_STATUS_SUCCESS;
        case EMUGEMM_ATTR_FP32_TILE:
            if (value != 0 && !emu::fp32_tile_code_ok(value)) return EMUGEMM_STATUS_INVALID_VALUE;
            h->fp32_tile = (int)value;
            return EMUGEMM_STATUS_SUCCESS;
        case EMUGEMM_ATTR_ROWS_PANELS:
            if (value < 0 || value > 16) return EMUGEMM_STATUS_INVALID_VALUE;
            h->rows_panels = (int)value;
            return EMUGEMM_STATUS_SUCCESS;
        case EMUGEMM_ATTR_COMM_SMS:
            if (value < 0 || value > 64 || (value & 1)) return EMUGEMM_STATUS_INVALID_VALUE;
            h->comm_sms = (int)value;
            return EMUGEMM_STATUS_SUCCESS;
        case EMUGEMM_ATTR_BCAST_NCCL:
            if (value != 0 && value != 1) return EMUGEMM_STATUS_INVALID_VALUE;
            h->bcast_nccl = (int)value;
            return EMUGEMM_STATUS_SUCCESS;
    }
    return EMUGEMM_STATUS_INVALID_VALUE;
}

emugemm_status_t emugemm_get_attr(emugemm_handle_t handle, int attr, long* value) {
    Handle* h = reinterpret_cast<Handle*>(handle);
    if (!h) return EMUGEMM_STATUS_INVALID_HANDLE;
    if (!value) return EMUGEMM_STATUS_INVALID_POINTER;
    switch (attr) {
        case EMUGEMM_ATTR_TC_KERNEL: *value = h->tc_kernel; return EMUGEMM_STATUS_SUCCESS;
        case EMUGEMM_ATTR_TC_SPLITK: *value = h->tc_splitk; return EMUGEMM_STATUS_SUCCESS;
        case EMUGEMM_ATTR_FP32_TILE: *value = h->fp32_tile; return EMUGEMM_STATUS_SUCCESS;
        case EMUGEMM_ATTR_ROWS_PANELS: *value = h->rows_panels; return EMUGEMM_STATUS_SUCCESS;
        case EMUGEMM_ATTR_COMM_SMS: *value = h->comm_sms; return EMUGEMM_STATUS_SUCCESS;
        case EMUGEMM_ATTR_BCAST_NCCL: *value = h->bcast_nccl; return EMUGEMM_STATUS_SUCCESS;
    }
    return EMUGEMM_STATUS_INVALID_VALUE;
}

emugemm_status_t emugemm_sync(emugemm_handle_t handle) {
    Handle* h = reinterpret_cast<Handle*>(handle);
    if (!h) return EMUGEMM_STATUS_INVALID_HANDLE;
    emu::DeviceGuard g(h->device);
    return emu::sync_check(h);
}

emugemm_status_t emugemm_peak_probe(emugemm_handle_t handle, int reps, double* rates, int n) {
    Handle* h = reinterpret_cast<Handle*>(handle);
    if (!h) return EMUGEMM_STATUS_INVALID_HANDLE;
    if (!rates && n > 0) return EMUGEMM_STATUS_INVALID_POINTER;
    if (reps < 1 || n < 0) return EMUGEMM_STATUS_INVALID_VALUE;
    emu::DeviceGuard g(h->device);
    emugemm_status_t s = emu::sync_check(h);
    if (s != EMUGEMM_STATUS_SUCCESS) return s;
    double r[EMU_PEAK_COUNT] = {};
    const int e = emu::run_peak_probe(reps, h->num_sms, h->err_dev, h->err_host, h->stream, r);
    if (e == -1) return emu::take_device_error(h);
    if (e) return emu::from_cuda(e);
    for (int i = 0; i < n && i < EMU_PEAK_COUNT; ++i) rates[i] = r[i];
    return EMUGEMM_STATUS_SUCCESS;
}

void emugemm_shutdown(void) { emu::tune_clear(); }

emugemm_status_t emugemm_sgemm_ex(emugemm_handle_t handle, int M, int N, long K, const float* A, long lda,
                                  const float* B, long ldb, float* C, long ldc, const emu_request_t* req,
                                  emu_hints_t* hints, emu_plan_t* out_plan) {
    Handle* h = reinterpret_cast<Handle*>(handle);
    if (!h) return EMUGEMM_STATUS_INVALID_HANDLE;
    if (M < 0 || N < 0 || K < 0) return EMUGEMM_STATUS_INVALID_SIZE;
    if (lda < (K > 0 ? K : 1) || ldb < (N > 0 ? N : 1) || ldc < (N > 0 ? N : 1)) return EMUGEMM_STATUS_INVALID_SIZE;
    if ((M > 0 && N > 0) && (!C || (K > 0 && (!A || !B)))) return EMUGEMM_STATUS_INVALID_POINTER;
    emu::DeviceGuard g(h->device);
    if (!g.ok) return EMUGEMM_STATUS_INTERNAL_ERROR;

    // src/emugemm.cpp:288-294: hints are in/out; NULL means measure everything with 64 probes.
    emu_hints_t local = hints ? *hints : emu_hints_t{-1.f, -1.f, 0, -1.f, 0};
    const bool have_a = (long)M * K > 0, have_b = K * (long)N > 0;
    if (local.a_absmax < 0) {
        float v = 0.f;
        if (have_a) {
            emugemm_status_t s = emu::absmax(h, A, M, K, lda, &v);
            if (s != EMUGEMM_STATUS_SUCCESS) return s;
        }
        local.a_absmax = v;
    }
    if (local.b_absmax < 0) {
        float v = 0.f;
        if (have_b) {
            emugemm_status_t s = emu::absmax(h, B, K, N, ldb, &v);
            if (s != EMUGEMM_STATUS_SUCCESS) return s;
        }
        local.b_absmax = v;
    }
    if (local.rho < 0) local.rho = (float)emu::estimate_rho(h, M, N, K, A, lda, B, ldb, local.rho_probes);
    if (hints) {
        hints->a_absmax = local.a_absmax;
        hints->b_absmax = local.b_absmax;
        hints->rho = local.rho;
    }
    emu_plan_t plan = emu::plan(emu::model(), M, N, K, req, &local);
    if (out_plan) *out_plan = plan;
    emu::log_plan("sgemm", M, N, K, plan, local);
    return emu::dispatch(h, plan.chosen, plan.chunks, M, N, K, A, lda, B, ldb, C, ldc, nullptr, 0,
                         hints && hints->a_is_reused);
}

emugemm_status_t emugemm_sgemm(emugemm_handle_t handle, int M, int N, long K, const float* A, const float* B,
                               float* C, const emu_request_t* req, emu_hints_t* hints, emu_plan_t* out_plan) {
    return emugemm_sgemm_ex(handle, M, N, K, A, K > 0 ? K : 1, B, N > 0 ? N : 1, C, N > 0 ? N : 1, req, hints,
                            out_plan);
}

emugemm_status_t emugemm_sgemm_host(emugemm_handle_t handle, int M, int N, long K, const float* A, const float* B,
                                    float* C, const emu_request_t* req, emu_hints_t* hints, emu_plan_t* out_plan) {
    Handle* h = reinterpret_cast<Handle*>(handle);
    if (!h) return EMUGEMM_STATUS_INVALID_HANDLE;
    if (M < 0 || N < 0 || K < 0) return EMUGEMM_STATUS_INVALID_SIZE;
    if ((M > 0 && N > 0) && (!C || (K > 0 && (!A || !B)))) return EMUGEMM_STATUS_INVALID_POINTER;
    emu::DeviceGuard g(h->device);
    if (!g.ok) return EMUGEMM_STATUS_INTERNAL_ERROR;
    if (M == 0 || N == 0) {
        if (out_plan) {
            emu_hints_t local = hints ? *hints : emu_hints_t{0.f, 0.f, 0, 0.f, 0};
            *out_plan = emu::plan(emu::model(), M, N, K, req, &local);
        }
        return EMUGEMM_STATUS_SUCCESS;
    }
    cudaStream_t cs = (cudaStream_t)h->stream;
    const size_t a_bytes = (size_t)M * K * 4, b_bytes = (size_t)K * N * 4, c_bytes = (size_t)M * N * 4;
    float* dA = (float*)emu::ws_get(h, emu::kWsHostA, a_bytes ? a_bytes : 4);
    float* dB = (float*)emu::ws_get(h, emu::kWsHostB, b_bytes ? b_bytes : 4);
    float* dC = (float*)emu::ws_get(h, emu::kWsHostC, c_bytes);
    if (!dA || !dB || !dC) return EMUGEMM_STATUS_MEMORY_ERROR;
    if (!h->copy_in) {
        if (cudaStreamCreateWithFlags((cudaStream_t*)&h->copy_in, cudaStreamNonBlocking) != cudaSuccess ||
            cudaStreamCreateWithFlags((cudaStream_t*)&h->copy_out, cudaStreamNonBlocking) != cudaSuccess) {
            cudaGetLastError();
            return EMUGEMM_STATUS_INTERNAL_ERROR;
        }
        for (void*& ev : h->host_ev)
            if (cudaEventCreateWithFlags((cudaEvent_t*)&ev, cudaEventDisableTiming) != cudaSuccess) {
                cudaGetLastError();
                return EMUGEMM_STATUS_INTERNAL_ERROR;
            }
    }
    cudaStream_t cin = (cudaStream_t)h->copy_in, cout = (cudaStream_t)h->copy_out;
    cudaEvent_t* ev = reinterpret_cast<cudaEvent_t*>(h->host_ev);
    cudaEvent_t ev_start = ev[0], ev_done = ev[1];
    cudaEvent_t* ev_b = ev + 2;                          // panel j of B has arrived
    cudaEvent_t* ev_c = ev + 2 + emu::kMaxHostPanels;    // panel j of C is computed
    int e = 0;
    // the copies must not overwrite the device operands while earlier work on the handle's stream reads them
    e = cudaEventRecord(ev_start, cs);
    if (!e) e = cudaStreamWaitEvent(cin, ev_start, 0);
    if (!e) e = cudaStreamWaitEvent(cout, ev_start, 0);
    if (e) return emu::from_cuda(e);

    // Hints that ask for scans need all of A and B on the device first: copy, then the device entry point.
    const bool measure = !hints || hints->a_absmax < 0 || hints->b_absmax < 0 || hints->rho < 0 || K == 0;
    if (measure) {
        if (a_bytes) e = cudaMemcpyAsync(dA, A, a_bytes, cudaMemcpyHostToDevice, cs);
        if (!e && b_bytes) e = cudaMemcpyAsync(dB, B, b_bytes, cudaMemcpyHostToDevice, cs);
        if (e) return emu::from_cuda(e);
        emugemm_status_t s = emugemm_sgemm_ex(handle, M, N, K, dA, K > 0 ? K : 1, dB, N, dC, N, req, hints, out_plan);
        if (s != EMUGEMM_STATUS_SUCCESS) return s;
        return emu::from_cuda(cudaMemcpyAsync(C, dC, c_bytes, cudaMemcpyDeviceToHost, cs));
    }

    emu_hints_t local = *hints;
    emu_plan_t plan = emu::plan(emu::model(), M, N, K, req, &local);
    if (out_plan) *out_plan = plan;
    emu::log_plan("sgemm_host", M, N, K, plan, local);
    // Row panels, so that every PCIe copy is contiguous: B crosses first in one copy; then panel i of A (its rows
    // [r0, r1)) travels on copy_in, its GEMM runs on the handle's stream as soon as it has landed, and panel i of C
    // travels back on copy_out while later panels of A arrive (PCIe carries both directions at once). B's column
    // panels had been pitched copies with 4 KB rows, which ran below the contiguous rate (8192^3: 12.2 ms per call
    // against about 11 for contiguous copies). Heights are multiples of 256 rows (whole CTA-pair tiles), about 8
    // panels.
    long hgt = ((long)M + 7) / 8;
    hgt = (hgt + 255) / 256 * 256;
    if (hgt < 256) hgt = 256;
    while ((M + hgt - 1) / hgt > emu::kMaxHostPanels) hgt += 256;
    const int np = (int)((M + hgt - 1) / hgt);
    // the panels use the kernel and K split count of the whole product, so C has the bits of the single call
    const bool tc = plan.chosen == EMU_SCHEME_BF16X3 || plan.chosen == EMU_SCHEME_BF16X6 ||
                    plan.chosen == EMU_SCHEME_FP16X3;
    if (tc) {
        const bool fp16 = plan.chosen == EMU_SCHEME_FP16X3;
        h->pin_tc_code = emu::tc_kernel_choice(h, M, N, K, fp16);
        h->pin_splits = emu::tc_split_count(emu::round_up(M, 256), emu::round_up(N, 256), K, h->num_sms, h->tc_splitk);
    }
    struct Unpin {
        Handle* h;
        ~Unpin() { h->pin_tc_code = 0; h->pin_splits = 0; }
    } unpin{h};
    e = cudaMemcpyAsync(dB, B, b_bytes, cudaMemcpyHostToDevice, cin);
    for (int i = 0; i < np && !e; ++i) {
        const long r0 = (long)i * hgt, rows = (r0 + hgt <= M) ? hgt : M - r0;
        e = cudaMemcpyAsync(dA + (size_t)r0 * K, A + (size_t)r0 * K, (size_t)rows * K * 4, cudaMemcpyHostToDevice,
                            cin);
        if (!e) e = cudaEventRecord(ev_b[i], cin);
        if (!e) e = cudaStreamWaitEvent(cs, ev_b[i], 0);
        if (e) break;
        emugemm_status_t s = emu::dispatch(h, plan.chosen, plan.chunks, (int)rows, N, K, dA + (size_t)r0 * K, K, dB,
                                           N, dC + (size_t)r0 * N, N, nullptr, 0);
        if (s != EMUGEMM_STATUS_SUCCESS) return s;
        e = cudaEventRecord(ev_c[i], cs);
        if (!e) e = cudaStreamWaitEvent(cout, ev_c[i], 0);
        if (!e)
            e = cudaMemcpyAsync(C + (size_t)r0 * N, dC + (size_t)r0 * N, (size_t)rows * N * 4, cudaMemcpyDeviceToHost,
                                cout);
    }
    // the call is complete, for the handle's stream, once the last panel of C has reached the host
    if (!e) e = cudaEventRecord(ev_done, cout);
    if (!e) e = cudaStreamWaitEvent(cs, ev_done, 0);
    return emu::from_cuda(e);
}

double emugemm_estimate_rho(emugemm_handle_t handle, int M, int N, long K, const float* A, const float* B,
                            int probes) {
    Handle* h = reinterpret_cast<Handle*>(handle);
    if (!h || !A || !B) return -1.0;
    emu::DeviceGuard g(h->device);
    return emu::estimate_rho(h, M, N, K, A, K, B, N, probes);
}

emugemm_status_t emugemm_absmax(emugemm_handle_t handle, const float* X, size_t n, float* out_absmax) {
    Handle* h = reinterpret_cast<Handle*>(handle);
    if (!h) return EMUGEMM_STATUS_INVALID_HANDLE;
    if (!out_absmax || (n && !X)) return EMUGEMM_STATUS_INVALID_POINTER;
    emu::DeviceGuard g(h->device);
    if (n == 0) { *out_absmax = 0.f; return EMUGEMM_STATUS_SUCCESS; }
    return emu::absmax(h, X, 1, (long)n, (long)n, out_absmax);
}

emugemm_status_t emugemm_split_bf16(emugemm_handle_t handle, const float* X, size_t n, unsigned short* hi,
                                    unsigned short* lo) {
    Handle* h = reinterpret_cast<Handle*>(handle);
    if (!h) return EMUGEMM_STATUS_INVALID_HANDLE;
    if (n && (!X || !hi || !lo)) return EMUGEMM_STATUS_INVALID_POINTER;
    emu::DeviceGuard g(h->device);
    return emu::from_cuda(emu::launch_split_bf16(X, n, hi, lo, h->stream));
}

emugemm_status_t emugemm_split_f16(emugemm_handle_t handle, const float* X, size_t n, unsigned short* hi,
                                   unsigned short* lo) {
    Handle* h = reinterpret_cast<Handle*>(handle);
    if (!h) return EMUGEMM_STATUS_INVALID_HANDLE;
    if (n && (!X || !hi || !lo)) return EMUGEMM_STATUS_INVALID_POINTER;
    emu::DeviceGuard g(h->device);
    return emu::from_cuda(emu::launch_split_f16(X, n, hi, lo, h->stream));
}

emugemm_status_t emugemm_sgemm_partial_f64(emugemm_handle_t handle, int M, int N, long K, const float* A, long lda,
                                           const float* B, long ldb, double* P, int scheme, int chunks) {
    Handle* h = reinterpret_cast<Handle*>(handle);
    if (!h) return EMUGEMM_STATUS_INVALID_HANDLE;
    if (M < 0 || N < 0 || K < 0) return EMUGEMM_STATUS_INVALID_SIZE;
    if (lda < (K > 0 ? K : 1) || ldb < (N > 0 ? N : 1)) return EMUGEMM_STATUS_INVALID_SIZE;
    if ((M > 0 && N > 0) && (!P || (K > 0 && (!A || !B)))) return EMUGEMM_STATUS_INVALID_POINTER;
    if (scheme == EMU_SCHEME_AUTO) return EMUGEMM_STATUS_INVALID_VALUE;
    emu::DeviceGuard g(h->device);
    return emu::dispatch(h, (emu_scheme_t)scheme, chunks, M, N, K, A, lda, B, ldb, nullptr, 0, P, N);
}

emugemm_status_t emugemm_reduce_f64(emugemm_handle_t handle, int M, int N, int G, const double* P, float* C) {
    Handle* h = reinterpret_cast<Handle*>(handle);
    if (!h) return EMUGEMM_STATUS_INVALID_HANDLE;
    if (M < 0 || N < 0 || G < 1) return EMUGEMM_STATUS_INVALID_SIZE;
    if ((long)M * N > 0 && (!P || !C)) return EMUGEMM_STATUS_INVALID_POINTER;
    emu::DeviceGuard g(h->device);
    return emu::from_cuda(emu::launch_reduce_f64(P, G, M, N, (long)M * N, C, N, nullptr, 0, h->stream));
}

int emugemm_fp32_groups_tile(int M, int N, long K, int chunks, int num_sms, int tile) {
    emu::Fp32GemmArgs f{};
    f.M = M; f.N = N; f.K = K; f.chunks = chunks < 1 ? 1 : chunks; f.num_sms = num_sms;
    f.lda = K; f.ldb = N;   // contiguous operands, as the caller's own rows would be
    f.bm = emu::fp32_tile_choice(M, N, K, f.chunks, tile);
    return emu::fp32_gemm_groups(f);
}

int emugemm_fp32_groups(int M, int N, long K, int chunks, int num_sms) {
    return emugemm_fp32_groups_tile(M, N, K, chunks, num_sms, emu::env_fp32_tile());
}

unsigned long long emugemm_kernel_launch_count(void) { return emu::g_launches.load(); }

emugemm_status_t emugemm_profile_begin(emugemm_handle_t handle) {
    Handle* h = reinterpret_cast<Handle*>(handle);
    if (!h) return EMUGEMM_STATUS_INVALID_HANDLE;
    emu::DeviceGuard g(h->device);
    emu::prof_clear(h);
    h->profiling = true;
    return EMUGEMM_STATUS_SUCCESS;
}

emugemm_status_t emugemm_profile_end(emugemm_handle_t handle, double* ms_by_kind, int* count_by_kind, int nkinds) {
    Handle* h = reinterpret_cast<Handle*>(handle);
    if (!h) return EMUGEMM_STATUS_INVALID_HANDLE;
    emu::DeviceGuard g(h->device);
    h->profiling = false;
    emugemm_status_t st = emu::sync_check(h);
    for (int k = 0; k < nkinds; ++k) {
        if (ms_by_kind) ms_by_kind[k] = 0.0;
        if (count_by_kind) count_by_kind[k] = 0;
    }
    for (int i = 0; i < h->prof_n; ++i) {
        const emu::ProfRec& r = h->prof[i];
        float ms = 0.f;
        if (r.kind < nkinds && cudaEventElapsedTime(&ms, (cudaEvent_t)r.a, (cudaEvent_t)r.b) == cudaSuccess) {
            if (ms_by_kind) ms_by_kind[r.kind] += ms;
            if (count_by_kind) count_by_kind[r.kind] += 1;
        }
    }
    emu::prof_clear(h);
    return st;
}

const char* emugemm_status_string(emugemm_status_t s) {
    switch (s) {
        case EMUGEMM_STATUS_SUCCESS: return "success";
        case EMUGEMM_STATUS_INVALID_HANDLE: return "invalid handle";
        case EMUGEMM_STATUS_NOT_IMPLEMENTED: return "not implemented";
        case EMUGEMM_STATUS_INVALID_POINTER: return "invalid pointer";
        case EMUGEMM_STATUS_INVALID_SIZE: return "invalid size";
        case EMUGEMM_STATUS_MEMORY_ERROR: return "memory error";
        case EMUGEMM_STATUS_INTERNAL_ERROR: return "internal error";
        case EMUGEMM_STATUS_INVALID_VALUE: return "invalid value";
        case EMUGEMM_STATUS_ARCH_MISMATCH: return "device is not sm_100";
        case EMUGEMM_STATUS_TIMEOUT: return "device wait timed out";
    }
    return "unknown status";
}

}  // extern "C"
