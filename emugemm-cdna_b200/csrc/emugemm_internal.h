// emugemm_internal.h - declarations shared by the host and kernel translation units of libemugemm.
#pragma once

#include "../../include/emugemm.h"

#include <cstddef>
#include <cstdint>

namespace emu {

// ---------------------------------------------------------------------------------------------------
// model.cpp
struct ChunkStep { int c_max; double cost; };

struct ModelConsts {
    const char* name;
    double a_fp32, a_lowp, a_fp16x3;
    double floor_bf16x3, floor_fp16x3, floor_bf16x6;
    double spd_bf16x3, spd_fp16x3, spd_bf16x6;
    float fp16_max, fp16_min;          // fp16 "range safe" test: min < absmax < max
    const ChunkStep* chunk_steps;
    int n_chunk_steps;
    double chunk_cost_beyond;
    int max_chunks;
    double hbm_bps, fp32_flops;
    double ovh_native, ovh_chunked, ovh_emulated, ovh_fp16x3;   // bytes per input element
    double rho_ref_coef;
    double rho_factor_min;   // lower clamp of rho/rho_ref(K); 0 = none (the reference's model)
};

const ModelConsts& model();
bool set_model_by_name(const char* name);
double chunk_cost(const ModelConsts& m, int c);
double model_err(const ModelConsts& m, emu_scheme_t s, long K, int c);
double model_err_rho(const ModelConsts& m, emu_scheme_t s, long K, int c, double rho);
double model_speed(const ModelConsts& m, emu_scheme_t s, int c);
emu_plan_t plan(const ModelConsts& m, int M, int N, long K, const emu_request_t* req,
                const emu_hints_t* hints);

extern const char* const kReasonUnreachable;
extern const char* const kReasonSlower;
extern const char* const kReasonFp16;
extern const char* const kReasonBf16;
extern const char* const kReasonChunked;
extern const char* const kReasonNative;

// ---------------------------------------------------------------------------------------------------
// tune.cpp: per-shape tile table
struct TileChoice {
    int tc_variant;     // tensor-core kernel: 0 = built-in choice, 1 = single-CTA, 2 = CTA pair (cta_group::2),
                        // 3 = CTA pair with the split fused in, 4 = CTA pair with A split into TMEM in the
                        // kernel and B pre-split (3 and 4: bf16x3 only)
    int fp32_bm;        // FP32 SIMT tile: 0 = auto, else a code of fp32_tile_code_ok
};
TileChoice lookup_tile(int M, int N, long K, int dtype /*0 fp32, 1 bf16, 2 fp16*/);

// ---------------------------------------------------------------------------------------------------
// Device-side error word: kernels OR these bits into the handle's mapped error word when a bounded wait
// gives up; the host reads it after synchronising.
enum : unsigned {
    kErrTimeoutProducer = 1u,
    kErrTimeoutMma = 2u,
    kErrTimeoutEpilogue = 4u,
    kErrTimeoutConvert = 8u,
    kErrTmemAlloc = 16u,
    kErrTimeoutComm = 32u,          // a wait for another GPU's flag in emugemm_sgemm_rows gave up
    kErrTimeoutFp32 = 64u,          // a wait for a TMA k-block in the FP32 SIMT kernel gave up
};

// Workspace slots of a handle (grow-only, freed with the handle).
enum WsSlot {
    kWsSplitA0 = 0, kWsSplitA1, kWsSplitB0, kWsSplitB1,
    kWsScaleA, kWsScaleB,
    kWsF64Acc,
    kWsRhoT1, kWsRhoT2, kWsRhoPart,
    kWsScalar,
    kWsHostA, kWsHostB, kWsHostC,   // device copies of the operands of emugemm_sgemm_host
    kWsSplitK,                      // FP64 partial planes of the split-K tensor-core GEMM
    kWsCommB,                       // emugemm_sgemm_rows: B's column panels as broadcast, panel after panel
    kWsCommP,                       // emugemm_sgemm_ksplit: the FP64 partial product and its sum over ranks
    // bank 1 of the per-product scratch (Handle::bank), for a second panel GEMM running beside the first
    kWsSplitB0b, kWsSplitB1b, kWsScaleBb, kWsSplitKb, kWsF64Accb,
    kWsCount
};

// emugemm_sgemm_host: column panels of B and C streamed over PCIe, at most this many per call.
constexpr int kMaxHostPanels = 16;

// Kernel classes timed by the optional per-handle profiler (CUDA events on the handle's stream).
enum ProfKind { kProfTcGemm = 0, kProfFp32Gemm, kProfSplit, kProfScan, kProfRho, kProfReduce, kProfCount };

struct ProfRec { void* a; void* b; int kind; };   // cudaEvent_t pair

struct Handle {
    int device = 0;
    void* stream = nullptr;         // cudaStream_t
    int num_sms = 0;
    size_t ws_limit = 0;            // 0 = no cap
    void* ws[kWsCount] = {};
    size_t ws_size[kWsCount] = {};
    unsigned* err_host = nullptr;   // mapped pinned word
    unsigned* err_dev = nullptr;
    bool profiling = false;
    ProfRec* prof = nullptr;        // growable array of event pairs
    int prof_n = 0, prof_cap = 0;
    // Identity of the A operand whose slices (and fp16 row exponents) the split workspace currently holds, so
    // a call with hints->a_is_reused can skip re-splitting an unchanged A (src/emugemm.h:53 of emugemm-cdna).
    struct ASplitKey {
        const float* A = nullptr; int M = 0; long K = 0, lda = 0; int kind = -1; long Mp = 0, Kp = 0;
        const void* ws0 = nullptr; const void* ws1 = nullptr; const void* rexp = nullptr;
    } a_key;
    // Kernel choices (emugemm_set_attr; defaults from the environment when the handle is created): tensor-core kernel
    // code (0 auto), K splits of the CTA-pair kernels (0 auto), FP32 SIMT tile code (0 auto).
    int tc_kernel = 0, tc_splitk = 0, fp32_tile = 0;
    // emugemm_sgemm_host: while its column panels run, the tensor-core kernel and K split count chosen for the whole
    // product (0: choose per call), so that the panels round like the single call would.
    int pin_tc_code = 0, pin_splits = 0;
    // emugemm_sgemm_host: copy streams (H2D, D2H) and events, created on first use.
    void* copy_in = nullptr;
    void* copy_out = nullptr;
    void* host_ev[2 * kMaxHostPanels + 2] = {};
    // multi-GPU state (multigpu.cpp): NCCL communicator, its stream and events; null until emugemm_comm_init
    void* mg = nullptr;
    int rows_panels = 0;            // EMUGEMM_ATTR_ROWS_PANELS: 0 = modelled schedule, n = n equal panels
    int comm_sms = 0;               // EMUGEMM_ATTR_COMM_SMS: SMs the GEMMs of emugemm_sgemm_rows leave to NCCL
    int tc_grid_sms = 0;            // while > 0: grid bound of the tensor-core kernels (set by emugemm_sgemm_rows)
    int bank = 0;                   // 1: the per-product B scratch comes from the bank-1 slots (two GEMMs at once)
    int bcast_nccl = 0;             // EMUGEMM_ATTR_BCAST_NCCL: 1 = B by NCCL broadcast, 0 = copy engines (peer memory)
};

// Workspace slot of the current bank: the scratch a product writes besides A's slices (B's slices and column
// exponents, split-K planes, FP64 chunk groups) is doubled, so that two panel GEMMs can run on two streams at once.
inline int bank_slot(const Handle* h, int slot) {
    if (!h->bank) return slot;
    switch (slot) {
        case kWsSplitB0: return kWsSplitB0b;
        case kWsSplitB1: return kWsSplitB1b;
        case kWsScaleB: return kWsScaleBb;
        case kWsSplitK: return kWsSplitKb;
        case kWsF64Acc: return kWsF64Accb;
        default: return slot;
    }
}

// Profiler scope: records an event before and after the launches inside it when the handle profiles.
struct ProfScope {
    Handle* h; int kind; ProfRec* rec = nullptr;
    ProfScope(Handle* h_, int kind_);
    ~ProfScope();
};

void* ws_get(Handle* h, int slot, size_t bytes);
void count_launch(unsigned n = 1);
// Testing hook (emugemm_test_stall_next_launches): true for each of the next n launches of a kernel that has one (the
// single-CTA tensor-core kernel, the TMA-fed FP32 kernel), which then gives up a 1 ms wait on a barrier nothing
// arrives on.
bool take_test_stall();

// ---------------------------------------------------------------------------------------------------
// api.cpp internals shared with multigpu.cpp
struct DeviceGuard {   // the handle's device current for the scope, the caller's restored afterwards
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int dev);
    ~DeviceGuard();
};
emugemm_status_t from_cuda(int e);
emugemm_status_t sync_check(Handle* h);
emugemm_status_t absmax(Handle* h, const float* X, long rows, long cols, long ld, float* out);
bool rho_sums(Handle* h, int M, int N, long K, const float* A, long lda, const float* B, long ldb, int P,
              double v[2]);
long round_up(long x, long m);
int tc_split_count(long Mp, long Np, long K, int num_sms, int forced);
int tc_kernel_choice(Handle* h, int M, int N, long K, bool fp16);
// One product (or panel) with scheme s into C (FP32) or C64 (FP64); a_reused: A's slices held by the handle are valid.
emugemm_status_t dispatch(Handle* h, emu_scheme_t s, int chunks, int M, int N, long K, const float* A, long lda,
                          const float* B, long ldb, float* C, long ldc, double* C64, long ldc64, bool a_reused = false);
// Make A's slices (and fp16x3 row exponents) for later dispatch calls with a_reused, sizing the B slots for panels of
// width N; nothing for the FP32 schemes and for the kernels that split A themselves.
emugemm_status_t prepare_a(Handle* h, emu_scheme_t s, int M, int N, long K, const float* A, long lda);
// multigpu.cpp: releases the handle's communicator, streams and events
void multigpu_release(Handle* h);

// ---------------------------------------------------------------------------------------------------
// Kernel launchers (return a cudaError_t as int; 0 = success).

// k_peak.cu: rates[0..5] = tcgen05 bf16 / fp16 / tf32 TFLOP/s, FFMA, DFMA TFLOP/s, copy GB/s (medians of
// `reps` interleaved runs). Returns a cudaError_t, or -1 when a tensor-core wait timed out.
int run_peak_probe(int reps, int num_sms, unsigned* err_dev, const unsigned* err_host, void* stream,
                   double* rates);

// k_split.cu
int launch_split_bf16(const float* X, size_t n, uint16_t* hi, uint16_t* lo, void* stream);
int launch_split_f16(const float* X, size_t n, uint16_t* hi, uint16_t* lo, void* stream);
int launch_absmax(const float* X, long rows, long cols, long ld, float* out, void* stream);
// Row exponents of A (MxK) / column exponents of B (KxN) for the scaled fp16 split: e such that
// max|x| * 2^-e < 2^15 (0 for an all-zero row or column).
int launch_row_exponents(const float* A, int M, long K, long lda, int* e_out, void* stream);
int launch_col_exponents(const float* B, long K, int N, long ldb, int* e_out, unsigned* scratch,
                         void* stream);
// Pre-split into K-major 16-bit slices: rows x Kp (zero padded to rows_p x Kp).
// kind 0 = bf16, 1 = scaled fp16 (hi = RNE(x*2^-e), lo = RNE((x*2^-e - hi)*2048)).
// Slices are stored in K panels, [Kp / KP][rows][KP] 16-bit values, so that the rows one TMA box touches sit
// 2 * KP bytes apart whatever K is. With plain rows of Kp values the bf16x3 kernel at M = N = 4096 ran at 43 % of
// tensor peak for K = 2^20 (rows 2 MB apart) against 72 % for K = 2^19. KP = Kp up to kSlicePanelMax values of
// K (one panel, plain rows), kSlicePanel beyond, with Kp rounded up to whole panels.
constexpr long kSlicePanel = 8192, kSlicePanelMax = 16384;
inline long slice_kp(long K) {
    const long k = (K + 63) / 64 * 64;
    return k <= kSlicePanelMax ? k : (k + kSlicePanel - 1) / kSlicePanel * kSlicePanel;
}
inline long slice_panel(long Kp) { return Kp <= kSlicePanelMax ? Kp : kSlicePanel; }
int launch_split_rows(const float* A, int M, long K, long lda, int Mp, long Kp, long KP, int kind,
                      const int* row_exp, uint16_t* hi, uint16_t* lo, void* stream);
// B (KxN, ldb) -> transposed K-major slices Np x Kp.
int launch_split_cols(const float* B, long K, int N, long ldb, int Np, long Kp, long KP, int kind,
                      const int* col_exp, uint16_t* hi, uint16_t* lo, void* stream);

// k_tc_gemm.cu: tensor-core 3-product GEMM over pre-split K-major slices.
struct TcGemmArgs {
    const uint16_t* a_hi; const uint16_t* a_lo;   // Mp x Kp
    const uint16_t* b_hi; const uint16_t* b_lo;   // Np x Kp
    int M, N, Mp, Np; long Kp;
    long KP;                                       // K panel width (slice_panel(Kp))
    float* C; long ldc;
    double* C64; long ldc64;                       // when non-null: write FP64 instead of C
    int fp16;                                      // 0 = bf16x3, 1 = scaled fp16x3
    const int* row_exp; const int* col_exp;        // fp16x3 only
    unsigned* err;
    int num_sms;
    // CTA-pair kernel only: K split into `splits` ranges of whole k-blocks (every range non-empty); each writes an
    // FP64 partial plane part64[s] (M x N, ld N) instead of C, and the caller sums the planes in order.
    int splits = 1;
    double* part64 = nullptr;
    long K = 0;          // the true K (split boundaries are 128-K chunks of it); 0: Kp
};
int launch_tc_gemm(const TcGemmArgs& a, void* stream);
int tc_gemm_bn(int fp16);   // output tile width of the bf16x3 (0) / fp16x3 (1) kernel
// k_tc_gemm2.cu: the same product on CTA pairs (cta_group::2); needs Mp % 256 == 0.
int launch_tc_gemm_pair(const TcGemmArgs& a, void* stream);
int tc_pair_bn(int fp16);
// k_tc_fused.cu: bf16x3 / fp16x3 with the split fused into the CTA-pair GEMM (FP32 tiles by TMA, no slices in HBM).
// splits / part64: K splits on 128-K chunk boundaries with FP64 partial planes, as for launch_tc_gemm_pair.
// Returns cudaErrorNotSupported unless lda, ldb are multiples of 4 and A, B are 16-byte aligned.
// fp16: the scaled fp16x3 form (row_exp / col_exp: the exponents of launch_row_exponents / launch_col_exponents),
// bit-identical to launch_tc_gemm_pair over the pre-split fp16 slices.
int launch_tc_fused(const float* A, long lda, const float* B, long ldb, int M, int N, long K, float* C, long ldc,
                    double* C64, long ldc64, unsigned* err, int num_sms, void* stream, int splits = 1,
                    double* part64 = nullptr, int fp16 = 0, const int* row_exp = nullptr,
                    const int* col_exp = nullptr);
// k_tc_fused_a.cu: bf16x3 on CTA pairs with A split in the kernel into TMEM and B's slices pre-split (b_hi, b_lo:
// Np x Kp in K panels of KP, Np a multiple of tc_fused_a_bn()). cudaErrorNotSupported unless lda % 4 == 0 and A is
// 16-byte aligned.
int tc_fused_a_bn();
int launch_tc_fused_a(const float* A, long lda, const uint16_t* b_hi, const uint16_t* b_lo, int M, int N, int Np,
                      long K, long Kp, long KP, float* C, long ldc, double* C64, long ldc64, unsigned* err,
                      int num_sms, void* stream);

// k_fp32_gemm.cu: FP32 SIMT GEMM with K-chunks summed in FP64.
struct Fp32GemmArgs {
    const float* A; long lda;
    const float* B; long ldb;
    float* C; long ldc;
    double* C64; long ldc64;     // when non-null: write FP64 sums here instead of C
    int M, N; long K;
    int chunks;
    double* ws64;                // G x M x N FP64 partials when G > 1
    int num_sms;
    int bm;                      // 0 = auto, else a tile code (fp32_tile_code_ok)
    unsigned* err = nullptr;     // device error word for the bounded waits (may be null)
};
// FP32 SIMT tile codes: 32, 64, 128 (square tiles), 16 (16 x 32, k_fp32_pipe_cp) and 3264 (32 x 64, k_fp32_pipe).
inline bool fp32_tile_code_ok(long t) {
    return t == 16 || t == 32 || t == 64 || t == 128 || t == 3264;
}
int fp32_gemm_groups(const Fp32GemmArgs& a);   // G chosen for this shape
size_t fp32_gemm_ws_bytes(const Fp32GemmArgs& a);
int launch_fp32_gemm(const Fp32GemmArgs& a, void* stream);
int launch_reduce_f64(const double* P, int G, int M, int N, long ldp, float* C, long ldc,
                      double* C64, long ldc64, void* stream);

// k_rho.cu: Hutchinson estimate of rho; out2[0] = sum |A|(|B| Omega) squared, out2[1] = sum (A B Omega)^2.
size_t rho_ws_bytes(int M, int N, long K, int P, int sms);
int launch_rho(const float* A, long lda, const float* B, long ldb, int M, int N, long K, int P, void* ws, int sms,
               double* out2, void* stream);

}  // namespace emu
