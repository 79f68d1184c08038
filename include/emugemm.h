/* emugemm.h - emulated-FP32 SGEMM for NVIDIA B200 (sm_100a) with an accuracy-contract planner.
 *
 * C ABI of the library libemugemm.so. Names, struct layouts, enum values and plan reason strings are
 * those of the emugemm C API (src/emugemm.h:37-99 of the emugemm-cdna project), so a caller written
 * against that header keeps working after two mechanical renames:
 *     rocblas_handle -> emugemm_handle_t      (opaque; created with emugemm_create_handle)
 *     rocblas_status -> emugemm_status_t      (same numeric values for the codes the API returns)
 * Defining EMUGEMM_ROCBLAS_COMPAT before including this header provides both spellings as typedefs.
 *
 * Semantics kept from the reference:
 *   - row-major, non-transposed: C(MxN) = A(MxK) * B(KxN), lda=K, ldb=N, ldc=N, alpha=1, beta=0;
 *   - A, B, C are DEVICE pointers owned by the caller;
 *   - the planner never returns a plan whose predicted error exceeds req->max_rel_err unless its reason
 *     starts with "TARGET UNREACHABLE" (it then still computes, with FP32_CHUNKED at the maximum chunk
 *     count, and returns success);
 *   - hints are in/out: a_absmax/b_absmax < 0 are measured, rho < 0 is estimated, and the measured
 *     values are written back.
 *
 * Error model (iid data, rho_ref(K) = 0.64*sqrt(K)):
 *     err(scheme, K, c, rho) = rho/rho_ref(K) * sqrt(floor_scheme^2 + a_scheme^2 * K/c)
 * The constants come from a named calibration table: "b200" (the default, measured on B200 with this
 * library's kernels) or "ref_mi250" (the reference's own constants, src/emugemm.cpp:16-23,92-93),
 * selectable with emugemm_set_model() so plans can be compared with the reference planner exactly.
 *
 * No CPU fallback exists: every compute entry point runs CUDA kernels built for sm_100a and fails with
 * EMUGEMM_STATUS_ARCH_MISMATCH on any other device.
 */
#ifndef EMUGEMM_H_
#define EMUGEMM_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- types kept from src/emugemm.h:37-71 ---------------------------------------------------------- */

typedef enum {
    EMU_SCHEME_AUTO = 0,
    EMU_SCHEME_NATIVE_FP32,
    EMU_SCHEME_FP32_CHUNKED,
    EMU_SCHEME_BF16X3,
    EMU_SCHEME_FP16X3,
    EMU_SCHEME_BF16X6       /* dominated; benchmarks only */
} emu_scheme_t;

typedef struct {
    double max_rel_err;   /* required normwise Frobenius relative error, e.g. 1e-5 */
    int    force_scheme;  /* emu_scheme_t; EMU_SCHEME_AUTO to let the dispatcher choose */
} emu_request_t;

typedef struct {
    float  a_absmax, b_absmax;  /* < 0 means "unknown, please scan" (an O(MK+KN) pass) */
    int    a_is_reused;         /* non-zero: A (same pointer, shape, lda) is unchanged since the previous
                                   emulated call on this handle, so its hi/lo split is reused */
    float  rho;                 /* cancellation ratio || |A||B| ||_F / ||AB||_F; < 0 = estimate it,
                                   0 = do not estimate and plan with the iid model */
    int    rho_probes;          /* Rademacher probes of the estimate; 0 -> 64 */
} emu_hints_t;

typedef struct {
    emu_scheme_t chosen;
    int          chunks;          /* c actually used */
    double       predicted_err;   /* from the model above */
    double       predicted_speedup;
    const char*  reason;          /* static string, never freed */
} emu_plan_t;

/* ---- status and handle (replace rocblas_status / rocblas_handle) -------------------------------------- */

typedef enum {
    EMUGEMM_STATUS_SUCCESS         = 0,   /* rocblas_status_success */
    EMUGEMM_STATUS_INVALID_HANDLE  = 1,   /* rocblas_status_invalid_handle */
    EMUGEMM_STATUS_NOT_IMPLEMENTED = 2,   /* rocblas_status_not_implemented */
    EMUGEMM_STATUS_INVALID_POINTER = 3,   /* rocblas_status_invalid_pointer */
    EMUGEMM_STATUS_INVALID_SIZE    = 4,   /* rocblas_status_invalid_size */
    EMUGEMM_STATUS_MEMORY_ERROR    = 5,   /* rocblas_status_memory_error */
    EMUGEMM_STATUS_INTERNAL_ERROR  = 6,   /* rocblas_status_internal_error */
    EMUGEMM_STATUS_INVALID_VALUE   = 11,  /* rocblas_status_invalid_value */
    EMUGEMM_STATUS_ARCH_MISMATCH   = 100, /* device is not sm_100 (no emugemm-cdna counterpart) */
    EMUGEMM_STATUS_TIMEOUT         = 101  /* a bounded device-side wait gave up; the context is intact */
} emugemm_status_t;

typedef struct emugemm_handle_s* emugemm_handle_t;

#ifdef EMUGEMM_ROCBLAS_COMPAT
typedef emugemm_status_t rocblas_status;
typedef emugemm_handle_t rocblas_handle;
#endif

/* Create a handle bound to the CURRENT CUDA device and the legacy default stream.
   Replaces rocblas_create_handle (the reference's harnesses call it before emugemm_init,
   bench/emugemm_test.cpp:64). Fails with ARCH_MISMATCH unless the device is compute capability 10.0. */
emugemm_status_t emugemm_create_handle(emugemm_handle_t* handle);
/* Frees the handle's workspace. Replaces rocblas_destroy_handle. */
emugemm_status_t emugemm_destroy_handle(emugemm_handle_t handle);
/* All work of the handle is enqueued on `stream` (a cudaStream_t; NULL = legacy default stream).
   Replaces rocblas_set_stream. */
emugemm_status_t emugemm_set_stream(emugemm_handle_t handle, void* stream);
/* Caps the handle's grow-only workspace; 0 = no cap. A call needing more returns MEMORY_ERROR. */
emugemm_status_t emugemm_set_workspace_limit(emugemm_handle_t handle, size_t bytes);

/* ---- functions kept from src/emugemm.h:77-99 ------------------------------------------------------------ */

/* Load the per-shape tile table (replaces the rocBLAS solution-index table, src/emugemm.cpp:107-128).
   Rows whose arch column does not match the live device ("sm_100a" on B200) are rejected and counted
   on stderr. A missing file runs with the built-in tile choice and still returns success. */
emugemm_status_t emugemm_init(const char* tune_csv_path);
void             emugemm_shutdown(void);

/* Decide only -- no GPU work (src/emugemm.cpp:216-282). */
emu_plan_t emugemm_plan(int M, int N, long K, const emu_request_t* req, const emu_hints_t* hints);

/* Row-major C = A*B on the handle's stream (src/emugemm.cpp:285-358). The call returns once the GEMM is
   enqueued; the absmax scan and rho estimate, when requested, synchronise the stream to read their
   results back to the host. */
emugemm_status_t emugemm_sgemm(emugemm_handle_t handle,
                               int M, int N, long K,
                               const float* A, const float* B, float* C,
                               const emu_request_t* req, emu_hints_t* hints,
                               emu_plan_t* out_plan);

double emugemm_model_err(emu_scheme_t s, long K, int chunks);          /* iid data (rho = rho_ref) */
double emugemm_model_err_rho(emu_scheme_t s, long K, int chunks, double rho);
/* Estimate rho on the device with `probes` Rademacher vectors (<= 0 -> 64). Returns < 0 on failure. */
double emugemm_estimate_rho(emugemm_handle_t h, int M, int N, long K,
                            const float* A, const float* B, int probes);
double emugemm_model_speed(emu_scheme_t s, int chunks);

/* ---- additions without an emugemm-cdna counterpart ------------------------------------------------------ */

/* Select the planner's constant table: "b200" (default) or "ref_mi250" (the reference constants, so that
   plans agree with the reference planner bit for bit). Returns INVALID_VALUE for an unknown name. */
emugemm_status_t emugemm_set_model(const char* name);
const char*      emugemm_get_model(void);

/* Device max |x| over n floats (the scan of src/emugemm.cpp:155-168), synchronous. */
emugemm_status_t emugemm_absmax(emugemm_handle_t h, const float* X, size_t n, float* out_absmax);

/* Debug split kernels for the bit-exact slice test (src/emugemm.cpp:143-148): element-wise, no scaling.
   bf16: hi = RNE_bf16(x), lo = RNE_bf16(x - hi).  fp16: hi = RNE_f16(x), lo = RNE_f16((x - hi)*2048).
   Outputs are n 16-bit words each (raw bit patterns). Asynchronous on the handle's stream. */
emugemm_status_t emugemm_split_bf16(emugemm_handle_t h, const float* X, size_t n,
                                    unsigned short* hi, unsigned short* lo);
emugemm_status_t emugemm_split_f16(emugemm_handle_t h, const float* X, size_t n,
                                   unsigned short* hi, unsigned short* lo);

/* Strided variant of emugemm_sgemm with explicit leading dimensions (lda >= K, ldb >= N, ldc >= N), used
   by the multi-GPU drivers to run on a panel of B or a block of rows of A in place. */
emugemm_status_t emugemm_sgemm_ex(emugemm_handle_t handle,
                                  int M, int N, long K,
                                  const float* A, long lda, const float* B, long ldb,
                                  float* C, long ldc,
                                  const emu_request_t* req, emu_hints_t* hints,
                                  emu_plan_t* out_plan);

/* emugemm_sgemm on HOST buffers (no emugemm-cdna counterpart; its callers copy to the device themselves):
   A (MxK), B (KxN), C (MxN) row-major in host memory, pinned (cudaHostAlloc / cudaHostRegister) for the
   copies to overlap. With every hint given (absmax >= 0, rho >= 0), B is copied to the device first in one piece,
   then A and C travel in row panels of about M/8 on two copy streams of the handle (every copy contiguous), each
   panel's GEMM starting as soon as its rows of A have landed and its rows of C leaving while later rows of A
   arrive.
   Hints that ask for measurements (or NULL hints) copy all of A and B first and then run emugemm_sgemm.
   C is identical to emugemm_sgemm's for BF16X3, FP16X3 and NATIVE_FP32; FP32_CHUNKED keeps the same FMA
   chains, but its FP64 chunk groups follow the panel's tile count. Asynchronous on the handle's stream: C is
   complete once that stream has been synchronized. The device copies of A, B, C live in the handle's
   workspace. */
emugemm_status_t emugemm_sgemm_host(emugemm_handle_t handle,
                                    int M, int N, long K,
                                    const float* A, const float* B, float* C,
                                    const emu_request_t* req, emu_hints_t* hints,
                                    emu_plan_t* out_plan);

/* K-split partial: P(MxN, FP64, ld=N) = A(MxK) * B(KxN) computed with `scheme` (BF16X3, FP16X3,
   NATIVE_FP32 or FP32_CHUNKED with `chunks`), written in FP64 so that partials from several devices can
   be summed exactly enough (ncclFloat64) before one final rounding to FP32. */
emugemm_status_t emugemm_sgemm_partial_f64(emugemm_handle_t handle,
                                           int M, int N, long K,
                                           const float* A, long lda, const float* B, long ldb,
                                           double* P, int scheme, int chunks);

/* C(MxN, FP32) = round(sum_{g<G} P[g]) for G FP64 partials of MxN each, summed in order g = 0..G-1. */
emugemm_status_t emugemm_reduce_f64(emugemm_handle_t handle, int M, int N, int G,
                                    const double* P, float* C);

/* Synchronise the handle's stream; returns TIMEOUT if a kernel of this handle gave up a bounded wait. */
emugemm_status_t emugemm_sync(emugemm_handle_t handle);

/* Peak rates of the handle's GPU, measured by micro-kernels run `reps` times each, interleaved round-robin,
   median kept (no function of the emugemm-cdna API; the counterpart of its bench/mfma_peak2.cpp probe).
   rates[EMU_PEAK_TC_*]: tcgen05 MMA TFLOP/s with operands resident in shared memory (bf16, fp16, tf32;
   FP32 accumulation); rates[EMU_PEAK_FFMA] / [EMU_PEAK_DFMA]: FP32 / FP64 FMA TFLOP/s; rates[EMU_PEAK_HBM_COPY]:
   device copy GB/s (read + written bytes). Fills the first min(n, EMU_PEAK_COUNT) entries; takes about
   reps * 4 ms and 2 GiB of device memory while it runs. */
enum {
    EMU_PEAK_TC_BF16 = 0,
    EMU_PEAK_TC_FP16 = 1,
    EMU_PEAK_TC_TF32 = 2,
    EMU_PEAK_FFMA = 3,
    EMU_PEAK_DFMA = 4,
    EMU_PEAK_HBM_COPY = 5,
    EMU_PEAK_COUNT = 6
};
emugemm_status_t emugemm_peak_probe(emugemm_handle_t handle, int reps, double* rates, int n);

/* emugemm_init with an explicit live arch string instead of the current device's, so the table parser
   and its arch rejection can be exercised without a GPU. */
emugemm_status_t emugemm_init_for_arch(const char* tune_csv_path, const char* live_arch);
/* Rows accepted by the last init, and the tile code the table gives a shape (0 = none within range).
   dtype: 0 fp32, 1 bf16, 2 fp16. */
int emugemm_tune_rows(void);
int emugemm_tune_lookup(int M, int N, long K, int dtype);

/* Number of FP64 partial groups the FP32_CHUNKED kernel uses for this shape on a GPU with num_sms SMs
   (fixes its summation order: chunk sums within a group in order, then the groups in order), for a handle
   created with the current environment (EMUGEMM_FP32_TILE read at this call). */
int emugemm_fp32_groups(int M, int N, long K, int chunks, int num_sms);

/* Per-handle kernel timing with CUDA events recorded on the handle's stream around each kernel class:
   0 tensor-core GEMM, 1 FP32 GEMM (+ FP64 reduce), 2 slice split, 3 absmax / exponent scans, 4 rho probe,
   5 FP64 reduce. profile_end synchronises and returns the summed milliseconds and launch counts of the
   first nkinds classes. */
emugemm_status_t emugemm_profile_begin(emugemm_handle_t handle);
emugemm_status_t emugemm_profile_end(emugemm_handle_t handle, double* ms_by_kind, int* count_by_kind,
                                     int nkinds);

/* bf16x3 emulated SGEMM that allocates nothing (no counterpart in the emugemm-cdna API). For callers that
   cannot let a library call cudaMalloc -- plugins inside an application whose own pool has reserved the
   device's memory, latency-critical paths that must not risk an allocation mid-run -- it computes the same
   product as emugemm_sgemm with force_scheme = EMU_SCHEME_BF16X3, with the slices of A and B held in a fixed
   64 MiB device array that every GPU loading the library keeps until the process exits. Limit:
   (Mp + Np) * Kp <= 16 Mi with Mp, Np, Kp = M, N, K rounded up to 128, 256, 64 (K: to 8192 beyond 16384;
   e.g. M = N = 2048, K <= 4096);
   larger sizes return EMUGEMM_STATUS_INVALID_SIZE. All calls on a device share the array: calls that overlap
   on the GPU race, so order them (e.g. one stream). The first call on a device looks the array up with
   cudaGetSymbolAddress; make that first call before any stream capture. Row-major, device pointers,
   asynchronous on `stream` (a cudaStream_t; NULL = legacy default stream), current device must be sm_100. */
emugemm_status_t emugemm_sgemm_bf16x3_noalloc(int M, int N, long K, const float* A, const float* B, float* C,
                                              void* stream);
/* Completion status of emugemm_sgemm_bf16x3_noalloc on the current device (no emugemm-cdna counterpart; the
   handle path reports the same event through emugemm_sync). Synchronises `stream`, then reads and clears the
   status word kept at the end of the static array: EMUGEMM_STATUS_TIMEOUT if a bounded device-side wait of any
   call since the previous query gave up (that call's C is incomplete), else SUCCESS. Allocates nothing. */
emugemm_status_t emugemm_noalloc_sync(void* stream);

/* Per-handle kernel choices (no emugemm-cdna counterpart; there rocBLAS picks the kernel). Every handle starts
   from the process environment, read when the handle is created: EMUGEMM_TC_KERNEL ("single", "pair", "fused",
   "fusea"), EMUGEMM_TC_SPLITK (a count >= 1) and EMUGEMM_FP32_TILE (16, 32, 64, 128, 3264); unset means 0, the tile
   table's choice and then the built-in one. A handle's setting changes only that handle's later calls. The K split
   count changes the order of the FP64 partial sums, so two handles with different settings may differ in the last
   bits of C; each setting on its own is deterministic. */
typedef enum {
    EMUGEMM_ATTR_TC_KERNEL = 0,   /* 0 auto, 1 single CTA, 2 CTA pair, 3 pair with the split fused in,
                                     4 pair with A split into TMEM (3, 4: bf16x3 only; fp16x3 runs 2) */
    EMUGEMM_ATTR_TC_SPLITK = 1,   /* 0 auto, n >= 1: K splits of the CTA-pair kernels */
    EMUGEMM_ATTR_FP32_TILE = 2,   /* 0 auto, 16 (16 x 32), 32, 64, 128, 3264 (32 x 64): tile of the FP32 SIMT
                                     kernel */
    EMUGEMM_ATTR_ROWS_PANELS = 3, /* emugemm_sgemm_rows: 0 = the modelled panel schedule, 1..16 = that many equal
                                     column panels of B (the same value on every rank) */
    EMUGEMM_ATTR_COMM_SMS = 4,    /* emugemm_sgemm_rows: SMs (even, 0..64) its tensor-core GEMMs leave free for the
                                     broadcast's NCCL kernels, so that neither waits for the other's SMs; C does
                                     not change (only the GEMMs' grid does) */
    EMUGEMM_ATTR_BCAST_NCCL = 5   /* emugemm_sgemm_rows: 0 = B travels by copy engines over peer memory (CUDA IPC,
                                     a tree of pulls; NCCL when the ranks cannot map each other's memory), 1 = NCCL
                                     broadcast (the same value on every rank) */
} emugemm_attr_t;
/* INVALID_VALUE for an unknown attribute or a value outside the ranges above. */
emugemm_status_t emugemm_set_attr(emugemm_handle_t handle, int attr, long value);
emugemm_status_t emugemm_get_attr(emugemm_handle_t handle, int attr, long* value);

/* emugemm_fp32_groups for an explicit FP32 tile code (0 = the tile table, then the built-in choice), as a handle
   with EMUGEMM_ATTR_FP32_TILE = tile uses it. */
int emugemm_fp32_groups_tile(int M, int N, long K, int chunks, int num_sms, int tile);

/* Testing hook for failure reporting (no emugemm-cdna counterpart). The next n launches of the single-CTA
   tensor-core kernel, from any entry point, make their MMA issuer wait before its second 128-K chunk on a
   barrier that nothing arrives on, with a 1 ms limit; the wait gives up and the kernel unwinds as after any
   timed-out wait (loads and MMAs in flight drained, TMEM freed, the timeout bit set in the error word), leaving
   that launch's C incomplete. The TMA-fed FP32 SIMT kernel (32 x 64 and 128 x 128 tiles) takes the hook the same
   way: its threads give up such a wait once the first k-blocks are issued, no further k-block is loaded, the loads in
   flight land before it exits, and its output is not meaningful. emugemm_sync (or emugemm_noalloc_sync) then
   returns EMUGEMM_STATUS_TIMEOUT. No fault, trap or hang is involved; n = 0 cancels. */
void emugemm_test_stall_next_launches(int n);

/* ---- several GPUs of one node: one process (and one handle) per GPU, NCCL between them ---------------------------
   No emugemm-cdna counterpart (the reference runs on one GPU); these are the two partitioned forms of its benchmark
   set. The library makes its own NCCL communicator and opens libnccl.so.2 at run time (the copy already loaded in
   the process, if any). Every rank calls the same entry points in the same order with the same M, N, K, root,
   request, hints and attributes; the calls are collective. */

/* 128 bytes (an ncclUniqueId) to be made on one rank and passed to every rank's emugemm_comm_init. */
emugemm_status_t emugemm_comm_unique_id(void* id_out);
/* Joins the handle to a communicator of `nranks` ranks (blocks until all ranks have joined). max_ctas > 0 caps the
   CTAs NCCL uses per collective (they share the SMs with the GEMMs); 0 = NCCL's choice. */
emugemm_status_t emugemm_comm_init(emugemm_handle_t handle, int nranks, int rank, const void* id, int max_ctas);
emugemm_status_t emugemm_comm_destroy(emugemm_handle_t handle);
/* The rows of an M-row product that this rank holds in emugemm_sgemm_rows: [row0, row0 + rows), contiguous blocks in
   rank order, the first M % nranks ranks one row longer. */
emugemm_status_t emugemm_comm_rows(emugemm_handle_t handle, int M, int* row0, int* rows);
/* The K range [k0, k0 + klen) this rank holds in emugemm_sgemm_ksplit: blocks of 64 values of K dealt like rows. */
emugemm_status_t emugemm_comm_krange(emugemm_handle_t handle, long K, long* k0, long* klen);

/* C = A * B (M x N x K) with the rows of A and C split over the ranks (emugemm_comm_rows) and B on `root`.
   A_local, C_local: this rank's rows (device, lda >= K, ldc >= N). B: K x N on the root (device, ldb >= N); on the
   other ranks a buffer that receives the root's B, or NULL. B travels in column panels over NCCL on a stream of the
   handle, each panel's GEMM starting as soon as it has arrived; A's slices are made once, while the first panel is
   on its way. Hints are those of emugemm_sgemm, agreed on by the ranks: a_absmax < 0 is the maximum over all row
   blocks, b_absmax < 0 the root's scan, rho < 0 the Hutchinson estimate of the whole product (all of B first, then
   each rank's sums over its rows added up). The plan is emugemm_plan of the whole product, the same on every rank,
   and every panel runs the tensor-core kernel and K split chosen for the whole product, so each rank's C rows equal
   those rows of the single-GPU emugemm_sgemm of the whole product bit for bit, whatever the number of ranks (BF16X3,
   FP16X3, NATIVE_FP32). Returns INVALID_VALUE without a communicator. Asynchronous on the handle's stream. */
emugemm_status_t emugemm_sgemm_rows(emugemm_handle_t handle, int M, int N, long K, const float* A_local, long lda,
                                    float* B, long ldb, float* C_local, long ldc, int root,
                                    const emu_request_t* req, emu_hints_t* hints, emu_plan_t* out_plan);
/* C = A * B with K split over the ranks (emugemm_comm_krange): A_local = A[:, k0:k0+klen] (M x klen, lda >= klen),
   B_local = B[k0:k0+klen, :] (klen x N). Each rank computes its partial product with `scheme` (and `chunks` for
   FP32_CHUNKED) in FP64, NCCL sums the partials in FP64, and one rounding gives C (M x N, ldc) on `root`, or on every
   rank when root = -1. Asynchronous on the handle's stream. */
emugemm_status_t emugemm_sgemm_ksplit(emugemm_handle_t handle, int M, int N, long K, const float* A_local, long lda,
                                      const float* B_local, long ldb, float* C, long ldc, int root, int scheme,
                                      int chunks);
/* The column panels [n0[i], n1[i]) emugemm_sgemm_rows uses for this product (up to `max` of them); returns their
   count. forced = EMUGEMM_ATTR_ROWS_PANELS. No GPU work. */
int emugemm_rows_panels(int M, int nranks, int N, long K, int num_sms, int forced, int* n0, int* n1, int max);

/* Number of kernels this library launched since the process started (all handles). */
unsigned long long emugemm_kernel_launch_count(void);

/* Human-readable name of a status code (static string). */
const char* emugemm_status_string(emugemm_status_t s);

#ifdef __cplusplus
}
#endif

#endif /* EMUGEMM_H_ */
