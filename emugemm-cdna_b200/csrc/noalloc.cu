// noalloc.cu - bf16x3 emulated SGEMM for callers that cannot allocate device memory.
//
// emugemm_sgemm needs scratch memory for the hi/lo bf16 slices of A and B, and takes it from a grow-only
// workspace that it allocates with cudaMalloc. Some callers cannot let a library do that: plugins inside an
// application whose own memory pool has reserved the device's memory (a cudaMalloc there fails or
// fragments that pool), and latency-critical paths that must not pay for, or risk the failure of, an
// allocation in the middle of a run. emugemm_sgemm_bf16x3_noalloc serves them: it computes the same bf16x3
// product with the same kernels, but its slices live in a fixed file-scope device array.
//
// Properties a caller must know:
//   - The scratch array holds 64 MiB on every GPU that loads this library, from the moment the module is
//     loaded (at the latest, this entry point's first call on the device) until the process exits. It
//     fits (Mp + Np) * Kp <= 16 Mi, where Mp = M rounded up to 128, Np = N rounded up to 256 and
//     Kp = K rounded up to 64, or to 8192 beyond K = 16384 (for example M = N = 2048 with K up to 4096);
//     larger problems are rejected
//     with EMUGEMM_STATUS_INVALID_SIZE and a message on stderr.
//   - Every call on a device uses the same array. Calls whose kernels overlap on the GPU (different
//     streams, or different host threads without ordering) race on it and produce wrong results; callers
//     must order them, for example by issuing them all on one stream.
//   - The array keeps the previous call's contents. Each call rewrites every slice element the GEMM reads
//     (zero padding included), so no stale slice value reaches the result.
//   - A bounded device-side wait that gives up (the kernel then unwinds and leaves C incomplete) sets a bit
//     in a status word at the end of the array. The call itself returns before its kernels run, so it
//     cannot report that; emugemm_noalloc_sync(stream) synchronises the stream, reads the word, clears it
//     and returns EMUGEMM_STATUS_TIMEOUT if any call since the previous query timed out. The word stays
//     set until it is read, so one query after several calls reports a timeout in any of them.
//   - The first call on a device resolves the array's device address with cudaGetSymbolAddress (once per
//     device, with that device current). That first call should come before any stream capture.
//   - The call is asynchronous on `stream` and allocates nothing: no cudaMalloc, cudaFree, host-pinned
//     allocation or allocating library routine.
#include "emugemm_internal.h"

#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

namespace emu {
namespace {
constexpr size_t kNoAllocScratchBytesDecl = size_t(64) << 20;
constexpr size_t kStatusBytesDecl = 256;
}  // namespace
}  // namespace emu

// File-scope scratch: 16-bit slices (A_hi, A_lo, B_hi, B_lo) followed by the device status word. In host code
// this name is only a host-side stand-in, not a device address: the address comes from
// cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[emu::kNoAllocScratchBytesDecl +
                                                                 emu::kStatusBytesDecl];

namespace emu {
namespace {

constexpr size_t kNoAllocScratchBytes = kNoAllocScratchBytesDecl;
constexpr size_t kStatusBytes = kStatusBytesDecl;   // status word of the tensor-core kernel (bounded waits)
constexpr int kMaxDevices = 64;

std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};
int g_num_sms[kMaxDevices] = {};

// Resolves (once per device, with that device current) the device address of the scratch array.
cudaError_t scratch_for_device(int dev, unsigned char** out, int* sms) {
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        int n = 0;
        e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        g_scratch_ptr[dev] = p;
        g_num_sms[dev] = n;
    }
    *out = static_cast<unsigned char*>(g_scratch_ptr[dev]);
    *sms = g_num_sms[dev];
    return cudaSuccess;
}

}  // namespace
}  // namespace emu

extern "C" emugemm_status_t emugemm_sgemm_bf16x3_noalloc(int M, int N, long K, const float* A, const float* B,
                                                         float* C, void* stream) {
    using namespace emu;
    if (M < 0 || N < 0 || K < 0) return EMUGEMM_STATUS_INVALID_SIZE;
    if (M == 0 || N == 0) return EMUGEMM_STATUS_SUCCESS;
    if (!C || (K > 0 && (!A || !B))) return EMUGEMM_STATUS_INVALID_POINTER;
    int dev = 0, major = 0, minor = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return EMUGEMM_STATUS_INTERNAL_ERROR;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
        return EMUGEMM_STATUS_INTERNAL_ERROR;
    if (major != 10 || minor != 0) return EMUGEMM_STATUS_ARCH_MISMATCH;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (K == 0) {
        return cudaMemset2DAsync(C, (size_t)N * 4, 0, (size_t)N * 4, (size_t)M, st) == cudaSuccess
                   ? EMUGEMM_STATUS_SUCCESS
                   : EMUGEMM_STATUS_INTERNAL_ERROR;
    }
    const int BN = tc_gemm_bn(0);
    const long Mp = round_up(M, 128), Np = round_up(N, BN), Kp = slice_kp(K), KP = slice_panel(Kp);
    const size_t need = (size_t)(Mp + Np) * (size_t)Kp * 2 /*slices*/ * 2 /*bytes*/;
    if (need > kNoAllocScratchBytes) {
        std::fprintf(stderr,
                     "emugemm_sgemm_bf16x3_noalloc: M=%d N=%d K=%ld needs %zu bytes of slices, above the %zu-byte "
                     "static scratch ((Mp + Np) * Kp must be <= %zu)\n",
                     M, N, K, need, kNoAllocScratchBytes, kNoAllocScratchBytes / 4);
        return EMUGEMM_STATUS_INVALID_SIZE;
    }
    unsigned char* base = nullptr;
    int sms = 0;
    if (scratch_for_device(dev, &base, &sms) != cudaSuccess) return EMUGEMM_STATUS_INTERNAL_ERROR;
    uint16_t* a_hi = reinterpret_cast<uint16_t*>(base);
    uint16_t* a_lo = a_hi + (size_t)Mp * Kp;
    uint16_t* b_hi = a_lo + (size_t)Mp * Kp;
    uint16_t* b_lo = b_hi + (size_t)Np * Kp;
    // sticky until emugemm_noalloc_sync reads it (zero when the module is loaded)
    unsigned* status = reinterpret_cast<unsigned*>(base + kNoAllocScratchBytes);
    int e = launch_split_rows(A, M, K, K, (int)Mp, Kp, KP, 0, nullptr, a_hi, a_lo, stream);
    if (!e) e = launch_split_cols(B, K, N, N, (int)Np, Kp, KP, 0, nullptr, b_hi, b_lo, stream);
    if (e) return EMUGEMM_STATUS_INTERNAL_ERROR;
    TcGemmArgs t;
    t.a_hi = a_hi; t.a_lo = a_lo; t.b_hi = b_hi; t.b_lo = b_lo;
    t.M = M; t.N = N; t.Mp = (int)Mp; t.Np = (int)Np; t.Kp = Kp; t.KP = KP;
    t.C = C; t.ldc = N; t.C64 = nullptr; t.ldc64 = 0;
    t.fp16 = 0;
    t.row_exp = nullptr; t.col_exp = nullptr;
    t.err = status;
    t.num_sms = sms;
    e = launch_tc_gemm(t, stream);
    if (e == (int)cudaErrorInvalidValue) return EMUGEMM_STATUS_INVALID_VALUE;
    return e ? EMUGEMM_STATUS_INTERNAL_ERROR : EMUGEMM_STATUS_SUCCESS;
}

extern "C" emugemm_status_t emugemm_noalloc_sync(void* stream) {
    using namespace emu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return EMUGEMM_STATUS_INTERNAL_ERROR;
    const cudaError_t se = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    unsigned char* base = nullptr;
    int sms = 0;
    if (scratch_for_device(dev, &base, &sms) != cudaSuccess) return EMUGEMM_STATUS_INTERNAL_ERROR;
    unsigned* status = reinterpret_cast<unsigned*>(base + kNoAllocScratchBytes);
    unsigned word = 0;
    // synchronous copies of one word between the static array and a host variable: nothing is allocated
    if (cudaMemcpy(&word, status, sizeof word, cudaMemcpyDeviceToHost) != cudaSuccess)
        return EMUGEMM_STATUS_INTERNAL_ERROR;
    if (word) {
        const unsigned zero = 0;
        if (cudaMemcpy(status, &zero, sizeof zero, cudaMemcpyHostToDevice) != cudaSuccess)
            return EMUGEMM_STATUS_INTERNAL_ERROR;
        std::fprintf(stderr, "emugemm_sgemm_bf16x3_noalloc: a device-side wait timed out (flags 0x%x)\n", word);
        return EMUGEMM_STATUS_TIMEOUT;
    }
    return se == cudaSuccess ? EMUGEMM_STATUS_SUCCESS : EMUGEMM_STATUS_INTERNAL_ERROR;
}
