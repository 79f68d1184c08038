// multigpu.cpp - the emulated SGEMM over the GPUs of one node: one process per GPU, NCCL between them.
//
// The reference runs one product on one GPU (src/emugemm.cpp:285-358); its benchmark set adds two partitioned forms
// for large products, both built here behind the same planner and kernels:
//   emugemm_sgemm_rows    row blocks of A (and C) on the ranks, B held by one rank and broadcast in column panels on
//                         a communication stream; the GEMM of panel j starts as soon as panel j has arrived, so the
//                         broadcast of later panels runs under the GEMMs of earlier ones. C equals the single-GPU
//                         emugemm_sgemm of the whole product bit for bit (its kernel and K split in every panel).
//   emugemm_sgemm_ksplit  K split over the ranks: every rank writes its partial product in FP64, NCCL sums the
//                         partials in FP64, one rounding to FP32 follows.
// NCCL is not linked: the library opens libnccl.so.2 when a communicator is first made, which resolves to the copy a
// host framework has already loaded, if any, so that the library and its caller use one NCCL. The communicator is
// the library's own (emugemm_comm_unique_id / emugemm_comm_init), so it never shares a stream or a sequence of
// collectives with the caller's.
//
// How B travels in emugemm_sgemm_rows. The panel GEMMs are persistent kernels with one CTA on every SM; NCCL's
// broadcast kernels need SMs of their own (about 27 GB/s per CTA measured), so they either wait for the GEMMs or take
// SMs from them. By default B therefore moves by COPY ENGINES over NVLink peer memory, which use no SM: every rank
// maps the staging buffers of the others (CUDA IPC, set up once per size), and the ranks form a binary tree rooted
// at `root`; the root copies B into its buffer in one piece, and each other rank pulls panel j from its parent's
// buffer into its own with one pitched cudaMemcpy2DAsync as soon as the parent has it, so every node sends B at
// most twice. Arrival and release are 32-bit sequence flags in device
// memory: one-warp kernels set them (a system-scope release store) and wait for them (bounded polls, which co-reside
// with the GEMM's CTAs on an SM); a wait that runs out sets the handle's timeout bit, so emugemm_sync reports it.
// The staging buffers alternate between two per call, and a rank refills one only after every rank has released
// the call that filled it last (which ranks pulled from it depended on that call's root). NCCL broadcasts remain the path when the ranks cannot map each other's memory, or on request.
#include "device_utils.cuh"
#include "emugemm_internal.h"

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

namespace emu {
namespace {

struct NcclApi {
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRankConfig) init_rank_config = nullptr;
    decltype(&ncclCommDestroy) destroy = nullptr;
    decltype(&ncclBroadcast) broadcast = nullptr;
    decltype(&ncclAllReduce) all_reduce = nullptr;
    decltype(&ncclReduce) reduce = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
    bool ok = false;
};

NcclApi g_nccl;
std::once_flag g_nccl_once;

const NcclApi* nccl() {
    std::call_once(g_nccl_once, [] {
        void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!lib) lib = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!lib) {
            std::fprintf(stderr, "emugemm: cannot open libnccl.so.2 (%s)\n", dlerror());
            return;
        }
        NcclApi& a = g_nccl;
        a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(lib, "ncclGetUniqueId"));
        a.init_rank_config = reinterpret_cast<decltype(a.init_rank_config)>(dlsym(lib, "ncclCommInitRankConfig"));
        a.destroy = reinterpret_cast<decltype(a.destroy)>(dlsym(lib, "ncclCommDestroy"));
        a.broadcast = reinterpret_cast<decltype(a.broadcast)>(dlsym(lib, "ncclBroadcast"));
        a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(dlsym(lib, "ncclAllReduce"));
        a.reduce = reinterpret_cast<decltype(a.reduce)>(dlsym(lib, "ncclReduce"));
        a.all_gather = reinterpret_cast<decltype(a.all_gather)>(dlsym(lib, "ncclAllGather"));
        a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(lib, "ncclGetErrorString"));
        a.ok = a.get_unique_id && a.init_rank_config && a.destroy && a.broadcast && a.all_reduce && a.reduce &&
               a.all_gather && a.error_string;
        if (!a.ok) std::fprintf(stderr, "emugemm: libnccl.so.2 lacks a needed entry point\n");
    });
    return g_nccl.ok ? &g_nccl : nullptr;
}

constexpr int kMaxRowPanels = 16;

struct Mg {
    ncclComm_t comm = nullptr;
    int rank = 0, size = 1;
    cudaStream_t stream = nullptr;                 // broadcasts of B's panels
    cudaStream_t stream2 = nullptr;                // every other panel GEMM, beside the handle's stream
    cudaEvent_t ev_start = nullptr, ev_done = nullptr, ev_a = nullptr, ev_join = nullptr;
    cudaEvent_t ev_panel[kMaxRowPanels] = {};
    void* small = nullptr;                         // 256 bytes: hint values agreed on by the ranks
    // copy-engine broadcast over peer memory
    int p2p = -1;                                  // -1 not yet tried, 0 unavailable (NCCL), 1 in use
    unsigned seq = 0;                              // emugemm_sgemm_rows calls so far (equal on every rank)
    size_t stage_bytes = 0;
    float* stage[2] = {};                          // this rank's staging buffers, mapped by the others
    unsigned* flags = nullptr;                     // [kFlagArrive + 16 b + j] arrivals, [kFlagRelease + c] releases
    std::vector<float*> peer_stage[2];             // the other ranks' staging buffers (by rank; null for this one)
    std::vector<unsigned*> peer_flags;
};

constexpr int kFlagArrive = 0;                     // + 16 * buffer + panel: the sequence number of the panel's call
constexpr int kFlagRelease = 32;                   // + rank: the last call whose panels that rank has pulled
constexpr int kMaxP2pRanks = 32;
constexpr size_t kFlagBytes = 4 * (kFlagRelease + kMaxP2pRanks);
constexpr unsigned long long kCommWaitNs = 10000000000ull;   // a peer that has not arrived within 10 s has failed

struct PeerFlags { unsigned* p[kMaxP2pRanks]; };

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Waits until flag[i] has reached `want` for every i < n except `skip` (sequence numbers compared modulo 2^32), all
// within limit_ns.
__global__ void k_wait_flags(const unsigned* flag, int n, int skip, unsigned want, unsigned* err,
                             unsigned long long limit_ns) {
    if (threadIdx.x != 0) return;
    const unsigned long long t0 = dev::globaltimer();
    for (int i = 0; i < n; ++i) {
        if (i == skip) continue;
        while ((int)(ld_acquire_sys(flag + i) - want) < 0) {
            if (dev::globaltimer() - t0 > limit_ns) {
                if (err) atomicOr(err, kErrTimeoutComm);
                return;
            }
            __nanosleep(200);
        }
    }
}

// Publishes `v` in *f.p[i] for every i < n that is not null, after every earlier operation of the stream (the copy
// it announces) has completed.
__global__ void k_set_flags(PeerFlags f, int n, unsigned v) {
    if (threadIdx.x != 0) return;
    __threadfence_system();
    for (int i = 0; i < n; ++i)
        if (f.p[i]) asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f.p[i]), "r"(v) : "memory");
}

int wait_flags(const unsigned* flag, int n, int skip, unsigned want, unsigned* err, cudaStream_t st) {
    k_wait_flags<<<1, 32, 0, st>>>(flag, n, skip, want, err, kCommWaitNs);
    count_launch();
    return (int)cudaGetLastError();
}

int set_flag(unsigned* flag, unsigned v, cudaStream_t st) {
    PeerFlags f{};
    f.p[0] = flag;
    k_set_flags<<<1, 32, 0, st>>>(f, 1, v);
    count_launch();
    return (int)cudaGetLastError();
}

void p2p_close(Mg* m) {
    for (int b = 0; b < 2; ++b) {
        for (float*& q : m->peer_stage[b])
            if (q) cudaIpcCloseMemHandle(q), q = nullptr;
        if (m->stage[b]) cudaFree(m->stage[b]), m->stage[b] = nullptr;
    }
    for (unsigned*& q : m->peer_flags)
        if (q) cudaIpcCloseMemHandle(q), q = nullptr;
    m->stage_bytes = 0;
}

Mg* mg_of(Handle* h) { return static_cast<Mg*>(h->mg); }

emugemm_status_t from_nccl(ncclResult_t r) {
    if (r == ncclSuccess) return EMUGEMM_STATUS_SUCCESS;
    const NcclApi* n = nccl();
    std::fprintf(stderr, "emugemm: NCCL error %d (%s)\n", (int)r, n ? n->error_string(r) : "?");
    return EMUGEMM_STATUS_INTERNAL_ERROR;
}

// Rows [r0, r1) of rank `rank` among `size`: contiguous blocks, the first M % size ranks one row longer.
void row_range(long M, int rank, int size, long* r0, long* r1) {
    const long base = M / size, extra = M % size;
    *r0 = rank * base + std::min<long>(rank, extra);
    *r1 = *r0 + base + (rank < extra ? 1 : 0);
}

// K range of rank `rank`: blocks of 64 values of K dealt like rows, so every rank's slices are whole k-blocks.
void k_range(long K, int rank, int size, long* k0, long* k1) {
    long b0, b1;
    row_range((K + 63) / 64, rank, size, &b0, &b1);
    *k0 = std::min(K, b0 * 64);
    *k1 = std::min(K, b1 * 64);
}

// Column panels of B for emugemm_sgemm_rows, in units of 256 columns (the CTA-pair tile width), chosen by a model of
// the pipeline so that every rank computes the same schedule from (M, ranks, N, K): panel j's broadcast ends at
// sum_{i<=j} (latency + bytes_i / bandwidth) on the communication stream; consecutive panel GEMMs run on two
// streams, so the CTAs of panel j+1 fill the SMs the last partial wave of panel j leaves idle, and the GPU works
// through the panels' tiles as one queue: panel j's tiles start once it has arrived and the tiles before it are
// done, and take tiles_j / SM pairs tile times, plus the split of the panel. A wide first panel leaves the GPU idle
// while it crosses NVLink; every further panel costs a collective's latency. The model's constants are round B200
// figures: 1.45 PFLOP/s of slice products over 74 SM pairs, 400 GB/s broadcast bandwidth, 25 us per collective,
// 5 TB/s for the split, 8 us per launch pair.
std::vector<std::pair<long, long>> rows_panels(long M, int size, long N, long K, int num_sms, int forced) {
    std::vector<std::pair<long, long>> out;
    const long nc = (N + 255) / 256;
    if (nc <= 0) return out;
    if (forced > 0 || size == 1) {
        const long np = std::min<long>(std::max(1, forced), std::min<long>(nc, kMaxRowPanels));
        const long per = (nc + np - 1) / np;
        for (long c = 0; c < nc; c += per) out.emplace_back(c * 256, std::min(N, (c + per) * 256));
        return out;
    }
    const long m_rows = (M + size - 1) / size;
    const long tiles_m = std::max<long>(1, (m_rows + 255) / 256);
    const long pairs = std::max(1, num_sms / 2);
    const double t_tile = 2.0 * 256 * 256 * (double)K * 3 / (1.45e15 / 74);
    const double col_bytes = (double)K * 256 * 4, bw = 400e9, lat = 25e-6, split = (double)K * 256 * 8 / 5e12,
                 launch = 8e-6;
    const int P = (int)std::min<long>(nc, kMaxRowPanels);
    const double inf = 1e30;
    // f[c][p]: earliest end of the GEMMs covering the first c tile columns with p panels (p broadcasts so far)
    std::vector<double> f((nc + 1) * (P + 1), inf);
    std::vector<int> from((nc + 1) * (P + 1), -1);
    auto at = [&](long c, int p) -> double& { return f[c * (P + 1) + p]; };
    at(0, 0) = 0.0;
    for (int p = 0; p < P; ++p)
        for (long c = 0; c < nc; ++c) {
            if (at(c, p) >= inf) continue;
            for (long w = 1; c + w <= nc; ++w) {
                const double arrive = (p + 1) * lat + (double)(c + w) * col_bytes / bw;
                const double work = (double)(tiles_m * w) / (double)pairs * t_tile;
                const double end = std::max(at(c, p), arrive + launch) + work + w * split + lat * 0.2;
                if (end < at(c + w, p + 1)) {
                    at(c + w, p + 1) = end;
                    from[(c + w) * (P + 1) + p + 1] = (int)c;
                }
            }
        }
    int best = 1;
    for (int p = 1; p <= P; ++p)
        if (at(nc, p) < at(nc, best)) best = p;
    std::vector<long> cuts;
    for (long c = nc; c > 0;) {
        cuts.push_back(c);
        c = from[c * (P + 1) + best];
        --best;
    }
    long c0 = 0;
    for (auto it = cuts.rbegin(); it != cuts.rend(); ++it) {
        out.emplace_back(c0 * 256, std::min(N, *it * 256));
        c0 = *it;
    }
    return out;
}

// Makes (or grows to `bytes`) the staging buffers of the copy-engine broadcast and maps every other rank's; collective:
// every rank calls it in the same emugemm_sgemm_rows call with the same size. Sets m->p2p to 1, or to 0 when some rank
// could not map the others' memory (all ranks then use NCCL broadcasts). On return every rank's earlier transfers of
// the old buffers have ended.
emugemm_status_t p2p_setup(Handle* h, Mg* m, const NcclApi* n, size_t bytes) {
    if (m->p2p == 0 || (m->p2p == 1 && m->stage_bytes >= bytes)) return EMUGEMM_STATUS_SUCCESS;
    if (m->size > kMaxP2pRanks) {
        m->p2p = 0;
        return EMUGEMM_STATUS_SUCCESS;
    }
    cudaStream_t cs = (cudaStream_t)h->stream;
    // every rank's device idle before any buffer is replaced: local sync, then a collective both ways
    if (cudaDeviceSynchronize() != cudaSuccess) return EMUGEMM_STATUS_INTERNAL_ERROR;
    struct Rec { cudaIpcMemHandle_t st[2], fl; int ok; char pad[256 - 3 * sizeof(cudaIpcMemHandle_t) - sizeof(int)]; };
    static_assert(sizeof(Rec) == 256, "record size");
    if (m->stage_bytes > 0) {
        // growing: the peers may still read this rank's old buffers until they, too, have drained
        int* d = static_cast<int*>(m->small);
        emugemm_status_t s = from_nccl(n->all_reduce(d, d, 1, ncclInt32, ncclSum, m->comm, cs));
        if (s == EMUGEMM_STATUS_SUCCESS) s = from_cuda((int)cudaStreamSynchronize(cs));
        if (s != EMUGEMM_STATUS_SUCCESS) return s;
    }
    Rec mine{};
    int ok = 1;
    const int P = m->size;
    p2p_close(m);
    if (!m->flags) {
        if (cudaMalloc(&m->flags, kFlagBytes) != cudaSuccess || cudaMemset(m->flags, 0, kFlagBytes) != cudaSuccess) {
            cudaGetLastError();
            m->flags = nullptr;
            ok = 0;
        }
    }
    for (int b = 0; b < 2 && ok; ++b) {
        void* q = nullptr;
        if (cudaMalloc(&q, bytes) != cudaSuccess) {
            cudaGetLastError();
            ok = 0;
            break;
        }
        m->stage[b] = static_cast<float*>(q);
    }
    if (ok)
        ok = cudaIpcGetMemHandle(&mine.st[0], m->stage[0]) == cudaSuccess &&
             cudaIpcGetMemHandle(&mine.st[1], m->stage[1]) == cudaSuccess &&
             cudaIpcGetMemHandle(&mine.fl, m->flags) == cudaSuccess;
    cudaGetLastError();
    mine.ok = ok;
    void* dev = nullptr;
    if (cudaMalloc(&dev, (size_t)(P + 1) * sizeof(Rec)) != cudaSuccess) {
        cudaGetLastError();
        return EMUGEMM_STATUS_MEMORY_ERROR;
    }
    std::vector<Rec> all(P);
    emugemm_status_t s = from_cuda((int)cudaMemcpy(dev, &mine, sizeof mine, cudaMemcpyHostToDevice));
    if (s == EMUGEMM_STATUS_SUCCESS)
        s = from_nccl(n->all_gather(dev, static_cast<char*>(dev) + sizeof(Rec), sizeof(Rec), ncclUint8, m->comm, cs));
    if (s == EMUGEMM_STATUS_SUCCESS)
        s = from_cuda((int)cudaMemcpyAsync(all.data(), static_cast<char*>(dev) + sizeof(Rec), P * sizeof(Rec),
                                           cudaMemcpyDeviceToHost, cs));
    if (s == EMUGEMM_STATUS_SUCCESS) s = from_cuda((int)cudaStreamSynchronize(cs));
    if (s != EMUGEMM_STATUS_SUCCESS) {
        cudaFree(dev);
        return s;
    }
    for (int r = 0; r < P; ++r) ok = ok && all[r].ok;
    for (int b = 0; b < 2; ++b) m->peer_stage[b].assign(P, nullptr);
    m->peer_flags.assign(P, nullptr);
    for (int r = 0; r < P && ok; ++r) {
        if (r == m->rank) continue;
        void* q[3] = {};
        const cudaIpcMemHandle_t* hs[3] = {&all[r].st[0], &all[r].st[1], &all[r].fl};
        for (int i = 0; i < 3 && ok; ++i)
            if (cudaIpcOpenMemHandle(&q[i], *hs[i], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                cudaGetLastError();
                ok = 0;
            }
        m->peer_stage[0][r] = static_cast<float*>(q[0]);
        m->peer_stage[1][r] = static_cast<float*>(q[1]);
        m->peer_flags[r] = static_cast<unsigned*>(q[2]);
    }
    // every rank must take the same path: the minimum of the ranks' outcomes
    int* d = static_cast<int*>(dev);
    s = from_cuda((int)cudaMemcpy(d, &ok, sizeof ok, cudaMemcpyHostToDevice));
    if (s == EMUGEMM_STATUS_SUCCESS) s = from_nccl(n->all_reduce(d, d, 1, ncclInt32, ncclMin, m->comm, cs));
    if (s == EMUGEMM_STATUS_SUCCESS) s = from_cuda((int)cudaMemcpyAsync(&ok, d, sizeof ok, cudaMemcpyDeviceToHost, cs));
    if (s == EMUGEMM_STATUS_SUCCESS) s = from_cuda((int)cudaStreamSynchronize(cs));
    cudaFree(dev);
    if (s != EMUGEMM_STATUS_SUCCESS) return s;
    if (!ok) {
        p2p_close(m);
        m->p2p = 0;
        std::fprintf(stderr, "emugemm: the ranks cannot map each other's memory; B travels by NCCL broadcast\n");
        return EMUGEMM_STATUS_SUCCESS;
    }
    m->stage_bytes = bytes;
    m->p2p = 1;
    return EMUGEMM_STATUS_SUCCESS;
}

bool is_tc(emu_scheme_t s) {
    return s == EMU_SCHEME_BF16X3 || s == EMU_SCHEME_BF16X6 || s == EMU_SCHEME_FP16X3;
}

}  // namespace

void multigpu_release(Handle* h) {
    Mg* m = mg_of(h);
    if (!m) return;
    if (m->stream) cudaStreamSynchronize(m->stream);
    const NcclApi* n = nccl();
    if (m->comm && n) n->destroy(m->comm);
    cudaDeviceSynchronize();   // no copy from or to a mapped buffer in flight
    p2p_close(m);
    if (m->flags) cudaFree(m->flags);
    for (cudaEvent_t e : m->ev_panel)
        if (e) cudaEventDestroy(e);
    if (m->ev_start) cudaEventDestroy(m->ev_start);
    if (m->ev_done) cudaEventDestroy(m->ev_done);
    if (m->stream) cudaStreamDestroy(m->stream);
    if (m->stream2) cudaStreamDestroy(m->stream2);
    if (m->ev_a) cudaEventDestroy(m->ev_a);
    if (m->ev_join) cudaEventDestroy(m->ev_join);
    if (m->small) cudaFree(m->small);
    delete m;
    h->mg = nullptr;
}

}  // namespace emu

using emu::Handle;

extern "C" {

emugemm_status_t emugemm_comm_unique_id(void* id_out) {
    if (!id_out) return EMUGEMM_STATUS_INVALID_POINTER;
    const emu::NcclApi* n = emu::nccl();
    if (!n) return EMUGEMM_STATUS_NOT_IMPLEMENTED;
    ncclUniqueId id;
    emugemm_status_t s = emu::from_nccl(n->get_unique_id(&id));
    if (s != EMUGEMM_STATUS_SUCCESS) return s;
    std::memcpy(id_out, &id, sizeof id);
    return EMUGEMM_STATUS_SUCCESS;
}

emugemm_status_t emugemm_comm_init(emugemm_handle_t handle, int nranks, int rank, const void* id, int max_ctas) {
    Handle* h = reinterpret_cast<Handle*>(handle);
    if (!h) return EMUGEMM_STATUS_INVALID_HANDLE;
    if (!id) return EMUGEMM_STATUS_INVALID_POINTER;
    if (nranks < 1 || rank < 0 || rank >= nranks || max_ctas < 0) return EMUGEMM_STATUS_INVALID_VALUE;
    const emu::NcclApi* n = emu::nccl();
    if (!n) return EMUGEMM_STATUS_NOT_IMPLEMENTED;
    emu::DeviceGuard g(h->device);
    if (!g.ok) return EMUGEMM_STATUS_INTERNAL_ERROR;
    emu::multigpu_release(h);
    emu::Mg* m = new emu::Mg();
    h->mg = m;
    m->rank = rank;
    m->size = nranks;
    bool ok = cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) == cudaSuccess &&
              cudaStreamCreateWithFlags(&m->stream2, cudaStreamNonBlocking) == cudaSuccess &&
              cudaEventCreateWithFlags(&m->ev_a, cudaEventDisableTiming) == cudaSuccess &&
              cudaEventCreateWithFlags(&m->ev_join, cudaEventDisableTiming) == cudaSuccess &&
              cudaEventCreateWithFlags(&m->ev_start, cudaEventDisableTiming) == cudaSuccess &&
              cudaEventCreateWithFlags(&m->ev_done, cudaEventDisableTiming) == cudaSuccess &&
              cudaMalloc(&m->small, 256) == cudaSuccess;
    for (cudaEvent_t& e : m->ev_panel) ok = ok && cudaEventCreateWithFlags(&e, cudaEventDisableTiming) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        emu::multigpu_release(h);
        return EMUGEMM_STATUS_MEMORY_ERROR;
    }
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof uid);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    if (max_ctas > 0) {
        cfg.minCTAs = 1;
        cfg.maxCTAs = max_ctas;
    }
    emugemm_status_t s = emu::from_nccl(n->init_rank_config(&m->comm, nranks, uid, rank, &cfg));
    if (s != EMUGEMM_STATUS_SUCCESS) {
        m->comm = nullptr;
        emu::multigpu_release(h);
    }
    return s;
}

emugemm_status_t emugemm_comm_destroy(emugemm_handle_t handle) {
    Handle* h = reinterpret_cast<Handle*>(handle);
    if (!h) return EMUGEMM_STATUS_INVALID_HANDLE;
    emu::DeviceGuard g(h->device);
    emu::multigpu_release(h);
    return EMUGEMM_STATUS_SUCCESS;
}

emugemm_status_t emugemm_comm_rows(emugemm_handle_t handle, int M, int* row0, int* rows) {
    Handle* h = reinterpret_cast<Handle*>(handle);
    if (!h) return EMUGEMM_STATUS_INVALID_HANDLE;
    emu::Mg* m = emu::mg_of(h);
    if (!m) return EMUGEMM_STATUS_INVALID_VALUE;
    if (M < 0) return EMUGEMM_STATUS_INVALID_SIZE;
    long r0, r1;
    emu::row_range(M, m->rank, m->size, &r0, &r1);
    if (row0) *row0 = (int)r0;
    if (rows) *rows = (int)(r1 - r0);
    return EMUGEMM_STATUS_SUCCESS;
}

emugemm_status_t emugemm_comm_krange(emugemm_handle_t handle, long K, long* k0, long* klen) {
    Handle* h = reinterpret_cast<Handle*>(handle);
    if (!h) return EMUGEMM_STATUS_INVALID_HANDLE;
    emu::Mg* m = emu::mg_of(h);
    if (!m) return EMUGEMM_STATUS_INVALID_VALUE;
    if (K < 0) return EMUGEMM_STATUS_INVALID_SIZE;
    long a, b;
    emu::k_range(K, m->rank, m->size, &a, &b);
    if (k0) *k0 = a;
    if (klen) *klen = b - a;
    return EMUGEMM_STATUS_SUCCESS;
}

int emugemm_rows_panels(int M, int nranks, int N, long K, int num_sms, int forced, int* n0, int* n1, int max) {
    if (nranks < 1 || M < 0 || N < 0 || K < 0) return -1;
    const auto p = emu::rows_panels(M, nranks, N, K, num_sms, forced);
    for (int i = 0; i < (int)p.size() && i < max; ++i) {
        if (n0) n0[i] = (int)p[i].first;
        if (n1) n1[i] = (int)p[i].second;
    }
    return (int)p.size();
}

emugemm_status_t emugemm_sgemm_rows(emugemm_handle_t handle, int M, int N, long K, const float* A_local, long lda,
                                    float* B, long ldb, float* C_local, long ldc, int root,
                                    const emu_request_t* req, emu_hints_t* hints, emu_plan_t* out_plan) {
    Handle* h = reinterpret_cast<Handle*>(handle);
    if (!h) return EMUGEMM_STATUS_INVALID_HANDLE;
    emu::Mg* m = emu::mg_of(h);
    if (!m) return EMUGEMM_STATUS_INVALID_VALUE;   // no communicator: emugemm_comm_init first
    if (M < 0 || N < 0 || K < 0) return EMUGEMM_STATUS_INVALID_SIZE;
    if (root < 0 || root >= m->size) return EMUGEMM_STATUS_INVALID_VALUE;
    long r0, r1;
    emu::row_range(M, m->rank, m->size, &r0, &r1);
    const int ml = (int)(r1 - r0);
    const bool is_root = m->rank == root;
    if (lda < (K > 0 ? K : 1) || ldc < (N > 0 ? N : 1) || (B && ldb < (N > 0 ? N : 1)))
        return EMUGEMM_STATUS_INVALID_SIZE;
    if ((ml > 0 && N > 0 && (!C_local || (K > 0 && !A_local))) || (is_root && K > 0 && N > 0 && !B))
        return EMUGEMM_STATUS_INVALID_POINTER;
    emu::DeviceGuard g(h->device);
    if (!g.ok) return EMUGEMM_STATUS_INTERNAL_ERROR;
    const emu::NcclApi* n = emu::nccl();
    if (!n) return EMUGEMM_STATUS_NOT_IMPLEMENTED;
    cudaStream_t cs = (cudaStream_t)h->stream;

    // Hints, agreed on by all ranks (every rank passes the same hints): max |A| over the row blocks, max |B| from
    // the root, and rho from the Hutchinson sums of all row blocks added up (after B has arrived, see below).
    emu_hints_t local = hints ? *hints : emu_hints_t{-1.f, -1.f, 0, -1.f, 0};
    const bool want_amax = local.a_absmax < 0 || local.b_absmax < 0, want_rho = local.rho < 0;
    if (want_amax) {
        float v[2] = {0.f, 0.f};
        if (local.a_absmax < 0 && ml > 0 && K > 0) {
            emugemm_status_t s = emu::absmax(h, A_local, ml, K, lda, &v[0]);
            if (s != EMUGEMM_STATUS_SUCCESS) return s;
        }
        if (local.b_absmax < 0 && is_root && K > 0 && N > 0) {
            emugemm_status_t s = emu::absmax(h, B, K, N, ldb, &v[1]);
            if (s != EMUGEMM_STATUS_SUCCESS) return s;
        }
        float* d = static_cast<float*>(m->small);
        int e = (int)cudaMemcpyAsync(d, v, sizeof v, cudaMemcpyHostToDevice, cs);
        if (e) return emu::from_cuda(e);
        emugemm_status_t s = emu::from_nccl(n->all_reduce(d, d, 2, ncclFloat, ncclMax, m->comm, cs));
        if (s != EMUGEMM_STATUS_SUCCESS) return s;
        e = (int)cudaMemcpyAsync(v, d, sizeof v, cudaMemcpyDeviceToHost, cs);
        if (!e) e = (int)cudaStreamSynchronize(cs);
        if (e) return emu::from_cuda(e);
        if (local.a_absmax < 0) local.a_absmax = v[0];
        if (local.b_absmax < 0) local.b_absmax = v[1];
    }

    // Column panels of B (one panel when rho must be measured: the probe reads all of B at once).
    const int gemm_sms = (m->size > 1 && h->comm_sms > 0) ? h->num_sms - h->comm_sms : h->num_sms;
    const auto pan = want_rho ? emu::rows_panels(M, m->size, N, K, gemm_sms, 1)
                              : emu::rows_panels(M, m->size, N, K, gemm_sms, h->rows_panels);
    long wmax = 0;
    for (const auto& p : pan) wmax = std::max(wmax, p.second - p.first);
    // B's path: copy engines over peer memory (default, when every rank can map the others' memory) or NCCL
    const bool use_p2p = m->size > 1 && !h->bcast_nccl && K > 0 && N > 0 &&
                         emu::p2p_setup(h, m, n, (size_t)K * N * 4) == EMUGEMM_STATUS_SUCCESS && m->p2p == 1;
    float* stage = nullptr;
    // calls that move B by copy engines are numbered alike on every rank (use_p2p is the same on all of them)
    const unsigned seq = use_p2p ? ++m->seq : 0u;
    const int buf = (int)(seq & 1u);
    if (use_p2p) {
        stage = m->stage[buf];
    } else if (K > 0 && N > 0) {
        stage = static_cast<float*>(emu::ws_get(h, emu::kWsCommB, (size_t)K * N * 4));
        if (!stage) return EMUGEMM_STATUS_MEMORY_ERROR;
    }
    // The transfers start once earlier work on the handle's stream is done with the staging buffer (and the root's B
    // is final); panel j is packed on the root (B's columns [n0, n1) made contiguous at stage + K*n0), moved to the
    // other ranks, and there copied into B's columns when the caller passed a B to receive it.
    int e = (int)cudaEventRecord(m->ev_start, cs);
    if (!e) e = (int)cudaStreamWaitEvent(m->stream, m->ev_start, 0);
    if (e) return emu::from_cuda(e);
    // the tree for this root: v = position after the root; parent (v - 1) / 2, children 2v + 1 and 2v + 2
    const int P = m->size, v = (m->rank - root + P) % P;
    const int parent = v > 0 ? ((v - 1) / 2 + root) % P : -1;
    if (use_p2p && seq > 2) {
        // this buffer was last filled two calls ago: wait until every rank has released that call (its pulls are
        // done; which ranks pulled from this one depended on that call's root)
        e = emu::wait_flags(m->flags + emu::kFlagRelease, P, m->rank, seq - 2, h->err_dev, m->stream);
        if (e) return emu::from_cuda(e);
    }
    // Staging layouts. Copy engines: B row-major (ld N) on every rank; the root fills its buffer with one contiguous
    // copy (a pitched same-GPU copy beside its GEMMs cost them 0.23 ms at 8192^3, a contiguous one 0.05 ms) and
    // announces every panel, and each other rank pulls panel j as a pitched copy over NVLink from its parent. NCCL:
    // panel j contiguous at stage + K * n0 (a broadcast buffer must be contiguous), packed on the root.
    if (use_p2p && is_root && K > 0 && N > 0) {
        // the first panel alone first (a small pitched copy), so that the other ranks start without waiting for all
        // of B; then B in one piece, which writes the first panel's bytes again with the same values
        const bool first_alone = pan.size() > 1;
        if (first_alone) {
            const long w0 = pan[0].second - pan[0].first;
            e = (int)cudaMemcpy2DAsync(stage, (size_t)N * 4, B, (size_t)ldb * 4, (size_t)w0 * 4, (size_t)K,
                                       cudaMemcpyDeviceToDevice, m->stream);
            if (!e) e = emu::set_flag(m->flags + emu::kFlagArrive + 16 * buf, seq, m->stream);
            if (e) return emu::from_cuda(e);
        }
        e = ldb == N ? (int)cudaMemcpyAsync(stage, B, (size_t)K * N * 4, cudaMemcpyDeviceToDevice, m->stream)
                     : (int)cudaMemcpy2DAsync(stage, (size_t)N * 4, B, (size_t)ldb * 4, (size_t)N * 4, (size_t)K,
                                              cudaMemcpyDeviceToDevice, m->stream);
        if (!e) {
            emu::PeerFlags f{};
            for (size_t j = first_alone ? 1 : 0; j < pan.size(); ++j) f.p[j] = m->flags + emu::kFlagArrive + 16 * buf + j;
            emu::k_set_flags<<<1, 32, 0, m->stream>>>(f, (int)pan.size(), seq);
            emu::count_launch();
            e = (int)cudaGetLastError();
        }
        if (e) return emu::from_cuda(e);
    }
    for (size_t j = 0; j < pan.size() && K > 0; ++j) {
        const long n0 = pan[j].first, w = pan[j].second - pan[j].first;
        float* sp = use_p2p ? stage + n0 : stage + (size_t)K * n0;
        const long sld = use_p2p ? N : w;
        if (use_p2p) {
            if (!is_root) {
                e = emu::wait_flags(m->peer_flags[parent] + emu::kFlagArrive + 16 * buf + j, 1, -1, seq, h->err_dev,
                                    m->stream);
                if (!e)
                    e = (int)cudaMemcpy2DAsync(sp, (size_t)N * 4, m->peer_stage[buf][parent] + n0, (size_t)N * 4,
                                               (size_t)w * 4, (size_t)K, cudaMemcpyDeviceToDevice, m->stream);
                if (!e) e = emu::set_flag(m->flags + emu::kFlagArrive + 16 * buf + j, seq, m->stream);
                if (e) return emu::from_cuda(e);
            }
        } else {
            if (is_root)
                e = (int)cudaMemcpy2DAsync(sp, (size_t)w * 4, B + n0, (size_t)ldb * 4, (size_t)w * 4, (size_t)K,
                                           cudaMemcpyDeviceToDevice, m->stream);
            if (e) return emu::from_cuda(e);
            emugemm_status_t s =
                emu::from_nccl(n->broadcast(sp, sp, (size_t)K * w, ncclFloat, root, m->comm, m->stream));
            if (s != EMUGEMM_STATUS_SUCCESS) return s;
        }
        if (!is_root && B)
            e = (int)cudaMemcpy2DAsync(B + n0, (size_t)ldb * 4, sp, (size_t)sld * 4, (size_t)w * 4, (size_t)K,
                                       cudaMemcpyDeviceToDevice, m->stream);
        if (!e) e = (int)cudaEventRecord(m->ev_panel[j], m->stream);
        if (e) return emu::from_cuda(e);
    }
    if (use_p2p) {
        // every panel pulled (the root pulls none): tell every rank, each may refill its buffer in two calls' time
        emu::PeerFlags f{};
        for (int r = 0; r < P; ++r)
            if (r != m->rank) f.p[r] = m->peer_flags[r] + emu::kFlagRelease + m->rank;
        emu::k_set_flags<<<1, 32, 0, m->stream>>>(f, P, seq);
        emu::count_launch();
        e = (int)cudaGetLastError();
        if (e) return emu::from_cuda(e);
    }
    e = (int)cudaEventRecord(m->ev_done, m->stream);
    if (e) return emu::from_cuda(e);

    if (want_rho) {
        // all of B has arrived (one panel): this rank's Hutchinson sums over its rows, added up over the ranks
        double v[2] = {0.0, 0.0};
        const int P = local.rho_probes > 0 ? local.rho_probes : 64;
        e = (int)cudaStreamWaitEvent(cs, m->ev_done, 0);
        if (e) return emu::from_cuda(e);
        if (ml > 0 && K > 0 && N > 0) {
            const float* Bsrc = is_root ? B : stage;
            const long bld = is_root ? ldb : N;
            if (!emu::rho_sums(h, ml, N, K, A_local, lda, Bsrc, bld, P, v)) return EMUGEMM_STATUS_INTERNAL_ERROR;
        }
        double* d = static_cast<double*>(m->small);
        e = (int)cudaMemcpyAsync(d, v, sizeof v, cudaMemcpyHostToDevice, cs);
        if (e) return emu::from_cuda(e);
        emugemm_status_t s = emu::from_nccl(n->all_reduce(d, d, 2, ncclDouble, ncclSum, m->comm, cs));
        if (s != EMUGEMM_STATUS_SUCCESS) return s;
        e = (int)cudaMemcpyAsync(v, d, sizeof v, cudaMemcpyDeviceToHost, cs);
        if (!e) e = (int)cudaStreamSynchronize(cs);
        if (e) return emu::from_cuda(e);
        const double num = std::sqrt(v[0] / P), den = std::sqrt(v[1] / P);
        local.rho = (num >= 0 && den > 0) ? (float)(num / den) : -1.f;
    }
    if (hints) {
        hints->a_absmax = local.a_absmax;
        hints->b_absmax = local.b_absmax;
        hints->rho = local.rho;
    }
    const emu_plan_t plan = emu::plan(emu::model(), M, N, K, req, &local);
    if (out_plan) *out_plan = plan;

    // The GEMMs on the handle's stream: A's slices once, before the first panel arrives; then panel j as soon as it
    // is there (the root reads its own B in place). Every panel of every rank runs the tensor-core kernel and K split
    // count chosen for the WHOLE M x N x K product, so C does not depend on the number of ranks: each rank's rows
    // are those of the single-GPU emugemm_sgemm of the whole product, bit for bit.
    emugemm_status_t st = EMUGEMM_STATUS_SUCCESS;
    if (ml > 0 && N > 0) {
        if (K == 0) {
            e = (int)cudaMemset2DAsync(C_local, (size_t)ldc * 4, 0, (size_t)N * 4, (size_t)ml, cs);
            if (e) return emu::from_cuda(e);
        } else {
            if (emu::is_tc(plan.chosen)) {
                const bool fp16 = plan.chosen == EMU_SCHEME_FP16X3;
                h->pin_tc_code = emu::tc_kernel_choice(h, M, N, K, fp16);
                h->pin_splits = emu::tc_split_count(emu::round_up(M, 256), emu::round_up(N, 256), K, h->num_sms,
                                                    h->tc_splitk);
            }
            struct Restore {
                Handle* h;
                void* stream;
                ~Restore() {
                    h->pin_tc_code = 0; h->pin_splits = 0; h->tc_grid_sms = 0;
                    h->stream = stream; h->bank = 0;
                }
            } restore{h, h->stream};
            if (m->size > 1 && h->comm_sms > 0) h->tc_grid_sms = h->num_sms - h->comm_sms;
            st = emu::prepare_a(h, plan.chosen, ml, (int)wmax, K, A_local, lda);
            // odd panels on the second stream with the bank-1 scratch, after A's split
            const bool two = pan.size() > 1;
            if (st == EMUGEMM_STATUS_SUCCESS && two) {
                e = (int)cudaEventRecord(m->ev_a, cs);
                if (!e) e = (int)cudaStreamWaitEvent(m->stream2, m->ev_a, 0);
                if (e) return emu::from_cuda(e);
            }
            for (size_t j = 0; j < pan.size() && st == EMUGEMM_STATUS_SUCCESS; ++j) {
                const long n0 = pan[j].first, w = pan[j].second - pan[j].first;
                const bool odd = two && (j & 1);
                cudaStream_t ps = odd ? m->stream2 : cs;
                if (!is_root) {
                    e = (int)cudaStreamWaitEvent(ps, m->ev_panel[j], 0);
                    if (e) return emu::from_cuda(e);
                }
                const float* Bp = is_root ? B + n0 : use_p2p ? stage + n0 : stage + (size_t)K * n0;
                const long bld = is_root ? ldb : use_p2p ? N : w;
                h->stream = ps;
                h->bank = odd ? 1 : 0;
                st = emu::dispatch(h, plan.chosen, plan.chunks, ml, (int)w, K, A_local, lda, Bp, bld, C_local + n0, ldc,
                                   nullptr, 0, /*a_reused*/ true);
                h->stream = cs;
                h->bank = 0;
            }
            if (two) {
                e = (int)cudaEventRecord(m->ev_join, m->stream2);
                if (!e) e = (int)cudaStreamWaitEvent(cs, m->ev_join, 0);
                if (e) return emu::from_cuda(e);
            }
        }
    }
    // the call is complete on the handle's stream once the broadcasts (and the copies into B) are done as well
    e = (int)cudaStreamWaitEvent(cs, m->ev_done, 0);
    if (st != EMUGEMM_STATUS_SUCCESS) return st;
    return emu::from_cuda(e);
}

emugemm_status_t emugemm_sgemm_ksplit(emugemm_handle_t handle, int M, int N, long K, const float* A_local, long lda,
                                      const float* B_local, long ldb, float* C, long ldc, int root, int scheme,
                                      int chunks) {
    Handle* h = reinterpret_cast<Handle*>(handle);
    if (!h) return EMUGEMM_STATUS_INVALID_HANDLE;
    emu::Mg* m = emu::mg_of(h);
    if (!m) return EMUGEMM_STATUS_INVALID_VALUE;
    if (M < 0 || N < 0 || K < 0) return EMUGEMM_STATUS_INVALID_SIZE;
    if (root >= m->size || root < -1) return EMUGEMM_STATUS_INVALID_VALUE;
    if (scheme <= EMU_SCHEME_AUTO || scheme > EMU_SCHEME_BF16X6) return EMUGEMM_STATUS_INVALID_VALUE;
    long k0, k1;
    emu::k_range(K, m->rank, m->size, &k0, &k1);
    const long kl = k1 - k0;
    const bool out_here = root < 0 || root == m->rank;
    if (lda < (kl > 0 ? kl : 1) || ldb < (N > 0 ? N : 1) || (out_here && ldc < (N > 0 ? N : 1)))
        return EMUGEMM_STATUS_INVALID_SIZE;
    if (M > 0 && N > 0 && ((kl > 0 && (!A_local || !B_local)) || (out_here && !C)))
        return EMUGEMM_STATUS_INVALID_POINTER;
    if (M == 0 || N == 0) return EMUGEMM_STATUS_SUCCESS;
    emu::DeviceGuard g(h->device);
    if (!g.ok) return EMUGEMM_STATUS_INTERNAL_ERROR;
    const emu::NcclApi* n = emu::nccl();
    if (!n) return EMUGEMM_STATUS_NOT_IMPLEMENTED;
    cudaStream_t cs = (cudaStream_t)h->stream;
    double* P = static_cast<double*>(emu::ws_get(h, emu::kWsCommP, (size_t)M * N * 8));
    if (!P) return EMUGEMM_STATUS_MEMORY_ERROR;
    emugemm_status_t st;
    if (kl > 0)
        st = emu::dispatch(h, (emu_scheme_t)scheme, chunks, M, N, kl, A_local, lda, B_local, ldb, nullptr, 0, P, N);
    else
        st = emu::from_cuda((int)cudaMemsetAsync(P, 0, (size_t)M * N * 8, cs));
    if (st != EMUGEMM_STATUS_SUCCESS) return st;
    const size_t cnt = (size_t)M * N;
    st = emu::from_nccl(root < 0 ? n->all_reduce(P, P, cnt, ncclDouble, ncclSum, m->comm, cs)
                                 : n->reduce(P, P, cnt, ncclDouble, ncclSum, root, m->comm, cs));
    if (st != EMUGEMM_STATUS_SUCCESS || !out_here) return st;
    emu::ProfScope ps(h, emu::kProfReduce);
    return emu::from_cuda(emu::launch_reduce_f64(P, 1, M, N, (long)M * N, C, ldc, nullptr, 0, cs));
}

}  // extern "C"
