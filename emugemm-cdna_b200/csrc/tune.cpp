// tune.cpp - per-shape tile table of emugemm (replaces the rocBLAS solution-index table of emugemm-cdna,
// src/emugemm.cpp:101-140).
//
// File format: the reference's 10-column CSV (data/tune_table.csv:1) with the rocBLAS columns reused:
//     arch,cuda_version,M,N,K,dtype,tile,best_ms,default_ms,gain
// dtype is fp32 | bf16 | fp16. `tile` is the kernel choice for that shape: for bf16/fp16 rows the
// tensor-core kernel (1 = single-CTA 128-row tiles, 2 = CTA pairs on 256-row tiles, 3 = CTA pairs with the
// split fused in, 4 = CTA pairs with A split into TMEM in the kernel), for fp32 rows the SIMT tile edge
// (32, 64 or 128). As in the reference, a row whose arch does not match the live device is rejected (a tile
// choice tuned on another GPU is not trusted), lines that do not parse as 10 fields are skipped (this
// skips the header), and the lookup takes the nearest shape in log2 space if its distance is below 1.
#include "emugemm_internal.h"

#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

namespace emu {
namespace {

struct TuneRow { int M, N; long K; int dt; int tile; };

std::mutex g_mu;
std::vector<TuneRow> g_tune;
std::string g_arch;
bool g_ready = false;

}  // namespace

std::string live_arch_string() {
    int dev = 0, major = 0, minor = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return std::string();
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return std::string();
    if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) return std::string();
    char buf[32];
    // The library is built for the architecture-specific target sm_100a.
    std::snprintf(buf, sizeof buf, "sm_%d%d%s", major, minor, (major == 10 && minor == 0) ? "a" : "");
    return std::string(buf);
}

emugemm_status_t init_for_arch(const char* path, const std::string& live) {
    std::lock_guard<std::mutex> lk(g_mu);
    g_tune.clear();
    g_ready = false;
    FILE* f = path ? std::fopen(path, "r") : nullptr;
    if (!f) {
        std::fprintf(stderr, "emugemm: no tune table at %s -- running with the built-in tile choice\n",
                     path ? path : "(null)");
        g_arch = live;
        g_ready = true;
        return EMUGEMM_STATUS_SUCCESS;
    }
    char line[512];
    int rejected = 0;
    while (std::fgets(line, sizeof line, f)) {
        char arch[96], ver[96], dt[16];
        int M, N, tile;
        long K;
        double bms, dms, gain;
        if (std::sscanf(line, "%95[^,],%95[^,],%d,%d,%ld,%15[^,],%d,%lf,%lf,%lf", arch, ver, &M, &N, &K, dt, &tile,
                        &bms, &dms, &gain) != 10)
            continue;
        if (live.find(arch) == std::string::npos && std::strncmp(arch, live.c_str(), 6) != 0) {
            ++rejected;
            continue;
        }
        int dcode = (std::strcmp(dt, "bf16") == 0) ? 1 : (std::strcmp(dt, "fp16") == 0) ? 2 : 0;
        if (M <= 0 || N <= 0 || K <= 0) continue;
        g_tune.push_back({M, N, K, dcode, tile});
    }
    std::fclose(f);
    if (rejected) std::fprintf(stderr, "emugemm: rejected %d rows from a different arch than %s\n", rejected, live.c_str());
    std::fprintf(stderr, "emugemm: loaded %zu tuned entries for %s\n", g_tune.size(), live.c_str());
    g_arch = live;
    g_ready = true;
    return EMUGEMM_STATUS_SUCCESS;
}

int tune_rows() {
    std::lock_guard<std::mutex> lk(g_mu);
    return (int)g_tune.size();
}

// Nearest shape in log2 space (src/emugemm.cpp:131-140); 0 when nothing is within distance 1.
static int lookup_raw(int M, int N, long K, int dt) {
    std::lock_guard<std::mutex> lk(g_mu);
    double best = 1e30;
    int tile = 0;
    for (const TuneRow& r : g_tune) {
        if (r.dt != dt) continue;
        double d = std::fabs(std::log2((double)r.M / M)) + std::fabs(std::log2((double)r.N / N)) +
                   std::fabs(std::log2((double)r.K / K));
        if (d < best) { best = d; tile = r.tile; }
    }
    return (best < 1.0) ? tile : 0;
}

TileChoice lookup_tile(int M, int N, long K, int dtype) {
    TileChoice t{0, 0};
    if (M <= 0 || N <= 0 || K <= 0) return t;
    int v = lookup_raw(M, N, K, dtype);
    if (dtype == 0) {
        if (fp32_tile_code_ok(v)) t.fp32_bm = v;
    } else {
        if (v >= 1 && v <= 4) t.tc_variant = v;
    }
    return t;
}

void tune_clear() {
    std::lock_guard<std::mutex> lk(g_mu);
    g_tune.clear();
    g_ready = false;
}

}  // namespace emu

extern "C" {

emugemm_status_t emugemm_init(const char* tune_csv_path) {
    std::string live = emu::live_arch_string();
    if (live.empty()) return EMUGEMM_STATUS_INTERNAL_ERROR;
    return emu::init_for_arch(tune_csv_path, live);
}

emugemm_status_t emugemm_init_for_arch(const char* tune_csv_path, const char* live_arch) {
    if (!live_arch) return EMUGEMM_STATUS_INVALID_POINTER;
    return emu::init_for_arch(tune_csv_path, std::string(live_arch));
}

int emugemm_tune_rows(void) { return emu::tune_rows(); }

int emugemm_tune_lookup(int M, int N, long K, int dtype) {
    emu::TileChoice t = emu::lookup_tile(M, N, K, dtype);
    return dtype == 0 ? t.fp32_bm : t.tc_variant;
}

}  // extern "C"
