// The engine-facing API of include/wex_decode.h over the GPU helper of this library
// (c/wex_decode.c is the reference's; its helper-loading and CPU-fallback branches have no
// counterpart here: the helper is this library and there is no CPU decoder).
#include <cuda_runtime.h>

#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "nr3_host.h"
#include "wex_cuda_helper.h"
#include "wex_decode.h"

#define WEXB_API extern "C" __attribute__((visibility("default")))

namespace wexb {
namespace {

std::atomic<uint64_t> g_host_ok{0}, g_device_ok{0};

// The GPU helper is used unless COLI_WEX_CUDA_LIB is "0" (c/wex_decode.c:42-44) and a device exists.
bool gpu_enabled() {
    static const bool on = [] {
        const char *v = std::getenv("COLI_WEX_CUDA_LIB");
        if (v && !std::strcmp(v, "0")) return false;
        int n = 0;
        if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) { (void)cudaGetLastError(); return false; }
        return true;
    }();
    return on;
}

void report_unavailable() {
    static std::atomic<int> once{0};
    if (!once.exchange(1))
        std::fprintf(stderr, "[wex] GPU decode unavailable (COLI_WEX_CUDA_LIB=0 or no CUDA device); this library has "
                             "no CPU decoder\n");
}

}  // namespace
}  // namespace wexb

using namespace wexb;

WEXB_API int coli_wex_register_model(const unsigned char *blob, size_t bytes, uint32_t *id) {
    uint32_t probe = 0;
    if (model_validate(blob, bytes, &probe)) return -1;
    if (model_register(blob, bytes)) return -1;   // an id collision or a full registry
    if (id) *id = probe;
    return 0;
}

WEXB_API int coli_wex_cuda_nr2_available(void) { return gpu_enabled(); }
WEXB_API int coli_wex_cuda_nr3_available(void) { return gpu_enabled(); }
WEXB_API int coli_wex_cuda_device_available(void) { return gpu_enabled(); }
WEXB_API int coli_wex_cuda_batch_available(void) { return gpu_enabled(); }
WEXB_API int coli_wex_cuda_batch_host_available(void) { return gpu_enabled(); }
WEXB_API uint64_t coli_wex_cuda_decode_count(void) { return g_host_ok.load(); }
WEXB_API uint64_t coli_wex_cuda_device_decode_count(void) { return g_device_ok.load(); }

WEXB_API int coli_wex_cuda_decode_to_device(const WexEntry *entry, const unsigned char *record, int device,
                                            unsigned char *const dst_scale[3], unsigned char *const dst_weight[3]) {
    if (!entry || (entry->flags != WEX_ENTRY_NEURAL_RANS && entry->flags != WEX_ENTRY_NEURAL_RANS2 &&
                   entry->flags != WEX_ENTRY_NEURAL_RANS3)) return -1;
    if (!gpu_enabled()) return 1;
    const int st = wex_cuda_decode_to_device(entry, record, device, dst_scale, dst_weight);
    if (!st) g_device_ok++;
    return st;
}

WEXB_API int coli_wex_cuda_decode_batch_to_device(int n, const WexEntry *const *entries,
                                                  const unsigned char *const *records, int device,
                                                  unsigned char *const *dst_scale, unsigned char *const *dst_weight,
                                                  int *status) {
    if (n <= 0) return 0;
    if (!status) return n;
    if (!gpu_enabled()) { for (int i = 0; i < n; ++i) status[i] = 1; return n; }
    const int bad = wex_cuda_decode_batch_to_device(n, entries, records, device, dst_scale, dst_weight, status);
    for (int i = 0; i < n; ++i) if (!status[i]) g_device_ok++;
    return bad;
}

WEXB_API int coli_wex_cuda_decode_batch_to_host(int n, const WexEntry *const *entries, const unsigned char *const *records,
                                                int device, unsigned char *const *dst, int *status) {
    if (n <= 0) return 0;
    if (!status) return n;
    if (!gpu_enabled()) { for (int i = 0; i < n; ++i) status[i] = 1; return n; }
    const int bad = wex_cuda_decode_batch_to_host(n, entries, records, device, dst, status);
    for (int i = 0; i < n; ++i) if (!status[i]) g_host_ok++;
    return bad;
}

WEXB_API int coli_wex_cuda_host_register(void *pointer, size_t bytes) {
    return gpu_enabled() ? wex_cuda_host_register(pointer, bytes) : 1;
}
WEXB_API int coli_wex_cuda_host_unregister(void *pointer) { return gpu_enabled() ? wex_cuda_host_unregister(pointer) : 1; }

WEXB_API int coli_wex_container_refused(uint32_t header_flags, const char *who) {
    const char *masked = std::getenv("DSV4_CUDA_MOE_MASKED");
    if (!(header_flags & WEX_HEADER_CANONICAL_ZERO)) return 0;
    if (masked && std::atoi(masked) != 0) {
        std::fprintf(stderr, "[%s] value-exact (canonical-zero) container refused: DSV4_CUDA_MOE_MASKED is not proven "
                             "value-exact\n", who ? who : "wex");
        return 1;
    }
    std::fprintf(stderr, "[%s] value-exact (canonical-zero) container\n", who ? who : "wex");
    return 0;
}

WEXB_API int coli_wex_decode_record(const WexEntry *entry, unsigned char *slab, size_t capacity) {
    uint64_t raw, aligned;
    if (!entry || !slab || entry_raw_sizes(entry, &raw, &aligned) || aligned > capacity) return -1;
    if (entry->flags == WEX_ENTRY_RAW) return entry->total_bytes == aligned ? 0 : -1;   // already a slab
    if (entry->flags != WEX_ENTRY_NEURAL_RANS2 && entry->flags != WEX_ENTRY_NEURAL_RANS3) return -1;
    // the record names its model at bytes 4..7 and must be registered (c/wex_decode.c:327-333)
    if (entry->total_bytes >= aligned || entry->total_bytes < 32) return -1;
    const size_t at = (size_t)(aligned - entry->total_bytes);
    if (at > capacity || entry->total_bytes > capacity - at || !model_registered(rd32(slab + at + 4))) return -1;
    if (!gpu_enabled()) { report_unavailable(); return -1; }
    const int st = wex_cuda_decode_to_host(entry, slab, capacity);
    if (!st) { g_host_ok++; return 0; }
    return -1;
}
