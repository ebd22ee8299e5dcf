// Decode of one WNR2/WNR3 record into caller-owned device buffers that allocates nothing.
//
// Who needs it: an engine that reserves all of its device memory at start-up in its own pool and may
// not call cudaMalloc / cudaFree afterwards (allocating later fragments its pool or fails under load),
// or one whose serving streams must never stall on the implicit device synchronisation that
// cudaMalloc and cudaFree can cause. Every other entry point of this library grows pooled device
// buffers on demand; this one works entirely inside a fixed array defined in this file.
//
// The scratch (record staging, the decoded slab before its gated commit, launch metadata with the work
// queue and its counters, model tables) is the file-scope device array below, of a fixed size: records
// of at most 24 MiB stored and 24 MiB decoded, at most 32,768 streams, at most 4 models per device. Every device on which this
// library's module is loaded holds the array (about 50 MiB) until the process exits; with CUDA's
// default lazy module loading that starts at the first call on the device. Every call shares the
// array and it keeps the last call's contents, so each call rewrites all the metadata it reads and
// clears the record's error word. Calls are synchronous and serialised by a process-wide lock; two
// calls that overlapped on the GPU would race on the array.
//
// In host code `g_na_scratch` is only a host-side stand-in for the device array, never a device
// address: the first call on each device, with that device current, asks the runtime for the real
// address (cudaGetSymbolAddress), creates the non-blocking stream its calls run on, and every pointer
// given to a kernel is derived from that address. That set-up call, and the first call that uses a
// model on a device (it copies the model's tables into the array with a synchronous cudaMemcpy),
// synchronise with the device; they should therefore come before any stream capture on that device.
// The call waits for its decode under the library's host wait limit; if that wait gives up it returns 1,
// and later calls on the device return 1 until the decode still using the array has ended. The caller's
// current device is restored on return.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <mutex>

#include "host_wait.h"
#include "nr3_host.h"
#include "wex_cuda_helper.h"
#include "wexb200.h"

#define WEXB_API extern "C" __attribute__((visibility("default")))

namespace wexb {
namespace {

constexpr size_t al256(size_t v) { return (v + 255) & ~(size_t)255; }

constexpr size_t kNaMaxRecord = 24ull << 20;    // stored record bytes
constexpr size_t kNaMaxSlab = 24ull << 20;      // decoded bytes (decode layout)
constexpr uint32_t kNaMaxStreams = 32768;
constexpr int kNaModels = 4;
constexpr uint32_t kNaMaxItems = kNaMaxStreams / 32u + 64u + (uint32_t)(kNaMaxSlab / kCommitChunk) + 8u;
// byte layout of the array
constexpr size_t kNaRec = 0;                                          // one Nr3Record
constexpr size_t kNaJob = al256(sizeof(Nr3Record));                   // one CommitJob
constexpr size_t kNaErr = kNaJob + al256(sizeof(CommitJob));          // the error word
constexpr size_t kNaCounters = kNaErr + 256;                          // the queue head, then 4 counters
constexpr size_t kNaItems = kNaCounters + 256;                        // the work queue
constexpr size_t kNaOffs = kNaItems + al256((size_t)kNaMaxItems * sizeof(Nr3Item));
constexpr size_t kNaMeta = kNaOffs + al256(((size_t)kNaMaxStreams + 1) * 4);   // per-call metadata ends here
constexpr size_t kNaTableStride = al256(kTableBytes);
constexpr size_t kNaTables = al256(kNaMeta);
constexpr size_t kNaRecord = kNaTables + kNaModels * kNaTableStride;
constexpr size_t kNaSlab = kNaRecord + al256(kNaMaxRecord + kRecordSlack);
constexpr size_t kNaBytes = kNaSlab + kNaMaxSlab;

static __device__ __align__(256) uint8_t g_na_scratch[kNaBytes];

std::mutex g_na_mu;
uint8_t *g_na_base[kMaxDevices];                 // device address of g_na_scratch, per device
cudaStream_t g_na_stream[kMaxDevices];           // the stream the calls on each device run on
uint32_t g_na_slot[kMaxDevices][kNaModels];      // model id held by each table slot (0 = free)
alignas(256) uint8_t g_na_host[kNaMeta];         // host image of the per-call metadata
// The record's error word is read back into this page, page-locked once per process at the first set-up
// (cudaHostRegister of static memory, no allocation): a read-back into pageable memory would block the
// host until the decode ends, outside the bounded wait.
alignas(4096) uint32_t g_na_word[1024];
bool g_na_word_locked = false;

}  // namespace
}  // namespace wexb

using namespace wexb;

WEXB_API int wexb_decode_to_device_noalloc(const WexEntry *entry, const unsigned char *record, int device,
                                           unsigned char *const *dst_scale, unsigned char *const *dst_weight) {
    if (!entry || !record || !dst_scale || !dst_weight) return -1;
    for (int m = 0; m < 3; ++m) if (!dst_scale[m] || !dst_weight[m]) return -1;
    if (entry->flags == WEX_ENTRY_NEURAL_RANS) return 1;   // WNR1: not built here, as the other entry points
    Plan p;
    if (plan_record(entry, record, &p)) return -1;
    if (p.total > kNaMaxRecord || p.scratch > kNaMaxSlab || p.streams() > kNaMaxStreams) {
        std::fprintf(stderr, "[wex] wexb_decode_to_device_noalloc: record of %u stored bytes, %llu decoded bytes and %u "
                             "streams exceeds its fixed scratch (%zu, %zu bytes, %u streams)\n", p.total,
                     (unsigned long long)p.scratch, p.streams(), kNaMaxRecord, kNaMaxSlab, kNaMaxStreams);
        return -2;
    }
    const uint8_t *image = model_image(p.model_id);
    if (!image || device < 0 || device >= kMaxDevices) return 1;
    std::lock_guard<std::mutex> lock(g_na_mu);
    KeepDevice keep;
    if (cudaSetDevice(device) != cudaSuccess) { (void)cudaGetLastError(); return 1; }
    if (!g_na_base[device]) {   // set-up, once per device, with that device current
        void *ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_na_scratch) != cudaSuccess || !ptr) { (void)cudaGetLastError(); return 1; }
        if (prepare_nr3_kernels() != cudaSuccess) { (void)cudaGetLastError(); return 1; }
        if (!g_na_stream[device] && cudaStreamCreateWithFlags(&g_na_stream[device], cudaStreamNonBlocking) != cudaSuccess) {
            (void)cudaGetLastError();
            g_na_stream[device] = nullptr;
            return 1;
        }
        if (!g_na_word_locked) {
            if (cudaHostRegister(g_na_word, sizeof g_na_word, cudaHostRegisterPortable) != cudaSuccess) {
                (void)cudaGetLastError();
                return 1;
            }
            g_na_word_locked = true;
        }
        g_na_base[device] = static_cast<uint8_t *>(ptr);
    }
    cudaStream_t st = g_na_stream[device];
    if (cudaStreamQuery(st) != cudaSuccess) { (void)cudaGetLastError(); return 1; }   // an earlier decode still runs
    uint8_t *const base = g_na_base[device];
    int slot = -1;
    for (int s = 0; s < kNaModels && slot < 0; ++s) if (g_na_slot[device][s] == p.model_id) slot = s;
    if (slot < 0) {
        for (int s = 0; s < kNaModels && slot < 0; ++s) if (!g_na_slot[device][s]) slot = s;
        if (slot < 0) {
            std::fprintf(stderr, "[wex] wexb_decode_to_device_noalloc: its %d model table slots are taken\n", kNaModels);
            return 1;
        }
        if (cudaMemcpy(base + kNaTables + slot * kNaTableStride, image, kTableBytes, cudaMemcpyHostToDevice) != cudaSuccess) {
            (void)cudaGetLastError();
            return 1;
        }
        g_na_slot[device][slot] = p.model_id;
    }
    const uint8_t *const tab = base + kNaTables + slot * kNaTableStride;
    const int sms = device_sms(device);
    if (!sms) return 1;
    // this call's metadata, written in full (the array keeps the previous call's bytes)
    plan_offsets(p, reinterpret_cast<uint32_t *>(g_na_host + kNaOffs));
    const Plan *plans[1] = {&p};
    LaunchSet launch;
    launch.plan(plans, &tab, 1, true);
    if (launch.items > kNaMaxItems) return -2;   // not reached within the stream and slab limits above
    launch.fill(plans, true, sms, kScalesFirst, reinterpret_cast<Nr3Item *>(g_na_host + kNaItems),
                reinterpret_cast<uint32_t *>(g_na_host + kNaCounters));
    uint32_t *derr = reinterpret_cast<uint32_t *>(base + kNaErr);
    const CommitJob *djob = reinterpret_cast<const CommitJob *>(base + kNaJob);
    plan_descriptor(p, base + kNaRecord, reinterpret_cast<const uint32_t *>(base + kNaOffs), base + kNaSlab, derr, djob,
                    reinterpret_cast<Nr3Record *>(g_na_host + kNaRec));
    CommitJob *job = reinterpret_cast<CommitJob *>(g_na_host + kNaJob);
    for (int m = 0; m < 3; ++m) {
        job->src[m] = base + kNaSlab + p.soff[m]; job->dst[m] = dst_scale[m]; job->bytes[m] = p.dst_bytes[m];
        job->src[3 + m] = base + kNaSlab + p.wout[m]; job->dst[3 + m] = dst_weight[m]; job->bytes[3 + m] = p.dst_bytes[3 + m];
    }
    *reinterpret_cast<uint32_t *>(g_na_host + kNaErr) = 0;   // the error word starts at zero every call
    const size_t meta_bytes = kNaOffs + 4ull * (p.streams() + 1);
    uint32_t &error = g_na_word[0];
    error = ~0u;
    const bool ok = cudaMemcpyAsync(base + kNaRecord, record, p.total, cudaMemcpyHostToDevice, st) == cudaSuccess &&
                    cudaMemcpyAsync(base, g_na_host, meta_bytes, cudaMemcpyHostToDevice, st) == cudaSuccess &&
                    launch.launch(reinterpret_cast<const Nr3Record *>(base + kNaRec), reinterpret_cast<const Nr3Item *>(base + kNaItems),
                                  reinterpret_cast<uint32_t *>(base + kNaCounters), sms, st) &&
                    cudaMemcpyAsync(&error, derr, 4, cudaMemcpyDeviceToHost, st) == cudaSuccess;
    const Waited waited = wait_stream(st);   // also after a failed step: whatever was queued must end
    if (!ok || waited != Waited::Done) { (void)cudaGetLastError(); return 1; }
    if (error) report_error_bits(error);
    return status_of_bits(error);
}
