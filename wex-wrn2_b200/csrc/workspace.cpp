// Per-device streams and the pool of call workspaces (workspace.h).
#include "workspace.h"

#include <algorithm>
#include <mutex>
#include <new>
#include <vector>

#include "host_wait.h"
#include "nr3_host.h"

namespace wexb {
namespace {

constexpr int kLanes = 4;   // kernel streams per device

struct Queues {
    cudaStream_t upload = nullptr, meta = nullptr, lane[kLanes] = {};
    unsigned next = 0;
    bool ok = false;
};
std::mutex g_queues_mu;
Queues g_queues[kMaxDevices];

constexpr int kHashLanes = 24;
struct HashLanes {
    cudaStream_t s[kHashLanes] = {};
    cudaEvent_t e[kHashLanes] = {};
    unsigned next = 0;
    bool ok = false;
};
HashLanes g_hash[kMaxDevices];

std::mutex g_pool_mu;
std::vector<Workspace *> g_idle[kMaxDevices];
std::vector<Workspace *> g_parked[kMaxDevices];   // gave up waiting: back to g_idle once `done` completes

Workspace *fresh(int device) {
    auto *w = new (std::nothrow) Workspace();
    if (!w) return nullptr;
    if (cudaEventCreateWithFlags(&w->meta_done, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&w->uploads_done, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&w->done, cudaEventDisableTiming) != cudaSuccess) {
        (void)cudaGetLastError();   // an event made before the failure leaks, on CUDA failure only
        delete w;
        return nullptr;
    }
    w->device = device;
    return w;
}

}  // namespace

bool device_streams(int device, cudaStream_t *up, cudaStream_t *st, cudaStream_t *meta) {
    if (device < 0 || device >= kMaxDevices) return false;
    std::lock_guard<std::mutex> lock(g_queues_mu);
    Queues &q = g_queues[device];
    if (!q.ok) {
        bool ok = cudaStreamCreateWithFlags(&q.upload, cudaStreamNonBlocking) == cudaSuccess &&
                  cudaStreamCreateWithFlags(&q.meta, cudaStreamNonBlocking) == cudaSuccess;
        for (int l = 0; ok && l < kLanes; ++l) ok = cudaStreamCreateWithFlags(&q.lane[l], cudaStreamNonBlocking) == cudaSuccess;
        if (!ok) { (void)cudaGetLastError(); return false; }   // streams made so far leak, on CUDA failure only
        q.ok = true;
    }
    *up = q.upload;
    if (meta) *meta = q.meta;
    *st = q.lane[q.next];
    q.next = (q.next + 1u) % kLanes;
    return true;
}

bool hash_lane(int device, cudaStream_t *hs, cudaEvent_t *hashed) {
    if (device < 0 || device >= kMaxDevices) return false;
    std::lock_guard<std::mutex> lock(g_queues_mu);
    HashLanes &h = g_hash[device];
    if (!h.ok) {
        for (int i = 0; i < kHashLanes; ++i)
            if ((!h.s[i] && cudaStreamCreateWithFlags(&h.s[i], cudaStreamNonBlocking) != cudaSuccess) ||
                (!h.e[i] && cudaEventCreateWithFlags(&h.e[i], cudaEventDisableTiming) != cudaSuccess)) {
                (void)cudaGetLastError();
                return false;   // what was made so far is kept for the next try
            }
        h.ok = true;
    }
    *hs = h.s[h.next];
    *hashed = h.e[h.next];
    h.next = (h.next + 1u) % kHashLanes;
    return true;
}

uint32_t Workspace::take_token(size_t records, cudaStream_t s) {
    const size_t bytes = std::max<size_t>(records, 1) * 4;
    if (bytes > dflags.cap || token == 0xffffffffu) {   // new words (or tokens exhausted): zero them first
        if (!dflags.grow(bytes) || !htoken.grow(16) || cudaMemsetAsync(dflags.p, 0, dflags.cap, s) != cudaSuccess ||
            wait_stream(s) != Waited::Done) {
            (void)cudaGetLastError();
            token = 0xffffffffu;   // zero again on the next call
            return 0;
        }
        token = 0;
    }
    ++token;
    *reinterpret_cast<uint32_t *>(htoken.p) = token;   // no copy of an earlier call from it is in flight
    return token;
}

Workspace *workspace_take(int device) {
    if (device < 0 || device >= kMaxDevices) return nullptr;
    {
        std::lock_guard<std::mutex> lock(g_pool_mu);
        std::vector<Workspace *> &parked = g_parked[device];
        for (size_t i = 0; i < parked.size();) {
            if (cudaEventQuery(parked[i]->done) == cudaSuccess) {
                g_idle[device].push_back(parked[i]);
                parked[i] = parked.back();
                parked.pop_back();
            } else {
                ++i;
            }
        }
        (void)cudaGetLastError();
        if (!g_idle[device].empty()) {
            Workspace *w = g_idle[device].back();
            g_idle[device].pop_back();
            return w;
        }
    }
    return fresh(device);
}

void workspace_give(Workspace *w, bool settled) {
    if (!w) return;
    std::lock_guard<std::mutex> lock(g_pool_mu);
    (settled ? g_idle : g_parked)[w->device].push_back(w);
}

}  // namespace wexb
