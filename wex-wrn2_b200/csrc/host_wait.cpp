// Deadline-bounded host waits (host_wait.h).
#include "host_wait.h"

#include <atomic>
#include <chrono>
#include <cstdlib>
#include <thread>

namespace wexb {
namespace {

double initial_limit() {
    const char *v = std::getenv("WEXB_WAIT_SECONDS");
    if (v && *v) {
        char *end = nullptr;
        const double s = std::strtod(v, &end);
        if (end != v && s > 0) return s;
    }
    return 60.0;
}
std::atomic<double> g_limit{initial_limit()};

inline void cpu_relax() {
#if defined(__x86_64__) || defined(__i386__)
    __builtin_ia32_pause();
#elif defined(__aarch64__)
    asm volatile("yield" ::: "memory");
#endif
}

// Polls `query` until the deadline: spinning for the first 100 us, then yielding the core between
// polls up to 5 ms (no sleep latency while the core is free, and the core is shared while other
// threads, such as the other ranks' submitting threads on a busy host, want it), then sleeping 20 us
// between polls.
template <class Query>
Waited poll(Query query, double seconds) {
    using clock = std::chrono::steady_clock;
    const auto start = clock::now();
    for (unsigned i = 0;; ++i) {
        const cudaError_t e = query();
        if (e == cudaSuccess) return Waited::Done;
        if (e != cudaErrorNotReady) { (void)cudaGetLastError(); return Waited::Failed; }
        if ((i & 7u) != 7u) { cpu_relax(); continue; }
        const double elapsed = std::chrono::duration<double>(clock::now() - start).count();
        if (elapsed > seconds) return Waited::TimedOut;
        if (elapsed > 5e-3) std::this_thread::sleep_for(std::chrono::microseconds(20));
        else if (elapsed > 1e-4) std::this_thread::yield();
    }
}

}  // namespace

double wait_limit() { return g_limit.load(std::memory_order_relaxed); }
void set_wait_limit(double seconds) { if (seconds > 0) g_limit.store(seconds, std::memory_order_relaxed); }

Waited wait_event(cudaEvent_t e, double seconds) { return poll([e] { return cudaEventQuery(e); }, seconds); }
Waited wait_stream(cudaStream_t s, double seconds) { return poll([s] { return cudaStreamQuery(s); }, seconds); }

KeepDevice::KeepDevice() {
    if (cudaGetDevice(&entry_device_) != cudaSuccess) { (void)cudaGetLastError(); entry_device_ = -1; }
}
KeepDevice::~KeepDevice() {
    if (entry_device_ < 0) return;
    int now = -1;
    if (cudaGetDevice(&now) != cudaSuccess || now != entry_device_) (void)cudaSetDevice(entry_device_);
    (void)cudaGetLastError();
}

}  // namespace wexb
