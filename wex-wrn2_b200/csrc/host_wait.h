// Host-side waits with a deadline, and a scope that gives the calling thread its current device back.
//
// No entry point of this library blocks on the GPU without a limit: every wait polls its event or
// stream (cudaEventQuery / cudaStreamQuery) until the work is done, CUDA reports an error, or the
// process-wide limit passes (WEXB_WAIT_SECONDS, default 60 s; wexb_set_wait_limit changes it). A call
// whose wait gives up returns status 1 ("unavailable, decode again"): its GPU work may still be running,
// so the buffers that work uses are parked (never handed to another call) until it ends.
#pragma once
#include <cuda_runtime.h>

namespace wexb {

// The current limit in seconds (> 0).
double wait_limit();
void set_wait_limit(double seconds);

enum class Waited { Done, Failed, TimedOut };
// Polls until `e` has completed (Done), CUDA reports an error (Failed; the error is cleared if it is
// not sticky), or `seconds` pass (TimedOut).
Waited wait_event(cudaEvent_t e, double seconds);
inline Waited wait_event(cudaEvent_t e) { return wait_event(e, wait_limit()); }
// The same for all work queued on `s`.
Waited wait_stream(cudaStream_t s, double seconds);
inline Waited wait_stream(cudaStream_t s) { return wait_stream(s, wait_limit()); }
// Done -> true; Failed / TimedOut -> false.
inline bool waited_ok(Waited w) { return w == Waited::Done; }

// Records the calling thread's current device when constructed and makes it current again when the
// scope ends, whatever the code in between selected.
class KeepDevice {
  public:
    KeepDevice();
    ~KeepDevice();
    KeepDevice(const KeepDevice &) = delete;
    KeepDevice &operator=(const KeepDevice &) = delete;

  private:
    int entry_device_;
};

}  // namespace wexb
