// Kernels of the WEX4 container layer besides SHA-256 (container_kernels.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace wexb {

// A RAW record's padding [begin, end) must be zero (c/wex4.h:678-682); any non-zero byte ORs `bit`
// into *error.
struct ZeroJob {
    const uint8_t *base;
    uint64_t begin, end;
    uint32_t *error;
    uint32_t bit;
};
cudaError_t launch_zero_check(const ZeroJob *jobs, uint32_t n, cudaStream_t st);

// The bounded wait every kernel puts on its shared-memory mbarriers, run on a barrier that expects one
// arrival: after `arrivals` arrivals (0 or 1), a wait of at most `polls` polls. bits[0] receives the
// timeout bit (16) when the wait gave up, else 0.
cudaError_t launch_wait_probe(uint32_t arrivals, uint32_t polls, uint32_t *bits, cudaStream_t st);
// The self-test's largest poll count: the kernels' own limit (kWaitPolls, wnr3.cuh).
constexpr uint32_t kSelftestMaxPolls = 1u << 24;

}  // namespace wexb
