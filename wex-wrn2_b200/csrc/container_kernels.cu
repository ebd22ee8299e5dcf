// RAW-record padding check on the GPU, and the probe of the bounded mbarrier wait (see container.cuh).
#include "container.cuh"
#include "rans_device.cuh"

namespace wexb {
namespace {

__global__ void zero_check(const ZeroJob *__restrict__ jobs) {
    const ZeroJob J = jobs[blockIdx.y];
    uint32_t any = 0;
    for (uint64_t i = J.begin + (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < J.end; i += (uint64_t)gridDim.x * blockDim.x)
        any |= J.base[i];
    if (__syncthreads_or(any) && threadIdx.x == 0) atomicOr(J.error, J.bit);
}

__global__ void wait_probe(uint32_t arrivals, uint32_t polls, uint32_t *bits) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) rans::mbar_init(&bar, 1);
    __syncthreads();
    if (threadIdx.x == 0 && arrivals)
        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" :: "r"((unsigned)__cvta_generic_to_shared(&bar)) : "memory");
    const bool done = rans::mbar_wait(&bar, 0, polls);
    if (threadIdx.x == 0) *bits = done ? 0u : kErrTimeout;
}

}  // namespace

cudaError_t launch_wait_probe(uint32_t arrivals, uint32_t polls, uint32_t *bits, cudaStream_t st) {
    wait_probe<<<1, 32, 0, st>>>(arrivals, polls, bits);
    return cudaGetLastError();
}

cudaError_t launch_zero_check(const ZeroJob *jobs, uint32_t n, cudaStream_t st) {
    if (!n) return cudaSuccess;
    zero_check<<<dim3(4, n), 256, 0, st>>>(jobs);
    return cudaGetLastError();
}

}  // namespace wexb
