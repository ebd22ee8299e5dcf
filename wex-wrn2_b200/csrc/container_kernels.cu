// RAW-record padding check on the GPU (see container.cuh).
#include "container.cuh"

namespace wexb {
namespace {

__global__ void zero_check(const ZeroJob *__restrict__ jobs) {
    const ZeroJob J = jobs[blockIdx.y];
    uint32_t any = 0;
    for (uint64_t i = J.begin + (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < J.end; i += (uint64_t)gridDim.x * blockDim.x)
        any |= J.base[i];
    if (__syncthreads_or(any) && threadIdx.x == 0) atomicOr(J.error, J.bit);
}

}  // namespace

cudaError_t launch_zero_check(const ZeroJob *jobs, uint32_t n, cudaStream_t st) {
    if (!n) return cudaSuccess;
    zero_check<<<dim3(4, n), 256, 0, st>>>(jobs);
    return cudaGetLastError();
}

}  // namespace wexb
