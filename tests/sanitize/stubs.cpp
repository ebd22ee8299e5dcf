// Host-only stand-ins for the kernel launchers, so that the library's host sources link into a
// sanitizer build without nvcc. The harness (fuzz_host.cpp) calls only host parsers; a launcher
// reached anyway reports "not supported", as a device without these kernels would.
#include "container.cuh"
#include "encode.cuh"
#include "sha256.cuh"
#include "wbp1.cuh"
#include "wnr3.cuh"
#include "wnr4.cuh"

namespace wexb {
cudaError_t launch_zero_check(const ZeroJob *, uint32_t, cudaStream_t) { return cudaErrorNotSupported; }
cudaError_t launch_wait_probe(uint32_t, uint32_t, uint32_t *, cudaStream_t) { return cudaErrorNotSupported; }
cudaError_t launch_encode(const uint8_t *, EncRecord *, uint32_t, uint32_t, const EncTask *, uint32_t, const uint32_t *,
                          uint32_t, cudaStream_t) { return cudaErrorNotSupported; }
cudaError_t launch_count(EncRecord *, uint32_t, const CountTask *, uint32_t, unsigned long long *, unsigned long long *,
                         cudaStream_t) { return cudaErrorNotSupported; }
cudaError_t launch_sha256_messages(const ShaMsg *, uint32_t, cudaStream_t) { return cudaErrorNotSupported; }
cudaError_t launch_sha256_parts(const ShaParts &, cudaStream_t) { return cudaErrorNotSupported; }
cudaError_t launch_sha256_segments(const ShaMsg *, uint32_t, uint8_t *, cudaStream_t) { return cudaErrorNotSupported; }
cudaError_t launch_wbp1_streams(const Wbp1Record *, const Wbp1Task *, uint32_t, cudaStream_t) { return cudaErrorNotSupported; }
cudaError_t launch_wbp1_join(const Wbp1Record *, uint32_t, cudaStream_t) { return cudaErrorNotSupported; }
cudaError_t prepare_wbp1_kernels() { return cudaErrorNotSupported; }
cudaError_t launch_nr3(const Nr3Launch &, int, cudaStream_t, bool) { return cudaErrorNotSupported; }
cudaError_t prepare_nr3_kernels() { return cudaErrorNotSupported; }
cudaError_t launch_wnr4(const W4Tables &, const W4Job *, uint32_t, const W4Rec *, cudaStream_t) { return cudaErrorNotSupported; }
}  // namespace wexb
