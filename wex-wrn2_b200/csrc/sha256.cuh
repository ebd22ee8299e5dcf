// SHA-256 kernels (sha256.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace wexb {

// One message (or, for the segment kernel, one piece of a message) in device memory.
struct ShaMsg {
    const uint8_t *data;
    uint64_t bytes;
    uint8_t *digest;          // optional: the 32-byte digest
    const uint8_t *expect;    // optional: a 32-byte digest to compare with
    uint32_t *verdict;        // optional: 0 equal (or no expect), 1 differs
    uint32_t or_bits;         // non-zero: on a difference OR these bits into *verdict, else leave it
};

// Digests and verdicts of n messages (each 16-byte aligned).
cudaError_t launch_sha256_messages(const ShaMsg *msgs, uint32_t n, cudaStream_t st);
// The same for up to kShaParts arrays of messages in one launch (say the records of several calls):
// messages [end[p - 1], end[p]) of the launch are part[p][0 ..] (end[-1] = 0).
//
// gate (optional): the messages are still being uploaded, in passes of 2^gate_shift bytes of every
// message (a multiple of 64); bytes [q 2^gate_shift, (q + 1) 2^gate_shift) of any message are in place
// once gate[q] >= gate_token (the upload stream copies the token there after pass q). The launch may
// then start before the uploads: each chain waits (bounded) for the pass it is about to read, so every
// record's chain starts with its first bytes instead of after the whole upload. A wait that gives up
// sets *gate_fail to 1 (the launch's digests are then meaningless).
constexpr int kShaParts = 16;
struct ShaParts {
    const ShaMsg *part[kShaParts];
    uint32_t end[kShaParts];
    uint32_t nparts;
    const uint32_t *gate;
    uint32_t gate_token, gate_shift;
    uint32_t *gate_fail;
};
cudaError_t launch_sha256_parts(const ShaParts &P, cudaStream_t st);
// One thread: the digest of the concatenation of n segments (data and bytes used).
cudaError_t launch_sha256_segments(const ShaMsg *segs, uint32_t n, uint8_t *digest, cudaStream_t st);

}  // namespace wexb
