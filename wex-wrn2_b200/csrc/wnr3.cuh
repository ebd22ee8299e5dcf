// WNR2/WNR3 record decode on sm_100a: shared host/device structures and the kernel launchers.
//
// Semantics follow the reference CPU decoder wex_nr2_decode (c/wex_neural_rans.h:468-521): per
// stream a 32-bit rANS state (L = 2^23, 14-bit CDFs, byte renormalisation, 4-byte big-endian
// initial state), scale streams with one 256-symbol CDF per matrix, weight streams with the
// 567-context rule, WNR3 per-stream MurmurHash3 end states, canonical-zero refusal and the
// ceil-form inverse. One CUDA thread decodes one stream; streams of every record of a launch are
// spread over CTAs that each serve one matrix of one record.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace wexb {

constexpr uint32_t kRansL = 1u << 23;
constexpr uint32_t kPrec = 14;
constexpr uint32_t kTotal = 1u << kPrec;
constexpr uint32_t kContexts = 567;
constexpr uint32_t kModelBytes = 32u + 3u * kContexts * 34u + 3u * 514u;   // 59,408

// error word bits (the reference's c/wex_cuda.cuh:295-298, plus a bounded-wait timeout)
constexpr uint32_t kErrStruct = 1, kErrHash = 2, kErrCeil = 4, kErrCz = 8, kErrTimeout = 16;
// Every wait inside a kernel (on an mbarrier, a flag or a counter) gives up after this many polls and
// sets kErrTimeout; the self-test entry point accepts at most this many polls as well.
constexpr uint32_t kWaitPolls = 1u << 24;

// Per model, per device: lookup tables derived from the WNM2 blob on the host.
//
// Weight contexts. The reference's context (srel * 9 + pm) * 9 + mx (c/wex_neural_rans.h:130-133, 498-512)
// only ever takes pm <= mx < 8 (pm the previous magnitude, mx the block's maximum so far) or the
// block start pm = mx = 8, so each srel has 37 reachable contexts: pair index mx (mx + 1) / 2 + pm,
// and 36 for the block start. The tables hold those 7 x 37 = 259 contexts of each matrix:
//   level 1 [259] of 8 B   cdf[4] | cdf[8] << 16,  cdf[12] | 2^14 << 16   (picks the quartile q; its
//                          fields are also cdf[4q + 4], the end of quartile q)
//   level 2 [259][4] of 8 B, quartile q: cdf[4q] | cdf[4q+1] << 16,  cdf[4q+2] | cdf[4q+3] << 16
//   ssym[m][slot]    the scale symbol owning slot (16,384 B per matrix)
//   scdf[m]          the scale CDF cdf[0..256] (u16), padded to 528 B
struct Nr3Tables {
    const uint8_t *wblk;
    const uint8_t *ssym;
    const uint16_t *scdf;
};
constexpr uint32_t kPairs = 37;                                        // contexts per srel
constexpr uint32_t kWContexts = 7u * kPairs;                           // 259
constexpr uint32_t kWL1Bytes = (kWContexts * 8u + 15u) & ~15u;         // 2,080
constexpr uint32_t kWBlockBytes = kWL1Bytes + kWContexts * 32u;        // 10,368 per matrix
constexpr size_t kWTableBytes = 3ull * kWBlockBytes;
constexpr size_t kSsymBytes = 3ull * kTotal;
constexpr uint32_t kScdfBytes = 528;   // 257 u16, padded to a multiple of 16 B
constexpr size_t kTableBytes = kWTableBytes + kSsymBytes + 3ull * kScdfBytes;

// One record of a launch, in device memory.
struct Nr3Record {
    const uint8_t *rec;        // the stored record (4-byte aligned)
    const uint32_t *offsets;   // absolute record offset of every stream, then the end: [streams + 1]
    uint8_t *out;              // decoded slab, decode layout: scales at soff[m], weights at wout[m]
    uint32_t *error;           // error bits of this record (cleared by the host before the launch)
    Nr3Tables t;
    uint32_t scount[3], wcount[3];   // scales / 4-bit weights of matrix m
    uint32_t soff[3], wout[3];       // their offsets in out (wout 16-byte aligned)
    uint32_t schunk, wchunk;         // symbols per stream
    uint32_t sbase[3], wbase[3];     // global index g of matrix m's first scale / weight stream
    uint32_t model_id, owner, word24;
    uint32_t flags;                  // bits 0-2 ceil mask, bit 3 canonical zero, bit 8 WNR3 (else WNR2)
    uint32_t pad;
};

// A CTA's work: streams [first, first + count) of one matrix of one record (stream index inside
// the matrix). count <= blockDim.x.
struct Nr3Task {
    uint32_t rec, matrix, first, count;
};

// Commit: copy a decoded record's six regions to the caller's buffers only if its error word is 0
// (the reference's c/wex_cuda.cuh:841-860 contract: destinations untouched on failure).
struct CommitJob {
    const uint8_t *src[6];
    uint8_t *dst[6];
    uint32_t bytes[6];
    const uint32_t *error;
};

constexpr int kScaleThreads = 128;
constexpr int kWeightThreadsMax = 256;   // weight CTAs have 128 or 256 threads (WEXB_WEIGHT_THREADS)

cudaError_t launch_nr3_scales(const Nr3Record *recs, const Nr3Task *tasks, uint32_t ntasks, cudaStream_t st);
cudaError_t launch_nr3_weights(const Nr3Record *recs, const Nr3Task *tasks, uint32_t ntasks, int threads,
                               cudaStream_t st);
cudaError_t launch_commit(const CommitJob *jobs, uint32_t njobs, cudaStream_t st);
cudaError_t prepare_nr3_kernels();   // sets the shared-memory opt-ins on the current device

}  // namespace wexb
