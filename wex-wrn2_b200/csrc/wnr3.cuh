// WNR2/WNR3 record decode on sm_100a: shared host/device structures and the kernel launcher.
//
// Semantics follow the reference CPU decoder wex_nr2_decode (c/wex_neural_rans.h:468-521): per
// stream a 32-bit rANS state (L = 2^23, 14-bit CDFs, byte renormalisation, 4-byte big-endian
// initial state), scale streams with one 256-symbol CDF per matrix, weight streams with the
// 567-context rule, WNR3 per-stream MurmurHash3 end states, canonical-zero refusal and the
// ceil-form inverse. One lane decodes one stream. A launch is one persistent grid (a CTA per SM,
// every table of the model in its shared memory) whose warps drain a work queue of scale, weight and
// commit items (nr3_decode.cu).
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
constexpr uint32_t kErrRecordSha = 32;   // verified batches: the record's SHA-256 differs from the index's
// Every wait inside a kernel (on an mbarrier, a flag or a counter) gives up after this many polls and
// sets kErrTimeout; the self-test entry point accepts at most this many polls as well.
constexpr uint32_t kWaitPolls = 1u << 24;

// Per model, per device: lookup tables derived from the WNM2 blob on the host, one block of
// kTableBytes that a decode CTA stages whole into its shared memory.
//
// Weight contexts. The reference's context (srel * 9 + pm) * 9 + mx (c/wex_neural_rans.h:130-133, 498-512)
// only ever takes pm <= mx < 8 (pm the previous magnitude, mx the block's maximum so far) or the
// block start pm = mx = 8, so each srel has 37 reachable contexts: pair index mx (mx + 1) / 2 + pm,
// and 36 for the block start. The tables hold those 7 x 37 = 259 contexts of each matrix:
//   level 1 [259] of 8 B   cdf[4] | cdf[8] << 16,  cdf[12] | 2^14 << 16   (picks the quartile q; its
//                          fields are also cdf[4q + 4], the end of quartile q)
//   level 2 [259][4] of 8 B, quartile q: cdf[4q] | cdf[4q+1] << 16,  cdf[4q+2] | cdf[4q+3] << 16
// Scales (256 symbols, one CDF per matrix):
//   ssym[m][slot]    the symbol owning slot (16,384 B per matrix)
//   sf[m][sym]       cdf[sym] | (cdf[sym + 1] - cdf[sym]) << 16 (256 words per matrix)
// Layout: wblk[3][kWBlockBytes], ssym[3][16384], sf[3][256] words.
constexpr uint32_t kPairs = 37;                                        // contexts per srel
constexpr uint32_t kWContexts = 7u * kPairs;                           // 259
constexpr uint32_t kWL1Bytes = (kWContexts * 8u + 15u) & ~15u;         // 2,080
constexpr uint32_t kWBlockBytes = kWL1Bytes + kWContexts * 32u;        // 10,368 per matrix
constexpr size_t kWTableBytes = 3ull * kWBlockBytes;
constexpr size_t kSsymBytes = 3ull * kTotal;
constexpr uint32_t kSfBytes = 256u * 4u;                               // per matrix
constexpr size_t kTableBytes = kWTableBytes + kSsymBytes + 3ull * kSfBytes;   // 83,328

// Commit: copy a decoded record's six regions to the caller's buffers only if its error word is 0
// (the reference's c/wex_cuda.cuh:841-860 contract: destinations untouched on failure).
struct CommitJob {
    const uint8_t *src[6];
    uint8_t *dst[6];
    uint32_t bytes[6];
};
constexpr uint32_t kCommitChunk = 128u << 10;   // bytes of a region one commit item copies

// One record of a launch, in device memory.
struct Nr3Record {
    const uint8_t *rec;        // the stored record (4-byte aligned, readable 16 bytes past its end)
    const uint32_t *offsets;   // absolute record offset of every stream, then the end: [streams + 1]
    uint8_t *out;              // decoded slab, decode layout: scales at soff[m], weights at wout[m]
    uint32_t *error;           // error bits of this record (zero when the launch starts)
    const CommitJob *job;      // the error-gated copy to the caller's buffers, or null (none)
    const uint32_t *landed;    // reaches landed_at once the record's upload has landed, or null (already there)
    uint32_t scount[3], wcount[3];   // scales / 4-bit weights of matrix m
    uint32_t soff[3], wout[3];       // their offsets in out (wout 16-byte aligned)
    uint32_t schunk, wchunk;         // symbols per stream
    uint32_t sbase[3], wbase[3];     // global index g of matrix m's first scale / weight stream
    uint32_t model_id, owner, word24;
    uint32_t flags;                  // bits 0-2 ceil mask, bit 3 canonical zero, bit 8 WNR3 (else WNR2)
    uint32_t sitems[3];              // scale items of matrix m (32 streams each)
    uint32_t witems;                 // weight items of the record (32 streams each, every matrix)
    uint32_t landed_at;              // the value the upload stream writes into *landed (never 0)
};

// The launch's work queue. A warp takes the next item (one atomic on the head counter) and runs it:
//   scale item   32 scale streams [first, first + 32) of matrix `sub`; a record still being uploaded
//                is waited for (bounded) first: after its bytes the upload stream copies the call's
//                token (landed_at, larger than any token of an earlier call) into its `landed` word
//   weight item  32 weight streams of matrix `sub`; it first waits until every scale item of that
//                matrix of its record is done (the streams' contexts read the decoded scales)
//   commit item  chunk `first` (kCommitChunk bytes) of region `sub` of the record's commit; it first
//                waits until every weight item of its record is done, then copies only if the
//                record's error word is 0
// Items only ever wait for items earlier in the queue, so the queue always drains.
constexpr uint32_t kItemScale = 0, kItemWeight = 1, kItemCommit = 2;
struct Nr3Item {
    uint32_t rec;    // index into the launch's records
    uint32_t what;   // kind << 28 | sub << 24 | first
};
__host__ __device__ constexpr uint32_t item_what(uint32_t kind, uint32_t sub, uint32_t first) {
    return kind << 28 | sub << 24 | first;
}

// One persistent launch: records of one model. Counters (zero when the launch starts): head, then
// per record j: done[4 j + m] = finished scale items of matrix m, done[4 j + 3] = finished weight items.
struct Nr3Launch {
    const Nr3Record *recs;
    const Nr3Item *items;
    uint32_t *head;
    uint32_t *done;
    const uint8_t *tables;     // the model's device tables (kTableBytes, 16-byte aligned)
    uint32_t nitems, nrecs;
};

// Threads of a decode CTA (one CTA per SM, persistent; 64 registers each, the whole register file).
constexpr int kDecodeThreads = 1024;
// Threads of a decode CTA beside record hashes: the register file then keeps room for two hash CTAs
// (64 threads of at most 72 registers), so a launch is never held back behind hash CTAs that run for
// the length of a whole record's SHA-256 chain.
constexpr int kBesideHashThreads = 832;

// One launch on `st`: one CTA per SM of the current device (`sms`), or, beside_hashes, CTAs of
// kBesideHashThreads threads on half of the SMs.
cudaError_t launch_nr3(const Nr3Launch &L, int sms, cudaStream_t st, bool beside_hashes = false);
cudaError_t prepare_nr3_kernels();   // sets the shared-memory opt-in on the current device

}  // namespace wexb
