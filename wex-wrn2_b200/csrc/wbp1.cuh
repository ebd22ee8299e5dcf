// WBP1 (codec 6, byte-plane rANS for non-expert tensors) on sm_100a: shared host/device structures.
//
// Semantics follow the reference CPU decoder wex4_bp_decode (c/wex4.h:527-577): the decoded bytes are
// elements of P bytes, plane p is byte p of every element; a plane is either order-0 rANS (the WNR3
// scale-stream coder with a 257-entry CDF carried in the record, streams of at most 2^chunk_log2
// symbols starting at L + h23) or raw, with one MurmurHash3 word per chunk. Transform 1 rotates every
// little-endian element right by one bit after the planes are joined. One thread decodes or checks one
// stream / chunk into a plane-major scratch; a second kernel joins the planes into the output.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace wexb {

constexpr uint32_t kWbp1Magic = 0x31504257u;   // "WBP1"
constexpr int kWbp1Threads = 256;

// One record of a launch, in device memory.
struct Wbp1Record {
    const uint8_t *rec;        // the stored record (4-byte aligned)
    const uint32_t *offsets;   // absolute record offset of every stream / chunk of every plane, then the end
    uint8_t *planes;           // plane-major scratch: plane p at plane_at[p]
    uint8_t *out;              // decoded bytes (decoded)
    uint32_t *error;           // error bits (cleared by the host)
    uint32_t decoded, P, chunk, mask, transform, owner, ident3;
    uint32_t n[8], gbase[8], cdf_at[8], table_at[8];   // per plane: bytes, first global stream, CDF and table offsets
    uint64_t plane_at[8];
};

// A CTA's work: streams [first, first + count) of one plane of one record (count <= kWbp1Threads).
struct Wbp1Task {
    uint32_t rec, plane, first, count;
};

cudaError_t launch_wbp1_streams(const Wbp1Record *recs, const Wbp1Task *tasks, uint32_t ntasks, cudaStream_t st);
// Joins the planes of records [0, nrecs) into their outputs (and undoes transform 1).
cudaError_t launch_wbp1_join(const Wbp1Record *recs, uint32_t nrecs, cudaStream_t st);
cudaError_t prepare_wbp1_kernels();

}  // namespace wexb
