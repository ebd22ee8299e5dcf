// GPU writer side of WNR3 / WNR2 records: the training counts of a WNM2 model and the record encoder,
// byte-identical to the reference encoder (c/wex_neural_rans.h:579-613 counts, :615-749 encoder).
//
// Encoder: one thread per stream. A stream's initial state is the MurmurHash3 of its ident words and
// its bytes (WNR3; WNR2 starts at L); its symbols are coded last to first into the stream's own
// scratch slot, bytes written downwards from the slot's end. A second kernel scans the stream lengths of
// each record, writes the header and the length table, and a third packs the payloads behind them.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace wexb {

constexpr uint32_t kEncContexts = 567;       // weight contexts of a WNM2 model: (srel * 9 + prev) * 9 + top
constexpr uint32_t kEncCdfRow = 17;          // u16 entries per weight-context CDF row
constexpr int kEncThreads = 128;             // streams per encoder CTA
constexpr uint32_t kEncErrCz = 1, kEncErrOverflow = 2;

// One record to encode. The coded slab is in device memory, canonical layout (scales m at soff[m],
// packed weights m at woff[m]).
struct EncRecord {
    const uint8_t *coded;
    uint32_t soff[3], woff[3], scount[3], wcount[3];
    uint32_t sbase[3], wbase[3];   // first stream (g) of each matrix's scale / weight streams
    uint32_t streams, schunk, wchunk, nr3, cz;
    uint32_t model_id, owner, flags;
    uint8_t anchor[3];             // set on the device by the anchor kernel
    uint8_t *scratch;              // streams slots of slot_bytes; a stream ends at its slot's end
    uint32_t slot_bytes;
    uint32_t *lens;                // [streams] stream lengths, then [streams] offsets in the record
    uint32_t *err;                 // error bits of the record
    uint8_t *out;                  // the record, cap bytes
    uint64_t cap, raw_aligned;
    uint64_t *result;              // [0] status (0, 1 RAW, -1 as uint64), [1] used, [2] total
};
// One encoder CTA: up to kEncThreads streams of one matrix of one record.
struct EncTask {
    uint32_t rec, m, scale, first, count;   // first: stream index within the matrix's scale or weight streams
};
// One counting CTA: weight blocks [first, first + count) of matrix m (32 nibbles a block), or its scales.
struct CountTask {
    uint32_t rec, m, scale, first, count;
};

// The model tables the kernels read: the WNM2 blob (32-byte header, [3][567][17] weight CDFs, [3][257]
// scale CDFs), in device memory.
// Both launches first set every record's three anchors from its scales (rule g for WNR3, the lower
// median for WNR2: c/wex_neural_rans.h:399-405, :526-534).
// One group of an encode launch: records [first, first + nrec) of recs, their tasks (whose rec fields index
// recs) and their streams (stream_rec: pairs of record index into recs and stream g).
cudaError_t launch_encode(const uint8_t *dblob, EncRecord *recs, uint32_t first, uint32_t nrec, const EncTask *tasks,
                          uint32_t ntasks, const uint32_t *stream_rec, uint32_t nstreams, cudaStream_t st);
cudaError_t launch_count(EncRecord *recs, uint32_t nrec, const CountTask *tasks, uint32_t ntasks, unsigned long long *wc,
                         unsigned long long *sc, cudaStream_t st);

}  // namespace wexb
