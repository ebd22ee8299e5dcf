// Host side of WBP1 (codec 6): record validation and planning for the GPU decoder, and the
// canonical encoder.
#pragma once
#include <cstddef>
#include <cstdint>
#include <vector>

#include "wbp1.cuh"

namespace wexb {

// A validated WBP1 record (c/wex4.h:487-525): per plane its byte count, streams, and where its CDF,
// stream table and payload start in the record.
struct Wbp1Plan {
    uint32_t decoded = 0, P = 0, chunk = 0, chunk_log2 = 0, mask = 0, transform = 0, owner = 0;
    uint32_t n[8] = {}, streams[8] = {}, gbase[8] = {}, cdf_at[8] = {}, table_at[8] = {}, payload_at[8] = {};
    uint32_t total_streams = 0;
};

// 0 when rec (total bytes) is a valid WBP1 record of `decoded` bytes owned by `owner`, else -1; the
// checks and their order are the reference's.
int wbp1_parse(const uint8_t *rec, size_t total, uint32_t decoded, uint32_t owner, Wbp1Plan *b);
// The absolute record offset of every stream / chunk (global numbering), then the end: total_streams + 1.
void wbp1_offsets(const Wbp1Plan &b, const uint8_t *rec, uint32_t *offsets);
// CTA tasks of one record (index rec in its launch).
void wbp1_tasks(const Wbp1Plan &b, uint32_t rec, std::vector<Wbp1Task> &tasks);
// Plane-major scratch bytes of a record (each plane 16-byte aligned) and the plane offsets.
uint64_t wbp1_scratch(const Wbp1Plan &b, uint64_t plane_at[8]);
// The device descriptor of a planned record.
Wbp1Record wbp1_descriptor(const Wbp1Plan &b, const uint8_t *drec, const uint32_t *doffsets, uint8_t *dplanes,
                           uint8_t *dout, uint32_t *derror);
// Sets the kernels' shared-memory opt-in on the current device (once per device).
bool wbp1_prepare(int device);

// The canonical encoder (c/wex4.h:579-660): the padded record of `decoded` bytes in elements of P
// bytes, streams of 2^chunk_log2, transform 0 or 1; 0 and *written, or -1.
int wbp1_encode(const uint8_t *data, uint32_t decoded, uint32_t P, uint32_t chunk_log2, uint32_t transform, uint32_t owner,
                uint8_t *out, size_t capacity, size_t *written);

}  // namespace wexb
