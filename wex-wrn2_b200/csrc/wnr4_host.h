// Host side of the WNR4 kind-MX decoder shared by the WNR4 ABI (wnr4_abi.cpp) and the WEX4 container
// check (wex4_api.cpp): model tables, slab geometry, record planning.
#pragma once
#include <cstddef>
#include <cstdint>
#include <vector>

#include "wnr4.cuh"

namespace wexb {

// Geometry of a kind-MX expert slab from its 13 words {kind, scount[3], scols[3], soff[3], woff[3]}
// (wnr4/wnr4.h:108-140).
struct W4Geo { uint32_t scount[3], scols[3]; };
bool wnr4_geo(const uint32_t *v, W4Geo *g);

// The device tables of a kind-MX WNM4 blob on `device`, registered once per model and device, and
// its id (FNV-1a, 0 read as 1): 0, -1 for an invalid blob, 1 on a CUDA failure.
int wnr4_tables(const uint8_t *blob, size_t bytes, int device, W4Tables *tab, uint32_t *id);

// One record's header, tile table, owner and model checks (wnr4/wnr4.h:317-346); appends its tiles
// (matrix by matrix) to jobs[m] with drec = the record's device copy and fills info (all but the
// destinations and the error word). False when the record is refused.
bool wnr4_plan(const uint8_t *rec, size_t total, const W4Geo &g, uint32_t owner, uint32_t model_id, const uint8_t *drec,
               uint32_t index, W4Rec *info, std::vector<W4Job> jobs[3]);

// Launch order of a batch: each matrix's tiles padded to whole CTAs.
std::vector<W4Job> wnr4_launch_order(const std::vector<W4Job> by_m[3]);

}  // namespace wexb
