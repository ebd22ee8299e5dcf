// WNR4 kind MX (draft codec 8 of the reference, wnr4/wnr4.h) on sm_100a: shared host/device structures.
//
// A record is a list of tiles; a tile is 32 rANS lanes (32-bit states, L = 2^16, 16-bit
// renormalisation) sharing one stream of u16 words, taken in lane order by the lanes that renormalise
// at each lockstep step. One warp decodes one tile (wnr4_kernel.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace wexb {

constexpr uint32_t kW4L = 0x10000u;
constexpr uint32_t kW4Classes = 7;           // MX: scale class = clamp(scale - anchor, -3, 3) + 3
constexpr uint32_t kW4Err = 1, kW4ErrHash = 2, kW4ErrCeil = 4, kW4ErrCz = 8;
constexpr uint32_t kW4ErrTimeout = 16;   // a bounded wait gave up (the host reports status 1)

// Per model and device, per matrix: the weight rows of the reachable contexts, then the scale block.
// A weight context (cls * 9 + pm) * 9 + mx (wnr4/wnr4.h, kind MX) only takes pm <= mx < 8 or the block
// start pm = mx = 8: 37 pairs per class (pair index mx (mx + 1) / 2 + pm, 36 for the block start), and
// pb position buckets each (pb = 5: bucket k - 27 for the last four nibbles of a cell). Row index
// (cls * 37 + pair) * pb + bucket, rows = 7 * 37 * pb:
//   level 1 [rows] of 8 B    cdf[4] | cdf[8] << 16,  cdf[12] | 2^14 << 16   (padded to 16 B)
//   level 2 [rows][4] of 8 B quartile q: cdf[4q] | cdf[4q+1] << 16,  cdf[4q+2] | cdf[4q+3] << 16
// The scale block: the coarse row cdf[0], cdf[16], .., cdf[240], then the scale CDF cdf[0..256] (u16).
struct W4Tables {
    const uint8_t *base;   // [3][matrix_bytes]
    uint32_t rows, pb, matrix_bytes, id;
};
constexpr uint32_t kW4Pairs = 37;
constexpr uint32_t kW4ScaleBlock = 32u + 514u + 30u;   // coarse row, cdf[0..256], padding to a multiple of 16 B
__host__ __device__ inline uint32_t w4_rows(uint32_t pb) { return kW4Classes * kW4Pairs * pb; }
__host__ __device__ inline uint32_t w4_l1_bytes(uint32_t rows) { return (rows * 8u + 15u) & ~15u; }
__host__ __device__ inline uint32_t w4_matrix_bytes(uint32_t rows) { return w4_l1_bytes(rows) + rows * 32u + kW4ScaleBlock; }

// One record of a batch.
struct W4Rec {
    uint32_t model_id, owner, flags, G, anchors;
    uint32_t *error;
    uint8_t *dst_s[3], *dst_w[3];
};

// One tile: the warp's work.
struct W4Job {
    const uint8_t *tile;   // its 32 initial states (u32 LE), then its words (u16 LE)
    uint32_t nwords, rec, t, m, c0, n;
};

constexpr int kW4Warps = 4;   // warps (tiles) per CTA; a CTA's tiles share one matrix

cudaError_t launch_wnr4(const W4Tables &tab, const W4Job *jobs, uint32_t njobs, const W4Rec *recs, cudaStream_t st);

}  // namespace wexb
