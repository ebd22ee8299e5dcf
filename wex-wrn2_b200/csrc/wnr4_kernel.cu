// WNR4 kind-MX tile decode on sm_100a (structures in wnr4.cuh). Semantics: the reference CPU decoder
// wnr4_decode_tile (wnr4/wnr4.h:388-478).
//
// One warp = one tile: its 32 lanes step in lockstep; at each step the lanes whose state fell below
// L = 2^16 take the next words of the tile's shared u16 stream in lane order (ballot, then each lane's
// rank = popc of the votes below it). The words come from a 64-word register window (lane l holds
// words base + l and base + 32 + l) by shuffle; when the read position passes base + 32 the window
// slides with one coalesced 64-byte load, consumed steps later. A CTA holds kW4Warps tiles of one
// matrix, with that matrix's weight rows and scale CDF staged into shared memory by one TMA bulk copy.
// A weight symbol takes two 8-byte shared loads: the row's level-1 entry gives the quartile q from
// three packed 16-bit comparisons, the quartile's four cumulative frequencies give the rank r in it,
// and start and end are adjacent fields taken by one funnel shift (tables in wnr4.cuh).
#include "wnr4.cuh"

namespace wexb {
namespace {

constexpr uint32_t kSpinLimit = 1u << 24;
constexpr uint32_t kFull = 0xffffffffu;

__device__ __forceinline__ uint32_t rotl32(uint32_t x, int r) { return __funnelshift_l(x, x, r); }
__device__ __forceinline__ uint32_t mm3_block(uint32_t h, uint32_t k) {
    k *= 0xcc9e2d51u; k = rotl32(k, 15); k *= 0x1b873593u;
    return rotl32(h ^ k, 13) * 5u + 0xe6546b64u;
}
__device__ __forceinline__ uint32_t mm3_final(uint32_t h, uint32_t len) {
    h ^= len; h ^= h >> 16; h *= 0x85ebca6bu; h ^= h >> 13; h *= 0xc2b2ae35u; h ^= h >> 16;
    return h;
}
// Number of the 16 entries of a cumulative row (a, b: 8 packed u16 pairs, all < 2^15) that are <= slot.
__device__ __forceinline__ uint32_t row_count(const uint4 a, const uint4 b, uint32_t slot) {
    const uint32_t g = slot * 0x10001u | 0x80008000u;
    const uint32_t p0 = __byte_perm(g - a.x, g - a.y, 0x7531), p1 = __byte_perm(g - a.z, g - a.w, 0x7531);
    const uint32_t p2 = __byte_perm(g - b.x, g - b.y, 0x7531), p3 = __byte_perm(g - b.z, g - b.w, 0x7531);
    const uint32_t m = 0x80808080u;
    return (uint32_t)__popc((p0 & m) | ((p1 & m) >> 1) | ((p2 & m) >> 2) | ((p3 & m) >> 3));
}
__device__ __forceinline__ uint32_t ceil_double(uint32_t w) {   // magnitudes a -> a + min(a, 2), signs kept
    const uint32_t mag = w & 0x77777777u, two_or_more = ((mag >> 1) | (mag >> 2)) & 0x11111111u;
    return (w & 0x88888888u) | (mag + ((two_or_more << 1) | (mag & 0x11111111u & ~two_or_more)));
}

struct Window {
    const uint16_t *words;
    uint32_t nwords, base, lo, hi;
    __device__ __forceinline__ uint32_t load(uint32_t i) const { return i < nwords ? (uint32_t)__ldg(words + i) : 0u; }
};

// The lanes with `need` take their words; false when the tile has too few words (warp-uniform).
__device__ __forceinline__ bool renorm(uint32_t &x, bool need, uint32_t &ptr, Window &w, uint32_t lane) {
    const uint32_t vote = __ballot_sync(kFull, need);
    if (!vote) return true;
    const uint32_t total = __popc(vote);
    if (ptr + total > w.nwords) return false;
    const uint32_t idx = ptr - w.base + __popc(vote & ((1u << lane) - 1u));   // < 64
    const uint32_t v0 = __shfl_sync(kFull, w.lo, idx & 31u), v1 = __shfl_sync(kFull, w.hi, idx & 31u);
    if (need) x = x << 16 | (idx < 32u ? v0 : v1);
    ptr += total;
    if (ptr - w.base >= 32u) { w.lo = w.hi; w.base += 32u; w.hi = w.load(w.base + 32u + lane); }
    return true;
}

__device__ __forceinline__ bool stage(uint64_t *bar, void *dst, const void *src, uint32_t bytes) {
    const unsigned b = (unsigned)__cvta_generic_to_shared(bar);
    if (threadIdx.x == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" :: "r"(b) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" :: "r"(b), "r"(bytes) : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n"
                     :: "r"((unsigned)__cvta_generic_to_shared(dst)), "l"(src), "r"(bytes), "r"(b) : "memory");
    }
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
        uint32_t done;
        asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n selp.u32 %0, 1, 0, p;\n}\n"
                     : "=r"(done) : "r"(b) : "memory");
        if (done) return true;
    }
    return false;
}

__global__ void __launch_bounds__(kW4Warps * 32) wnr4_tiles(W4Tables tab, const W4Job *__restrict__ jobs,
                                                            const W4Rec *__restrict__ recs) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bar;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t m = jobs[blockIdx.x * kW4Warps].m;   // every tile of the CTA is of this matrix
    const W4Job J = jobs[blockIdx.x * kW4Warps + warp];
    if (!stage(&bar, smem, tab.base + (size_t)m * tab.matrix_bytes, tab.matrix_bytes)) {
        if (J.n && lane == 0) atomicOr(recs[J.rec].error, kW4Err);
        return;
    }
    if (!J.n) return;
    const W4Rec &R = recs[J.rec];
    const uint2 *level1 = reinterpret_cast<const uint2 *>(smem);
    const uint2 *level2 = reinterpret_cast<const uint2 *>(smem + w4_l1_bytes(tab.rows));
    const uint8_t *sblock = smem + w4_l1_bytes(tab.rows) + tab.rows * 32u;
    const uint4 *coarse = reinterpret_cast<const uint4 *>(sblock);
    const uint16_t *scdf = reinterpret_cast<const uint16_t *>(sblock + 32);
    const uint16_t *tile16 = reinterpret_cast<const uint16_t *>(J.tile);   // 2-byte aligned only
    uint32_t x = (uint32_t)tile16[2 * lane] | (uint32_t)tile16[2 * lane + 1] << 16;
    if (__any_sync(kFull, x < kW4L)) { if (lane == 0) atomicOr(R.error, kW4Err); return; }
    Window win{tile16 + 64, J.nwords, 0, 0, 0};
    win.lo = win.load(lane); win.hi = win.load(32u + lane);
    uint32_t ptr = 0, err = 0;
    // lane hash start: ident words {model, owner, tile, lane, kind | flags << 8 | G << 16, anchors}
    uint32_t hash = 0x34524e57u;
    hash = mm3_block(hash, R.model_id); hash = mm3_block(hash, R.owner); hash = mm3_block(hash, J.t);
    hash = mm3_block(hash, lane); hash = mm3_block(hash, R.flags << 8 | R.G << 16); hash = mm3_block(hash, R.anchors);
    uint8_t *so = R.dst_s[m];
    uint4 *wo = reinterpret_cast<uint4 *>(R.dst_w[m]);
    const uint32_t n = J.n, c0 = J.c0, rounds = (n + 31) / 32;
    // phase 1: the tile's scales, lane l owning scale c0 + 32k + l (order 0: one 256-symbol CDF)
    for (uint32_t k = 0; k < rounds; ++k) {
        const uint32_t i = 32u * k + lane;
        const bool act = i < n;
        if (act) {
            const uint32_t slot = x & 0x3fffu;
            const uint32_t g = row_count(coarse[0], coarse[1], slot) - 1u;                    // group of 16 symbols
            const uint4 *fine = reinterpret_cast<const uint4 *>(scdf + 16u * g);
            const uint32_t y = 16u * g + row_count(fine[0], fine[1], slot) - 1u;
            const uint32_t start = scdf[y], freq = scdf[y + 1] - start;
            x = freq * (x >> 14) + slot - start;
            so[c0 + i] = (uint8_t)y;
            hash = mm3_block(hash, y);
        }
        if (!renorm(x, act && x < kW4L, ptr, win, lane)) { if (lane == 0) atomicOr(R.error, kW4Err); return; }
    }
    // phase 2: rounds of 32 cells, lane l owning cell c0 + 32j + l, its 32 nibbles in order
    const bool ceil = (R.flags >> m) & 1u, cz = (R.flags & 8u) != 0;
    const int anchor = (int)((R.anchors >> (8u * m)) & 0xffu);
    for (uint32_t j = 0; j < rounds; ++j) {
        const bool active = lane < min(32u, n - 32u * j);
        const uint32_t cell = c0 + 32u * j + lane;
        const bool tail = active && lane >= 2 && j == (n - lane - 1) / 32;   // last 4 nibbles live in the state
        uint32_t scale = 0, cls = 0;
        if (active) {
            scale = so[cell];
            const int d = (int)scale - anchor;
            cls = (uint32_t)(min(max(d, -3), 3) + 3);
        }
        // the context as a row index (cls * 37 + pair) * pb + bucket; pair 36 = the block start
        const uint32_t pb = tab.pb, cls_row = cls * kW4Pairs * pb;
        uint32_t pair = kW4Pairs - 1u, top = 0, w0 = 0, w1 = 0, w2 = 0, w3 = 0;
        // four groups of 8 nibbles, one packed word each (the words rotate through w0..w3), so that only
        // 8 copies of the step are unrolled
#pragma unroll 1
        for (uint32_t g8 = 0; g8 < 4; ++g8) {
            uint32_t word = 0;
#pragma unroll
            for (uint32_t kk = 0; kk < 8; ++kk) {
                const uint32_t k = 8u * g8 + kk;
                const bool act = active && !(tail && k >= 28u);
                if (act) {
                    const uint32_t row = cls_row + pair * pb + ((k + 5u <= 32u || pb == 1u) ? 0u : k - 27u);
                    const uint2 c = level1[row];
                    const uint32_t slot = x & 0x3fffu, gs = slot * 0x10001u + 0x80008000u;
                    // q = [cdf[4] <= slot] + [cdf[8] <= slot] + [cdf[12] <= slot]: flag bits of packed subtractions
                    const uint32_t q = __popc(((gs - c.x) & 0x80008000u) | (((gs - c.y) >> 1) & 0x4000u));
                    const uint2 rq = level2[4u * row + q];   // cdf[4q] | cdf[4q+1] << 16, cdf[4q+2] | cdf[4q+3] << 16
                    const uint32_t r = __popc(((gs - rq.y) & 0x80008000u) | ((gs - rq.x) >> 31));
                    const uint32_t bound = __byte_perm(c.x, c.y, 0x10u + 0x22u * q);   // cdf[4q+4] in bits 0..15
                    const uint32_t pr = __funnelshift_r((r & 2u) ? rq.y : rq.x, (r & 2u) ? bound : rq.y, r << 4);   // mod 32
                    const uint32_t start = pr & 0xffffu, y = 4u * q + r;
                    x = ((pr >> 16) - start) * (x >> 14) + slot - start;
                    if (cz && y == 8u) err |= kW4ErrCz;
                    word |= y << (4u * kk);
                    const uint32_t mag = y & 7u;
                    top = max(top, mag);
                    pair = ((top * top + top) >> 1) + mag;
                }
                // out of words: the structure bit alone, as the reference reports it (earlier bits dropped)
                if (!renorm(x, act && x < kW4L, ptr, win, lane)) { if (lane == 0) atomicOr(R.error, kW4Err); return; }
            }
            w0 = w1; w1 = w2; w2 = w3; w3 = word;
        }
        uint32_t w[4] = {w0, w1, w2, w3};
        const uint32_t left = x - kW4L;
        if (__any_sync(kFull, tail && (x < kW4L || left > 0xffffu))) { atomicOr(R.error, kW4Err | err); return; }
        if (active) {
            if (tail) {
                for (uint32_t q = 0; q < 4; ++q) {
                    const uint32_t y = (left >> (4u * q)) & 15u;
                    if (cz && y == 8u) err |= kW4ErrCz;
                    top = max(top, y & 7u);
                }
                w[3] |= left << 16;
                x = kW4L;
            }
            hash = mm3_block(mm3_block(mm3_block(mm3_block(hash, w[0]), w[1]), w[2]), w[3]);
            if (ceil && top == 5u) {
                if (!scale) err |= kW4ErrCeil;
                else {
                    so[cell] = (uint8_t)(scale - 1u);
                    for (int q = 0; q < 4; ++q) w[q] = ceil_double(w[q]);
                }
            }
            wo[cell] = make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
    // tile hash: XOR over the lanes of each lane's final MurmurHash3 (length 24 + 4 per scale + 16 per cell)
    const uint32_t mine = lane < n ? (n - lane + 31) / 32 : 0u;
    uint32_t H = mm3_final(hash, 24u + 20u * mine);
#pragma unroll
    for (int s = 16; s; s >>= 1) H ^= __shfl_xor_sync(kFull, H, s);
    if (ptr != J.nwords) err |= kW4Err;
    if (lane == 0 && x != kW4L + (H & 0xffffu)) err |= kW4ErrHash;
    if (lane == 1 && x != kW4L + (H >> 16)) err |= kW4ErrHash;
    if (lane >= 2 && x != kW4L) err |= kW4Err;
    if (err) atomicOr(R.error, err);
}

}  // namespace

cudaError_t launch_wnr4(const W4Tables &tab, const W4Job *jobs, uint32_t njobs, const W4Rec *recs, cudaStream_t st) {
    if (!njobs) return cudaSuccess;
    if (njobs % kW4Warps) return cudaErrorInvalidValue;   // the host pads every matrix's tiles to whole CTAs
    static thread_local int configured_device = -1;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return cudaGetLastError();
    if (dev != configured_device) {
        const cudaError_t e = cudaFuncSetAttribute(wnr4_tiles, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)w4_matrix_bytes(w4_rows(5)));
        if (e != cudaSuccess) return e;
        configured_device = dev;
    }
    wnr4_tiles<<<njobs / kW4Warps, kW4Warps * 32, tab.matrix_bytes, st>>>(tab, jobs, recs);
    return cudaGetLastError();
}

}  // namespace wexb
