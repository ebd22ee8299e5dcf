// WNR4 kind-MX tile decode on sm_100a (structures in wnr4.cuh). Semantics: the reference CPU decoder
// wnr4_decode_tile (wnr4/wnr4.h:388-478).
//
// One warp = one tile: its 32 lanes step in lockstep; at each step the lanes whose state fell below
// L = 2^16 take the next words of the tile's shared u16 stream in lane order (the format's rule: a
// lane's word is the one at the stream position plus the number of needing lanes below it). The
// stream reaches the warp through shared memory: TMA bulk copies move it in 1 KB chunks (16-byte
// aligned spans of the record, the first one starting at or below the tile's first word) into a
// two-chunk ring per warp, each chunk completing on its own mbarrier; the next chunk is requested as
// soon as the warp has left the one before it, and each lane reads its word with one 2-byte shared
// load. A CTA holds kW4Warps tiles of one matrix, with that matrix's weight rows and scale CDF staged
// into shared memory by one TMA bulk copy. A weight symbol takes two 8-byte shared loads: the row's
// level-1 entry gives the quartile q from three packed 16-bit comparisons, the quartile's four
// cumulative frequencies give the rank r in it, and start and end are adjacent fields taken by one
// funnel shift (tables in wnr4.cuh).
#include "wnr4.cuh"
#include "rans_device.cuh"

namespace wexb {
namespace {

using namespace rans;

constexpr uint32_t kFull = 0xffffffffu;
constexpr uint32_t kChunkBytes = 1024, kChunkWords = kChunkBytes / 2;
constexpr uint32_t kRingBytesPerWarp = 2 * kChunkBytes;

// Number of the 16 entries of a cumulative row (a, b: 8 packed u16 pairs, all < 2^15) that are <= slot.
__device__ __forceinline__ uint32_t row_count(const uint4 a, const uint4 b, uint32_t slot) {
    const uint32_t g = slot * 0x10001u | 0x80008000u;
    const uint32_t p0 = __byte_perm(g - a.x, g - a.y, 0x7531), p1 = __byte_perm(g - a.z, g - a.w, 0x7531);
    const uint32_t p2 = __byte_perm(g - b.x, g - b.y, 0x7531), p3 = __byte_perm(g - b.z, g - b.w, 0x7531);
    const uint32_t m = 0x80808080u;
    return (uint32_t)__popc((p0 & m) | ((p1 & m) >> 1) | ((p2 & m) >> 2) | ((p3 & m) >> 3));
}

__device__ __forceinline__ uint32_t lds_u16(uint32_t a) {
    uint16_t v;
    asm volatile("ld.shared.u16 %0, [%1];\n" : "=h"(v) : "r"(a));
    return v;
}

// A warp's tile word stream (see the file comment). Word k of the stream is byte 2 (k + shift) of the
// aligned span that starts at `from`; chunk c is that span's bytes [1024 c, 1024 (c + 1)), held in ring
// half c % 2 and completed on barrier c % 2 in phase (c / 2) % 2.
struct TileStream {
    uint32_t ring, bars;        // shared addresses: this warp's 2 KB ring and its two mbarriers
    const uint8_t *from;        // 16-byte aligned, at or below the first word
    uint32_t shift;             // words from `from` to the first word (0..7)
    uint32_t span;              // bytes from `from` to the end of the last word
    uint32_t nwords, ptr;       // words in the tile; the next unread one
    uint32_t ready, issued;     // chunks landed; chunks requested

    // The next chunk, by lane 0 (called by the whole warp); bytes a multiple of 16. The warp barrier and
    // the proxy fence order every lane's earlier reads of that ring half before the copy's writes.
    __device__ __forceinline__ void request() {
        const uint32_t c = issued++;
        __syncwarp();
        if ((threadIdx.x & 31u) == 0) {
            asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
            const uint32_t at = c * kChunkBytes, bytes = min(kChunkBytes, (span - at + 15u) & ~15u);
            const uint32_t bar = bars + 8u * (c & 1u);
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" :: "r"(bar), "r"(bytes) : "memory");
            asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n"
                         :: "r"(ring + kChunkBytes * (c & 1u)), "l"(from + at), "r"(bytes), "r"(bar) : "memory");
        }
    }
    __device__ __forceinline__ bool more() const { return issued * kChunkBytes < span; }
    // Waits (bounded) for the oldest requested chunk that has not landed; false when the wait gave up.
    __device__ __forceinline__ bool land() {
        const uint32_t c = ready;
        unsigned done = 0;
        for (uint32_t i = 0; i < kWaitPolls && !done; ++i)
            asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
                         : "=r"(done) : "r"(bars + 8u * (c & 1u)), "r"((c >> 1) & 1u) : "memory");
        if (done) ++ready;
        return done != 0;
    }
    // Before the warp leaves: every requested chunk has landed, so no copy can reach shared memory
    // that another CTA may own later (bounded like every wait).
    __device__ __forceinline__ void drain() { while (ready < issued && land()) {} }
    __device__ __forceinline__ uint32_t word(uint32_t k) const {
        return lds_u16(ring + 2u * ((k + shift) % (2u * kChunkWords)));
    }
    // Opens the stream (the warp's barriers initialised by the caller) and requests its first two chunks.
    __device__ __forceinline__ bool open(const uint8_t *words, uint32_t n, uint32_t ring_addr, uint32_t bar_addr) {
        ring = ring_addr; bars = bar_addr; nwords = n; ptr = 0; ready = 0; issued = 0;
        from = reinterpret_cast<const uint8_t *>(reinterpret_cast<uintptr_t>(words) & ~(uintptr_t)15);
        shift = (uint32_t)(words - from) / 2u;
        span = 2u * (shift + n);
        if (!span) return true;
        request();
        if (more()) request();
        return land();
    }
};

// The lanes with `need` take the next words of the stream, in lane order. 0, or kW4Err when the tile has
// too few words, or kW4ErrTimeout when a chunk did not land in time (both warp-uniform).
__device__ __forceinline__ uint32_t take_words(uint32_t &x, bool need, TileStream &s, uint32_t lane) {
    const uint32_t vote = __ballot_sync(kFull, need);
    if (!vote) return 0;
    const uint32_t total = __popc(vote);
    if (s.ptr + total > s.nwords) return kW4Err;
    if (s.shift + s.ptr + total > kChunkWords * s.ready && !s.land()) return kW4ErrTimeout;
    if (need) x = x << 16 | s.word(s.ptr + __popc(vote & ((1u << lane) - 1u)));
    s.ptr += total;
    // the chunk before the current one is used up: its half of the ring takes the one after the next
    if (s.more() && s.shift + s.ptr >= kChunkWords * (s.issued - 1u)) s.request();
    return 0;
}

__global__ void __launch_bounds__(kW4Warps * 32) wnr4_tiles(W4Tables tab, const W4Job *__restrict__ jobs,
                                                            const W4Rec *__restrict__ recs) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bar;
    __shared__ uint64_t stream_bars[kW4Warps][2];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t m = jobs[blockIdx.x * kW4Warps].m;   // every tile of the CTA is of this matrix
    const W4Job J = jobs[blockIdx.x * kW4Warps + warp];
    if (threadIdx.x < 2 * kW4Warps) mbar_init(&stream_bars[threadIdx.x >> 1][threadIdx.x & 1u], 1);
    {
        void *dst[1] = {smem};
        const void *src[1] = {tab.base + (size_t)m * tab.matrix_bytes};
        const uint32_t bytes[1] = {tab.matrix_bytes};
        if (!stage_tables(&bar, dst, src, bytes, 1)) {   // the table copy may still be in flight: read nothing
            if (J.n && lane == 0) atomicOr(recs[J.rec].error, kW4ErrTimeout);
            return;
        }
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
    TileStream ts;
    const uint32_t ring = smem_addr(smem + tab.matrix_bytes) + warp * kRingBytesPerWarp;
    if (!ts.open(J.tile + 128, J.nwords, ring, smem_addr(&stream_bars[warp][0]))) {
        ts.drain();
        if (lane == 0) atomicOr(R.error, kW4ErrTimeout);
        return;
    }
    uint32_t err = 0;
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
        if (const uint32_t e = take_words(x, act && x < kW4L, ts, lane)) {
            ts.drain();
            if (lane == 0) atomicOr(R.error, e);
            return;
        }
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
                if (const uint32_t e = take_words(x, act && x < kW4L, ts, lane)) {
                    ts.drain();
                    if (lane == 0) atomicOr(R.error, e);
                    return;
                }
            }
            w0 = w1; w1 = w2; w2 = w3; w3 = word;
        }
        uint32_t w[4] = {w0, w1, w2, w3};
        const uint32_t left = x - kW4L;
        if (__any_sync(kFull, tail && (x < kW4L || left > 0xffffu))) { ts.drain(); atomicOr(R.error, kW4Err | err); return; }
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
                    for (int q = 0; q < 4; ++q) w[q] = ceil_inverse_word(w[q]);
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
    ts.drain();
    if (ts.ptr != J.nwords) err |= kW4Err;
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
                                                   (int)(w4_matrix_bytes(w4_rows(5)) + kW4Warps * kRingBytesPerWarp));
        if (e != cudaSuccess) return e;
        configured_device = dev;
    }
    wnr4_tiles<<<njobs / kW4Warps, kW4Warps * 32, tab.matrix_bytes + kW4Warps * kRingBytesPerWarp, st>>>(tab, jobs, recs);
    return cudaGetLastError();
}

}  // namespace wexb
