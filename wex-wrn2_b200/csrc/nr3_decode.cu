// WNR2/WNR3 decode on sm_100a: one persistent launch per model and call (structures in wnr3.cuh).
//
// Every CTA (one per SM, 1024 threads) stages the model's whole table block (83 KB: both weight lookup
// levels of the three matrices, the scale slot tables and the packed scale CDFs) into shared memory
// with one TMA bulk copy, then its 32 warps drain the launch's work queue. A warp takes an item with
// one atomic and runs it on its 32 lanes, one stream per lane:
//   - scale items decode the order-0 scale streams into the decode layout;
//   - weight items wait (bounded) until their matrix's scales are decoded, then decode the weight
//     streams: 32 context-modelled 4-bit symbols per block, checked (stream hash, canonical zero) and
//     ceil-inverted per block, each block one 16-byte vector store (a 32-byte store of two blocks
//     would hold four more registers than the loop has: measured as spills);
//   - commit items wait (bounded) until their record's weight items are done and copy one chunk of
//     the decoded slab to the caller's buffer when the record's error word is 0.
// The host interleaves commit items with later records' weight items, so the copies run beside the
// decode instead of as a pass after it. Every lane reads its stream through a PayloadWindow
// (rans_device.cuh).
//
// Weight symbol lookup, two 8-byte shared loads: the context's level-1 entry gives the quartile q of
// the slot from three packed 16-bit comparisons (each a subtraction whose flag bit is set exactly when
// cdf <= slot), then the quartile's four cumulative frequencies give the symbol's rank r in it the
// same way; start and end are the two adjacent 16-bit fields r, r + 1 of the quartile row followed by
// its end (a field of the level-1 entry), taken by one funnel shift. Renormalisation is branch-free:
// from a valid state a symbol leaves at least 2^9, so it takes 0, 1 or 2 bytes (from the count of
// leading zeros), read as one big-endian window shared by a pair of symbols.
#include "wnr3.cuh"
#include "rans_device.cuh"

namespace wexb {
namespace {

using namespace rans;

// dynamic shared memory of a CTA of kThreads threads: the table block, then every lane's payload ring
template <int kThreads> constexpr size_t decode_smem() { return kTableBytes + (size_t)(kWinWords + 1) * 4u * kThreads; }
static_assert(kTableBytes % 16 == 0, "the table block is one TMA bulk copy");

// ---- queue plumbing ---------------------------------------------------------------------------
// Lane 0 polls `counter` until it reaches `target` (acquire loads, at most kWaitPolls polls, with a sleep
// between polls that doubles from 128 ns to 8 us: a waiting warp must not take issue slots from the
// decoding warps beside it); the whole warp then goes on (true) or gives up (false). The warp barrier
// orders every lane's later reads after lane 0's acquire.
__device__ __forceinline__ bool warp_wait_count(const uint32_t *counter, uint32_t target) {
    uint32_t ok = 1;
    if ((threadIdx.x & 31u) == 0) {
        ok = 0;
        uint32_t nap = 128;
        for (uint32_t n = 0; n < kWaitPolls; ++n) {
            uint32_t v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(counter) : "memory");
            if (v >= target) { ok = 1; break; }
            __nanosleep(nap);
            nap = min(2u * nap, 8192u);
        }
    }
    ok = __shfl_sync(~0u, ok, 0);
    __syncwarp();
    return ok != 0;
}
// Publishes a finished item: every lane's writes, then one increment of `counter`.
__device__ __forceinline__ void item_done(uint32_t *counter) {
    __threadfence();
    __syncwarp();
    if ((threadIdx.x & 31u) == 0) atomicAdd(counter, 1u);
}

// ---- block checks of the coded nibbles ----------------------------------------------------------
// Non-zero iff a nibble of the four words is 8 (a coded -0). Per word t = w ^ 0x8888...: a nibble of t
// is zero exactly when neither its bit 3 nor (its low three bits + 7) reaches bit 3; the sums stay
// inside their nibbles (7 + 7 < 16).
__device__ __forceinline__ uint32_t coded_neg_zero(const uint32_t w[4]) {
    uint32_t nonzero = 0x88888888u;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const uint32_t t = w[q] ^ 0x88888888u;
        nonzero &= ((t & 0x77777777u) + 0x77777777u) | t;
    }
    return ~nonzero & 0x88888888u;
}
// ---- scale streams ----------------------------------------------------------------------------
// tables, lane_slots: shared addresses of the staged table block and of the lane's payload slot 0.
template <int kThreads>
__device__ __noinline__ uint32_t scale_stream(const Nr3Record &R, uint32_t m, uint32_t j, uint32_t tables,
                                              uint32_t lane_slots) {
    const uint32_t g = R.sbase[m] + j, begin = R.offsets[g], end = R.offsets[g + 1];
    const uint32_t first = j * R.schunk, count = min(R.schunk, R.scount[m] - first);
    const uint32_t ssym = tables + (uint32_t)kWTableBytes + m * kTotal;
    const uint32_t sf = tables + (uint32_t)(kWTableBytes + kSsymBytes) + m * kSfBytes;
    PayloadWindow<kThreads> pw;
    uint32_t x = pw.open(R.rec, begin, end, lane_slots);
    uint32_t err = (x - kRansL >= 255u * kRansL) ? kErrStruct : 0u;   // a valid initial state is in [L, 256 L)
    const bool nr3 = R.flags & 256u;
    uint32_t h = nr3 ? ident_hash(R.model_id, R.owner, g, R.word24) : 0u;
    x = order0_stream(pw, x, ssym, sf, count, R.out + R.soff[m] + first, h);
    pw.close();
    const uint32_t expect = nr3 ? kRansL + (mm3_final(h, 16u + count) & 0x7fffffu) : kRansL;
    if (pw.byte_pos() != end - (begin & ~3u)) err |= kErrStruct;
    else if (x != expect) err |= nr3 ? kErrHash : kErrStruct;
    return err;
}

// ---- weight streams ---------------------------------------------------------------------------
// active: the lanes of the warp decoding a stream of this item (every one of them calls this).
template <int kThreads>
__device__ __noinline__ uint32_t weight_stream(const Nr3Record &R, uint32_t m, uint32_t j, uint32_t tables,
                                               uint32_t lane_slots, uint32_t active) {
    const uint32_t g = R.wbase[m] + j, begin = R.offsets[g], end = R.offsets[g + 1];
    const uint32_t first = j * R.wchunk, blocks = min(R.wchunk, R.wcount[m] - first) / 32u;
    uint8_t *scales = R.out + R.soff[m] + first / 32u;   // coded scales; the ceil inverse edits them
    uint8_t *dst = R.out + R.wout[m] + first / 2u;        // 16 bytes per block
    const uint32_t level1 = tables + m * kWBlockBytes, level2 = level1 + kWL1Bytes;   // rows of 8 bytes
    const bool nr3 = R.flags & 256u, cz = nr3 && (R.flags & 8u), ceil = nr3 && ((R.flags >> m) & 1u);
    const int anchor = (int)((R.word24 >> (8u * m)) & 0xffu);
    PayloadWindow<kThreads> pw;
    uint32_t x = pw.open(R.rec, begin, end, lane_slots);
    uint32_t err = (x - kRansL >= 255u * kRansL) ? kErrStruct : 0u;
    uint32_t h = nr3 ? ident_hash(R.model_id, R.owner, g, R.word24) : 0u;
    uint32_t scale = blocks ? scales[0] : 0u;
    // The lanes run in lockstep only if nothing makes them part: a rare branch (a ceil-form block)
    // could otherwise leave the warp split in two halves for the rest of the stream, each issuing every
    // instruction. When every active lane has the same number of blocks (all but a matrix's last item),
    // the warp meets at the end of each block.
    const bool lockstep = __reduce_min_sync(active, blocks) == __reduce_max_sync(active, blocks);
#pragma unroll 1
    for (uint32_t b = 0; b < blocks; ++b) {
        const uint32_t next_scale = b + 1 < blocks ? scales[b + 1] : 0u;
        const int d = (int)scale - anchor;
        const uint32_t srel = (uint32_t)(min(max(d, -3), 3) + 3) * kPairs;
        const uint32_t l1 = level1 + 8u * srel, l2 = level2 + 32u * srel;
        // row1: the shared address of the context's level-1 row (8 bytes a pair index); its level-2 rows
        // (32 bytes a pair index) sit at 4 row1 + to2. The block starts at pair index 36.
        const uint32_t to2 = l2 - 4u * l1;   // (wraps mod 2^32; 4 row1 + to2 does not)
        uint32_t row1 = l1 + 8u * (kPairs - 1u), top = 0, w[4] = {0, 0, 0, 0};
        // one symbol: its quartile and rank from the two 8-byte rows of the context, the state update,
        // then the next context (pair index top (top + 1) / 2 + mag: 4 top (top + 1) + 8 mag bytes)
        auto step = [&](uint32_t k) {
            const uint2 c = lds_v2(row1);
            const uint32_t slot = x & (kTotal - 1u), gs = slot * 0x10001u + 0x80008000u;
            // q = [cdf[4] <= slot] + [cdf[8] <= slot] + [cdf[12] <= slot]
            uint32_t d0, d1;
            asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(d0) : "r"(c.x), "r"(0xffffffffu), "r"(gs));
            asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(d1) : "r"(c.y), "r"(0xffffffffu), "r"(gs));
            const uint32_t q = __popc((d0 & 0x80008000u) | ((d1 >> 1) & 0x4000u));
            const uint2 row = lds_v2(4u * row1 + to2 + 8u * q);   // cdf[4q] | cdf[4q+1] << 16, cdf[4q+2] | cdf[4q+3] << 16
            // r = [cdf[4q+1] <= slot] + [cdf[4q+2] <= slot] + [cdf[4q+3] <= slot]
            uint32_t e0, e1;
            asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(e0) : "r"(row.x), "r"(0xffffffffu), "r"(gs));
            asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(e1) : "r"(row.y), "r"(0xffffffffu), "r"(gs));
            const uint32_t r = __popc((e1 & 0x80008000u) | (e0 >> 31));
            // cdf[4q+4] in bits 0..15: field q of cdf[4], cdf[8], cdf[12], 2^14 (bytes 2q, 2q + 1)
            const uint32_t bound = __byte_perm(c.x, c.y, 0x10u + 0x22u * q);
            // start | end << 16 = fields r, r + 1 of cdf[4q .. 4q+3], bound (only its low half reaches pair)
            const uint32_t lo = (r & 2u) ? row.y : row.x, hi = (r & 2u) ? bound : row.y;
            const uint32_t pair = __funnelshift_r(lo, hi, r << 4);   // the shift counts mod 32: 0 or 16
            const uint32_t start = pair & 0xffffu, freq = (pair >> 16) - start;
            x = freq * (x >> kPrec) + slot - start;
            const uint32_t sym = 4u * q + r;
            w[k / 8u] += sym << (4u * (k % 8u));
            const uint32_t mag = sym & 7u;
            top = max(top, mag);
            row1 = l1 + 4u * (top * top + top) + 8u * mag;
        };
#pragma unroll
        for (uint32_t k = 0; k < 32; k += 2) {
            if (k % 8u == 0) pw.top_up();
            uint32_t win = pw.take32();   // the bytes of both symbols of the pair
            step(k);
            const uint32_t b1 = renorm_bits(x);
            x = __funnelshift_l(win, x, b1);
            win <<= b1;
            step(k + 1);
            const uint32_t b2 = renorm_bits(x);
            x = __funnelshift_l(win, x, b2);
            pw.bit += b1 + b2;
        }
        if (nr3) {   // the stream hash runs over the coded nibbles; then the canonical-zero and ceil rules
            h = mm3_block(mm3_block(mm3_block(mm3_block(h, w[0]), w[1]), w[2]), w[3]);
            if (cz && coded_neg_zero(w)) err |= kErrCz;
            if (ceil && top == 5u) {
                if (!scale) {
                    err |= kErrCeil;
                } else {
#pragma unroll
                    for (int q = 0; q < 4; ++q) w[q] = ceil_inverse_word(w[q]);
                    scales[b] = (uint8_t)(scale - 1u);
                }
            }
        }
        reinterpret_cast<uint4 *>(dst)[b] = make_uint4(w[0], w[1], w[2], w[3]);
        scale = next_scale;
        if (lockstep) __syncwarp(active);
    }
    pw.close();
    const uint32_t expect = nr3 ? kRansL + (mm3_final(h, 16u + blocks * 16u) & 0x7fffffu) : kRansL;
    if (pw.byte_pos() != end - (begin & ~3u)) err |= kErrStruct;
    else if (x != expect) err |= nr3 ? kErrHash : kErrStruct;
    return err;
}

// ---- commit -----------------------------------------------------------------------------------
// Chunk `chunk` of region `region` of the record's commit, by one warp. The decoded bytes were written
// by other SMs during this launch, so they are read from L2 (ld.global.cg), never from a possibly
// stale L1 line.
__device__ __noinline__ void commit_chunk(const CommitJob &J, uint32_t region, uint32_t chunk) {
    const uint32_t lane = threadIdx.x & 31u;
    const size_t at = (size_t)chunk * kCommitChunk;
    if (at >= J.bytes[region]) return;
    const uint32_t n = (uint32_t)min((size_t)kCommitChunk, J.bytes[region] - at);
    const uint8_t *s = J.src[region] + at;
    uint8_t *d = J.dst[region] + at;
    uint32_t i = 0;
    if (!((reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(d)) & 15u)) {
        const uint4 *s16 = reinterpret_cast<const uint4 *>(s);
        uint4 *d16 = reinterpret_cast<uint4 *>(d);
        const uint32_t n16 = n / 16u;
        uint32_t k = lane;
        for (; k + 96u < n16; k += 128u) {   // four 16-byte loads in flight per lane
            const uint4 a = __ldcg(s16 + k), b = __ldcg(s16 + k + 32u), c = __ldcg(s16 + k + 64u), e = __ldcg(s16 + k + 96u);
            d16[k] = a; d16[k + 32u] = b; d16[k + 64u] = c; d16[k + 96u] = e;
        }
        for (; k < n16; k += 32u) d16[k] = __ldcg(s16 + k);
        i = n16 * 16u;
    }
    for (uint32_t k = i + lane; k < n; k += 32u) d[k] = __ldcg(s + k);
}

// ---- the persistent kernel --------------------------------------------------------------------
// 64 registers a thread in both CTA sizes (1,024 threads: the whole register file; 832 threads: room
// for two record-hash CTAs beside it)
template <int kThreads>
__global__ void __maxnreg__(64) nr3_decode(const Nr3Launch L) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bar;
    {
        void *dst[1] = {smem};
        const void *src[1] = {L.tables};
        const uint32_t bytes[1] = {(uint32_t)kTableBytes};
        if (!stage_tables(&bar, dst, src, bytes, 1)) {
            // the tables may still be landing: this CTA never reads them and takes no item; every
            // record reports the timeout bit (the host makes that status 1: decode again)
            for (uint32_t r = threadIdx.x; r < L.nrecs; r += blockDim.x) atomicOr(L.recs[r].error, kErrTimeout);
            return;
        }
    }
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t tables = smem_addr(smem), lane_slots = tables + (uint32_t)kTableBytes + 4u * threadIdx.x;
    for (;;) {
        uint32_t i = 0;
        if (lane == 0) i = atomicAdd(L.head, 1u);
        i = __shfl_sync(~0u, i, 0);
        if (i >= L.nitems) break;
        const Nr3Item it = L.items[i];
        const uint32_t kind = it.what >> 28, sub = (it.what >> 24) & 15u, first = it.what & 0xffffffu;
        const Nr3Record &R = L.recs[it.rec];
        uint32_t *done = L.done + 4u * it.rec;
        uint32_t err = 0;
        if (kind == kItemScale) {
            if (R.landed && !warp_wait_count(R.landed, R.landed_at)) {   // the record's bytes never arrived
                if (lane == 0) atomicOr(R.error, kErrTimeout);
                item_done(done + sub);
                continue;
            }
            const uint32_t j = first + lane;
            if (j < (R.scount[sub] + R.schunk - 1u) / R.schunk) err = scale_stream<kThreads>(R, sub, j, tables, lane_slots);
            if (err) atomicOr(R.error, err);
            item_done(done + sub);
        } else if (kind == kItemWeight) {
            if (!warp_wait_count(done + sub, R.sitems[sub])) {   // its scales never completed
                if (lane == 0) atomicOr(R.error, kErrTimeout);
                continue;
            }
            const uint32_t j = first + lane;
            const bool mine = j < (R.wcount[sub] + R.wchunk - 1u) / R.wchunk;
            const uint32_t active = __ballot_sync(~0u, mine);
            if (mine) err = weight_stream<kThreads>(R, sub, j, tables, lane_slots, active);
            if (err) atomicOr(R.error, err);
            item_done(done + 3);
        } else {
            if (!warp_wait_count(done + 3, R.witems)) {
                if (lane == 0) atomicOr(R.error, kErrTimeout);
                continue;
            }
            if (!*reinterpret_cast<const volatile uint32_t *>(R.error)) commit_chunk(*R.job, sub, first);
        }
    }
}

}  // namespace

cudaError_t prepare_nr3_kernels() {
    const cudaError_t e = cudaFuncSetAttribute(nr3_decode<kDecodeThreads>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)decode_smem<kDecodeThreads>());
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(nr3_decode<kBesideHashThreads>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)decode_smem<kBesideHashThreads>());
}

cudaError_t launch_nr3(const Nr3Launch &L, int sms, cudaStream_t st, bool beside_hashes) {
    if (!L.nitems) return cudaSuccess;
    if (beside_hashes)
        nr3_decode<kBesideHashThreads>
            <<<(sms + 1) / 2, kBesideHashThreads, decode_smem<kBesideHashThreads>(), st>>>(L);
    else
        nr3_decode<kDecodeThreads><<<sms, kDecodeThreads, decode_smem<kDecodeThreads>(), st>>>(L);
    return cudaGetLastError();
}

}  // namespace wexb
