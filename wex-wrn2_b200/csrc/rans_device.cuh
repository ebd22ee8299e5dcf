// Device helpers shared by the rANS stream kernels (WNR2/WNR3 in nr3_decode.cu, WBP1 in
// wbp1_kernels.cu): MurmurHash3 words, bounded mbarrier waits around TMA bulk copies, and the payload
// window through which one lane reads its stream's bytes.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "wnr3.cuh"

namespace wexb {
namespace rans {

// ---- MurmurHash3_x86_32 (Austin Appleby's published algorithm), one 32-bit block at a time ---------
__device__ __forceinline__ uint32_t rotl32(uint32_t x, int r) { return __funnelshift_l(x, x, r); }
__device__ __forceinline__ uint32_t mm3_mix(uint32_t k) { return rotl32(k * 0xcc9e2d51u, 15) * 0x1b873593u; }
__device__ __forceinline__ uint32_t mm3_block(uint32_t h, uint32_t k) { return rotl32(h ^ mm3_mix(k), 13) * 5u + 0xe6546b64u; }
__device__ __forceinline__ uint32_t mm3_final(uint32_t h, uint32_t len) {
    h ^= len;
    h ^= h >> 16; h *= 0x85ebca6bu; h ^= h >> 13; h *= 0xc2b2ae35u; h ^= h >> 16;
    return h;
}
// MurmurHash3 state after a WNR3 stream's ident words {model, owner, g, word24}, seed "WNR3"
// (c/wex_neural_rans.h:225-233).
__device__ __forceinline__ uint32_t ident_hash(uint32_t model, uint32_t owner, uint32_t g, uint32_t word24) {
    uint32_t h = 0x33524e57u;
    h = mm3_block(h, model); h = mm3_block(h, owner); h = mm3_block(h, g);
    return mm3_block(h, word24);
}

// ---- TMA bulk copies into shared memory, completed on an mbarrier, waited for with a limit --------
__device__ __forceinline__ unsigned smem_addr(const void *p) { return (unsigned)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" :: "r"(smem_addr(bar)), "r"(count) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
__device__ __forceinline__ void mbar_expect(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" :: "r"(smem_addr(bar)), "r"(bytes) : "memory");
}
// Global -> this CTA's shared memory; both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n"
                 :: "r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar)) : "memory");
}
// Waits for phase `parity` of the mbarrier, at most `limit` polls; false when it gave up.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint32_t limit = kWaitPolls) {
    const unsigned a = smem_addr(bar);
    for (uint32_t i = 0; i < limit; ++i) {
        uint32_t done;
        asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
                     : "=r"(done) : "r"(a), "r"(parity) : "memory");
        if (done) return true;
    }
    return false;
}

// Stages `n` blocks of table bytes into shared memory with TMA; every thread of the CTA returns once
// they landed, or false after a bounded wait (the copies may then still be in flight: the caller
// reports kErrTimeout, which the host turns into status 1, and never reads the tables).
__device__ __forceinline__ bool stage_tables(uint64_t *bar, void *const *dst, const void *const *src,
                                             const uint32_t *bytes, int n) {
    if (threadIdx.x == 0) mbar_init(bar, 1);
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t total = 0;
        for (int i = 0; i < n; ++i) total += bytes[i];
        mbar_expect(bar, total);
        for (int i = 0; i < n; ++i) bulk_g2s(dst[i], src[i], bytes[i], bar);
    }
    return mbar_wait(bar, 0);
}

// ---- one stream's payload, as its lane sees it -----------------------------------------------------
// The stream's bytes go through a window of kWinWords words in shared memory, laid out across the
// CTA's lanes: word w of the stream (counted from its first 4-byte aligned word) sits in slot
// w % kWinWords of the lane, slot s of lane l at ring[s * lanes + l], so every shared access of a warp
// is conflict-free whatever position each lane has reached. Slot kWinWords repeats slot 0, so the two
// words under any position are adjacent slots with no wrap.
//
// Words arrive in groups of 4 by 4-byte cp.async copies (the stream's bytes are not 16-byte aligned,
// and the transposed layout needs word-sized pieces). Each top_up() keeps at least 12 words requested
// ahead of the read position and waits for all but the newest group; it is called before every 8
// symbols, which read at most 16 bytes. A group is requested whole even when it ends past the stream's
// last word, so a stream's reads run at most 12 bytes past its end (record buffers carry that slack);
// bytes past the end are never valid data: a decoder that reaches them fails its final position check.
constexpr uint32_t kWinWords = 16;

// Shared-memory accesses by 32-bit shared-window address. Table loads may be reordered freely (the
// tables do not change once staged); payload loads are volatile asm, which the compiler keeps in order
// with the (volatile) cp.async waits.
__device__ __forceinline__ uint32_t lds_u8(uint32_t a) {
    uint32_t v;
    asm("ld.shared.u8 %0, [%1];\n" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
    uint32_t v;
    asm("ld.shared.u32 %0, [%1];\n" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 lds_v2(uint32_t a) {
    uint2 v;
    asm("ld.shared.v2.u32 {%0, %1}, [%2];\n" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds_payload(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];\n" : "=r"(v) : "r"(a));
    return v;
}

// Four 4-byte asynchronous copies global -> shared, src[k] to dst + k * stride, when `go`, and a fifth of
// src[0] to `mirror` when `go` and `also`. The copies are predicated (one predicate for the four), so the
// lanes of a warp that copy and those that do not stay converged.
template <uint32_t kStrideBytes>
__device__ __forceinline__ void cp_async4x4(uint32_t dst, const uint32_t *src, uint32_t mirror, bool go, bool also) {
    asm volatile("{\n"
                 "  .reg .pred p, q;\n"
                 "  setp.ne.u32 p, %3, 0;\n"
                 "  setp.ne.and.u32 q, %4, 0, p;\n"
                 "  @p cp.async.ca.shared.global [%0], [%1], 4;\n"
                 "  @p cp.async.ca.shared.global [%0+%5], [%1+4], 4;\n"
                 "  @p cp.async.ca.shared.global [%0+%6], [%1+8], 4;\n"
                 "  @p cp.async.ca.shared.global [%0+%7], [%1+12], 4;\n"
                 "  @q cp.async.ca.shared.global [%2], [%1], 4;\n"
                 "}\n" :: "r"(dst), "l"(src), "r"(mirror), "r"((uint32_t)go), "r"((uint32_t)also),
                 "n"(kStrideBytes), "n"(2 * kStrideBytes), "n"(3 * kStrideBytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" :: "n"(N) : "memory"); }

template <int kLanes>
struct PayloadWindow {
    static constexpr uint32_t kStride = 4u * kLanes;   // bytes from one slot of a lane to its next
    uint32_t slots;           // shared address of this lane's slot 0
    const uint32_t *words;    // the stream's first aligned word
    uint32_t bit;             // bit position of the next unread byte, from `words`
    uint32_t ask;             // next word to request (a multiple of 4)
    uint32_t stop;            // words at or past this are never requested (one past the stream's last word)

    // The next group when `go` (every lane runs the same predicated instructions: no divergence).
    __device__ __forceinline__ void request_group(bool go) {
        const uint32_t s = ask % kWinWords;
        // the group's four words, and the mirror of slot 0 when the group starts there
        cp_async4x4<kStride>(slots + s * kStride, words + ask, slots + kWinWords * kStride, go, s == 0);
        ask += go ? 4u : 0u;
    }
    // Opens the stream of record bytes [begin, end) (length >= 4, checked on the host) and returns its
    // initial state, the big-endian word at begin. lane_slots: shared address of the lane's slot 0.
    __device__ __forceinline__ uint32_t open(const uint8_t *rec, uint32_t begin, uint32_t end, uint32_t lane_slots) {
        slots = lane_slots;
        words = reinterpret_cast<const uint32_t *>(rec) + (begin >> 2);
        stop = ((end + 3u) >> 2) - (begin >> 2);
        ask = 0;
        for (int k = 0; k < 3; ++k) request_group(ask < stop);
        cp_async_commit();
        cp_async_wait<0>();
        bit = (begin & 3u) * 8u;
        const uint32_t v = take32();
        bit += 32;
        return v;
    }
    // Before each 8 symbols: a new group when fewer than 12 words are requested ahead.
    __device__ __forceinline__ void top_up() {
        request_group(ask < stop && ask - (bit >> 5) < 12u);
        cp_async_commit();
        cp_async_wait<1>();
    }
    // The 4 bytes at the read position, big-endian (the first byte in bits 24..31).
    __device__ __forceinline__ uint32_t take32() const {
        const uint32_t a = slots + ((bit >> 5) % kWinWords) * kStride;
        return __byte_perm(__funnelshift_r(lds_payload(a), lds_payload(a + kStride), bit), 0, 0x0123);
    }
    // Byte offset of the read position from the stream's first aligned word.
    __device__ __forceinline__ uint32_t byte_pos() const { return bit >> 3; }
    // Waits for every copy this lane still has in flight (before the lane leaves the stream).
    __device__ __forceinline__ void close() const { cp_async_wait<0>(); }
};

// The ceil-form inverse of the eight nibbles of w (c/wex_neural_rans.h:446-461, the same rule in WNR4
// kind MX): magnitude a becomes a + min(a, 2), i.e. 0 1 2 3 4 5 -> 0 2 4 5 6 7, read from a nibble
// table; signs are kept. A block whose coded maximum is 5 holds magnitudes 0..5 only.
__device__ __forceinline__ uint32_t ceil_inverse_word(uint32_t w) {
    constexpr uint32_t kDoubled = 0x00765420u;   // nibble a: the magnitude a stands for
    uint32_t out = w & 0x88888888u;
#pragma unroll
    for (int k = 0; k < 32; k += 4) out |= ((kDoubled >> (4u * ((w >> k) & 7u))) & 7u) << k;
    return out;
}

// Bits (0, 8 or 16) a state in [2^9, 2^31) shifts in until it is at least 2^23.
__device__ __forceinline__ uint32_t renorm_bits(uint32_t x) { return ((uint32_t)__clz(x) - 1u) & 24u; }

// Decodes `count` order-0 byte symbols of one stream (the WNR3 scale coder, also WBP1's coded planes):
// slot -> symbol from the shared table at `ssym` (16,384 bytes), the symbol's start | freq << 16 from
// the shared table at `sf` (256 words). The bytes go to out (4-byte stores when out is 4-byte aligned)
// and through the MurmurHash3 state h, the last partial word as a hash tail. Returns the final state.
template <int kLanes>
__device__ __forceinline__ uint32_t order0_stream(PayloadWindow<kLanes> &pw, uint32_t x, uint32_t ssym, uint32_t sf,
                                                  uint32_t count, uint8_t *out, uint32_t &h) {
    const bool words_ok = !(reinterpret_cast<uintptr_t>(out) & 3u);
    uint32_t i = 0;
    for (; i + 8 <= count; i += 8) {
        pw.top_up();
        uint32_t word[2] = {0, 0};
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const uint32_t win = pw.take32();
            const uint32_t slot = x & (kTotal - 1u), sym = lds_u8(ssym + slot), e = lds_u32(sf + 4u * sym);
            x = (e >> 16) * (x >> kPrec) + slot - (e & 0xffffu);
            const uint32_t b = renorm_bits(x);
            x = __funnelshift_l(win, x, b);
            pw.bit += b;
            word[k >> 2] |= sym << (8 * (k & 3));
        }
        h = mm3_block(mm3_block(h, word[0]), word[1]);
        if (words_ok) {
            reinterpret_cast<uint32_t *>(out + i)[0] = word[0];
            reinterpret_cast<uint32_t *>(out + i)[1] = word[1];
        } else {
            for (int k = 0; k < 8; ++k) out[i + k] = (uint8_t)(word[k >> 2] >> (8 * (k & 3)));
        }
    }
    if (i < count) {   // the last stream of a matrix or plane: fewer than 8 symbols left
        pw.top_up();
        uint32_t word = 0, held = 0;
        for (; i < count; ++i) {
            const uint32_t win = pw.take32();
            const uint32_t slot = x & (kTotal - 1u), sym = lds_u8(ssym + slot), e = lds_u32(sf + 4u * sym);
            x = (e >> 16) * (x >> kPrec) + slot - (e & 0xffffu);
            const uint32_t b = renorm_bits(x);
            x = __funnelshift_l(win, x, b);
            pw.bit += b;
            out[i] = (uint8_t)sym;
            word |= sym << (8 * held);
            if (++held == 4) { h = mm3_block(h, word); word = 0; held = 0; }
        }
        if (held) h ^= mm3_mix(word);   // MurmurHash3's tail: the last 1-3 bytes, mixed without a round
    }
    return x;
}

}  // namespace rans
}  // namespace wexb
