// Device helpers shared by the rANS stream kernels (WNR3/WNR2 in wnr3_kernels.cu, WBP1 in
// wbp1_kernels.cu): MurmurHash3 words, bounded mbarrier waits around TMA bulk copies, cp.async, and the
// per-lane payload ring that one stream's decoder reads its bytes from.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "wnr3.cuh"

namespace wexb {
namespace rans {

constexpr uint32_t kRingWords = 32;
constexpr uint32_t kAhead = 24;
constexpr uint32_t kSpinLimit = kWaitPolls;   // bounded waits: never spin forever on a barrier

__device__ __forceinline__ uint32_t rotl32(uint32_t x, int r) { return __funnelshift_l(x, x, r); }
__device__ __forceinline__ uint32_t mm3_mix(uint32_t k) { return rotl32(k * 0xcc9e2d51u, 15) * 0x1b873593u; }
__device__ __forceinline__ uint32_t mm3_block(uint32_t h, uint32_t k) { return rotl32(h ^ mm3_mix(k), 13) * 5u + 0xe6546b64u; }
__device__ __forceinline__ uint32_t mm3_final(uint32_t h, uint32_t len) {
    h ^= len;
    h ^= h >> 16; h *= 0x85ebca6bu; h ^= h >> 13; h *= 0xc2b2ae35u; h ^= h >> 16;
    return h;
}
// MurmurHash3 state after the stream's ident words {model, owner, g, word24}, seed "WNR3"
// (c/wex_neural_rans.h:225-233).
__device__ __forceinline__ uint32_t ident_hash(uint32_t model, uint32_t owner, uint32_t g, uint32_t word24) {
    uint32_t h = 0x33524e57u;
    h = mm3_block(h, model); h = mm3_block(h, owner); h = mm3_block(h, g);
    return mm3_block(h, word24);
}

// ---- async copies ----------------------------------------------------------------------------
__device__ __forceinline__ void cp4(uint32_t *dst, const uint32_t *src, bool pred) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %2, 0;\n @p cp.async.ca.shared.global [%0], [%1], 4;\n}\n"
                 :: "r"(d), "l"(src), "r"((int)pred) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" :: "n"(N) : "memory"); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" :: "r"((unsigned)__cvta_generic_to_shared(bar)), "r"(count) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
__device__ __forceinline__ void mbar_expect(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n"
                 :: "r"((unsigned)__cvta_generic_to_shared(bar)), "r"(bytes) : "memory");
}
// TMA bulk copy global -> this CTA's shared memory, completing `bytes` on the mbarrier. Both
// addresses 16-byte aligned, bytes a multiple of 16 (every table block here is).
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n"
                 :: "r"((unsigned)__cvta_generic_to_shared(dst)), "l"(src), "r"(bytes),
                    "r"((unsigned)__cvta_generic_to_shared(bar)) : "memory");
}
// Waits for phase `parity` of the mbarrier, at most `limit` polls; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint32_t limit = kSpinLimit) {
    const unsigned a = (unsigned)__cvta_generic_to_shared(bar);
    for (uint32_t i = 0; i < limit; ++i) {
        uint32_t done;
        asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
                     : "=r"(done) : "r"(a), "r"(parity) : "memory");
        if (done) return true;
    }
    return false;
}

// Stages `n` blocks of table bytes into shared memory with TMA; every thread returns once they
// landed (or, after a bounded wait, with false).
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

// ---- one stream's payload: a per-lane ring in shared memory ------------------------------------
struct Reader {
    uint32_t *lane;          // this lane's ring base; word w lives at lane[(w % kRingWords) * stride]
    uint32_t stride;
    const uint32_t *src;     // the record as 32-bit words (4-byte aligned)
    uint32_t pos;            // record offset of the next payload byte
    uint32_t req;            // next word to request
    uint32_t last;           // the stream's last word

    __device__ __forceinline__ uint32_t *slot(uint32_t w) const { return lane + (w & (kRingWords - 1)) * stride; }

    // Opens [begin, end) (length >= 4, checked on the host) and returns its initial state.
    __device__ __forceinline__ uint32_t open(uint32_t begin, uint32_t end) {
        const uint32_t first = begin >> 2;
        last = (end - 1) >> 2;
        const uint32_t target = min(first + kAhead, last + 1);
        for (uint32_t w = first; w < target; ++w) cp4(slot(w), src + w, true);
        req = target;
        cp_commit();
        cp_wait<0>();
        const uint32_t v = __funnelshift_r(*slot(first), *slot(first + 1), (begin & 3u) * 8u);
        pos = begin + 4;
        return __byte_perm(v, 0, 0x0123);   // big-endian bytes begin .. begin + 3
    }
    // Every 16 symbols (at most 32 bytes): keep kAhead words requested, then wait for the words of
    // the previous request, which cover every byte the next 16 symbols can read.
    __device__ __forceinline__ void refill() {
        const uint32_t target = min((pos >> 2) + kAhead, last + 1);
#pragma unroll
        for (uint32_t k = 0; k < 8; ++k) {
            const uint32_t w = req + k;
            cp4(slot(w), src + w, w < target);
        }
        req = max(req, min(req + 8, target));
        cp_commit();
        cp_wait<1>();
    }
    // The next two payload bytes as a big-endian pair in bits 16..31 (read before the lookup, so
    // the shared loads overlap it). Past the stream's end the ring holds stale words: consuming
    // them is caught by the final pos == end check.
    __device__ __forceinline__ uint32_t peek() const {
        const uint32_t w = pos >> 2;
        return __byte_perm(__funnelshift_r(*slot(w), *slot(w + 1), (pos & 3u) * 8u), 0, 0x0144);
    }
    // Waits for every copy this lane still has in flight (before the lane returns).
    __device__ __forceinline__ void drain() const { cp_wait<0>(); }
    // while (x < L) x = x << 8 | next byte, as one funnel shift of 0, 8 or 16 bits.
    __device__ __forceinline__ uint32_t renorm(uint32_t x, uint32_t two) {
        const uint32_t bits = x < (1u << 15) ? 16u : (x < kRansL ? 8u : 0u);
        pos += bits >> 3;
        return __funnelshift_l(two, x, bits);
    }
};

}  // namespace rans
}  // namespace wexb
