// WNR2/WNR3 decode kernels for sm_100a (see wnr3.cuh for the structures).
//
// Layout per CTA: the CTA serves one matrix of one record; its lookup tables are staged into shared
// memory by TMA bulk copies (cp.async.bulk, completion on an mbarrier), and every lane owns a
// 32-word ring of its stream's payload in shared memory, refilled every 16 symbols by 4-byte
// cp.async copies kept 24 words ahead of the read position (ring word w of lane l at
// ring[(w % 32) * blockDim + l]: conflict-free whatever position each lane is at).
//
// Weight symbol lookup, two 8-byte shared loads: the context's level-1 entry gives the quartile q of
// the slot from three packed 16-bit comparisons (each a subtraction whose flag bit is set exactly when
// cdf <= slot), then the quartile's four cumulative frequencies give the symbol's rank r in it the
// same way; start and end are the two adjacent 16-bit fields r, r + 1 of the quartile row followed by
// its end (a field of the level-1 entry), taken by one funnel shift. Renormalisation is branch-free:
// from a valid state a symbol leaves at least 2^9, so it takes 0, 1 or 2 bytes (from the count of
// leading zeros), read as one big-endian pair.
#include "wnr3.cuh"
#include "rans_device.cuh"

namespace wexb {
namespace {

using namespace rans;

// Non-zero iff one of the eight nibbles of w is 8 (-0).
__device__ __forceinline__ uint32_t has_neg_zero(uint32_t w) {
    const uint32_t t = w ^ 0x88888888u;
    return (t - 0x11111111u) & ~t & 0x88888888u;
}
// Ceil-form inverse of eight nibbles: magnitude a -> a + min(a, 2), signs kept.
__device__ __forceinline__ uint32_t ceil_double(uint32_t w) {
    const uint32_t mag = w & 0x77777777u;
    const uint32_t two_or_more = ((mag >> 1) | (mag >> 2)) & 0x11111111u;
    const uint32_t least = (two_or_more << 1) | (mag & 0x11111111u & ~two_or_more);
    return (w & 0x88888888u) | (mag + least);
}

// ---- kernel A: scale streams ------------------------------------------------------------------
__global__ void __launch_bounds__(kScaleThreads) nr3_scales(const Nr3Record *__restrict__ recs,
                                                            const Nr3Task *__restrict__ tasks) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bar;
    uint8_t *ssym = smem;
    uint16_t *scdf = reinterpret_cast<uint16_t *>(smem + kTotal);
    uint32_t *ring = reinterpret_cast<uint32_t *>(smem + kTotal + kScdfBytes);
    const Nr3Task task = tasks[blockIdx.x];
    const Nr3Record &R = recs[task.rec];
    const uint32_t m = task.matrix;
    {
        void *dst[2] = {ssym, scdf};
        const void *src[2] = {R.t.ssym + (size_t)m * kTotal, reinterpret_cast<const uint8_t *>(R.t.scdf) + (size_t)m * kScdfBytes};
        const uint32_t bytes[2] = {kTotal, kScdfBytes};
        if (!stage_tables(&bar, dst, src, bytes, 2)) {
            if (threadIdx.x == 0) atomicOr(R.error, kErrTimeout);
            return;
        }
    }
    if (threadIdx.x >= task.count) return;
    const uint32_t j = task.first + threadIdx.x, g = R.sbase[m] + j;
    const uint32_t begin = R.offsets[g], end = R.offsets[g + 1];
    const uint32_t first = j * R.schunk, count = min(R.schunk, R.scount[m] - first);
    uint8_t *out = R.out + R.soff[m] + first;
    Reader rd{ring + threadIdx.x, blockDim.x, reinterpret_cast<const uint32_t *>(R.rec), 0, 0, 0};
    uint32_t x = rd.open(begin, end);
    if (x < kRansL || x >= (kRansL << 8)) { atomicOr(R.error, kErrStruct); rd.drain(); return; }
    const bool nr3 = R.flags & 256u, aligned = !(reinterpret_cast<uintptr_t>(out) & 3u);
    uint32_t h = nr3 ? ident_hash(R.model_id, R.owner, g, R.word24) : 0u;
    const uint32_t full = count & ~15u;
    for (uint32_t i = 0; i < full; i += 16) {
        rd.refill();
#pragma unroll
        for (uint32_t q = 0; q < 4; ++q) {
            uint32_t word = 0;
#pragma unroll
            for (uint32_t k = 0; k < 4; ++k) {
                const uint32_t two = rd.peek(), slot = x & (kTotal - 1u), y = ssym[slot], start = scdf[y];
                word |= y << (8u * k);
                x = (scdf[y + 1] - start) * (x >> kPrec) + slot - start;
                x = rd.renorm(x, two);
            }
            if (nr3) h = mm3_block(h, word);
            if (aligned) *reinterpret_cast<uint32_t *>(out + i + 4u * q) = word;
            else for (uint32_t k = 0; k < 4; ++k) out[i + 4u * q + k] = (uint8_t)(word >> (8u * k));
        }
    }
    if (full < count) {   // the last stream of a matrix: a partial group of 16
        rd.refill();
        uint32_t word = 0, held = 0;
        for (uint32_t i = full; i < count; ++i) {
            const uint32_t two = rd.peek(), slot = x & (kTotal - 1u), s = ssym[slot], start = scdf[s];
            out[i] = (uint8_t)s;
            word |= s << (8u * held);
            x = (scdf[s + 1] - start) * (x >> kPrec) + slot - start;
            x = rd.renorm(x, two);
            if (++held == 4) { if (nr3) h = mm3_block(h, word); word = 0; held = 0; }
        }
        if (nr3 && held) h ^= mm3_mix(word);
    }
    rd.drain();
    const uint32_t expect = nr3 ? kRansL + (mm3_final(h, 16u + count) & 0x7fffffu) : kRansL;
    if (rd.pos != end) atomicOr(R.error, kErrStruct);
    else if (x != expect) atomicOr(R.error, nr3 ? kErrHash : kErrStruct);
}

// a - b as a multiply-add on the FMA pipe (the integer ALU pipe is this kernel's limit)
__device__ __forceinline__ uint32_t sub_fma(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(b), "r"(0xffffffffu), "r"(a));
    return d;
}

// ---- kernel B: weight streams -----------------------------------------------------------------
// A lane's payload ring for the weight kernel: word w of the stream (counted from the stream's
// first word) lives in slot w % 32, slot 32 repeats slot 0, so the two words under any read
// position are slots s and s + 1 with no wrap. Slot s of lane l is ring[s * kThreads + l].
template <int kThreads>
struct WeightReader {
    uint32_t *ring;          // this lane's slot 0
    const uint32_t *src;     // the stream's first word in the record
    uint32_t bit;            // bit offset of the next payload byte from the stream's first word
    uint32_t req;            // next word to request
    uint32_t last;           // the stream's last word

    __device__ __forceinline__ void copy(uint32_t w, bool pred) { cp4(ring + (w & 31u) * kThreads, src + w, pred); }

    // Opens [begin, end) of the record (length >= 4, checked on the host); returns the initial state.
    __device__ __forceinline__ uint32_t open(const uint32_t *rec, uint32_t begin, uint32_t end) {
        src = rec + (begin >> 2);
        last = ((end - 1u) >> 2) - (begin >> 2);
        const uint32_t target = min(kAhead, last + 1u);
        for (uint32_t w = 0; w < target; ++w) copy(w, true);
        cp4(ring + 32u * kThreads, src, true);
        req = target;
        cp_commit();
        cp_wait<0>();
        const uint32_t v = __funnelshift_r(ring[0], ring[kThreads], (begin & 3u) * 8u);
        bit = (begin & 3u) * 8u + 32u;
        return __byte_perm(v, 0, 0x0123);   // big-endian bytes begin .. begin + 3
    }
    // Every 16 symbols (at most 32 bytes): keep kAhead words requested, then wait for the words of
    // the previous request, which cover every byte the next 16 symbols can read.
    __device__ __forceinline__ void refill() {
        const uint32_t target = min((bit >> 5) + kAhead, last + 1u);
#pragma unroll
        for (uint32_t k = 0; k < 8; ++k) copy(req + k, req + k < target);
        const uint32_t k0 = (0u - req) & 31u;   // the word of slot 0 among them, mirrored to slot 32
        cp4(ring + 32u * kThreads, src + req + k0, k0 < 8u && req + k0 < target);
        req = max(req, min(req + 8u, target));
        cp_commit();
        cp_wait<1>();
    }
    // The next four payload bytes, big-endian: enough for two symbols, each of which takes at most two.
    // Past the stream's end the ring holds stale words: consuming them is caught by the final position
    // check.
    __device__ __forceinline__ uint32_t peek4() const {
        const uint32_t *p = ring + ((bit >> 5) & 31u) * kThreads;
        return __byte_perm(__funnelshift_r(p[0], p[kThreads], bit), 0, 0x0123);
    }
    __device__ __forceinline__ void drain() const { cp_wait<0>(); }
};
// x in [2^9, 2^31) after a symbol: the bits (0, 8 or 16) to shift in until x >= 2^23.
__device__ __forceinline__ uint32_t renorm_bits(uint32_t x) { return ((uint32_t)__clz(x) - 1u) & 24u; }

template <int kThreads>
__global__ void __launch_bounds__(kThreads, 1024 / kThreads) nr3_weights(const Nr3Record *__restrict__ recs,
                                                                         const Nr3Task *__restrict__ tasks) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bar;
    const uint2 *level1 = reinterpret_cast<const uint2 *>(smem);
    const uint2 *level2 = reinterpret_cast<const uint2 *>(smem + kWL1Bytes);
    uint32_t *ring = reinterpret_cast<uint32_t *>(smem + kWBlockBytes);
    const Nr3Task task = tasks[blockIdx.x];
    const Nr3Record &R = recs[task.rec];
    const uint32_t m = task.matrix;
    {
        void *dst[1] = {smem};
        const void *src[1] = {R.t.wblk + (size_t)m * kWBlockBytes};
        const uint32_t bytes[1] = {kWBlockBytes};
        if (!stage_tables(&bar, dst, src, bytes, 1)) {
            if (threadIdx.x == 0) atomicOr(R.error, kErrTimeout);
            return;
        }
    }
    if (threadIdx.x >= task.count) return;
    const uint32_t j = task.first + threadIdx.x, g = R.wbase[m] + j;
    const uint32_t begin = R.offsets[g], end = R.offsets[g + 1];
    const uint32_t first = j * R.wchunk, blocks = min(R.wchunk, R.wcount[m] - first) / 32u;
    uint8_t *scales = R.out + R.soff[m] + first / 32u;   // coded scales; the ceil inverse edits them
    uint4 *out = reinterpret_cast<uint4 *>(R.out + R.wout[m] + first / 2u);
    WeightReader<kThreads> rd{ring + threadIdx.x, nullptr, 0, 0, 0};
    uint32_t x = rd.open(reinterpret_cast<const uint32_t *>(R.rec), begin, end);
    if (x < kRansL || x >= (kRansL << 8)) { atomicOr(R.error, kErrStruct); rd.drain(); return; }
    const bool nr3 = R.flags & 256u, cz = nr3 && (R.flags & 8u), ceil = nr3 && ((R.flags >> m) & 1u);
    const int anchor = (int)((R.word24 >> (8u * m)) & 0xffu);
    uint32_t h = nr3 ? ident_hash(R.model_id, R.owner, g, R.word24) : 0u;
    uint32_t scale = scales[0];
#pragma unroll 1
    for (uint32_t b = 0; b < blocks; ++b) {
        const uint32_t next_scale = b + 1 < blocks ? scales[b + 1] : 0u;
        const int d = (int)scale - anchor;
        const uint32_t srel = (uint32_t)(min(max(d, -3), 3) + 3) * kPairs;
        const uint2 *l1 = level1 + srel;
        const uint2 *l2 = level2 + 4u * srel;
        uint32_t idx = kPairs - 1u, top = 0, w[4] = {0, 0, 0, 0};   // the block-start context
        // one symbol: its quartile and rank from the two 8-byte rows of context idx, the state update,
        // then the next context (pair index top (top + 1) / 2 + mag)
        auto step = [&](uint32_t k) {
            const uint2 c = l1[idx];
            const uint32_t slot = x & (kTotal - 1u), gs = slot * 0x10001u + 0x80008000u;
            // q = [cdf[4] <= slot] + [cdf[8] <= slot] + [cdf[12] <= slot]
            const uint32_t d1 = sub_fma(gs, c.y);
            const uint32_t q = __popc((sub_fma(gs, c.x) & 0x80008000u) | ((d1 >> 1) & 0x4000u));
            const uint2 row = l2[4u * idx + q];   // cdf[4q] | cdf[4q+1] << 16, cdf[4q+2] | cdf[4q+3] << 16
            // r = [cdf[4q+1] <= slot] + [cdf[4q+2] <= slot] + [cdf[4q+3] <= slot]
            const uint32_t r = __popc((sub_fma(gs, row.y) & 0x80008000u) | (sub_fma(gs, row.x) >> 31));
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
            idx = ((top * top + top) >> 1) + mag;
        };
#pragma unroll
        for (uint32_t k = 0; k < 32; k += 2) {
            if (k == 0 || k == 16) rd.refill();
            uint32_t win = rd.peek4();   // the bytes of both symbols of the pair
            step(k);
            const uint32_t b1 = renorm_bits(x);
            x = __funnelshift_l(win, x, b1);
            win <<= b1;
            step(k + 1);
            const uint32_t b2 = renorm_bits(x);
            x = __funnelshift_l(win, x, b2);
            rd.bit += b1 + b2;
        }
        if (nr3) {   // hash and checks on the coded nibbles, then the ceil inverse
            h = mm3_block(mm3_block(mm3_block(mm3_block(h, w[0]), w[1]), w[2]), w[3]);
            if (cz && (has_neg_zero(w[0]) | has_neg_zero(w[1]) | has_neg_zero(w[2]) | has_neg_zero(w[3]))) {
                atomicOr(R.error, kErrCz);
                rd.drain();
                return;
            }
            if (ceil && top == 5u) {
                if (!scale) { atomicOr(R.error, kErrCeil); rd.drain(); return; }
#pragma unroll
                for (int q = 0; q < 4; ++q) w[q] = ceil_double(w[q]);
                scales[b] = (uint8_t)(scale - 1u);
            }
        }
        out[b] = make_uint4(w[0], w[1], w[2], w[3]);
        scale = next_scale;
    }
    rd.drain();
    const uint32_t expect = nr3 ? kRansL + (mm3_final(h, 16u + blocks * 16u) & 0x7fffffu) : kRansL;
    if (rd.bit != (end - (begin & ~3u)) * 8u) atomicOr(R.error, kErrStruct);
    else if (x != expect) atomicOr(R.error, nr3 ? kErrHash : kErrStruct);
}

// ---- commit -----------------------------------------------------------------------------------
__global__ void commit_regions(const CommitJob *__restrict__ jobs) {
    const CommitJob &J = jobs[blockIdx.z];
    if (*reinterpret_cast<const volatile uint32_t *>(J.error)) return;
    const uint32_t r = blockIdx.y;
    const uint8_t *from = J.src[r];
    uint8_t *to = J.dst[r];
    const size_t bytes = J.bytes[r], stride = (size_t)gridDim.x * blockDim.x;
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (!((reinterpret_cast<uintptr_t>(from) | reinterpret_cast<uintptr_t>(to)) & 15u)) {
        const size_t n16 = bytes / 16u;
        for (size_t k = i; k < n16; k += stride) reinterpret_cast<uint4 *>(to)[k] = reinterpret_cast<const uint4 *>(from)[k];
        for (size_t k = n16 * 16u + i; k < bytes; k += stride) to[k] = from[k];
    } else {
        for (size_t k = i; k < bytes; k += stride) to[k] = from[k];
    }
}

constexpr size_t scale_smem(int threads) { return kTotal + kScdfBytes + (size_t)kRingWords * 4u * threads; }
constexpr size_t weight_smem(int threads) { return kWBlockBytes + (size_t)(kRingWords + 1u) * 4u * threads; }

}  // namespace

cudaError_t prepare_nr3_kernels() {
    cudaError_t e = cudaFuncSetAttribute(nr3_scales, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)scale_smem(kScaleThreads));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(nr3_weights<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)weight_smem(128));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(nr3_weights<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)weight_smem(256));
    return e;
}

cudaError_t launch_nr3_scales(const Nr3Record *recs, const Nr3Task *tasks, uint32_t ntasks, cudaStream_t st) {
    if (!ntasks) return cudaSuccess;
    nr3_scales<<<ntasks, kScaleThreads, scale_smem(kScaleThreads), st>>>(recs, tasks);
    return cudaGetLastError();
}

cudaError_t launch_nr3_weights(const Nr3Record *recs, const Nr3Task *tasks, uint32_t ntasks, int threads, cudaStream_t st) {
    if (!ntasks) return cudaSuccess;
    if (threads == 256) nr3_weights<256><<<ntasks, 256, weight_smem(256), st>>>(recs, tasks);
    else if (threads == 128) nr3_weights<128><<<ntasks, 128, weight_smem(128), st>>>(recs, tasks);
    else return cudaErrorInvalidValue;
    return cudaGetLastError();
}

cudaError_t launch_commit(const CommitJob *jobs, uint32_t njobs, cudaStream_t st) {
    if (!njobs) return cudaSuccess;
    commit_regions<<<dim3(32, 6, njobs), 256, 0, st>>>(jobs);
    return cudaGetLastError();
}

}  // namespace wexb
