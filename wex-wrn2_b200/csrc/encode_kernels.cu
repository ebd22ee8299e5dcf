// Kernels of the GPU record writer (encode.cuh): training counts, stream encoder, length scan, packing.
#include <cstdint>

#include "encode.cuh"
#include "rans_device.cuh"

namespace wexb {
namespace {

using rans::ident_hash;
using rans::mm3_block;
using rans::mm3_final;
using rans::mm3_mix;

constexpr uint32_t kL = 1u << 23, kPrec = 14;
constexpr uint32_t kWnr3Magic = 0x33524e57u, kWnr2Magic = 0x32524e57u;

__device__ __forceinline__ uint32_t ld_u32(const uint8_t *p, bool aligned) {
    if (aligned) return *reinterpret_cast<const uint32_t *>(p);
    return p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24;
}

// The stream's bytes written downwards from `top`, four at a time once four are pending. The slot below
// `top` holds at least 2 bytes per symbol plus the flush (a symbol emits at most 2 bytes: x < 2^31 and
// the renormalisation bound is freq << 17), so `room` never runs out for a valid slot size; it is
// checked anyway and an overflow is reported instead of written.
struct Sink {
    uint8_t *p;
    uint32_t room, acc, pending;
    bool overflow;
    __device__ __forceinline__ void emit(uint32_t b) {
        acc = acc << 8 | b;
        if (++pending == 4) {
            if (room >= 4) { p -= 4; room -= 4; *reinterpret_cast<uint32_t *>(p) = acc; }
            else overflow = true;
            pending = 0;
        }
    }
    __device__ __forceinline__ void put(uint32_t &x, uint32_t start, uint32_t freq) {
        const uint32_t bound = freq << 17;   // ((L >> 14) << 8) * freq
        while (x >= bound) { emit(x & 0xffu); x >>= 8; }
        x = ((x / freq) << kPrec) + x % freq + start;
    }
    __device__ __forceinline__ void finish(uint32_t x) {
        for (int b = 0; b < 4; ++b) { emit(x & 0xffu); x >>= 8; }
        if (pending > room) { overflow = true; return; }
        for (uint32_t i = 0; i < pending; ++i) p[-1 - (int)i] = (uint8_t)(acc >> (8 * (pending - 1 - i)));
        p -= pending; room -= pending;
    }
};

__device__ __forceinline__ uint32_t word24_of(const EncRecord &R) {
    return R.anchor[0] | (uint32_t)R.anchor[1] << 8 | (uint32_t)R.anchor[2] << 16 | R.flags << 24;
}

// One CTA per (record, matrix): the histogram of the matrix's scales, then its anchor.
__global__ void __launch_bounds__(256) enc_anchor(EncRecord *recs) {
    __shared__ uint32_t hist[256];
    EncRecord &R = recs[blockIdx.x / 3];
    const uint32_t m = blockIdx.x % 3, n = R.scount[m];
    const uint8_t *s = R.coded + R.soff[m];
    hist[threadIdx.x] = 0;
    __syncthreads();
    uint32_t i0 = 0;
    if (!(reinterpret_cast<uintptr_t>(s) & 15u)) {   // 16 scales a load
        const uint4 *v = reinterpret_cast<const uint4 *>(s);
        for (uint32_t i = threadIdx.x; i < n / 16; i += blockDim.x) {
            const uint4 q = v[i];
            const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int k = 0; k < 16; ++k) atomicAdd(&hist[(w[k >> 2] >> (8 * (k & 3))) & 0xffu], 1u);
        }
        i0 = n & ~15u;
    }
    for (uint32_t i = i0 + threadIdx.x; i < n; i += blockDim.x) atomicAdd(&hist[s[i]], 1u);
    __syncthreads();
    if (threadIdx.x) return;
    uint32_t best = 0;
    if (R.nr3) {   // rule g: the lower value of the adjacent pair holding most scales, first on ties
        uint32_t top = 0;
        for (uint32_t v = 0; v < 255; ++v)
            if (hist[v] + hist[v + 1] > top) { top = hist[v] + hist[v + 1]; best = v; }
    } else {       // the lower median
        uint32_t seen = 0;
        best = 255;
        for (uint32_t v = 0; v < 256; ++v) { seen += hist[v]; if (seen * 2u >= n) { best = v; break; } }
    }
    R.anchor[m] = (uint8_t)best;
}

// One CTA: up to kEncThreads streams of one matrix (c/wex_neural_rans.h:615-713).
__global__ void __launch_bounds__(kEncThreads) enc_streams(const uint8_t *__restrict__ blob, const EncRecord *recs,
                                                           const EncTask *tasks) {
    __shared__ uint16_t cdf[kEncContexts * kEncCdfRow];
    const EncTask T = tasks[blockIdx.x];
    const EncRecord &R = recs[T.rec];
    const uint32_t m = T.m;
    const uint16_t *src = reinterpret_cast<const uint16_t *>(
        blob + 32 + (T.scale ? 3u * kEncContexts * 34u + 514u * m : 34u * kEncContexts * m));
    const uint32_t entries = T.scale ? 257u : kEncContexts * kEncCdfRow;
    for (uint32_t i = threadIdx.x; i < entries; i += blockDim.x) cdf[i] = src[i];
    __syncthreads();
    if (threadIdx.x >= T.count) return;
    const uint32_t k = T.first + threadIdx.x;
    const uint32_t chunk = T.scale ? R.schunk : R.wchunk, all = T.scale ? R.scount[m] : R.wcount[m];
    const uint32_t first = k * chunk, count = min(chunk, all - first);
    const uint32_t g = (T.scale ? R.sbase[m] : R.wbase[m]) + k;
    const uint8_t *s = R.coded + R.soff[m];
    const uint8_t *bytes = T.scale ? s + first : R.coded + R.woff[m] + first / 2;
    const uint32_t nbytes = T.scale ? count : count / 2;
    const bool aligned = (reinterpret_cast<uintptr_t>(bytes) & 3u) == 0;
    // initial state = the state the decoder must end in (c/wex_neural_rans.h:225-245)
    uint32_t x = kL;
    if (R.nr3) {
        uint32_t h = ident_hash(R.model_id, R.owner, g, word24_of(R)), i = 0;
        for (; i + 4 <= nbytes; i += 4) h = mm3_block(h, ld_u32(bytes + i, aligned));
        if (nbytes & 3u) {
            uint32_t t = 0;
            for (uint32_t q = nbytes & 3u; q-- > 0;) t = t << 8 | bytes[i + q];
            h ^= mm3_mix(t);
        }
        x = kL + (mm3_final(h, 16u + nbytes) & 0x7fffffu);
    }
    Sink out{R.scratch + (size_t)(g + 1) * R.slot_bytes, R.slot_bytes, 0, 0, false};
    uint32_t err = 0;
    if (T.scale) {
        for (uint32_t j = count; j-- > 0;) {
            const uint32_t sym = bytes[j], start = cdf[sym];
            out.put(x, start, cdf[sym + 1] - start);
        }
    } else {
        const uint8_t anchor = R.anchor[m];
        for (uint32_t b = count / 32; b-- > 0;) {   // 32-nibble blocks, last to first
            const uint8_t *q8 = bytes + 16 * b;
            uint32_t q[4];
#pragma unroll
            for (int w = 0; w < 4; ++w) q[w] = ld_u32(q8 + 4 * w, aligned);
            const int d = (int)s[(first >> 5) + b] - (int)anchor;
            const uint32_t srel = (uint32_t)(max(-3, min(3, d)) + 3);
            uint32_t ctx[32], prev = 8, top = 8;
#pragma unroll
            for (int j = 0; j < 32; ++j) {   // contexts run forwards
                const uint32_t v = (q[j >> 3] >> (4 * (j & 7))) & 15u;
                ctx[j] = ((srel * 9 + prev) * 9 + top) * kEncCdfRow;
                if (R.cz && v == 8u) err |= kEncErrCz;
                prev = v & 7u;
                if (top == 8 || prev > top) top = prev;
            }
#pragma unroll
            for (int j = 31; j >= 0; --j) {   // the coder runs backwards
                const uint32_t v = (q[j >> 3] >> (4 * (j & 7))) & 15u;
                const uint16_t *row = cdf + ctx[j];
                const uint32_t start = row[v];
                out.put(x, start, row[v + 1] - start);
            }
        }
    }
    out.finish(x);
    if (out.overflow) err |= kEncErrOverflow;
    R.lens[g] = R.slot_bytes - out.room;
    if (err) atomicOr(R.err, err);
}

// One CTA per record: stream offsets (exclusive scan of the lengths), the verdict, header, length
// table and zero padding (c/wex_neural_rans.h:714-749).
__global__ void __launch_bounds__(1024) enc_scan(const EncRecord *recs) {
    __shared__ uint32_t warp_sum[32];
    __shared__ uint64_t bytes_of[2];
    const EncRecord &R = recs[blockIdx.x];
    const uint32_t S = R.streams, per = (S + blockDim.x - 1) / blockDim.x;
    const uint32_t lo = min(S, threadIdx.x * per), hi = min(S, lo + per), sstreams = R.wbase[0];
    if (threadIdx.x < 2) bytes_of[threadIdx.x] = 0;
    uint32_t sum = 0, ssum = 0, big = 0;
    for (uint32_t g = lo; g < hi; ++g) {
        const uint32_t n = R.lens[g];
        sum += n;
        if (g < sstreams) ssum += n;
        big |= n > 65535u;
    }
    // block-wide exclusive scan of the per-thread sums (32 warps)
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    uint32_t incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= (uint32_t)o) incl += t;
    }
    if (lane == 31) warp_sum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const uint32_t v = lane < (blockDim.x >> 5) ? warp_sum[lane] : 0u;
        uint32_t w = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t t = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= (uint32_t)o) w += t;
        }
        warp_sum[lane] = w - v;
    }
    if (big) atomicOr(R.err, kEncErrOverflow);
    atomicAdd(reinterpret_cast<unsigned long long *>(&bytes_of[0]), (unsigned long long)ssum);
    atomicAdd(reinterpret_cast<unsigned long long *>(&bytes_of[1]), (unsigned long long)(sum - ssum));
    __syncthreads();
    uint32_t at = warp_sum[warp] + incl - sum;
    for (uint32_t g = lo; g < hi; ++g) { R.lens[S + g] = at; at += R.lens[g]; }
    const uint64_t meta = 32ull + 2ull * S, used = meta + bytes_of[0] + bytes_of[1];
    const uint64_t padded = (used + 4095u) & ~4095ull;
    const uint32_t err = *R.err;
    const int64_t status = err ? -1 : (used > R.cap || padded > R.cap) ? -1 : padded >= R.raw_aligned ? 1 : 0;
    if (threadIdx.x == 0) { R.result[0] = (uint64_t)status; R.result[1] = used; R.result[2] = padded; }
    if (status != 0) return;
    uint8_t *o = R.out;
    if (threadIdx.x == 0) {
        const uint32_t head[8] = {R.nr3 ? kWnr3Magic : kWnr2Magic, R.model_id, (uint32_t)bytes_of[0], (uint32_t)bytes_of[1],
                                  R.wchunk, R.schunk, word24_of(R), R.owner};
        for (int i = 0; i < 8; ++i)
            for (int b = 0; b < 4; ++b) o[4 * i + b] = (uint8_t)(head[i] >> (8 * b));
    }
    for (uint32_t g = threadIdx.x; g < S; g += blockDim.x) {
        o[32 + 2 * g] = (uint8_t)R.lens[g];
        o[33 + 2 * g] = (uint8_t)(R.lens[g] >> 8);
    }
    for (uint64_t i = used + threadIdx.x; i < padded; i += blockDim.x) o[i] = 0;
}

// One warp per stream: the payload behind the length table, for records whose verdict is 0.
__global__ void __launch_bounds__(256) enc_pack(const EncRecord *recs, const uint32_t *stream_rec, uint32_t total) {
    const uint32_t gs = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31u;
    if (gs >= total) return;
    const EncRecord &R = recs[stream_rec[2 * gs]];
    if (R.result[0] != 0) return;
    const uint32_t g = stream_rec[2 * gs + 1], len = R.lens[g];
    const uint8_t *src = R.scratch + (size_t)(g + 1) * R.slot_bytes - len;
    uint8_t *dst = R.out + 32 + 2 * (size_t)R.streams + R.lens[R.streams + g];
    for (uint32_t i = lane; i < len; i += 32) dst[i] = src[i];
}

// Training counts (c/wex_neural_rans.h:579-613): a shared histogram per CTA, added to the global u64
// counters at the end.
__global__ void __launch_bounds__(256) enc_count(const EncRecord *recs, const CountTask *tasks, unsigned long long *wc,
                                                 unsigned long long *sc) {
    __shared__ uint32_t hist[kEncContexts * 16];
    const CountTask T = tasks[blockIdx.x];
    const EncRecord &R = recs[T.rec];
    const uint32_t m = T.m, bins = T.scale ? 256u : kEncContexts * 16u;
    for (uint32_t i = threadIdx.x; i < bins; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const uint8_t *s = R.coded + R.soff[m];
    if (T.scale) {
        for (uint32_t i = T.first + threadIdx.x; i < T.first + T.count; i += blockDim.x) atomicAdd(&hist[s[i]], 1u);
    } else {
        const uint8_t *w = R.coded + R.woff[m];
        const bool aligned = (reinterpret_cast<uintptr_t>(w) & 3u) == 0;
        const uint8_t anchor = R.anchor[m];
        for (uint32_t b = T.first + threadIdx.x; b < T.first + T.count; b += blockDim.x) {
            uint32_t q[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) q[k] = ld_u32(w + 16 * (size_t)b + 4 * k, aligned);
            const int d = (int)s[b] - (int)anchor;
            const uint32_t srel = (uint32_t)(max(-3, min(3, d)) + 3);
            uint32_t prev = 8, top = 8;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const uint32_t v = (q[j >> 3] >> (4 * (j & 7))) & 15u;
                atomicAdd(&hist[((srel * 9 + prev) * 9 + top) * 16u + v], 1u);
                prev = v & 7u;
                if (top == 8 || prev > top) top = prev;
            }
        }
    }
    __syncthreads();
    unsigned long long *dst = T.scale ? sc + 256u * m : wc + (size_t)kEncContexts * 16u * m;
    for (uint32_t i = threadIdx.x; i < bins; i += blockDim.x)
        if (hist[i]) atomicAdd(dst + i, (unsigned long long)hist[i]);
}

}  // namespace

cudaError_t launch_encode(const uint8_t *dblob, EncRecord *recs, uint32_t first, uint32_t nrec, const EncTask *tasks,
                          uint32_t ntasks, const uint32_t *stream_rec, uint32_t nstreams, cudaStream_t st) {
    if (!nrec) return cudaSuccess;
    enc_anchor<<<3 * nrec, 256, 0, st>>>(recs + first);
    enc_streams<<<ntasks, kEncThreads, 0, st>>>(dblob, recs, tasks);
    enc_scan<<<nrec, 1024, 0, st>>>(recs + first);
    const uint32_t warps_per_cta = 256 / 32;
    enc_pack<<<(nstreams + warps_per_cta - 1) / warps_per_cta, 256, 0, st>>>(recs, stream_rec, nstreams);
    return cudaGetLastError();
}

cudaError_t launch_count(EncRecord *recs, uint32_t nrec, const CountTask *tasks, uint32_t ntasks, unsigned long long *wc,
                         unsigned long long *sc, cudaStream_t st) {
    if (!ntasks) return cudaSuccess;
    enc_anchor<<<3 * nrec, 256, 0, st>>>(recs);
    enc_count<<<ntasks, 256, 0, st>>>(recs, tasks, wc, sc);
    return cudaGetLastError();
}

}  // namespace wexb
