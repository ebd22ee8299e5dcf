// WBP1 decode kernels for sm_100a (structures in wbp1.cuh).
//
// wbp1_streams: a CTA serves one plane of one record. For a rANS plane it first builds the
// slot -> symbol table of the record's CDF in shared memory (each thread 64 consecutive slots: one
// binary search, then a walk) and the packed start | freq << 16 word of every symbol, then every lane
// decodes one stream through its payload window with the order-0 stream decoder the WNR3 scale
// streams use (rans_device.cuh), hashing the decoded bytes as it stores them; for a raw plane every
// lane copies one chunk and checks its MurmurHash3 word. wbp1_join writes each element's P bytes as
// one store, rotating it right by one bit under transform 1.
#include "wnr3.cuh"
#include "rans_device.cuh"
#include "wbp1.cuh"

namespace wexb {
namespace {

using namespace rans;

constexpr uint32_t kCdfBytes = 528;   // 257 u16, padded
constexpr uint32_t kSfWords = 256;
constexpr size_t kStreamSmem = kTotal + kCdfBytes + 4u * kSfWords + (size_t)(kWinWords + 1) * 4u * kWbp1Threads;

__device__ __forceinline__ uint32_t ident_hash(uint32_t owner, uint32_t g, uint32_t word) {
    uint32_t h = 0x33524e57u;
    h = mm3_block(h, kWbp1Magic); h = mm3_block(h, owner); h = mm3_block(h, g);
    return mm3_block(h, word);
}
__device__ __forceinline__ uint32_t rd32_bytes(const uint8_t *p) {
    return p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24;
}

__global__ void __launch_bounds__(kWbp1Threads) wbp1_streams(const Wbp1Record *__restrict__ recs,
                                                             const Wbp1Task *__restrict__ tasks) {
    extern __shared__ __align__(16) uint8_t smem[];
    uint8_t *ssym = smem;
    uint16_t *cdf = reinterpret_cast<uint16_t *>(smem + kTotal);
    uint32_t *sf = reinterpret_cast<uint32_t *>(smem + kTotal + kCdfBytes);
    uint32_t *ring = reinterpret_cast<uint32_t *>(smem + kTotal + kCdfBytes + 4u * kSfWords);
    const Wbp1Task task = tasks[blockIdx.x];
    const Wbp1Record &R = recs[task.rec];
    const uint32_t p = task.plane;
    const bool coded = (R.mask >> p) & 1u;
    if (coded) {   // the plane's CDF (validated on the host) and its slot -> symbol table
        const uint8_t *g = R.rec + R.cdf_at[p];
        for (uint32_t i = threadIdx.x; i < 257u; i += blockDim.x) cdf[i] = (uint16_t)(g[2 * i] | g[2 * i + 1] << 8);
        __syncthreads();
        for (uint32_t base = threadIdx.x * 64u; base < kTotal; base += blockDim.x * 64u) {
            uint32_t lo = 0, hi = 256;   // largest s with cdf[s] <= base
            while (hi - lo > 1) { const uint32_t mid = (lo + hi) / 2; if (cdf[mid] <= base) lo = mid; else hi = mid; }
            for (uint32_t k = 0; k < 64; ++k) {
                while (cdf[lo + 1] <= base + k) ++lo;
                ssym[base + k] = (uint8_t)lo;
            }
        }
        for (uint32_t i = threadIdx.x; i < kSfWords; i += blockDim.x) sf[i] = cdf[i] | (uint32_t)(cdf[i + 1] - cdf[i]) << 16;
        __syncthreads();
    }
    if (threadIdx.x >= task.count) return;
    const uint32_t s = task.first + threadIdx.x, g = R.gbase[p] + s;
    const uint32_t begin = R.offsets[g], end = R.offsets[g + 1];
    const uint32_t first = s * R.chunk, count = min(R.chunk, R.n[p] - first);
    uint8_t *out = R.planes + R.plane_at[p] + first;   // 4-byte aligned: plane_at and chunk are
    uint32_t h = ident_hash(R.owner, g, R.ident3);
    if (!coded) {   // raw chunk: copy, then its hash against the table word
        const uint8_t *src = R.rec + begin;
        uint32_t i = 0;
        for (; i + 4 <= count; i += 4) {
            const uint32_t w = rd32_bytes(src + i);
            *reinterpret_cast<uint32_t *>(out + i) = w;
            h = mm3_block(h, w);
        }
        if (i < count) {
            uint32_t k = 0;
            for (uint32_t t = count; t-- > i;) { k = k << 8 | src[t]; out[t] = src[t]; }
            h ^= mm3_mix(k);
        }
        if (mm3_final(h, 16u + count) != rd32_bytes(R.rec + R.table_at[p] + 4ull * s)) atomicOr(R.error, kErrHash);
        return;
    }
    PayloadWindow<kWbp1Threads> pw;
    uint32_t x = pw.open(R.rec, begin, end, smem_addr(ring + threadIdx.x));
    uint32_t err = (x - kRansL >= 255u * kRansL) ? kErrStruct : 0u;   // a valid initial state is in [L, 256 L)
    x = order0_stream(pw, x, smem_addr(ssym), smem_addr(sf), count, out, h);
    pw.close();
    if (pw.byte_pos() != end - (begin & ~3u)) err |= kErrStruct;
    else if (x != kRansL + (mm3_final(h, 16u + count) & 0x7fffffu)) err |= kErrHash;
    if (err) atomicOr(R.error, err);
}

// Element e of a record: byte p from plane p; under transform 1 the element (little-endian, P bytes)
// rotates right by one bit.
template <int P>
__device__ __forceinline__ void join_element(const Wbp1Record &R, uint64_t e) {
    uint8_t b[P];
#pragma unroll
    for (int p = 0; p < P; ++p) b[p] = R.planes[R.plane_at[p] + e];
    if (R.transform) {
        const uint8_t low = b[0] & 1u;
#pragma unroll
        for (int p = 0; p < P - 1; ++p) b[p] = (uint8_t)(b[p] >> 1 | (b[p + 1] & 1u) << 7);
        b[P - 1] = (uint8_t)(b[P - 1] >> 1 | low << 7);
    }
    uint8_t *o = R.out + e * P;
    if constexpr (P == 1) {
        o[0] = b[0];
    } else if constexpr (P == 2) {
        *reinterpret_cast<uint16_t *>(o) = (uint16_t)(b[0] | b[1] << 8);
    } else {
        uint32_t w[P / 4];
#pragma unroll
        for (int k = 0; k < P / 4; ++k) w[k] = b[4 * k] | (uint32_t)b[4 * k + 1] << 8 | (uint32_t)b[4 * k + 2] << 16 | (uint32_t)b[4 * k + 3] << 24;
        if constexpr (P == 4) *reinterpret_cast<uint32_t *>(o) = w[0];
        else *reinterpret_cast<uint2 *>(o) = make_uint2(w[0], w[1]);
    }
}

__global__ void wbp1_join(const Wbp1Record *__restrict__ recs) {
    const Wbp1Record &R = recs[blockIdx.y];
    const uint64_t whole = R.decoded / R.P, stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t e = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; e < whole; e += stride) {
        switch (R.P) {
            case 1: join_element<1>(R, e); break;
            case 2: join_element<2>(R, e); break;
            case 4: join_element<4>(R, e); break;
            default: join_element<8>(R, e); break;
        }
    }
    // a partial last element (no transform then): its bytes one by one
    const uint32_t tail = R.decoded - (uint32_t)(whole * R.P);
    if (tail && blockIdx.x == 0 && threadIdx.x < tail) R.out[whole * R.P + threadIdx.x] = R.planes[R.plane_at[threadIdx.x] + whole];
}

}  // namespace

cudaError_t prepare_wbp1_kernels() {
    return cudaFuncSetAttribute(wbp1_streams, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kStreamSmem);
}

cudaError_t launch_wbp1_streams(const Wbp1Record *recs, const Wbp1Task *tasks, uint32_t ntasks, cudaStream_t st) {
    if (!ntasks) return cudaSuccess;
    wbp1_streams<<<ntasks, kWbp1Threads, kStreamSmem, st>>>(recs, tasks);
    return cudaGetLastError();
}

cudaError_t launch_wbp1_join(const Wbp1Record *recs, uint32_t nrecs, cudaStream_t st) {
    if (!nrecs) return cudaSuccess;
    wbp1_join<<<dim3(64, nrecs), 256, 0, st>>>(recs);
    return cudaGetLastError();
}

}  // namespace wexb
