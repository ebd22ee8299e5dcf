// SHA-256 (FIPS 180-4) on the GPU: the per-record hash of stored bytes checked against a WEX4 index
// (c/wex4.h:673-677) and the content digest of a container (wex4/wex4_tools.c:125-158).
//
// A SHA-256 chain is serial, so one thread hashes one message; records hash concurrently, one thread
// each. The content digest is one message over many segments (tensor metadata from the host,
// decoded bytes on the device), hashed by a single thread in order.
#include "sha256.cuh"

namespace wexb {
namespace {

__constant__ uint32_t kSha[64] = {
    0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5,
    0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174,
    0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da,
    0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967,
    0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85,
    0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070,
    0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
    0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7, 0xc67178f2};

__device__ __forceinline__ uint32_t ror(uint32_t x, int r) { return __funnelshift_r(x, x, r); }
__device__ __forceinline__ uint32_t bswap(uint32_t x) { return __byte_perm(x, 0, 0x0123); }

// One compression of the big-endian message words w[0..15] into st.
__device__ __forceinline__ void compress(uint32_t st[8], uint32_t w[16]) {
    uint32_t a = st[0], b = st[1], c = st[2], d = st[3], e = st[4], f = st[5], g = st[6], h = st[7];
#pragma unroll
    for (int i = 0; i < 64; ++i) {
        uint32_t wi;
        if (i < 16) {
            wi = w[i];
        } else {   // the schedule kept in a 16-word circular window
            const uint32_t w15 = w[(i - 15) & 15], w2 = w[(i - 2) & 15];
            wi = w[i & 15] + (ror(w15, 7) ^ ror(w15, 18) ^ (w15 >> 3)) + w[(i - 7) & 15] +
                 (ror(w2, 17) ^ ror(w2, 19) ^ (w2 >> 10));
            w[i & 15] = wi;
        }
        const uint32_t t1 = h + (ror(e, 6) ^ ror(e, 11) ^ ror(e, 25)) + ((e & f) ^ (~e & g)) + kSha[i] + wi;
        const uint32_t t2 = (ror(a, 2) ^ ror(a, 13) ^ ror(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
        h = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
    }
    st[0] += a; st[1] += b; st[2] += c; st[3] += d; st[4] += e; st[5] += f; st[6] += g; st[7] += h;
}

__device__ __forceinline__ void init(uint32_t st[8]) {
    st[0] = 0x6a09e667; st[1] = 0xbb67ae85; st[2] = 0x3c6ef372; st[3] = 0xa54ff53a;
    st[4] = 0x510e527f; st[5] = 0x9b05688c; st[6] = 0x1f83d9ab; st[7] = 0x5be0cd19;
}

// Streaming state of one thread: the chaining value, a partial block of `fill` bytes, the length. The
// partial block lives in a byte buffer; the message words handed to compress() are always a fresh
// statically indexed array, so they stay in registers.
struct Sha {
    uint32_t st[8];
    uint8_t buf[64];
    uint32_t fill;
    uint64_t len;
    __device__ void start() { init(st); fill = 0; len = 0; }
    __device__ __forceinline__ void flush_buf() {
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
            w[i] = (uint32_t)buf[4 * i] << 24 | (uint32_t)buf[4 * i + 1] << 16 | (uint32_t)buf[4 * i + 2] << 8 | buf[4 * i + 3];
        compress(st, w);
    }
    __device__ __forceinline__ void byte(uint32_t v) {
        buf[fill] = (uint8_t)v;
        if (++fill == 64) { flush_buf(); fill = 0; }
    }
    __device__ void update(const uint8_t *p, uint64_t n) {
        len += n;
        while (n && fill) { byte(*p++); --n; }
        if (n >= 64 && !(reinterpret_cast<uintptr_t>(p) & 15)) {   // aligned whole blocks: four 16-byte loads each,
            const uint4 *q = reinterpret_cast<const uint4 *>(p);     // the next block's issued before this block's
            const uint4 *stop = q + 4 * (n / 64);                     // compression, an L2 prefetch 8 blocks ahead
            uint4 v[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) v[k] = __ldg(q + k);
            for (; n >= 64; n -= 64, p += 64, q += 4) {
                if (q + 32 < stop) asm volatile("prefetch.global.L2 [%0];" :: "l"(q + 32));
                uint32_t w[16];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    w[4 * k] = bswap(v[k].x); w[4 * k + 1] = bswap(v[k].y); w[4 * k + 2] = bswap(v[k].z); w[4 * k + 3] = bswap(v[k].w);
                }
                if (n >= 128) {
#pragma unroll
                    for (int k = 0; k < 4; ++k) v[k] = __ldg(q + 4 + k);
                }
                compress(st, w);
            }
        } else if (n >= 64) {   // unaligned whole blocks: aligned 4-byte words joined by funnel shifts
            const uint32_t shift = (uint32_t)(reinterpret_cast<uintptr_t>(p) & 3u) * 8u;
            const uint32_t *q = reinterpret_cast<const uint32_t *>(reinterpret_cast<uintptr_t>(p) & ~(uintptr_t)3);
            for (; n >= 64; n -= 64, p += 64, q += 16) {
                uint32_t w[16], next = __ldg(q);
#pragma unroll
                for (int k = 0; k < 16; ++k) {
                    const uint32_t cur = next;
                    // the 17th word holds the block's last bytes only when the block is unaligned
                    next = (k < 15 || shift) ? __ldg(q + k + 1) : 0u;
                    w[k] = bswap(__funnelshift_r(cur, next, shift));
                }
                compress(st, w);
            }
        }
        while (n) { byte(*p++); --n; }
    }
    __device__ void finish(uint8_t *out) {
        const uint64_t bits = len * 8;
        byte(0x80);
        while (fill != 56) byte(0);
        for (int i = 7; i >= 0; --i) byte((uint32_t)(bits >> (8 * i)) & 0xffu);
        for (int i = 0; i < 32; ++i) out[i] = (uint8_t)(st[i / 4] >> (24 - 8 * (i % 4)));
    }
};

// Record hashes, two warps per 32 messages (lane l of both warps serves message l of the CTA). A single
// thread's chain is issue-bound on the integer pipe, so the work is split: warp 1 loads each 64-byte
// block (or builds the padded last blocks) and expands its schedule into W[t] + K[t] in shared memory;
// warp 0 runs only the 64 rounds from there. Two slots alternate, with one CTA barrier per block;
// messages shorter than the CTA's longest keep their final state through the extra blocks. A slot
// holds the rounds of a lane four at a time ([group of 4 rounds][lane], 16 bytes), so the round warp
// reads them with one 16-byte load per four rounds, issued a group ahead: its chain never waits on
// shared memory.
constexpr int kShaLanes = 32;
__device__ __forceinline__ uint32_t msg_blocks(uint64_t bytes) { return (uint32_t)((bytes + 9 + 63) / 64); }

__device__ __forceinline__ void produce_block(const uint8_t *data, uint64_t bytes, uint32_t b, uint32_t w[16]) {
    const uint64_t at = 64ull * b;
    if (at + 64 <= bytes) {   // a whole data block (data is 16-byte aligned)
        const uint4 *q = reinterpret_cast<const uint4 *>(data + at);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint4 v = __ldcg(q + k);
            w[4 * k] = bswap(v.x); w[4 * k + 1] = bswap(v.y); w[4 * k + 2] = bswap(v.z); w[4 * k + 3] = bswap(v.w);
        }
        return;
    }
    // the message end: data bytes, 0x80, zeros, and in the last block the bit length (big-endian)
    const uint64_t bits = bytes * 8;
    const bool last = b + 1 == msg_blocks(bytes);
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        uint32_t v = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint64_t pos = at + 4 * k + j;
            const uint32_t byte = pos < bytes ? __ldcg(data + pos) : pos == bytes ? 0x80u : 0u;
            v = v << 8 | byte;
        }
        w[k] = v;
    }
    if (last) { w[14] = (uint32_t)(bits >> 32); w[15] = (uint32_t)bits; }
}

// The producer warp, before it reads block b of its lanes' messages (every lane at the same block):
// waits (bounded, lane 0 polling with a sleep that doubles up to 8 us) until the upload pass holding
// that block has landed. `landed`: passes known to be in place. False when the wait gave up.
__device__ __forceinline__ bool gate_wait(const ShaParts &P, uint32_t b, uint32_t &landed) {
    if (!P.gate) return true;
    const uint32_t pass = (uint32_t)((64ull * b) >> P.gate_shift);
    if (pass < landed) return true;
    uint32_t ok = 1;
    if ((threadIdx.x & 31u) == 0) {
        ok = 0;
        uint32_t nap = 64;
        for (uint32_t n = 0; n < (1u << 24); ++n) {
            uint32_t v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(P.gate + pass) : "memory");
            if (v >= P.gate_token) { ok = 1; break; }
            __nanosleep(nap);
            nap = min(2u * nap, 8192u);
        }
        if (!ok) atomicExch(P.gate_fail, 1u);
    }
    ok = __shfl_sync(~0u, ok, 0);
    __syncwarp();
    if (ok) landed = pass + 1;
    return ok != 0;
}

__global__ void __launch_bounds__(2 * kShaLanes) sha256_messages(const ShaParts P) {
    __shared__ uint4 sched[2][16][kShaLanes];   // [slot][rounds 4g .. 4g+3][lane]: W[t] + K[t]
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t i = blockIdx.x * kShaLanes + lane;
    const bool active = P.nparts && i < P.end[P.nparts - 1];
    uint32_t part = 0;
    while (active && i >= P.end[part]) ++part;
    const ShaMsg m = active ? P.part[part][i - (part ? P.end[part - 1] : 0u)] : ShaMsg{nullptr, 0, nullptr, nullptr, nullptr, 0};
    const uint32_t mine = active ? msg_blocks(m.bytes) : 0u;
    const uint32_t blocks = __reduce_max_sync(0xffffffffu, mine);
    if (warp == 1) {   // producer
        // a whole data block's four 16-byte loads are issued one block ahead, before the schedule work of
        // the current block, so their latency is hidden behind it
        // (coherent L2 loads: with a gate the bytes land while the launch runs)
        uint4 v[4];
        bool ahead = false;
        uint32_t landed = 0;   // upload passes known to be in place (gated launches)
        auto load = [&](uint32_t b) {
            ahead = 64ull * b + 64 <= m.bytes;
            if (!ahead) return;
            const uint4 *q = reinterpret_cast<const uint4 *>(m.data + 64ull * b);
#pragma unroll
            for (int k = 0; k < 4; ++k) v[k] = __ldcg(q + k);
        };
        if (blocks) gate_wait(P, 0, landed);
        if (mine) load(0);
        for (uint32_t b = 0; b < blocks; ++b) {
            if (b + 1 < blocks) gate_wait(P, b + 1, landed);   // the block loaded one ahead (warp-uniform)
            if (b < mine) {
                uint32_t w[16];
                if (ahead) {
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        w[4 * k] = bswap(v[k].x); w[4 * k + 1] = bswap(v[k].y);
                        w[4 * k + 2] = bswap(v[k].z); w[4 * k + 3] = bswap(v[k].w);
                    }
                } else {
                    produce_block(m.data, m.bytes, b, w);
                }
                if (b + 1 < mine) load(b + 1);
                if (64ull * (b + 8) + 64 <= m.bytes && (!P.gate || ((64ull * (b + 8)) >> P.gate_shift) < landed))
                    asm volatile("prefetch.global.L2 [%0];" :: "l"(m.data + 64ull * (b + 8)));
                uint4 (*out)[kShaLanes] = sched[b & 1];
                uint32_t wk[4];
#pragma unroll
                for (int t = 0; t < 64; ++t) {
                    uint32_t wt;
                    if (t < 16) {
                        wt = w[t];
                    } else {
                        const uint32_t w15 = w[(t - 15) & 15], w2 = w[(t - 2) & 15];
                        wt = w[t & 15] + (ror(w15, 7) ^ ror(w15, 18) ^ (w15 >> 3)) + w[(t - 7) & 15] +
                             (ror(w2, 17) ^ ror(w2, 19) ^ (w2 >> 10));
                        w[t & 15] = wt;
                    }
                    wk[t & 3] = wt + kSha[t];
                    if ((t & 3) == 3) out[t >> 2][lane] = make_uint4(wk[0], wk[1], wk[2], wk[3]);
                }
            }
            __syncthreads();
        }
        return;
    }
    uint32_t st[8];   // consumer
    init(st);
    for (uint32_t b = 0; b < blocks; ++b) {
        __syncthreads();
        if (b >= mine) continue;
        const uint4 (*in)[kShaLanes] = sched[b & 1];
        uint32_t a = st[0], bb = st[1], c = st[2], d = st[3], e = st[4], f = st[5], g = st[6], h = st[7];
        // W + K of rounds 4q .. 4q+3 (cur) and of the next group (ahead, loaded a group early)
        uint4 cur = in[0][lane], ahead = in[1][lane];
        // hk = h + W[t] + K[t], formed a round early (the next round's h is this round's g), so that the
        // new e and a are one three-input add after the round's rotations and logic functions
        uint32_t hk = h + cur.x;
#pragma unroll
        for (int t = 0; t < 64; ++t) {
            const uint32_t s1 = ror(e, 6) ^ ror(e, 11) ^ ror(e, 25), ch = (e & f) ^ (~e & g);
            const uint32_t s0 = ror(a, 2) ^ ror(a, 13) ^ ror(a, 22), mj = (a & bb) ^ (a & c) ^ (bb & c);
            const uint32_t dhk = d + hk, t1 = hk + s1 + ch;
            uint32_t next_hk = 0;
            if (t < 63) {
                const int u = (t + 1) & 3;
                if (u == 0) {   // round t + 1 opens the next group: shift, and load the one after it
                    cur = ahead;
                    if ((t + 1) / 4 + 1 < 16) ahead = in[(t + 1) / 4 + 1][lane];
                }
                next_hk = g + (u == 0 ? cur.x : u == 1 ? cur.y : u == 2 ? cur.z : cur.w);
            }
            h = g; g = f; f = e; e = dhk + s1 + ch; d = c; c = bb; bb = a; a = t1 + (s0 + mj);
            hk = next_hk;
        }
        st[0] += a; st[1] += bb; st[2] += c; st[3] += d; st[4] += e; st[5] += f; st[6] += g; st[7] += h;
    }
    if (!active) return;
    uint32_t differ = 0;
    for (int k = 0; k < 32; ++k) {
        const uint8_t got = (uint8_t)(st[k / 4] >> (24 - 8 * (k % 4)));
        if (m.digest) m.digest[k] = got;
        if (m.expect) differ |= got ^ m.expect[k];
    }
    if (!m.verdict) return;
    if (m.or_bits) { if (m.expect && differ) atomicOr(m.verdict, m.or_bits); }
    else *m.verdict = m.expect ? (differ ? 1u : 0u) : 0u;
}

__global__ void sha256_segments(const ShaMsg *__restrict__ segs, uint32_t n, uint8_t *digest) {
    if (blockIdx.x || threadIdx.x) return;
    Sha s;
    s.start();
    for (uint32_t i = 0; i < n; ++i) s.update(segs[i].data, segs[i].bytes);
    s.finish(digest);
}

}  // namespace

cudaError_t launch_sha256_parts(const ShaParts &P, cudaStream_t st) {
    const uint32_t n = P.nparts ? P.end[P.nparts - 1] : 0u;
    if (!n) return cudaSuccess;
    if (P.nparts > (uint32_t)kShaParts) return cudaErrorInvalidValue;
    sha256_messages<<<(n + kShaLanes - 1) / kShaLanes, 2 * kShaLanes, 0, st>>>(P);
    return cudaGetLastError();
}

cudaError_t launch_sha256_messages(const ShaMsg *msgs, uint32_t n, cudaStream_t st) {
    ShaParts P{};   // no gate
    P.part[0] = msgs;
    P.end[0] = n;
    P.nparts = 1;
    return launch_sha256_parts(P, st);
}

cudaError_t launch_sha256_segments(const ShaMsg *segs, uint32_t n, uint8_t *digest, cudaStream_t st) {
    sha256_segments<<<1, 1, 0, st>>>(segs, n, digest);
    return cudaGetLastError();
}

}  // namespace wexb
