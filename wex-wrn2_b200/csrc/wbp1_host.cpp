// Host side of WBP1 (codec 6): validation and planning for wbp1_kernels.cu, and the canonical encoder
// (the record layout of the reference's docs/WEX4-SPEC.md section 7.2, c/wex4.h:446-660).
#include "wbp1_host.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "nr3_host.h"

namespace wexb {
namespace {

constexpr uint32_t kPage = 4096, kHeader = 16, kMaxDecoded = 1u << 30, kRansLHost = 1u << 23, kPrecHost = 14;
constexpr uint32_t kTotalHost = 1u << kPrecHost;

uint32_t plane_bytes(uint32_t decoded, uint32_t P, uint32_t p) { return decoded > p ? (decoded - p + P - 1) / P : 0; }
bool cdf_ok(const uint8_t *c) {
    if (rd16(c) != 0 || rd16(c + 512) != kTotalHost) return false;
    for (uint32_t s = 0; s < 256; ++s) if (rd16(c + 2 * s) >= rd16(c + 2 * s + 2)) return false;
    return true;
}

// MurmurHash3_x86_32 pieces with the WNR3 seed, over an ident block then data (c/wex_neural_rans.h:196-233)
uint32_t rotl(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }
uint32_t mix(uint32_t k) { return rotl(k * 0xcc9e2d51u, 15) * 0x1b873593u; }
uint32_t block(uint32_t h, uint32_t k) { return rotl(h ^ mix(k), 13) * 5u + 0xe6546b64u; }
uint32_t final(uint32_t h, uint32_t len) {
    h ^= len; h ^= h >> 16; h *= 0x85ebca6bu; h ^= h >> 13; h *= 0xc2b2ae35u; h ^= h >> 16;
    return h;
}
uint32_t h32(const uint32_t ident[4], const uint8_t *p, uint32_t n) {
    uint32_t h = 0x33524e57u, i = 0;
    for (int k = 0; k < 4; ++k) h = block(h, ident[k]);
    for (; i + 4 <= n; i += 4) h = block(h, rd32(p + i));
    if (n & 3u) {
        uint32_t k = 0;
        for (uint32_t t = n & 3u; t-- > 0;) k = k << 8 | p[i + t];
        h ^= mix(k);
    }
    return final(h, 16u + n);
}

// 14-bit CDF of 256 counts: every symbol at least 1, the rest in proportion, the remainder one each to
// the largest fractional parts, the lower symbol first on ties (c/wex_neural_rans.h:536-562).
void quantize(const uint64_t counts[256], uint16_t cdf[257]) {
    uint64_t total = 0, rem[256];
    uint32_t freq[256], used = 0;
    const uint32_t spare = kTotalHost - 256;
    bool taken[256] = {};
    for (int s = 0; s < 256; ++s) total += counts[s];
    for (int s = 0; s < 256; ++s) {
        const uint64_t scaled = total ? counts[s] * spare : spare, div = total ? total : 256;
        freq[s] = 1u + (uint32_t)(scaled / div);
        rem[s] = scaled % div;
        used += freq[s];
    }
    for (uint32_t extra = kTotalHost - used; extra; --extra) {
        int best = -1;
        for (int s = 0; s < 256; ++s) if (!taken[s] && (best < 0 || rem[s] > rem[best])) best = s;
        taken[best] = true; ++freq[best];
    }
    uint32_t at = 0;
    for (int s = 0; s <= 256; ++s) { cdf[s] = (uint16_t)at; if (s < 256) at += freq[s]; }
}

std::mutex g_prep_mu;
bool g_prepared[kMaxDevices];

}  // namespace

int wbp1_parse(const uint8_t *rec, size_t total, uint32_t decoded, uint32_t owner, Wbp1Plan *b) {
    if (!rec || !b || total < kPage || (total & (kPage - 1)) || rd32(rec) != kWbp1Magic || rd32(rec + 4) != owner ||
        rd32(rec + 8) != decoded || !decoded || decoded > kMaxDecoded) return -1;
    Wbp1Plan v;
    v.decoded = decoded; v.owner = owner; v.P = rec[12]; v.chunk_log2 = rec[13]; v.mask = rec[14]; v.transform = rec[15];
    if ((v.P != 1 && v.P != 2 && v.P != 4 && v.P != 8) || v.chunk_log2 < 10 || v.chunk_log2 > 15 || (v.mask >> v.P) ||
        v.transform > 1 || (v.transform && (v.P == 1 || decoded % v.P))) return -1;
    v.chunk = 1u << v.chunk_log2;
    uint64_t at = kHeader;
    uint32_t g = 0;
    for (uint32_t p = 0; p < v.P; ++p) {
        v.n[p] = plane_bytes(decoded, v.P, p);
        v.streams[p] = (uint32_t)(((uint64_t)v.n[p] + v.chunk - 1) / v.chunk);
        v.gbase[p] = g; g += v.streams[p];
        if (!((v.mask >> p) & 1u)) continue;
        if (!v.n[p] || total - at < 514) return -1;
        v.cdf_at[p] = (uint32_t)at; at += 514;
        if (!cdf_ok(rec + v.cdf_at[p])) return -1;
    }
    v.total_streams = g;
    for (uint32_t p = 0; p < v.P; ++p) {
        const uint64_t bytes = (uint64_t)v.streams[p] * (((v.mask >> p) & 1u) ? 2u : 4u);
        if (total - at < bytes) return -1;
        v.table_at[p] = (uint32_t)at; at += bytes;
    }
    for (uint32_t p = 0; p < v.P; ++p) {
        uint64_t bytes = v.n[p];
        if ((v.mask >> p) & 1u) {
            bytes = 0;
            for (uint32_t s = 0; s < v.streams[p]; ++s) {
                const uint32_t length = rd16(rec + v.table_at[p] + 2ull * s);
                if (length < 4) return -1;
                bytes += length;
            }
        }
        if (total - at < bytes) return -1;
        v.payload_at[p] = (uint32_t)at; at += bytes;
    }
    if (align_up(at, kPage) != total) return -1;
    for (; at < total; ++at) if (rec[at]) return -1;
    *b = v;
    return 0;
}

void wbp1_offsets(const Wbp1Plan &b, const uint8_t *rec, uint32_t *offsets) {
    uint32_t at = 0;
    for (uint32_t p = 0; p < b.P; ++p) {
        at = b.payload_at[p];
        for (uint32_t s = 0; s < b.streams[p]; ++s) {
            offsets[b.gbase[p] + s] = at;
            at += ((b.mask >> p) & 1u) ? rd16(rec + b.table_at[p] + 2ull * s) : std::min(b.chunk, b.n[p] - s * b.chunk);
        }
    }
    offsets[b.total_streams] = at;
}

void wbp1_tasks(const Wbp1Plan &b, uint32_t rec, std::vector<Wbp1Task> &tasks) {
    for (uint32_t p = 0; p < b.P; ++p)
        for (uint32_t f = 0; f < b.streams[p]; f += kWbp1Threads)
            tasks.push_back({rec, p, f, std::min<uint32_t>(kWbp1Threads, b.streams[p] - f)});
}

uint64_t wbp1_scratch(const Wbp1Plan &b, uint64_t plane_at[8]) {
    uint64_t at = 0;
    for (uint32_t p = 0; p < 8; ++p) {
        plane_at[p] = at;
        if (p < b.P) at = align_up(at + b.n[p], 16);
    }
    return std::max<uint64_t>(at, 16);
}

Wbp1Record wbp1_descriptor(const Wbp1Plan &b, const uint8_t *drec, const uint32_t *doffsets, uint8_t *dplanes, uint8_t *dout,
                           uint32_t *derror) {
    Wbp1Record r{};
    r.rec = drec; r.offsets = doffsets; r.planes = dplanes; r.out = dout; r.error = derror;
    r.decoded = b.decoded; r.P = b.P; r.chunk = b.chunk; r.mask = b.mask; r.transform = b.transform; r.owner = b.owner;
    r.ident3 = b.P | b.chunk_log2 << 8 | b.transform << 24;
    wbp1_scratch(b, r.plane_at);
    for (uint32_t p = 0; p < 8; ++p) {
        r.n[p] = b.n[p]; r.gbase[p] = b.gbase[p]; r.cdf_at[p] = b.cdf_at[p]; r.table_at[p] = b.table_at[p];
    }
    return r;
}

bool wbp1_prepare(int device) {
    if (device < 0 || device >= kMaxDevices) return false;
    std::lock_guard<std::mutex> lock(g_prep_mu);
    if (g_prepared[device]) return true;
    if (prepare_wbp1_kernels() != cudaSuccess) { (void)cudaGetLastError(); return false; }
    g_prepared[device] = true;
    return true;
}

int wbp1_encode(const uint8_t *data, uint32_t decoded, uint32_t P, uint32_t chunk_log2, uint32_t transform, uint32_t owner,
                uint8_t *out, size_t capacity, size_t *written) {
    if (!data || !out || !written || !decoded || decoded > kMaxDecoded || (P != 1 && P != 2 && P != 4 && P != 8) ||
        chunk_log2 < 10 || chunk_log2 > 15 || transform > 1 || (transform && (P == 1 || decoded % P))) return -1;
    const uint32_t chunk = 1u << chunk_log2;
    std::vector<uint8_t> coded;
    if (transform) {   // every little-endian element rotated left by one bit
        coded.assign(data, data + decoded);
        for (size_t i = 0; i + P <= decoded; i += P) {
            uint32_t carry = coded[i + P - 1] >> 7;
            for (uint32_t k = 0; k < P; ++k) {
                const uint32_t next = coded[i + k] >> 7;
                coded[i + k] = (uint8_t)(coded[i + k] << 1 | carry);
                carry = next;
            }
        }
        data = coded.data();
    }
    uint32_t ident[4] = {kWbp1Magic, owner, 0, P | chunk_log2 << 8 | transform << 24}, g = 0, mask = 0;
    uint32_t n[8] = {}, streams[8] = {};
    uint16_t cdf[8][257] = {};
    std::vector<uint8_t> enc[8], table[8], plane;
    std::vector<uint8_t> tmp(2 * chunk + 16);
    for (uint32_t p = 0; p < P; ++p) {
        n[p] = plane_bytes(decoded, P, p);
        streams[p] = (n[p] + chunk - 1) / chunk;
        if (!n[p]) continue;
        uint64_t counts[256] = {};
        plane.resize(n[p]);
        for (uint32_t i = 0; i < n[p]; ++i) counts[plane[i] = data[(size_t)i * P + p]]++;
        quantize(counts, cdf[p]);
        table[p].resize(4ull * streams[p]);
        for (uint32_t s = 0, first = 0; first < n[p]; first += chunk, ++s) {   // rANS, coded backwards
            const uint32_t count = std::min(chunk, n[p] - first);
            ident[2] = g + s;
            uint32_t x = kRansLHost + (h32(ident, plane.data() + first, count) & 0x7fffffu);
            uint8_t *const top = tmp.data() + tmp.size();
            uint8_t *cur = top;
            for (uint32_t j = count; j-- > 0;) {
                const uint32_t y = plane[first + j], start = cdf[p][y], freq = cdf[p][y + 1] - start;
                const uint32_t bound = ((kRansLHost >> kPrecHost) << 8) * freq;
                while (x >= bound) {
                    if (cur == tmp.data()) return -1;
                    *--cur = (uint8_t)x; x >>= 8;
                }
                x = (x / freq << kPrecHost) + x % freq + start;
            }
            for (int k = 0; k < 4; ++k) {
                if (cur == tmp.data()) return -1;
                *--cur = (uint8_t)x; x >>= 8;
            }
            const size_t len = (size_t)(top - cur);
            if (len > 65535) return -1;
            enc[p].insert(enc[p].end(), cur, top);
            table[p][2 * s] = (uint8_t)len; table[p][2 * s + 1] = (uint8_t)(len >> 8);
        }
        if (514u + 2ull * streams[p] + enc[p].size() < 4ull * streams[p] + n[p]) {
            mask |= 1u << p;
            table[p].resize(2ull * streams[p]);
        } else {   // raw: the plane bytes and one hash word per chunk
            for (uint32_t s = 0, first = 0; first < n[p]; first += chunk, ++s) {
                ident[2] = g + s;
                const uint32_t h = h32(ident, plane.data() + first, std::min(chunk, n[p] - first));
                for (int k = 0; k < 4; ++k) table[p][4 * s + k] = (uint8_t)(h >> (8 * k));
            }
            enc[p].assign(plane.begin(), plane.end());
        }
        g += streams[p];
    }
    size_t at = kHeader;
    for (uint32_t p = 0; p < P; ++p) at += (((mask >> p) & 1u) ? 514u : 0u) + table[p].size() + enc[p].size();
    const size_t padded = align_up(at, kPage);
    if (padded > capacity) return -1;
    std::memset(out, 0, padded);
    const uint32_t head[3] = {kWbp1Magic, owner, decoded};
    for (int i = 0; i < 12; ++i) out[i] = (uint8_t)(head[i / 4] >> (8 * (i % 4)));
    out[12] = (uint8_t)P; out[13] = (uint8_t)chunk_log2; out[14] = (uint8_t)mask; out[15] = (uint8_t)transform;
    at = kHeader;
    for (uint32_t p = 0; p < P; ++p)
        if ((mask >> p) & 1u)
            for (int s = 0; s <= 256; ++s) { out[at++] = (uint8_t)cdf[p][s]; out[at++] = (uint8_t)(cdf[p][s] >> 8); }
    for (uint32_t p = 0; p < P; ++p) { if (!table[p].empty()) std::memcpy(out + at, table[p].data(), table[p].size()); at += table[p].size(); }
    for (uint32_t p = 0; p < P; ++p) { if (!enc[p].empty()) std::memcpy(out + at, enc[p].data(), enc[p].size()); at += enc[p].size(); }
    *written = padded;
    return 0;
}

}  // namespace wexb
