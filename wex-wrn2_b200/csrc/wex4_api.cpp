// The WEX4 container ABI of include/wex4_tools.h.
//
// Host: the header page and the index are validated with the reference's rules, in the reference's
// order, so a refused file gets the same WEX4_E_* class (c/wex4.h:185-437; each check below names
// its rule). GPU: every record's stored bytes go up once; record SHA-256 checks, RAW padding checks,
// WNR3 decodes (the persistent launch of nr3_decode.cu), WBP1 and WNR4 decodes and the content digest
// run there.
#include <cuda_runtime.h>
#include <sys/mman.h>
#include <unistd.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "bufs.h"
#include "container.cuh"
#include "host_wait.h"
#include "nr3_host.h"
#include "sha256.cuh"
#include "wex4_index.h"
#include "wex4_tools.h"
#include "wbp1_host.h"
#include "wnr4_host.h"

#define WEXB_API extern "C" __attribute__((visibility("default")))

namespace wexb {
namespace {

enum { OK = 0, E_ARG = -1, E_MAGIC = -2, E_HASH = -3, E_VERSION = -4, E_FEATURE = -5, E_HEADER = -6, E_INDEX = -7,
       E_BLOB = -8, E_RECORD = -9, E_TENSOR = -10, E_NAME = -11, E_LAYOUT = -12, E_EXPERT = -13, E_DATA = -14,
       E_UNSUPPORTED = -15 };
constexpr uint32_t kMagic = 0x57455834u, kPage = 4096;
constexpr uint64_t kMaxBlobs = 1u << 16, kMaxRecords = 1u << 24, kMaxTensors = 1u << 24, kMaxIndex = 1ull << 28,
                   kMaxDecoded = 1u << 30;
constexpr uint32_t kCodecRaw = 0, kCodecWnr3 = 5, kCodecWbp1 = 6, kCodecWnr4 = 8, kRecValueExact = 1, kRecExpert = 2,
                   kBlobWnm2 = 1, kBlobWnm4 = 3;

uint64_t page_align(uint64_t n) { return (n + kPage - 1) & ~(uint64_t)(kPage - 1); }

// ---- host SHA-256 (FIPS 180-4) for the header page, the index and blobs -------------------------
struct HostSha {
    static uint32_t ror(uint32_t x, int r) { return (x >> r) | (x << (32 - r)); }
    uint32_t h[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a, 0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
    uint8_t buf[64];
    uint64_t n = 0;
    void block(const uint8_t *p) {
        static const uint32_t K[64] = {
            0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5,
            0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174,
            0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da,
            0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967,
            0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85,
            0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070,
            0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
            0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7, 0xc67178f2};
        uint32_t w[64], s[8];
        for (int i = 0; i < 16; ++i) w[i] = (uint32_t)p[4 * i] << 24 | (uint32_t)p[4 * i + 1] << 16 | (uint32_t)p[4 * i + 2] << 8 | p[4 * i + 3];
        for (int i = 16; i < 64; ++i)
            w[i] = w[i - 16] + (ror(w[i - 15], 7) ^ ror(w[i - 15], 18) ^ (w[i - 15] >> 3)) + w[i - 7] +
                   (ror(w[i - 2], 17) ^ ror(w[i - 2], 19) ^ (w[i - 2] >> 10));
        std::memcpy(s, h, sizeof s);
        for (int i = 0; i < 64; ++i) {
            const uint32_t t1 = s[7] + (ror(s[4], 6) ^ ror(s[4], 11) ^ ror(s[4], 25)) + ((s[4] & s[5]) ^ (~s[4] & s[6])) + K[i] + w[i];
            const uint32_t t2 = (ror(s[0], 2) ^ ror(s[0], 13) ^ ror(s[0], 22)) + ((s[0] & s[1]) ^ (s[0] & s[2]) ^ (s[1] & s[2]));
            s[7] = s[6]; s[6] = s[5]; s[5] = s[4]; s[4] = s[3] + t1; s[3] = s[2]; s[2] = s[1]; s[1] = s[0]; s[0] = t1 + t2;
        }
        for (int i = 0; i < 8; ++i) h[i] += s[i];
    }
    void update(const uint8_t *p, size_t len) {
        size_t fill = (size_t)(n & 63);
        n += len;
        if (fill) {
            const size_t take = std::min<size_t>(64 - fill, len);
            std::memcpy(buf + fill, p, take); p += take; len -= take;
            if (fill + take < 64) return;
            block(buf);
        }
        for (; len >= 64; p += 64, len -= 64) block(p);
        if (len) std::memcpy(buf, p, len);
    }
    void final(uint8_t out[32]) {
        const uint64_t bits = n * 8;
        uint8_t pad[72] = {0x80}, l[8];
        for (int i = 0; i < 8; ++i) l[i] = (uint8_t)(bits >> (56 - 8 * i));
        update(pad, ((119 - (n & 63)) & 63) + 1);
        update(l, 8);
        for (int i = 0; i < 32; ++i) out[i] = (uint8_t)(h[i / 4] >> (24 - 8 * (i % 4)));
    }
};
void sha256(const uint8_t *p, size_t n, uint8_t out[32]) { HostSha s; s.update(p, n); s.final(out); }

// ---- the index -------------------------------------------------------------------------------------
struct Header {
    uint32_t major, minor, blobs, records, tensors, layers, experts, max_decoded;
    uint64_t required, optional, file_bytes, index_offset, index_bytes, names_bytes, meta_bytes, total_decoded;
    uint8_t index_sha[32], root[32];
};
struct Blob { uint32_t kind, id; uint64_t offset, bytes; const uint8_t *sha; };
struct Record { uint64_t offset; uint32_t stored, decoded, codec, flags, blob, owner, first_tensor, tensor_count; const uint8_t *sha; };
struct Tensor { const uint8_t *name; uint32_t name_len, dtype, rank, record, record_count; uint64_t shape[8], offset, nbytes; };
struct View {
    Header h;
    const uint8_t *blobs, *records, *tensors, *order, *names, *meta;
    Blob blob(uint32_t i) const {
        const uint8_t *p = blobs + (size_t)i * 64;
        return {rd32(p), rd32(p + 4), rd64(p + 8), rd64(p + 16), p + 24};
    }
    Record record(uint32_t i) const {
        const uint8_t *p = records + (size_t)i * 72;
        return {rd64(p), rd32(p + 8), rd32(p + 12), rd16(p + 16), rd16(p + 18), rd32(p + 20), rd32(p + 24), rd32(p + 28),
                rd32(p + 32), p + 36};
    }
    Tensor tensor(uint32_t i) const {
        const uint8_t *p = tensors + (size_t)i * 96;
        Tensor t;
        t.name = names + rd32(p); t.name_len = rd16(p + 4); t.dtype = p[6]; t.rank = p[7];
        for (int d = 0; d < 8; ++d) t.shape[d] = rd64(p + 8 + 8 * d);
        t.record = rd32(p + 72); t.record_count = rd32(p + 76); t.offset = rd64(p + 80); t.nbytes = rd64(p + 88);
        return t;
    }
};

// bits per element of the safetensors dtype codes 1..22 (0: opaque bytes) (c/wex4.h:178-179)
const uint8_t kDtypeBits[23] = {0, 8, 8, 8, 8, 8, 8, 16, 16, 16, 16, 32, 32, 32, 64, 64, 64, 64, 4, 6, 6, 8, 8};

// the header page (c/wex4.h:185-215)
int parse_header(const uint8_t *page, uint64_t file_bytes, Header *h) {
    uint8_t digest[32];
    if (!page || !h) return E_ARG;
    if (rd32(page) != kMagic) return E_MAGIC;
    sha256(page, 4064, digest);
    if (std::memcmp(digest, page + 4064, 32)) return E_HASH;
    h->major = rd16(page + 4); h->minor = rd16(page + 6);
    if (h->major != 4) return E_VERSION;
    h->required = rd64(page + 8); h->optional = rd64(page + 16);
    if (h->required & ~1ull) return E_FEATURE;
    h->file_bytes = rd64(page + 24); h->index_offset = rd64(page + 32); h->index_bytes = rd64(page + 40);
    h->blobs = rd32(page + 48); h->records = rd32(page + 52); h->tensors = rd32(page + 56);
    h->layers = rd32(page + 60); h->experts = rd32(page + 64); h->max_decoded = rd32(page + 68);
    h->names_bytes = rd64(page + 72); h->meta_bytes = rd64(page + 80); h->total_decoded = rd64(page + 88);
    std::memcpy(h->index_sha, page + 96, 32); std::memcpy(h->root, digest, 32);
    if (h->file_bytes != file_bytes || file_bytes < kPage || (file_bytes & (kPage - 1)) || h->blobs > kMaxBlobs ||
        h->records > kMaxRecords || h->tensors > kMaxTensors || h->names_bytes > kMaxIndex || h->meta_bytes > kMaxIndex ||
        h->layers > 65536 || h->experts > 65536 || !h->layers != !h->experts ||
        (uint64_t)h->layers * h->experts > kMaxRecords || h->max_decoded > kMaxDecoded ||
        (!h->records && (h->max_decoded || h->total_decoded)))
        return E_HEADER;
    const uint64_t need = (uint64_t)h->blobs * 64 + (uint64_t)h->records * 72 + (uint64_t)h->tensors * 100 + h->names_bytes +
                          h->meta_bytes;
    if (need != h->index_bytes || need > kMaxIndex || h->index_offset < kPage || (h->index_offset & (kPage - 1)) ||
        h->index_offset > file_bytes || page_align(need) > file_bytes - h->index_offset ||
        (!need && h->index_offset != kPage))
        return E_HEADER;
    return OK;
}

// strict UTF-8 without NUL (c/wex4.h:238-260)
bool utf8_ok(const uint8_t *p, size_t n) {
    size_t i = 0;
    while (i < n) {
        const uint32_t c = p[i];
        uint32_t extra, cp;
        if (!c) return false;
        if (c < 0x80) { ++i; continue; }
        if (c >= 0xc2 && c <= 0xdf) { extra = 1; cp = c & 0x1f; }
        else if (c >= 0xe0 && c <= 0xef) { extra = 2; cp = c & 0x0f; }
        else if (c >= 0xf0 && c <= 0xf4) { extra = 3; cp = c & 0x07; }
        else return false;
        if (n - i <= extra) return false;
        for (uint32_t k = 1; k <= extra; ++k) {
            if ((p[i + k] & 0xc0) != 0x80) return false;
            cp = cp << 6 | (p[i + k] & 0x3f);
        }
        if ((extra == 2 && (cp < 0x800 || (cp >= 0xd800 && cp <= 0xdfff))) || (extra == 3 && (cp < 0x10000 || cp > 0x10ffff)))
            return false;
        i += extra + 1;
    }
    return true;
}

// The 72-byte legacy entry of an EXPERT record: 3 scale then 3 weight tensors (c/wex4.h:264-290).
int expert_entry(const View &v, uint32_t r, WexEntry *e) {
    if (r >= v.h.records) return E_ARG;
    const Record rec = v.record(r);
    if (!(rec.flags & kRecExpert) || rec.tensor_count != 6) return E_EXPERT;
    std::memset(e, 0, sizeof *e);
    e->file_offset = rec.offset; e->total_bytes = rec.stored; e->flags = rec.codec;
    for (uint32_t m = 0; m < 6; ++m) {
        const Tensor t = v.tensor(rec.first_tensor + m);
        if (t.rank != 2 || t.record_count != 1 || !t.shape[0] || !t.shape[1] || t.shape[0] > 65535 || t.shape[1] > 65535)
            return E_EXPERT;
        if (m < 3) {
            if (t.dtype != 2 && t.dtype != 6) return E_EXPERT;   // U8 or F8_E8M0
            e->scale_shapes[m][0] = (uint16_t)t.shape[0]; e->scale_shapes[m][1] = (uint16_t)t.shape[1];
            e->scale_offsets[m] = (uint32_t)t.offset; e->scale_bytes += (uint32_t)t.nbytes;
        } else {
            if (t.dtype != 2 && t.dtype != 3) return E_EXPERT;   // U8 or I8
            e->weight_shapes[m - 3][0] = (uint16_t)t.shape[0]; e->weight_shapes[m - 3][1] = (uint16_t)t.shape[1];
            e->weight_offsets[m - 3] = (uint32_t)t.offset; e->weight_bytes += (uint32_t)t.nbytes;
        }
    }
    uint64_t raw, aligned;
    if (entry_raw_sizes(e, &raw, &aligned) || raw != rec.decoded) return E_EXPERT;
    return OK;
}

// the whole index (c/wex4.h:294-437)
int open_index(const Header &h, const uint8_t *index, size_t index_len, View *v) {
    uint8_t digest[32];
    if (!v || (!index && h.index_bytes) || index_len != page_align(h.index_bytes)) return E_ARG;
    sha256(index, (size_t)h.index_bytes, digest);
    if (std::memcmp(digest, h.index_sha, 32)) return E_HASH;
    for (uint64_t i = h.index_bytes; i < index_len; ++i) if (index[i]) return E_INDEX;
    v->h = h;
    v->blobs = index;
    v->records = v->blobs + (size_t)h.blobs * 64;
    v->tensors = v->records + (size_t)h.records * 72;
    v->order = v->tensors + (size_t)h.tensors * 96;
    v->names = v->order + (size_t)h.tensors * 4;
    v->meta = v->names + (size_t)h.names_bytes;
    // tensors: the canonical name pool, dtype / shape / size
    uint64_t name_at = 0;
    for (uint32_t i = 0; i < h.tensors; ++i) {
        const uint8_t *p = v->tensors + (size_t)i * 96;
        if (rd32(p) != name_at || rd16(p + 4) > h.names_bytes - name_at) return E_NAME;
        const Tensor t = v->tensor(i);
        name_at += t.name_len;
        if (!utf8_ok(t.name, t.name_len)) return E_NAME;
        if (t.rank > 8) return E_TENSOR;
        uint64_t elements = 1;
        for (uint32_t d = 0; d < 8; ++d) {
            if (d >= t.rank) { if (t.shape[d]) return E_TENSOR; continue; }
            if (t.shape[d] && elements > UINT64_MAX / t.shape[d]) return E_TENSOR;
            elements *= t.shape[d];
        }
        const uint32_t bits = t.dtype < 23 ? kDtypeBits[t.dtype] : 0;
        if (bits && (elements > UINT64_MAX / 64 || t.nbytes > UINT64_MAX / 8 || elements * bits != t.nbytes * 8)) return E_TENSOR;
    }
    if (name_at != h.names_bytes) return E_NAME;
    // name order: strictly increasing names (a permutation, unique names)
    for (uint32_t i = 0; i < h.tensors; ++i) {
        const uint32_t at = rd32(v->order + (size_t)i * 4);
        if (at >= h.tensors) return E_NAME;
        if (i) {
            const Tensor prev = v->tensor(rd32(v->order + (size_t)(i - 1) * 4)), cur = v->tensor(at);
            const int c = std::memcmp(prev.name, cur.name, std::min(prev.name_len, cur.name_len));
            if (c > 0 || (!c && prev.name_len >= cur.name_len)) return E_NAME;
        }
    }
    // blobs
    for (uint32_t i = 0; i < h.blobs; ++i) {
        const Blob b = v->blob(i);
        if (!b.bytes || b.bytes > kMaxDecoded || rd64(b.sha + 32)) return E_BLOB;
        if (b.kind == kBlobWnm2 && (b.bytes != kModelBytes || !b.id)) return E_BLOB;
    }
    // records and the tensors that tile them
    uint64_t total = 0, pending_bytes = 0;
    uint32_t t = 0, pending = 0, maximum = 0;
    int64_t last_owner = -1;
    for (uint32_t r = 0; r < h.records; ++r) {
        const Record rec = v->record(r);
        uint64_t cursor = 0;
        if (!rec.stored || (rec.stored & (kPage - 1)) || !rec.decoded || rec.decoded > kMaxDecoded ||
            rec.stored > page_align(rec.decoded) || (rec.flags & ~(kRecValueExact | kRecExpert)) || rd32(rec.sha + 32) ||
            rec.blob > h.blobs) return E_RECORD;
        if (rec.codec == kCodecRaw ? (rec.stored != page_align(rec.decoded) || rec.blob) : rec.stored == page_align(rec.decoded))
            return E_RECORD;
        if (rec.codec == kCodecWbp1 &&
            (rec.blob || rec.flags || rec.stored < page_align(16 + 6ull * (((uint64_t)rec.decoded + 32767) >> 15))))
            return E_RECORD;
        if ((rec.flags & kRecValueExact) && (rec.codec != kCodecWnr3 || !(h.required & 1))) return E_RECORD;
        if (rec.codec == kCodecWnr3) {
            if (!(rec.flags & kRecExpert) || !rec.blob) return E_RECORD;
            if (v->blob(rec.blob - 1).kind != kBlobWnm2) return E_RECORD;
        }
        total += rec.decoded;
        if (rec.decoded > maximum) maximum = rec.decoded;
        if (pending) {   // continuation part of tensor t - 1
            if (rec.tensor_count || rec.first_tensor != t - 1 || (rec.flags & kRecExpert) || rec.owner != r ||
                rec.decoded > pending_bytes) return E_RECORD;
            pending_bytes -= rec.decoded;
            if (!--pending && pending_bytes) return E_RECORD;
            continue;
        }
        if (!rec.tensor_count || rec.first_tensor != t || rec.tensor_count > h.tensors - t) return E_RECORD;
        for (uint32_t k = 0; k < rec.tensor_count; ++k) {
            const Tensor ten = v->tensor(t + k);
            if (ten.record != r || !ten.nbytes) return E_TENSOR;
            if (ten.record_count == 1) {
                if (ten.offset != cursor || ten.nbytes > rec.decoded - cursor) return E_TENSOR;
                cursor += ten.nbytes;
            } else {
                if (ten.record_count < 2 || rec.tensor_count != 1 || ten.offset || (rec.flags & kRecExpert) ||
                    ten.record_count > h.records - r || ten.nbytes <= rec.decoded) return E_TENSOR;
                pending = ten.record_count - 1; pending_bytes = ten.nbytes - rec.decoded; cursor = rec.decoded;
            }
        }
        if (cursor != rec.decoded) return E_TENSOR;
        t += rec.tensor_count;
        if (rec.flags & kRecExpert) {
            WexEntry e;
            if (rec.codec != kCodecRaw && rec.codec != kCodecWnr3) return E_EXPERT;
            if ((rec.owner >> 16) >= h.layers || (rec.owner & 0xffff) >= h.experts || (int64_t)rec.owner <= last_owner ||
                expert_entry(*v, r, &e)) return E_EXPERT;
            last_owner = rec.owner;
            if (rec.codec == kCodecWnr3) {   // the smallest legal WNR3 record: longest chunks, 4-byte streams
                uint64_t streams = 0;
                for (int m = 0; m < 3; ++m)
                    streams += ((uint64_t)e.scale_shapes[m][0] * e.scale_shapes[m][1] + 16383) / 16384 +
                               ((uint64_t)e.weight_shapes[m][0] * e.weight_shapes[m][1] * 2 + 16383) / 16384;
                if (rec.stored < page_align(32 + streams * 6)) return E_EXPERT;
            }
        } else if (rec.owner != r) return E_RECORD;
    }
    if (pending || total != h.total_decoded || maximum != h.max_decoded) return E_RECORD;
    if (h.layers && last_owner < 0) return E_EXPERT;
    for (; t < h.tensors; ++t) {   // zero-size tensors close the table
        const Tensor ten = v->tensor(t);
        if (ten.nbytes || ten.record_count || ten.record || ten.offset) return E_TENSOR;
    }
    // header page, blobs, records and the index tile the file, in offset order
    uint64_t pos = kPage;
    uint32_t b = 0, r = 0;
    bool index_done = !h.index_bytes;
    for (;;) {
        uint64_t size;
        if (b < h.blobs && v->blob(b).offset == pos) { size = page_align(v->blob(b).bytes); ++b; }
        else if (r < h.records && v->record(r).offset == pos) { size = v->record(r).stored; ++r; }
        else if (!index_done && h.index_offset == pos) { size = index_len; index_done = true; }
        else break;
        if (size > h.file_bytes - pos) return E_LAYOUT;
        pos += size;
    }
    if (b != h.blobs || r != h.records || !index_done || pos != h.file_bytes) return E_LAYOUT;
    return OK;
}

int view_of(const uint8_t *page, uint64_t file_bytes, const uint8_t *index, size_t index_len, View *v) {
    Header h;
    const int st = parse_header(page, file_bytes, &h);
    return st ? st : open_index(h, index, index_len, v);
}

// ---- records on the GPU --------------------------------------------------------------------------
// One record to check and decode: its stored bytes in host memory and what to do with them.
struct Job {
    uint32_t r = 0;
    Record rec{};
    const uint8_t *stored = nullptr;
    const uint8_t *expect_sha = nullptr;   // non-null: verify the stored bytes' SHA-256
    int pre = OK;                          // a host verdict that precedes the GPU (WEX4_E_*)
    bool nr3 = false;
    Plan plan{};
    const uint8_t *tabs = nullptr;          // device tables of its WNM2 model
    bool w4 = false;                       // a codec-8 (WNR4 kind MX) expert slab
    W4Geo geo{};
    W4Tables w4tab{};
    uint64_t soff[3] = {}, woff[3] = {};   // its six tensors in the decoded record
    bool host_refused = false;             // its header or tile table failed the host checks
    bool bp = false;                       // a WBP1 (codec 6) record
    Wbp1Plan bpp{};
    uint8_t *out_dev = nullptr;            // decoded bytes on the device (after the run)
    int status = OK;
};

struct Space {   // the container layer's device workspace: one call at a time
    std::mutex mu;
    int device = -1;
    cudaStream_t st = nullptr, sh[1] = {};     // uploads and decodes; the record hashes
    std::vector<cudaEvent_t> landed;           // the metadata in place; the hashes done
    DevBuf stage, out, scratch, meta;
    PinBuf hmeta;
    // upload passes of a hashed check: gate[q] is set to the call's token after pass q (sha256.cuh)
    DevBuf gates;
    PinBuf htoken;
    uint32_t token = 0;
    bool unsettled = false;   // a bounded wait gave up: its work may still use the buffers and streams
    bool events(size_t n) {
        while (landed.size() < n) {
            cudaEvent_t e;
            if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return false;
            landed.push_back(e);
        }
        return true;
    }
};
// Record hashes: one serial chain per record (a single thread hashes a large record at tens of MB/s),
// so every record's chain must run at once with all the others, and start as early as it can. The
// records are uploaded in passes of kPassBytes of every record (pass q: bytes [q P, (q + 1) P) of each),
// each pass followed by its gate word; one hash launch over all records starts before the uploads and
// each chain waits only for the pass it is about to read. Every chain thus starts within the first pass
// (about 1 GB of a 10 GB check) instead of after its record's turn in a record-by-record upload, and
// the copies stay ahead of the chains (a record's share of the link is above a chain's speed).
constexpr int kShaStreams = 1;
constexpr uint32_t kPassShift = 21, kPassBytes = 1u << kPassShift;
Space g_space;

// Host verdicts of a WNR3 record before its decode (c/wex4.h:685-697): entry, model id, owner and
// value-exact flag cross-checks, then the record parse.
int prepare_wnr3(const View &v, Job &j, uint32_t model_id, int device) {
    WexEntry e;
    if (!model_id || expert_entry(v, j.r, &e)) return E_ARG;
    const Blob b = v.blob(j.rec.blob - 1);
    if (model_id != b.id || rd32(j.stored + 28) != j.rec.owner ||
        !(j.stored[27] & 8) != !(j.rec.flags & kRecValueExact)) return E_DATA;
    if (plan_record(&e, j.stored, &j.plan) || j.plan.model_id != model_id || !j.plan.nr3) return E_DATA;
    if (model_tables(model_id, device, &j.tabs)) return E_ARG;
    j.nr3 = true;
    return OK;
}

// Host verdicts of a codec-8 record (draft WNR4 kind MX, decoded on request): a non-EXPERT record
// holding the six tensors of an expert slab (scales [rows, cols] of U8 / F8_E8M0, then weights
// [rows, 16 cols] of U8 / I8), owning itself, with a kind-3 WNM4 blob whose FNV-1a id is the entry's.
// The record's own header, tile table, owner and model are checked when its tiles are planned.
int prepare_wnr4(const View &v, Job &j, const uint8_t *file, int device) {
    const Record &rec = j.rec;
    if (rec.flags || rec.tensor_count != 6 || !rec.blob) return E_UNSUPPORTED;
    const Blob b = v.blob(rec.blob - 1);
    if (b.kind != kBlobWnm4) return E_UNSUPPORTED;
    uint32_t geo[13] = {0};
    for (int m = 0; m < 3; ++m) {
        const Tensor s = v.tensor(rec.first_tensor + m), w = v.tensor(rec.first_tensor + 3 + m);
        if (s.rank != 2 || w.rank != 2 || (s.dtype != 2 && s.dtype != 6) || (w.dtype != 2 && w.dtype != 3) ||
            w.shape[0] != s.shape[0] || w.shape[1] != 16 * s.shape[1] || s.shape[0] > 65535 || s.shape[1] > 4095)
            return E_UNSUPPORTED;
        geo[1 + m] = (uint32_t)(s.shape[0] * s.shape[1]); geo[4 + m] = (uint32_t)s.shape[1];
        geo[7 + m] = (uint32_t)s.offset; geo[10 + m] = (uint32_t)w.offset;
        j.soff[m] = s.offset; j.woff[m] = w.offset;
        if (w.offset & 15) return E_UNSUPPORTED;   // 16-byte stores of packed weights
    }
    if (!wnr4_geo(geo, &j.geo)) return E_UNSUPPORTED;
    uint32_t id = 0;
    const int st = wnr4_tables(file + b.offset, (size_t)b.bytes, device, &j.w4tab, &id);
    if (st < 0 || id != b.id) return E_BLOB;
    if (st) return E_ARG;
    j.w4 = true;
    return OK;
}

// Host verdict of a WBP1 record before its decode (c/wex4.h:487-525, :684-685): the record header,
// planes, CDFs, stream tables and padding.
int prepare_wbp1(Job &j, int device) {
    if (wbp1_parse(j.stored, j.rec.stored, j.rec.decoded, j.rec.owner, &j.bpp)) return E_DATA;
    if (!wbp1_prepare(device)) return E_ARG;
    j.bp = true;
    return OK;
}

// Runs every job with pre == OK: upload, SHA-256 checks, RAW padding checks, WNR3 decodes into device
// memory. Sets job.status (E_HASH before E_DATA, as the reference orders them) and job.out_dev.
// Returns false on a CUDA failure. The caller holds g_space.mu.
bool run_jobs(std::vector<Job> &jobs, int device) {
    Space &S = g_space;
    if (cudaSetDevice(device) != cudaSuccess) { (void)cudaGetLastError(); return false; }
    if (S.unsettled) {   // reuse the workspace only once the work of the call that gave up has ended
        bool ended = cudaStreamQuery(S.st) == cudaSuccess;
        for (cudaStream_t h : S.sh) ended = ended && cudaStreamQuery(h) == cudaSuccess;
        (void)cudaGetLastError();
        if (!ended) return false;
        S.unsettled = false;
    }
    if (S.device != device) {
        if (S.st) {
            S.stage.release(); S.out.release(); S.scratch.release(); S.meta.release();
            cudaStreamDestroy(S.st);
            for (cudaStream_t h : S.sh) cudaStreamDestroy(h);
            for (cudaEvent_t e : S.landed) cudaEventDestroy(e);
            S.landed.clear();
        }
        bool made = cudaStreamCreateWithFlags(&S.st, cudaStreamNonBlocking) == cudaSuccess;
        for (int h = 0; made && h < kShaStreams; ++h) made = cudaStreamCreateWithFlags(&S.sh[h], cudaStreamNonBlocking) == cudaSuccess;
        if (!made) { (void)cudaGetLastError(); S.device = -1; return false; }   // streams made so far leak
        S.device = device;
    }
    std::vector<size_t> at(jobs.size()), scr(jobs.size()), offs(jobs.size());
    size_t stage_bytes = 0, out_bytes = 0, scr_bytes = 0, noffs = 0;
    std::vector<size_t> nr3_of, w4_of, bp_of;   // job index of each WNR3 / WNR4 / WBP1 descriptor
    std::vector<size_t> bp_scr(jobs.size()), bp_offs(jobs.size());
    std::vector<Wbp1Task> bptasks;
    for (size_t i = 0; i < jobs.size(); ++i) {
        Job &j = jobs[i];
        if (j.pre != OK) continue;
        at[i] = stage_bytes; stage_bytes += align_up(j.rec.stored + kRecordSlack, 256);
        if (j.nr3) {
            scr[i] = scr_bytes; scr_bytes += align_up(j.plan.scratch, 256);
            offs[i] = noffs; noffs += j.plan.streams() + 1;
            nr3_of.push_back(i);
            out_bytes += align_up(j.rec.decoded, 256);
        }
        if (j.w4) { w4_of.push_back(i); out_bytes += align_up(j.rec.decoded, 256); }
        if (j.bp) {
            uint64_t plane_at[8];
            bp_scr[i] = scr_bytes; scr_bytes += align_up(wbp1_scratch(j.bpp, plane_at), 256);
            bp_offs[i] = noffs; noffs += j.bpp.total_streams + 1;
            wbp1_tasks(j.bpp, (uint32_t)bp_of.size(), bptasks);
            bp_of.push_back(i);
            out_bytes += align_up(j.rec.decoded, 256);
        }
    }
    const size_t kb = bp_of.size();
    const size_t n = jobs.size(), k = nr3_of.size(), k4 = w4_of.size();
    // WNR3 records: one persistent launch per model, its records contiguous
    std::stable_sort(nr3_of.begin(), nr3_of.end(), [&](size_t a, size_t b) { return jobs[a].tabs < jobs[b].tabs; });
    std::vector<const Plan *> nr3_plans(k);
    std::vector<const uint8_t *> nr3_tabs(k);
    for (size_t q = 0; q < k; ++q) { nr3_plans[q] = &jobs[nr3_of[q]].plan; nr3_tabs[q] = jobs[nr3_of[q]].tabs; }
    LaunchSet launches;
    launches.plan(nr3_plans.data(), nr3_tabs.data(), (uint32_t)k, true);
    const int sms = k ? device_sms(device) : 1;
    if (!sms) return false;
    // codec-8 tiles, planned from the host bytes against the staged copies, grouped by model
    std::vector<W4Rec> w4info(k4);
    std::vector<W4Job> w4jobs;
    std::vector<std::pair<size_t, size_t>> w4runs;   // (first job, job count) per model
    std::vector<const W4Tables *> w4tabs;
    std::vector<int> w4bad(k4, 0);
    for (size_t q0 = 0; q0 < k4;) {
        const uint32_t id = jobs[w4_of[q0]].w4tab.id;
        std::vector<W4Job> by_m[3];
        size_t q = q0;
        for (; q < k4 && jobs[w4_of[q]].w4tab.id == id; ++q) {
            Job &j = jobs[w4_of[q]];
            std::vector<W4Job> mine[3];
            std::memset(&w4info[q], 0, sizeof(W4Rec));
            // tile addresses as offsets into the staging buffer until it has its final size
            if (!wnr4_plan(j.stored, j.rec.stored, j.geo, j.r, id, reinterpret_cast<const uint8_t *>(at[w4_of[q]]), (uint32_t)q,
                           &w4info[q], mine)) {
                w4bad[q] = 1;
                continue;
            }
            for (int m = 0; m < 3; ++m) by_m[m].insert(by_m[m].end(), mine[m].begin(), mine[m].end());
        }
        const std::vector<W4Job> order = wnr4_launch_order(by_m);
        w4runs.push_back({w4jobs.size(), order.size()});
        w4tabs.push_back(&jobs[w4_of[q0]].w4tab);
        w4jobs.insert(w4jobs.end(), order.begin(), order.end());
        q0 = q;
    }
    size_t m = 0;
    auto take = [&](size_t bytes) { size_t a = m; m = align_up(m + bytes, 256); return a; };
    const size_t o_recs = take(k * sizeof(Nr3Record)), o_items = take(launches.items * sizeof(Nr3Item)),
                 o_counters = take(launches.counter_words() * 4), o_jobs = take(k * sizeof(CommitJob)),
                 o_sha = take(n * sizeof(ShaMsg)), o_exp = take(n * 32), o_zero = take(n * sizeof(ZeroJob)),
                 o_err = take(n * 4), o_ver = take(n * 4), o_offs = take(noffs * 4),
                 o_w4rec = take(k4 * sizeof(W4Rec)), o_w4job = take(w4jobs.size() * sizeof(W4Job)),
                 o_bprec = take(kb * sizeof(Wbp1Record)), o_bptask = take(bptasks.size() * sizeof(Wbp1Task)),
                 o_gfail = take(4);
    if (!S.stage.grow(stage_bytes) || !S.out.grow(out_bytes) || !S.scratch.grow(scr_bytes) || !S.meta.grow(m) ||
        !S.hmeta.grow(m)) return false;
    uint8_t *hm = S.hmeta.p, *dm = S.meta.p;
    std::memset(hm, 0, m);
    ShaMsg *hsha = reinterpret_cast<ShaMsg *>(hm + o_sha);
    ZeroJob *hzero = reinterpret_cast<ZeroJob *>(hm + o_zero);
    uint32_t *derr = reinterpret_cast<uint32_t *>(dm + o_err), *dver = reinterpret_cast<uint32_t *>(dm + o_ver);
    uint32_t nsha = 0, nzero = 0;
    size_t out_at = 0;
    for (size_t i = 0; i < n; ++i) {
        Job &j = jobs[i];
        if (j.pre != OK) continue;
        uint8_t *stage = S.stage.p + at[i];
        if (j.expect_sha) {
            std::memcpy(hm + o_exp + 32 * i, j.expect_sha, 32);
            hsha[nsha++] = {stage, j.rec.stored, nullptr, dm + o_exp + 32 * i, dver + i, 0};
        }
        if (j.rec.codec == kCodecRaw) {
            hzero[nzero++] = {stage, j.rec.decoded, j.rec.stored, derr + i, 1u};
            j.out_dev = stage;   // a RAW record decodes to its own first `decoded` bytes
        }
    }
    for (size_t q = 0; q < k; ++q) {
        Job &j = jobs[nr3_of[q]];
        const size_t i = nr3_of[q];
        plan_offsets(j.plan, reinterpret_cast<uint32_t *>(hm + o_offs) + offs[i]);
        plan_descriptor(j.plan, S.stage.p + at[i], reinterpret_cast<const uint32_t *>(dm + o_offs) + offs[i],
                        S.scratch.p + scr[i], derr + i, reinterpret_cast<const CommitJob *>(dm + o_jobs) + q,
                        reinterpret_cast<Nr3Record *>(hm + o_recs) + q);
        j.out_dev = S.out.p + out_at; out_at += align_up(j.rec.decoded, 256);
        CommitJob &J = reinterpret_cast<CommitJob *>(hm + o_jobs)[q];
        for (int mm = 0; mm < 3; ++mm) {
            J.src[mm] = S.scratch.p + scr[i] + j.plan.soff[mm]; J.dst[mm] = j.out_dev + j.plan.soff[mm];
            J.bytes[mm] = j.plan.dst_bytes[mm];
            J.src[3 + mm] = S.scratch.p + scr[i] + j.plan.wout[mm];
            J.dst[3 + mm] = j.out_dev + j.plan.scale_bytes + (j.plan.wout[mm] - j.plan.weight_at);
            J.bytes[3 + mm] = j.plan.dst_bytes[3 + mm];
        }
    }
    launches.fill(nr3_plans.data(), true, sms, kScalesFirst, reinterpret_cast<Nr3Item *>(hm + o_items),
                  reinterpret_cast<uint32_t *>(hm + o_counters));
    for (W4Job &t : w4jobs)
        if (t.tile) t.tile = S.stage.p + reinterpret_cast<uintptr_t>(t.tile);
    for (size_t q = 0; q < k4; ++q) {
        Job &j = jobs[w4_of[q]];
        j.out_dev = S.out.p + out_at; out_at += align_up(j.rec.decoded, 256);
        if (w4bad[q]) { j.host_refused = true; continue; }
        for (int mm = 0; mm < 3; ++mm) { w4info[q].dst_s[mm] = j.out_dev + j.soff[mm]; w4info[q].dst_w[mm] = j.out_dev + j.woff[mm]; }
        w4info[q].error = derr + w4_of[q];
    }
    for (size_t q = 0; q < kb; ++q) {
        Job &j = jobs[bp_of[q]];
        const size_t i = bp_of[q];
        j.out_dev = S.out.p + out_at; out_at += align_up(j.rec.decoded, 256);
        wbp1_offsets(j.bpp, j.stored, reinterpret_cast<uint32_t *>(hm + o_offs) + bp_offs[i]);
        reinterpret_cast<Wbp1Record *>(hm + o_bprec)[q] =
            wbp1_descriptor(j.bpp, S.stage.p + at[i], reinterpret_cast<const uint32_t *>(dm + o_offs) + bp_offs[i],
                            S.scratch.p + bp_scr[i], j.out_dev, derr + i);
    }
    if (!bptasks.empty()) std::memcpy(hm + o_bptask, bptasks.data(), bptasks.size() * sizeof(Wbp1Task));
    if (k4) std::memcpy(hm + o_w4rec, w4info.data(), k4 * sizeof(W4Rec));
    if (!w4jobs.empty()) std::memcpy(hm + o_w4job, w4jobs.data(), w4jobs.size() * sizeof(W4Job));
    cudaStream_t st = S.st, sh = S.sh[0];
    bool ok = S.events(2) && cudaMemcpyAsync(dm, hm, m, cudaMemcpyHostToDevice, st) == cudaSuccess;
    if (nsha) {   // passes of every record, gated; the hash launch first (it waits for each pass)
        size_t passes = 0;
        for (size_t i = 0; i < n; ++i)
            if (jobs[i].pre == OK) passes = std::max<size_t>(passes, (jobs[i].rec.stored + kPassBytes - 1) / kPassBytes);
        const size_t gate_bytes = 4 * (passes + 1);   // the last word covers the padding blocks past the data
        if (ok && (gate_bytes > S.gates.cap || S.token == 0xffffffffu)) {   // new words: zero them first
            ok = S.gates.grow(gate_bytes) && S.htoken.grow(16) &&
                 cudaMemsetAsync(S.gates.p, 0, S.gates.cap, st) == cudaSuccess && wait_stream(st) == Waited::Done;
            S.token = 0;
            if (!ok) S.token = 0xffffffffu;
        }
        const uint32_t token = ++S.token;
        if (ok) *reinterpret_cast<uint32_t *>(S.htoken.p) = token;   // the previous check's copies have ended
        uint32_t *gates = reinterpret_cast<uint32_t *>(S.gates.p);
        ShaParts P{};
        P.part[0] = reinterpret_cast<const ShaMsg *>(dm + o_sha);
        P.end[0] = nsha;
        P.nparts = 1;
        P.gate = gates; P.gate_token = token; P.gate_shift = kPassShift;
        P.gate_fail = reinterpret_cast<uint32_t *>(dm + o_gfail);
        ok = ok && cudaEventRecord(S.landed[0], st) == cudaSuccess && cudaStreamWaitEvent(sh, S.landed[0], 0) == cudaSuccess &&
             launch_sha256_parts(P, sh) == cudaSuccess;
        const bool hashing = ok;   // from here on, every gate word must be set, whatever fails
        for (size_t q = 0; ok && q < passes; ++q) {
            const size_t from = q * kPassBytes;
            for (size_t i = 0; ok && i < n; ++i)
                if (jobs[i].pre == OK && jobs[i].rec.stored > from)
                    ok = cudaMemcpyAsync(S.stage.p + at[i] + from, jobs[i].stored + from,
                                         std::min<size_t>(kPassBytes, jobs[i].rec.stored - from), cudaMemcpyHostToDevice,
                                         st) == cudaSuccess;
            ok = ok && cudaMemcpyAsync(gates + q, S.htoken.p, 4, cudaMemcpyHostToDevice, st) == cudaSuccess;
        }
        ok = ok && cudaMemcpyAsync(gates + passes, S.htoken.p, 4, cudaMemcpyHostToDevice, st) == cudaSuccess;
        if (hashing && !ok) {   // an upload failed: open every gate, so the hash launch ends at once (its
            (void)cudaGetLastError();   // verdicts are then discarded with the call) instead of at its wait limit
            for (size_t q = 0; q <= passes; ++q)
                (void)cudaMemcpyAsync(gates + q, S.htoken.p, 4, cudaMemcpyHostToDevice, st);
            (void)cudaGetLastError();
        }
    } else {
        for (size_t i = 0; ok && i < n; ++i)
            if (jobs[i].pre == OK)
                ok = cudaMemcpyAsync(S.stage.p + at[i], jobs[i].stored, jobs[i].rec.stored, cudaMemcpyHostToDevice, st) == cudaSuccess;
    }
    for (uint32_t z = 0; ok && z < nzero; z += 65535)
        ok = launch_zero_check(reinterpret_cast<const ZeroJob *>(dm + o_zero) + z, std::min<uint32_t>(65535, nzero - z), st) == cudaSuccess;
    const Nr3Record *drecs = reinterpret_cast<const Nr3Record *>(dm + o_recs);
    ok = ok && launches.launch(drecs, reinterpret_cast<const Nr3Item *>(dm + o_items), reinterpret_cast<uint32_t *>(dm + o_counters),
                               sms, st, nsha != 0);   // beside the hash launch's CTAs
    ok = ok && launch_wbp1_streams(reinterpret_cast<const Wbp1Record *>(dm + o_bprec),
                                   reinterpret_cast<const Wbp1Task *>(dm + o_bptask), (uint32_t)bptasks.size(), st) == cudaSuccess &&
         launch_wbp1_join(reinterpret_cast<const Wbp1Record *>(dm + o_bprec), (uint32_t)kb, st) == cudaSuccess;
    for (size_t g = 0; ok && g < w4runs.size(); ++g)
        ok = launch_wnr4(*w4tabs[g], reinterpret_cast<const W4Job *>(dm + o_w4job) + w4runs[g].first,
                         (uint32_t)w4runs[g].second, reinterpret_cast<const W4Rec *>(dm + o_w4rec), st) == cudaSuccess;
    // the hashes rejoin the decode stream before the verdicts come back
    if (nsha)
        ok = ok && cudaEventRecord(S.landed[1], sh) == cudaSuccess && cudaStreamWaitEvent(st, S.landed[1], 0) == cudaSuccess;
    ok = ok &&
         cudaMemcpyAsync(hm + o_err, dm + o_err, 4 * n, cudaMemcpyDeviceToHost, st) == cudaSuccess &&
         cudaMemcpyAsync(hm + o_ver, dm + o_ver, 4 * n, cudaMemcpyDeviceToHost, st) == cudaSuccess &&
         cudaMemcpyAsync(hm + o_gfail, dm + o_gfail, 4, cudaMemcpyDeviceToHost, st) == cudaSuccess;
    // bounded waits, also after a failed step: whatever was queued must end before the space is reused
    Waited waited = wait_stream(st);
    for (cudaStream_t h : S.sh) {
        const Waited w = wait_stream(h);
        if (w != Waited::Done && waited == Waited::Done) waited = w;
    }
    if (waited == Waited::TimedOut) S.unsettled = true;
    if (!ok || waited != Waited::Done) { (void)cudaGetLastError(); return false; }
    if (*reinterpret_cast<const uint32_t *>(hm + o_gfail)) return false;   // a chain gave up waiting for its bytes
    const uint32_t *herr = reinterpret_cast<const uint32_t *>(hm + o_err), *hver = reinterpret_cast<const uint32_t *>(hm + o_ver);
    for (size_t i = 0; i < n; ++i) {
        Job &j = jobs[i];
        if (j.pre != OK) { j.status = j.pre; continue; }
        if (j.expect_sha && hver[i]) j.status = E_HASH;
        else if (j.host_refused) j.status = E_DATA;
        else if (herr[i]) { j.status = E_DATA; if (j.nr3) report_error_bits(herr[i]); }
        else j.status = OK;
    }
    return true;
}

int current_device() {
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess) { (void)cudaGetLastError(); return -1; }
    return d;
}

}  // namespace

// ---- the expert records of an index, for file readers (wex4_index.h) --------------------------------
int file_header(const uint8_t *page, uint64_t file_bytes, FileIndex *out) {
    Header h;
    if (!out) return E_ARG;
    const int st = parse_header(page, file_bytes, &h);
    if (st) return st;
    out->file_bytes = file_bytes; out->index_offset = h.index_offset; out->index_len = page_align(h.index_bytes);
    out->layers = h.layers; out->experts = h.experts;
    return OK;
}

int file_index(const uint8_t *page, const uint8_t *index, FileIndex *out) {
    View v;
    if (!out) return E_ARG;
    int st = view_of(page, out->file_bytes, index, (size_t)out->index_len, &v);
    if (st) return st;
    out->records.clear(); out->models.clear();
    for (uint32_t i = 0; i < v.h.blobs; ++i) {
        const Blob b = v.blob(i);
        if (b.kind != kBlobWnm2) continue;
        FileModel m{b.offset, b.bytes, b.id, {}};
        std::memcpy(m.sha, b.sha, 32);
        out->models.push_back(m);
    }
    for (uint32_t r = 0; r < v.h.records; ++r) {
        const Record rec = v.record(r);
        if (!(rec.flags & kRecExpert)) continue;
        FileExpert f{};
        if ((st = expert_entry(v, r, &f.entry)) != OK) return st;
        if (rec.codec != kCodecRaw && rec.codec != kCodecWnr3) return E_UNSUPPORTED;
        f.owner = rec.owner; f.codec = rec.codec; f.stored = rec.stored; f.value_exact = (rec.flags & kRecValueExact) != 0;
        f.model = rec.codec == kCodecWnr3 ? v.blob(rec.blob - 1).id : 0;
        std::memcpy(f.sha, rec.sha, 32);
        out->records.push_back(f);
    }
    return OK;
}

void host_sha256(const uint8_t *p, size_t n, uint8_t out[32]) { sha256(p, n, out); }

}  // namespace wexb

using namespace wexb;

WEXB_API uint32_t wex4_tools_abi(void) { return 1u; }

WEXB_API void wex4_sha256_bytes(const unsigned char *p, size_t n, unsigned char *out) { sha256(p, n, out); }

WEXB_API int wex4_validate(const unsigned char *page, uint64_t file_bytes, const unsigned char *index, size_t index_len) {
    View v;
    return view_of(page, file_bytes, index, index_len, &v);
}

WEXB_API int wex4_expert_table(const unsigned char *page, uint64_t file_bytes, const unsigned char *index,
                               size_t index_len, unsigned char *out) {
    View v;
    int st = view_of(page, file_bytes, index, index_len, &v);
    if (st || !out) return st ? st : E_ARG;
    std::memset(out, 0, (size_t)v.h.layers * v.h.experts * sizeof(WexEntry));
    for (uint32_t r = 0; r < v.h.records; ++r) {
        const Record rec = v.record(r);
        if (!(rec.flags & kRecExpert)) continue;
        WexEntry e;
        if ((st = expert_entry(v, r, &e)) != OK) return st;
        std::memcpy(out + ((size_t)(rec.owner >> 16) * v.h.experts + (rec.owner & 0xffff)) * sizeof e, &e, sizeof e);
    }
    return OK;
}

WEXB_API int wex4_decode_record_buf(const unsigned char *page, uint64_t file_bytes, const unsigned char *index,
                                    size_t index_len, uint32_t r, const unsigned char *stored, const unsigned char *blob,
                                    int check_sha, unsigned char *out) {
    View v;
    int st = view_of(page, file_bytes, index, index_len, &v);
    if (st) return st;
    if (r >= v.h.records) return E_ARG;
    const Record rec = v.record(r);
    uint32_t model_id = 0;
    if (rec.blob && blob) {
        const Blob b = v.blob(rec.blob - 1);
        if (b.kind == kBlobWnm2) {
            if (model_validate(blob, (size_t)b.bytes, &model_id) || model_id != b.id) return E_BLOB;
            if (model_register(blob, (size_t)b.bytes)) return E_ARG;
        }
    }
    if (!stored || !out) return E_ARG;
    const int device = current_device();
    if (device < 0) return E_ARG;
    std::vector<Job> jobs(1);
    Job &j = jobs[0];
    j.r = r; j.rec = rec; j.stored = stored;
    j.expect_sha = check_sha ? rec.sha : nullptr;
    // codec 8 and unknown codecs are unsupported, as in the reference
    if (rec.codec == kCodecWnr3) j.pre = prepare_wnr3(v, j, model_id, device);
    else if (rec.codec == kCodecWbp1) j.pre = prepare_wbp1(j, device);
    else if (rec.codec != kCodecRaw) j.pre = E_UNSUPPORTED;
    const int pre = j.pre;
    if (pre != OK && !j.expect_sha) return pre;
    if (pre != OK) { j.pre = OK; j.nr3 = false; j.w4 = false; j.bp = false; j.rec.codec = 0xffff; }   // its hash is still checked first
    std::lock_guard<std::mutex> lock(g_space.mu);
    if (!run_jobs(jobs, device)) return E_ARG;
    if (j.status == E_HASH) return E_HASH;
    if (pre != OK) return pre;
    if (j.status != OK) return j.status;
    if (cudaMemcpy(out, j.out_dev, rec.decoded, cudaMemcpyDeviceToHost) != cudaSuccess) { (void)cudaGetLastError(); return E_ARG; }
    return OK;
}

WEXB_API int wex4_check(const unsigned char *file, uint64_t len, int flags, unsigned char *digest) {
    View v;
    if (!file || len < kPage) return E_HEADER;
    Header h;
    int st = parse_header(file, len, &h);
    if (st) return st;
    if ((st = open_index(h, file + h.index_offset, (size_t)page_align(h.index_bytes), &v)) != OK) return st;
    std::vector<uint32_t> model_ids(h.blobs ? h.blobs : 1, 0);
    for (uint32_t i = 0; i < h.blobs; ++i) {   // blobs (wex4/wex4_tools.c:82-97)
        const Blob b = v.blob(i);
        if (flags & WEX4_CHECK_HASHES) {
            uint8_t d[32];
            sha256(file + b.offset, (size_t)b.bytes, d);
            if (std::memcmp(d, b.sha, 32)) return E_HASH;
            for (uint64_t a = b.bytes; a < page_align(b.bytes); ++a) if (file[b.offset + a]) return E_BLOB;
        }
        if (b.kind == kBlobWnm2) {
            uint32_t id = 0;
            if (model_validate(file + b.offset, (size_t)b.bytes, &id) || id != b.id) return E_BLOB;
            if (model_register(file + b.offset, (size_t)b.bytes)) return E_ARG;
            model_ids[i] = id;
        }
    }
    if (!(flags & (WEX4_CHECK_HASHES | WEX4_CHECK_DECODE))) return OK;
    const int device = current_device();
    if (device < 0) return E_ARG;
    std::vector<Job> jobs(h.records);
    for (uint32_t r = 0; r < h.records; ++r) {
        Job &j = jobs[r];
        j.r = r; j.rec = v.record(r); j.stored = file + j.rec.offset;
        j.expect_sha = (flags & WEX4_CHECK_HASHES) ? j.rec.sha : nullptr;
        if (!(flags & WEX4_CHECK_DECODE)) {   // hashes only: RAW-like upload, nothing decoded
            j.rec.codec = kCodecRaw; j.rec.decoded = j.rec.stored;
            continue;
        }
        if (j.rec.codec == kCodecWnr3) j.pre = prepare_wnr3(v, j, j.rec.blob ? model_ids[j.rec.blob - 1] : 0, device);
        else if (j.rec.codec == kCodecWnr4 && (flags & WEX4_CHECK_CODEC8)) j.pre = prepare_wnr4(v, j, file, device);
        else if (j.rec.codec == kCodecWbp1) j.pre = prepare_wbp1(j, device);
        else if (j.rec.codec != kCodecRaw) j.pre = E_UNSUPPORTED;
    }
    std::lock_guard<std::mutex> lock(g_space.mu);
    // a record refused on the host still has its hash checked first: run its SHA on the GPU too
    std::vector<int> pre(h.records);
    for (uint32_t r = 0; r < h.records; ++r) {
        pre[r] = jobs[r].pre;
        if (jobs[r].pre != OK && jobs[r].expect_sha) {
            jobs[r].pre = OK; jobs[r].nr3 = false; jobs[r].w4 = false; jobs[r].bp = false; jobs[r].rec.codec = 0xffff;
        }
    }
    if (!run_jobs(jobs, device)) return E_ARG;
    for (uint32_t r = 0; r < h.records; ++r) {   // the first failing record, in record order
        const Job &j = jobs[r];
        if (j.status == E_HASH) return E_HASH;
        if (pre[r] != OK) return pre[r];
        if (j.status != OK) return j.status;
    }
    if (!(flags & WEX4_CHECK_DECODE) || (flags & WEX4_CHECK_NO_DIGEST)) return OK;
    // the content digest: per tensor in table order {u16 name_len, name, u8 dtype, u8 rank, u64 shape[8],
    // u64 nbytes, bytes} (wex4/wex4_tools.c:125-158), hashed on the GPU by one thread over the segments
    std::vector<uint8_t> metas;
    struct Seg { bool host; size_t at; const uint8_t *dev; uint64_t bytes; };
    std::vector<Seg> segs;
    auto meta = [&](const Tensor &t, uint64_t nbytes) {
        const size_t a = metas.size();
        metas.push_back((uint8_t)t.name_len); metas.push_back((uint8_t)(t.name_len >> 8));
        metas.insert(metas.end(), t.name, t.name + t.name_len);
        metas.push_back((uint8_t)t.dtype); metas.push_back((uint8_t)t.rank);
        for (int d = 0; d < 8; ++d) for (int b = 0; b < 8; ++b) metas.push_back((uint8_t)(t.shape[d] >> (8 * b)));
        for (int b = 0; b < 8; ++b) metas.push_back((uint8_t)(nbytes >> (8 * b)));
        segs.push_back({true, a, nullptr, metas.size() - a});
    };
    for (uint32_t r = 0; r < h.records; ++r) {
        const Job &j = jobs[r];
        if (!j.rec.tensor_count) segs.push_back({false, 0, j.out_dev, j.rec.decoded});
        for (uint32_t q = 0; q < j.rec.tensor_count; ++q) {
            const Tensor t = v.tensor(j.rec.first_tensor + q);
            meta(t, t.nbytes);
            segs.push_back({false, 0, j.out_dev + t.offset, t.record_count == 1 ? t.nbytes : j.rec.decoded});
        }
    }
    uint32_t first_empty = h.tensors;
    while (first_empty && !v.tensor(first_empty - 1).nbytes) --first_empty;
    for (uint32_t i = first_empty; i < h.tensors; ++i) meta(v.tensor(i), 0);
    DevBuf dmeta, dsegs;
    std::vector<ShaMsg> msgs(segs.size());
    bool ok = dmeta.grow(metas.size() + 32) && dsegs.grow(msgs.size() * sizeof(ShaMsg) + 256);
    for (size_t i = 0; ok && i < segs.size(); ++i)
        msgs[i] = {segs[i].host ? dmeta.p + 32 + segs[i].at : segs[i].dev, segs[i].bytes, nullptr, nullptr, nullptr, 0};
    ok = ok && cudaMemcpy(dmeta.p + 32, metas.data(), metas.size(), cudaMemcpyHostToDevice) == cudaSuccess &&
         cudaMemcpy(dsegs.p, msgs.data(), msgs.size() * sizeof(ShaMsg), cudaMemcpyHostToDevice) == cudaSuccess &&
         launch_sha256_segments(reinterpret_cast<const ShaMsg *>(dsegs.p), (uint32_t)msgs.size(), dmeta.p, g_space.st) == cudaSuccess;
    const Waited waited = wait_stream(g_space.st);
    if (waited == Waited::TimedOut) { g_space.unsettled = true; return E_ARG; }   // dmeta / dsegs stay allocated
    ok = ok && waited == Waited::Done;
    uint8_t dg[32];
    ok = ok && cudaMemcpy(dg, dmeta.p, 32, cudaMemcpyDeviceToHost) == cudaSuccess;
    dmeta.release(); dsegs.release();
    if (!ok) { (void)cudaGetLastError(); return E_ARG; }
    if (digest) std::memcpy(digest, dg, 32);
    return OK;
}

WEXB_API int wex4_bp_encode_record(const unsigned char *data, uint32_t decoded, uint32_t planes, uint32_t chunk_log2,
                                   uint32_t transform, uint32_t owner, unsigned char *out, size_t capacity, size_t *written) {
    return wbp1_encode(data, decoded, planes, chunk_log2, transform, owner, out, capacity, written);
}

WEXB_API int wex4_bp_decode_record(const unsigned char *record, size_t total, uint32_t decoded, uint32_t owner,
                                   unsigned char *out) {
    if (!record || !out) return -1;
    const int device = current_device();
    if (device < 0) return -1;
    std::vector<Job> jobs(1);
    Job &j = jobs[0];
    j.rec.codec = kCodecWbp1; j.rec.stored = (uint32_t)total; j.rec.decoded = decoded; j.rec.owner = owner;
    j.stored = record;
    if (total > 0xffffffffull || prepare_wbp1(j, device) != OK) return -1;
    std::lock_guard<std::mutex> lock(g_space.mu);
    if (!run_jobs(jobs, device) || j.status != OK) return -1;
    if (cudaMemcpy(out, j.out_dev, decoded, cudaMemcpyDeviceToHost) != cudaSuccess) { (void)cudaGetLastError(); return -1; }
    return 0;
}
// The same check as wex4_check on a copy of the file that ends right before an inaccessible page, so
// that any host read past the end of the file faults instead of passing silently (the reference's
// guard-paged check, wex4/wex4_tools.c:36-59, :170-178). The decoded bytes live in device memory here,
// where host guard pages do not apply: a kernel never reads past a record's stored bytes by design
// (every stream read is bounded by its offsets, the record lengths checked on the host first).
WEXB_API int wex4_fuzz_check(const unsigned char *file, uint64_t len, int flags, unsigned char *digest) {
    if (!file && len) return E_ARG;
    const long ps = sysconf(_SC_PAGESIZE);
    const size_t page = ps > 0 ? (size_t)ps : 4096;
    if (len > (uint64_t)SIZE_MAX - 2 * page) return E_ARG;
    const size_t body = ((size_t)len + page - 1) / page * page;
    void *base = mmap(nullptr, body + page, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
    if (base == MAP_FAILED) return E_ARG;
    uint8_t *const guard = static_cast<uint8_t *>(base) + body;
    if (mprotect(guard, page, PROT_NONE) != 0) { munmap(base, body + page); return E_ARG; }
    uint8_t *copy = guard - len;
    if (len) std::memcpy(copy, file, (size_t)len);
    const int st = wex4_check(copy, len, flags, digest);
    munmap(base, body + page);
    return st;
}
WEXB_API int wex4_fuzz_run(const unsigned char *, uint64_t, uint64_t, uint32_t, int, uint64_t *) { return E_UNSUPPORTED; }
WEXB_API int wex4_store_probe(const char *, const unsigned char *, unsigned char *, uint64_t, uint32_t *) { return E_UNSUPPORTED; }
