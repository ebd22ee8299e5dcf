/* ORACLE — test infrastructure only (see oracle.h). CPU restatement of the WNR2/WNR3 record
 * decode (reference c/wex_neural_rans.h, c/wex_format.h) and of SHA-256 (c/wex4.h:49-151).
 * Written for clarity, not speed: one symbol at a time, binary CDF search, like the reference. */
#include "oracle.h"
#include <stdlib.h>
#include <string.h>

#define RANS_L (1u << 23)          /* c/wex_neural_rans.h:20 */
#define PREC 14u                   /* :146 */
#define CONTEXTS 567u              /* :148 */
#define MODEL_BYTES (32u + 3u * CONTEXTS * 34u + 3u * 514u)   /* :153 = 59408 */
#define MAGIC_WNR2 0x32524e57u     /* :144 */
#define MAGIC_WNR3 0x33524e57u     /* :190 */
#define MAGIC_WNM2 0x324d4e57u     /* :145 */

static uint32_t rd32(const uint8_t *p) { return p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24; }
static uint32_t rd16(const uint8_t *p) { return p[0] | (uint32_t)p[1] << 8; }
static uint32_t rotl(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }

/* ---- MurmurHash3_x86_32 (Appleby's public algorithm), streaming form ----------------------- */
typedef struct { uint32_t h, len, carry, nc; } Mm3;
static uint32_t mm3_mix(uint32_t k) { k *= 0xcc9e2d51u; k = rotl(k, 15); return k * 0x1b873593u; }
static void mm3_word(Mm3 *s, uint32_t k) { s->h = rotl(s->h ^ mm3_mix(k), 13) * 5u + 0xe6546b64u; }
static void mm3_bytes(Mm3 *s, const uint8_t *p, size_t n) {
    for (size_t i = 0; i < n; i++) {
        s->carry |= (uint32_t)p[i] << (8u * s->nc);
        if (++s->nc == 4u) { mm3_word(s, s->carry); s->carry = 0; s->nc = 0; }
    }
    s->len += (uint32_t)n;
}
static uint32_t mm3_final(Mm3 *s) {
    uint32_t h = s->h;
    if (s->nc) h ^= mm3_mix(s->carry);
    h ^= s->len;
    h ^= h >> 16; h *= 0x85ebca6bu; h ^= h >> 13; h *= 0xc2b2ae35u; h ^= h >> 16;
    return h;
}
uint32_t oracle_murmur3(const uint8_t *p, size_t n, uint32_t seed) {
    Mm3 s = {seed, 0, 0, 0};
    mm3_bytes(&s, p, n);
    return mm3_final(&s);
}
/* c/wex_neural_rans.h:225-233: the ident words then the stream's decoded bytes, seed "WNR3". */
uint32_t oracle_nr3_x0(const uint32_t ident[4], const uint8_t *data, uint32_t n) {
    uint8_t head[16];
    for (int i = 0; i < 16; i++) head[i] = (uint8_t)(ident[i / 4] >> (8 * (i % 4)));
    Mm3 s = {MAGIC_WNR3, 0, 0, 0};
    mm3_bytes(&s, head, 16);
    mm3_bytes(&s, data, n);
    return RANS_L + (mm3_final(&s) & 0x7fffffu);
}

uint32_t oracle_fnv1a(const uint8_t *p, size_t n) {   /* c/wex_neural_rans.h:235-240 */
    uint32_t h = 2166136261u;
    for (size_t i = 0; i < n; i++) h = (h ^ p[i]) * 16777619u;
    return h ? h : 1u;
}

/* c/wex_neural_rans.h:399-405: lower member of the densest adjacent pair of values, first wins. */
uint8_t oracle_anchor(const uint8_t *scales, uint32_t n) {
    uint32_t hist[256] = {0}, best = 0, top = 0;
    for (uint32_t i = 0; i < n; i++) hist[scales[i]]++;
    for (uint32_t v = 0; v + 1 < 256; v++)
        if (hist[v] + hist[v + 1] > top) { top = hist[v] + hist[v + 1]; best = v; }
    return (uint8_t)best;
}

/* A CDF of `symbols` entries (+1): starts at 0, ends at 2^14, strictly increasing (:249-255). */
static int cdf_ok(const uint8_t *cdf, uint32_t symbols) {
    if (rd16(cdf) != 0 || rd16(cdf + 2 * symbols) != (1u << PREC)) return 0;
    for (uint32_t s = 0; s < symbols; s++) if (rd16(cdf + 2 * s) >= rd16(cdf + 2 * s + 2)) return 0;
    return 1;
}
/* c/wex_neural_rans.h:258-274 */
int oracle_wnm2_open(const uint8_t *blob, size_t bytes, uint32_t *id) {
    static const uint32_t head[8] = {MAGIC_WNM2, 1u, PREC, CONTEXTS, 3u, 0, 0, 0};
    if (!blob || bytes != MODEL_BYTES) return -1;
    for (int i = 0; i < 8; i++) if (rd32(blob + 4 * i) != head[i]) return -1;
    for (uint32_t r = 0; r < 3u * CONTEXTS; r++) if (!cdf_ok(blob + 32 + 34u * r, 16)) return -1;
    for (uint32_t m = 0; m < 3u; m++) if (!cdf_ok(blob + 32 + 3u * CONTEXTS * 34u + 514u * m, 256)) return -1;
    if (id) *id = oracle_fnv1a(blob, bytes);
    return 0;
}

/* ---- one rANS stream (c/wex_neural_rans.h:356-380) ------------------------------------------- */
typedef struct { const uint8_t *p, *end; uint32_t x; } Stream;
static int stream_open(Stream *s, const uint8_t *begin, uint32_t length) {
    if (length < 4) return -1;
    s->x = (uint32_t)begin[0] << 24 | (uint32_t)begin[1] << 16 | (uint32_t)begin[2] << 8 | begin[3];
    s->p = begin + 4; s->end = begin + length;
    return s->x >= RANS_L && s->x < (RANS_L << 8) ? 0 : -1;
}
/* Largest symbol s with cdf[s] <= slot, then the state step and byte renormalisation. */
static int stream_symbol(Stream *s, const uint8_t *cdf, uint32_t symbols, uint32_t *out) {
    uint32_t slot = s->x & ((1u << PREC) - 1u), lo = 0, hi = symbols;
    while (hi - lo > 1) { uint32_t mid = (lo + hi) / 2; if (rd16(cdf + 2 * mid) <= slot) lo = mid; else hi = mid; }
    uint32_t start = rd16(cdf + 2 * lo), freq = rd16(cdf + 2 * lo + 2) - start;
    s->x = freq * (s->x >> PREC) + slot - start;
    while (s->x < RANS_L) {
        if (s->p == s->end) return -1;
        s->x = (s->x << 8) | *s->p++;
    }
    *out = lo;
    return 0;
}

/* ---- legacy 72-byte entry (c/wex_format.h:57-67, raw sizes :130-159) ---------------------------- */
typedef struct {
    uint32_t total, scale_bytes, weight_bytes, codec;
    uint32_t srows[3], scols[3], wrows[3], wcols[3], soff[3], woff[3];
} Entry;
static int entry_read(const uint8_t *e, Entry *v, uint64_t *raw) {
    uint64_t scales = 0, weights = 0;
    v->total = rd32(e + 8); v->scale_bytes = rd32(e + 12); v->weight_bytes = rd32(e + 16); v->codec = rd32(e + 68);
    for (int m = 0; m < 3; m++) {
        v->srows[m] = rd16(e + 20 + 4 * m); v->scols[m] = rd16(e + 22 + 4 * m);
        v->wrows[m] = rd16(e + 32 + 4 * m); v->wcols[m] = rd16(e + 34 + 4 * m);
        v->soff[m] = rd32(e + 44 + 4 * m); v->woff[m] = rd32(e + 56 + 4 * m);
    }
    for (int m = 0; m < 3; m++) {
        if (!v->srows[m] || !v->scols[m] || !v->wrows[m] || !v->wcols[m] || v->srows[m] != v->wrows[m] ||
            v->scols[m] * 16u != v->wcols[m] || v->soff[m] != scales) return -1;
        scales += (uint64_t)v->srows[m] * v->scols[m];
    }
    if (scales != v->scale_bytes) return -1;
    for (int m = 0; m < 3; m++) {
        if (v->woff[m] != scales + weights) return -1;
        weights += (uint64_t)v->wrows[m] * v->wcols[m];
    }
    if (weights != v->weight_bytes || scales + weights > 0xffffffffull) return -1;
    *raw = scales + weights;
    return ((*raw + 4095) & ~4095ull) > 0xffffffffull ? -1 : 0;
}

/* WNR2/WNR3 record decode: parse (c/wex_neural_rans.h:287-337), streams (:468-519), ceil inverse
 * (:446-461), scratch-then-copy (c/wex_format.h:530-556). */
int oracle_nrx_decode(const uint8_t *blob, const uint8_t *entry, const uint8_t *rec, uint8_t *out, int *where) {
    Entry e;
    uint64_t raw;
    uint32_t model_id = 0, scount[3], wcount[3];
    int dummy;
    if (!where) where = &dummy;
    *where = 1;
    if (!blob || !entry || !rec || !out || entry_read(entry, &e, &raw)) return -1;
    if (e.codec != 4 && e.codec != 5) return -1;
    if ((uint64_t)e.total >= ((raw + 4095) & ~4095ull)) return -1;   /* a coded record is smaller than raw */
    *where = 6;
    if (oracle_wnm2_open(blob, MODEL_BYTES, &model_id)) return -1;
    *where = 1;
    const int nr3 = e.codec == 5;
    const uint32_t magic = nr3 ? MAGIC_WNR3 : MAGIC_WNR2, total = e.total;
    if (total < 32 || (total & 4095u) || rd32(rec) != magic) return -1;
    const uint32_t flags = rec[27];
    if (nr3 ? (flags & ~0x0fu) != 0 : (flags != 0 || rd32(rec + 28) != 0)) return -1;
    const uint32_t rid = rd32(rec + 4), sp = rd32(rec + 8), wp = rd32(rec + 12), wchunk = rd32(rec + 16),
                   schunk = rd32(rec + 20), owner = rd32(rec + 28), word24 = rd32(rec + 24);
    if (!rid) return -1;
    if (rid != model_id) { *where = 6; return -1; }
#define POW2_IN(v, lo) ((v) >= (lo) && (v) <= 16384u && !((v) & ((v) - 1u)))
    if (!POW2_IN(wchunk, 512u) || !POW2_IN(schunk, 256u)) return -1;
    uint32_t sstreams = 0, wstreams = 0;
    for (int m = 0; m < 3; m++) {
        scount[m] = e.srows[m] * e.scols[m];
        wcount[m] = e.wrows[m] * e.wcols[m] * 2u;
        if (!scount[m] || !wcount[m] || wcount[m] % 32u || (uint64_t)scount[m] * 32u != wcount[m]) return -1;
        sstreams += (scount[m] + schunk - 1) / schunk;
        wstreams += (wcount[m] + wchunk - 1) / wchunk;
    }
    const uint64_t meta = 32u + 2ull * (sstreams + wstreams), used = meta + sp + wp;
    if (used > total || ((used + 4095) & ~4095ull) != total) return -1;
    const uint8_t *lengths = rec + 32;
    uint64_t sum = 0;
    for (uint32_t g = 0; g < sstreams + wstreams; g++) {
        uint32_t n = rd16(lengths + 2 * g);
        if (n < 4) return -1;
        sum += n;
        if (g + 1 == sstreams) { if (sum != sp) return -1; sum = 0; }
    }
    if (sum != wp) return -1;
    for (uint64_t i = used; i < total; i++) if (rec[i]) return -1;   /* canonical zero padding */

    uint8_t *slab = (uint8_t *)malloc((size_t)raw);
    if (!slab) return -1;
    const uint8_t *scdf_base = blob + 32 + 3u * CONTEXTS * 34u, *wcdf_base = blob + 32;
    const uint8_t *payload = rec + meta;
    const int cz = nr3 && (flags & 0x08u);
    uint32_t ident[4] = {rid, owner, 0, word24}, g = 0, sym;
    int status = -1;
    Stream s;
    /* scale streams, matrix by matrix */
    for (int m = 0; m < 3; m++) {
        uint8_t *so = slab + e.soff[m];
        for (uint32_t first = 0; first < scount[m]; first += schunk, g++) {
            uint32_t count = scount[m] - first < schunk ? scount[m] - first : schunk, len = rd16(lengths + 2 * g);
            *where = 2;
            if (stream_open(&s, payload, len)) goto done;
            for (uint32_t j = 0; j < count; j++) {
                if (stream_symbol(&s, scdf_base + 514u * m, 256, &sym)) goto done;
                so[first + j] = (uint8_t)sym;
            }
            if (s.p != s.end) goto done;
            ident[2] = g;
            if (s.x != (nr3 ? oracle_nr3_x0(ident, so + first, count) : RANS_L)) { *where = nr3 ? 3 : 2; goto done; }
            payload += len;
        }
    }
    /* weight streams: context = (srel * 9 + previous magnitude) * 9 + running maximum */
    payload = rec + meta + sp;
    for (int m = 0; m < 3; m++) {
        const uint8_t *so = slab + e.soff[m], anchor = rec[24 + m];
        uint8_t *wo = slab + e.woff[m];
        for (uint32_t first = 0; first < wcount[m]; first += wchunk, g++) {
            uint32_t count = wcount[m] - first < wchunk ? wcount[m] - first : wchunk, len = rd16(lengths + 2 * g);
            uint32_t srel = 0, prev = 8, maxm = 8;
            *where = 2;
            if (stream_open(&s, payload, len)) goto done;
            for (uint32_t j = 0; j < count; j++) {
                uint32_t i = first + j;
                if (i % 32u == 0) {
                    int d = (int)so[i / 32u] - (int)anchor;
                    srel = (uint32_t)((d < -3 ? -3 : d > 3 ? 3 : d) + 3);
                    prev = 8; maxm = 8;
                }
                if (stream_symbol(&s, wcdf_base + 34u * (m * CONTEXTS + (srel * 9 + prev) * 9 + maxm), 16, &sym)) goto done;
                if (cz && sym == 8) { *where = 4; goto done; }
                if (i & 1u) wo[i / 2] |= (uint8_t)(sym << 4); else wo[i / 2] = (uint8_t)sym;
                prev = sym & 7u;
                if (maxm == 8 || prev > maxm) maxm = prev;
            }
            if (s.p != s.end) goto done;
            ident[2] = g;
            if (s.x != (nr3 ? oracle_nr3_x0(ident, wo + first / 2, count / 2) : RANS_L)) { *where = nr3 ? 3 : 2; goto done; }
            payload += len;
        }
    }
    /* ceil form inverse: in a flagged matrix every block whose coded maximum magnitude is 5 maps
     * magnitudes a -> a + min(a, 2) and its scale drops by one (scale 0 there is an error) */
    if (nr3) {
        for (int m = 0; m < 3; m++) {
            if (!((flags >> m) & 1u)) continue;
            uint8_t *so = slab + e.soff[m], *wo = slab + e.woff[m];
            for (uint32_t b = 0; b < scount[m]; b++) {
                uint8_t *q = wo + 16u * b;
                uint32_t top = 0;
                for (int k = 0; k < 32; k++) { uint32_t a = (q[k / 2] >> (4 * (k & 1))) & 7u; if (a > top) top = a; }
                if (top != 5) continue;
                if (!so[b]) { *where = 5; goto done; }
                for (int k = 0; k < 16; k++) {
                    uint32_t lo = q[k] & 7u, hi = (q[k] >> 4) & 7u;
                    lo += lo < 2 ? lo : 2; hi += hi < 2 ? hi : 2;
                    q[k] = (uint8_t)((q[k] & 0x88u) | lo | hi << 4);
                }
                so[b]--;
            }
        }
    }
    memcpy(out, slab, (size_t)raw);
    *where = 0;
    status = 0;
done:
    free(slab);
    return status;
}

/* ---- SHA-256, FIPS 180-4 ------------------------------------------------------------------- */
static const uint32_t SHA_K[64] = {
    0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5,
    0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174,
    0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da,
    0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967,
    0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85,
    0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070,
    0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
    0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7, 0xc67178f2};
static uint32_t ror(uint32_t x, int r) { return (x >> r) | (x << (32 - r)); }
static void sha_compress(uint32_t st[8], const uint8_t *blk) {
    uint32_t w[64], a[8];
    for (int i = 0; i < 16; i++)
        w[i] = (uint32_t)blk[4 * i] << 24 | (uint32_t)blk[4 * i + 1] << 16 | (uint32_t)blk[4 * i + 2] << 8 | blk[4 * i + 3];
    for (int i = 16; i < 64; i++) {
        uint32_t s0 = ror(w[i - 15], 7) ^ ror(w[i - 15], 18) ^ (w[i - 15] >> 3);
        uint32_t s1 = ror(w[i - 2], 17) ^ ror(w[i - 2], 19) ^ (w[i - 2] >> 10);
        w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    memcpy(a, st, sizeof a);
    for (int i = 0; i < 64; i++) {
        uint32_t t1 = a[7] + (ror(a[4], 6) ^ ror(a[4], 11) ^ ror(a[4], 25)) + ((a[4] & a[5]) ^ (~a[4] & a[6])) + SHA_K[i] + w[i];
        uint32_t t2 = (ror(a[0], 2) ^ ror(a[0], 13) ^ ror(a[0], 22)) + ((a[0] & a[1]) ^ (a[0] & a[2]) ^ (a[1] & a[2]));
        memmove(a + 1, a, 7 * sizeof(uint32_t));
        a[4] += t1;
        a[0] = t1 + t2;
    }
    for (int i = 0; i < 8; i++) st[i] += a[i];
}
void oracle_sha256(const uint8_t *p, size_t n, uint8_t out[32]) {
    uint32_t st[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a, 0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
    uint8_t tail[128] = {0};
    size_t full = n / 64, rest = n % 64, pad;
    for (size_t b = 0; b < full; b++) sha_compress(st, p + 64 * b);
    memcpy(tail, p + 64 * full, rest);
    tail[rest] = 0x80;
    pad = rest < 56 ? 64 : 128;
    for (int i = 0; i < 8; i++) tail[pad - 1 - i] = (uint8_t)(((uint64_t)n * 8u) >> (8 * i));
    sha_compress(st, tail);
    if (pad == 128) sha_compress(st, tail + 64);
    for (int i = 0; i < 32; i++) out[i] = (uint8_t)(st[i / 4] >> (24 - 8 * (i % 4)));
}
