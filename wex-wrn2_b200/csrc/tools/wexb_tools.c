/* wexb_tools: the writer side of the WNR3 codec, host C, no CUDA. It makes the inputs the GPU
 * decoder consumes: seeded synthetic MXFP4 experts, the WNR3 coded domain (canonical zero, ceil
 * form), WNM2 model training, and the WNR3/WNR2 record encoder. The byte layout it writes is the
 * reference's (c/wex_neural_rans.h:123-189, encoder :615-749); its output is compared byte for
 * byte with the reference encoder in tests/. Thread-safe: no globals, caller-owned buffers.
 *
 * Expert slab layout (the legacy 72-byte entry, c/wex_format.h:57-67): scales of w1, w2, w3, then
 * the packed E2M1 nibbles of w1, w2, w3 (even element in the low nibble). */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define EXPORT __attribute__((visibility("default")))
#define RANS_L (1u << 23)
#define PREC 14u
#define TOTAL (1u << PREC)
#define CONTEXTS 567u
#define MODEL_BYTES (32u + 3u * CONTEXTS * 34u + 3u * 514u)
#define MAGIC_WNR2 0x32524e57u
#define MAGIC_WNR3 0x33524e57u
#define MAGIC_WNM2 0x324d4e57u
#define MAX_CHUNK 16384u

static uint32_t rd32(const uint8_t *p) { return p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24; }
static uint32_t rd16(const uint8_t *p) { return p[0] | (uint32_t)p[1] << 8; }
static void wr32(uint8_t *p, uint32_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); p[2] = (uint8_t)(v >> 16); p[3] = (uint8_t)(v >> 24); }
static void wr16(uint8_t *p, uint32_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); }
static uint32_t rotl(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }

EXPORT uint32_t wexb_tools_abi(void) { return 1u; }
EXPORT uint32_t wexb_model_bytes(void) { return MODEL_BYTES; }

/* ---- deterministic generator: splitmix64 + Box-Muller ---------------------------------------- */
typedef struct { uint64_t s; int have; double spare; } Rng;
static uint64_t rng_u64(Rng *r) {
    uint64_t z = (r->s += 0x9e3779b97f4a7c15ull);
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}
static double rng_unit(Rng *r) { return ((rng_u64(r) >> 11) + 0.5) * (1.0 / 9007199254740992.0); }
/* Standard normal by inverse CDF: quantiles of 65536 equal-probability buckets (bisection on erfc,
 * built once), linear inside a bucket; the two outermost buckets draw an exact Box-Muller tail. */
#define QBUCKETS 65536
static double g_quantile[QBUCKETS + 1];   /* [1 .. QBUCKETS - 1] used */
static pthread_once_t g_quantile_once = PTHREAD_ONCE_INIT;
static void quantile_init(void) {
    for (int i = 1; i < QBUCKETS; i++) {
        double p = (double)i / QBUCKETS, lo = -10, hi = 10;
        for (int it = 0; it < 80; it++) {
            double mid = 0.5 * (lo + hi);
            if (0.5 * erfc(-mid / 1.4142135623730951) < p) lo = mid; else hi = mid;
        }
        g_quantile[i] = 0.5 * (lo + hi);
    }
}
static double rng_normal(Rng *r) {
    const uint32_t u = (uint32_t)(rng_u64(r) >> 32), i = u >> 16;
    if (i == 0 || i == QBUCKETS - 1) {   /* tails beyond the first / last quantile: Marsaglia's tail method */
        const double a = g_quantile[QBUCKETS - 1];
        double x, y;
        do { x = -log(rng_unit(r)) / a; y = -log(rng_unit(r)); } while (2.0 * y < x * x);
        return i ? a + x : -(a + x);
    }
    const double f = (u & 0xffffu) * (1.0 / 65536.0);
    return g_quantile[i] + f * (g_quantile[i + 1] - g_quantile[i]);
}

/* OCP MXFP4 of one 32-element block: E8M0 exponent floor(log2(amax)) - 2 (amax 0: -127), E2M1
 * magnitudes {0, .5, 1, 1.5, 2, 3, 4, 6} rounded to nearest with ties to the even code, the sign
 * bit only on non-zero codes (the rule of the reference's c/tools/make_qwen38_tiny_mxfp4.py:44-64). */
static uint8_t e2m1_code(double mag) {   /* midpoints; a tie goes to the even code */
    return (uint8_t)((mag > 0.25) + (mag >= 0.75) + (mag > 1.25) + (mag >= 1.75) + (mag > 2.5) + (mag >= 3.5) +
                     (mag > 5.0));
}
static uint8_t quantize_block(const double *g, uint8_t nib[32]) {
    double amax = 0;
    for (int i = 0; i < 32; i++) amax = fmax(amax, fabs(g[i]));
    int e = -127;
    if (amax > 0) e = ilogb(amax) - 2;   /* floor(log2 amax) - 2, exact */
    if (e < -127) e = -127;
    if (e > 127) e = 127;
    const double inv = ldexp(1.0, -e);   /* a power of two: the products below are exact */
    for (int i = 0; i < 32; i++) {
        double x = g[i] * inv, mag = fmin(fabs(x), 6.0);
        uint8_t c = e2m1_code(mag);
        nib[i] = (x < 0 && c) ? (uint8_t)(c | 8u) : c;
    }
    return (uint8_t)(e + 127);
}

/* One matrix of rows x cols FP4 elements (cols a multiple of 32): packed[rows * cols / 2] and
 * scales[rows * cols / 32]. mode 0: N(0, sigma) quantized; mode 1: uniform random nibbles and
 * scales in 118..126 (incompressible); mode 2: mode 0 with every WNR3 block case mixed in (a quarter
 * of the blocks "even": maximum magnitude 7 and no magnitude 1 or 3, some of them at scale 254 or
 * 255; blocks of maximum 0..4; all-zero blocks with random signs), like the reference's test fill
 * (c/tests/test_wex_format.c:694-730); mode 3: mode 2 plus one block of maximum 5, which keeps the
 * ceil form off for the matrix. neg_zero: the fraction of zero nibbles written as -0 (0x8). */
EXPORT int wexb_synth_matrix(uint64_t seed, uint32_t rows, uint32_t cols, double sigma, int mode, double neg_zero,
                             uint8_t *packed, uint8_t *scales) {
    if (!rows || !cols || cols % 32u || !packed || !scales) return -1;
    pthread_once(&g_quantile_once, quantile_init);
    Rng r = {seed * 0x9e3779b97f4a7c15ull + 0x632be59bd9b4e019ull, 0, 0};
    double g[32];
    uint8_t nib[32];
    const uint32_t blocks = cols / 32u;
    const uint64_t nz = neg_zero > 0 ? (uint64_t)(neg_zero * 9007199254740992.0) : 0;   /* of 2^53 */
    for (uint64_t b = 0; b < (uint64_t)rows * blocks; b++) {
        if (mode == 1) {
            uint64_t bits = rng_u64(&r), more = rng_u64(&r);
            for (int i = 0; i < 16; i++) nib[i] = (uint8_t)((bits >> (4 * i)) & 15u);
            for (int i = 0; i < 16; i++) nib[16 + i] = (uint8_t)((more >> (4 * i)) & 15u);
            scales[b] = (uint8_t)(118u + rng_u64(&r) % 9u);
        } else {
            for (int i = 0; i < 32; i++) g[i] = sigma * rng_normal(&r);
            scales[b] = quantize_block(g, nib);
            if (mode >= 2) {
                static const uint8_t even[6] = {0, 2, 4, 5, 6, 7};
                const uint32_t pick = (uint32_t)(rng_u64(&r) % 16u);
                if (pick < 4) {            /* even block, maximum 7 */
                    for (int i = 0; i < 32; i++) nib[i] = even[rng_u64(&r) % 6u];
                    nib[rng_u64(&r) % 32u] = 7;
                    if (pick == 0) scales[b] = (uint8_t)(254u + rng_u64(&r) % 2u);
                } else if (pick == 4) {    /* maximum 0..4 */
                    const uint32_t top = (uint32_t)(rng_u64(&r) % 5u);
                    for (int i = 0; i < 32; i++) nib[i] = (uint8_t)(rng_u64(&r) % (top + 1u));
                } else if (pick == 5) {    /* all zero, random signs */
                    for (int i = 0; i < 32; i++) nib[i] = (uint8_t)((rng_u64(&r) & 1u) << 3);
                }
                if (pick < 5)
                    for (int i = 0; i < 32; i++) if (nib[i] && (rng_u64(&r) & 1u)) nib[i] |= 8u;
                if (mode == 3 && b == 0) { for (int i = 0; i < 32; i++) nib[i] &= 0xbu; nib[5] = 5; }
            }
            if (nz)
                for (int i = 0; i < 32; i++)
                    if (nib[i] == 0 && (rng_u64(&r) >> 11) < nz) nib[i] = 8;
        }
        for (int i = 0; i < 16; i++) packed[b * 16 + i] = (uint8_t)(nib[2 * i] | nib[2 * i + 1] << 4);
    }
    return 0;
}

/* ---- expert views (the caller's 72-byte entry) ------------------------------------------------- */
typedef struct { uint32_t scount[3], wcount[3], soff[3], woff[3], scale_bytes, weight_bytes; uint64_t raw; } View;
static int view_of(const uint8_t *e, View *v) {
    uint64_t s = 0, w = 0;
    if (!e) return -1;
    v->scale_bytes = rd32(e + 12); v->weight_bytes = rd32(e + 16);
    for (int m = 0; m < 3; m++) {
        uint32_t sr = rd16(e + 20 + 4 * m), sc = rd16(e + 22 + 4 * m), wr = rd16(e + 32 + 4 * m), wc = rd16(e + 34 + 4 * m);
        v->soff[m] = rd32(e + 44 + 4 * m); v->woff[m] = rd32(e + 56 + 4 * m);
        if (!sr || !sc || sr != wr || sc * 16u != wc || v->soff[m] != s) return -1;
        v->scount[m] = sr * sc; v->wcount[m] = wr * wc * 2u;
        s += v->scount[m];
    }
    if (s != v->scale_bytes) return -1;
    for (int m = 0; m < 3; m++) { if (v->woff[m] != s + w) return -1; w += v->wcount[m] / 2u; }
    if (w != v->weight_bytes) return -1;
    v->raw = s + w;
    return 0;
}

/* c/wex_neural_rans.h:399-405 (rule g) and :526-534 (lower median, WNR2) */
static uint8_t anchor_g(const uint8_t *s, uint32_t n) {
    uint32_t h[256] = {0}, best = 0, top = 0;
    for (uint32_t i = 0; i < n; i++) h[s[i]]++;
    for (uint32_t v = 0; v < 255; v++) if (h[v] + h[v + 1] > top) { top = h[v] + h[v + 1]; best = v; }
    return (uint8_t)best;
}
static uint8_t lower_median(const uint8_t *s, uint32_t n) {
    uint32_t h[256] = {0}, seen = 0;
    for (uint32_t i = 0; i < n; i++) h[s[i]]++;
    for (uint32_t v = 0; v < 256; v++) { seen += h[v]; if (seen * 2u >= n) return (uint8_t)v; }
    return 255;
}
static uint32_t block_max(const uint8_t *q, int *odd) {
    uint32_t top = 0, o = 0;
    for (int k = 0; k < 32; k++) {
        uint32_t a = (q[k / 2] >> (4 * (k & 1))) & 7u;
        if (a > top) top = a;
        o |= a == 1 || a == 3;
    }
    if (odd) *odd = (int)o;
    return top;
}

/* Coded domain (c/wex_neural_rans.h:407-442): coded = source, then -0 -> +0 (cz), then the ceil
 * form on every matrix with no block of maximum 5: blocks of maximum 7 with only even magnitudes
 * (0, 2, 4, 5, 6, 7) and scale < 255 are halved to 0..5 and their scale raised by one. Returns the
 * record flags (ceil mask | 8 for cz) or -1. */
EXPORT int wexb_nr3_prepare(const uint8_t *entry, const uint8_t *source, int cz, uint8_t *coded) {
    static const uint8_t halve[8] = {0, 0, 1, 0, 2, 3, 4, 5};
    View v;
    if (!coded || !source || view_of(entry, &v)) return -1;
    memmove(coded, source, (size_t)v.raw);
    if (cz)
        for (uint64_t i = v.scale_bytes; i < v.raw; i++) {
            if ((coded[i] & 15u) == 8u) coded[i] &= 0xf0u;
            if ((coded[i] >> 4) == 8u) coded[i] &= 0x0fu;
        }
    uint32_t mask = 0;
    for (int m = 0; m < 3; m++) {
        uint8_t *s = coded + v.soff[m], *w = coded + v.woff[m];
        uint32_t fives = 0;
        for (uint32_t b = 0; b < v.scount[m]; b++) fives += block_max(w + 16u * b, NULL) == 5u;
        if (fives) continue;
        mask |= 1u << m;
        for (uint32_t b = 0; b < v.scount[m]; b++) {
            uint8_t *q = w + 16u * b;
            int odd;
            if (block_max(q, &odd) != 7u || odd || s[b] == 255u) continue;
            for (int k = 0; k < 16; k++)
                q[k] = (uint8_t)((q[k] & 0x88u) | halve[q[k] & 7u] | halve[(q[k] >> 4) & 7u] << 4);
            s[b]++;
        }
    }
    return (int)(mask | (cz ? 8u : 0u));
}

/* Training counts of one coded expert (c/wex_neural_rans.h:579-613): weights wc[3][567][16], scales
 * sc[3][256], contexts relative to the rule-g anchors (nr3 = 1) or lower medians (nr3 = 0). */
EXPORT int wexb_count_expert(const uint8_t *entry, const uint8_t *coded, int nr3, uint64_t *wc, uint64_t *sc) {
    View v;
    if (!coded || !wc || !sc || view_of(entry, &v)) return -1;
    for (int m = 0; m < 3; m++) {
        const uint8_t *s = coded + v.soff[m], *w = coded + v.woff[m];
        uint8_t a = nr3 ? anchor_g(s, v.scount[m]) : lower_median(s, v.scount[m]);
        uint32_t srel = 0, prev = 8, top = 8;
        for (uint32_t i = 0; i < v.scount[m]; i++) sc[256u * m + s[i]]++;
        for (uint32_t i = 0; i < v.wcount[m]; i++) {
            uint32_t x = (w[i / 2] >> (4 * (i & 1))) & 15u;
            if (i % 32u == 0) {
                int d = (int)s[i / 32] - (int)a;
                srel = (uint32_t)((d < -3 ? -3 : d > 3 ? 3 : d) + 3);
                prev = 8; top = 8;
            }
            wc[((size_t)m * CONTEXTS + (srel * 9 + prev) * 9 + top) * 16u + x]++;
            prev = x & 7u;
            if (top == 8 || prev > top) top = prev;
        }
    }
    return 0;
}

/* Counts -> 14-bit CDF, every symbol at least 1, the spare in proportion, the remainder one each
 * to the largest fractional parts, lower symbol first on ties (c/wex_neural_rans.h:536-562). */
static void quantize(const uint64_t *counts, uint32_t n, uint8_t *cdf) {
    uint64_t total = 0, rem[256];
    uint32_t freq[256], used = 0, spare = TOTAL - n;
    uint8_t taken[256] = {0};
    for (uint32_t s = 0; s < n; s++) total += counts[s];
    for (uint32_t s = 0; s < n; s++) {
        uint64_t scaled = total ? counts[s] * spare : spare, div = total ? total : n;
        freq[s] = 1u + (uint32_t)(scaled / div);
        rem[s] = scaled % div;
        used += freq[s];
    }
    for (uint32_t extra = TOTAL - used; extra; extra--) {
        uint32_t best = n;
        for (uint32_t s = 0; s < n; s++)
            if (!taken[s] && (best == n || rem[s] > rem[best])) best = s;
        taken[best] = 1; freq[best]++;
    }
    uint32_t at = 0;
    for (uint32_t s = 0; s <= n; s++) { wr16(cdf + 2 * s, at); if (s < n) at += freq[s]; }
}
static uint32_t fnv1a(const uint8_t *p, size_t n) {
    uint32_t h = 2166136261u;
    for (size_t i = 0; i < n; i++) h = (h ^ p[i]) * 16777619u;
    return h ? h : 1u;
}
/* WNM2 blob (c/wex_neural_rans.h:564-575); returns its id (FNV-1a), 0 on bad arguments. */
EXPORT uint32_t wexb_build_model(const uint64_t *wc, const uint64_t *sc, uint8_t *blob) {
    static const uint32_t head[8] = {MAGIC_WNM2, 1u, PREC, CONTEXTS, 3u, 0, 0, 0};
    if (!wc || !sc || !blob) return 0;
    for (int i = 0; i < 8; i++) wr32(blob + 4 * i, head[i]);
    for (uint32_t r = 0; r < 3u * CONTEXTS; r++) quantize(wc + 16u * r, 16, blob + 32 + 34u * r);
    for (uint32_t m = 0; m < 3u; m++) quantize(sc + 256u * m, 256, blob + 32 + 3u * CONTEXTS * 34u + 514u * m);
    return fnv1a(blob, MODEL_BYTES);
}

/* ---- MurmurHash3 of a stream's ident words + decoded bytes -> its initial (= final) state ------ */
static uint32_t mm3_mix(uint32_t k) { k *= 0xcc9e2d51u; k = rotl(k, 15); return k * 0x1b873593u; }
static uint32_t stream_x0(const uint32_t ident[4], const uint8_t *p, uint32_t n) {
    uint32_t h = MAGIC_WNR3, i;
    for (i = 0; i < 4; i++) h = rotl(h ^ mm3_mix(ident[i]), 13) * 5u + 0xe6546b64u;
    for (i = 0; i + 4 <= n; i += 4) h = rotl(h ^ mm3_mix(rd32(p + i)), 13) * 5u + 0xe6546b64u;
    if (n & 3u) {
        uint32_t k = 0;
        for (uint32_t t = n & 3u; t-- > 0;) k = k << 8 | p[i + t];
        h ^= mm3_mix(k);
    }
    h ^= 16u + n;
    h ^= h >> 16; h *= 0x85ebca6bu; h ^= h >> 13; h *= 0xc2b2ae35u; h ^= h >> 16;
    return RANS_L + (h & 0x7fffffu);
}

/* rANS encoder of one stream: symbols coded last to first, bytes written downwards from `top`,
 * then the state as 4 big-endian bytes. Returns the stream length or 0 on overflow. */
typedef struct { uint32_t x; uint8_t *p, *floor; } Enc;
static int enc_put(Enc *e, uint32_t start, uint32_t freq) {
    const uint32_t bound = ((RANS_L >> PREC) << 8) * freq;
    while (e->x >= bound) {
        if (e->p == e->floor) return -1;
        *--e->p = (uint8_t)e->x;
        e->x >>= 8;
    }
    e->x = (e->x / freq << PREC) + e->x % freq + start;
    return 0;
}
static int enc_flush(Enc *e) {
    for (int b = 0; b < 4; b++) {
        if (e->p == e->floor) return -1;
        *--e->p = (uint8_t)e->x;
        e->x >>= 8;
    }
    return 0;
}

/* Encode a coded expert as a WNR3 record (magic WNR3: rule-g anchors, flags and owner in bytes
 * 24..31, each stream starting at L + h23) or a WNR2 record (nr3 = 0: lower medians, flags and
 * owner 0, streams starting at L), with the chunk pair wchunk:schunk, into out (cap bytes,
 * zero-padded to 4096). Returns 0, 1 when the record is not smaller than the 4096-aligned raw slab
 * (the writer then stores the expert RAW), -1 on error. */
EXPORT int wexb_encode_record(const uint8_t *blob, const uint8_t *entry, const uint8_t *coded, int nr3, uint32_t flags,
                              uint32_t owner, uint32_t wchunk, uint32_t schunk, uint8_t *out, size_t cap,
                              size_t *used, size_t *total) {
    View v;
    if (!blob || !coded || !out || !used || !total || view_of(entry, &v) || rd32(blob) != MAGIC_WNM2) return -1;
    if (wchunk < 512 || wchunk > MAX_CHUNK || (wchunk & (wchunk - 1)) || schunk < 256 || schunk > MAX_CHUNK ||
        (schunk & (schunk - 1)) || (flags & ~0x0fu) || (!nr3 && (flags || owner))) return -1;
    const uint32_t model_id = fnv1a(blob, MODEL_BYTES);
    uint8_t anchor[3];
    uint32_t sstreams = 0, streams = 0;
    for (int m = 0; m < 3; m++) {
        const uint8_t *s = coded + v.soff[m];
        anchor[m] = nr3 ? anchor_g(s, v.scount[m]) : lower_median(s, v.scount[m]);
        if ((flags & 8u))
            for (uint32_t i = 0; i < v.wcount[m] / 2; i++) {
                uint8_t b = coded[v.woff[m] + i];
                if ((b & 15u) == 8u || (b >> 4) == 8u) return -1;   /* a CZ record carries no -0 */
            }
        sstreams += (v.scount[m] + schunk - 1) / schunk;
        streams += (v.wcount[m] + wchunk - 1) / wchunk;
    }
    streams += sstreams;
    const size_t meta = 32u + 2u * (size_t)streams;
    if (cap < meta) return -1;
    const uint32_t word24 = anchor[0] | (uint32_t)anchor[1] << 8 | (uint32_t)anchor[2] << 16 | flags << 24;
    uint32_t ident[4] = {model_id, owner, 0, word24}, g = 0;
    uint64_t sbytes = 0, wbytes = 0;
    size_t cursor = meta;
    uint8_t *tmp = (uint8_t *)malloc(2u * MAX_CHUNK + 16u);
    uint16_t *ctx = (uint16_t *)malloc(sizeof(uint16_t) * MAX_CHUNK);
    int status = -1;
    if (!tmp || !ctx) goto done;
    for (int pass = 0; pass < 6; pass++) {
        const int m = pass % 3, scale_pass = pass < 3;
        const uint8_t *s = coded + v.soff[m], *w = coded + v.woff[m];
        const uint32_t count_all = scale_pass ? v.scount[m] : v.wcount[m], chunk = scale_pass ? schunk : wchunk;
        const uint8_t *scdf = blob + 32 + 3u * CONTEXTS * 34u + 514u * m;
        const uint8_t *wcdf = blob + 32 + 34u * CONTEXTS * m;
        for (uint32_t first = 0; first < count_all; first += chunk, g++) {
            const uint32_t count = count_all - first < chunk ? count_all - first : chunk;
            if (!scale_pass) {   /* contexts run forwards; the coder runs backwards */
                uint32_t srel = 0, prev = 8, top = 8;
                for (uint32_t j = 0; j < count; j++) {
                    uint32_t i = first + j, x = (w[i / 2] >> (4 * (i & 1))) & 15u;
                    if (i % 32u == 0) {
                        int d = (int)s[i / 32] - (int)anchor[m];
                        srel = (uint32_t)((d < -3 ? -3 : d > 3 ? 3 : d) + 3);
                        prev = 8; top = 8;
                    }
                    ctx[j] = (uint16_t)((srel * 9 + prev) * 9 + top);
                    prev = x & 7u;
                    if (top == 8 || prev > top) top = prev;
                }
            }
            ident[2] = g;
            Enc e = {RANS_L, tmp + 2u * MAX_CHUNK + 16u, tmp};
            if (nr3) e.x = scale_pass ? stream_x0(ident, s + first, count) : stream_x0(ident, w + first / 2, count / 2);
            for (uint32_t j = count; j-- > 0;) {
                uint32_t i = first + j, sym;
                const uint8_t *cdf;
                if (scale_pass) { sym = s[i]; cdf = scdf; }
                else { sym = (w[i / 2] >> (4 * (i & 1))) & 15u; cdf = wcdf + 34u * ctx[j]; }
                uint32_t start = rd16(cdf + 2 * sym);
                if (enc_put(&e, start, rd16(cdf + 2 * sym + 2) - start)) goto done;
            }
            if (enc_flush(&e)) goto done;
            const size_t len = (size_t)(tmp + 2u * MAX_CHUNK + 16u - e.p);
            if (len > 65535u || cap - cursor < len) goto done;
            memcpy(out + cursor, e.p, len);
            cursor += len;
            wr16(out + 32 + 2u * g, (uint32_t)len);
            if (scale_pass) sbytes += len; else wbytes += len;
        }
    }
    wr32(out, nr3 ? MAGIC_WNR3 : MAGIC_WNR2); wr32(out + 4, model_id);
    wr32(out + 8, (uint32_t)sbytes); wr32(out + 12, (uint32_t)wbytes);
    wr32(out + 16, wchunk); wr32(out + 20, schunk); wr32(out + 24, word24); wr32(out + 28, owner);
    {
        size_t padded = (cursor + 4095u) & ~(size_t)4095u;
        if (padded > cap) goto done;
        memset(out + cursor, 0, padded - cursor);
        *used = cursor; *total = padded;
        status = padded >= ((v.raw + 4095u) & ~(uint64_t)4095u) ? 1 : 0;
    }
done:
    free(tmp); free(ctx);
    return status;
}
