/* wexb_wnr4: the writer side of the draft WNR4 codec (codec 8), kind MX only, host C, no CUDA:
 * WNM4 model training and the record encoder for MXFP4 expert slabs in the coded domain of
 * wexb_nr3_prepare (canonical zero, ceil form, the same flag bits). The byte layout is the
 * reference's (wnr4/wnr4.h: geometry :108-140, model :142-199, record :317-346, tile :388-478);
 * tests/ check that the reference's own decoder accepts what it writes.
 *
 * A tile is 32 rANS lanes (32-bit states, L = 2^16, 16-bit words) over 32 G cells of one matrix; lane
 * l owns cells l, l + 32, ... Decode order: phase 1 the tile's scales, 32 at a time in lane order;
 * phase 2 rounds of 32 cells, nibble k of every lane's cell before nibble k + 1, lanes 2..31 keeping
 * the last four nibbles of their last cell in their final state. The lanes share one word stream,
 * read in that lockstep order; the encoder runs the same order backwards and reverses its words. The
 * final states of lanes 0 and 1 hold the tile hash, those of lanes 2..31 are L. */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define EXPORT __attribute__((visibility("default")))
#define W4_L 0x10000u
#define W4_PREC 14u
#define W4_TOTAL (1u << W4_PREC)
#define W4_MAGIC 0x34524e57u   /* "WNR4" */
#define W4_MODEL 0x344d4e57u   /* "WNM4" */
#define MX_CLASSES 7u

static uint32_t rd32(const uint8_t *p) { return p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24; }
static uint32_t rd16(const uint8_t *p) { return p[0] | (uint32_t)p[1] << 8; }
static void wr32(uint8_t *p, uint32_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); p[2] = (uint8_t)(v >> 16); p[3] = (uint8_t)(v >> 24); }
static void wr16(uint8_t *p, uint32_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); }
static uint32_t rotl(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }
static uint32_t mm3_word(uint32_t h, uint32_t k) {
    k *= 0xcc9e2d51u; k = rotl(k, 15); k *= 0x1b873593u;
    return rotl(h ^ k, 13) * 5u + 0xe6546b64u;
}
static uint32_t mm3_final(uint32_t h, uint32_t len) {
    h ^= len; h ^= h >> 16; h *= 0x85ebca6bu; h ^= h >> 13; h *= 0xc2b2ae35u; h ^= h >> 16;
    return h;
}
static uint32_t fnv1a(const uint8_t *p, size_t n) {
    uint32_t h = 2166136261u;
    for (size_t i = 0; i < n; i++) h = (h ^ p[i]) * 16777619u;
    return h ? h : 1u;
}

/* An expert slab from its 72-byte entry: cells (= scales) and offsets per matrix. */
typedef struct { uint32_t cells[3], soff[3], woff[3]; uint64_t raw; } Slab;
static int slab_of(const uint8_t *e, Slab *s) {
    if (!e) return -1;
    uint64_t raw = 0;
    for (int m = 0; m < 3; m++) {
        uint32_t sr = rd16(e + 20 + 4 * m), sc = rd16(e + 22 + 4 * m), wr = rd16(e + 32 + 4 * m), wc = rd16(e + 34 + 4 * m);
        if (!sr || !sc || sr != wr || sc * 16u != wc) return -1;
        s->cells[m] = sr * sc; s->soff[m] = rd32(e + 44 + 4 * m); s->woff[m] = rd32(e + 56 + 4 * m);
        if ((uint64_t)s->soff[m] + s->cells[m] > raw) raw = (uint64_t)s->soff[m] + s->cells[m];
        if ((uint64_t)s->woff[m] + 16ull * s->cells[m] > raw) raw = (uint64_t)s->woff[m] + 16ull * s->cells[m];
    }
    s->raw = raw;
    return 0;
}
/* rule g of the WNR3 writer: the v maximising count(v) + count(v + 1) */
static uint8_t anchor_g(const uint8_t *s, uint32_t n) {
    uint32_t h[256] = {0}, best = 0, top = 0;
    for (uint32_t i = 0; i < n; i++) h[s[i]]++;
    for (uint32_t v = 0; v < 255; v++) if (h[v] + h[v + 1] > top) { top = h[v] + h[v + 1]; best = v; }
    return (uint8_t)best;
}
static uint32_t wctx_of(uint32_t pb) { return MX_CLASSES * 81u * pb; }
static uint32_t row_of(uint32_t pb, uint32_t cls, uint32_t pm, uint32_t mx, uint32_t k) {
    const uint32_t ctx = (cls * 9u + pm) * 9u + mx;
    return pb == 1 ? ctx : ctx * 5u + (k + 5u <= 32u ? 0u : k - 27u);
}
static uint32_t cls_of(uint8_t scale, uint8_t anchor) {
    const int d = (int)scale - (int)anchor;
    return (uint32_t)((d < -3 ? -3 : d > 3 ? 3 : d) + 3);
}

EXPORT size_t wexb_w4_model_bytes(uint32_t pb) { return (pb == 1 || pb == 5) ? 32u + 3ull * wctx_of(pb) * 34u + 3u * 514u : 0; }
EXPORT size_t wexb_w4_counts_words(uint32_t pb) { return 3ull * wctx_of(pb) * 16u + 3u * 256u; }

/* Training counts of one coded expert: weights [3][wctx][16], then scales [3][256]. */
EXPORT int wexb_w4_count(const uint8_t *entry, const uint8_t *coded, uint32_t pb, uint64_t *counts) {
    Slab s;
    if ((pb != 1 && pb != 5) || !coded || !counts || slab_of(entry, &s)) return -1;
    const uint32_t wctx = wctx_of(pb);
    uint64_t *sc = counts + 3ull * wctx * 16u;
    for (int m = 0; m < 3; m++) {
        const uint8_t *sb = coded + s.soff[m], *wb = coded + s.woff[m], a = anchor_g(sb, s.cells[m]);
        for (uint32_t c = 0; c < s.cells[m]; c++) {
            const uint32_t cls = cls_of(sb[c], a);
            uint32_t pm = 8, mx = 8;
            sc[256u * m + sb[c]]++;
            for (uint32_t k = 0; k < 32; k++) {
                const uint32_t y = (wb[16u * c + k / 2] >> (4 * (k & 1))) & 15u;
                counts[((size_t)m * wctx + row_of(pb, cls, pm, mx, k)) * 16u + y]++;
                pm = y & 7u;
                mx = mx == 8 ? pm : (pm > mx ? pm : mx);
            }
        }
    }
    return 0;
}

/* Counts -> 14-bit CDF: every symbol at least 1, the rest in proportion, the remainder one each to
 * the largest fractional parts (lower symbol first on ties). */
static void quantize(const uint64_t *counts, uint32_t n, uint8_t *cdf) {
    uint64_t total = 0, rem[256];
    uint32_t freq[256], used = 0, spare = W4_TOTAL - n;
    uint8_t taken[256] = {0};
    for (uint32_t i = 0; i < n; i++) total += counts[i];
    for (uint32_t i = 0; i < n; i++) {
        const uint64_t scaled = total ? counts[i] * spare : spare, div = total ? total : n;
        freq[i] = 1u + (uint32_t)(scaled / div);
        rem[i] = scaled % div;
        used += freq[i];
    }
    for (uint32_t extra = W4_TOTAL - used; extra; extra--) {
        uint32_t best = n;
        for (uint32_t i = 0; i < n; i++) if (!taken[i] && (best == n || rem[i] > rem[best])) best = i;
        taken[best] = 1; freq[best]++;
    }
    uint32_t at = 0;
    for (uint32_t i = 0; i <= n; i++) { wr16(cdf + 2 * i, at); if (i < n) at += freq[i]; }
}

/* WNM4 blob of kind MX: {magic, version 1, kind 0, precision 14, weight contexts, 1 scale context,
 * pb, 0}, the weight CDFs [3][wctx][17] and the scale CDFs [3][257]. Returns its id, 0 on error. */
EXPORT uint32_t wexb_w4_build(uint32_t pb, const uint64_t *counts, uint8_t *blob) {
    if ((pb != 1 && pb != 5) || !counts || !blob) return 0;
    const uint32_t wctx = wctx_of(pb), head[8] = {W4_MODEL, 1u, 0u, W4_PREC, wctx, 1u, pb, 0u};
    for (int i = 0; i < 8; i++) wr32(blob + 4 * i, head[i]);
    for (uint32_t r = 0; r < 3u * wctx; r++) quantize(counts + 16ull * r, 16, blob + 32 + 34ull * r);
    for (uint32_t m = 0; m < 3; m++) quantize(counts + 3ull * wctx * 16u + 256u * m, 256, blob + 32 + 3ull * wctx * 34u + 514u * m);
    return fnv1a(blob, wexb_w4_model_bytes(pb));
}

/* One rANS symbol onto a lane state (the decode step inverted), pushing at most one word. */
typedef struct { uint16_t *w; size_t n, cap; } Words;
static int put(uint32_t *x, uint32_t start, uint32_t freq, Words *ws) {
    if (*x >= (W4_L >> W4_PREC << 16) * freq) {
        if (ws->n == ws->cap) return -1;
        ws->w[ws->n++] = (uint16_t)*x;
        *x >>= 16;
    }
    *x = (*x / freq << W4_PREC) + *x % freq + start;
    return 0;
}

/* Encode one tile into dst (its 32 states, then its words); returns its byte size or 0. */
static size_t encode_tile(const uint8_t *blob, uint32_t pb, uint32_t model_id, uint32_t owner, uint32_t flags, uint32_t G,
                          uint32_t anchors, const uint8_t *sb, const uint8_t *wb, uint8_t anchor, uint32_t m, uint32_t t,
                          uint32_t c0, uint32_t n, Words *ws, uint8_t *dst, size_t room) {
    const uint32_t wctx = wctx_of(pb);
    const uint8_t *wcdf = blob + 32 + 34ull * m * wctx, *scdf = blob + 32 + 3ull * wctx * 34u + 514u * m;
    uint32_t x[32], hash[32], H = 0;
    for (uint32_t l = 0; l < 32; l++) {   /* lane hashes over the coded values (the decoder's order per lane) */
        uint32_t h = W4_MAGIC;
        h = mm3_word(h, model_id); h = mm3_word(h, owner); h = mm3_word(h, t);
        h = mm3_word(h, l); h = mm3_word(h, flags << 8 | G << 16); h = mm3_word(h, anchors);
        for (uint32_t i = l; i < n; i += 32) h = mm3_word(h, sb[c0 + i]);
        for (uint32_t i = l; i < n; i += 32)
            for (int q = 0; q < 4; q++) h = mm3_word(h, rd32(wb + 16ull * (c0 + i) + 4 * q));
        const uint32_t nsl = l < n ? (n - l + 31) / 32 : 0;
        hash[l] = mm3_final(h, 24u + 4u * nsl + 16u * nsl);
        H ^= hash[l];
        x[l] = W4_L;
    }
    x[0] = W4_L + (H & 0xffffu);
    x[1] = W4_L + (H >> 16);
    ws->n = 0;
    /* phase 2 backwards */
    for (uint32_t j = (n - 1) / 32 + 1; j-- > 0;) {
        const uint32_t act = n - 32 * j < 32 ? n - 32 * j : 32;
        uint32_t rows[32][32];
        for (uint32_t l = 0; l < act; l++) {   /* contexts run forwards */
            const uint32_t cell = c0 + 32 * j + l, cls = cls_of(sb[cell], anchor);
            uint32_t pm = 8, mx = 8;
            for (uint32_t k = 0; k < 32; k++) {
                const uint32_t y = (wb[16ull * cell + k / 2] >> (4 * (k & 1))) & 15u;
                rows[l][k] = row_of(pb, cls, pm, mx, k);
                pm = y & 7u;
                mx = mx == 8 ? pm : (pm > mx ? pm : mx);
            }
            if (l >= 2 && j == (n - l - 1) / 32) x[l] = W4_L + rd16(wb + 16ull * cell + 14);   /* the tail */
        }
        for (uint32_t k = 32; k-- > 0;)
            for (uint32_t l = act; l-- > 0;) {
                if (l >= 2 && k >= 28 && j == (n - l - 1) / 32) continue;
                const uint32_t cell = c0 + 32 * j + l, y = (wb[16ull * cell + k / 2] >> (4 * (k & 1))) & 15u;
                const uint8_t *cdf = wcdf + 34ull * rows[l][k];
                const uint32_t start = rd16(cdf + 2 * y);
                if (put(&x[l], start, rd16(cdf + 2 * y + 2) - start, ws)) return 0;
            }
    }
    /* phase 1 backwards */
    for (uint32_t k = (n - 1) / 32 + 1; k-- > 0;)
        for (uint32_t l = 32; l-- > 0;) {
            const uint32_t i = 32 * k + l;
            if (i >= n) continue;
            const uint32_t y = sb[c0 + i], start = rd16(scdf + 2 * y);
            if (put(&x[l], start, rd16(scdf + 2 * y + 2) - start, ws)) return 0;
        }
    const size_t bytes = 128u + 2u * ws->n;
    if (bytes > room) return 0;
    for (uint32_t l = 0; l < 32; l++) wr32(dst + 4 * l, x[l]);
    for (size_t i = 0; i < ws->n; i++) wr16(dst + 128 + 2 * i, ws->w[ws->n - 1 - i]);
    return bytes;
}

/* Encode a coded expert (flags from wexb_nr3_prepare) as a kind-MX WNR4 record of G cells per lane
 * (32 G cells per tile), zero-padded to 4096, into out (cap bytes). Returns the record size, 0 when
 * it is not smaller than the 4096-aligned raw slab, -1 on error. */
EXPORT long long wexb_w4_encode(const uint8_t *blob, size_t blob_bytes, const uint8_t *entry, const uint8_t *coded,
                                uint32_t flags, uint32_t owner, uint32_t G, uint8_t *out, size_t cap) {
    Slab s;
    if (!blob || blob_bytes < 32 || !coded || !out || slab_of(entry, &s) || G < 1 || G > 4096 || (flags & ~0x0fu)) return -1;
    const uint32_t pb = rd32(blob + 24);
    if (rd32(blob) != W4_MODEL || (pb != 1 && pb != 5) || blob_bytes != wexb_w4_model_bytes(pb)) return -1;
    const uint32_t model_id = fnv1a(blob, blob_bytes);
    uint8_t anchor[3];
    uint32_t base[4], ntiles = 0;
    for (int m = 0; m < 3; m++) {
        anchor[m] = anchor_g(coded + s.soff[m], s.cells[m]);
        base[m] = ntiles;
        ntiles += (s.cells[m] + 32u * G - 1) / (32u * G);
    }
    base[3] = ntiles;
    const uint32_t anchors = anchor[0] | (uint32_t)anchor[1] << 8 | (uint32_t)anchor[2] << 16;
    const size_t head = 64u + 4ull * (ntiles + 1u);
    if (cap < head) return -1;
    memset(out, 0, head);
    Words ws = {NULL, 0, 0};
    ws.cap = 16u * 32u * G + 32u * G + 64u;   /* at most one word per symbol of a tile */
    ws.w = (uint16_t *)malloc(sizeof(uint16_t) * ws.cap);
    if (!ws.w) return -1;
    size_t at = head;
    long long result = -1;
    for (uint32_t t = 0; t < ntiles; t++) {
        const uint32_t m = t >= base[2] ? 2 : t >= base[1] ? 1 : 0;
        const uint32_t c0 = (t - base[m]) * 32u * G, n = s.cells[m] - c0 < 32u * G ? s.cells[m] - c0 : 32u * G;
        const size_t bytes = encode_tile(blob, pb, model_id, owner, flags, G, anchors, coded + s.soff[m], coded + s.woff[m],
                                         anchor[m], m, t, c0, n, &ws, out + at, cap - at);
        if (!bytes) goto done;
        at += bytes;
        if (at - head > 0xffffffffull) goto done;
        wr32(out + 64 + 4ull * (t + 1), (uint32_t)(at - head));
    }
    wr32(out, W4_MAGIC); wr32(out + 4, model_id); wr32(out + 8, owner);
    out[12] = 0; out[13] = (uint8_t)flags; wr16(out + 14, G);
    out[16] = anchor[0]; out[17] = anchor[1]; out[18] = anchor[2]; out[19] = 0;
    wr32(out + 20, ntiles); wr32(out + 24, (uint32_t)(at - head));
    {
        const size_t padded = (at + 4095u) & ~(size_t)4095u;
        if (padded > cap) goto done;
        memset(out + at, 0, padded - at);
        result = padded >= ((s.raw + 4095u) & ~4095ull) ? 0 : (long long)padded;
    }
done:
    free(ws.w);
    return result;
}
