/* ORACLE — test infrastructure only (see oracle.h). CPU restatement of the WNR4 kind-MX record
 * decode of the reference draft codec 8 (wnr4/wnr4.h): geometry :108-140, WNM4 model :142-199,
 * record parse :317-346, tile decode :388-478, record decode :481-493. Kind NV (NVFP4) is not
 * restated: only MXFP4 experts are on this path. */
#include "oracle.h"
#include <stdlib.h>
#include <string.h>

#define W4_L 0x10000u
#define W4_PREC 14u
#define W4_MAGIC 0x34524e57u   /* "WNR4" */
#define W4_MODEL 0x344d4e57u   /* "WNM4" */
#define W4_ERR_STRUCT 1u
#define W4_ERR_HASH 2u
#define W4_ERR_CEIL 4u
#define W4_ERR_CZ 8u
#define MX_CLASSES 7u
#define MX_R 3

static uint32_t rd32(const uint8_t *p) { return p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24; }
static uint32_t rd16(const uint8_t *p) { return p[0] | (uint32_t)p[1] << 8; }
static uint32_t rotl(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }
static uint32_t mm3_word(uint32_t h, uint32_t k) {
    k *= 0xcc9e2d51u; k = rotl(k, 15); k *= 0x1b873593u;
    return rotl(h ^ k, 13) * 5u + 0xe6546b64u;
}
static uint32_t mm3_final(uint32_t h, uint32_t len) {
    h ^= len; h ^= h >> 16; h *= 0x85ebca6bu; h ^= h >> 13; h *= 0xc2b2ae35u; h ^= h >> 16;
    return h;
}

typedef struct {
    uint32_t pb, wctx;
    const uint8_t *wcdf, *scdf;   /* [3][wctx][17] and [3][1][257] u16 LE */
    uint32_t id;
} Model4;

static int cdf_ok(const uint8_t *c, uint32_t n) {
    if (rd16(c) != 0 || rd16(c + 2 * n) != (1u << W4_PREC)) return 0;
    for (uint32_t i = 0; i < n; i++) if (rd16(c + 2 * i + 2) <= rd16(c + 2 * i)) return 0;
    return 1;
}
/* wnr4/wnr4.h:170-190, kind MX only */
static int model_open(const uint8_t *b, size_t bytes, Model4 *m) {
    if (!b || bytes < 32) return -1;
    uint32_t kind = rd32(b + 8), pb = rd32(b + 24);
    if (rd32(b) != W4_MODEL || rd32(b + 4) != 1 || kind != 0 || (pb != 1 && pb != 5)) return -1;
    m->pb = pb; m->wctx = MX_CLASSES * 81u * pb;
    if (bytes != 32u + 3u * (size_t)m->wctx * 34u + 3u * 514u || rd32(b + 12) != W4_PREC || rd32(b + 16) != m->wctx ||
        rd32(b + 20) != 1 || rd32(b + 28)) return -1;
    m->wcdf = b + 32;
    m->scdf = b + 32 + 3u * (size_t)m->wctx * 34u;
    for (uint32_t i = 0; i < 3u * m->wctx; i++) if (!cdf_ok(m->wcdf + 34u * i, 16)) return -1;
    for (uint32_t i = 0; i < 3u; i++) if (!cdf_ok(m->scdf + 514u * i, 256)) return -1;
    uint32_t h = 2166136261u;
    for (size_t i = 0; i < bytes; i++) h = (h ^ b[i]) * 16777619u;
    m->id = h ? h : 1u;
    return 0;
}
uint32_t oracle_wnm4_id(const uint8_t *blob, size_t bytes) {
    Model4 m;
    return model_open(blob, bytes, &m) ? 0u : m.id;
}

typedef struct { uint32_t scount[3], scols[3], soff[3], woff[3]; uint64_t raw; } Geo;
static int geo_read(const uint32_t *v, Geo *g) {
    uint64_t lo[6], hi[6];
    if (!v || v[0] != 0) return -1;   /* kind MX */
    memset(g, 0, sizeof *g);
    for (int m = 0; m < 3; m++) {
        g->scount[m] = v[1 + m]; g->scols[m] = v[4 + m]; g->soff[m] = v[7 + m]; g->woff[m] = v[10 + m];
        if (!g->scount[m] || !g->scols[m] || g->scount[m] % g->scols[m] || g->scount[m] >= (1u << 27)) return -1;
        lo[2 * m] = g->soff[m]; hi[2 * m] = (uint64_t)g->soff[m] + g->scount[m];
        lo[2 * m + 1] = g->woff[m]; hi[2 * m + 1] = (uint64_t)g->woff[m] + 16ull * g->scount[m];
        if (hi[2 * m] > g->raw) g->raw = hi[2 * m];
        if (hi[2 * m + 1] > g->raw) g->raw = hi[2 * m + 1];
    }
    for (int i = 0; i < 6; i++)
        for (int j = i + 1; j < 6; j++) if (lo[i] < hi[j] && lo[j] < hi[i]) return -1;
    return 0;
}

/* symbol of `slot` in a CDF of n symbols: largest s with cdf[s] <= slot */
static uint32_t find(const uint8_t *cdf, uint32_t n, uint32_t slot) {
    uint32_t lo = 0, hi = n;
    while (hi - lo > 1) { uint32_t mid = (lo + hi) / 2; if (rd16(cdf + 2 * mid) <= slot) lo = mid; else hi = mid; }
    return lo;
}
static uint32_t dbl8(uint32_t w) {   /* magnitudes a -> a + min(a, 2) on 8 nibbles, signs kept */
    uint32_t r = w & 0x88888888u;
    for (int q = 0; q < 8; q++) { uint32_t a = (w >> (4 * q)) & 7u; r |= (a + (a < 2 ? a : 2)) << (4 * q); }
    return r;
}

typedef struct {
    uint32_t model_id, owner, flags, G, ntiles, payload, tile_base[4];
    uint8_t anchor[3];
    const uint8_t *offsets, *data;
} Rec4;

/* One tile: 32 lanes in lockstep over a shared stream of u16 words (wnr4/wnr4.h:388-478). */
static uint32_t tile_decode(const Model4 *md, const Geo *g, const Rec4 *r, uint32_t t, uint8_t *out) {
    uint32_t m = t >= r->tile_base[2] ? 2 : t >= r->tile_base[1] ? 1 : 0;
    uint32_t c0 = (t - r->tile_base[m]) * 32u * r->G, n = g->scount[m] - c0;
    if (n > 32u * r->G) n = 32u * r->G;
    uint32_t o0 = rd32(r->offsets + 4 * t), o1 = rd32(r->offsets + 4 * t + 4);
    if (o1 < o0 || o1 - o0 < 128 || o1 > r->payload) return W4_ERR_STRUCT;
    const uint8_t *tile = r->data + o0, *words = tile + 128;
    const uint32_t nwords = (o1 - o0 - 128) / 2;
    const uint8_t *wt = md->wcdf + 34u * (size_t)m * md->wctx, *st = md->scdf + 514u * m;
    const int ceil = (r->flags >> m) & 1u, cz = (r->flags & 8u) != 0;
    uint8_t *so = out + g->soff[m], *wo = out + g->woff[m];
    const uint32_t anchors = r->anchor[0] | (uint32_t)r->anchor[1] << 8 | (uint32_t)r->anchor[2] << 16;
    const uint32_t word = 0u | r->flags << 8 | r->G << 16;
    uint32_t x[32], hash[32], ptr = 0, err = 0;
    for (uint32_t l = 0; l < 32; l++) {
        x[l] = rd32(tile + 4 * l);
        if (x[l] < W4_L) return W4_ERR_STRUCT;
        uint32_t h = W4_MAGIC;
        h = mm3_word(h, r->model_id); h = mm3_word(h, r->owner); h = mm3_word(h, t);
        h = mm3_word(h, l); h = mm3_word(h, word); hash[l] = mm3_word(h, anchors);
    }
#define STEP(lane, cdf, nsym, sym)                                                         \
    do {                                                                                   \
        uint32_t slot_ = x[lane] & 0x3fffu;                                                \
        sym = find(cdf, nsym, slot_);                                                      \
        uint32_t s0_ = rd16(cdf + 2 * sym);                                                \
        x[lane] = (rd16(cdf + 2 * sym + 2) - s0_) * (x[lane] >> W4_PREC) + slot_ - s0_;    \
    } while (0)
#define RENORM(lane)                                                                       \
    do {                                                                                   \
        if (x[lane] < W4_L) {                                                              \
            if (ptr >= nwords) return W4_ERR_STRUCT;   /* the bits seen so far are dropped */ \
            x[lane] = x[lane] << 16 | rd16(words + 2 * ptr); ptr++;                        \
        }                                                                                  \
    } while (0)
    /* phase 1: the tile's scales, 32 at a time, lane l owning scale c0 + 32k + l */
    for (uint32_t k = 0; 32 * k < n; k++)
        for (uint32_t l = 0; l < 32; l++) {
            uint32_t i = 32 * k + l, y;
            if (i >= n) continue;
            STEP(l, st, 256, y);
            so[c0 + i] = (uint8_t)y;
            hash[l] = mm3_word(hash[l], y);
            RENORM(l);
        }
    /* phase 2: rounds of 32 cells, lane l owning cell c0 + 32j + l, 32 nibbles each */
    for (uint32_t j = 0; 32 * j < n; j++) {
        uint32_t act = n - 32 * j < 32 ? n - 32 * j : 32, pm[32], mx[32], cls[32], wd[32][4];
        memset(wd, 0, sizeof wd);
        for (uint32_t l = 0; l < act; l++) {
            int d = (int)so[c0 + 32 * j + l] - (int)r->anchor[m];
            cls[l] = (uint32_t)((d < -MX_R ? -MX_R : d > MX_R ? MX_R : d) + MX_R);
            pm[l] = mx[l] = 8;
        }
        for (uint32_t k = 0; k < 32; k++)
            for (uint32_t l = 0; l < act; l++) {
                /* lanes 2..31 keep the last 4 nibbles of their last cell in the state */
                if (l >= 2 && k >= 28 && j == (n - l - 1) / 32) continue;
                uint32_t ctx = (cls[l] * 9 + pm[l]) * 9 + mx[l], row = md->pb == 1 ? ctx : ctx * 5 + (k + 5 <= 32 ? 0 : k - 27), y;
                STEP(l, wt + 34u * row, 16, y);
                if (cz && y == 8) err |= W4_ERR_CZ;
                wd[l][k / 8] |= y << (4 * (k % 8));
                pm[l] = y & 7u;
                mx[l] = mx[l] == 8 ? pm[l] : (pm[l] > mx[l] ? pm[l] : mx[l]);
                RENORM(l);
            }
        for (uint32_t l = 0; l < act; l++) {
            uint32_t cell = c0 + 32 * j + l;
            if (l >= 2 && j == (n - l - 1) / 32) {
                uint32_t tail = x[l] - W4_L;
                if (x[l] < W4_L || tail > 0xffffu) return err | W4_ERR_STRUCT;
                for (int q = 0; q < 4; q++) {
                    uint32_t y = (tail >> (4 * q)) & 15u, a = y & 7u;
                    if (cz && y == 8) err |= W4_ERR_CZ;
                    mx[l] = mx[l] == 8 ? a : (a > mx[l] ? a : mx[l]);
                }
                wd[l][3] |= tail << 16;
                x[l] = W4_L;
            }
            for (int q = 0; q < 4; q++) hash[l] = mm3_word(hash[l], wd[l][q]);
            if (ceil && mx[l] == 5) {
                if (!so[cell]) err |= W4_ERR_CEIL;
                else { so[cell]--; for (int q = 0; q < 4; q++) wd[l][q] = dbl8(wd[l][q]); }
            }
            for (int q = 0; q < 4; q++)
                for (int b = 0; b < 4; b++) wo[16u * cell + 4 * q + b] = (uint8_t)(wd[l][q] >> (8 * b));
        }
    }
#undef STEP
#undef RENORM
    uint32_t H = 0;
    for (uint32_t l = 0; l < 32; l++) {
        uint32_t nsl = l < n ? (n - l + 31) / 32 : 0;   /* MX: one scale per cell */
        H ^= mm3_final(hash[l], 24u + 4u * nsl + 16u * nsl);
    }
    if (ptr != nwords) err |= W4_ERR_STRUCT;
    if (x[0] != W4_L + (H & 0xffffu) || x[1] != W4_L + (H >> 16)) err |= W4_ERR_HASH;
    for (uint32_t l = 2; l < 32; l++) if (x[l] != W4_L) err |= W4_ERR_STRUCT;
    return err;
}

/* wnr4/wnr4.h:317-346 (parse) and :481-493 (record decode) */
uint32_t oracle_wnr4_decode(const uint8_t *blob, size_t model_bytes, const uint32_t *geo, const uint8_t *rec,
                            size_t total, uint32_t owner, uint8_t *out) {
    Model4 md;
    Geo g;
    Rec4 r;
    if (model_open(blob, model_bytes, &md) || geo_read(geo, &g) || !rec || !out) return W4_ERR_STRUCT;
    if (total < 64 || (total & 4095u) || rd32(rec) != W4_MAGIC) return W4_ERR_STRUCT;
    memset(&r, 0, sizeof r);
    r.model_id = rd32(rec + 4); r.owner = rd32(rec + 8);
    r.flags = rec[13]; r.G = rec[14] | (uint32_t)rec[15] << 8;
    memcpy(r.anchor, rec + 16, 3);
    r.ntiles = rd32(rec + 20); r.payload = rd32(rec + 24);
    if (!r.model_id || rec[12] != 0 || rec[19] || r.G < 1 || r.G > 4096 || (r.flags & ~0x0fu)) return W4_ERR_STRUCT;
    for (int i = 28; i < 64; i++) if (rec[i]) return W4_ERR_STRUCT;
    uint32_t t = 0;
    for (int m = 0; m < 3; m++) { r.tile_base[m] = t; t += (g.scount[m] + 32u * r.G - 1) / (32u * r.G); }
    r.tile_base[3] = t;
    if (t != r.ntiles) return W4_ERR_STRUCT;
    uint64_t used = 64ull + 4ull * (r.ntiles + 1ull) + r.payload;
    if (used > total || ((used + 4095) & ~4095ull) != total) return W4_ERR_STRUCT;
    r.offsets = rec + 64;
    r.data = r.offsets + 4ull * (r.ntiles + 1ull);
    uint32_t prev = rd32(r.offsets);
    if (prev) return W4_ERR_STRUCT;
    for (uint32_t i = 1; i <= r.ntiles; i++) {
        uint32_t o = rd32(r.offsets + 4 * i);
        if (o < prev || o - prev < 128 || ((o - prev) & 1u)) return W4_ERR_STRUCT;
        prev = o;
    }
    if (prev != r.payload) return W4_ERR_STRUCT;
    for (uint64_t i = used; i < total; i++) if (rec[i]) return W4_ERR_STRUCT;
    if (r.model_id != md.id || r.owner != owner) return W4_ERR_STRUCT;
    uint8_t *tmp = (uint8_t *)calloc(1, (size_t)g.raw);
    if (!tmp) return W4_ERR_STRUCT;
    uint32_t err = 0;
    for (uint32_t i = 0; i < r.ntiles; i++) err |= tile_decode(&md, &g, &r, i, tmp);
    if (!err) memcpy(out, tmp, (size_t)g.raw);
    free(tmp);
    return err;
}
