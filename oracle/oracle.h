/* ORACLE — test infrastructure only. Never linked, loaded or called by the product.
 *
 * A plain-C restatement of the reference's CPU semantics for the WEX4 expert decode path, used by
 * tests/, the smoke check and the bench's CPU-baseline leg to check the CUDA decoder against.
 * Each function names the reference lines it follows (paths inside the reference project).
 * Parity of this restatement is pinned in tests/ against:
 *   - the reference's own compiled CPU tools (oracle/_ref/, built by `make -C oracle ref`),
 *   - the reference's hash known answers (c/tests/test_wex_format.c:668-693),
 *   - the content digests of the reference's WNR3 conformance vectors (wex4/vectors/MANIFEST.tsv).
 */
#ifndef WEXB_ORACLE_H
#define WEXB_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* MurmurHash3_x86_32 of p[0..n) under `seed`. */
uint32_t oracle_murmur3(const uint8_t *p, size_t n, uint32_t seed);
/* WNR3 stream end state: L + (MurmurHash3(ident[4] LE || data, seed "WNR3") & 0x7fffff). */
uint32_t oracle_nr3_x0(const uint32_t ident[4], const uint8_t *data, uint32_t n);
/* FNV-1a, 0 mapped to 1 (model ids). */
uint32_t oracle_fnv1a(const uint8_t *p, size_t n);
/* Rule-g anchor of n coded scales. */
uint8_t oracle_anchor(const uint8_t *scales, uint32_t n);
/* 0 and *id when blob is a valid WNM2 model of `bytes` bytes, else -1. */
int oracle_wnm2_open(const uint8_t *blob, size_t bytes, uint32_t *id);
/* Decode a codec-4 (WNR2) or codec-5 (WNR3) expert record described by the 72-byte legacy entry
 * `entry` (its total_bytes bytes at `record`) with the WNM2 model `blob` into the canonical slab
 * out[0 .. scale_bytes + weight_bytes). Returns 0, or -1 with out unspecified (callers decode into
 * scratch). *where (optional) receives the failing check: 1 entry/parse, 2 stream structure,
 * 3 stream hash, 4 canonical zero, 5 ceil at scale 0, 6 model. */
int oracle_nrx_decode(const uint8_t *blob, const uint8_t *entry, const uint8_t *record, uint8_t *out, int *where);
/* SHA-256 (FIPS 180-4). */
void oracle_sha256(const uint8_t *p, size_t n, uint8_t out[32]);

/* WNR4 kind MX (MXFP4). geo = u32[13]: kind, scount[3], scols[3], soff[3], woff[3]. Decodes the
 * record (total bytes) of owner `owner` into out (the geometry's raw bytes). Returns 0 or the OR of
 * the error bits 1 structure, 2 hash, 4 ceil, 8 canonical zero. */
uint32_t oracle_wnr4_decode(const uint8_t *model_blob, size_t model_bytes, const uint32_t *geo,
                            const uint8_t *rec, size_t total, uint32_t owner, uint8_t *out);
/* Id of a valid WNM4 model blob, 0 if invalid. */
uint32_t oracle_wnm4_id(const uint8_t *blob, size_t bytes);

#ifdef __cplusplus
}
#endif
#endif
