/* The WEX4 container ABI that the reference's Python reader binds through ctypes (CLib,
 * wex4/wex4.py:292-310), implemented over the GPU decoder: a library exporting these names is a
 * drop-in for `python wex4/wex4.py verify FILE --dll libwexb200.so`.
 * Return values are the reference's WEX4_E_* codes (c/wex4.h:45-47): 0 ok, -1 ARG, -2 MAGIC, -3 HASH,
 * -4 VERSION, -5 FEATURE, -6 HEADER, -7 INDEX, -8 BLOB, -9 RECORD, -10 TENSOR, -11 NAME, -12 LAYOUT,
 * -13 EXPERT, -14 DATA, -15 UNSUPPORTED.
 * Header page and index are validated on the host with the reference's rules and order
 * (c/wex4.h:185-437); record SHA-256 checks, RAW padding checks, WNR3 decodes and the content digest
 * run on the GPU. */
#ifndef WEXB_WEX4_TOOLS_H
#define WEXB_WEX4_TOOLS_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define WEX4_CHECK_HASHES 1     /* verify every blob and record SHA-256 */
#define WEX4_CHECK_DECODE 2     /* decode every record and write the content digest */
#define WEX4_CHECK_CODEC8 4     /* addition: also decode draft codec-8 (WNR4 kind MX) records */
#define WEX4_CHECK_NO_DIGEST 8  /* addition: with WEX4_CHECK_DECODE, decode and verify but skip the digest */

/* 1 (wex4/wex4_tools.c:25) */
uint32_t wex4_tools_abi(void);
/* SHA-256 of host bytes (wex4/wex4_tools.c:26) */
void wex4_sha256_bytes(const unsigned char *p, size_t n, unsigned char *out);
/* Whole file in host memory: header, index, then (flags) every hash and every record; the content
 * digest (32 bytes) with WEX4_CHECK_DECODE (wex4/wex4_tools.c:67-168). */
int wex4_check(const unsigned char *file, uint64_t len, int flags, unsigned char *digest);
/* 0 when the header page and the index (as read from disk, 4096-aligned) are valid
 * (wex4/wex4_tools.c:188-191). */
int wex4_validate(const unsigned char *page, uint64_t file_bytes, const unsigned char *index, size_t index_len);
/* Decode record r from its stored bytes into out (rec.decoded bytes; scratch until it returns 0);
 * blob = the bytes of its model blob or NULL; check_sha also verifies the record's SHA-256
 * (wex4/wex4_tools.c:193-212). */
int wex4_decode_record_buf(const unsigned char *page, uint64_t file_bytes, const unsigned char *index,
                           size_t index_len, uint32_t r, const unsigned char *stored, const unsigned char *blob,
                           int check_sha, unsigned char *out);
/* The legacy layers x experts table of 72-byte entries rebuilt from the index (wex4/wex4_tools.c:215-231). */
int wex4_expert_table(const unsigned char *page, uint64_t file_bytes, const unsigned char *index, size_t index_len,
                      unsigned char *out);
/* WBP1 (codec 6, non-expert tensors; wex4/wex4_tools.c:27-35): the canonical encoder (host) and the
 * GPU decoder of one record into host memory (out is scratch until it returns 0); 0 or -1. */
int wex4_bp_encode_record(const unsigned char *data, uint32_t decoded, uint32_t planes, uint32_t chunk_log2,
                          uint32_t transform, uint32_t owner, unsigned char *out, size_t capacity, size_t *written);
int wex4_bp_decode_record(const unsigned char *record, size_t total, uint32_t decoded, uint32_t owner,
                          unsigned char *out);
/* wex4_check on a copy of the file that ends right before an inaccessible page, so that a host read past
 * the end faults instead of passing silently (wex4/wex4_tools.c:170-178; the reference also guard-pages
 * its host decode buffer: here the decoded bytes are in device memory). Same return values. */
int wex4_fuzz_check(const unsigned char *file, uint64_t len, int flags, unsigned char *digest);
/* Test tooling of the reference (mutation fuzzing, an engine store on disk), not part of the decode
 * path: they return WEX4_E_UNSUPPORTED (-15) (wex4/wex4_tools.c:250-312, :317-348). */
int wex4_fuzz_run(const unsigned char *file, uint64_t len, uint64_t seed, uint32_t iterations, int mode,
                  uint64_t *counts);
int wex4_store_probe(const char *path, const unsigned char *root, unsigned char *out, uint64_t capacity,
                     uint32_t *info);

#ifdef __cplusplus
}
#endif
#endif
