/* The 72-byte legacy expert entry every decode entry point takes, and its codec ids.
 * Same wire layout as the reference's WexEntry (c/wex_format.h:57-67, packed, little-endian):
 * a record of total_bytes bytes decodes to a canonical slab of scale_bytes + weight_bytes bytes,
 * the scales of matrix m (w1 gate, w2 down, w3 up) at scale_offsets[m] and its packed E2M1 nibbles
 * at weight_offsets[m]. */
#ifndef WEXB_WEX_ENTRY_H
#define WEXB_WEX_ENTRY_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#pragma pack(push, 1)
typedef struct {
    uint64_t file_offset;
    uint32_t total_bytes;            /* stored record bytes (a multiple of 4096) */
    uint32_t scale_bytes;            /* decoded scales, w1/w2/w3 */
    uint32_t weight_bytes;           /* decoded packed FP4, w1/w2/w3 */
    uint16_t scale_shapes[3][2];
    uint16_t weight_shapes[3][2];
    uint32_t scale_offsets[3];
    uint32_t weight_offsets[3];
    uint32_t flags;                  /* codec (low 8 bits) */
} WexEntry;
#pragma pack(pop)

typedef char wexb_entry_is_72_bytes[(sizeof(WexEntry) == 72) ? 1 : -1];

/* codec ids of the entry's flags (c/wex_format.h:34-38) */
#define WEX_ENTRY_RAW 0u
#define WEX_ENTRY_NEURAL_RANS 3u     /* WNR1: legacy, not decoded by this library */
#define WEX_ENTRY_NEURAL_RANS2 4u    /* WNR2 records (container model) */
#define WEX_ENTRY_NEURAL_RANS3 5u    /* WNR3 records (codec 5 of WEX4) */

/* container header flag of canonical-zero (value-exact) WNR3 containers (c/wex_format.h:33) */
#define WEX_HEADER_CANONICAL_ZERO 64u

#ifdef __cplusplus
}
#endif
#endif
