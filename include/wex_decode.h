/* The engine-facing WEX decode API of the reference (c/wex_decode.h:26-79), implemented in this library
 * directly over the GPU helper of wex_cuda_helper.h (the reference loads its helper DLL by name,
 * c/wex_decode.c:41-105, Windows only). Same signatures and return conventions. Differences:
 *   - there is no CPU decoder: with COLI_WEX_CUDA_LIB=0 or without a CUDA device the cuda entry points
 *     report "unavailable" (1) as the reference's non-Windows build does, and coli_wex_decode_record
 *     returns -1 for a WNR2/WNR3 record (it cannot fall back to a CPU decode);
 *   - legacy codecs 1..3 (scale tiles, palette3, WNR1; not in WEX4) return -1 from
 *     coli_wex_decode_record. */
#ifndef WEXB_WEX_DECODE_H
#define WEXB_WEX_DECODE_H
#include <stddef.h>
#include <stdint.h>

#include "wex_entry.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Canonical host slab of a record held at slab + read offset: RAW entries (codec 0) are already a slab
 * (0 when total_bytes is the aligned raw size), WNR2/WNR3 records decode on the GPU; 0 or -1, the slab
 * untouched on failure (c/wex_decode.h:26, c/wex_decode.c:323-352). */
int coli_wex_decode_record(const WexEntry *entry, unsigned char *slab, size_t capacity);
/* Successful GPU decodes to host / to device so far (c/wex_decode.h:27, :40). */
uint64_t coli_wex_cuda_decode_count(void);
uint64_t coli_wex_cuda_device_decode_count(void);
/* 1 when the direct-to-device decode is available (c/wex_decode.h:34). */
int coli_wex_cuda_device_available(void);
/* (c/wex_decode.h:35-36) */
int coli_wex_cuda_decode_to_device(const WexEntry *entry, const unsigned char *record, int device,
                                   unsigned char *const dst_scale[3], unsigned char *const dst_weight[3]);
/* Page-lock a staging buffer: 0 registered, 1 unavailable (c/wex_decode.h:38-39). */
int coli_wex_cuda_host_register(void *pointer, size_t bytes);
int coli_wex_cuda_host_unregister(void *pointer);
/* Register a container's WNM2 model (process-wide, kept until exit; again is a no-op): 0 and *id, or
 * -1 for an invalid blob or a full registry (c/wex_decode.h:46). */
int coli_wex_register_model(const unsigned char *blob, size_t bytes, uint32_t *id);
/* 1 when WNR2 / WNR3 records decode on the GPU (c/wex_decode.h:48, :51). */
int coli_wex_cuda_nr2_available(void);
int coli_wex_cuda_nr3_available(void);
/* 1 (and a stderr line prefixed by `who`) when a canonical-zero container must be refused because
 * DSV4_CUDA_MOE_MASKED != 0; otherwise 0 (c/wex_decode.h:56, c/wex_decode.c:309-321). */
int coli_wex_container_refused(uint32_t header_flags, const char *who);
/* Batched direct-to-device decode (c/wex_decode.h:63-67). */
int coli_wex_cuda_batch_available(void);
int coli_wex_cuda_decode_batch_to_device(int n, const WexEntry *const *entries, const unsigned char *const *records,
                                         int device, unsigned char *const *dst_scale, unsigned char *const *dst_weight,
                                         int *status);
/* Batched decode to host slabs (c/wex_decode.h:76-79). */
int coli_wex_cuda_batch_host_available(void);
int coli_wex_cuda_decode_batch_to_host(int n, const WexEntry *const *entries, const unsigned char *const *records,
                                       int device, unsigned char *const *dst, int *status);

#ifdef __cplusplus
}
#endif
#endif
