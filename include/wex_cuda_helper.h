/* The CUDA helper C ABI: a drop-in for the reference's kaira_wex_cuda helper library
 * (c/tools/wex_cuda_bridge.cu), resolved by name by the engine glue (c/wex_decode.c:69-102).
 * Every function keeps the reference's signature, return codes and guarantees:
 *   0 ok, 1 unavailable (CUDA, resources, model not registered), -1 invalid input;
 *   batch calls write status[i] and return the number of non-zero statuses;
 *   _to_device and _batch_to_device write the destination only after a clean decode;
 *   every call is synchronous (all copies and kernels completed on return, under the bounded host
 *   wait of wexb200.h: a wait that gives up returns 1), thread-safe, and leaves `device` current (as
 *   the reference does).
 * Records are host memory (page-locked for full speed). WNR2 (codec 4) and WNR3 (codec 5) records
 * are decoded on the GPU; WNR1 (codec 3) returns 1 (unavailable: legacy codec, not built). */
#ifndef WEXB_WEX_CUDA_HELPER_H
#define WEXB_WEX_CUDA_HELPER_H
#include "wex_entry.h"

#ifdef __cplusplus
extern "C" {
#endif

#define WEX_CUDA_FEATURE_DEVICE 1u
#define WEX_CUDA_FEATURE_REGISTER 2u
#define WEX_CUDA_FEATURE_NR2 4u
#define WEX_CUDA_FEATURE_BATCH 8u
#define WEX_CUDA_FEATURE_NR3 16u
#define WEX_CUDA_FEATURE_BATCH_HOST 32u

/* 1 (c/tools/wex_cuda_bridge.cu:325) */
unsigned int wex_cuda_helper_abi(void);
/* 63: every feature bit above (c/tools/wex_cuda_bridge.cu:370-373) */
unsigned int wex_cuda_helper_features(void);
/* Register a WNM2 model blob (59,408 B; process-wide, kept until exit): 0 registered or already
 * registered with the same bytes, -1 invalid or another blob with the same id, 1 registry full
 * (64 models here; the reference holds 16) (c/tools/wex_cuda_bridge.cu:213-243). */
int wex_cuda_register_model(const unsigned char *blob, size_t bytes);
/* Decode the record at slab + read offset (entry->total_bytes, in the tail of the slab) into the
 * canonical slab at slab[0 .. scale_bytes + weight_bytes); the slab is untouched unless it returns
 * 0 (c/tools/wex_cuda_bridge.cu:327-362). */
int wex_cuda_decode_to_host(const WexEntry *entry, unsigned char *slab, size_t slab_capacity);
/* Decode one record (host memory) into caller-owned device buffers dst_scale[m] / dst_weight[m] on
 * `device` (c/tools/wex_cuda_bridge.cu:414-454). */
int wex_cuda_decode_to_device(const WexEntry *entry, const unsigned char *record, int device,
                              unsigned char *const *dst_scale, unsigned char *const *dst_weight);
/* n records; record i's matrix m to dst_scale[3i + m] / dst_weight[3i + m]; status[i] 0 written,
 * -1 invalid (untouched), 1 unavailable (untouched or correct) (c/tools/wex_cuda_bridge.cu:608-613). */
int wex_cuda_decode_batch_to_device(int n, const WexEntry *const *entries, const unsigned char *const *records,
                                    int device, unsigned char *const *dst_scale, unsigned char *const *dst_weight,
                                    int *status);
/* n records decoded into host buffers dst[i] (canonical slab; dst[i] may overlap record i itself,
 * never another record); on a non-zero status dst[i] may be partially written
 * (c/tools/wex_cuda_bridge.cu:628-633). */
int wex_cuda_decode_batch_to_host(int n, const WexEntry *const *entries, const unsigned char *const *records,
                                  int device, unsigned char *const *dst, int *status);
/* Page-lock / release a caller staging buffer (portable): 0, 1 CUDA error, -1 bad arguments
 * (c/tools/wex_cuda_bridge.cu:635-644). */
int wex_cuda_host_register(void *pointer, size_t bytes);
int wex_cuda_host_unregister(void *pointer);

#ifdef __cplusplus
}
#endif
#endif
