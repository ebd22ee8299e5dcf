/* The WNR4 CUDA helper ABI 5 of the reference (wnr4/tools/wnr4_cuda_bridge.cu:160-361), kind MX
 * (MXFP4 experts). geo = u32[13]: kind, scount[3], scols[3], soff[3], woff[3] (wnr4_geo, wnr4/wnr4.h:108-140).
 * Records are decoded straight into the destinations (device; weights 16-byte aligned), as the
 * reference does: a failed record's destination may hold partial data (status != 0: do not use it).
 * Every call leaves the caller's current device as it found it. Kinds NV (NVFP4) and GG (GGUF slices)
 * are not built: their models and batches are refused (-1 / WNR4_E_ARGS). */
#ifndef WEXB_WNR4_CUDA_H
#define WEXB_WNR4_CUDA_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define WNR4_CUDA_SLOTS 4      /* batches in flight per calling thread and device */
#define WNR4_E_ARGS (-1)       /* submit: bad arguments or geometry */
#define WNR4_E_MODEL (-2)      /* submit: model not registered on that device */
#define WNR4_E_CUDA (-3)       /* submit: CUDA or memory error, nothing queued */
#define WNR4_E_BUSY (-4)       /* submit: the next slot holds a batch not yet waited for */

/* 5 (wnr4/tools/wnr4_cuda_bridge.cu:160) */
unsigned int wnr4_cuda_abi(void);
/* Validate a WNM4 blob (kind MX) and upload its tables to `device`: 0 ok (also when already
 * registered), -1 invalid blob, 1 CUDA error (wnr4/tools/wnr4_cuda_bridge.cu:162-184). */
int wnr4_cuda_register_model(const unsigned char *blob, size_t bytes, int device);
/* Queue n records of one geometry (page-locked host memory; records[i] holds totals[i] bytes) for
 * decoding into dst_scale[3i + m] / dst_weight[3i + m] on `stream` (a cudaStream_t, NULL = the slot's
 * own non-blocking stream). A ticket >= 0, or WNR4_E_ARGS / _MODEL / _CUDA / _BUSY
 * (wnr4/tools/wnr4_cuda_bridge.cu:186-236). */
int wnr4_cuda_batch_submit(int n, const uint32_t *geo, const unsigned char *const *records, const size_t *totals,
                           const uint32_t *owners, uint32_t model_id, int device, unsigned char *const *dst_scale,
                           unsigned char *const *dst_weight, void *stream);
/* Wait for a ticket (on the thread that submitted it): status[i] 0 decoded, -1 invalid or failed an
 * integrity check, 1 CUDA error; the number of non-zero statuses, or -1 for an unknown ticket
 * (wnr4/tools/wnr4_cuda_bridge.cu:238-251). */
int wnr4_cuda_batch_wait(int ticket, int *status);
/* Synchronous submit + wait (wnr4/tools/wnr4_cuda_bridge.cu:253-270). */
int wnr4_cuda_decode_batch(int n, const uint32_t *geo, const unsigned char *const *records, const size_t *totals,
                           const uint32_t *owners, uint32_t model_id, int device, unsigned char *const *dst_scale,
                           unsigned char *const *dst_weight, int *status);
/* Free this thread's slots on every device, after waiting for their batches (:361). */
void wnr4_cuda_release_thread(void);
/* Kind GG is not built: -1 (invalid blob) / WNR4_E_ARGS / every status -1 (:273-359). */
int wnr4_cuda_gg_register_model(const unsigned char *blob, size_t bytes, int device, uint32_t *id);
int wnr4_cuda_gg_batch_submit(int n, uint32_t nseg, const uint32_t *types, const uint32_t *bytes,
                              const unsigned char *const *records, const size_t *totals, const uint32_t *owners,
                              uint32_t model_id, int device, unsigned char *const *dst, void *stream);
int wnr4_cuda_gg_decode_batch(int n, uint32_t nseg, const uint32_t *types, const uint32_t *bytes,
                              const unsigned char *const *records, const size_t *totals, const uint32_t *owners,
                              uint32_t model_id, int device, unsigned char *const *dst, int *status);

#ifdef __cplusplus
}
#endif
#endif
