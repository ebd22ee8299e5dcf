/* B200 additions to the helper ABI. None of these has a counterpart in the reference; they sit beside
 * the drop-in entry points of wex_cuda_helper.h and use the same status codes (0 ok, 1 unavailable,
 * -1 invalid) and the same fail-closed destinations.
 *
 * Resident records: an engine that keeps compressed experts in HBM uploads and validates them once
 * (wexb_resident_create) and then decodes any subset straight from device memory into its own
 * device buffers, asynchronously on its own stream (wexb_resident_decode + wexb_resident_wait).
 * Two decodes of a resident set may be queued at once, so the host plans the next one while the GPU
 * runs the previous one; a wait returns the oldest queued decode. */
#ifndef WEXB_WEXB200_H
#define WEXB_WEXB200_H
#include "wex_entry.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Library ABI of these additions. */
unsigned int wexb_abi(void);

/* Queued batches: the device-destination batch of wex_cuda_decode_batch_to_device
 * (the reference's c/tools/wex_cuda_bridge.cu:388-487) split into a submit that returns once the
 * uploads and kernels are queued and a wait that returns the statuses, so that a caller can keep
 * several batches in flight. Host records and destination pointers must stay valid until the wait.
 * Returns a ticket >= 0 (also when no record could be queued: the wait then reports why), -1 for
 * bad arguments, -3 when out of host memory. */
int wexb_batch_submit(int n, const WexEntry *const *entries, const unsigned char *const *records, int device,
                      unsigned char *const *dst_scale, unsigned char *const *dst_weight);
/* wexb_batch_submit with every record's stored bytes checked on the GPU against sha256[32 i .. 32 i + 32)
 * (the digest a WEX4 index keeps for the record, c/wex4.h:673-677) before its decode may write the
 * destination: a record whose bytes hash to anything else gets status -1 (error bit 32) and its
 * destination stays untouched. Verified calls of a device gather in windows of up to 64 records (or 16
 * calls): a window's hashes are one launch on one of the device's 24 hash streams once its records have
 * landed, and its calls' decodes follow them. A window is queued when it is full or when one of its calls
 * is waited for, so a call may start only at the wait. One SHA-256 chain per record: keep many calls in
 * flight (tens) so that hundreds of chains run at once, and run the process with
 * CUDA_DEVICE_MAX_CONNECTIONS=32 so that no stream waits behind another's hash launch. Wait with
 * wexb_batch_wait. Returns as wexb_batch_submit; -1 also when sha256 is NULL. */
int wexb_batch_submit_verified(int n, const WexEntry *const *entries, const unsigned char *const *records,
                               const unsigned char *sha256, int device, unsigned char *const *dst_scale,
                               unsigned char *const *dst_weight);
/* Wait for a ticket: status[i] as wex_cuda_decode_batch_to_device (0 ok, -1 invalid, 1 unavailable;
 * destinations untouched unless 0). Returns the number of non-zero statuses, -1 for an unknown or
 * already-waited ticket. status may be NULL. */
int wexb_batch_wait(int ticket, int *status);

typedef struct WexbResident WexbResident;

/* Validate n WNR2/WNR3 records (host memory) and copy them, with their stream offset tables, to
 * `device`. status[i]: 0 resident, -1 invalid, 1 unavailable (model not registered, CUDA error).
 * Resident record j is the j-th record whose status is 0. Returns the number of non-zero statuses;
 * *out is NULL only when no record could be kept. */
int wexb_resident_create(int n, const WexEntry *const *entries, const unsigned char *const *records, int device,
                         WexbResident **out, int *status);
/* Device bytes held by a resident set (records, offset tables). */
size_t wexb_resident_bytes(const WexbResident *r);
/* Queue the decode of resident records index[0 .. k) on `stream` (a cudaStream_t, NULL = the set's own
 * stream): record index[j]'s matrix m goes to dst_scale[3j + m] / dst_weight[3j + m] (device), each
 * written only if that record decoded cleanly. With two decodes already queued, the oldest is waited
 * for first and its statuses are dropped. Returns 0 queued, -1 bad arguments (nothing queued), 1 CUDA
 * error. */
int wexb_resident_decode(WexbResident *r, int k, const int *index, unsigned char *const *dst_scale,
                         unsigned char *const *dst_weight, void *stream);
/* Wait for the oldest queued decode; status[j] of its record index[j]: 0 written, -1 failed its checks
 * (destination untouched), 1 CUDA error. Returns the number of non-zero statuses, -1 when nothing is
 * queued. */
int wexb_resident_wait(WexbResident *r, int *status);
/* 1: bracket each kernel of the following decodes with CUDA events on its stream; 0: stop. Returns 0
 * (a decode returns 1 when its events cannot be created). */
int wexb_resident_profile(WexbResident *r, int on);
/* Milliseconds of the last waited decode (profiling on), on its stream: ms3[0] the upload of its launch
 * metadata, ms3[1] the decode launch (scale, weight and commit work of every record), ms3[2] the
 * read-back of the error words. 0, or -1 when there is nothing to report. */
int wexb_resident_kernel_ms(const WexbResident *r, float *ms3);
/* Kernel launches of the last queued decode: one persistent launch per model among its records. */
int wexb_resident_launches(const WexbResident *r);
void wexb_resident_destroy(WexbResident *r);

/* No counterpart in the reference. wex_cuda_decode_to_device for callers that may not allocate device
 * memory at run time (an engine that reserves all of HBM in its own pool at start-up, or whose serving
 * streams must not stall on the device synchronisation cudaMalloc / cudaFree can cause): it calls no
 * cudaMalloc, cudaFree or other allocating routine and works in a fixed ~50 MiB device array defined
 * in the library, held by every device that loads the library until the process exits. Limits:
 * records of at most 24 MiB stored and 24 MiB decoded and 32,768 streams (larger ones return -2 with
 * a message on stderr), at most 4 models per device (a fifth returns 1). The first call on a device
 * sets that device up (looks up the array's address, creates the stream its calls run on) and the first
 * call with a model on a device copies that model's tables into the array; both synchronise with the
 * device and should come before any stream capture there. Calls are synchronous and serialised by a
 * process-wide lock; calls that overlapped on the GPU would race on the shared array. The wait for the
 * decode is bounded (wexb_set_wait_limit): after a wait that gave up, calls on that device return 1
 * until the decode still using the array has ended. The caller's current device is restored. Returns
 * 0, -1 invalid (destination untouched), 1 unavailable, -2 too large. */
int wexb_decode_to_device_noalloc(const WexEntry *entry, const unsigned char *record, int device,
                                  unsigned char *const *dst_scale, unsigned char *const *dst_weight);

/* Self-test of the bounded waits. Every kernel waits on its shared-memory mbarriers for at most a fixed
 * number of polls (2^24), then sets error bit 16 in the record's error word and returns: it never spins
 * forever. This runs the same wait, limited to `polls` polls (1 .. 2^24; more is refused with -1), on a
 * barrier that completes and on one that nothing arrives on; *bits receives the second one's error bits
 * (16). The host waits for the probe under the library's wait limit (wexb_set_wait_limit). Returns 0
 * when the first completes and the second gives up, -1 otherwise or for bad arguments, 1 when CUDA is
 * unavailable, when the host's wait gave up before the probe ended (the probe then ends on its own),
 * or while the previous probe on that device is still running. */
int wexb_selftest_bounded_wait(int device, unsigned int polls, unsigned int *bits);

/* Host waits. No entry point of this library blocks on the GPU without a limit: each polls its CUDA
 * event or stream until the work ends or `seconds` pass (default 60, or WEXB_WAIT_SECONDS at load),
 * and a call whose wait gave up returns status 1 ("unavailable, decode again") for the records it had
 * queued. Their GPU work may still be running: the buffers it uses are not handed to another call
 * until it ends, and a device destination may still be written afterwards by that work's error-gated
 * commit (with correct bytes only). Returns 0, or -1 for a limit outside (0, 86400]. */
int wexb_set_wait_limit(double seconds);
double wexb_wait_limit(void);

/* Error bits of the last failed record seen by this process (1 structure, 2 stream hash, 4 ceil form
 * at scale 0, 8 canonical zero, 16 bounded wait expired, 32 record SHA-256 of a verified batch); 0 if
 * none failed. */
unsigned int wexb_last_error_bits(void);

/* Expert records read from a WEX4 container file: the step before the upload. The reference's expert
 * store reads each record with one pread (O_DIRECT where it can) into a pageable slab and decodes it
 * there (c/expert_store_wex.c:92-121, :305-337; its read paths are timed by bench/wex_io.c). Here the
 * reads run on a pool of reader threads, in page-aligned pieces of at most 2 MiB, into a ring of
 * page-locked buffers of 8 records each; each batch is uploaded and decoded (wexb_batch_submit) while
 * the next ones are read. A WexbFile serves one call at a time. */
typedef struct WexbFile WexbFile;
#define WEXB_FILE_DIRECT 1u   /* open with O_DIRECT: reads bypass the page cache */

/* Opens `path`: reads and validates the header page and the index (the WEX4 rules of wex4_validate),
 * reads every WNM2 model blob, checks it against its SHA-256 and registers it (wex_cuda_register_model).
 * readers: reader threads, 0 = 8, at most 64. Returns 0 and *out; -1 for bad arguments or a container
 * that fails validation; 1 when the file cannot be opened or read (with WEXB_FILE_DIRECT: also when
 * the filesystem refuses O_DIRECT) or memory runs out. */
int wexb_file_open(const char *path, unsigned int flags, int readers, WexbFile **out);
/* The expert grid of the header, the number of expert records, the largest stored record (page-aligned). */
int wexb_file_info(const WexbFile *f, unsigned int *layers, unsigned int *experts, unsigned int *records,
                   unsigned long long *max_stored);
/* Drops the file's pages from the page cache (POSIX_FADV_DONTNEED): 0, or 1 if refused. */
int wexb_file_evict(WexbFile *f);
/* Reads the stored records of experts (layer[i], expert[i]) through the ring and discards them: the
 * read stage alone. check != 0: each record's SHA-256 is checked against the index on the host.
 * status[i]: 0 read, -1 no such expert or (check) a SHA-256 mismatch, 1 the read failed. *bytes (may
 * be NULL): stored bytes read. Returns the number of non-zero statuses, -1 for bad arguments. */
int wexb_file_read(WexbFile *f, int n, const unsigned int *layer, const unsigned int *expert, int check,
                   int *status, unsigned long long *bytes);
/* Reads, uploads and decodes experts (layer[i], expert[i]) into device buffers, as
 * wex_cuda_decode_batch_to_device does from host memory: dst_scale[3i + m] and dst_weight[3i + m] for
 * matrix m, written only when status[i] is 0. WNR3 records are decoded on `device`; RAW records are
 * copied region by region. status[i]: 0 ok; -1 no such expert, or a record that fails its checks (the
 * record header against the index, the decode's own checks); 1 unavailable (read failed, model not
 * registered, CUDA error: the caller may try again). Returns the number of non-zero statuses, -1 for
 * bad arguments. */
int wexb_file_decode(WexbFile *f, int device, int n, const unsigned int *layer, const unsigned int *expert,
                     unsigned char *const *dst_scale, unsigned char *const *dst_weight, int *status);
void wexb_file_close(WexbFile *f);

/* The writer side on the GPU. The reference writes records on the CPU, one at a time
 * (c/tools/wex_nr3_tools.c:87-120 -> wex_nr3_encode, c/wex_neural_rans.h:615-749), after counting
 * its training experts (c/wex_neural_rans.h:579-613). These run every stream of every record of a call
 * at once and give the same bytes.
 *
 * Encodes n coded experts (the canonical-zero / ceil-form domain: canonical slab layout of entries[i],
 * in host memory) as WNR3 records (nr3 = 1; flags[i] = the record flags, owners[i] = layer << 16 |
 * expert) or WNR2 records (nr3 = 0; flags and owners 0) with the chunk pair wchunk:schunk under the
 * WNM2 model `blob`. status[i]: 0 encoded (out[i] holds total[i] bytes: used[i] bytes of record, then
 * zero padding to 4096); 1 the record would not be smaller than the 4096-aligned raw slab (the writer
 * stores the expert RAW; out[i] untouched, used / total still given); -1 invalid (entry layout, chunk
 * sizes, flags, a -0 nibble in a canonical-zero record, a record larger than cap[i]); -2 CUDA
 * unavailable. Returns the number of non-zero statuses, -1 for bad arguments. */
int wexb_encode_batch(int n, const WexEntry *const *entries, const unsigned char *const *coded,
                      const unsigned int *flags, const unsigned int *owners, int nr3, unsigned int wchunk,
                      unsigned int schunk, const unsigned char *blob, size_t blob_bytes, int device,
                      unsigned char *const *out, const size_t *cap, size_t *used, size_t *total, int *status);
/* Adds the training counts of n coded experts to wc[3][567][16] (weight symbols per matrix and
 * context) and sc[3][256] (scale values per matrix), contexts taken against the rule-g anchors (nr3 =
 * 1) or the lower medians (nr3 = 0). status[i]: 0 counted, -1 invalid entry, -2 CUDA unavailable (then
 * nothing is added). Returns the number of non-zero statuses, -1 for bad arguments. */
int wexb_count_batch(int n, const WexEntry *const *entries, const unsigned char *const *coded, int nr3, int device,
                     unsigned long long *wc, unsigned long long *sc, int *status);

#ifdef __cplusplus
}
#endif
#endif
