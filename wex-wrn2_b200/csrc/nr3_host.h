// Host side of the WNR2/WNR3 decoder: model registry with per-device lookup tables, record
// validation and launch planning. Shared by the helper ABI (helper_abi.cpp) and the WEX4 entry
// points (wex4_api.cpp).
#pragma once
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <vector>

#include "wex_entry.h"
#include "wnr3.cuh"

namespace wexb {

inline uint32_t rd32(const uint8_t *p) { return p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24; }
inline uint32_t rd16(const uint8_t *p) { return p[0] | (uint32_t)p[1] << 8; }
inline uint64_t rd64(const uint8_t *p) { return rd32(p) | (uint64_t)rd32(p + 4) << 32; }
inline size_t align_up(size_t v, size_t a) { return (v + a - 1) & ~(a - 1); }

constexpr uint32_t kMagicWnr2 = 0x32524e57u, kMagicWnr3 = 0x33524e57u, kMagicWnm2 = 0x324d4e57u;
constexpr int kMaxModels = 64, kMaxDevices = 64;   // the reference registry holds 16 models

// ---- WNM2 model registry (process-wide, never freed; c/tools/wex_cuda_bridge.cu:161-202) -------
// 0 and *id when blob is a valid WNM2 model (c/wex_neural_rans.h:258-274), else -1.
int model_validate(const uint8_t *blob, size_t bytes, uint32_t *id);
// 0 registered (or already, same bytes), -1 invalid or id collision, 1 registry full.
int model_register(const uint8_t *blob, size_t bytes);
bool model_registered(uint32_t id);
// Device tables of model `id` on `device` (the current device; kTableBytes, wnr3.cuh), built on first
// use: 0, or 1 when the model is not registered or CUDA failed.
int model_tables(uint32_t id, int device, const uint8_t **out);
// Host image (kTableBytes, the device table layout) of registered model `id`, or nullptr. Registered
// models are never freed, so the pointer stays valid.
const uint8_t *model_image(uint32_t id);

// ---- one validated record ---------------------------------------------------------------------
struct Plan {
    uint32_t nr3, flags, model_id, owner, word24, schunk, wchunk;
    uint32_t scount[3], wcount[3], soff[3], wout[3], sbase[3], wbase[3];
    uint32_t sstreams, wstreams, meta, total;
    uint32_t scale_bytes, weight_bytes, weight_at;   // weights at weight_at (16-aligned) in the decode layout
    uint64_t raw, scratch;                           // canonical slab bytes, decode-layout bytes
    uint32_t dst_bytes[6];                           // bytes of the six regions (scales m, weights m)
    const uint8_t *lengths;
    uint32_t streams() const { return sstreams + wstreams; }
};

// wex_entry_raw_sizes (c/wex_format.h:130-159): 0 and the raw / 4096-aligned sizes, else -1.
int entry_raw_sizes(const WexEntry *e, uint64_t *raw, uint64_t *aligned);
// Validates a codec-4/5 record of entry e (e->total_bytes at rec, host memory) and plans it; any model
// id is accepted (the caller resolves it). The checks are the reference's parse (c/wex_neural_rans.h:
// 287-337) behind its entry checks (c/wex_cuda.cuh:421-459). 0 or -1.
int plan_record(const WexEntry *e, const uint8_t *rec, Plan *p);
// Absolute record offsets of every stream, then the end: streams() + 1 words.
void plan_offsets(const Plan &p, uint32_t *off);
// Fills the device descriptor of a planned record: its record copy, stream offsets, decode layout,
// error word and commit job (null: the decode layout is the output) on the device.
void plan_descriptor(const Plan &p, const uint8_t *drec, const uint32_t *doff, uint8_t *dout, uint32_t *derr,
                     const CommitJob *djob, Nr3Record *out);

// ---- the work queue of a launch (wnr3.cuh) ------------------------------------------------------
// Items a record adds to a queue: its scale and weight items, and its commit items when `commit`.
uint32_t queue_items(const Plan &p, bool commit);
// Writes the queue of one launch over records 0 .. n-1 (their plans, all of one model) into items and
// returns how many. Record by record: its weight items, preceded by the scale items of the record
// `scale_lead` places later (the first scale_lead records' scale items open the queue; scale_lead >= n
// puts every scale item first, the order for records already in device memory, while a small lead
// suits records still being uploaded in order) and followed by the commit items of an earlier record
// (`delay` records back, about one wave of the device's warps); the commits still missing at the end.
uint32_t queue_fill(const Plan *const *plans, uint32_t n, bool commit, int sms, uint32_t scale_lead, Nr3Item *items);
// scale_lead for records already in device memory: every scale item first.
constexpr uint32_t kScalesFirst = 0xffffffffu;
// SMs of a device (cached), or 0 when CUDA fails.
int device_sms(int device);

// The launches of one call: its records grouped by model (equal tables contiguous in call order), one
// persistent launch per group. Counters: one head per group, then 4 words per record.
struct LaunchSet {
    struct Group { uint32_t first_rec, nrecs, first_item, nitems; const uint8_t *tables; };
    std::vector<Group> groups;
    uint32_t items = 0, records = 0;
    // Groups records [0, k) by their tables (already ordered so that equal tables are contiguous).
    void plan(const Plan *const *plans, const uint8_t *const *tables, uint32_t k, bool commit);
    size_t counter_words() const { return groups.size() + 4ull * records; }
    // Writes every group's queue (`items` entries; scale_lead as for queue_fill) and zeroes the counters
    // (counter_words()).
    void fill(const Plan *const *plans, bool commit, int sms, uint32_t scale_lead, Nr3Item *items_out,
              uint32_t *counters) const;
    // Launches every group on st over the device copies of the records, items and counters
    // (beside_hashes: the footprint that leaves room for record-hash CTAs, launch_nr3).
    bool launch(const Nr3Record *drecs, const Nr3Item *ditems, uint32_t *dcounters, int sms, cudaStream_t st,
                bool beside_hashes = false) const;
};
// Slack a record buffer keeps after each record: a stream's payload window may read up to 12 bytes
// past the stream's end (rans_device.cuh).
constexpr size_t kRecordSlack = 64;

// Reports an integrity failure once per process (c/tools/wex_cuda_bridge.cu:117-122).
void report_error_bits(uint32_t bits);
// The status of a record from its error word: 0 clean, -1 the record failed a check, 1 a bounded
// device wait gave up (kErrTimeout). A TMA copy may still have been in flight when that CTA returned,
// so the device is suspect and the record must be decoded again (status 1, "unavailable"), never
// reported as invalid data.
inline int status_of_bits(uint32_t bits) { return !bits ? 0 : (bits & kErrTimeout) ? 1 : -1; }
uint32_t last_error_bits();

// Queued batches (helper_abi.cpp): waits until the host records of ticket `t` (wexb_batch_submit) have
// been copied to the device, so their host memory may be reused before the wait for the decode. False
// for an unknown ticket or a CUDA error.
bool batch_uploads_wait(int t);

}  // namespace wexb
