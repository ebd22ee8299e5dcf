// The CUDA helper C ABI (include/wex_cuda_helper.h) and the resident-record additions
// (include/wexb200.h), over the sm_100a WNR2/WNR3 kernels.
//
// One call = a pooled workspace (grown buffers, three events, upload flags) on the device's shared
// streams: each record is parsed and its upload queued at once (upload stream, call order, a flag word
// after each record); the launch metadata (record descriptors, work queue, commit jobs, error words,
// stream offsets) follows in one copy on the metadata stream; one persistent decode launch per model
// and the read-back of the error words run on the call's kernel stream, the records decoding as their
// flags land. Queued calls therefore overlap one call's decode with its own later uploads and the next
// call's. A record's destinations are written by the launch's error-gated commit items (device
// destinations), or copied back after it (host destinations). Verified calls add a hash window
// (window_flush below).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <utility>
#include <vector>

#include "bufs.h"
#include "container.cuh"
#include "host_wait.h"
#include "nr3_host.h"
#include "sha256.cuh"
#include "wex_cuda_helper.h"
#include "workspace.h"
#include "wexb200.h"

#define WEXB_API extern "C" __attribute__((visibility("default")))

namespace wexb {
namespace {

// Byte layout of a call's metadata block (host pinned, copied to the device in one piece): record
// descriptors, the work queue, its counters, commit jobs, error words, stream offsets.
struct MetaLayout {
    size_t recs = 0, items = 0, counters = 0, jobs = 0, errs = 0, offs = 0, digests = 0, msgs = 0, total = 0;
    // nhash: records whose SHA-256 is checked (their expected digests and hash jobs)
    void compute(size_t k, size_t nitems, size_t ncounters, size_t njobs, size_t noffs, size_t nhash = 0) {
        size_t at = 0;
        recs = at; at = align_up(at + k * sizeof(Nr3Record), 256);
        items = at; at = align_up(at + nitems * sizeof(Nr3Item), 256);
        counters = at; at = align_up(at + ncounters * 4, 256);
        jobs = at; at = align_up(at + njobs * sizeof(CommitJob), 256);
        errs = at; at = align_up(at + k * 4, 256);
        offs = at; at = align_up(at + noffs * 4, 256);
        digests = at; at = align_up(at + nhash * 32, 256);
        msgs = at; at = align_up(at + nhash * sizeof(ShaMsg), 256);
        total = at;
    }
};

enum class Dest { Device, Host, HostChecked };
constexpr int kPending = 2;

// One batch call between its submit and its finish.
struct Call {
    int n = 0, device = -1;
    Dest mode = Dest::Device;
    unsigned char *const *dst_host = nullptr;
    std::vector<Plan> plans;
    std::vector<int> status, pend;
    std::vector<size_t> scr_off;
    Workspace *w = nullptr;
    size_t k = 0, broken_at = 0;
    bool unsettled = false;   // a bounded wait during submit gave up: the workspace may still be in use
    MetaLayout L;
    // queued after the uploads by launch_rest(): at once, or for a verified call once its window's
    // record hashes are queued
    LaunchSet launches;
    cudaStream_t up = nullptr, st = nullptr, ms = nullptr;
    int sms = 0;
    bool ok = false, queued_meta = false, verify = false, launched = false;
    int failures() const { int bad = 0; for (int v : status) bad += v != 0; return bad; }
    void settle(int v) { for (int &s : status) if (s == kPending) s = v; }
};

// The part of a call queued after its uploads and metadata: the decode launch (behind the record
// hashes of a verified call: `hashed`, recorded on hs after them; hash_ok: they were queued), the
// read-back of the error words and the call's `done` event.
void launch_rest(Call &c, cudaEvent_t hashed, cudaStream_t hs, bool hash_ok) {
    Workspace *w = c.w;
    const MetaLayout &L = c.L;
    uint8_t *dm = w->dmeta.p;
    const size_t k = c.k;
    cudaStream_t st = c.st;
    bool ok = c.ok && (!c.verify || hash_ok);
    if (ok)
        ok = cudaStreamWaitEvent(st, c.verify ? hashed : w->meta_done, 0) == cudaSuccess &&
             c.launches.launch(reinterpret_cast<const Nr3Record *>(dm + L.recs), reinterpret_cast<const Nr3Item *>(dm + L.items),
                               reinterpret_cast<uint32_t *>(dm + L.counters), c.sms, st, c.verify);
    // the read-back and `done` come after every upload (records, flags, metadata) and every hash
    if (cudaStreamWaitEvent(st, w->uploads_done, 0) != cudaSuccess ||
        (c.queued_meta && cudaStreamWaitEvent(st, w->meta_done, 0) != cudaSuccess) ||
        (hashed && cudaStreamWaitEvent(st, hashed, 0) != cudaSuccess)) {
        (void)cudaGetLastError();
        if (wait_stream(c.up) == Waited::TimedOut || wait_stream(c.ms) == Waited::TimedOut ||
            (hs && wait_stream(hs) == Waited::TimedOut))
            c.unsettled = true;
        ok = false;
    }
    for (size_t j = 0; ok && c.mode == Dest::Host && j < k; ++j) {
        const int i = c.pend[j];
        const Plan &p = c.plans[(size_t)i];
        const uint8_t *scr = w->dscratch.p + c.scr_off[j];
        ok = cudaMemcpyAsync(c.dst_host[i], scr, p.scale_bytes, cudaMemcpyDeviceToHost, st) == cudaSuccess &&
             cudaMemcpyAsync(c.dst_host[i] + p.scale_bytes, scr + p.weight_at, p.weight_bytes, cudaMemcpyDeviceToHost,
                             st) == cudaSuccess;
    }
    c.broken_at = ok ? k : 0;
    if (!ok) (void)cudaGetLastError();
    uint32_t *herrs = reinterpret_cast<uint32_t *>(w->hmeta.p + L.errs);
    const uint32_t *derrs = reinterpret_cast<const uint32_t *>(dm + L.errs);
    if (!c.queued_meta || cudaMemcpyAsync(herrs, derrs, k * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaEventRecord(w->done, st) != cudaSuccess) {
        (void)cudaGetLastError();
        if (cudaEventRecord(w->done, st) != cudaSuccess) {   // `done` must still cover the queued copies
            (void)cudaGetLastError();
            c.unsettled = true;
        }
        if (wait_stream(st) == Waited::TimedOut) c.unsettled = true;
        c.broken_at = 0;
    }
    c.launched = true;
}

// ---- hash windows of verified calls --------------------------------------------------------------
// A record's SHA-256 is one serial chain, so a verified stream needs hundreds of records hashing at
// once. The verified calls of a device therefore gather in a window (up to kWindowRecords records or
// kShaParts calls) whose hashes are one launch on the next of the device's hash lanes, behind the
// uploads of all its calls; each call's decode then waits for that launch. A window is flushed when it
// is full, or when one of its calls is waited for. Few long launches on few streams keep the hash
// launches apart from the upload, metadata and kernel streams.
constexpr uint32_t kWindowRecords = 64;
std::mutex g_window_mu;
struct Window { std::vector<Call *> calls; uint32_t records = 0; };
Window g_window[kMaxDevices];

// (g_window_mu held) Queues the window's hashes and the rest of each of its calls.
void window_flush(int device) {
    Window &win = g_window[device];
    if (win.calls.empty()) return;
    KeepDevice keep;
    (void)cudaSetDevice(device);
    ShaParts P{};
    uint32_t total = 0;
    for (Call *c : win.calls)
        if (c->ok) {
            total += (uint32_t)c->k;
            P.part[P.nparts] = reinterpret_cast<const ShaMsg *>(c->w->dmeta.p + c->L.msgs);
            P.end[P.nparts++] = total;
        }
    cudaStream_t hs = nullptr;
    cudaEvent_t hashed = nullptr;
    bool hash_ok = false;
    if (P.nparts && hash_lane(device, &hs, &hashed)) {
        bool ok = true;
        for (Call *c : win.calls)
            if (c->ok)
                ok = ok && cudaStreamWaitEvent(hs, c->w->uploads_done, 0) == cudaSuccess &&
                     cudaStreamWaitEvent(hs, c->w->meta_done, 0) == cudaSuccess;
        ok = ok && launch_sha256_parts(P, hs) == cudaSuccess;
        if (cudaEventRecord(hashed, hs) != cudaSuccess) {   // nothing can wait for the hashes: wait here (bounded)
            (void)cudaGetLastError();
            const bool gave_up = wait_stream(hs) == Waited::TimedOut;
            for (Call *c : win.calls) c->unsettled = c->unsettled || gave_up;
            hashed = nullptr;
            ok = false;
        }
        hash_ok = ok;
    }
    if (!hash_ok) (void)cudaGetLastError();
    for (Call *c : win.calls) launch_rest(*c, hashed, hs, hash_ok);
    win.calls.clear();
    win.records = 0;
}

void window_add(Call &c) {
    std::lock_guard<std::mutex> lock(g_window_mu);
    Window &win = g_window[c.device];
    win.calls.push_back(&c);
    win.records += (uint32_t)c.k;
    if (win.records >= kWindowRecords || win.calls.size() >= (size_t)kShaParts) window_flush(c.device);
}

// Before a wait: a verified call still in its window is queued now.
void ensure_launched(Call &c) {
    if (!c.w) return;
    std::lock_guard<std::mutex> lock(g_window_mu);   // `launched` is written under this lock
    if (!c.launched) window_flush(c.device);
}

// Validates n records (host memory) and queues their pipeline: dst_scale / dst_weight (Device) or
// dst_host (Host: copied back after the kernels; HostChecked: copied back by finish() only after a
// clean decode). Argument and status rules of the reference batch (c/tools/wex_cuda_bridge.cu:388-487).
// expect (verified calls, device destinations): 32 bytes per record, the SHA-256 its stored bytes must
// have; the hashes run on the GPU before the decode, and a record that differs is refused (-1) with its
// destination untouched. False when nothing could be queued (c.status then final).
//
// Each record's upload is queued as soon as that record is validated, so the copy engine starts on
// the first record while the host still parses the others; the launch metadata (built once every
// record is planned) goes up on the device's metadata stream, beside the record copies.
bool submit(Call &c, int n, const WexEntry *const *entries, const unsigned char *const *records, int device,
            unsigned char *const *dst_scale, unsigned char *const *dst_weight, unsigned char *const *dst_host, Dest mode,
            const uint8_t *expect = nullptr) {
    const bool host_dst = mode != Dest::Device;
    c.n = n; c.device = device; c.mode = mode; c.dst_host = dst_host;
    c.plans.assign((size_t)n, Plan{});
    c.status.assign((size_t)n, -1);
    // argument checks only; each record is parsed just before its upload
    std::vector<int> cand;
    size_t rec_cap = 0, scr_cap = 0;
    for (int i = 0; i < n; ++i) {
        const WexEntry *e = entries[i];
        if (!e || !records[i]) continue;
        bool targets = host_dst ? dst_host[i] != nullptr : true;
        if (!host_dst) for (int m = 0; m < 3; ++m) if (!dst_scale[3 * i + m] || !dst_weight[3 * i + m]) targets = false;
        uint64_t raw, aligned;
        if (!targets || entry_raw_sizes(e, &raw, &aligned) || e->total_bytes >= aligned) continue;   // -1 as parsed
        cand.push_back(i);
        rec_cap += align_up((size_t)e->total_bytes + kRecordSlack, 256);
        scr_cap += align_up((size_t)raw + 16, 256);   // decode layout: scales, then weights 16-aligned
    }
    if (cand.empty()) return false;
    // the device side: streams, a workspace, its token (every failure: valid records report 1)
    const bool commit = mode == Dest::Device;
    const bool verify = expect != nullptr && commit;
    cudaStream_t up = nullptr, st = nullptr, ms = nullptr;
    Workspace *w = nullptr;
    int sms = 0;
    uint32_t token = 0;
    if (device >= 0 && device < kMaxDevices && cudaSetDevice(device) == cudaSuccess && device_streams(device, &up, &st, &ms) &&
        (sms = device_sms(device)) > 0 && (w = workspace_take(device)) != nullptr)
        token = w->drec.grow(rec_cap) && w->dscratch.grow(scr_cap) ? w->take_token(cand.size(), ms) : 0u;
    if (!token) {
        (void)cudaGetLastError();
        if (w) workspace_give(w, true);
        for (int i : cand) if (!plan_record(entries[i], records[i], &c.plans[(size_t)i])) c.status[(size_t)i] = 1;
        return false;
    }
    c.w = w;
    // plan and upload record by record (call order). A flag word follows the records at least every
    // kFlagBytes (and after the last): a 4-byte copy costs the copy engine about as much as several
    // microseconds of record bytes, so small records share a flag (a record's flag is the first one after
    // its bytes)
    constexpr size_t kFlagBytes = 8u << 20;
    uint32_t *dflags = reinterpret_cast<uint32_t *>(w->dflags.p);
    const uint32_t *htoken = reinterpret_cast<const uint32_t *>(w->htoken.p);
    std::vector<const uint8_t *> tabs_of((size_t)n, nullptr);
    std::vector<size_t> rec_off((size_t)n, 0);
    std::vector<uint32_t> flag_of((size_t)n, 0);
    bool ok = true;
    size_t rec_bytes = 0, since_flag = 0;
    uint32_t flags = 0;
    std::vector<int> unflagged;
    auto flag_now = [&]() {
        for (int r : unflagged) flag_of[(size_t)r] = flags;
        ok = ok && cudaMemcpyAsync(dflags + flags, htoken, 4, cudaMemcpyHostToDevice, up) == cudaSuccess;
        ++flags;
        unflagged.clear();
        since_flag = 0;
    };
    for (int i : cand) {
        Plan &p = c.plans[(size_t)i];
        if (plan_record(entries[i], records[i], &p)) continue;
        if (!model_registered(p.model_id) || model_tables(p.model_id, device, &tabs_of[(size_t)i])) {
            c.status[(size_t)i] = 1;
            continue;
        }
        c.status[(size_t)i] = kPending;
        c.pend.push_back(i);
        rec_off[(size_t)i] = rec_bytes;
        rec_bytes += align_up(p.total + kRecordSlack, 256);
        ok = ok && cudaMemcpyAsync(w->drec.p + rec_off[(size_t)i], records[i], p.total, cudaMemcpyHostToDevice, up) == cudaSuccess;
        unflagged.push_back(i);
        since_flag += p.total;
        if (since_flag >= kFlagBytes) flag_now();
    }
    if (!unflagged.empty()) flag_now();
    if (cudaEventRecord(w->uploads_done, up) != cudaSuccess) {
        (void)cudaGetLastError();
        if (!c.pend.empty() && wait_stream(up) == Waited::TimedOut) c.unsettled = true;
        ok = false;
    }
    if (c.pend.empty()) {   // nothing was queued
        c.w = nullptr;
        workspace_give(w, !c.unsettled);
        return false;
    }
    // one launch per model: the records of a model contiguous (call order otherwise)
    std::stable_sort(c.pend.begin(), c.pend.end(), [&](int a, int b) { return tabs_of[(size_t)a] < tabs_of[(size_t)b]; });
    const size_t k = c.k = c.pend.size();
    std::vector<size_t> off_off(k);
    std::vector<const Plan *> plans(k);
    std::vector<const uint8_t *> tabs(k);
    c.scr_off.assign(k, 0);
    size_t scr_bytes = 0, noffs = 0;
    for (size_t j = 0; j < k; ++j) {
        const Plan &p = c.plans[(size_t)c.pend[j]];
        plans[j] = &p;
        tabs[j] = tabs_of[(size_t)c.pend[j]];
        c.scr_off[j] = scr_bytes; scr_bytes += align_up(p.scratch, 256);
        off_off[j] = noffs; noffs += p.streams() + 1;
    }
    LaunchSet launches;
    launches.plan(plans.data(), tabs.data(), (uint32_t)k, commit);
    MetaLayout &L = c.L;
    L.compute(k, launches.items, launches.counter_words(), commit ? k : 0, noffs, verify ? k : 0);
    // (the scratch was grown for the entries' raw sizes before the uploads; a plan's scratch is that
    // raw size rounded up to 16, so this grow does not reallocate)
    ok = ok && w->dscratch.grow(scr_bytes) && w->dmeta.grow(L.total) && w->hmeta.grow(L.total);
    uint8_t *hm = w->hmeta.p, *dm = w->dmeta.p;
    Nr3Record *hrecs = reinterpret_cast<Nr3Record *>(hm + L.recs);
    CommitJob *hjobs = reinterpret_cast<CommitJob *>(hm + L.jobs);
    uint32_t *herrs = reinterpret_cast<uint32_t *>(hm + L.errs);
    uint32_t *hoffs = reinterpret_cast<uint32_t *>(hm + L.offs);
    const CommitJob *djobs = reinterpret_cast<const CommitJob *>(dm + L.jobs);
    uint32_t *derrs = reinterpret_cast<uint32_t *>(dm + L.errs);
    if (ok) {
        // records are decoded as their uploads land (one record's scale items ahead of the weight items)
        launches.fill(plans.data(), commit, sms, 1, reinterpret_cast<Nr3Item *>(hm + L.items),
                      reinterpret_cast<uint32_t *>(hm + L.counters));
        for (size_t j = 0; j < k; ++j) {
            const int i = c.pend[j];
            const Plan &p = c.plans[(size_t)i];
            uint8_t *scr = w->dscratch.p + c.scr_off[j];
            plan_offsets(p, hoffs + off_off[j]);
            plan_descriptor(p, w->drec.p + rec_off[(size_t)i], reinterpret_cast<const uint32_t *>(dm + L.offs) + off_off[j],
                            scr, derrs + j, commit ? djobs + j : nullptr, &hrecs[j]);
            hrecs[j].landed = dflags + flag_of[(size_t)i];
            hrecs[j].landed_at = token;
            herrs[j] = 0;
            if (verify) {   // the record's SHA-256 against the expected digest; a difference ORs kErrRecordSha
                std::memcpy(hm + L.digests + 32 * j, expect + 32 * (size_t)i, 32);
                reinterpret_cast<ShaMsg *>(hm + L.msgs)[j] = {w->drec.p + rec_off[(size_t)i], p.total, nullptr,
                                                              dm + L.digests + 32 * j, derrs + j, kErrRecordSha};
            }
            if (commit) {
                CommitJob &J = hjobs[j];
                for (int m = 0; m < 3; ++m) {
                    J.src[m] = scr + p.soff[m]; J.dst[m] = dst_scale[3 * i + m]; J.bytes[m] = p.dst_bytes[m];
                    J.src[3 + m] = scr + p.wout[m]; J.dst[3 + m] = dst_weight[3 * i + m]; J.bytes[3 + m] = p.dst_bytes[3 + m];
                }
            }
        }
        // metadata stream: the whole block in one copy. Kernel stream: once it is there, one persistent
        // launch per model, whose scale items wait for each record's flag, so the records decode as
        // they land; then, after every upload, the read-back of the error words (`done`, recorded
        // last, covers the whole call)
        ok = cudaMemcpyAsync(dm, hm, L.total, cudaMemcpyHostToDevice, ms) == cudaSuccess &&
             cudaEventRecord(w->meta_done, ms) == cudaSuccess;
    }
    c.launches = std::move(launches);
    c.up = up; c.st = st; c.ms = ms; c.sms = sms;
    c.ok = ok; c.queued_meta = ok; c.verify = verify;
    if (verify) window_add(c);   // its decode is queued once its window's record hashes are
    else launch_rest(c, nullptr, nullptr, false);
    return true;
}

// Waits (bounded) for a submitted call, writes its statuses, releases its workspace. A call whose wait
// gives up reports status 1 for its records and parks its workspace.
void finish(Call &c) {
    Workspace *w = c.w;
    if (!w) { c.settle(1); return; }
    ensure_launched(c);
    (void)cudaSetDevice(c.device);
    const Waited waited = c.unsettled ? Waited::TimedOut : wait_event(w->done);
    const bool synced = waited == Waited::Done;
    const uint32_t *herrs = reinterpret_cast<const uint32_t *>(w->hmeta.p + c.L.errs);
    for (size_t j = 0; j < c.k; ++j) {
        const int i = c.pend[j];
        c.status[(size_t)i] = (j >= c.broken_at || !synced) ? 1 : status_of_bits(herrs[j]);
        if (c.status[(size_t)i] == -1) report_error_bits(herrs[j]);
    }
    if (c.mode == Dest::HostChecked && synced) {   // the single to-host call: copy back only a clean decode
        for (size_t j = 0; j < c.k; ++j) {
            const int i = c.pend[j];
            if (c.status[(size_t)i]) continue;
            const Plan &p = c.plans[(size_t)i];
            const uint8_t *scr = w->dscratch.p + c.scr_off[j];
            if (cudaMemcpy(c.dst_host[i], scr, p.scale_bytes, cudaMemcpyDeviceToHost) != cudaSuccess ||
                cudaMemcpy(c.dst_host[i] + p.scale_bytes, scr + p.weight_at, p.weight_bytes, cudaMemcpyDeviceToHost) != cudaSuccess) {
                (void)cudaGetLastError();
                c.status[(size_t)i] = 1;   // the slab may now be partly written: the caller treats 1 as "decode again"
            }
        }
    }
    workspace_give(w, synced);
    c.w = nullptr;
}

int run_batch(int n, const WexEntry *const *entries, const unsigned char *const *records, int device,
              unsigned char *const *dst_scale, unsigned char *const *dst_weight, unsigned char *const *dst_host,
              Dest mode, int *status) {
    if (n <= 0) return 0;
    const bool host_dst = mode != Dest::Device;
    if (!entries || !records || !(host_dst ? dst_host != nullptr : (dst_scale && dst_weight)) || !status) return n;
    Call c;
    if (submit(c, n, entries, records, device, dst_scale, dst_weight, dst_host, mode)) finish(c);
    for (int i = 0; i < n; ++i) status[i] = c.status[(size_t)i];
    return c.failures();
}

// ---- queued calls (tickets) ----------------------------------------------------------------------
std::mutex g_calls_mu;
std::vector<std::pair<int, Call *>> g_calls;
int g_next_ticket = 0;

}  // namespace
}  // namespace wexb

using namespace wexb;

// ---- the helper ABI ----------------------------------------------------------------------------
WEXB_API unsigned int wex_cuda_helper_abi(void) { return 1u; }

WEXB_API unsigned int wex_cuda_helper_features(void) {
    return WEX_CUDA_FEATURE_DEVICE | WEX_CUDA_FEATURE_REGISTER | WEX_CUDA_FEATURE_NR2 | WEX_CUDA_FEATURE_BATCH |
           WEX_CUDA_FEATURE_NR3 | WEX_CUDA_FEATURE_BATCH_HOST;
}

WEXB_API int wex_cuda_register_model(const unsigned char *blob, size_t bytes) { return model_register(blob, bytes); }

WEXB_API int wex_cuda_decode_to_host(const WexEntry *entry, unsigned char *slab, size_t slab_capacity) {
    uint64_t raw, aligned;
    if (!entry || !slab) return -1;
    if (entry->flags == WEX_ENTRY_NEURAL_RANS) return 1;   // WNR1: legacy codec, not built here
    if (entry->flags != WEX_ENTRY_NEURAL_RANS2 && entry->flags != WEX_ENTRY_NEURAL_RANS3) return -1;
    if (entry_raw_sizes(entry, &raw, &aligned) || aligned > slab_capacity || entry->total_bytes >= aligned) return -1;
    const size_t offset = (size_t)(aligned - entry->total_bytes);   // wex_record_read_offset (c/wex_format.h:161-176)
    if (offset > slab_capacity || entry->total_bytes > slab_capacity - offset) return -1;
    const unsigned char *rec = slab + offset;
    unsigned char *dst = slab;
    int status = -1, device = 0;   // the caller's current device (c/tools/wex_cuda_bridge.cu:141-142)
    if (cudaGetDevice(&device) != cudaSuccess) { (void)cudaGetLastError(); return 1; }
    run_batch(1, &entry, &rec, device, nullptr, nullptr, &dst, Dest::HostChecked, &status);
    return status;
}

WEXB_API int wex_cuda_decode_to_device(const WexEntry *entry, const unsigned char *record, int device,
                                       unsigned char *const *dst_scale, unsigned char *const *dst_weight) {
    if (!entry || !record || !dst_scale || !dst_weight) return -1;
    if (entry->flags == WEX_ENTRY_NEURAL_RANS) return 1;
    int status = -1;
    run_batch(1, &entry, &record, device, dst_scale, dst_weight, nullptr, Dest::Device, &status);
    return status;
}

WEXB_API int wex_cuda_decode_batch_to_device(int n, const WexEntry *const *entries, const unsigned char *const *records,
                                             int device, unsigned char *const *dst_scale, unsigned char *const *dst_weight,
                                             int *status) {
    if (!dst_scale || !dst_weight) return n > 0 ? n : 0;
    return run_batch(n, entries, records, device, dst_scale, dst_weight, nullptr, Dest::Device, status);
}

WEXB_API int wex_cuda_decode_batch_to_host(int n, const WexEntry *const *entries, const unsigned char *const *records,
                                           int device, unsigned char *const *dst, int *status) {
    if (!dst) return n > 0 ? n : 0;
    return run_batch(n, entries, records, device, nullptr, nullptr, dst, Dest::Host, status);
}

WEXB_API int wex_cuda_host_register(void *pointer, size_t bytes) {
    if (!pointer || !bytes) return -1;
    if (cudaHostRegister(pointer, bytes, cudaHostRegisterPortable) != cudaSuccess) { (void)cudaGetLastError(); return 1; }
    return 0;
}

WEXB_API int wex_cuda_host_unregister(void *pointer) {
    if (!pointer) return -1;
    if (cudaHostUnregister(pointer) != cudaSuccess) { (void)cudaGetLastError(); return 1; }
    return 0;
}

namespace wexb {
namespace {
// Per device, for the self-test: two result words (device), their page-locked copy, a stream and an
// event. Made once and kept, so a call whose host wait gave up never frees memory its probe may still
// write; the next call refuses (1) until that probe has ended.
struct ProbeSpace {
    uint32_t *dev = nullptr, *host = nullptr;
    cudaStream_t st = nullptr;
    cudaEvent_t done = nullptr;
    bool ok = false;
};
std::mutex g_probe_mu;
ProbeSpace g_probe[kMaxDevices];
}  // namespace
}  // namespace wexb

WEXB_API int wexb_selftest_bounded_wait(int device, unsigned int polls, unsigned int *bits) {
    if (!bits || !polls || polls > kSelftestMaxPolls || device < 0 || device >= kMaxDevices) return -1;
    KeepDevice keep;
    if (cudaSetDevice(device) != cudaSuccess) { (void)cudaGetLastError(); return 1; }
    std::lock_guard<std::mutex> lock(g_probe_mu);
    ProbeSpace &P = g_probe[device];
    if (!P.ok) {
        if (cudaMalloc(&P.dev, 8) != cudaSuccess || cudaMallocHost(&P.host, 8) != cudaSuccess ||
            cudaStreamCreateWithFlags(&P.st, cudaStreamNonBlocking) != cudaSuccess ||
            cudaEventCreateWithFlags(&P.done, cudaEventDisableTiming) != cudaSuccess) {
            (void)cudaGetLastError();
            return 1;   // whatever was made stays allocated; nothing is retried on a failing device
        }
        P.ok = true;
    } else if (cudaEventQuery(P.done) != cudaSuccess) {   // the previous probe has not ended yet
        (void)cudaGetLastError();
        return 1;
    }
    P.host[0] = P.host[1] = ~0u;
    const bool queued = launch_wait_probe(1, polls, P.dev, P.st) == cudaSuccess &&       // a barrier that completes
                        launch_wait_probe(0, polls, P.dev + 1, P.st) == cudaSuccess &&   // one that nothing arrives on
                        cudaMemcpyAsync(P.host, P.dev, 8, cudaMemcpyDeviceToHost, P.st) == cudaSuccess &&
                        cudaEventRecord(P.done, P.st) == cudaSuccess;
    if (!queued) { (void)cudaGetLastError(); return 1; }
    if (wait_event(P.done) != Waited::Done) return 1;   // the host gave up first: the probe ends on its own
    *bits = P.host[1];
    return P.host[0] == 0 && P.host[1] == kErrTimeout ? 0 : -1;
}

WEXB_API int wexb_set_wait_limit(double seconds) {
    if (!(seconds > 0) || seconds > 86400.0) return -1;
    set_wait_limit(seconds);
    return 0;
}

WEXB_API double wexb_wait_limit(void) { return wait_limit(); }

WEXB_API int wexb_batch_submit(int n, const WexEntry *const *entries, const unsigned char *const *records, int device,
                               unsigned char *const *dst_scale, unsigned char *const *dst_weight) {
    if (n <= 0 || !entries || !records || !dst_scale || !dst_weight) return -1;
    Call *c = new (std::nothrow) Call();
    if (!c) return -3;
    (void)submit(*c, n, entries, records, device, dst_scale, dst_weight, nullptr, Dest::Device);   // statuses final if not queued
    std::lock_guard<std::mutex> lock(g_calls_mu);
    const int t = g_next_ticket;
    g_next_ticket = (g_next_ticket + 1) & 0x7fffffff;
    g_calls.emplace_back(t, c);
    return t;
}

WEXB_API int wexb_batch_submit_verified(int n, const WexEntry *const *entries, const unsigned char *const *records,
                                        const unsigned char *sha256, int device, unsigned char *const *dst_scale,
                                        unsigned char *const *dst_weight) {
    if (n <= 0 || !entries || !records || !sha256 || !dst_scale || !dst_weight) return -1;
    Call *c = new (std::nothrow) Call();
    if (!c) return -3;
    (void)submit(*c, n, entries, records, device, dst_scale, dst_weight, nullptr, Dest::Device, sha256);
    std::lock_guard<std::mutex> lock(g_calls_mu);
    const int t = g_next_ticket;
    g_next_ticket = (g_next_ticket + 1) & 0x7fffffff;
    g_calls.emplace_back(t, c);
    return t;
}

WEXB_API int wexb_batch_wait(int ticket, int *status) {
    Call *c = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_calls_mu);
        for (size_t i = 0; i < g_calls.size(); ++i)
            if (g_calls[i].first == ticket) { c = g_calls[i].second; g_calls.erase(g_calls.begin() + (std::ptrdiff_t)i); break; }
    }
    if (!c) return -1;
    if (c->w) finish(*c);
    if (status) for (int i = 0; i < c->n; ++i) status[i] = c->status[(size_t)i];
    const int bad = c->failures();
    delete c;
    return bad;
}

namespace wexb {
bool batch_uploads_wait(int t) {
    cudaEvent_t e = nullptr;
    int device = 0;
    {
        std::lock_guard<std::mutex> lock(g_calls_mu);
        const Call *c = nullptr;
        for (const auto &q : g_calls) if (q.first == t) { c = q.second; break; }
        if (!c) return false;
        if (!c->w) return true;   // nothing was queued
        e = c->w->uploads_done; device = c->device;
    }
    if (cudaSetDevice(device) != cudaSuccess) { (void)cudaGetLastError(); return false; }
    return wait_event(e) == Waited::Done;
}
}  // namespace wexb

// ---- resident records --------------------------------------------------------------------------
// One queued decode of a resident set: its metadata (host and device), scratch, events and statuses.
struct ResSlot {
    DevBuf dscratch, dmeta;
    PinBuf hmeta;
    MetaLayout L;
    cudaEvent_t done = nullptr;
    cudaEvent_t marks[4] = {};
    bool timed = false;
    bool stale = false;   // its wait gave up: the GPU may still be using it until `done` completes
    int k = 0;
    std::vector<int> order;   // launch position -> the caller's index j (records grouped by model)
};
// Two decodes may be queued at once: the host plans the next one while the GPU runs the previous one.
struct WexbResident {
    int device = -1;
    cudaStream_t own = nullptr;
    std::vector<Plan> plans;          // lengths pointers cleared: the records live on the device
    std::vector<const uint8_t *> tabs;
    std::vector<size_t> rec_off, off_off;
    DevBuf store;                     // records, then offset tables
    size_t offs_at = 0, bytes = 0;
    bool profiling = false;
    int launches = 0;
    ResSlot slot[2];
    int head = 0, queued = 0;         // the oldest queued decode's slot, and how many are queued
    int waited = -1;                  // the slot of the last waited decode (kernel times)
};

WEXB_API unsigned int wexb_abi(void) { return 1u; }

WEXB_API unsigned int wexb_last_error_bits(void) { return last_error_bits(); }

WEXB_API int wexb_resident_create(int n, const WexEntry *const *entries, const unsigned char *const *records, int device,
                                  WexbResident **out, int *status) {
    if (!out) return n > 0 ? n : 0;
    *out = nullptr;
    if (n <= 0 || !entries || !records || !status) return n > 0 ? n : 0;
    auto *r = new (std::nothrow) WexbResident();
    if (!r) { for (int i = 0; i < n; ++i) status[i] = 1; return n; }
    int bad = 0;
    const bool dev_ok = device >= 0 && device < kMaxDevices && cudaSetDevice(device) == cudaSuccess;
    if (!dev_ok) (void)cudaGetLastError();
    size_t rec_bytes = 0, noffs = 0;
    std::vector<std::vector<uint32_t>> offs;
    for (int i = 0; i < n; ++i) {
        Plan p{};
        const uint8_t *t = nullptr;
        status[i] = -1;
        if (!entries[i] || !records[i] || plan_record(entries[i], records[i], &p)) { ++bad; continue; }
        if (!dev_ok || !model_registered(p.model_id) || model_tables(p.model_id, device, &t)) { status[i] = 1; ++bad; continue; }
        status[i] = 0;
        std::vector<uint32_t> o(p.streams() + 1);
        plan_offsets(p, o.data());
        offs.push_back(std::move(o));
        r->rec_off.push_back(rec_bytes); rec_bytes += align_up(p.total + kRecordSlack, 256);
        r->off_off.push_back(noffs); noffs += p.streams() + 1;
        p.lengths = nullptr;
        r->plans.push_back(p);
        r->tabs.push_back(t);
    }
    if (r->plans.empty()) { delete r; return bad; }
    r->device = device;
    r->offs_at = align_up(rec_bytes, 256);
    r->bytes = r->offs_at + noffs * 4;
    bool ok = cudaStreamCreateWithFlags(&r->own, cudaStreamNonBlocking) == cudaSuccess &&
              cudaEventCreateWithFlags(&r->slot[0].done, cudaEventDisableTiming) == cudaSuccess &&
              cudaEventCreateWithFlags(&r->slot[1].done, cudaEventDisableTiming) == cudaSuccess && r->store.grow(r->bytes);
    for (int i = 0, j = 0; ok && i < n; ++i) {
        if (status[i]) continue;
        ok = cudaMemcpy(r->store.p + r->rec_off[(size_t)j], records[i], r->plans[(size_t)j].total, cudaMemcpyHostToDevice) == cudaSuccess &&
             cudaMemcpy(r->store.p + r->offs_at + 4 * r->off_off[(size_t)j], offs[(size_t)j].data(), 4 * offs[(size_t)j].size(),
                        cudaMemcpyHostToDevice) == cudaSuccess;
        ++j;
    }
    if (!ok) {
        (void)cudaGetLastError();
        for (int i = 0; i < n; ++i) if (!status[i]) { status[i] = 1; ++bad; }
        wexb_resident_destroy(r);
        return bad;
    }
    // resident index j <-> caller index: the j-th record with status 0
    *out = r;
    return bad;
}

WEXB_API size_t wexb_resident_bytes(const WexbResident *r) { return r ? r->bytes : 0; }

namespace {
// Waits for the oldest queued decode of r and releases its slot: its statuses (may be NULL), or
// nullptr-safe counts. Returns the number of non-zero statuses.
int resident_retire(WexbResident *r, int *status) {
    ResSlot &q = r->slot[r->head];
    Waited waited = Waited::Failed;
    if (cudaSetDevice(r->device) == cudaSuccess) waited = wait_event(q.done);
    else (void)cudaGetLastError();
    const bool ok = waited == Waited::Done;
    q.stale = waited == Waited::TimedOut;
    const uint32_t *herrs = reinterpret_cast<const uint32_t *>(q.hmeta.p + q.L.errs);
    int bad = 0;
    for (int j = 0; j < q.k; ++j) {   // launch position j holds the caller's record order[j]
        const int v = !ok ? 1 : status_of_bits(herrs[j]);
        if (v == -1) report_error_bits(herrs[j]);
        if (status) status[q.order[(size_t)j]] = v;
        bad += v != 0;
    }
    r->waited = r->head;
    r->head ^= 1;
    --r->queued;
    return bad;
}
}  // namespace

WEXB_API int wexb_resident_decode(WexbResident *r, int k, const int *index, unsigned char *const *dst_scale,
                                  unsigned char *const *dst_weight, void *stream) {
    if (!r || k <= 0 || !index || !dst_scale || !dst_weight) return -1;
    for (int j = 0; j < k; ++j) {
        if (index[j] < 0 || (size_t)index[j] >= r->plans.size()) return -1;
        for (int m = 0; m < 3; ++m) if (!dst_scale[3 * j + m] || !dst_weight[3 * j + m]) return -1;
    }
    if (cudaSetDevice(r->device) != cudaSuccess) { (void)cudaGetLastError(); return 1; }
    if (r->queued == 2) (void)resident_retire(r, nullptr);   // both slots busy: the oldest decode's statuses are dropped
    const int si = (r->head + r->queued) & 1;
    ResSlot &q = r->slot[si];
    if (q.stale) {   // an earlier wait on this slot gave up: reuse it only once its work has ended
        if (cudaEventQuery(q.done) != cudaSuccess) { (void)cudaGetLastError(); return 1; }
        q.stale = false;
    }
    cudaStream_t st = stream ? (cudaStream_t)stream : r->own;
    const int sms = device_sms(r->device);
    if (!sms) return 1;
    // launch order: the records of a model contiguous, the caller's order otherwise
    std::vector<int> &order = q.order;
    order.resize((size_t)k);
    for (int j = 0; j < k; ++j) order[(size_t)j] = j;
    std::stable_sort(order.begin(), order.end(),
                     [&](int a, int b) { return r->tabs[(size_t)index[a]] < r->tabs[(size_t)index[b]]; });
    std::vector<const Plan *> plans((size_t)k);
    std::vector<const uint8_t *> tabs((size_t)k);
    size_t scr_bytes = 0;
    std::vector<size_t> scr_off((size_t)k);
    for (int j = 0; j < k; ++j) {
        const size_t x = (size_t)index[order[(size_t)j]];
        plans[(size_t)j] = &r->plans[x];
        tabs[(size_t)j] = r->tabs[x];
        scr_off[(size_t)j] = scr_bytes; scr_bytes += align_up(r->plans[x].scratch, 256);
    }
    LaunchSet launches;
    launches.plan(plans.data(), tabs.data(), (uint32_t)k, true);
    q.L.compute((size_t)k, launches.items, launches.counter_words(), (size_t)k, 0);
    if (!q.dscratch.grow(scr_bytes) || !q.dmeta.grow(q.L.total) || !q.hmeta.grow(q.L.total)) return 1;
    uint8_t *hm = q.hmeta.p, *dm = q.dmeta.p;
    Nr3Record *hrecs = reinterpret_cast<Nr3Record *>(hm + q.L.recs);
    CommitJob *hjobs = reinterpret_cast<CommitJob *>(hm + q.L.jobs);
    uint32_t *herrs = reinterpret_cast<uint32_t *>(hm + q.L.errs);
    uint32_t *derrs = reinterpret_cast<uint32_t *>(dm + q.L.errs);
    const CommitJob *djobs = reinterpret_cast<const CommitJob *>(dm + q.L.jobs);
    launches.fill(plans.data(), true, sms, kScalesFirst, reinterpret_cast<Nr3Item *>(hm + q.L.items),
                  reinterpret_cast<uint32_t *>(hm + q.L.counters));
    for (int j = 0; j < k; ++j) {
        const int cj = order[(size_t)j];   // the caller's index of the record at launch position j
        const size_t x = (size_t)index[cj];
        const Plan &p = r->plans[x];
        uint8_t *scr = q.dscratch.p + scr_off[(size_t)j];
        plan_descriptor(p, r->store.p + r->rec_off[x], reinterpret_cast<const uint32_t *>(r->store.p + r->offs_at) + r->off_off[x],
                        scr, derrs + j, djobs + j, &hrecs[j]);
        herrs[j] = 0;
        CommitJob &J = hjobs[j];
        for (int m = 0; m < 3; ++m) {
            J.src[m] = scr + p.soff[m]; J.dst[m] = dst_scale[3 * cj + m]; J.bytes[m] = p.dst_bytes[m];
            J.src[3 + m] = scr + p.wout[m]; J.dst[3 + m] = dst_weight[3 * cj + m]; J.bytes[3 + m] = p.dst_bytes[3 + m];
        }
    }
    if (r->profiling && !q.marks[0])
        for (auto &e : q.marks)
            if (cudaEventCreate(&e) != cudaSuccess) { (void)cudaGetLastError(); return 1; }
    const Nr3Record *drecs = reinterpret_cast<const Nr3Record *>(dm + q.L.recs);
    auto mark = [&](int i) { return !r->profiling || cudaEventRecord(q.marks[i], st) == cudaSuccess; };
    // events around: the metadata upload, the decode launch(es), the read-back of the error words
    bool ok = mark(0) && cudaMemcpyAsync(dm, hm, q.L.total, cudaMemcpyHostToDevice, st) == cudaSuccess && mark(1) &&
              launches.launch(drecs, reinterpret_cast<const Nr3Item *>(dm + q.L.items),
                              reinterpret_cast<uint32_t *>(dm + q.L.counters), sms, st) &&
              mark(2) && cudaMemcpyAsync(herrs, derrs, 4 * (size_t)k, cudaMemcpyDeviceToHost, st) == cudaSuccess &&
              mark(3) && cudaEventRecord(q.done, st) == cudaSuccess;
    if (!ok) { (void)cudaGetLastError(); return 1; }
    r->launches = (int)launches.groups.size();
    q.timed = r->profiling;
    q.k = k;
    if (r->waited == si) r->waited = -1;   // its kernel times are being overwritten
    ++r->queued;
    return 0;
}

WEXB_API int wexb_resident_wait(WexbResident *r, int *status) {
    if (!r || !r->queued) return -1;
    return resident_retire(r, status);
}

WEXB_API int wexb_resident_launches(const WexbResident *r) { return r ? r->launches : 0; }

WEXB_API int wexb_resident_profile(WexbResident *r, int on) {
    if (!r) return -1;
    r->profiling = on != 0;
    return 0;
}

WEXB_API int wexb_resident_kernel_ms(const WexbResident *r, float *ms3) {
    if (!r || !ms3 || r->waited < 0 || !r->slot[r->waited].timed) return -1;
    const ResSlot &q = r->slot[r->waited];
    for (int i = 0; i < 3; ++i)
        if (cudaEventElapsedTime(&ms3[i], q.marks[i], q.marks[i + 1]) != cudaSuccess) { (void)cudaGetLastError(); return -1; }
    return 0;
}

WEXB_API void wexb_resident_destroy(WexbResident *r) {
    if (!r) return;
    if (r->device >= 0) {
        KeepDevice keep;
        if (cudaSetDevice(r->device) == cudaSuccess) {
            // bounded: if queued work does not end, the device memory it may use is left allocated
            bool ended = !r->own || wait_stream(r->own) == Waited::Done;
            for (ResSlot &q : r->slot) if (q.done) ended = wait_event(q.done) == Waited::Done && ended;
            for (ResSlot &q : r->slot) {
                if (q.done) cudaEventDestroy(q.done);
                for (auto &e : q.marks) if (e) cudaEventDestroy(e);
                if (ended) { q.dscratch.release(); q.dmeta.release(); q.hmeta.release(); }
            }
            if (ended) {
                if (r->own) cudaStreamDestroy(r->own);
                r->store.release();
            }
        }
        (void)cudaGetLastError();
    }
    delete r;
}
