// Host side of the GPU record writer: wexb_encode_batch and wexb_count_batch (include/wexb200.h).
//
// The reference writes WNR3 records on the CPU, one at a time (c/tools/wex_nr3_tools.c:87-120 ->
// wex_nr3_encode, c/wex_neural_rans.h:615-749) after counting its training experts
// (c/wex_neural_rans.h:579-613). Here the entry checks and chunk rules run on the host; anchors, counts
// and streams run on the GPU, every stream of every record of a call at once (encode_kernels.cu).
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <vector>

#include "bufs.h"
#include "encode.cuh"
#include "host_wait.h"
#include "nr3_host.h"
#include "wexb200.h"

#define WEXB_API extern "C" __attribute__((visibility("default")))

namespace wexb {
namespace {

constexpr uint32_t kMaxChunk = 16384;
constexpr size_t kLaunchBytes = size_t(1) << 30;   // device bytes one launch may hold (slabs, slots, records)

// The writer's view of a 72-byte entry: canonical layout, scales then packed weights, with the
// shape rules of the reference writer (scale [rows, cols], weights [rows, 16 cols]).
struct Layout {
    uint32_t scount[3], wcount[3], soff[3], woff[3];
    uint64_t raw;
};
bool layout_of(const WexEntry *e, Layout *v) {
    if (!e) return false;
    uint64_t s = 0, w = 0;
    for (int m = 0; m < 3; ++m) {
        const uint32_t sr = e->scale_shapes[m][0], sc = e->scale_shapes[m][1];
        const uint32_t wr = e->weight_shapes[m][0], wc = e->weight_shapes[m][1];
        v->soff[m] = e->scale_offsets[m]; v->woff[m] = e->weight_offsets[m];
        if (!sr || !sc || sr != wr || sc * 16u != wc || v->soff[m] != s) return false;
        v->scount[m] = sr * sc; v->wcount[m] = wr * wc * 2u;
        s += v->scount[m];
    }
    if (s != e->scale_bytes) return false;
    for (int m = 0; m < 3; ++m) { if (v->woff[m] != s + w) return false; w += v->wcount[m] / 2u; }
    if (w != e->weight_bytes) return false;
    v->raw = s + w;
    return true;
}

bool pow2_in(uint32_t v, uint32_t lo) { return v >= lo && v <= kMaxChunk && !(v & (v - 1)); }

struct Job {
    int i;
    Layout L;
    uint32_t streams, sstreams;
    size_t dev_bytes;
};

// Device buffers of one launch (grown, kept per process; one call at a time per device).
struct EncSpace {
    std::mutex mu;
    DevBuf slabs, scratch, outs, meta, blob;
    PinBuf hmeta;
    cudaStream_t st[2] = {}, down = nullptr;   // uploads and kernels of groups in turn; downloads
    cudaEvent_t meta_done = nullptr, verdicts[2] = {};
    bool unsettled = false;   // a bounded wait gave up: the buffers may still be in use on the GPU
    bool ready() {
        for (cudaStream_t *s : {&st[0], &st[1], &down})
            if (!*s && cudaStreamCreateWithFlags(s, cudaStreamNonBlocking) != cudaSuccess) return false;
        for (cudaEvent_t *e : {&meta_done, &verdicts[0], &verdicts[1]})
            if (!*e && cudaEventCreateWithFlags(e, cudaEventDisableTiming) != cudaSuccess) return false;
        if (unsettled) {   // reuse the buffers only once the work of the call that gave up has ended
            for (cudaStream_t s : {st[0], st[1], down})
                if (cudaStreamQuery(s) != cudaSuccess) { (void)cudaGetLastError(); return false; }
            unsettled = false;
        }
        return true;
    }
    // Bounded waits for every stream of the space; false (and unsettled on a timeout) unless all ended.
    bool settle() {
        bool ok = true;
        for (cudaStream_t s : {st[0], st[1], down}) {
            const Waited w = wait_stream(s);
            if (w == Waited::TimedOut) unsettled = true;
            ok = ok && w == Waited::Done;
        }
        return ok;
    }
};
constexpr size_t kGroup = 16;   // records per pipelined group of an encode launch
EncSpace g_enc[kMaxDevices];

template <class T> T *carve(uint8_t *&p, size_t n) {
    T *r = reinterpret_cast<T *>(p);
    p += align_up(n * sizeof(T), 256);
    return r;
}

}  // namespace
}  // namespace wexb

using namespace wexb;

WEXB_API int wexb_encode_batch(int n, const WexEntry *const *entries, const unsigned char *const *coded,
                               const unsigned int *flags, const unsigned int *owners, int nr3, unsigned int wchunk,
                               unsigned int schunk, const unsigned char *blob, size_t blob_bytes, int device,
                               unsigned char *const *out, const size_t *cap, size_t *used, size_t *total, int *status) {
    if (n < 0 || (n && (!entries || !coded || !flags || !owners || !out || !cap || !used || !total || !status))) return -1;
    if (!n) return 0;
    for (int i = 0; i < n; ++i) { status[i] = -1; used[i] = total[i] = 0; }
    uint32_t model_id = 0;
    if (model_validate(blob, blob_bytes, &model_id) || !pow2_in(wchunk, 512) || !pow2_in(schunk, 256)) return n;
    std::vector<Job> jobs;
    for (int i = 0; i < n; ++i) {
        Job j{};
        j.i = i;
        if (!coded[i] || !out[i] || !layout_of(entries[i], &j.L) || (flags[i] & ~0x0fu) || (!nr3 && (flags[i] || owners[i])))
            continue;
        for (int m = 0; m < 3; ++m) {
            j.sstreams += (j.L.scount[m] + schunk - 1) / schunk;
            j.streams += (j.L.wcount[m] + wchunk - 1) / wchunk;
        }
        j.streams += j.sstreams;
        const size_t slot = align_up(2 * (size_t)std::max(wchunk, schunk) + 16, 16);
        j.dev_bytes = align_up(j.L.raw, 256) + j.streams * slot + align_up(j.L.raw, 4096) + 8 * (size_t)j.streams + 1024;
        jobs.push_back(j);
    }
    if (device < 0 || device >= kMaxDevices || cudaSetDevice(device) != cudaSuccess) {
        (void)cudaGetLastError();
        for (const Job &j : jobs) status[j.i] = -2;
        return n;
    }
    EncSpace &S = g_enc[device];
    std::lock_guard<std::mutex> lock(S.mu);
    const size_t slot = align_up(2 * (size_t)std::max(wchunk, schunk) + 16, 16);
    bool cuda_ok = S.ready() && S.blob.grow(blob_bytes) &&
                   cudaMemcpyAsync(S.blob.p, blob, blob_bytes, cudaMemcpyHostToDevice, S.st[0]) == cudaSuccess;
    size_t at = 0;
    while (cuda_ok && at < jobs.size()) {
        // one launch: as many records as fit kLaunchBytes (at least one)
        size_t end = at, bytes = 0;
        while (end < jobs.size() && (end == at || bytes + jobs[end].dev_bytes <= kLaunchBytes)) bytes += jobs[end++].dev_bytes;
        const size_t k = end - at;
        size_t slab_bytes = 0, scratch_bytes = 0, out_bytes = 0, streams = 0;
        std::vector<size_t> slab_at(k), scratch_at(k), out_at(k), lens_at(k);
        for (size_t q = 0; q < k; ++q) {
            const Job &j = jobs[at + q];
            slab_at[q] = slab_bytes; slab_bytes += align_up(j.L.raw, 256);
            scratch_at[q] = scratch_bytes; scratch_bytes += (size_t)j.streams * slot;
            out_at[q] = out_bytes; out_bytes += align_up(j.L.raw, 4096);
            lens_at[q] = streams; streams += j.streams;
        }
        // metadata: records, tasks, stream map, lengths and offsets, error words, results
        std::vector<EncTask> tasks;
        std::vector<size_t> task_at(k + 1);
        for (size_t q = 0; q < k; ++q) {
            task_at[q] = tasks.size();
            const Job &j = jobs[at + q];
            for (uint32_t m = 0; m < 3; ++m) {
                const uint32_t ss = (j.L.scount[m] + schunk - 1) / schunk, ws = (j.L.wcount[m] + wchunk - 1) / wchunk;
                for (uint32_t f = 0; f < ss; f += kEncThreads) tasks.push_back({(uint32_t)q, m, 1, f, std::min<uint32_t>(kEncThreads, ss - f)});
                for (uint32_t f = 0; f < ws; f += kEncThreads) tasks.push_back({(uint32_t)q, m, 0, f, std::min<uint32_t>(kEncThreads, ws - f)});
            }
        }
        task_at[k] = tasks.size();
        const size_t meta_bytes = align_up(k * sizeof(EncRecord), 256) + align_up(tasks.size() * sizeof(EncTask), 256) +
                                  align_up(streams * 8, 256) + align_up(streams * 8, 256) + align_up(k * 4, 256) +
                                  align_up(k * 24, 256);
        if (!S.slabs.grow(slab_bytes) || !S.scratch.grow(scratch_bytes) || !S.outs.grow(out_bytes) ||
            !S.meta.grow(meta_bytes) || !S.hmeta.grow(meta_bytes)) { cuda_ok = false; break; }
        uint8_t *hp = S.hmeta.p, *dp = S.meta.p;
        EncRecord *hrec = carve<EncRecord>(hp, k);
        EncTask *htask = carve<EncTask>(hp, tasks.size());
        uint32_t *hmap = carve<uint32_t>(hp, 2 * streams);
        carve<uint32_t>(hp, 2 * streams);
        uint32_t *herr = carve<uint32_t>(hp, k);
        uint64_t *hres = carve<uint64_t>(hp, 3 * k);
        EncRecord *drec = carve<EncRecord>(dp, k);
        EncTask *dtask = carve<EncTask>(dp, tasks.size());
        uint32_t *dmap = carve<uint32_t>(dp, 2 * streams);
        uint32_t *dlens = carve<uint32_t>(dp, 2 * streams);
        uint32_t *derr = carve<uint32_t>(dp, k);
        uint64_t *dres = carve<uint64_t>(dp, 3 * k);
        std::memcpy(htask, tasks.data(), tasks.size() * sizeof(EncTask));
        for (size_t q = 0; q < k; ++q) {
            const Job &j = jobs[at + q];
            EncRecord &R = hrec[q];
            std::memset(&R, 0, sizeof R);
            R.coded = S.slabs.p + slab_at[q];
            uint32_t sb = 0, wb = j.sstreams;
            for (int m = 0; m < 3; ++m) {
                R.soff[m] = j.L.soff[m]; R.woff[m] = j.L.woff[m]; R.scount[m] = j.L.scount[m]; R.wcount[m] = j.L.wcount[m];
                R.sbase[m] = sb; sb += (j.L.scount[m] + schunk - 1) / schunk;
                R.wbase[m] = wb; wb += (j.L.wcount[m] + wchunk - 1) / wchunk;
            }
            R.streams = j.streams; R.schunk = schunk; R.wchunk = wchunk; R.nr3 = nr3 ? 1 : 0; R.cz = (flags[j.i] & 8u) ? 1 : 0;
            R.model_id = model_id; R.owner = owners[j.i]; R.flags = flags[j.i];
            R.scratch = S.scratch.p + scratch_at[q]; R.slot_bytes = (uint32_t)slot;
            R.lens = dlens + 2 * lens_at[q];   // its stream lengths, then their offsets
            R.err = derr + q;
            // the device copy of a record holds raw_aligned bytes: only records below that (verdict 0) are
            // written; the caller's cap decides -1 before the RAW verdict, as in the reference writer
            R.out = S.outs.p + out_at[q];
            R.cap = cap[j.i];
            R.raw_aligned = align_up(j.L.raw, 4096);
            R.result = dres + 3 * q;
            herr[q] = 0;
            for (uint32_t g = 0; g < j.streams; ++g) { hmap[2 * (lens_at[q] + g)] = (uint32_t)q; hmap[2 * (lens_at[q] + g) + 1] = g; }
        }
        // The metadata first. Then groups of kGroup records on the two streams in turn: uploads, kernels and
        // verdicts. A group's records come back, on the download stream, once its verdicts are read, while
        // the next groups upload and encode: uploads, kernels and downloads overlap.
        cuda_ok = cudaMemcpyAsync(S.meta.p, S.hmeta.p, meta_bytes, cudaMemcpyHostToDevice, S.st[0]) == cudaSuccess &&
                  cudaEventRecord(S.meta_done, S.st[0]) == cudaSuccess &&
                  cudaStreamWaitEvent(S.st[1], S.meta_done, 0) == cudaSuccess;
        const size_t groups = (k + kGroup - 1) / kGroup;
        auto fetch = [&](size_t gi) {   // group gi's verdicts, then its records' copies back
            const Waited w = wait_event(S.verdicts[gi & 1]);
            if (w == Waited::TimedOut) S.unsettled = true;
            if (w != Waited::Done) return false;
            for (size_t q = gi * kGroup; q < std::min(k, (gi + 1) * kGroup); ++q) {
                const Job &j = jobs[at + q];
                const int64_t st = (int64_t)hres[3 * q];
                status[j.i] = (int)st;
                used[j.i] = (size_t)hres[3 * q + 1];
                total[j.i] = (size_t)hres[3 * q + 2];
                if (st == 0 && cudaMemcpyAsync(out[j.i], S.outs.p + out_at[q], total[j.i], cudaMemcpyDeviceToHost,
                                               S.down) != cudaSuccess)
                    return false;
            }
            return true;
        };
        for (size_t gi = 0; cuda_ok && gi < groups; ++gi) {
            const size_t q0 = gi * kGroup, q1 = std::min(k, q0 + kGroup);
            cudaStream_t sg = S.st[gi & 1];
            for (size_t q = q0; cuda_ok && q < q1; ++q)
                cuda_ok = cudaMemcpyAsync(S.slabs.p + slab_at[q], coded[jobs[at + q].i], jobs[at + q].L.raw,
                                          cudaMemcpyHostToDevice, sg) == cudaSuccess;
            const size_t s0 = lens_at[q0], s1 = q1 < k ? lens_at[q1] : streams;
            cuda_ok = cuda_ok &&
                      launch_encode(S.blob.p, drec, (uint32_t)q0, (uint32_t)(q1 - q0), dtask + task_at[q0],
                                    (uint32_t)(task_at[q1] - task_at[q0]), dmap + 2 * s0, (uint32_t)(s1 - s0), sg) == cudaSuccess &&
                      cudaMemcpyAsync(hres + 3 * q0, dres + 3 * q0, 24 * (q1 - q0), cudaMemcpyDeviceToHost, sg) == cudaSuccess &&
                      cudaEventRecord(S.verdicts[gi & 1], sg) == cudaSuccess;
            if (cuda_ok && gi) cuda_ok = fetch(gi - 1);
        }
        if (cuda_ok && groups) cuda_ok = fetch(groups - 1);
        cuda_ok = S.settle() && cuda_ok;   // also after a failed step: what was queued must end first
        if (!cuda_ok)
            for (size_t q = 0; q < k; ++q) status[jobs[at + q].i] = -2;
        at = end;
    }
    if (!cuda_ok) {
        (void)cudaGetLastError();
        for (size_t q = at; q < jobs.size(); ++q) status[jobs[q].i] = -2;
    }
    int bad = 0;
    for (int i = 0; i < n; ++i) bad += status[i] != 0;
    return bad;
}

WEXB_API int wexb_count_batch(int n, const WexEntry *const *entries, const unsigned char *const *coded, int nr3,
                              int device, unsigned long long *wc, unsigned long long *sc, int *status) {
    if (n < 0 || (n && (!entries || !coded || !wc || !sc || !status))) return -1;
    if (!n) return 0;
    std::vector<Job> jobs;
    for (int i = 0; i < n; ++i) {
        Job j{};
        j.i = i;
        status[i] = -1;
        if (!coded[i] || !layout_of(entries[i], &j.L)) continue;
        jobs.push_back(j);
    }
    if (device < 0 || device >= kMaxDevices || cudaSetDevice(device) != cudaSuccess) {
        (void)cudaGetLastError();
        for (const Job &j : jobs) status[j.i] = -2;
        return n;
    }
    EncSpace &S = g_enc[device];
    std::lock_guard<std::mutex> lock(S.mu);
    const size_t counters = (3 * kEncContexts * 16 + 3 * 256) * sizeof(unsigned long long);
    bool ok = S.ready() && S.outs.grow(counters) && cudaMemsetAsync(S.outs.p, 0, counters, S.st[0]) == cudaSuccess;
    unsigned long long *dwc = reinterpret_cast<unsigned long long *>(S.outs.p), *dsc = dwc + 3 * kEncContexts * 16;
    size_t at = 0;
    while (ok && at < jobs.size()) {
        size_t end = at, bytes = 0;
        while (end < jobs.size() && (end == at || bytes + align_up(jobs[end].L.raw, 256) <= kLaunchBytes))
            bytes += align_up(jobs[end++].L.raw, 256);
        const size_t k = end - at;
        std::vector<size_t> slab_at(k);
        size_t slab_bytes = 0;
        std::vector<CountTask> tasks;
        constexpr uint32_t kBlocksPerTask = 4096, kScalesPerTask = 65536;
        for (size_t q = 0; q < k; ++q) {
            const Job &j = jobs[at + q];
            slab_at[q] = slab_bytes; slab_bytes += align_up(j.L.raw, 256);
            for (uint32_t m = 0; m < 3; ++m) {
                for (uint32_t f = 0; f < j.L.scount[m]; f += kScalesPerTask)
                    tasks.push_back({(uint32_t)q, m, 1, f, std::min(kScalesPerTask, j.L.scount[m] - f)});
                const uint32_t blocks = j.L.wcount[m] / 32;
                for (uint32_t f = 0; f < blocks; f += kBlocksPerTask)
                    tasks.push_back({(uint32_t)q, m, 0, f, std::min(kBlocksPerTask, blocks - f)});
            }
        }
        const size_t meta_bytes = align_up(k * sizeof(EncRecord), 256) + align_up(tasks.size() * sizeof(CountTask), 256);
        if (!S.slabs.grow(slab_bytes) || !S.meta.grow(meta_bytes) || !S.hmeta.grow(meta_bytes)) { ok = false; break; }
        uint8_t *hp = S.hmeta.p, *dp = S.meta.p;
        EncRecord *hrec = carve<EncRecord>(hp, k);
        CountTask *htask = carve<CountTask>(hp, tasks.size());
        EncRecord *drec = carve<EncRecord>(dp, k);
        CountTask *dtask = carve<CountTask>(dp, tasks.size());
        std::memcpy(htask, tasks.data(), tasks.size() * sizeof(CountTask));
        for (size_t q = 0; q < k; ++q) {
            const Job &j = jobs[at + q];
            EncRecord &R = hrec[q];
            std::memset(&R, 0, sizeof R);
            R.coded = S.slabs.p + slab_at[q];
            for (int m = 0; m < 3; ++m) {
                R.soff[m] = j.L.soff[m]; R.woff[m] = j.L.woff[m]; R.scount[m] = j.L.scount[m]; R.wcount[m] = j.L.wcount[m];
            }
            R.nr3 = nr3 ? 1 : 0;
        }
        ok = cudaMemcpyAsync(S.meta.p, S.hmeta.p, meta_bytes, cudaMemcpyHostToDevice, S.st[0]) == cudaSuccess;
        for (size_t q = 0; ok && q < k; ++q)
            ok = cudaMemcpyAsync(S.slabs.p + slab_at[q], coded[jobs[at + q].i], jobs[at + q].L.raw, cudaMemcpyHostToDevice,
                                 S.st[0]) == cudaSuccess;
        ok = ok && launch_count(drec, (uint32_t)k, dtask, (uint32_t)tasks.size(), dwc, dsc, S.st[0]) == cudaSuccess;
        ok = S.settle() && ok;   // the slabs and metadata are reused by the next launch
        at = end;
    }
    std::vector<unsigned long long> hwc(3 * kEncContexts * 16), hsc(3 * 256);
    ok = ok && cudaMemcpy(hwc.data(), dwc, hwc.size() * 8, cudaMemcpyDeviceToHost) == cudaSuccess &&
         cudaMemcpy(hsc.data(), dsc, hsc.size() * 8, cudaMemcpyDeviceToHost) == cudaSuccess;
    if (!ok) {
        (void)cudaGetLastError();
        for (const Job &j : jobs) status[j.i] = -2;
    } else {
        for (size_t i = 0; i < hwc.size(); ++i) wc[i] += hwc[i];
        for (size_t i = 0; i < hsc.size(); ++i) sc[i] += hsc[i];
        for (const Job &j : jobs) status[j.i] = 0;
    }
    int bad = 0;
    for (int i = 0; i < n; ++i) bad += status[i] != 0;
    return bad;
}
