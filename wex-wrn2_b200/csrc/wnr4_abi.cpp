// The WNR4 ABI 5 of include/wnr4_cuda.h (kind MX) over wnr4_kernel.cu: WNM4 model registry with
// per-device tables, host validation of records and geometry (wnr4/wnr4.h:108-140, :170-190,
// :317-346), and batches queued on tickets. A ticket is served by the same pooled workspaces and
// per-device streams as the WNR3 helper's queued batches (workspace.h): the records and one metadata
// block (record descriptors, tile jobs, zeroed error words) go up on the device's upload stream (or the
// caller's stream), the tile kernel and the read-back of the error words run on a kernel stream, and
// the wait is bounded (host_wait.h). The ABI's in-flight rule is kept: a thread's n-th ticket takes
// lane n mod WNR4_CUDA_SLOTS on its device, and a submit whose lane still holds a ticket that was not
// waited for is refused with WNR4_E_BUSY.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <vector>

#include "bufs.h"
#include "host_wait.h"
#include "nr3_host.h"
#include "wnr4.cuh"
#include "wnr4_cuda.h"
#include "wnr4_host.h"
#include "workspace.h"

#define WEXB_API extern "C" __attribute__((visibility("default")))

namespace wexb {
namespace {

constexpr uint32_t kWnm4 = 0x344d4e57u, kWnr4 = 0x34524e57u;

struct Model4 {
    uint32_t id = 0, pb = 0, rows = 0;
    int device = -1;
    uint8_t *dev = nullptr;
    W4Tables tab{};
};
std::mutex g_m4_mu;
std::vector<Model4 *> g_m4;

bool cdf_ok(const uint8_t *c, uint32_t n) {
    if (rd16(c) != 0 || rd16(c + 2 * n) != (1u << 14)) return false;
    for (uint32_t i = 0; i < n; ++i) if (rd16(c + 2 * i + 2) <= rd16(c + 2 * i)) return false;
    return true;
}

// A WNM4 blob of kind MX: 0 and its pb / id (wnr4/wnr4.h:170-190), else -1.
int model4_validate(const uint8_t *b, size_t bytes, uint32_t *pb, uint32_t *id) {
    if (!b || bytes < 32 || rd32(b) != kWnm4 || rd32(b + 4) != 1 || rd32(b + 8) != 0) return -1;
    const uint32_t p = rd32(b + 24), wctx = kW4Classes * 81u * p;
    if ((p != 1 && p != 5) || bytes != 32u + 3ull * wctx * 34u + 3u * 514u || rd32(b + 12) != 14 || rd32(b + 16) != wctx ||
        rd32(b + 20) != 1 || rd32(b + 28)) return -1;
    for (uint32_t i = 0; i < 3 * wctx; ++i) if (!cdf_ok(b + 32 + 34ull * i, 16)) return -1;
    for (uint32_t i = 0; i < 3; ++i) if (!cdf_ok(b + 32 + 3ull * wctx * 34u + 514u * i, 256)) return -1;
    uint32_t h = 2166136261u;
    for (size_t i = 0; i < bytes; ++i) h = (h ^ b[i]) * 16777619u;
    *pb = p; *id = h ? h : 1u;
    return 0;
}

// Device image (wnr4.cuh): per matrix the two-level weight rows of the reachable contexts, then the
// scale block.
std::vector<uint8_t> model4_image(const uint8_t *b, uint32_t pb) {
    const uint32_t full = kW4Classes * 81u * pb, rows = w4_rows(pb), mb = w4_matrix_bytes(rows), l1b = w4_l1_bytes(rows);
    std::vector<uint8_t> img(3ull * mb, 0);
    for (uint32_t m = 0; m < 3; ++m) {
        uint8_t *dst = img.data() + (size_t)m * mb;
        uint32_t *l1 = reinterpret_cast<uint32_t *>(dst), *l2 = reinterpret_cast<uint32_t *>(dst + l1b);
        for (uint32_t cls = 0; cls < kW4Classes; ++cls)
            for (uint32_t pair = 0; pair < kW4Pairs; ++pair) {
                uint32_t pm = 8, mx = 8;   // pair 36: the block start
                if (pair + 1 < kW4Pairs) {
                    for (mx = 0; (mx + 1) * (mx + 2) / 2 <= pair; ++mx) {}
                    pm = pair - mx * (mx + 1) / 2;
                }
                for (uint32_t bucket = 0; bucket < pb; ++bucket) {
                    const uint32_t ctx = (cls * 9u + pm) * 9u + mx, src = pb == 1 ? ctx : ctx * 5u + bucket;
                    const uint32_t row = (cls * kW4Pairs + pair) * pb + bucket;
                    const uint8_t *c = b + 32 + 34ull * (m * full + src);
                    uint32_t cdf[16];
                    for (uint32_t k = 0; k < 16; ++k) cdf[k] = rd16(c + 2 * k);
                    l1[2 * row] = cdf[4] | cdf[8] << 16;
                    l1[2 * row + 1] = cdf[12] | (1u << 14) << 16;
                    for (uint32_t q = 0; q < 4; ++q) {
                        l2[8 * row + 2 * q] = cdf[4 * q] | cdf[4 * q + 1] << 16;
                        l2[8 * row + 2 * q + 1] = cdf[4 * q + 2] | cdf[4 * q + 3] << 16;
                    }
                }
            }
        const uint8_t *sc = b + 32 + 3ull * full * 34u + 514u * m;
        uint8_t *blk = dst + l1b + 32ull * rows;
        for (uint32_t k = 0; k < 16; ++k) std::memcpy(blk + 2 * k, sc + 32 * k, 2);   // cdf[16k]
        std::memcpy(blk + 32, sc, 514);
    }
    return img;
}

Model4 *find4(uint32_t id, int device) {
    std::lock_guard<std::mutex> lock(g_m4_mu);
    for (Model4 *m : g_m4) if (m->id == id && m->device == device) return m;
    return nullptr;
}

// Device tables of a validated blob on `device` (once per model and device): 0, or 1 on a CUDA failure.
int register4(const uint8_t *blob, size_t, uint32_t pb, uint32_t id, int device) {
    KeepDevice keep;
    std::lock_guard<std::mutex> lock(g_m4_mu);
    for (Model4 *m : g_m4) if (m->id == id && m->device == device) return 0;
    const std::vector<uint8_t> img = model4_image(blob, pb);
    auto *m = new Model4();
    m->id = id; m->pb = pb; m->rows = w4_rows(pb); m->device = device;
    if (cudaSetDevice(device) != cudaSuccess || cudaMalloc(&m->dev, img.size()) != cudaSuccess ||
        cudaMemcpy(m->dev, img.data(), img.size(), cudaMemcpyHostToDevice) != cudaSuccess) {
        (void)cudaGetLastError();
        if (m->dev) cudaFree(m->dev);
        delete m;
        return 1;
    }
    m->tab = {m->dev, m->rows, pb, w4_matrix_bytes(m->rows), id};
    g_m4.push_back(m);
    return 0;
}

}  // namespace

// Geometry of a kind-MX expert slab (wnr4_geo, wnr4/wnr4.h:108-140).
bool wnr4_geo(const uint32_t *v, W4Geo *g) {
    if (!v || v[0] != 0) return false;
    uint64_t lo[6], hi[6];
    for (int m = 0; m < 3; ++m) {
        g->scount[m] = v[1 + m]; g->scols[m] = v[4 + m];
        if (!v[1 + m] || !v[4 + m] || v[1 + m] % v[4 + m] || v[1 + m] >= (1u << 27)) return false;
        lo[2 * m] = v[7 + m]; hi[2 * m] = (uint64_t)v[7 + m] + v[1 + m];
        lo[2 * m + 1] = v[10 + m]; hi[2 * m + 1] = (uint64_t)v[10 + m] + 16ull * v[1 + m];
    }
    for (int i = 0; i < 6; ++i)
        for (int j = i + 1; j < 6; ++j) if (lo[i] < hi[j] && lo[j] < hi[i]) return false;
    return true;
}

// One record's header and tile table (wnr4/wnr4.h:317-346), its owner and model; appends its tiles
// (matrix by matrix) to jobs[m]. drec = the record's device copy.
bool wnr4_plan(const uint8_t *rec, size_t total, const W4Geo &g, uint32_t owner, uint32_t model_id, const uint8_t *drec,
                  uint32_t index, W4Rec *info, std::vector<W4Job> jobs[3]) {
    if (!rec || total < 64 || (total & 4095) || rd32(rec) != kWnr4) return false;
    const uint32_t mid = rd32(rec + 4), own = rd32(rec + 8), kind = rec[12], flags = rec[13], G = rd16(rec + 14);
    const uint32_t ntiles = rd32(rec + 20), payload = rd32(rec + 24);
    if (!mid || kind != 0 || rec[19] || G < 1 || G > 4096 || (flags & ~0x0fu)) return false;
    for (int i = 28; i < 64; ++i) if (rec[i]) return false;
    uint32_t base[4], t = 0;
    for (int m = 0; m < 3; ++m) { base[m] = t; t += (g.scount[m] + 32u * G - 1) / (32u * G); }
    base[3] = t;
    if (t != ntiles) return false;
    const uint64_t used = 64ull + 4ull * (ntiles + 1ull) + payload;
    if (used > total || align_up(used, 4096) != total) return false;
    const uint8_t *offs = rec + 64;
    if (rd32(offs)) return false;
    uint32_t prev = 0;
    for (uint32_t i = 1; i <= ntiles; ++i) {
        const uint32_t o = rd32(offs + 4ull * i);
        if (o < prev || o - prev < 128 || ((o - prev) & 1u)) return false;
        prev = o;
    }
    if (prev != payload) return false;
    for (uint64_t i = used; i < total; ++i) if (rec[i]) return false;
    if (mid != model_id || own != owner) return false;
    info->model_id = mid; info->owner = own; info->flags = flags; info->G = G;
    info->anchors = rec[16] | (uint32_t)rec[17] << 8 | (uint32_t)rec[18] << 16;
    const uint64_t data = 64ull + 4ull * (ntiles + 1ull);
    for (uint32_t tt = 0; tt < ntiles; ++tt) {
        const uint32_t m = tt >= base[2] ? 2 : tt >= base[1] ? 1 : 0;
        const uint32_t c0 = (tt - base[m]) * 32u * G, n = std::min(32u * G, g.scount[m] - c0);
        const uint32_t o0 = rd32(offs + 4ull * tt), o1 = rd32(offs + 4ull * tt + 4);
        jobs[m].push_back({drec + data + o0, (o1 - o0 - 128) / 2, index, tt, m, c0, n});
    }
    return true;
}

std::vector<W4Job> wnr4_launch_order(const std::vector<W4Job> by_m[3]) {
    std::vector<W4Job> jobs;
    for (int m = 0; m < 3; ++m) {   // each matrix's tiles padded to whole CTAs (a CTA holds one matrix)
        jobs.insert(jobs.end(), by_m[m].begin(), by_m[m].end());
        while (jobs.size() % kW4Warps) jobs.push_back({nullptr, 0, 0, 0, (uint32_t)m, 0, 0});
    }
    return jobs;
}

int wnr4_tables(const uint8_t *blob, size_t bytes, int device, W4Tables *tab, uint32_t *id) {
    uint32_t pb = 0;
    if (model4_validate(blob, bytes, &pb, id)) return -1;
    const int st = register4(blob, bytes, pb, *id, device);
    if (st) return st;
    Model4 *m = find4(*id, device);
    if (!m) return 1;
    *tab = m->tab;
    return 0;
}

namespace {

// ---- tickets ------------------------------------------------------------------------------------
// One submitted batch of the calling thread: its workspace and the host verdict of each record
// (-1 refused before queueing, 0 queued).
struct Batch4 {
    int ticket = -1, device = -1;
    Workspace *w = nullptr;
    size_t err_at = 0;          // byte offset of the error words in the metadata block
    bool queued = false;        // every queueing step succeeded
    std::vector<int> pre;
};

// The calling thread's tickets: those it submitted and has not waited for yet.
struct TicketBook {
    uint32_t issued = 0;
    std::vector<Batch4> open;

    bool lane_taken(int device, int lane) const {
        for (const Batch4 &b : open)
            if (b.device == device && (b.ticket % WNR4_CUDA_SLOTS) == lane) return true;
        return false;
    }
    // Waits (bounded) for open[i], writes its statuses, gives its workspace back and removes it.
    int close(size_t i, int *status) {
        Batch4 b = std::move(open[i]);
        open.erase(open.begin() + (std::ptrdiff_t)i);
        Waited waited = Waited::Failed;
        if (b.w) {
            KeepDevice keep;
            if (cudaSetDevice(b.device) == cudaSuccess) waited = wait_event(b.w->done);
            else (void)cudaGetLastError();
        }
        const bool ok = b.queued && waited == Waited::Done;
        const uint32_t *err = b.w ? reinterpret_cast<const uint32_t *>(b.w->hmeta.p + b.err_at) : nullptr;
        int bad = 0;
        for (size_t r = 0; r < b.pre.size(); ++r) {
            const int v = b.pre[r] ? b.pre[r] : !ok ? 1 : status_of_bits(err[r]);
            if (status) status[r] = v;
            bad += v != 0;
        }
        workspace_give(b.w, waited != Waited::TimedOut);
        return bad;
    }
    void close_all() { while (!open.empty()) close(open.size() - 1, nullptr); }
    ~TicketBook() { close_all(); }
};
thread_local TicketBook t_book;

}  // namespace
}  // namespace wexb

using namespace wexb;

WEXB_API unsigned int wnr4_cuda_abi(void) { return 5u; }

WEXB_API int wnr4_cuda_register_model(const unsigned char *blob, size_t bytes, int device) {
    uint32_t pb = 0, id = 0;
    if (model4_validate(blob, bytes, &pb, &id)) return -1;
    return register4(blob, bytes, pb, id, device);
}

WEXB_API int wnr4_cuda_batch_submit(int n, const uint32_t *geo, const unsigned char *const *records, const size_t *totals,
                                    const uint32_t *owners, uint32_t model_id, int device, unsigned char *const *dst_scale,
                                    unsigned char *const *dst_weight, void *stream) {
    W4Geo g;
    if (n <= 0 || !geo || !records || !totals || !owners || !dst_scale || !dst_weight || !wnr4_geo(geo, &g)) return WNR4_E_ARGS;
    Model4 *md = find4(model_id, device);
    if (!md) return WNR4_E_MODEL;
    const int ticket = (int)(t_book.issued & 0x7fffffffu);
    if (t_book.lane_taken(device, ticket % WNR4_CUDA_SLOTS)) return WNR4_E_BUSY;   // unread verdicts are never dropped
    KeepDevice keep;
    if (cudaSetDevice(device) != cudaSuccess) { (void)cudaGetLastError(); return WNR4_E_CUDA; }
    Batch4 b;
    b.ticket = ticket; b.device = device;
    b.pre.assign((size_t)n, -1);
    // records, 256-byte aligned, in the workspace's record buffer
    std::vector<size_t> rec_at((size_t)n);
    size_t rec_bytes = 0;
    for (int i = 0; i < n; ++i) { rec_at[(size_t)i] = rec_bytes; rec_bytes += align_up(totals[i], 256); }
    Workspace *w = workspace_take(device);
    if (!w) return WNR4_E_CUDA;
    if (!w->drec.grow(rec_bytes + 256)) { workspace_give(w, true); return WNR4_E_CUDA; }
    std::vector<W4Rec> info((size_t)n);
    std::vector<W4Job> by_m[3];
    for (int i = 0; i < n; ++i) {
        W4Rec &R = info[(size_t)i];
        std::memset(&R, 0, sizeof R);
        bool targets = records[i] != nullptr;
        uintptr_t wbits = 0;
        for (int m = 0; m < 3; ++m) {
            targets = targets && dst_scale[3 * i + m] && dst_weight[3 * i + m];
            wbits |= reinterpret_cast<uintptr_t>(dst_weight[3 * i + m]);
        }
        if (!targets || (wbits & 15u)) continue;   // packed weights take 16-byte stores
        std::vector<W4Job> tiles[3];
        if (!wnr4_plan(records[i], totals[i], g, owners[i], model_id, w->drec.p + rec_at[(size_t)i], (uint32_t)i, &R, tiles))
            continue;
        for (int m = 0; m < 3; ++m) {
            R.dst_s[m] = dst_scale[3 * i + m];
            R.dst_w[m] = dst_weight[3 * i + m];
            by_m[m].insert(by_m[m].end(), tiles[m].begin(), tiles[m].end());
        }
        b.pre[(size_t)i] = 0;
    }
    const std::vector<W4Job> jobs = wnr4_launch_order(by_m);
    // one metadata block: record descriptors, tile jobs, zeroed error words
    const size_t info_at = 0, job_at = align_up(sizeof(W4Rec) * (size_t)n, 256);
    b.err_at = align_up(job_at + sizeof(W4Job) * (jobs.size() + 1), 256);
    const size_t meta_bytes = b.err_at + 4ull * (size_t)n;
    if (!w->dmeta.grow(meta_bytes) || !w->hmeta.grow(meta_bytes)) { workspace_give(w, true); return WNR4_E_CUDA; }
    uint8_t *hm = w->hmeta.p, *dm = w->dmeta.p;
    uint32_t *derr = reinterpret_cast<uint32_t *>(dm + b.err_at);
    for (int i = 0; i < n; ++i) if (!b.pre[(size_t)i]) info[(size_t)i].error = derr + i;
    std::memcpy(hm + info_at, info.data(), sizeof(W4Rec) * (size_t)n);
    if (!jobs.empty()) std::memcpy(hm + job_at, jobs.data(), sizeof(W4Job) * jobs.size());
    std::memset(hm + b.err_at, 0, 4ull * (size_t)n);
    // uploads, then the kernel and the read-back of the error words
    cudaStream_t up = (cudaStream_t)stream, st = (cudaStream_t)stream;
    if (!stream && !device_streams(device, &up, &st)) { workspace_give(w, true); return WNR4_E_CUDA; }
    bool ok = cudaMemcpyAsync(dm, hm, meta_bytes, cudaMemcpyHostToDevice, up) == cudaSuccess;
    for (int i = 0; ok && i < n; ++i)
        if (!b.pre[(size_t)i])
            ok = cudaMemcpyAsync(w->drec.p + rec_at[(size_t)i], records[i], totals[i], cudaMemcpyHostToDevice, up) == cudaSuccess;
    if (ok && up != st)
        ok = cudaEventRecord(w->uploads_done, up) == cudaSuccess && cudaStreamWaitEvent(st, w->uploads_done, 0) == cudaSuccess;
    ok = ok &&
         launch_wnr4(md->tab, reinterpret_cast<const W4Job *>(dm + job_at), (uint32_t)jobs.size(),
                     reinterpret_cast<const W4Rec *>(dm + info_at), st) == cudaSuccess &&
         cudaMemcpyAsync(hm + b.err_at, derr, 4ull * (size_t)n, cudaMemcpyDeviceToHost, st) == cudaSuccess;
    // `done` is recorded even after a failed step, so the wait covers whatever was queued
    if (cudaEventRecord(w->done, st) != cudaSuccess) {
        (void)cudaGetLastError();
        ok = false;
        if (wait_stream(st) == Waited::TimedOut || (up != st && wait_stream(up) == Waited::TimedOut)) {
            workspace_give(w, false);   // its work may still be running; nothing else will wait for it
            return WNR4_E_CUDA;
        }
    }
    if (!ok) (void)cudaGetLastError();
    b.w = w;
    b.queued = ok;
    t_book.open.push_back(std::move(b));
    t_book.issued++;
    return ticket;
}

WEXB_API int wnr4_cuda_batch_wait(int ticket, int *status) {
    if (ticket < 0) return -1;
    for (size_t i = 0; i < t_book.open.size(); ++i)
        if (t_book.open[i].ticket == ticket) return t_book.close(i, status);
    return -1;
}

WEXB_API int wnr4_cuda_decode_batch(int n, const uint32_t *geo, const unsigned char *const *records, const size_t *totals,
                                    const uint32_t *owners, uint32_t model_id, int device, unsigned char *const *dst_scale,
                                    unsigned char *const *dst_weight, int *status) {
    if (n <= 0) return 0;
    if (!status) return n;
    const int t = wnr4_cuda_batch_submit(n, geo, records, totals, owners, model_id, device, dst_scale, dst_weight, nullptr);
    if (t >= 0) return wnr4_cuda_batch_wait(t, status);
    const int v = t == WNR4_E_ARGS ? -1 : 1;
    for (int i = 0; i < n; ++i) status[i] = v;
    return n;
}

WEXB_API void wnr4_cuda_release_thread(void) { t_book.close_all(); }

WEXB_API int wnr4_cuda_gg_register_model(const unsigned char *, size_t, int, uint32_t *id) {
    if (id) *id = 0;
    return -1;
}
WEXB_API int wnr4_cuda_gg_batch_submit(int, uint32_t, const uint32_t *, const uint32_t *, const unsigned char *const *,
                                       const size_t *, const uint32_t *, uint32_t, int, unsigned char *const *, void *) {
    return WNR4_E_ARGS;
}
WEXB_API int wnr4_cuda_gg_decode_batch(int n, uint32_t, const uint32_t *, const uint32_t *, const unsigned char *const *,
                                       const size_t *, const uint32_t *, uint32_t, int, unsigned char *const *, int *status) {
    if (n <= 0) return 0;
    if (!status) return n;
    for (int i = 0; i < n; ++i) status[i] = -1;
    return n;
}
