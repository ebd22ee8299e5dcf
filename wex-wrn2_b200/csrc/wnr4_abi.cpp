// The WNR4 ABI 5 of include/wnr4_cuda.h (kind MX) over wnr4_kernel.cu: WNM4 model registry with
// per-device tables, host validation of records and geometry (wnr4/wnr4.h:108-140, :170-190,
// :317-346), batches queued on tickets, up to WNR4_CUDA_SLOTS in flight per thread and device.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <vector>

#include "bufs.h"
#include "nr3_host.h"
#include "wnr4.cuh"
#include "wnr4_cuda.h"
#include "wnr4_host.h"

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

struct DeviceGuard {
    int saved = -1;
    DeviceGuard() { if (cudaGetDevice(&saved) != cudaSuccess) { (void)cudaGetLastError(); saved = -1; } }
    ~DeviceGuard() { if (saved >= 0) (void)cudaSetDevice(saved); }
};

// Device tables of a validated blob on `device` (once per model and device): 0, or 1 on a CUDA failure.
int register4(const uint8_t *blob, size_t, uint32_t pb, uint32_t id, int device) {
    DeviceGuard guard;
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
struct Slot {
    DevBuf drec, djob, dinfo, derr;
    PinBuf hjob, hinfo, herr;
    cudaEvent_t done = nullptr;
    cudaStream_t own = nullptr;
    std::vector<int> status;
    bool busy = false, broken = false;
    int ticket = -1;
    void release() {
        if (busy && done) (void)cudaEventSynchronize(done);
        drec.release(); djob.release(); dinfo.release(); derr.release();
        hjob.release(); hinfo.release(); herr.release();
        if (done) cudaEventDestroy(done);
        if (own) cudaStreamDestroy(own);
        (void)cudaGetLastError();
        done = nullptr; own = nullptr; busy = false; ticket = -1; status.clear();
    }
};
struct Ring { int device = -1; Slot slot[WNR4_CUDA_SLOTS]; };
struct Rings {
    std::vector<Ring *> rings;
    unsigned next = 0;
    Ring *get(int device) {
        for (Ring *r : rings) if (r->device == device) return r;
        Ring *r = new Ring();
        r->device = device;
        rings.push_back(r);
        return r;
    }
    void release() {
        int cur = -1;
        if (cudaGetDevice(&cur) != cudaSuccess) { (void)cudaGetLastError(); cur = -1; }
        for (Ring *r : rings) {
            if (cudaSetDevice(r->device) == cudaSuccess) for (Slot &s : r->slot) s.release();
            (void)cudaGetLastError();
            delete r;
        }
        rings.clear();
        if (cur >= 0) (void)cudaSetDevice(cur);
    }
    ~Rings() { release(); }
};
thread_local Rings t_rings;

int finish(Slot &s, int *status) {
    const int n = (int)s.status.size();
    const bool ok = !s.broken && cudaEventSynchronize(s.done) == cudaSuccess;
    if (!ok) (void)cudaGetLastError();
    const uint32_t *herr = reinterpret_cast<const uint32_t *>(s.herr.p);
    int bad = 0;
    for (int i = 0; i < n; ++i) {
        int v = s.status[(size_t)i];
        if (!v) v = !ok ? 1 : herr[i] ? -1 : 0;
        if (status) status[i] = v;
        bad += v != 0;
    }
    s.busy = false;
    s.ticket = -1;
    return bad;
}

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
    DeviceGuard guard;
    if (cudaSetDevice(device) != cudaSuccess) { (void)cudaGetLastError(); return WNR4_E_CUDA; }
    Ring *R = t_rings.get(device);
    const int ticket = (int)(t_rings.next & 0x7fffffffu);
    Slot &s = R->slot[(unsigned)ticket % WNR4_CUDA_SLOTS];
    if (s.busy) return WNR4_E_BUSY;   // never drop verdicts the caller has not read
    if ((!s.done && cudaEventCreateWithFlags(&s.done, cudaEventDisableTiming) != cudaSuccess) ||
        (!s.own && cudaStreamCreateWithFlags(&s.own, cudaStreamNonBlocking) != cudaSuccess)) {
        (void)cudaGetLastError();
        return WNR4_E_CUDA;
    }
    cudaStream_t st = stream ? (cudaStream_t)stream : s.own;
    std::vector<size_t> at((size_t)n);
    size_t bytes = 0;
    for (int i = 0; i < n; ++i) { at[(size_t)i] = bytes; bytes += align_up(totals[i], 256); }
    if (!s.drec.grow(bytes) || !s.dinfo.grow(sizeof(W4Rec) * (size_t)n) || !s.hinfo.grow(sizeof(W4Rec) * (size_t)n) ||
        !s.derr.grow(4ull * n) || !s.herr.grow(4ull * n)) return WNR4_E_CUDA;
    s.status.assign((size_t)n, -1);
    std::vector<W4Job> by_m[3];
    W4Rec *info = reinterpret_cast<W4Rec *>(s.hinfo.p);
    for (int i = 0; i < n; ++i) {
        uint8_t *ds[3] = {dst_scale[3 * i], dst_scale[3 * i + 1], dst_scale[3 * i + 2]};
        uint8_t *dw[3] = {dst_weight[3 * i], dst_weight[3 * i + 1], dst_weight[3 * i + 2]};
        std::memset(&info[i], 0, sizeof(W4Rec));
        const bool targets = records[i] && ds[0] && ds[1] && ds[2] && dw[0] && dw[1] && dw[2] &&
                             !((reinterpret_cast<uintptr_t>(dw[0]) | reinterpret_cast<uintptr_t>(dw[1]) |
                                reinterpret_cast<uintptr_t>(dw[2])) & 15u);
        std::vector<W4Job> mine[3];
        if (targets && wnr4_plan(records[i], totals[i], g, owners[i], model_id, s.drec.p + at[(size_t)i], (uint32_t)i,
                                 &info[i], mine)) {
            for (int m = 0; m < 3; ++m) {
                info[i].dst_s[m] = ds[m]; info[i].dst_w[m] = dw[m];
                by_m[m].insert(by_m[m].end(), mine[m].begin(), mine[m].end());
            }
            info[i].error = reinterpret_cast<uint32_t *>(s.derr.p) + i;
            s.status[(size_t)i] = 0;
        }
    }
    const std::vector<W4Job> jobs = wnr4_launch_order(by_m);
    if (!s.djob.grow(sizeof(W4Job) * (jobs.size() + 1)) || !s.hjob.grow(sizeof(W4Job) * (jobs.size() + 1))) return WNR4_E_CUDA;
    if (!jobs.empty()) std::memcpy(s.hjob.p, jobs.data(), sizeof(W4Job) * jobs.size());
    cudaError_t e = cudaSuccess;
    for (int i = 0; i < n && e == cudaSuccess; ++i)
        if (!s.status[(size_t)i]) e = cudaMemcpyAsync(s.drec.p + at[(size_t)i], records[i], totals[i], cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(s.dinfo.p, s.hinfo.p, sizeof(W4Rec) * (size_t)n, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess && !jobs.empty())
        e = cudaMemcpyAsync(s.djob.p, s.hjob.p, sizeof(W4Job) * jobs.size(), cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(s.derr.p, 0, 4ull * n, st);
    if (e == cudaSuccess)
        e = launch_wnr4(md->tab, reinterpret_cast<const W4Job *>(s.djob.p), (uint32_t)jobs.size(),
                        reinterpret_cast<const W4Rec *>(s.dinfo.p), st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(s.herr.p, s.derr.p, 4ull * n, cudaMemcpyDeviceToHost, st);
    const cudaError_t ev = cudaEventRecord(s.done, st);   // recorded even after a failed step: wait waits for what was queued
    s.broken = e != cudaSuccess || ev != cudaSuccess;
    if (s.broken) (void)cudaGetLastError();
    s.busy = true;
    s.ticket = ticket;
    t_rings.next++;
    return ticket;
}

WEXB_API int wnr4_cuda_batch_wait(int ticket, int *status) {
    if (ticket < 0) return -1;
    for (Ring *R : t_rings.rings) {
        Slot &s = R->slot[(unsigned)ticket % WNR4_CUDA_SLOTS];
        if (s.busy && s.ticket == ticket) {
            DeviceGuard guard;
            (void)cudaSetDevice(R->device);
            return finish(s, status);
        }
    }
    return -1;
}

WEXB_API int wnr4_cuda_decode_batch(int n, const uint32_t *geo, const unsigned char *const *records, const size_t *totals,
                                    const uint32_t *owners, uint32_t model_id, int device, unsigned char *const *dst_scale,
                                    unsigned char *const *dst_weight, int *status) {
    if (n <= 0) return 0;
    if (!status) return n;
    const int t = wnr4_cuda_batch_submit(n, geo, records, totals, owners, model_id, device, dst_scale, dst_weight, nullptr);
    if (t < 0) {
        const int v = t == WNR4_E_ARGS ? -1 : 1;
        for (int i = 0; i < n; ++i) status[i] = v;
        return n;
    }
    return wnr4_cuda_batch_wait(t, status);
}

WEXB_API void wnr4_cuda_release_thread(void) { t_rings.release(); }

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
