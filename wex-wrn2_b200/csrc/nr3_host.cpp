// Host side of the WNR2/WNR3 decoder (see nr3_host.h).
#include "nr3_host.h"

#include <cstring>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <mutex>

namespace wexb {

// ---- models ------------------------------------------------------------------------------------
namespace {

struct Model {
    uint32_t id = 0;
    std::vector<uint8_t> blob, image;        // image: the device table layout, built once on the host
    uint8_t *dev[kMaxDevices] = {};
};
std::mutex g_models_mu;
Model *g_models[kMaxModels];
int g_nmodels = 0;
bool g_prepared[kMaxDevices];

bool cdf_ok(const uint8_t *c, uint32_t n) {
    if (rd16(c) != 0 || rd16(c + 2 * n) != kTotal) return false;
    for (uint32_t s = 0; s < n; ++s) if (rd16(c + 2 * s) >= rd16(c + 2 * s + 2)) return false;
    return true;
}
uint32_t fnv1a(const uint8_t *p, size_t n) {
    uint32_t h = 2166136261u;
    for (size_t i = 0; i < n; ++i) h = (h ^ p[i]) * 16777619u;
    return h ? h : 1u;
}

// Table image (wnr3.cuh): per matrix the two-level weight block, then ssym [3][16384 u8], then sf [3][256 u32].
void build_image(const uint8_t *blob, std::vector<uint8_t> &img) {
    img.assign(kTableBytes, 0);
    uint8_t *ssym = img.data() + kWTableBytes;
    uint32_t *sf = reinterpret_cast<uint32_t *>(img.data() + kWTableBytes + kSsymBytes);
    for (uint32_t m = 0; m < 3; ++m) {
        uint32_t *l1 = reinterpret_cast<uint32_t *>(img.data() + (size_t)m * kWBlockBytes);
        uint32_t *l2 = reinterpret_cast<uint32_t *>(img.data() + (size_t)m * kWBlockBytes + kWL1Bytes);
        for (uint32_t srel = 0; srel < 7; ++srel) {
            for (uint32_t pair = 0; pair < kPairs; ++pair) {
                uint32_t pm = 8, mx = 8;   // pair 36: the block start
                if (pair + 1 < kPairs) {
                    for (mx = 0; (mx + 1) * (mx + 2) / 2 <= pair; ++mx) {}
                    pm = pair - mx * (mx + 1) / 2;
                }
                const uint32_t idx = srel * kPairs + pair;
                const uint8_t *c = blob + 32 + 34u * (m * kContexts + (srel * 9u + pm) * 9u + mx);
                uint32_t cdf[17];
                for (uint32_t k = 0; k < 17; ++k) cdf[k] = rd16(c + 2 * k);
                l1[2 * idx] = cdf[4] | cdf[8] << 16;
                l1[2 * idx + 1] = cdf[12] | kTotal << 16;
                for (uint32_t q = 0; q < 4; ++q) {
                    l2[8 * idx + 2 * q] = cdf[4 * q] | cdf[4 * q + 1] << 16;
                    l2[8 * idx + 2 * q + 1] = cdf[4 * q + 2] | cdf[4 * q + 3] << 16;
                }
            }
        }
    }
    for (uint32_t m = 0; m < 3; ++m) {
        const uint8_t *c = blob + 32 + 3u * kContexts * 34u + 514u * m;
        for (uint32_t s = 0; s < 256; ++s) {
            const uint32_t lo = rd16(c + 2 * s), hi = rd16(c + 2 * s + 2);
            for (uint32_t slot = lo; slot < hi; ++slot) ssym[m * kTotal + slot] = (uint8_t)s;
            sf[m * 256u + s] = lo | (hi - lo) << 16;
        }
    }
}
Model *find_locked(uint32_t id) {
    for (int i = 0; i < g_nmodels; ++i) if (g_models[i]->id == id) return g_models[i];
    return nullptr;
}

}  // namespace

int model_validate(const uint8_t *blob, size_t bytes, uint32_t *id) {
    static const uint32_t head[8] = {kMagicWnm2, 1u, kPrec, kContexts, 3u, 0, 0, 0};
    if (!blob || bytes != kModelBytes) return -1;
    for (int i = 0; i < 8; ++i) if (rd32(blob + 4 * i) != head[i]) return -1;
    for (uint32_t r = 0; r < 3 * kContexts; ++r) if (!cdf_ok(blob + 32 + 34u * r, 16)) return -1;
    for (uint32_t m = 0; m < 3; ++m) if (!cdf_ok(blob + 32 + 3u * kContexts * 34u + 514u * m, 256)) return -1;
    if (id) *id = fnv1a(blob, bytes);
    return 0;
}

int model_register(const uint8_t *blob, size_t bytes) {
    uint32_t id;
    if (model_validate(blob, bytes, &id)) return -1;
    std::lock_guard<std::mutex> lock(g_models_mu);
    if (Model *known = find_locked(id)) return std::memcmp(known->blob.data(), blob, kModelBytes) ? -1 : 0;
    if (g_nmodels >= kMaxModels) return 1;
    Model *m = new (std::nothrow) Model();
    if (!m) return 1;
    m->id = id;
    m->blob.assign(blob, blob + kModelBytes);
    build_image(blob, m->image);
    g_models[g_nmodels++] = m;
    return 0;
}

bool model_registered(uint32_t id) {
    std::lock_guard<std::mutex> lock(g_models_mu);
    return find_locked(id) != nullptr;
}

int model_tables(uint32_t id, int device, const uint8_t **out) {
    std::lock_guard<std::mutex> lock(g_models_mu);
    Model *m = find_locked(id);
    if (!m || device < 0 || device >= kMaxDevices) return 1;
    if (!g_prepared[device]) {
        if (prepare_nr3_kernels() != cudaSuccess) { (void)cudaGetLastError(); return 1; }
        g_prepared[device] = true;
    }
    if (!m->dev[device]) {
        uint8_t *p = nullptr;
        if (cudaMalloc(&p, kTableBytes) != cudaSuccess) { (void)cudaGetLastError(); return 1; }
        if (cudaMemcpy(p, m->image.data(), kTableBytes, cudaMemcpyHostToDevice) != cudaSuccess) {
            (void)cudaGetLastError(); cudaFree(p); return 1;
        }
        m->dev[device] = p;
    }
    *out = m->dev[device];
    return 0;
}

const uint8_t *model_image(uint32_t id) {
    std::lock_guard<std::mutex> lock(g_models_mu);
    Model *m = find_locked(id);
    return m ? m->image.data() : nullptr;
}

// ---- records ----------------------------------------------------------------------------------
int entry_raw_sizes(const WexEntry *e, uint64_t *raw, uint64_t *aligned) {
    uint64_t s = 0, w = 0;
    if (!e) return -1;
    for (int m = 0; m < 3; ++m) {
        const uint32_t sr = e->scale_shapes[m][0], sc = e->scale_shapes[m][1];
        const uint32_t wr = e->weight_shapes[m][0], wc = e->weight_shapes[m][1];
        if (!sr || !sc || !wr || !wc || sr != wr || sc * 16u != wc || e->scale_offsets[m] != s) return -1;
        s += (uint64_t)sr * sc;
    }
    if (s != e->scale_bytes) return -1;
    for (int m = 0; m < 3; ++m) {
        if (e->weight_offsets[m] != s + w) return -1;
        w += (uint64_t)e->weight_shapes[m][0] * e->weight_shapes[m][1];
    }
    if (w != e->weight_bytes || s + w > 0xffffffffull) return -1;
    *raw = s + w;
    *aligned = align_up(*raw, 4096);
    return *aligned > 0xffffffffull ? -1 : 0;
}

static bool pow2_in(uint32_t v, uint32_t lo) { return v >= lo && v <= 16384u && !(v & (v - 1)); }

int plan_record(const WexEntry *e, const uint8_t *rec, Plan *p) {
    uint64_t raw, aligned;
    if (!e || !rec || !p || (e->flags != WEX_ENTRY_NEURAL_RANS2 && e->flags != WEX_ENTRY_NEURAL_RANS3) ||
        entry_raw_sizes(e, &raw, &aligned) || e->total_bytes >= aligned) return -1;
    const uint32_t total = e->total_bytes, nr3 = e->flags == WEX_ENTRY_NEURAL_RANS3;
    if (total < 32 || (total & 4095u) || rd32(rec) != (nr3 ? kMagicWnr3 : kMagicWnr2)) return -1;
    const uint32_t flags = rec[27];
    if (nr3 ? (flags & ~0x0fu) != 0 : (flags != 0 || rd32(rec + 28) != 0)) return -1;
    Plan v{};
    v.nr3 = nr3;
    v.flags = (nr3 ? flags : 0u) | (nr3 ? 256u : 0u);
    v.model_id = rd32(rec + 4);
    v.owner = rd32(rec + 28);
    v.word24 = rd32(rec + 24);
    const uint32_t sp = rd32(rec + 8), wp = rd32(rec + 12);
    v.wchunk = rd32(rec + 16);
    v.schunk = rd32(rec + 20);
    if (!v.model_id || !pow2_in(v.wchunk, 512) || !pow2_in(v.schunk, 256)) return -1;
    v.scale_bytes = e->scale_bytes;
    v.weight_bytes = e->weight_bytes;
    v.weight_at = (uint32_t)align_up(e->scale_bytes, 16);
    v.raw = raw;
    v.scratch = (uint64_t)v.weight_at + e->weight_bytes;
    for (int m = 0; m < 3; ++m) {
        v.scount[m] = (uint32_t)e->scale_shapes[m][0] * e->scale_shapes[m][1];
        v.wcount[m] = (uint32_t)e->weight_shapes[m][0] * e->weight_shapes[m][1] * 2u;
        if (!v.scount[m] || !v.wcount[m] || v.wcount[m] % 32u || (uint64_t)v.scount[m] * 32u != v.wcount[m]) return -1;
        v.soff[m] = e->scale_offsets[m];
        v.wout[m] = v.weight_at + (e->weight_offsets[m] - e->scale_bytes);
        v.dst_bytes[m] = v.scount[m];
        v.dst_bytes[3 + m] = v.wcount[m] / 2u;
    }
    for (int m = 0; m < 3; ++m) { v.sbase[m] = v.sstreams; v.sstreams += (v.scount[m] + v.schunk - 1) / v.schunk; }
    for (int m = 0; m < 3; ++m) { v.wbase[m] = v.sstreams + v.wstreams; v.wstreams += (v.wcount[m] + v.wchunk - 1) / v.wchunk; }
    const uint64_t meta = 32u + 2ull * v.streams(), used = meta + sp + wp;
    if (used > total || align_up(used, 4096) != total) return -1;
    v.meta = (uint32_t)meta;
    v.total = total;
    v.lengths = rec + 32;
    uint64_t sum = 0;
    for (uint32_t g = 0; g < v.streams(); ++g) {
        const uint32_t n = rd16(v.lengths + 2 * g);
        if (n < 4) return -1;
        sum += n;
        if (g + 1 == v.sstreams) { if (sum != sp) return -1; sum = 0; }
    }
    if (sum != wp) return -1;
    for (uint64_t i = used; i < total; ++i) if (rec[i]) return -1;   // canonical zero padding
    *p = v;
    return 0;
}

void plan_offsets(const Plan &p, uint32_t *off) {
    uint32_t at = p.meta;
    for (uint32_t g = 0; g < p.streams(); ++g) { off[g] = at; at += rd16(p.lengths + 2 * g); }
    off[p.streams()] = at;
}

void plan_descriptor(const Plan &p, const uint8_t *drec, const uint32_t *doff, uint8_t *dout, uint32_t *derr,
                     const CommitJob *djob, Nr3Record *r) {
    std::memset(r, 0, sizeof *r);
    r->rec = drec; r->offsets = doff; r->out = dout; r->error = derr; r->job = djob;
    r->witems = 0;
    for (int m = 0; m < 3; ++m) {
        r->scount[m] = p.scount[m]; r->wcount[m] = p.wcount[m];
        r->soff[m] = p.soff[m]; r->wout[m] = p.wout[m];
        r->sbase[m] = p.sbase[m]; r->wbase[m] = p.wbase[m];
        r->sitems[m] = ((p.scount[m] + p.schunk - 1) / p.schunk + 31) / 32;
        r->witems += ((p.wcount[m] + p.wchunk - 1) / p.wchunk + 31) / 32;
    }
    r->schunk = p.schunk; r->wchunk = p.wchunk;
    r->model_id = p.model_id; r->owner = p.owner; r->word24 = p.word24; r->flags = p.flags;
}

namespace {
uint32_t warp_items(uint32_t symbols, uint32_t chunk) { return ((symbols + chunk - 1) / chunk + 31) / 32; }
uint32_t commit_items(const Plan &p) {
    uint32_t n = 0;
    for (int r = 0; r < 6; ++r) n += (p.dst_bytes[r] + kCommitChunk - 1) / kCommitChunk;
    return n;
}
uint32_t weight_items(const Plan &p) {
    uint32_t n = 0;
    for (int m = 0; m < 3; ++m) n += warp_items(p.wcount[m], p.wchunk);
    return n;
}
}  // namespace

uint32_t queue_items(const Plan &p, bool commit) {
    uint32_t n = weight_items(p) + (commit ? commit_items(p) : 0u);
    for (int m = 0; m < 3; ++m) n += warp_items(p.scount[m], p.schunk);
    return n;
}

uint32_t queue_fill(const Plan *const *plans, uint32_t n, bool commit, int sms, uint32_t scale_lead, Nr3Item *items) {
    uint32_t at = 0;
    auto scales = [&](uint32_t r) {
        for (uint32_t m = 0; m < 3; ++m)
            for (uint32_t i = 0, k = warp_items(plans[r]->scount[m], plans[r]->schunk); i < k; ++i)
                items[at++] = {r, item_what(kItemScale, m, 32u * i)};
    };
    auto weights = [&](uint32_t r) {
        for (uint32_t m = 0; m < 3; ++m)
            for (uint32_t i = 0, k = warp_items(plans[r]->wcount[m], plans[r]->wchunk); i < k; ++i)
                items[at++] = {r, item_what(kItemWeight, m, 32u * i)};
    };
    auto commits = [&](uint32_t r) {
        for (uint32_t region = 0; region < 6; ++region)
            for (uint32_t c = 0, k = (plans[r]->dst_bytes[region] + kCommitChunk - 1) / kCommitChunk; c < k; ++c)
                items[at++] = {r, item_what(kItemCommit, region, c)};
    };
    // commits trail the decode by about one wave of warps (every warp of the device busy with weight items)
    const uint32_t per_record = n ? std::max(1u, weight_items(*plans[0])) : 1u;
    const uint32_t delay = (uint32_t)std::max(1, sms) * (kDecodeThreads / 32u) / per_record + 1u;
    const uint32_t lead = std::min(std::max(scale_lead, 1u), n);
    for (uint32_t r = 0; r < lead; ++r) scales(r);
    for (uint32_t r = 0; r < n; ++r) {
        if (r + lead < n) scales(r + lead);
        weights(r);
        if (commit && r >= delay) commits(r - delay);
    }
    if (commit)
        for (uint32_t r = n > delay ? n - delay : 0; r < n; ++r) commits(r);
    return at;
}

void LaunchSet::plan(const Plan *const *plans, const uint8_t *const *tables, uint32_t k, bool commit) {
    groups.clear();
    items = 0;
    records = k;
    for (uint32_t j = 0; j < k; ++j) {
        if (groups.empty() || groups.back().tables != tables[j]) groups.push_back({j, 0, items, 0, tables[j]});
        Group &g = groups.back();
        const uint32_t n = queue_items(*plans[j], commit);
        ++g.nrecs;
        g.nitems += n;
        items += n;
    }
}

void LaunchSet::fill(const Plan *const *plans, bool commit, int sms, uint32_t scale_lead, Nr3Item *items_out,
                     uint32_t *counters) const {
    for (const Group &g : groups) queue_fill(plans + g.first_rec, g.nrecs, commit, sms, scale_lead, items_out + g.first_item);
    std::memset(counters, 0, 4 * counter_words());
}

bool LaunchSet::launch(const Nr3Record *drecs, const Nr3Item *ditems, uint32_t *dcounters, int sms, cudaStream_t st,
                       bool beside_hashes) const {
    const size_t heads = groups.size();
    for (size_t i = 0; i < heads; ++i) {
        const Group &g = groups[i];
        const Nr3Launch L{drecs + g.first_rec, ditems + g.first_item, dcounters + i, dcounters + heads + 4ull * g.first_rec,
                          g.tables, g.nitems, g.nrecs};
        if (launch_nr3(L, sms, st, beside_hashes) != cudaSuccess) return false;
    }
    return true;
}

int device_sms(int device) {
    static std::atomic<int> cache[kMaxDevices];
    if (device < 0 || device >= kMaxDevices) return 0;
    int v = cache[device].load();
    if (!v) {
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) {
            (void)cudaGetLastError();
            return 0;
        }
        cache[device].store(v);
    }
    return v;
}

static std::atomic<uint32_t> g_last_bits{0};
void report_error_bits(uint32_t bits) {
    static std::atomic<int> reported{0};
    if (!bits) return;
    g_last_bits.store(bits);
    if ((bits & (kErrHash | kErrCeil | kErrCz)) && !reported.exchange(1))
        std::fprintf(stderr, "[wex] WNR3 record failed its integrity check (error 0x%x); rejected\n", bits);
}
uint32_t last_error_bits() { return g_last_bits.load(); }

}  // namespace wexb
