// Expert records read from a WEX4 container file into HBM: the wexb_file_* entry points of
// include/wexb200.h.
//
// The reference's expert store reads one record per pread (O_DIRECT where the platform has it) into a
// pageable slab and then decodes it (c/expert_store_wex.c:92-121, :305-337); its read benchmark times
// pread on threads and io_uring (bench/wex_io.c). Here the read is the first stage of a pipeline:
//   1. reads: every record is split into page-aligned pieces of at most 2 MiB, spread over a pool of
//      reader threads (pread; O_DIRECT on request), into a ring of kSlots page-locked host buffers of
//      kBatch records each;
//   2. once the last piece of a slot has landed, its WNR3 records are checked on the host (owner,
//      value-exact flag, model id) and queued to the device by wexb_batch_submit, and its RAW records
//      are copied to their six destinations on the file's own stream;
//   3. the slot is read again as soon as its uploads have finished, before its decodes have;
// so the reads of later batches overlap the uploads and decodes of earlier ones.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <mutex>
#include <new>
#include <thread>
#include <unordered_map>
#include <vector>

#include "host_wait.h"
#include "nr3_host.h"
#include "wex4_index.h"
#include "wexb200.h"

#define WEXB_API extern "C" __attribute__((visibility("default")))

namespace wexb {
namespace {

constexpr size_t kPage = 4096, kPiece = size_t(2) << 20;
constexpr int kBatch = 8;      // records per ring slot, per queued decode call
constexpr int kSlots = 3;      // ring slots: batches being read while an earlier one uploads
constexpr int kInflight = 3;   // queued decode calls before the oldest is waited for
constexpr int kDefaultReaders = 8, kMaxReaders = 64;

// The reads of one ring slot.
struct Gate {
    std::mutex mu;
    std::condition_variable cv;
    uint32_t open = 0;
    uint8_t bad[kBatch] = {};   // a read of record j of the slot failed
};
struct Piece {
    uint8_t *dst;
    size_t len, need;   // bytes asked for (page-aligned), bytes that must arrive (the record's share)
    uint64_t off;
    Gate *gate;
    int j;
};

// Reads len bytes at off, or up to the end of the file; true when at least `need` bytes arrived.
bool read_piece(int fd, const Piece &p) {
    size_t got = 0;
    while (got < p.len) {
        const ssize_t r = pread(fd, p.dst + got, p.len - got, (off_t)(p.off + got));
        if (r < 0 && errno == EINTR) continue;
        if (r <= 0) break;
        got += (size_t)r;
    }
    return got >= p.need;
}

}  // namespace
}  // namespace wexb

using namespace wexb;

struct WexbFile {
    int fd = -1;
    bool direct = false;
    FileIndex idx;
    std::unordered_map<uint32_t, uint32_t> by_owner;   // layer << 16 | expert -> index of idx.records
    std::vector<uint32_t> model_of;                     // per record: its model id (WNR3), else 0
    size_t slot_rec = 0;                                // ring bytes per record: largest stored, page-aligned
    // reader pool
    std::vector<std::thread> readers;
    std::mutex qmu;
    std::condition_variable qcv;
    std::deque<Piece> queue;
    bool stop = false;
    // ring and device state; one call at a time
    std::mutex call_mu;
    uint8_t *ring = nullptr;
    size_t ring_bytes = 0;
    bool pinned = false;
    Gate gates[kSlots];
    int device = -1;
    cudaStream_t raw_st = nullptr;
    cudaEvent_t raw_done[kSlots] = {};
    // A bounded wait for a slot's uploads gave up: the GPU may still read the ring, so no later call
    // reuses it (every record then reports 1).
    bool stuck = false;

    void reader_loop() {
        for (;;) {
            Piece p;
            {
                std::unique_lock<std::mutex> lock(qmu);
                qcv.wait(lock, [&] { return stop || !queue.empty(); });
                if (queue.empty()) return;
                p = queue.front();
                queue.pop_front();
            }
            const bool ok = read_piece(fd, p);
            std::lock_guard<std::mutex> lock(p.gate->mu);
            if (!ok) p.gate->bad[p.j] = 1;
            if (--p.gate->open == 0) p.gate->cv.notify_all();
        }
    }
    uint8_t *slot(int s) { return ring + (size_t)s * kBatch * slot_rec; }
    // Queues the reads of records rec[0 .. k) into ring slot s.
    void issue(int s, const uint32_t *rec, int k) {
        Gate &g = gates[s];
        std::vector<Piece> ps;
        for (int j = 0; j < k; ++j) {
            const FileExpert &e = idx.records[rec[j]];
            const size_t len = align_up(e.stored, kPage);
            for (size_t at = 0; at < len; at += kPiece) {
                const size_t n = std::min(kPiece, len - at);
                ps.push_back({slot(s) + (size_t)j * slot_rec + at, n, std::min(n, (size_t)e.stored - std::min((size_t)e.stored, at)),
                              e.entry.file_offset + at, &g, j});
            }
        }
        {
            std::lock_guard<std::mutex> lock(g.mu);
            g.open = (uint32_t)ps.size();
            std::memset(g.bad, 0, sizeof g.bad);
        }
        {
            std::lock_guard<std::mutex> lock(qmu);
            for (const Piece &p : ps) queue.push_back(p);
        }
        qcv.notify_all();
    }
    void wait_reads(int s) {
        Gate &g = gates[s];
        std::unique_lock<std::mutex> lock(g.mu);
        g.cv.wait(lock, [&] { return g.open == 0; });
    }
    bool alloc_ring() {
        if (ring) return true;
        const size_t bytes = (size_t)kSlots * kBatch * slot_rec;
        void *p = nullptr;
        if (posix_memalign(&p, kPage, bytes)) return false;
        std::memset(p, 0, bytes);   // touched before any read
        ring = (uint8_t *)p;
        ring_bytes = bytes;
        return true;
    }
    // Device-side state for `dev`: the ring page-locked, the RAW copy stream and its slot events.
    bool bind(int dev) {
        if (cudaSetDevice(dev) != cudaSuccess) { (void)cudaGetLastError(); return false; }
        if (!pinned) {
            if (cudaHostRegister(ring, ring_bytes, cudaHostRegisterPortable) != cudaSuccess) { (void)cudaGetLastError(); return false; }
            pinned = true;
        }
        if (device == dev) return true;
        drop_stream();
        if (cudaStreamCreateWithFlags(&raw_st, cudaStreamNonBlocking) != cudaSuccess) { (void)cudaGetLastError(); return false; }
        for (auto &e : raw_done)
            if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) { (void)cudaGetLastError(); return false; }
        device = dev;
        return true;
    }
    void drop_stream() {
        if (device >= 0) (void)cudaSetDevice(device);
        for (auto &e : raw_done) { if (e) cudaEventDestroy(e); e = nullptr; }
        if (raw_st) cudaStreamDestroy(raw_st);
        raw_st = nullptr;
        device = -1;
    }
    ~WexbFile() {
        {
            std::lock_guard<std::mutex> lock(qmu);
            stop = true;
        }
        qcv.notify_all();
        for (auto &t : readers) t.join();
        drop_stream();
        if (pinned) cudaHostUnregister(ring);
        std::free(ring);
        if (fd >= 0) close(fd);
    }
};

namespace {

// Reads len bytes at off into a fresh page-aligned buffer (O_DIRECT-safe), or nullptr.
uint8_t *read_aligned(int fd, uint64_t off, size_t len) {
    void *p = nullptr;
    const size_t cap = align_up(len ? len : 1, kPage);
    if (posix_memalign(&p, kPage, cap)) return nullptr;
    Piece piece{(uint8_t *)p, cap, len, off, nullptr, 0};
    if (!read_piece(fd, piece)) { std::free(p); return nullptr; }
    return (uint8_t *)p;
}

// The requests that name an expert of the file, in order, cut into ring batches.
struct Work {
    std::vector<int> who;        // request index of each resolved record
    std::vector<uint32_t> rec;   // its record
    size_t batches() const { return (rec.size() + kBatch - 1) / kBatch; }
    int size(size_t b) const { return (int)std::min<size_t>(kBatch, rec.size() - b * kBatch); }
};
Work resolve(const WexbFile &f, int n, const unsigned *layer, const unsigned *expert, int *status) {
    Work w;
    for (int i = 0; i < n; ++i) {
        status[i] = -1;
        if (layer[i] > 0xffff || expert[i] > 0xffff) continue;
        const auto it = f.by_owner.find(layer[i] << 16 | expert[i]);
        if (it == f.by_owner.end()) continue;
        w.who.push_back(i);
        w.rec.push_back(it->second);
    }
    return w;
}

}  // namespace

WEXB_API int wexb_file_open(const char *path, unsigned int flags, int readers, WexbFile **out) {
    if (!path || !out || (flags & ~WEXB_FILE_DIRECT) || readers < 0 || readers > kMaxReaders) return -1;
    *out = nullptr;
    WexbFile *f = new (std::nothrow) WexbFile();
    if (!f) return 1;
    f->direct = (flags & WEXB_FILE_DIRECT) != 0;
    f->fd = open(path, O_RDONLY | O_CLOEXEC | (f->direct ? O_DIRECT : 0));
    struct stat st;
    if (f->fd < 0 || fstat(f->fd, &st)) { delete f; return 1; }   // EINVAL with O_DIRECT: the filesystem refuses it
    // header page, index, models (c/wex4.h:185-437), as the stores open a container
    uint8_t *page = read_aligned(f->fd, 0, kPage);
    int rc = page ? file_header(page, (uint64_t)st.st_size, &f->idx) : -1;
    uint8_t *index = nullptr;
    if (!rc) {
        index = read_aligned(f->fd, f->idx.index_offset, (size_t)f->idx.index_len);
        rc = index ? file_index(page, index, &f->idx) : -1;
    }
    std::free(index);
    std::free(page);
    for (size_t m = 0; !rc && m < f->idx.models.size(); ++m) {
        const FileModel &b = f->idx.models[m];
        uint8_t *blob = read_aligned(f->fd, b.offset, (size_t)b.bytes), digest[32];
        uint32_t id = 0;
        if (!blob) { rc = -1; break; }
        host_sha256(blob, (size_t)b.bytes, digest);
        if (std::memcmp(digest, b.sha, 32) || model_validate(blob, (size_t)b.bytes, &id) || id != b.id ||
            model_register(blob, (size_t)b.bytes))
            rc = -1;
        std::free(blob);
    }
    if (rc) { delete f; return -1; }
    size_t largest = kPage;
    for (uint32_t r = 0; r < f->idx.records.size(); ++r) {
        const FileExpert &e = f->idx.records[r];
        f->by_owner.emplace(e.owner, r);
        largest = std::max(largest, align_up(e.stored, kPage));
    }
    f->slot_rec = largest;
    const int nthreads = readers ? readers : kDefaultReaders;
    try {
        for (int t = 0; t < nthreads; ++t) f->readers.emplace_back(&WexbFile::reader_loop, f);
    } catch (...) {
        delete f;
        return 1;
    }
    *out = f;
    return 0;
}

WEXB_API void wexb_file_close(WexbFile *f) { delete f; }

WEXB_API int wexb_file_info(const WexbFile *f, unsigned int *layers, unsigned int *experts, unsigned int *records,
                            unsigned long long *max_stored) {
    if (!f) return -1;
    if (layers) *layers = f->idx.layers;
    if (experts) *experts = f->idx.experts;
    if (records) *records = (unsigned)f->idx.records.size();
    if (max_stored) *max_stored = f->slot_rec;
    return 0;
}

WEXB_API int wexb_file_evict(WexbFile *f) {
    if (!f) return -1;
    return posix_fadvise(f->fd, 0, 0, POSIX_FADV_DONTNEED) ? 1 : 0;
}

WEXB_API int wexb_file_read(WexbFile *f, int n, const unsigned int *layer, const unsigned int *expert, int check,
                            int *status, unsigned long long *bytes) {
    if (!f || n < 0 || (n && (!layer || !expert || !status))) return -1;
    if (bytes) *bytes = 0;
    if (!n) return 0;
    std::lock_guard<std::mutex> lock(f->call_mu);
    Work w = resolve(*f, n, layer, expert, status);
    if (!w.rec.empty() && !f->alloc_ring()) {
        for (int i : w.who) status[i] = 1;
        w.rec.clear();
    }
    const size_t nb = w.batches();
    for (size_t b = 0; b < nb && b < (size_t)kSlots; ++b) f->issue((int)(b % kSlots), &w.rec[b * kBatch], w.size(b));
    unsigned long long got = 0;
    for (size_t b = 0; b < nb; ++b) {
        const int s = (int)(b % kSlots), k = w.size(b);
        f->wait_reads(s);
        for (int j = 0; j < k; ++j) {
            const size_t q = b * kBatch + (size_t)j;
            const FileExpert &e = f->idx.records[w.rec[q]];
            int &st = status[w.who[q]];
            st = f->gates[s].bad[j] ? 1 : 0;
            if (!st && check) {   // SHA-256 of the stored bytes against the index
                uint8_t d[32];
                host_sha256(f->slot(s) + (size_t)j * f->slot_rec, e.stored, d);
                if (std::memcmp(d, e.sha, 32)) st = -1;
            }
            if (!st) got += e.stored;
        }
        if (b + kSlots < nb) f->issue(s, &w.rec[(b + kSlots) * kBatch], w.size(b + kSlots));
    }
    if (bytes) *bytes = got;
    int bad = 0;
    for (int i = 0; i < n; ++i) bad += status[i] != 0;
    return bad;
}

WEXB_API int wexb_file_decode(WexbFile *f, int device, int n, const unsigned int *layer, const unsigned int *expert,
                              unsigned char *const *dst_scale, unsigned char *const *dst_weight, int *status) {
    if (!f || n < 0 || (n && (!layer || !expert || !dst_scale || !dst_weight || !status))) return -1;
    if (!n) return 0;
    std::lock_guard<std::mutex> lock(f->call_mu);
    Work w = resolve(*f, n, layer, expert, status);
    if (!w.rec.empty() && (f->stuck || !f->alloc_ring() || !f->bind(device))) {
        for (int i : w.who) status[i] = 1;
        w.rec.clear();
    }
    const size_t nb = w.batches();
    std::vector<int> ticket(nb, -1);
    std::vector<std::vector<int>> queued(nb);   // request index of each record of a queued call
    std::vector<int> raw;                       // requests copied as RAW records
    bool raw_ok = true;
    auto retire = [&](size_t b) {
        if (ticket[b] < 0) return;
        int st[kBatch];
        wexb_batch_wait(ticket[b], st);
        for (size_t j = 0; j < queued[b].size(); ++j) status[queued[b][j]] = st[j];
        ticket[b] = -1;
    };
    for (size_t b = 0; b < nb && b < (size_t)kSlots; ++b) f->issue((int)(b % kSlots), &w.rec[b * kBatch], w.size(b));
    size_t issued = std::min(nb, (size_t)kSlots), done_at = nb;
    for (size_t b = 0; b < nb; ++b) {
        const int s = (int)(b % kSlots), k = w.size(b);
        f->wait_reads(s);
        const WexEntry *ents[kBatch];
        const unsigned char *recs[kBatch];
        unsigned char *ds[3 * kBatch], *dw[3 * kBatch];
        int q = 0;
        for (int j = 0; j < k; ++j) {
            const size_t at = b * kBatch + (size_t)j;
            const int i = w.who[at];
            const FileExpert &e = f->idx.records[w.rec[at]];
            const uint8_t *p = f->slot(s) + (size_t)j * f->slot_rec;
            if (f->gates[s].bad[j]) { status[i] = 1; continue; }
            if (e.codec == WEX_ENTRY_RAW) {   // the stored bytes are the slab: six region copies
                const uint32_t *so = e.entry.scale_offsets, *wo = e.entry.weight_offsets;
                for (int m = 0; m < 3 && raw_ok; ++m) {
                    const size_t sb = (size_t)e.entry.scale_shapes[m][0] * e.entry.scale_shapes[m][1];
                    const size_t wb = (size_t)e.entry.weight_shapes[m][0] * e.entry.weight_shapes[m][1];
                    raw_ok = cudaMemcpyAsync(dst_scale[3 * i + m], p + so[m], sb, cudaMemcpyHostToDevice, f->raw_st) == cudaSuccess &&
                             cudaMemcpyAsync(dst_weight[3 * i + m], p + wo[m], wb, cudaMemcpyHostToDevice, f->raw_st) == cudaSuccess;
                }
                raw.push_back(i);
                continue;
            }
            // WNR3: the record header against the index (c/wex4.h:685-697)
            if (rd32(p + 28) != e.owner || !(p[27] & 8) != !e.value_exact || rd32(p + 4) != e.model) { status[i] = -1; continue; }
            ents[q] = &e.entry; recs[q] = p;
            for (int m = 0; m < 3; ++m) { ds[3 * q + m] = dst_scale[3 * i + m]; dw[3 * q + m] = dst_weight[3 * i + m]; }
            queued[b].push_back(i);
            ++q;
        }
        if (q) {
            ticket[b] = wexb_batch_submit(q, ents, recs, device, ds, dw);
            if (ticket[b] < 0) { for (int i : queued[b]) status[i] = 1; queued[b].clear(); }
        }
        if (cudaEventRecord(f->raw_done[s], f->raw_st) != cudaSuccess) { (void)cudaGetLastError(); raw_ok = false; }
        if (b + kSlots < nb) {   // the slot is read again once its uploads have landed (bounded waits)
            const bool uploaded = ticket[b] < 0 || batch_uploads_wait(ticket[b]);
            const Waited copied = wait_event(f->raw_done[s]);
            if (copied != Waited::Done) raw_ok = false;
            if (!uploaded || copied != Waited::Done) {   // the slot may still be read: stop here
                f->stuck = true;
                done_at = b + 1;
                break;
            }
            f->issue(s, &w.rec[(b + kSlots) * kBatch], w.size(b + kSlots));
            ++issued;
        }
        if (b >= (size_t)kInflight) retire(b - kInflight);
    }
    for (size_t b = done_at; b < issued; ++b) f->wait_reads((int)(b % kSlots));   // reads already handed out
    for (size_t b = done_at; b < nb; ++b)
        for (int j = 0; j < w.size(b); ++j) status[w.who[b * kBatch + (size_t)j]] = 1;
    for (size_t b = 0; b < nb; ++b) retire(b);
    if (!raw.empty()) {
        const Waited copied = wait_stream(f->raw_st);
        if (copied == Waited::TimedOut) f->stuck = true;
        if (copied != Waited::Done) raw_ok = false;
    }
    for (int i : raw) status[i] = raw_ok ? 0 : 1;
    int bad = 0;
    for (int i = 0; i < n; ++i) bad += status[i] != 0;
    return bad;
}
