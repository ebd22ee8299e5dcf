// Host parsers of the library under AddressSanitizer / UndefinedBehaviorSanitizer: every container
// given on the command line, and seeded mutants of it, go through the WEX4 header and index checks
// (wex4_validate, wex4_expert_table, wex4_check without decode, the file reader's index parse), and
// every record's stored bytes, and mutants of them, through the record parsers the GPU paths run
// before a launch (WNR2/WNR3 plan_record, WBP1 wbp1_parse, WNR4 kind-MX wnr4_plan). Verdicts are not
// compared here (the parity tests do that); the run fails only if a sanitizer reports an error.
//
//   fuzz_host SEED MUTANTS FILE...      prints the number of parser runs, then the record parses by codec
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <vector>

#include "nr3_host.h"
#include "wbp1_host.h"
#include "wex4_index.h"
#include "wex4_tools.h"
#include "wnr4_host.h"

using namespace wexb;

extern "C" int wex4_validate(const unsigned char *page, uint64_t file_bytes, const unsigned char *index, size_t index_len);
extern "C" int wex4_expert_table(const unsigned char *page, uint64_t file_bytes, const unsigned char *index,
                                 size_t index_len, unsigned char *out);
extern "C" int wex4_check(const unsigned char *file, uint64_t len, int flags, unsigned char *digest);

namespace {

uint64_t u64(const std::vector<uint8_t> &b, size_t at) {
    uint64_t v = 0;
    if (at + 8 <= b.size()) std::memcpy(&v, b.data() + at, 8);
    return v;
}
uint32_t u32(const std::vector<uint8_t> &b, size_t at) {
    uint32_t v = 0;
    if (at + 4 <= b.size()) std::memcpy(&v, b.data() + at, 4);
    return v;
}

// The container-level checks on one file image (any bytes).
void containers(const std::vector<uint8_t> &f) {
    if (f.size() < 4096) { (void)wex4_check(f.data(), f.size(), 0, nullptr); return; }
    const uint64_t index_offset = u64(f, 32), index_bytes = u64(f, 40);
    const uint64_t index_len = (index_bytes + 4095) & ~4095ull;
    std::vector<uint8_t> index(index_len < (1u << 28) ? index_len : 0, 0);
    if (index_offset < f.size() && !index.empty())
        std::memcpy(index.data(), f.data() + index_offset, std::min<uint64_t>(index.size(), f.size() - index_offset));
    (void)wex4_validate(f.data(), f.size(), index.data(), index.size());
    const uint32_t layers = u32(f, 60), experts = u32(f, 64);
    if ((uint64_t)layers * experts <= (1u << 16)) {
        std::vector<uint8_t> table((size_t)layers * experts * 72 + 72);
        (void)wex4_expert_table(f.data(), f.size(), index.data(), index.size(), table.data());
    }
    (void)wex4_check(f.data(), f.size(), 0, nullptr);
    FileIndex fi;
    if (!file_header(f.data(), f.size(), &fi) && fi.index_len == index.size()) (void)file_index(f.data(), index.data(), &fi);
}

// The record parsers on one record of a valid container: its stored bytes s (any bytes).
struct Rec {
    uint32_t codec, owner, decoded;
    bool expert;
    WexEntry entry;
    uint32_t geo[13];
};
size_t g_by_codec[16];
void records(const Rec &r, const std::vector<uint8_t> &s) {
    ++g_by_codec[r.codec & 15];
    if (r.codec == 4 || r.codec == 5) {
        WexEntry e = r.entry;
        e.total_bytes = (uint32_t)s.size();
        Plan p;
        (void)plan_record(&e, s.data(), &p);
    } else if (r.codec == 6) {
        Wbp1Plan p;
        (void)wbp1_parse(s.data(), s.size(), r.decoded, r.owner, &p);
    } else if (r.codec == 8) {
        W4Geo g;
        if (!wnr4_geo(r.geo, &g)) return;
        W4Rec info;
        std::vector<W4Job> jobs[3];
        (void)wnr4_plan(s.data(), s.size(), g, r.owner, u32(s, 4), s.data(), 0, &info, jobs);
    }
}

// The records of a container that validates, with what the parsers need from the index.
std::vector<std::pair<Rec, std::vector<uint8_t>>> list_records(const std::vector<uint8_t> &f) {
    std::vector<std::pair<Rec, std::vector<uint8_t>>> out;
    const uint64_t io = u64(f, 32), index_bytes = u64(f, 40);
    const uint32_t nblobs = u32(f, 48), nrec = u32(f, 52), ntens = u32(f, 56), experts = u32(f, 64);
    std::vector<uint8_t> index(f.begin() + (long)io, f.begin() + (long)(io + ((index_bytes + 4095) & ~4095ull)));
    const uint32_t layers = u32(f, 60);
    std::vector<uint8_t> table((size_t)layers * experts * 72 + 72);
    if (wex4_expert_table(f.data(), f.size(), index.data(), index.size(), table.data())) table.clear();
    const size_t rows = io + 64ull * nblobs, tens = rows + 72ull * nrec;
    for (uint32_t i = 0; i < nrec; ++i) {
        const size_t at = rows + 72ull * i;
        Rec r{};
        const uint64_t off = u64(f, at);
        const uint32_t stored = u32(f, at + 8);
        r.decoded = u32(f, at + 12);
        r.codec = u32(f, at + 16) & 0xffff;
        r.expert = (u32(f, at + 16) >> 16) & 2;
        r.owner = u32(f, at + 24);
        const uint32_t first = u32(f, at + 28);
        if (r.expert && !table.empty())
            std::memcpy(&r.entry, table.data() + ((size_t)(r.owner >> 16) * experts + (r.owner & 0xffff)) * 72, 72);
        if (r.codec == 8 && first + 6 <= ntens) {   // geometry from the six tensor rows
            r.geo[0] = 0;
            for (int m = 0; m < 3; ++m) {
                const size_t s = tens + 96ull * (first + m), w = tens + 96ull * (first + 3 + m);
                const uint64_t rws = u64(f, s + 8), cols = u64(f, s + 16);
                r.geo[1 + m] = (uint32_t)(rws * cols); r.geo[4 + m] = (uint32_t)cols;
                r.geo[7 + m] = (uint32_t)u64(f, s + 80); r.geo[10 + m] = (uint32_t)u64(f, w + 80);
            }
        }
        if (off + stored <= f.size()) out.push_back({r, std::vector<uint8_t>(f.begin() + (long)off, f.begin() + (long)(off + stored))});
    }
    return out;
}

void mutate(std::vector<uint8_t> &b, std::mt19937_64 &rng, size_t lo, size_t hi) {
    if (hi <= lo) return;
    const int flips = 1 + (int)(rng() % 4);
    for (int k = 0; k < flips; ++k) b[lo + rng() % (hi - lo)] ^= (uint8_t)(1u << (rng() % 8));
}

}  // namespace

int main(int argc, char **argv) {
    if (argc < 4) { std::fprintf(stderr, "usage: %s SEED MUTANTS FILE...\n", argv[0]); return 2; }
    std::mt19937_64 rng(std::strtoull(argv[1], nullptr, 10));
    const int mutants = std::atoi(argv[2]);
    size_t runs = 0;
    for (int a = 3; a < argc; ++a) {
        FILE *fp = std::fopen(argv[a], "rb");
        if (!fp) { std::fprintf(stderr, "cannot open %s\n", argv[a]); return 2; }
        std::vector<uint8_t> f;
        uint8_t buf[1 << 16];
        size_t n;
        while ((n = std::fread(buf, 1, sizeof buf, fp)) > 0) f.insert(f.end(), buf, buf + n);
        std::fclose(fp);
        containers(f);
        ++runs;
        const bool valid = f.size() >= 4096 && !wex4_check(f.data(), f.size(), 0, nullptr);
        for (int k = 0; k < mutants; ++k) {   // the file: anywhere, then the header page and index only
            std::vector<uint8_t> m = f;
            const size_t head = std::min<size_t>(f.size(), 4096 + ((u64(f, 40) + 4095) & ~4095ull));
            mutate(m, rng, 0, (k & 1) ? head : m.size());
            if ((k % 7) == 3) m.resize(rng() % (m.size() + 1));   // truncated
            containers(m);
            ++runs;
        }
        if (!valid) continue;
        for (auto &rs : list_records(f)) {
            records(rs.first, rs.second);
            ++runs;
            for (int k = 0; k < mutants; ++k) {   // a record: its header and tables, then anywhere
                std::vector<uint8_t> m = rs.second;
                mutate(m, rng, 0, (k & 1) ? std::min<size_t>(m.size(), 4096) : m.size());
                records(rs.first, m);
                ++runs;
            }
        }
    }
    std::printf("%zu parser runs; record parses by codec: 0 %zu, 5 %zu, 6 %zu, 8 %zu\n", runs, g_by_codec[0],
                g_by_codec[5], g_by_codec[6], g_by_codec[8]);
    return 0;
}
