// The decode launch's work queue (queue_fill, nr3_host.cpp) against the rules the kernel's items wait
// by (wnr3.cuh): a weight item of matrix m of a record waits for every scale item of that matrix of
// that record, and a commit item for every weight item of its record. Each wait is for items earlier in
// the queue, so the queue always drains; this checks that on seeded random launches (record shapes,
// chunk sizes, SM counts, scale leads, with and without commits), and that every stream and every
// commit chunk is covered exactly once and the descriptors' item counts match the queue.
//
//   queue_order SEED LAUNCHES      prints the number of items checked; exits non-zero on a violation
#include <cstdio>
#include <cstdlib>
#include <random>
#include <set>
#include <tuple>
#include <vector>

#include "nr3_host.h"

using namespace wexb;

namespace {

int fail(const char *what, uint32_t launch, uint32_t at) {
    std::fprintf(stderr, "launch %u, item %u: %s\n", launch, at, what);
    return 1;
}

// A plan with the shape fields queue_fill and plan_descriptor read (the rest is not used by them).
Plan random_plan(std::mt19937_64 &rng) {
    static const uint32_t wchunks[] = {512, 1024, 2048, 4096, 16384};
    static const uint32_t schunks[] = {256, 512, 1024, 16384};
    Plan p{};
    p.wchunk = wchunks[rng() % 5];
    p.schunk = schunks[rng() % 4];
    for (int m = 0; m < 3; ++m) {
        const uint32_t rows = 1 + (uint32_t)(rng() % 3000), cols = 1 + (uint32_t)(rng() % 80);   // scales
        p.scount[m] = rows * cols;
        p.wcount[m] = 32u * p.scount[m];
        p.dst_bytes[m] = p.scount[m];
        p.dst_bytes[3 + m] = p.wcount[m] / 2u;
    }
    return p;
}

}  // namespace

int main(int argc, char **argv) {
    if (argc < 3) { std::fprintf(stderr, "usage: %s SEED LAUNCHES\n", argv[0]); return 2; }
    std::mt19937_64 rng(std::strtoull(argv[1], nullptr, 10));
    const uint32_t launches = (uint32_t)std::atoi(argv[2]);
    size_t checked = 0;
    for (uint32_t L = 0; L < launches; ++L) {
        const uint32_t n = 1 + (uint32_t)(rng() % 24);
        const bool commit = rng() & 1;
        const int sms = (int)(1 + rng() % 160);
        const uint32_t leads[] = {1u, 2u, 5u, kScalesFirst};
        const uint32_t lead = leads[rng() % 4];
        std::vector<Plan> plans(n);
        std::vector<const Plan *> ptr(n);
        for (uint32_t r = 0; r < n; ++r) { plans[r] = random_plan(rng); ptr[r] = &plans[r]; }
        uint32_t expect = 0;
        for (uint32_t r = 0; r < n; ++r) expect += queue_items(plans[r], commit);
        std::vector<Nr3Item> items(expect + 1);
        const uint32_t got = queue_fill(ptr.data(), n, commit, sms, lead, items.data());
        if (got != expect) return fail("queue_fill wrote a different number of items than queue_items counts", L, got);
        // descriptors: items per matrix / record as the kernel's waits count them
        std::vector<Nr3Record> desc(n);
        for (uint32_t r = 0; r < n; ++r) plan_descriptor(plans[r], nullptr, nullptr, nullptr, nullptr, nullptr, &desc[r]);
        std::vector<uint32_t> scales_done(3 * n, 0), weights_done(n, 0);
        std::set<std::tuple<uint32_t, uint32_t, uint32_t, uint32_t>> seen;   // (record, kind, sub, first)
        for (uint32_t at = 0; at < got; ++at) {
            const Nr3Item it = items[at];
            const uint32_t kind = it.what >> 28, sub = (it.what >> 24) & 15u, first = it.what & 0xffffffu;
            if (it.rec >= n) return fail("record index out of range", L, at);
            if (!seen.insert({it.rec, kind, sub, first}).second) return fail("item repeated", L, at);
            const Plan &p = plans[it.rec];
            const Nr3Record &R = desc[it.rec];
            if (kind == kItemScale) {
                if (sub > 2 || first % 32u || first >= (p.scount[sub] + p.schunk - 1) / p.schunk) return fail("bad scale item", L, at);
                ++scales_done[3 * it.rec + sub];
            } else if (kind == kItemWeight) {
                if (sub > 2 || first % 32u || first >= (p.wcount[sub] + p.wchunk - 1) / p.wchunk) return fail("bad weight item", L, at);
                if (scales_done[3 * it.rec + sub] != R.sitems[sub]) return fail("a weight item before its matrix's scales", L, at);
                ++weights_done[it.rec];
            } else if (kind == kItemCommit) {
                if (!commit || sub > 5 || (size_t)first * kCommitChunk >= p.dst_bytes[sub]) return fail("bad commit item", L, at);
                if (weights_done[it.rec] != R.witems) return fail("a commit item before its record's weights", L, at);
            } else {
                return fail("unknown item kind", L, at);
            }
            ++checked;
        }
        for (uint32_t r = 0; r < n; ++r) {
            for (int m = 0; m < 3; ++m)
                if (scales_done[3 * r + m] != desc[r].sitems[m]) return fail("scale items missing", L, r);
            if (weights_done[r] != desc[r].witems) return fail("weight items missing", L, r);
        }
    }
    std::printf("%zu\n", checked);
    return 0;
}
