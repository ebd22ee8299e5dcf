// Grown device / page-locked host buffers (reused by every call that owns them; never shrunk). They
// grow geometrically: a reallocation frees the old buffer, and cudaFree waits for the whole device,
// so a pipeline of calls of slowly rising sizes must not reallocate on every call.
#pragma once
#include <cuda_runtime.h>

#include <algorithm>
#include <cstddef>
#include <cstdint>

namespace wexb {

// New capacity for n bytes after `cap`: at least 1.5 x cap, rounded up to 64 KiB.
inline size_t grown(size_t cap, size_t n) {
    const size_t want = std::max(n, cap + cap / 2);
    return (want + 65535) & ~(size_t)65535;
}

struct DevBuf {
    uint8_t *p = nullptr;
    size_t cap = 0;
    bool grow(size_t n) {
        if (n <= cap) return true;
        if (p) cudaFree(p);
        p = nullptr;
        const size_t want = grown(cap, n);
        cap = 0;
        if (cudaMalloc(&p, want) != cudaSuccess) { (void)cudaGetLastError(); return false; }
        cap = want;
        return true;
    }
    void release() { if (p) cudaFree(p); p = nullptr; cap = 0; }
};
struct PinBuf {
    uint8_t *p = nullptr;
    size_t cap = 0;
    bool grow(size_t n) {
        if (n <= cap) return true;
        if (p) cudaFreeHost(p);
        p = nullptr;
        const size_t want = grown(cap, n);
        cap = 0;
        if (cudaMallocHost(&p, want) != cudaSuccess) { (void)cudaGetLastError(); return false; }
        cap = want;
        return true;
    }
    void release() { if (p) cudaFreeHost(p); p = nullptr; cap = 0; }
};

}  // namespace wexb
