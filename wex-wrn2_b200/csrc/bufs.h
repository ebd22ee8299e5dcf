// Grown device / page-locked host buffers (reused by every call that owns them; never shrunk).
#pragma once
#include <cuda_runtime.h>

#include <algorithm>
#include <cstddef>
#include <cstdint>

namespace wexb {

struct DevBuf {
    uint8_t *p = nullptr;
    size_t cap = 0;
    bool grow(size_t n) {
        if (n <= cap) return true;
        if (p) cudaFree(p);
        p = nullptr; cap = 0;
        if (cudaMalloc(&p, std::max<size_t>(n, 256)) != cudaSuccess) { (void)cudaGetLastError(); return false; }
        cap = n;
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
        p = nullptr; cap = 0;
        if (cudaMallocHost(&p, std::max<size_t>(n, 256)) != cudaSuccess) { (void)cudaGetLastError(); return false; }
        cap = n;
        return true;
    }
    void release() { if (p) cudaFreeHost(p); p = nullptr; cap = 0; }
};

}  // namespace wexb
