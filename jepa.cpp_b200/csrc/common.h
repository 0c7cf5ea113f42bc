// Shared host-side helpers: diagnostics (stderr + the thread-local capture buffer behind
// jepa_error_text), CUDA error checks that turn a failed call into a logged -1, and small device
// buffer utilities.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>
#include <vector>

namespace jb {

// stderr + the calling thread's capture buffer (reference contract: include/jepa.h:597-611,
// src/jepa.cpp:16-36)
void log(const char * fmt, ...) __attribute__((format(printf, 1, 2)));

// true when `e` is cudaSuccess; otherwise logs "<what>: <cuda error>" and returns false
bool cuda_ok(cudaError_t e, const char * what);

#define JB_CUDA(call) do { if (!::jb::cuda_ok((call), #call)) return -1; } while (0)
#define JB_CUDA_B(call) do { if (!::jb::cuda_ok((call), #call)) return false; } while (0)

// One device allocation that is carved into aligned sub-buffers (a workspace). Freed as a whole.
struct Arena {
    char * base = nullptr;
    size_t size = 0, used = 0;
    int device = -1;
    ~Arena() { release(); }
    void release() {
        if (base) { cudaSetDevice(device); cudaFree(base); }
        base = nullptr; size = used = 0;
    }
    bool reserve(size_t bytes, int dev) {
        release();
        device = dev;
        if (bytes == 0) return true;
        if (cudaMalloc((void **) &base, bytes) != cudaSuccess) {
            cudaGetLastError();
            log("jepa: could not allocate %.1f MiB of device memory for the planner workspace\n", bytes / 1048576.0);
            base = nullptr;
            return false;
        }
        size = bytes;
        used = 0;
        return true;
    }
    template <class T> T * take(size_t n) {
        const size_t bytes = (n * sizeof(T) + 255) & ~(size_t) 255;
        if (!base || used + bytes > size) return nullptr;
        T * p = (T *) (base + used);
        used += bytes;
        return p;
    }
};

// Byte count of a carve plan, computed before the allocation is made.
struct ArenaPlan {
    size_t bytes = 0;
    template <class T> void add(size_t n) { bytes += (n * sizeof(T) + 255) & ~(size_t) 255; }
};

}  // namespace jb
