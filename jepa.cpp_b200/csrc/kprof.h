// Per-kernel device timing for measurement runs: while enabled (jepa_b200_kprof_begin / _end), every
// instrumented launch is bracketed by two CUDA events on its stream and booked under a kind name with
// its algorithmic FLOPs and bytes. Disabled, a KTimer costs one load of a global flag.
#pragma once

#include <cuda_runtime.h>

namespace jb {

extern bool g_kprof_on;

struct KTimer {
    cudaEvent_t e0 = nullptr;
    cudaStream_t st = nullptr;
    const char * kind = nullptr;
    double flops = 0, bytes = 0;
    KTimer(const char * kind, cudaStream_t st, double flops = 0, double bytes = 0);
    ~KTimer();
};

}  // namespace jb
