// jepa_b200_gemm_noalloc: the planner's tcgen05 3xTF32 GEMM for callers that cannot allocate device
// memory (see include/jepa_b200.h). Its device working set -- the copies of A, B and C and the hi / lo
// split planes of both operands -- lives in one file-scope device array of a fixed size, so the call
// makes no cudaMalloc / cudaFree. Host code never passes the array's name to a kernel (in host code
// that name is only a stand-in for the symbol); it passes the per-device address that
// cudaGetSymbolAddress returns, looked up once per device with that device current.
#include "kernels.h"
#include "common.h"
#include "../../include/jepa_b200.h"

#include <mutex>

namespace {

constexpr size_t SCRATCH_FLOATS = JEPA_B200_NOALLOC_MAX_FLOATS;
__device__ __align__(256) float g_noalloc_scratch[SCRATCH_FLOATS];

constexpr int MAX_DEVICES = 128;
std::mutex g_mu;
float * g_scratch_ptr[MAX_DEVICES] = {};

// this device's address of the array (looked up on the first call made on the device)
float * scratch_of_current_device() {
    int dev = 0;
    if (!jb::cuda_ok(cudaGetDevice(&dev), "cudaGetDevice")) return nullptr;
    if (dev < 0 || dev >= MAX_DEVICES) { jb::log("jepa: jepa_b200_gemm_noalloc: device %d is out of range\n", dev); return nullptr; }
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_scratch_ptr[dev]) {
        void * p = nullptr;
        if (!jb::cuda_ok(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress")) return nullptr;
        g_scratch_ptr[dev] = (float *) p;
    }
    return g_scratch_ptr[dev];
}

size_t round64(size_t n) { return (n + 63) & ~(size_t) 63; }

}  // namespace

extern "C" int jepa_b200_gemm_noalloc(const float * A, const float * B, int M, int N, int K, float * C) {
    if (!A || !B || !C || M < 1 || N < 1 || K < 1 || (K & 3)) {
        jb::log("jepa: jepa_b200_gemm_noalloc: need host buffers and M, N, K >= 1 with K a multiple of 4\n");
        return -1;
    }
    const size_t mk = round64((size_t) M * K), nk = round64((size_t) N * K), mn = round64((size_t) M * N);
    const size_t need = 3 * mk + 3 * nk + mn;
    if (need > SCRATCH_FLOATS) {
        jb::log("jepa: jepa_b200_gemm_noalloc: M %d N %d K %d needs %zu floats of device scratch, the fixed array holds %zu "
                "(3 (M K + N K) + M N must stay within JEPA_B200_NOALLOC_MAX_FLOATS)\n", M, N, K, need, SCRATCH_FLOATS);
        return -1;
    }
    float * s = scratch_of_current_device();
    if (!s) return -1;
    float * a = s, * a_hi = a + mk, * a_lo = a_hi + mk;
    float * b = a_lo + mk, * b_hi = b + nk, * b_lo = b_hi + nk;
    float * c = b_lo + nk;
    cudaStream_t st = 0;   // the legacy default stream: no stream object to create
    // a timeout flag left by an earlier call that failed before reading it must not fail this one
    if (jb::gemm_error_clear(st) != 0) return -1;
    JB_CUDA(cudaMemcpyAsync(a, A, (size_t) M * K * 4, cudaMemcpyHostToDevice, st));
    JB_CUDA(cudaMemcpyAsync(b, B, (size_t) N * K * 4, cudaMemcpyHostToDevice, st));
    // every element the kernels read is written first (the split planes, then C in full), so stale
    // contents left by an earlier call need no clearing
    jb::split_f32(a, K, a_hi, a_lo, K, M, K, st);
    jb::split_f32(b, K, b_hi, b_lo, K, N, K, st);
    // a launch that failed (configuration errors are not sticky, so the synchronise below would not
    // report it) would leave the GEMM reading the split planes of the previous call
    JB_CUDA(cudaGetLastError());
    jb::GemmEpi ep;
    ep.mode = jb::EPI_F32;
    ep.out0 = c;
    ep.ld0 = N;
    if (jb::gemm_tc({a_hi, a_lo, K}, {b_hi, b_lo, K}, M, N, K, ep, st) != 0) return -1;
    JB_CUDA(cudaMemcpyAsync(C, c, (size_t) M * N * 4, cudaMemcpyDeviceToHost, st));
    JB_CUDA(cudaStreamSynchronize(st));
    if (jb::gemm_error_flag(st) != 0) {
        jb::log("jepa: jepa_b200_gemm_noalloc: the tensor-core kernel timed out waiting on its pipeline (or its flag could not be read)\n");
        return -1;
    }
    return 0;
}
