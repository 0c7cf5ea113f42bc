// Kernel-level entry points of include/jepa_b200.h: the planner's GEMM and dequantisation kernels
// reached through the C ABI with host buffers, for parity tests and isolated timing.
#include "kernels.h"
#include "common.h"
#include "gguf.h"
#include "../../include/jepa_b200.h"

#include <vector>

namespace {

struct DevBuf {
    void * p = nullptr;
    ~DevBuf() { if (p) cudaFree(p); }
    bool alloc(size_t bytes) { return cudaMalloc(&p, bytes) == cudaSuccess; }
    float * f() const { return (float *) p; }
};

__global__ void k_fill_h(__half * p, size_t n, uint32_t seed, float scale) {
    for (size_t i = blockIdx.x * (size_t) blockDim.x + threadIdx.x; i < n; i += (size_t) gridDim.x * blockDim.x) {
        uint32_t h = (uint32_t) i * 2654435761u ^ seed;
        h ^= h >> 15; h *= 2246822519u; h ^= h >> 13;
        p[i] = __float2half_rn(((float) (h & 0xffff) / 65535.0f - 0.5f) * scale);
    }
}

__global__ void k_h2f(const __half * x, float * y, size_t n) {
    for (size_t i = blockIdx.x * (size_t) blockDim.x + threadIdx.x; i < n; i += (size_t) gridDim.x * blockDim.x) y[i] = __half2float(x[i]);
}

// split planes of a host matrix, uploaded
bool upload_split(const float * h, size_t n, DevBuf & raw, DevBuf & hi, DevBuf & lo, int rows, int cols, cudaStream_t st) {
    if (!raw.alloc(n * 4) || !hi.alloc(n * 4) || !lo.alloc(n * 4)) return false;
    if (cudaMemcpyAsync(raw.p, h, n * 4, cudaMemcpyHostToDevice, st) != cudaSuccess) return false;
    jb::split_f32(raw.f(), cols, hi.f(), lo.f(), cols, rows, cols, st);
    return true;
}

}  // namespace

extern "C" const char * jepa_b200_version(void) { return "jepa-b200 0.1.0"; }

namespace {

// fix-up scratch for the GEMM's K split (the planner's configuration): partial tiles and zeroed counters
bool alloc_fixup(DevBuf & fix, DevBuf & cnt, int M, int N, int K, jb::GemmEpi & ep, cudaStream_t st) {
    const size_t nf = jb::gemm_fixup_floats(M, N, K), nc = jb::gemm_fixup_counters(M, N, K);
    if (!nf) return true;
    if (!fix.alloc(nf * 4) || !cnt.alloc(nc * sizeof(int))) return false;
    if (cudaMemsetAsync(cnt.p, 0, nc * sizeof(int), st) != cudaSuccess) return false;
    ep.fix = fix.f();
    ep.fix_floats = nf;
    ep.fix_count = (int *) cnt.p;
    ep.fix_counters = nc;
    return true;
}

int gemm_host(const float * A, const float * B, int M, int N, int K, float * C, bool ksplit, const char * fn) {
    if (!A || !B || !C || M < 1 || N < 1 || K < 1 || (K & 3)) {
        jb::log("jepa: %s: need host buffers and M, N, K >= 1 with K a multiple of 4\n", fn);
        return -1;
    }
    cudaStream_t st;
    JB_CUDA(cudaStreamCreate(&st));
    if (jb::gemm_error_clear(st) != 0) { cudaStreamDestroy(st); return -1; }
    DevBuf ar, ah, al, br, bh, bl, c, fix, cnt;
    int rc = -1;
    jb::GemmEpi ep;
    if (upload_split(A, (size_t) M * K, ar, ah, al, M, K, st) && upload_split(B, (size_t) N * K, br, bh, bl, N, K, st) &&
        c.alloc((size_t) M * N * 4) && (!ksplit || alloc_fixup(fix, cnt, M, N, K, ep, st))) {
        ep.mode = jb::EPI_F32;
        ep.out0 = c.f();
        ep.ld0 = N;
        rc = jb::gemm_tc({ah.f(), al.f(), K}, {bh.f(), bl.f(), K}, M, N, K, ep, st);
        if (rc == 0 && !jb::cuda_ok(cudaMemcpyAsync(C, c.p, (size_t) M * N * 4, cudaMemcpyDeviceToHost, st), "copy C")) rc = -1;
        if (rc == 0 && !jb::cuda_ok(cudaStreamSynchronize(st), "gemm")) rc = -1;
        if (rc == 0 && jb::gemm_error_flag(st) != 0) {
            jb::log("jepa: %s: the tensor-core kernel timed out waiting on its pipeline\n", fn);
            rc = -1;
        }
    } else {
        jb::log("jepa: %s: device allocation or upload failed\n", fn);
    }
    cudaStreamDestroy(st);
    return rc;
}

}  // namespace

extern "C" int jepa_b200_gemm(const float * A, const float * B, int M, int N, int K, float * C) {
    return gemm_host(A, B, M, N, K, C, false, "jepa_b200_gemm");
}

extern "C" int jepa_b200_gemm_ksplit(const float * A, const float * B, int M, int N, int K, float * C) {
    return gemm_host(A, B, M, N, K, C, true, "jepa_b200_gemm_ksplit");
}

extern "C" int jepa_b200_gemm_plan(int M, int N, int K, int * out) {
    if (!out || M <= 0 || N <= 0 || K <= 0) return -1;
    const jb::GemmPlan p = jb::gemm_plan(M, N, K);
    out[0] = p.persistent ? 1 : 0;
    out[1] = p.k_parts;
    out[2] = p.m_fast;
    return 0;
}

extern "C" int jepa_b200_gemm_tile_walk(int M, int N, int K, int * m0, int * n0, int cap) {
    if (!m0 || !n0 || cap < 0 || M <= 0 || N <= 0 || K <= 0) return -1;
    return jb::gemm_tile_walk(M, N, K, m0, n0, cap);
}

namespace {

// a weight's block planes on the device, from its raw GGUF rows (host)
struct QuantWeight {
    DevBuf raw, q, qt, d;
    bool make(uint32_t type, const void * w_raw, int rows, int ne0, cudaStream_t st) {
        const size_t rb = jb::row_bytes(type, ne0);
        const size_t nq = jb::quant_plane_bytes(type, rows, ne0), nd = jb::quant_scale_count(type, rows, ne0);
        if (!rb || !nq || !raw.alloc(rb * (size_t) rows) || !q.alloc(nq) || !qt.alloc(nq) || !d.alloc(std::max<size_t>(nd, 1) * 2)) return false;
        if (cudaMemcpyAsync(raw.p, w_raw, rb * (size_t) rows, cudaMemcpyHostToDevice, st) != cudaSuccess) return false;
        return jb::quant_planes(type, raw.p, rows, ne0, q.p, qt.p, (uint16_t *) d.p, st) == 0;
    }
    jb::SplitMat operand(uint32_t type, int transposed) const {
        jb::SplitMat m;
        m.q.fmt = type == 8 ? jb::QF_Q8 : type == 2 ? jb::QF_Q4 : jb::QF_F16;
        m.q.orient = transposed ? 1 : 0;
        m.q.q = transposed ? qt.p : q.p;
        m.q.d = type == 1 ? nullptr : (const uint16_t *) d.p;
        return m;
    }
};

}  // namespace

// C = A W^T (transposed = 0: A [M][ne0], C [M][rows]) or C = A W (transposed = 1: A [M][rows], C [M][ne0]),
// W [rows][ne0] the raw rows of a GGUF weight of `type` (8 q8_0, 2 q4_0, 1 f16), read by the GEMM in its
// block planes and dequantised in the mainloop. ksplit = 1: the planner's K-split configuration.
extern "C" int jepa_b200_gemm_quant(uint32_t type, const void * w_raw, int rows, int ne0, int transposed, const float * A, int M,
                                    float * C, int ksplit) {
    if (!w_raw || !A || !C || M < 1 || !jb::quant_ok(type, rows, ne0)) {
        jb::log("jepa: jepa_b200_gemm_quant: need host buffers, M >= 1 and a q8_0 / q4_0 / f16 weight in whole 32 x 32 blocks\n");
        return -1;
    }
    const int N = transposed ? ne0 : rows, K = transposed ? rows : ne0;
    cudaStream_t st;
    JB_CUDA(cudaStreamCreate(&st));
    if (jb::gemm_error_clear(st) != 0) { cudaStreamDestroy(st); return -1; }
    QuantWeight w;
    DevBuf ar, ah, al, c, fix, cnt;
    int rc = -1;
    jb::GemmEpi ep;
    if (w.make(type, w_raw, rows, ne0, st) && upload_split(A, (size_t) M * K, ar, ah, al, M, K, st) && c.alloc((size_t) M * N * 4) &&
        (!ksplit || alloc_fixup(fix, cnt, M, N, K, ep, st))) {
        ep.out0 = c.f();
        ep.ld0 = N;
        rc = jb::gemm_tc({ah.f(), al.f(), K}, w.operand(type, transposed), M, N, K, ep, st);
        if (rc == 0 && !jb::cuda_ok(cudaMemcpyAsync(C, c.p, (size_t) M * N * 4, cudaMemcpyDeviceToHost, st), "copy C")) rc = -1;
        if (rc == 0 && !jb::cuda_ok(cudaStreamSynchronize(st), "gemm")) rc = -1;
        if (rc == 0 && jb::gemm_error_flag(st) != 0) {
            jb::log("jepa: jepa_b200_gemm_quant: the tensor-core kernel timed out waiting on its pipeline\n");
            rc = -1;
        }
    } else {
        jb::log("jepa: jepa_b200_gemm_quant: device allocation, upload or block planes failed\n");
    }
    cudaStreamDestroy(st);
    return rc;
}

// mean device time of `reps` back-to-back launches of the planner's GEMM at (M, N, K) with B a q8_0 / q4_0 /
// f16 weight in block planes (zero values), forward or transposed
extern "C" int jepa_b200_gemm_quant_bench(uint32_t type, int M, int N, int K, int transposed, int reps, double * ms) {
    const int rows = transposed ? K : N, ne0 = transposed ? N : K;
    if (M < 1 || reps < 1 || !ms || !jb::quant_ok(type, rows, ne0)) return -1;
    cudaStream_t st;
    JB_CUDA(cudaStreamCreate(&st));
    QuantWeight w;
    DevBuf ah, al, c, fix, cnt;
    int rc = -1;
    jb::GemmEpi ep;
    std::vector<uint8_t> zeros(jb::row_bytes(type, ne0) * (size_t) rows, 0);
    if (w.make(type, zeros.data(), rows, ne0, st) && ah.alloc((size_t) M * K * 4) && al.alloc((size_t) M * K * 4) &&
        c.alloc((size_t) M * N * 4) && alloc_fixup(fix, cnt, M, N, K, ep, st)) {
        cudaMemsetAsync(ah.p, 0, (size_t) M * K * 4, st);
        cudaMemsetAsync(al.p, 0, (size_t) M * K * 4, st);
        ep.out0 = c.f();
        ep.ld0 = N;
        const jb::SplitMat B = w.operand(type, transposed);
        rc = jb::gemm_tc({ah.f(), al.f(), K}, B, M, N, K, ep, st);   // warm-up
        cudaEvent_t e0, e1;
        cudaEventCreate(&e0);
        cudaEventCreate(&e1);
        cudaEventRecord(e0, st);
        for (int i = 0; i < reps && rc == 0; i++) rc = jb::gemm_tc({ah.f(), al.f(), K}, B, M, N, K, ep, st);
        cudaEventRecord(e1, st);
        if (rc == 0 && jb::cuda_ok(cudaEventSynchronize(e1), "gemm bench")) {
            float t = 0;
            cudaEventElapsedTime(&t, e0, e1);
            *ms = t / reps;
        } else {
            rc = -1;
        }
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
        if (rc == 0 && jb::gemm_error_flag(st) != 0) rc = -1;
    }
    cudaStreamDestroy(st);
    return rc;
}

extern "C" int jepa_b200_gemm_bench(int M, int N, int K, int reps, double * ms) {
    if (M < 1 || N < 1 || K < 1 || (K & 3) || reps < 1 || !ms) return -1;
    cudaStream_t st;
    JB_CUDA(cudaStreamCreate(&st));
    DevBuf ah, al, bh, bl, c, fix, cnt;
    int rc = -1;
    jb::GemmEpi ep;
    if (ah.alloc((size_t) M * K * 4) && al.alloc((size_t) M * K * 4) && bh.alloc((size_t) N * K * 4) &&
        bl.alloc((size_t) N * K * 4) && c.alloc((size_t) M * N * 4) && alloc_fixup(fix, cnt, M, N, K, ep, st)) {
        cudaMemsetAsync(ah.p, 0, (size_t) M * K * 4, st);
        cudaMemsetAsync(al.p, 0, (size_t) M * K * 4, st);
        cudaMemsetAsync(bh.p, 0, (size_t) N * K * 4, st);
        cudaMemsetAsync(bl.p, 0, (size_t) N * K * 4, st);
        ep.out0 = c.f();
        ep.ld0 = N;
        rc = jb::gemm_tc({ah.f(), al.f(), K}, {bh.f(), bl.f(), K}, M, N, K, ep, st);   // warm-up
        cudaEvent_t e0, e1;
        cudaEventCreate(&e0);
        cudaEventCreate(&e1);
        cudaEventRecord(e0, st);
        for (int i = 0; i < reps && rc == 0; i++) rc = jb::gemm_tc({ah.f(), al.f(), K}, {bh.f(), bl.f(), K}, M, N, K, ep, st);
        cudaEventRecord(e1, st);
        if (rc == 0 && jb::cuda_ok(cudaEventSynchronize(e1), "gemm bench")) {
            float t = 0;
            cudaEventElapsedTime(&t, e0, e1);
            *ms = t / reps;
        } else {
            rc = -1;
        }
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
    }
    cudaStreamDestroy(st);
    return rc;
}

// C = f16(A) f16(B)^T through the V-JEPA 2-AC tensor-core GEMM (f32 accumulate, plain f32 epilogue)
extern "C" int jepa_b200_gemm_f16(const float * A, const float * B, int M, int N, int K, float * C) {
    if (!A || !B || !C || M < 1 || N < 1 || K < 1 || (K & 7)) return -1;
    cudaStream_t st;
    JB_CUDA(cudaStreamCreate(&st));
    DevBuf a32, b32, a16, b16, c;
    int rc = -1;
    if (a32.alloc((size_t) M * K * 4) && b32.alloc((size_t) N * K * 4) && a16.alloc((size_t) M * K * 2) &&
        b16.alloc((size_t) N * K * 2) && c.alloc((size_t) M * N * 4)) {
        cudaMemcpyAsync(a32.p, A, (size_t) M * K * 4, cudaMemcpyHostToDevice, st);
        cudaMemcpyAsync(b32.p, B, (size_t) N * K * 4, cudaMemcpyHostToDevice, st);
        jb::to_f16(a32.f(), K, (__half *) a16.p, K, M, K, jb::RowMap{}, st);
        jb::to_f16(b32.f(), K, (__half *) b16.p, K, N, K, jb::RowMap{}, st);
        jb::AcGemmEpi ep;
        ep.mode = jb::AEPI_F32;
        ep.out_f32 = c.f();
        ep.ld_f32 = N;
        rc = jb::gemm_f16((const __half *) a16.p, K, (const __half *) b16.p, K, M, N, K, ep, st);
        if (rc == 0) {
            rc = jb::cuda_ok(cudaMemcpyAsync(C, c.p, (size_t) M * N * 4, cudaMemcpyDeviceToHost, st), "gemm_f16") &&
                 jb::cuda_ok(cudaStreamSynchronize(st), "gemm_f16") ? 0 : -1;
        }
        if (rc == 0 && jb::gemm_f16_error_flag(st) != 0) { jb::log("jepa: gemm_f16: pipeline wait timed out\n"); rc = -1; }
    }
    cudaStreamDestroy(st);
    return rc;
}

// the same product timed on device-resident operands (zeros): mean ms per launch over `reps` launches
extern "C" int jepa_b200_gemm_f16_bench(int M, int N, int K, int reps, double * ms) {
    if (M < 1 || N < 1 || K < 1 || (K & 7) || reps < 1 || !ms) return -1;
    cudaStream_t st;
    JB_CUDA(cudaStreamCreate(&st));
    DevBuf a16, b16, c;
    int rc = -1;
    if (a16.alloc((size_t) M * K * 2) && b16.alloc((size_t) N * K * 2) && c.alloc((size_t) M * N * 4)) {
        k_fill_h<<<1184, 256, 0, st>>>((__half *) a16.p, (size_t) M * K, 3u, 2.0f);
        k_fill_h<<<1184, 256, 0, st>>>((__half *) b16.p, (size_t) N * K, 4u, 0.1f);
        jb::AcGemmEpi ep;
        ep.mode = jb::AEPI_F32;
        ep.out_f32 = c.f();
        ep.ld_f32 = N;
        rc = jb::gemm_f16((const __half *) a16.p, K, (const __half *) b16.p, K, M, N, K, ep, st);
        cudaEvent_t e0, e1;
        cudaEventCreate(&e0);
        cudaEventCreate(&e1);
        cudaEventRecord(e0, st);
        for (int i = 0; i < reps && rc == 0; i++) rc = jb::gemm_f16((const __half *) a16.p, K, (const __half *) b16.p, K, M, N, K, ep, st);
        cudaEventRecord(e1, st);
        if (rc == 0 && jb::cuda_ok(cudaEventSynchronize(e1), "gemm_f16 bench")) {
            float t = 0;
            cudaEventElapsedTime(&t, e0, e1);
            *ms = t / reps;
        } else {
            rc = -1;
        }
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
    }
    cudaStreamDestroy(st);
    return rc;
}


// The AC predictor's attention timed alone: the last of `n_frames` frames of `rows` rows attends to all
// of them, for `n_cand` candidates and `heads` heads of width `hd` (keys / values contiguous per
// candidate, pseudo-random f16 values). Mean milliseconds per launch over `reps` launches.
extern "C" int jepa_b200_attention_bench(int n_cand, int n_frames, int rows, int heads, int hd, int impl, int reps, double * ms) {
    if (n_cand < 1 || n_frames < 1 || n_frames > jb::AC_MAX_FRAMES || rows < 1 || heads < 1 || reps < 1 || !ms) return -1;
    const int D = heads * hd;
    cudaStream_t st;
    JB_CUDA(cudaStreamCreate(&st));
    DevBuf q, kv, o;
    int rc = -1;
    const size_t nq = (size_t) n_cand * rows * D, nkv = (size_t) n_cand * n_frames * rows * 2 * D;
    if (q.alloc(nq * 2) && kv.alloc(nkv * 2) && o.alloc(nq * 2)) {
        k_fill_h<<<1184, 256, 0, st>>>((__half *) q.p, nq, 1u, 2.0f);
        k_fill_h<<<1184, 256, 0, st>>>((__half *) kv.p, nkv, 2u, 2.0f);
        jb::AttnArgs a;
        a.q = (const __half *) q.p; a.ldq = D; a.q_cand = (long long) rows * D; a.nq = rows; a.n_qframes = 1; a.q_frame = rows;
        a.out = (__half *) o.p; a.ldo = D; a.o_cand = a.q_cand;
        a.key_frames0 = n_frames; a.key_step = 0;
        for (int f = 0; f < n_frames; f++) {
            a.kv[f] = (const __half *) kv.p + (size_t) f * rows * 2 * D;
            a.kv_cand_stride[f] = (long long) n_frames * rows * 2 * D;
        }
        a.kv_rows = rows; a.ld_kv = 2 * D; a.D = D; a.n_head = heads; a.hd = hd; a.n_cand = n_cand;
        a.scale = 1.0f / sqrtf((float) hd);
        a.impl = impl;
        rc = jb::attention_f16(a, st);
        cudaEvent_t e0, e1;
        cudaEventCreate(&e0);
        cudaEventCreate(&e1);
        cudaEventRecord(e0, st);
        for (int i = 0; i < reps && rc == 0; i++) rc = jb::attention_f16(a, st);
        cudaEventRecord(e1, st);
        if (rc == 0 && jb::cuda_ok(cudaEventSynchronize(e1), "attention bench")) {
            float t = 0;
            cudaEventElapsedTime(&t, e0, e1);
            *ms = t / reps;
        } else {
            rc = -1;
        }
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
    }
    cudaStreamDestroy(st);
    return rc;
}

// The AC predictor's attention on host inputs: the last of `n_frames` frames of `rows` rows attends to all
// of them. q [n_cand][rows][heads hd], kv [n_cand][n_frames rows][2 heads hd] (k then v), out like q; all
// f32 on the host, f16 on the device. impl: 0 auto, 1 the mma.sync kernel, 2 the tcgen05 kernel.
extern "C" int jepa_b200_attention(const float * q, const float * kv, int n_cand, int n_frames, int rows, int heads, int hd,
                                   int impl, float * out) {
    if (!q || !kv || !out || n_cand < 1 || n_frames < 1 || n_frames > jb::AC_MAX_FRAMES || rows < 1 || heads < 1) return -1;
    const int D = heads * hd;
    cudaStream_t st;
    JB_CUDA(cudaStreamCreate(&st));
    const size_t nq = (size_t) n_cand * rows * D, nkv = (size_t) n_cand * n_frames * rows * 2 * D;
    DevBuf q32, kv32, q16, kv16, o16, o32;
    int rc = -1;
    if (q32.alloc(nq * 4) && kv32.alloc(nkv * 4) && q16.alloc(nq * 2) && kv16.alloc(nkv * 2) && o16.alloc(nq * 2) && o32.alloc(nq * 4)) {
        cudaMemcpyAsync(q32.p, q, nq * 4, cudaMemcpyHostToDevice, st);
        cudaMemcpyAsync(kv32.p, kv, nkv * 4, cudaMemcpyHostToDevice, st);
        jb::to_f16(q32.f(), D, (__half *) q16.p, D, n_cand * rows, D, jb::RowMap{}, st);
        jb::to_f16(kv32.f(), 2 * D, (__half *) kv16.p, 2 * D, n_cand * n_frames * rows, 2 * D, jb::RowMap{}, st);
        jb::AttnArgs a;
        a.q = (const __half *) q16.p; a.ldq = D; a.q_cand = (long long) rows * D; a.nq = rows; a.n_qframes = 1; a.q_frame = rows;
        a.out = (__half *) o16.p; a.ldo = D; a.o_cand = a.q_cand;
        a.key_frames0 = n_frames; a.key_step = 0;
        for (int f = 0; f < n_frames; f++) {
            a.kv[f] = (const __half *) kv16.p + (size_t) f * rows * 2 * D;
            a.kv_cand_stride[f] = (long long) n_frames * rows * 2 * D;
        }
        a.kv_rows = rows; a.ld_kv = 2 * D; a.D = D; a.n_head = heads; a.hd = hd; a.n_cand = n_cand;
        a.scale = 1.0f / sqrtf((float) hd);
        a.impl = impl;
        rc = jb::attention_f16(a, st);
        if (rc == 0) {
            k_h2f<<<1184, 256, 0, st>>>((const __half *) o16.p, o32.f(), nq);
            rc = jb::cuda_ok(cudaMemcpyAsync(out, o32.p, nq * 4, cudaMemcpyDeviceToHost, st), "attention") &&
                 jb::cuda_ok(cudaStreamSynchronize(st), "attention") ? 0 : -1;
        }
        if (rc == 0 && jb::attention_tc_error_flag(st) != 0) { jb::log("jepa: attention: pipeline wait timed out\n"); rc = -1; }
    }
    cudaStreamDestroy(st);
    return rc;
}

extern "C" int jepa_b200_dequant(uint32_t type, const void * src, int64_t rows, int64_t ne0, float * dst) {
    if (!src || !dst || rows < 1 || ne0 < 1) return -1;
    size_t row_bytes = 0;
    switch (type) {
        case 0: row_bytes = (size_t) ne0 * 4; break;
        case 1: case 30: row_bytes = (size_t) ne0 * 2; break;
        case 8: row_bytes = (size_t) (ne0 / 32) * 34; break;
        case 2: row_bytes = (size_t) (ne0 / 32) * 18; break;
        default: jb::log("jepa: jepa_b200_dequant: unsupported ggml type %u\n", type); return -1;
    }
    cudaStream_t st;
    JB_CUDA(cudaStreamCreate(&st));
    DevBuf s, d;
    int rc = -1;
    if (s.alloc(row_bytes * (size_t) rows) && d.alloc((size_t) rows * ne0 * 4) &&
        cudaMemcpyAsync(s.p, src, row_bytes * (size_t) rows, cudaMemcpyHostToDevice, st) == cudaSuccess) {
        rc = jb::dequant_rows(type, s.p, d.f(), rows, ne0, st);
        if (rc == 0 && !jb::cuda_ok(cudaMemcpyAsync(dst, d.p, (size_t) rows * ne0 * 4, cudaMemcpyDeviceToHost, st), "copy")) rc = -1;
        if (rc == 0 && !jb::cuda_ok(cudaStreamSynchronize(st), "dequant")) rc = -1;
    }
    cudaStreamDestroy(st);
    return rc;
}

extern "C" int jepa_b200_check_wait_timeout(long long limit_cycles, int * code) {
    if (!code || limit_cycles < 1 || limit_cycles > 4000000000LL) {
        jb::log("jepa: jepa_b200_check_wait_timeout: need an output and 1 <= limit_cycles <= 4e9\n");
        return -1;
    }
    constexpr int CODE = 9;   // the code this check's wait reports (the GEMM's own waits use 1..5)
    cudaStream_t st;
    JB_CUDA(cudaStreamCreate(&st));
    int rc = -1;
    if (jb::gemm_error_clear(st) == 0 && jb::wait_timeout_check(limit_cycles, CODE, st) == 0 &&
        jb::cuda_ok(cudaStreamSynchronize(st), "jepa_b200_check_wait_timeout")) {
        *code = jb::gemm_error_flag(st);            // the timeout, read once ...
        const int after = jb::gemm_error_flag(st);   // ... and reset by that read
        rc = (*code >= 0 && after == 0) ? 0 : -1;
        if (after != 0) jb::log("jepa: jepa_b200_check_wait_timeout: the flag was not reset by its read (%d)\n", after);
    }
    cudaStreamDestroy(st);
    return rc;
}

extern "C" int jepa_b200_host_dequant(uint32_t type, const void * src, int64_t rows, int64_t ne0, float * dst) {
    if (!src || !dst || rows < 1 || ne0 < 1) return -1;
    size_t row_bytes = 0;
    switch (type) {
        case 0: row_bytes = (size_t) ne0 * 4; break;
        case 1: case 30: row_bytes = (size_t) ne0 * 2; break;
        case 8: row_bytes = (size_t) (ne0 / 32) * 34; break;
        case 2: row_bytes = (size_t) (ne0 / 32) * 18; break;
        default: jb::log("jepa: jepa_b200_host_dequant: unsupported ggml type %u\n", type); return -1;
    }
    if ((type == 8 || type == 2) && ne0 % 32) { jb::log("jepa: jepa_b200_host_dequant: block rows need ne0 %% 32 == 0\n"); return -1; }
    for (int64_t r = 0; r < rows; r++) jb::dequant_row(type, (const uint8_t *) src + (size_t) r * row_bytes, dst + r * ne0, ne0);
    return 0;
}
