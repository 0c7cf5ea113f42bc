// Row kernels of the V-JEPA 2-AC predictor and CEM: LayerNorm to f16 (with a row gather, so the final
// norm reads only the patch rows of the trailing frames), the reference's non-affine normalisation
// between rollout steps, the action / state conditioning rows, row broadcast of shared embeddings, and
// the L1 energy. One warp per row, coalesced float4 loads, stats in double like the reference's host
// code (src/vjepa2_ac.cpp:182-196 normalize, :253-263 energy).
#include "kernels.h"
#include "common.h"
#include "launch.h"

namespace jb {

namespace {

__device__ __forceinline__ void pdl_enter() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ int map_row(const RowMap & m, int r) {
    if (m.g1 == 0) return r;
    const int blk = m.g1 * m.g2;
    return (r / blk) * m.s2 + ((r / m.g1) % m.g2) * m.s1 + m.off + r % m.g1;
}

constexpr int WARPS = 8;   // rows per 256-thread block

// register-resident: V float4 per lane, D == 128 V
template <int V>
__global__ void __launch_bounds__(256) k_ln_f16_v(const float * __restrict__ x, int ldx, const float * __restrict__ w,
                                                   const float * __restrict__ b, float eps, __half * __restrict__ y, int ldy,
                                                   int M, RowMap map) {
    pdl_enter();
    const int lane = threadIdx.x & 31;
    const int r = blockIdx.x * WARPS + (threadIdx.x >> 5);
    if (r >= M) return;
    constexpr int D = V * 128;
    const float * xr = x + (size_t) map_row(map, r) * ldx;
    float4 v[V];
#pragma unroll
    for (int i = 0; i < V; i++) v[i] = *(const float4 *) (xr + i * 128 + lane * 4);
    double s = 0;
#pragma unroll
    for (int i = 0; i < V; i++) s += (double) v[i].x + (double) v[i].y + (double) v[i].z + (double) v[i].w;
    const float mu = (float) (warp_sum_d(s) / D);
    double q = 0;
#pragma unroll
    for (int i = 0; i < V; i++) {
        const float a0 = v[i].x - mu, a1 = v[i].y - mu, a2 = v[i].z - mu, a3 = v[i].w - mu;
        q += (double) a0 * a0 + (double) a1 * a1 + (double) a2 * a2 + (double) a3 * a3;
    }
    const float inv = 1.0f / sqrtf((float) (warp_sum_d(q) / D) + eps);
    __half * yr = y + (size_t) r * ldy;
#pragma unroll
    for (int i = 0; i < V; i++) {
        const int c = i * 128 + lane * 4;
        float o[4] = {(v[i].x - mu) * inv, (v[i].y - mu) * inv, (v[i].z - mu) * inv, (v[i].w - mu) * inv};
        if (w) {
            const float4 ww = *(const float4 *) (w + c);
            o[0] *= ww.x; o[1] *= ww.y; o[2] *= ww.z; o[3] *= ww.w;
        }
        if (b) {
            const float4 bb = *(const float4 *) (b + c);
            o[0] += bb.x; o[1] += bb.y; o[2] += bb.z; o[3] += bb.w;
        }
        __half2 h0 = __floats2half2_rn(o[0], o[1]), h1 = __floats2half2_rn(o[2], o[3]);
        uint2 u;
        u.x = *(uint32_t *) &h0;
        u.y = *(uint32_t *) &h1;
        *(uint2 *) (yr + c) = u;
    }
}

// any D: strided loops over the row (re-read from L1 / L2)
__global__ void __launch_bounds__(256) k_ln_f16(const float * __restrict__ x, int ldx, const float * __restrict__ w,
                                                 const float * __restrict__ b, float eps, __half * __restrict__ y, int ldy,
                                                 int M, int D, RowMap map) {
    pdl_enter();
    const int lane = threadIdx.x & 31;
    const int r = blockIdx.x * WARPS + (threadIdx.x >> 5);
    if (r >= M) return;
    const float * xr = x + (size_t) map_row(map, r) * ldx;
    double s = 0;
    for (int c = lane; c < D; c += 32) s += xr[c];
    const float mu = (float) (warp_sum_d(s) / D);
    double q = 0;
    for (int c = lane; c < D; c += 32) { const float a = xr[c] - mu; q += (double) a * a; }
    const float inv = 1.0f / sqrtf((float) (warp_sum_d(q) / D) + eps);
    __half * yr = y + (size_t) r * ldy;
    for (int c = lane; c < D; c += 32) {
        float o = (xr[c] - mu) * inv;
        if (w) o *= w[c];
        if (b) o += b[c];
        yr[c] = __float2half_rn(o);
    }
}

// jepa_ac_normalize: double mean, double variance of (x - mean), float inverse std of (float) var + eps,
// then (x - (float) mean) * inv in float
__global__ void __launch_bounds__(256) k_ac_normalize(float * __restrict__ x, int ld, __half * __restrict__ y16, int ldy,
                                                       int M, int D, float eps) {
    pdl_enter();
    const int lane = threadIdx.x & 31;
    const int r = blockIdx.x * WARPS + (threadIdx.x >> 5);
    if (r >= M) return;
    float * xr = x + (size_t) r * ld;
    double s = 0;
    for (int c = lane; c < D; c += 32) s += xr[c];
    const double mu = warp_sum_d(s) / D;
    double q = 0;
    for (int c = lane; c < D; c += 32) { const double d = (double) xr[c] - mu; q += d * d; }
    const float inv = 1.0f / sqrtf((float) (warp_sum_d(q) / D) + eps);
    const float muf = (float) mu;
    __half * yr = y16 ? y16 + (size_t) r * ldy : nullptr;
    for (int c = lane; c < D; c += 32) {
        const float o = (xr[c] - muf) * inv;
        xr[c] = o;
        if (yr) yr[c] = __float2half_rn(o);
    }
}

__global__ void k_to_f16(const float * __restrict__ x, int ldx, __half * __restrict__ y, int ldy, int M, int N, RowMap map) {
    pdl_enter();
    const long long total = (long long) M * N;
    for (long long i = blockIdx.x * (long long) blockDim.x + threadIdx.x; i < total; i += (long long) gridDim.x * blockDim.x) {
        const int r = (int) (i / N), c = (int) (i % N);
        y[(size_t) r * ldy + c] = __float2half_rn(x[(size_t) map_row(map, r) * ldx + c]);
    }
}

// one thread per output column of the two conditioning rows of one (candidate, frame) block
__global__ void k_ac_cond(const float * __restrict__ acts, long long act_cand, const float * __restrict__ sts, long long st_cand,
                          int A, int S, const float * __restrict__ wa, const float * __restrict__ ba, const float * __restrict__ ws,
                          const float * __restrict__ bs, float * __restrict__ resid, int ld, int n_frames, int n_blocks, int rows_per_frame, int D) {
    pdl_enter();
    const int d = blockIdx.x * blockDim.x + threadIdx.x;
    if (d >= D) return;
    for (int blk = blockIdx.y; blk < n_blocks; blk += gridDim.y) {   // candidate * n_frames + frame
        const int c = blk / n_frames, t = blk % n_frames;
        const float * a = acts + (size_t) c * act_cand + (size_t) t * A;
        const float * s = sts + (size_t) c * st_cand + (size_t) t * S;
        float acc = 0.0f;
        for (int k = 0; k < A; k++) acc += wa[(size_t) d * A + k] * a[k];
        const float ya = (ba ? ba[d] : 0.0f) + acc;
        acc = 0.0f;
        for (int k = 0; k < S; k++) acc += ws[(size_t) d * S + k] * s[k];
        const float ys = (bs ? bs[d] : 0.0f) + acc;
        float * row = resid + (size_t) blk * rows_per_frame * ld;
        row[d] = ya;
        row[ld + d] = ys;
    }
}

__global__ void k_ac_broadcast(float * __restrict__ x, int ld, long long cand_rows, int row0, int rows, int n_cand, int D) {
    pdl_enter();
    const long long per = (long long) rows * D;
    const long long total = per * (n_cand - 1);
    for (long long i = blockIdx.x * (long long) blockDim.x + threadIdx.x; i < total; i += (long long) gridDim.x * blockDim.x) {
        const int c = 1 + (int) (i / per);
        const long long e = i % per;
        const int r = row0 + (int) (e / D), col = (int) (e % D);
        x[((size_t) c * cand_rows + r) * ld + col] = x[(size_t) r * ld + col];
    }
}

// one block per candidate: sum |pred - goal| in double, tree-reduced
__global__ void __launch_bounds__(256) k_ac_energy(const float * __restrict__ pred, long long cand_stride,
                                                    const float * __restrict__ goal, long long n, float * __restrict__ energy) {
    pdl_enter();
    const float * p = pred + (size_t) blockIdx.x * cand_stride;
    double acc = 0;
    const bool vec = ((n & 3) == 0) && (((uintptr_t) p & 15) == 0) && (((uintptr_t) goal & 15) == 0);
    if (vec) {
        const long long n4 = n >> 2;
        for (long long i = threadIdx.x; i < n4; i += blockDim.x) {
            const float4 a = ((const float4 *) p)[i], g = ((const float4 *) goal)[i];
            acc += fabs((double) a.x - (double) g.x) + fabs((double) a.y - (double) g.y) +
                   fabs((double) a.z - (double) g.z) + fabs((double) a.w - (double) g.w);
        }
    } else {
        for (long long i = threadIdx.x; i < n; i += blockDim.x) acc += fabs((double) p[i] - (double) goal[i]);
    }
    acc = warp_sum_d(acc);
    __shared__ double part[8];
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0;
        for (int i = 0; i < (int) (blockDim.x >> 5); i++) t += part[i];
        energy[blockIdx.x] = (float) (t / (double) n);
    }
}

int grid_for(long long total) {
    long long b = (total + 255) / 256;
    if (b > 148 * 16) b = 148 * 16;
    return (int) (b < 1 ? 1 : b);
}

}  // namespace

void ln_to_f16(const float * x, int ldx, const float * w, const float * b, float eps, __half * y, int ldy, int M, int D,
               RowMap map, cudaStream_t st) {
    if (M <= 0) return;
    const dim3 grid((unsigned) ((M + WARPS - 1) / WARPS));
    const bool vec = (D % 128 == 0) && (ldx % 4 == 0) && (ldy % 4 == 0) && (((uintptr_t) x & 15) == 0) && (((uintptr_t) y & 7) == 0);
    if (vec) {
        switch (D / 128) {
            case 1: launch_pdl(k_ln_f16_v<1>, grid, dim3(256), 0, st, x, ldx, w, b, eps, y, ldy, M, map); return;
            case 2: launch_pdl(k_ln_f16_v<2>, grid, dim3(256), 0, st, x, ldx, w, b, eps, y, ldy, M, map); return;
            case 4: launch_pdl(k_ln_f16_v<4>, grid, dim3(256), 0, st, x, ldx, w, b, eps, y, ldy, M, map); return;
            case 8: launch_pdl(k_ln_f16_v<8>, grid, dim3(256), 0, st, x, ldx, w, b, eps, y, ldy, M, map); return;
            case 16: launch_pdl(k_ln_f16_v<16>, grid, dim3(256), 0, st, x, ldx, w, b, eps, y, ldy, M, map); return;
            default: break;
        }
    }
    launch_pdl(k_ln_f16, grid, dim3(256), 0, st, x, ldx, w, b, eps, y, ldy, M, D, map);
}

void ac_normalize_rows(float * x, int ld, __half * y16, int ldy, int M, int D, float eps, cudaStream_t st) {
    if (M <= 0) return;
    launch_pdl(k_ac_normalize, dim3((unsigned) ((M + WARPS - 1) / WARPS)), dim3(256), 0, st, x, ld, y16, ldy, M, D, eps);
}

void to_f16(const float * x, int ldx, __half * y, int ldy, int M, int N, RowMap map, cudaStream_t st) {
    if (M <= 0 || N <= 0) return;
    launch_pdl(k_to_f16, dim3((unsigned) grid_for((long long) M * N)), dim3(256), 0, st, x, ldx, y, ldy, M, N, map);
}

void ac_cond_rows(const float * acts, long long act_cand, const float * states, long long st_cand, int A, int S,
                  const float * wa, const float * ba, const float * ws, const float * bs, float * resid, int ld,
                  int n_cand, int n_frames, int rows_per_frame, int D, cudaStream_t st) {
    if (n_cand <= 0 || n_frames <= 0) return;
    const int n_blocks = n_cand * n_frames;
    const dim3 grid((unsigned) ((D + 127) / 128), (unsigned) (n_blocks < 65535 ? n_blocks : 65535));
    launch_pdl(k_ac_cond, grid, dim3(128), 0, st, acts, act_cand, states, st_cand, A, S, wa, ba, ws, bs, resid, ld, n_frames,
               n_blocks, rows_per_frame, D);
}

void ac_broadcast_rows(float * x, int ld, long long cand_rows, int row0, int rows, int n_cand, int D, cudaStream_t st) {
    if (n_cand <= 1 || rows <= 0) return;
    launch_pdl(k_ac_broadcast, dim3((unsigned) grid_for((long long) rows * D * (n_cand - 1))), dim3(256), 0, st,
               x, ld, cand_rows, row0, rows, n_cand, D);
}

void ac_energy(const float * pred, long long cand_stride, const float * goal, long long n, int n_cand, float * energy,
               cudaStream_t st) {
    if (n_cand <= 0 || n <= 0) return;
    launch_pdl(k_ac_energy, dim3((unsigned) n_cand), dim3(256), 0, st, pred, cand_stride, goal, n, energy);
}

}  // namespace jb
