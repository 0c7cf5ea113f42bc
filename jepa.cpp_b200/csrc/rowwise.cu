// Row-wise and element-wise kernels of the planner: the adaLN block prologue (LayerNorm + FiLM +
// inner LayerNorm, written as split tensor-core operands), the fused block backward halves, LayerNorm
// forward / backward, activations, the squared-L2 cost, the AdamW step and small helpers.
//
// The arithmetic restates the reference's host ops expression by expression
// (src/hjepa-plan.cpp:290-475): LayerNorm statistics in double, the inverse std rounded to float,
// x_hat = (float)(x - mean) * inv, gradients with the float64 row means m1 / m2. The library is built
// with -fmad=false so that no multiply-add is contracted where the reference (built with
// -ffp-contract=off) rounds twice; these kernels then agree with the host ops bit for bit except
// where a transcendental (erff / expf) differs in its last bit.
//
// The loop kernels below take one warp per row and re-read the row from L1 for each pass; the register-
// resident kernels further down (one or four warps per row) serve every row width that is a multiple of 32.
#include "kernels.h"
#include "common.h"
#include "launch.h"

namespace jb {

namespace {

constexpr int ROWS_PER_BLOCK = 8;   // 8 warps

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float split_hi(float v) { return __uint_as_float(__float_as_uint(v) & 0xFFFFE000u); }

__device__ __forceinline__ void store_split(float * hi, float * lo, size_t i, float v) {
    const float h = split_hi(v);
    hi[i] = h;
    lo[i] = v - h;
}

// mean and float inverse std of a row (two passes in double, as the reference)
__device__ __forceinline__ void row_stats(const float * xr, int D, float eps, int lane, double & mean, float & inv) {
    double s = 0;
    for (int i = lane; i < D; i += 32) s += (double) xr[i];
    mean = warp_sum(s) / D;
    double v = 0;
    for (int i = lane; i < D; i += 32) { const double c = (double) xr[i] - mean; v += c * c; }
    const double var = warp_sum(v) / D;
    inv = (float) (1.0 / sqrt(var + (double) eps));
}

__device__ __forceinline__ float xhat_of(float x, double mean, float inv) { return (float) ((double) x - mean) * inv; }

// ---------------------------------------------------------------------------------------------
__global__ void k_block_pre(const float * __restrict__ x, int ldx, const float * __restrict__ mod, int ld_mod,
                            int sh_off, int sc_off, const float * __restrict__ ln_w, const float * __restrict__ ln_b,
                            float eps0, float eps1, float * __restrict__ h_hi, float * __restrict__ h_lo, int ldh,
                            LnStats * __restrict__ st0, LnStats * __restrict__ st1, int M, int D) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * ROWS_PER_BLOCK + (threadIdx.x >> 5);
    if (row >= M) return;
    const float * xr = x + (size_t) row * ldx;
    const float * sh = mod + (size_t) row * ld_mod + sh_off;
    const float * sc = mod + (size_t) row * ld_mod + sc_off;
    double mean0; float inv0;
    row_stats(xr, D, eps0, lane, mean0, inv0);
    if (lane == 0) st0[row] = LnStats{mean0, inv0, 0.0f};
    float * hh = h_hi + (size_t) row * ldh;
    float * hl = h_lo + (size_t) row * ldh;
    if (!ln_w) {
        for (int i = lane; i < D; i += 32) {
            const float z = xhat_of(xr[i], mean0, inv0) * (1.0f + sc[i]) + sh[i];
            store_split(hh, hl, i, z);
        }
        return;
    }
    double s = 0;
    for (int i = lane; i < D; i += 32) s += (double) (xhat_of(xr[i], mean0, inv0) * (1.0f + sc[i]) + sh[i]);
    const double mean1 = warp_sum(s) / D;
    double v = 0;
    for (int i = lane; i < D; i += 32) {
        const double c = (double) (xhat_of(xr[i], mean0, inv0) * (1.0f + sc[i]) + sh[i]) - mean1;
        v += c * c;
    }
    const float inv1 = (float) (1.0 / sqrt(warp_sum(v) / D + (double) eps1));
    if (lane == 0) st1[row] = LnStats{mean1, inv1, 0.0f};
    for (int i = lane; i < D; i += 32) {
        const float z = xhat_of(xr[i], mean0, inv0) * (1.0f + sc[i]) + sh[i];
        const float y = xhat_of(z, mean1, inv1) * ln_w[i] + (ln_b ? ln_b[i] : 0.0f);
        store_split(hh, hl, i, y);
    }
}

__global__ void k_layer_norm(const float * __restrict__ x, int ldx, const float * __restrict__ w, const float * __restrict__ b,
                             float eps, float * __restrict__ y, int ldy, float * __restrict__ hi, float * __restrict__ lo,
                             LnStats * __restrict__ stats, int M, int D) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * ROWS_PER_BLOCK + (threadIdx.x >> 5);
    if (row >= M) return;
    const float * xr = x + (size_t) row * ldx;
    double mean; float inv;
    row_stats(xr, D, eps, lane, mean, inv);
    if (stats && lane == 0) stats[row] = LnStats{mean, inv, 0.0f};
    for (int i = lane; i < D; i += 32) {
        const float v = xhat_of(xr[i], mean, inv) * (w ? w[i] : 1.0f) + (b ? b[i] : 0.0f);
        if (y) y[(size_t) row * ldy + i] = v;
        if (hi) store_split(hi + (size_t) row * ldy, lo + (size_t) row * ldy, i, v);
    }
}

// gx = gres + ln_bwd(gy) ; optional gated-residual head
__global__ void k_layer_norm_bwd(const float * __restrict__ gy, int ldgy, const float * __restrict__ x, int ldx,
                                 const LnStats * __restrict__ stats, const float * __restrict__ w,
                                 const float * __restrict__ gres, int ldres, float * __restrict__ gx, int ldgx,
                                 const float * __restrict__ dn, int lddn, const float * __restrict__ gate, int ld_gate,
                                 float * __restrict__ dmod_hi, float * __restrict__ dmod_lo, int ld_dmod,
                                 float * __restrict__ d_hi, float * __restrict__ d_lo, int ldd, int M, int D) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * ROWS_PER_BLOCK + (threadIdx.x >> 5);
    if (row >= M) return;
    const float * g = gy + (size_t) row * ldgy;
    const float * xr = x + (size_t) row * ldx;
    const LnStats stt = stats[row];
    double m1 = 0, m2 = 0;
    for (int i = lane; i < D; i += 32) {
        const float gh = g[i] * (w ? w[i] : 1.0f);
        m1 += gh;
        m2 += (double) gh * xhat_of(xr[i], stt.mean, stt.inv);
    }
    m1 = warp_sum(m1) / D;
    m2 = warp_sum(m2) / D;
    for (int i = lane; i < D; i += 32) {
        const float gh = g[i] * (w ? w[i] : 1.0f);
        const float xh = xhat_of(xr[i], stt.mean, stt.inv);
        float v = (float) (((double) gh - m1 - (double) xh * m2) * (double) stt.inv);
        if (gres) v = gres[(size_t) row * ldres + i] + v;
        gx[(size_t) row * ldgx + i] = v;
        if (dn) {
            store_split(dmod_hi + (size_t) row * ld_dmod, dmod_lo + (size_t) row * ld_dmod, i, v * dn[(size_t) row * lddn + i]);
            store_split(d_hi + (size_t) row * ldd, d_lo + (size_t) row * ldd, i, v * gate[(size_t) row * ld_gate + i]);
        }
    }
}

__global__ void k_block_bwd(BlockBwdArgs a) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * ROWS_PER_BLOCK + (threadIdx.x >> 5);
    if (row >= a.M) return;
    const int D = a.D;
    const float * gh = a.gh + (size_t) row * a.ldgh;
    const float * xr = a.x + (size_t) row * a.ldx;
    const float * sh = a.mod + (size_t) row * a.ld_mod + a.sh_off;
    const float * sc = a.mod + (size_t) row * a.ld_mod + a.sc_off;
    const LnStats s0 = a.st0[row];
    float * dmh = a.dmod_hi + (size_t) row * a.ld_dmod;
    float * dml = a.dmod_lo + (size_t) row * a.ld_dmod;
    // inner ln backward statistics (when there is an inner ln)
    double n1 = 0, n2 = 0;
    LnStats s1{0.0, 1.0f, 0.0f};
    if (a.ln_w) {
        s1 = a.st1[row];
        for (int i = lane; i < D; i += 32) {
            const float z = xhat_of(xr[i], s0.mean, s0.inv) * (1.0f + sc[i]) + sh[i];
            const float g = gh[i] * a.ln_w[i];
            n1 += g;
            n2 += (double) g * xhat_of(z, s1.mean, s1.inv);
        }
        n1 = warp_sum(n1) / D;
        n2 = warp_sum(n2) / D;
    }
    // gz_i: gradient into the FiLM output; dmod (scale, shift); m1 / m2 of the LN0 backward
    double m1 = 0, m2 = 0;
    for (int i = lane; i < D; i += 32) {
        const float xh = xhat_of(xr[i], s0.mean, s0.inv);
        float gz = gh[i];
        if (a.ln_w) {
            const float z = xh * (1.0f + sc[i]) + sh[i];
            const float g = gh[i] * a.ln_w[i];
            gz = (float) (((double) g - n1 - (double) xhat_of(z, s1.mean, s1.inv) * n2) * (double) s1.inv);
        }
        store_split(dmh, dml, a.sc_off + i, gz * xh);
        store_split(dmh, dml, a.sh_off + i, gz);
        const float gxh = gz * (1.0f + sc[i]);
        m1 += gxh;
        m2 += (double) gxh * xh;
    }
    m1 = warp_sum(m1) / D;
    m2 = warp_sum(m2) / D;
    for (int i = lane; i < D; i += 32) {
        const float xh = xhat_of(xr[i], s0.mean, s0.inv);
        float gz = gh[i];
        if (a.ln_w) {
            const float z = xh * (1.0f + sc[i]) + sh[i];
            const float g = gh[i] * a.ln_w[i];
            gz = (float) (((double) g - n1 - (double) xhat_of(z, s1.mean, s1.inv) * n2) * (double) s1.inv);
        }
        const float gxh = gz * (1.0f + sc[i]);
        const float v = a.gres[(size_t) row * a.ldres + i] + (float) (((double) gxh - m1 - (double) xh * m2) * (double) s0.inv);
        a.gx[(size_t) row * a.ldgx + i] = v;
        if (a.a2) {
            store_split(a.dmod2_hi + (size_t) row * a.ld_dmod2, a.dmod2_lo + (size_t) row * a.ld_dmod2, a.gate2_off + i,
                        v * a.a2[(size_t) row * a.lda2 + i]);
            store_split(a.d_hi + (size_t) row * a.ldd, a.d_lo + (size_t) row * a.ldd, i,
                        v * a.mod2[(size_t) row * a.ld_mod2 + a.gate2_off + i]);
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Register-resident variants: a row of D floats is held by W warps (32 W threads), V values per thread,
// element i = t + 32 W k for thread t of the row (coalesced per warp instruction). Every pass over the row
// issues all of its loads at once and keeps the values in registers, so a pass costs one memory latency
// instead of one per element. Narrow rows take one warp each (W = 1, FAST_ROWS rows per block); rows of 512
// floats and more take four warps (W = 4, two rows per block): a 768-wide row is then 6 values per thread
// instead of 24, which keeps the block backward's eight row arrays in ~70 registers rather than 252 and
// lets an SM hold four times the warps to cover the memory latency. Row sums reduce each warp's lanes by
// shuffles, then the W warp partials in shared memory in warp order (a fixed order: deterministic). Same
// element-wise arithmetic and expression order as the loop kernels above.
// ---------------------------------------------------------------------------------------------
constexpr int FAST_ROWS = 4;   // rows per block with one warp per row
constexpr int WIDE_ROWS = 2;   // rows per block with four warps per row

// Programmatic dependent launch: wait for the grid this one depends on (its writes become visible),
// then let the next grid in the stream begin launching while this one runs.
__device__ __forceinline__ void pdl_enter() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// where a thread sits: its row in the block, its index t within the row, its warp within the row
template <int W>
struct RowPos {
    int rr, t, wir, lane;
    __device__ RowPos() {
        lane = threadIdx.x & 31;
        t = threadIdx.x % (32 * W);
        rr = threadIdx.x / (32 * W);
        wir = t >> 5;
    }
};

template <int V, int W>
__device__ __forceinline__ void load_row(const float * __restrict__ p, int D, int t, float (&v)[V]) {
#pragma unroll
    for (int k = 0; k < V; k++) { const int i = t + 32 * W * k; v[k] = i < D ? p[i] : 0.0f; }
}

// The sum of a row's per-thread partials (every thread of the block calls it, valid row or not). The W warp
// partials go through one of two shared slots, which calls alternate: a slot is written again only two
// reductions later, after the intervening reduction's barrier, which every thread reaches after its reads of
// this one -- so one barrier per reduction suffices.
template <int W>
__device__ __forceinline__ double row_sum(double v, const RowPos<W> & p, int slot) {
    v = warp_sum(v);
    if (W == 1) return v;
    __shared__ double red[2][8][W];
    if (p.lane == 0) red[slot][p.rr][p.wir] = v;
    __syncthreads();
    double s = red[slot][p.rr][0];
#pragma unroll
    for (int w = 1; w < W; w++) s += red[slot][p.rr][w];
    return s;
}

// two row sums at once (the same sums in the same order as two row_sum calls: the same bits), one exchange
// through shared memory instead of two
template <int W>
__device__ __forceinline__ void row_sum2(double & a, double & b, const RowPos<W> & p, int slot) {
    a = warp_sum(a);
    b = warp_sum(b);
    if (W == 1) return;
    __shared__ double red2[2][8][W][2];
    if (p.lane == 0) { red2[slot][p.rr][p.wir][0] = a; red2[slot][p.rr][p.wir][1] = b; }
    __syncthreads();
    double sa = red2[slot][p.rr][0][0], sb = red2[slot][p.rr][0][1];
#pragma unroll
    for (int w = 1; w < W; w++) { sa += red2[slot][p.rr][w][0]; sb += red2[slot][p.rr][w][1]; }
    a = sa;
    b = sb;
}

template <int V, int W>
__device__ __forceinline__ void stats_of(const float (&v)[V], int D, const RowPos<W> & p, float eps, double & mean, float & inv) {
    double s = 0;
#pragma unroll
    for (int k = 0; k < V; k++) if (p.t + 32 * W * k < D) s += (double) v[k];
    mean = row_sum<W>(s, p, 0) / D;
    double q = 0;
#pragma unroll
    for (int k = 0; k < V; k++) if (p.t + 32 * W * k < D) { const double c = (double) v[k] - mean; q += c * c; }
    inv = (float) (1.0 / sqrt(row_sum<W>(q, p, 1) / D + (double) eps));
}

template <int W> __host__ __device__ constexpr int rows_per_block() { return W == 1 ? FAST_ROWS : WIDE_ROWS; }

template <int V, int W>
__global__ void __launch_bounds__(32 * W * rows_per_block<W>())
k_block_pre_v(const float * __restrict__ x, int ldx, const float * __restrict__ mod, int ld_mod, int sh_off, int sc_off,
              const float * __restrict__ ln_w, const float * __restrict__ ln_b, float eps0, float eps1,
              float * __restrict__ h_hi, float * __restrict__ h_lo, int ldh, LnStats * __restrict__ st0,
              LnStats * __restrict__ st1, int M, int D) {
    const RowPos<W> p;
    const int row = blockIdx.x * rows_per_block<W>() + p.rr;
    const bool valid = row < M;
    // the modulation and the norm weights come from kernels that finished before this grid was launched:
    // they are read while the preceding kernel (the producer of x) still runs
    float xv[V], sc[V], sh[V], lw[V], lb[V];
#pragma unroll
    for (int k = 0; k < V; k++) { lb[k] = 0.0f; sc[k] = sh[k] = lw[k] = xv[k] = 0.0f; }
    if (valid) {
        load_row<V, W>(mod + (size_t) row * ld_mod + sc_off, D, p.t, sc);
        load_row<V, W>(mod + (size_t) row * ld_mod + sh_off, D, p.t, sh);
        if (ln_w) load_row<V, W>(ln_w, D, p.t, lw);
        if (ln_b) load_row<V, W>(ln_b, D, p.t, lb);
    }
    pdl_enter();
    if (valid) load_row<V, W>(x + (size_t) row * ldx, D, p.t, xv);
    double mean0; float inv0;
    stats_of<V, W>(xv, D, p, eps0, mean0, inv0);
    if (valid && p.t == 0) st0[row] = LnStats{mean0, inv0, 0.0f};
#pragma unroll
    for (int k = 0; k < V; k++) xv[k] = xhat_of(xv[k], mean0, inv0) * (1.0f + sc[k]) + sh[k];   // z, the FiLM output
    if (ln_w) {
        double mean1; float inv1;
        stats_of<V, W>(xv, D, p, eps1, mean1, inv1);
        if (valid && p.t == 0) st1[row] = LnStats{mean1, inv1, 0.0f};
#pragma unroll
        for (int k = 0; k < V; k++) xv[k] = xhat_of(xv[k], mean1, inv1) * lw[k] + lb[k];
    }
    if (!valid) return;
    float * hh = h_hi + (size_t) row * ldh;
    float * hl = h_lo + (size_t) row * ldh;
#pragma unroll
    for (int k = 0; k < V; k++) {
        const int i = p.t + 32 * W * k;
        if (i < D) store_split(hh, hl, i, xv[k]);
    }
}

template <int V, int W>
__global__ void __launch_bounds__(32 * W * rows_per_block<W>())
k_layer_norm_v(const float * __restrict__ x, int ldx, const float * __restrict__ w, const float * __restrict__ b, float eps,
               float * __restrict__ y, int ldy, float * __restrict__ hi, float * __restrict__ lo, LnStats * __restrict__ stats,
               int M, int D) {
    pdl_enter();
    const RowPos<W> p;
    const int row = blockIdx.x * rows_per_block<W>() + p.rr;
    const bool valid = row < M;
    float xv[V], wv[V], bv[V];
#pragma unroll
    for (int k = 0; k < V; k++) { wv[k] = 1.0f; bv[k] = 0.0f; xv[k] = 0.0f; }
    if (valid) {
        load_row<V, W>(x + (size_t) row * ldx, D, p.t, xv);
        if (w) load_row<V, W>(w, D, p.t, wv);
        if (b) load_row<V, W>(b, D, p.t, bv);
    }
    double mean; float inv;
    stats_of<V, W>(xv, D, p, eps, mean, inv);
    if (!valid) return;
    if (stats && p.t == 0) stats[row] = LnStats{mean, inv, 0.0f};
#pragma unroll
    for (int k = 0; k < V; k++) {
        const int i = p.t + 32 * W * k;
        if (i >= D) continue;
        const float v = xhat_of(xv[k], mean, inv) * wv[k] + bv[k];
        if (y) y[(size_t) row * ldy + i] = v;
        if (hi) store_split(hi + (size_t) row * ldy, lo + (size_t) row * ldy, i, v);
    }
}

template <int V, int W>
__global__ void __launch_bounds__(32 * W * rows_per_block<W>())
k_layer_norm_bwd_v(const float * __restrict__ gy, int ldgy, const float * __restrict__ x, int ldx,
                   const LnStats * __restrict__ stats, const float * __restrict__ w, const float * __restrict__ gres, int ldres,
                   float * __restrict__ gx, int ldgx, const float * __restrict__ dn, int lddn, const float * __restrict__ gate,
                   int ld_gate, float * __restrict__ dmod_hi, float * __restrict__ dmod_lo, int ld_dmod,
                   float * __restrict__ d_hi, float * __restrict__ d_lo, int ldd, int M, int D) {
    pdl_enter();
    const RowPos<W> p;
    const int row = blockIdx.x * rows_per_block<W>() + p.rr;
    const bool valid = row < M;
    const LnStats stt = valid ? stats[row] : LnStats{0.0, 0.0f, 0.0f};
    float gh[V], xh[V], wv[V], gr[V], dv[V], gt[V];
#pragma unroll
    for (int k = 0; k < V; k++) { wv[k] = 1.0f; gr[k] = 0.0f; gh[k] = xh[k] = dv[k] = gt[k] = 0.0f; }
    if (valid) {
        load_row<V, W>(gy + (size_t) row * ldgy, D, p.t, gh);
        load_row<V, W>(x + (size_t) row * ldx, D, p.t, xh);
        if (w) load_row<V, W>(w, D, p.t, wv);
        if (gres) load_row<V, W>(gres + (size_t) row * ldres, D, p.t, gr);
        if (dn) {
            load_row<V, W>(dn + (size_t) row * lddn, D, p.t, dv);
            load_row<V, W>(gate + (size_t) row * ld_gate, D, p.t, gt);
        }
    }
    double m1 = 0, m2 = 0;
#pragma unroll
    for (int k = 0; k < V; k++) {
        if (p.t + 32 * W * k >= D) continue;
        gh[k] = gh[k] * wv[k];
        xh[k] = xhat_of(xh[k], stt.mean, stt.inv);
        m1 += gh[k];
        m2 += (double) gh[k] * xh[k];
    }
    row_sum2<W>(m1, m2, p, 0);
    m1 = m1 / D;
    m2 = m2 / D;
    if (!valid) return;
#pragma unroll
    for (int k = 0; k < V; k++) {
        const int i = p.t + 32 * W * k;
        if (i >= D) continue;
        float v = (float) (((double) gh[k] - m1 - (double) xh[k] * m2) * (double) stt.inv);
        if (gres) v = gr[k] + v;
        gx[(size_t) row * ldgx + i] = v;
        if (dn) {
            store_split(dmod_hi + (size_t) row * ld_dmod, dmod_lo + (size_t) row * ld_dmod, i, v * dv[k]);
            store_split(d_hi + (size_t) row * ldd, d_lo + (size_t) row * ldd, i, v * gt[k]);
        }
    }
}

template <int V, int W>
__global__ void __launch_bounds__(32 * W * rows_per_block<W>()) k_block_bwd_v(BlockBwdArgs a) {
    const RowPos<W> p;
    const int row = blockIdx.x * rows_per_block<W>() + p.rr;
    const bool valid = row < a.M;
    const int D = a.D;
    // every load of the row up front (the struct's pointers may alias as far as the compiler knows). All but
    // gh were written at least two kernels earlier in the stream (the forward pass, the modulation, the
    // residual gradient of the half above), by grids that finished before this one was launched: they are
    // read while the preceding kernel (the producer of gh) still runs.
    float gz[V], xh[V], sc[V], z[V], lw[V], gr[V], av[V], gt[V];
#pragma unroll
    for (int k = 0; k < V; k++) gz[k] = xh[k] = sc[k] = z[k] = lw[k] = gr[k] = av[k] = gt[k] = 0.0f;
    LnStats s0{}, s1{};
    if (valid) {
        s0 = a.st0[row];
        if (a.ln_w) s1 = a.st1[row];
        load_row<V, W>(a.x + (size_t) row * a.ldx, D, p.t, xh);
        load_row<V, W>(a.mod + (size_t) row * a.ld_mod + a.sc_off, D, p.t, sc);
        load_row<V, W>(a.gres + (size_t) row * a.ldres, D, p.t, gr);
        if (a.ln_w) {
            load_row<V, W>(a.mod + (size_t) row * a.ld_mod + a.sh_off, D, p.t, z);
            load_row<V, W>(a.ln_w, D, p.t, lw);
        }
        if (a.a2) {
            load_row<V, W>(a.a2 + (size_t) row * a.lda2, D, p.t, av);
            load_row<V, W>(a.mod2 + (size_t) row * a.ld_mod2 + a.gate2_off, D, p.t, gt);
        }
    }
    pdl_enter();
    if (valid) load_row<V, W>(a.gh + (size_t) row * a.ldgh, D, p.t, gz);
#pragma unroll
    for (int k = 0; k < V; k++) xh[k] = xhat_of(xh[k], s0.mean, s0.inv);
    if (a.ln_w) {
        // inner ln backward: gz = ln_bwd(gh) over the ln's normalised input
        double n1 = 0, n2 = 0;
#pragma unroll
        for (int k = 0; k < V; k++) {
            if (p.t + 32 * W * k >= D) continue;
            z[k] = xhat_of(xh[k] * (1.0f + sc[k]) + z[k], s1.mean, s1.inv);
            gz[k] = gz[k] * lw[k];
            n1 += gz[k];
            n2 += (double) gz[k] * z[k];
        }
        row_sum2<W>(n1, n2, p, 0);
        n1 = n1 / D;
        n2 = n2 / D;
#pragma unroll
        for (int k = 0; k < V; k++) gz[k] = (float) (((double) gz[k] - n1 - (double) z[k] * n2) * (double) s1.inv);
    }
    float * dmh = a.dmod_hi + (size_t) row * a.ld_dmod;
    float * dml = a.dmod_lo + (size_t) row * a.ld_dmod;
    double m1 = 0, m2 = 0;
#pragma unroll
    for (int k = 0; k < V; k++) {
        const int i = p.t + 32 * W * k;
        if (i >= D) continue;
        if (valid) {
            store_split(dmh, dml, a.sc_off + i, gz[k] * xh[k]);
            store_split(dmh, dml, a.sh_off + i, gz[k]);
        }
        gz[k] = gz[k] * (1.0f + sc[k]);   // now the gradient into LN0's output
        m1 += gz[k];
        m2 += (double) gz[k] * xh[k];
    }
    row_sum2<W>(m1, m2, p, 1);   // (slot 0: the inner LayerNorm's sums)
    m1 = m1 / D;
    m2 = m2 / D;
    if (!valid) return;
#pragma unroll
    for (int k = 0; k < V; k++) {
        const int i = p.t + 32 * W * k;
        if (i >= D) continue;
        const float v = gr[k] + (float) (((double) gz[k] - m1 - (double) xh[k] * m2) * (double) s0.inv);
        a.gx[(size_t) row * a.ldgx + i] = v;
        if (a.a2) {
            store_split(a.dmod2_hi + (size_t) row * a.ld_dmod2, a.dmod2_lo + (size_t) row * a.ld_dmod2, a.gate2_off + i,
                        v * av[k]);
            store_split(a.d_hi + (size_t) row * a.ldd, a.d_lo + (size_t) row * a.ldd, i, v * gt[k]);
        }
    }
}

// values per thread of the register kernels for a row of D floats at W warps per row (0 = use the loop
// kernels): four warps per row from 512 floats, one below
inline int fast_w(int D) { return D >= 512 && D % 128 == 0 ? 4 : 1; }
inline int fast_v(int D) {
    const int lanes = 32 * fast_w(D);
    if (D % 32 != 0) return 0;
    const int v = (D + lanes - 1) / lanes;
    for (int c : {1, 2, 4, 6, 8, 12, 16, 24, 32}) if (v <= c) return c;
    return 0;
}

#define JB_DISPATCH_V(V, ...)                                      \
    switch (V) {                                                   \
        case 1: { constexpr int VV = 1; __VA_ARGS__; } break;      \
        case 2: { constexpr int VV = 2; __VA_ARGS__; } break;      \
        case 4: { constexpr int VV = 4; __VA_ARGS__; } break;      \
        case 6: { constexpr int VV = 6; __VA_ARGS__; } break;      \
        case 8: { constexpr int VV = 8; __VA_ARGS__; } break;      \
        case 12: { constexpr int VV = 12; __VA_ARGS__; } break;    \
        case 16: { constexpr int VV = 16; __VA_ARGS__; } break;    \
        case 24: { constexpr int VV = 24; __VA_ARGS__; } break;    \
        default: { constexpr int VV = 32; __VA_ARGS__; } break;    \
    }
// one warp per row, or four for rows of 512 floats and more (a multiple of 128, at most 32 x 128)
#define JB_DISPATCH_VW(D, ...)                                                                      \
    if (fast_w(D) == 4) {                                                                           \
        constexpr int WW = 4;                                                                       \
        const unsigned nb = (unsigned) ((M_ + WIDE_ROWS - 1) / WIDE_ROWS);                          \
        JB_DISPATCH_V(fast_v(D), __VA_ARGS__);                                                      \
    } else {                                                                                        \
        constexpr int WW = 1;                                                                       \
        const unsigned nb = (unsigned) ((M_ + FAST_ROWS - 1) / FAST_ROWS);                          \
        JB_DISPATCH_V(fast_v(D), __VA_ARGS__);                                                      \
    }

// ---------------------------------------------------------------------------------------------
__global__ void k_linear_simt(const float * __restrict__ x, int ldx, const float * __restrict__ w, const float * __restrict__ b,
                              float * __restrict__ y, int ldy, int M, int N, int K) {
    const size_t idx = (size_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (size_t) M * N) return;
    const int r = (int) (idx / N), o = (int) (idx % N);
    const float * xr = x + (size_t) r * ldx;
    const float * wr = w + (size_t) o * K;
    float acc = b ? b[o] : 0.0f;
    for (int i = 0; i < K; i++) acc = acc + xr[i] * wr[i];
    y[(size_t) r * ldy + o] = acc;
}

__global__ void k_split(const float * __restrict__ x, int ldx, float * __restrict__ hi, float * __restrict__ lo, int ldo, int M, int N) {
    const size_t idx = (size_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (size_t) M * N) return;
    const int r = (int) (idx / N), c = (int) (idx % N);
    store_split(hi + (size_t) r * ldo, lo + (size_t) r * ldo, c, x[(size_t) r * ldx + c]);
}

__global__ void k_add_row(const float * __restrict__ x, int ldx, const float * __restrict__ row, float * __restrict__ y, int ldy, int M, int N) {
    const size_t idx = (size_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (size_t) M * N) return;
    const int r = (int) (idx / N), c = (int) (idx % N);
    y[(size_t) r * ldy + c] = x[(size_t) r * ldx + c] + row[c];
}

// activation codes: 1 GELU (erf), 2 SiLU, 3 ReLU, 4 GELU (tanh form: 0.5 v (1 + tanh(sqrt(2 / pi) (v + 0.044715 v^3))))
__device__ __forceinline__ float act_f(float v, int act) {
    if (act == 2) return v / (1.0f + expf(-v));
    if (act == 3) return v > 0 ? v : 0.0f;
    if (act == 4) return 0.5f * v * (1.0f + tanhf(0.79788456080286536f * (v + 0.044715f * v * v * v)));
    return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
}
__device__ __forceinline__ float act_d(float v, int act) {
    if (act == 2) { const float s = 1.0f / (1.0f + expf(-v)); return s * (1.0f + v * (1.0f - s)); }
    if (act == 3) return v > 0 ? 1.0f : 0.0f;
    if (act == 4) {
        const float t = tanhf(0.79788456080286536f * (v + 0.044715f * v * v * v));
        return 0.5f * (1.0f + t) + 0.5f * v * (1.0f - t * t) * 0.79788456080286536f * (1.0f + 3.0f * 0.044715f * v * v);
    }
    return 0.5f * (1.0f + erff(v * 0.70710678118654752f)) + v * 0.39894228040143268f * expf(-0.5f * v * v);
}

__global__ void k_act_fwd(const float * __restrict__ x, int ldx, float * __restrict__ y, int ldy, int M, int N, int act) {
    const size_t idx = (size_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (size_t) M * N) return;
    const int r = (int) (idx / N), c = (int) (idx % N);
    y[(size_t) r * ldy + c] = act_f(x[(size_t) r * ldx + c], act);
}

__global__ void k_act_bwd(const float * __restrict__ gy, int ldgy, const float * __restrict__ x, int ldx, float * __restrict__ gx,
                          int ldgx, int M, int N, int act, int accumulate) {
    const size_t idx = (size_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (size_t) M * N) return;
    const int r = (int) (idx / N), c = (int) (idx % N);
    const float v = gy[(size_t) r * ldgy + c] * act_d(x[(size_t) r * ldx + c], act);
    float * o = gx + (size_t) r * ldgx + c;
    *o = accumulate ? *o + v : v;
}

__global__ void k_gated_add(const float * __restrict__ x, int ldx, const float * __restrict__ a, int lda,
                            const float * __restrict__ gate, int ld_gate, float * __restrict__ y, int ldy, int M, int N) {
    const size_t idx = (size_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (size_t) M * N) return;
    const int r = (int) (idx / N), c = (int) (idx % N);
    y[(size_t) r * ldy + c] = x[(size_t) r * ldx + c] + a[(size_t) r * lda + c] * gate[(size_t) r * ld_gate + c];
}

__global__ void k_add_inplace(float * __restrict__ y, int ldy, const float * __restrict__ x, int ldx, int M, int N) {
    const size_t idx = (size_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (size_t) M * N) return;
    const int r = (int) (idx / N), c = (int) (idx % N);
    y[(size_t) r * ldy + c] = y[(size_t) r * ldy + c] + x[(size_t) r * ldx + c];
}

__global__ void k_copy_rows(const float * __restrict__ x, int ldx, float * __restrict__ y, int ldy, int M, int N) {
    const size_t idx = (size_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (size_t) M * N) return;
    const int r = (int) (idx / N), c = (int) (idx % N);
    y[(size_t) r * ldy + c] = x[(size_t) r * ldx + c];
}

__global__ void k_fill(float * y, float v, size_t n) {
    const size_t idx = (size_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (idx < n) y[idx] = v;
}

__global__ void k_gather_actions(const float * __restrict__ x, float * __restrict__ a_all, int S, int T, int A) {
    const size_t idx = (size_t) blockIdx.x * blockDim.x + threadIdx.x;   // over [T][S][A]
    if (idx >= (size_t) S * T * A) return;
    const int a = (int) (idx % A);
    const size_t ts = idx / A;
    const int r = (int) (ts % S), t = (int) (ts / S);
    a_all[idx] = x[((size_t) r * T + t) * A + a];
}

__global__ void k_scatter_actions(const float * __restrict__ da, float * __restrict__ grad, int S, int T, int A) {
    const size_t idx = (size_t) blockIdx.x * blockDim.x + threadIdx.x;   // over [S][T][A]
    if (idx >= (size_t) S * T * A) return;
    const int a = (int) (idx % A);
    const size_t rt = idx / A;
    const int t = (int) (rt % T), r = (int) (rt / T);
    grad[idx] = da[((size_t) t * S + r) * A + a];
}

struct CostArgs {
    const float * const * preds;
    const float * goals;
    const float * weights;
    float * const * gpreds;
    int W, M, D, ldp;
    float * cost;
    int want_grad;
};

// one warp per row: cost[r] = sum_j w_j * (float) sum_i (p - g)^2 (double per j), as chunk_cost
__global__ void k_cost_l2(CostArgs c) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * ROWS_PER_BLOCK + (threadIdx.x >> 5);
    if (row >= c.M) return;
    float total = c.cost[row];
    for (int j = 0; j < c.W; j++) {
        const float * p = c.preds[j] + (size_t) row * c.ldp;
        const float * g = c.goals + (size_t) j * c.D;
        const float w = c.weights[j];
        double acc = 0;
        for (int i = lane; i < c.D; i += 32) {
            const float diff = p[i] - g[i];
            acc += (double) diff * diff;
            if (c.want_grad) {
                float * gp = c.gpreds[j] + (size_t) row * c.ldp;
                gp[i] = gp[i] + 2.0f * w * diff;
            }
        }
        acc = warp_sum(acc);
        total = total + w * (float) acc;
    }
    if (lane == 0) c.cost[row] = total;
}

__global__ void k_adam(float * __restrict__ x, float * __restrict__ m, float * __restrict__ v, const float * __restrict__ g_t,
                       float * __restrict__ a_all, const float * __restrict__ sched, int * step_ctr, float lr_wd,
                       const float * __restrict__ z, float noise_std, size_t z_stride, const float * __restrict__ lo,
                       const float * __restrict__ hi, int S, int T, int A) {
    const size_t idx = (size_t) blockIdx.x * blockDim.x + threadIdx.x;   // over [S][T][A]
    const size_t N = (size_t) S * T * A;
    const int k = *(volatile int *) step_ctr;
    if (idx < N) {
        const int a = (int) (idx % A);
        const size_t rt = idx / A;
        const int t = (int) (rt % T), r = (int) (rt / T);
        const size_t tm = ((size_t) t * S + r) * A + a;
        const float g = g_t[tm];
        const float step_size = sched[2 * k], c2s = sched[2 * k + 1];
        const float b1 = 0.9f, b2 = 0.999f, eps = 1e-8f;
        float xv = x[idx] * (1.0f - lr_wd);
        const float mv = b1 * m[idx] + (1.0f - b1) * g;
        const float vv = b2 * v[idx] + (1.0f - b2) * g * g;
        xv = xv - step_size * mv / (sqrtf(vv) / c2s + eps);
        if (z) xv = xv + z[(size_t) k * z_stride + idx] * noise_std;
        if (lo) xv = fminf(fmaxf(xv, lo[a]), hi[a]);
        x[idx] = xv;
        m[idx] = mv;
        v[idx] = vv;
        a_all[tm] = xv;
    }
    // the step counter moves once every block has read it: the last block to finish bumps it
    __shared__ bool last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        last = atomicAdd(step_ctr + 1, 1) == (int) gridDim.x - 1;
    }
    __syncthreads();
    if (last && threadIdx.x == 0) {
        step_ctr[1] = 0;
        __threadfence();
        step_ctr[0] = k + 1;
    }
}

__global__ void k_argmin(const float * __restrict__ cost, int n, int * idx, float * val) {
    __shared__ float sv[1024];
    __shared__ int si[1024];
    float best = INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float c = cost[i];
        if (bi == 0x7fffffff || c < best) { best = c; bi = i; }   // strict: the first minimum wins
    }
    sv[threadIdx.x] = best;
    si[threadIdx.x] = bi;
    __syncthreads();
    for (int s = blockDim.x / 2; s > 0; s >>= 1) {
        if ((int) threadIdx.x < s) {
            const float o = sv[threadIdx.x + s];
            const int oi = si[threadIdx.x + s];
            if (o < sv[threadIdx.x] || (o == sv[threadIdx.x] && oi < si[threadIdx.x])) { sv[threadIdx.x] = o; si[threadIdx.x] = oi; }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) { *idx = si[0] == 0x7fffffff ? 0 : si[0]; *val = sv[0]; }
}

inline unsigned blocks_for(size_t n, int t = 256) { return (unsigned) ((n + t - 1) / t); }
inline unsigned row_blocks(int M) { return (unsigned) ((M + ROWS_PER_BLOCK - 1) / ROWS_PER_BLOCK); }

}  // namespace

// ---------------------------------------------------------------------------------------------
void block_pre(const float * x, int ldx, const float * mod, int ld_mod, int sh_off, int sc_off, const float * ln_w,
               const float * ln_b, float eps0, float eps1, float * h_hi, float * h_lo, int ldh, LnStats * st0,
               LnStats * st1, int M, int D, cudaStream_t st) {
    if (M <= 0) return;
    if (fast_v(D)) {
        const int M_ = M;
        JB_DISPATCH_VW(D, (launch_pdl(k_block_pre_v<VV, WW>, nb, 32 * WW * rows_per_block<WW>(), 0, st, x, ldx, mod, ld_mod,
                                      sh_off, sc_off, ln_w, ln_b, eps0, eps1, h_hi, h_lo, ldh, st0, st1, M, D)));
        return;
    }
    k_block_pre<<<row_blocks(M), 32 * ROWS_PER_BLOCK, 0, st>>>(x, ldx, mod, ld_mod, sh_off, sc_off, ln_w, ln_b, eps0,
                                                              eps1, h_hi, h_lo, ldh, st0, st1, M, D);
}

void layer_norm(const float * x, int ldx, const float * w, const float * b, float eps, float * y, int ldy, float * hi,
                float * lo, LnStats * stats, int M, int D, cudaStream_t st) {
    if (M <= 0) return;
    if (fast_v(D)) {
        const int M_ = M;
        JB_DISPATCH_VW(D, (launch_pdl(k_layer_norm_v<VV, WW>, nb, 32 * WW * rows_per_block<WW>(), 0, st, x, ldx, w, b, eps, y,
                                      ldy, hi, lo, stats, M, D)));
        return;
    }
    k_layer_norm<<<row_blocks(M), 32 * ROWS_PER_BLOCK, 0, st>>>(x, ldx, w, b, eps, y, ldy, hi, lo, stats, M, D);
}

void layer_norm_bwd(const float * gy, int ldgy, const float * x, int ldx, const LnStats * stats, const float * w,
                    const float * gres, int ldres, float * gx, int ldgx, const float * dn, int lddn, const float * gate,
                    int ld_gate, float * dmod_hi, float * dmod_lo, int ld_dmod, float * d_hi, float * d_lo, int ldd,
                    int M, int D, cudaStream_t st) {
    if (M <= 0) return;
    if (fast_v(D)) {
        const int M_ = M;
        JB_DISPATCH_VW(D, (launch_pdl(k_layer_norm_bwd_v<VV, WW>, nb, 32 * WW * rows_per_block<WW>(), 0, st, gy, ldgy, x, ldx,
                                      stats, w, gres, ldres, gx, ldgx, dn, lddn, gate, ld_gate, dmod_hi, dmod_lo, ld_dmod, d_hi,
                                      d_lo, ldd, M, D)));
        return;
    }
    k_layer_norm_bwd<<<row_blocks(M), 32 * ROWS_PER_BLOCK, 0, st>>>(gy, ldgy, x, ldx, stats, w, gres, ldres, gx, ldgx, dn,
                                                                   lddn, gate, ld_gate, dmod_hi, dmod_lo, ld_dmod, d_hi,
                                                                   d_lo, ldd, M, D);
}

void block_bwd(const BlockBwdArgs & a, cudaStream_t st) {
    if (a.M <= 0) return;
    if (fast_v(a.D)) {
        const int M_ = a.M;
        JB_DISPATCH_VW(a.D, (launch_pdl(k_block_bwd_v<VV, WW>, nb, 32 * WW * rows_per_block<WW>(), 0, st, a)));
        return;
    }
    k_block_bwd<<<row_blocks(a.M), 32 * ROWS_PER_BLOCK, 0, st>>>(a);
}

void linear_simt(const float * x, int ldx, const float * w, const float * b, float * y, int ldy, int M, int N, int K,
                 cudaStream_t st) {
    const size_t n = (size_t) M * N;
    if (n) k_linear_simt<<<blocks_for(n), 256, 0, st>>>(x, ldx, w, b, y, ldy, M, N, K);
}

void split_f32(const float * x, int ldx, float * hi, float * lo, int ldo, int M, int N, cudaStream_t st) {
    const size_t n = (size_t) M * N;
    if (n) k_split<<<blocks_for(n), 256, 0, st>>>(x, ldx, hi, lo, ldo, M, N);
}

void add_row_vec(const float * x, int ldx, const float * row, float * y, int ldy, int M, int N, cudaStream_t st) {
    const size_t n = (size_t) M * N;
    if (n) k_add_row<<<blocks_for(n), 256, 0, st>>>(x, ldx, row, y, ldy, M, N);
}

void act_fwd(const float * x, int ldx, float * y, int ldy, int M, int N, int act, cudaStream_t st) {
    const size_t n = (size_t) M * N;
    if (n) k_act_fwd<<<blocks_for(n), 256, 0, st>>>(x, ldx, y, ldy, M, N, act);
}

void act_bwd(const float * gy, int ldgy, const float * x, int ldx, float * gx, int ldgx, int M, int N, int act,
             bool accumulate, cudaStream_t st) {
    const size_t n = (size_t) M * N;
    if (n) k_act_bwd<<<blocks_for(n), 256, 0, st>>>(gy, ldgy, x, ldx, gx, ldgx, M, N, act, accumulate ? 1 : 0);
}

void gated_add(const float * x, int ldx, const float * a, int lda, const float * gate, int ld_gate, float * y, int ldy,
               int M, int N, cudaStream_t st) {
    const size_t n = (size_t) M * N;
    if (n) k_gated_add<<<blocks_for(n), 256, 0, st>>>(x, ldx, a, lda, gate, ld_gate, y, ldy, M, N);
}

void add_inplace(float * y, int ldy, const float * x, int ldx, int M, int N, cudaStream_t st) {
    const size_t n = (size_t) M * N;
    if (n) k_add_inplace<<<blocks_for(n), 256, 0, st>>>(y, ldy, x, ldx, M, N);
}

void copy_rows(const float * x, int ldx, float * y, int ldy, int M, int N, cudaStream_t st) {
    const size_t n = (size_t) M * N;
    if (n) k_copy_rows<<<blocks_for(n), 256, 0, st>>>(x, ldx, y, ldy, M, N);
}

void fill_f32(float * y, float v, size_t n, cudaStream_t st) {
    if (n) k_fill<<<blocks_for(n), 256, 0, st>>>(y, v, n);
}

void gather_actions(const float * x, float * a_all, int S, int T, int A, cudaStream_t st) {
    const size_t n = (size_t) S * T * A;
    if (n) k_gather_actions<<<blocks_for(n), 256, 0, st>>>(x, a_all, S, T, A);
}

void scatter_actions(const float * da, float * grad, int S, int T, int A, cudaStream_t st) {
    const size_t n = (size_t) S * T * A;
    if (n) k_scatter_actions<<<blocks_for(n), 256, 0, st>>>(da, grad, S, T, A);
}

void cost_l2(const float * const * preds, const float * goals, const float * weights, float * const * gpreds, int W,
             int M, int D, int ldp, float * cost, bool want_grad, cudaStream_t st) {
    if (M <= 0) return;
    CostArgs c{preds, goals, weights, gpreds, W, M, D, ldp, cost, want_grad ? 1 : 0};
    k_cost_l2<<<row_blocks(M), 32 * ROWS_PER_BLOCK, 0, st>>>(c);
}

void adam_step(float * x, float * m, float * v, const float * grad_tmajor, float * a_all, const float * sched,
               int * step_ctr, float lr_wd, const float * z, float noise_std, size_t z_stride, const float * lo,
               const float * hi, int S, int T, int A, cudaStream_t st) {
    const size_t n = (size_t) S * T * A;
    k_adam<<<blocks_for(n), 256, 0, st>>>(x, m, v, grad_tmajor, a_all, sched, step_ctr, lr_wd, z, noise_std, z_stride, lo, hi, S, T, A);
}

void argmin_first(const float * cost, int n, int * idx, float * val, cudaStream_t st) {
    k_argmin<<<1, 1024, 0, st>>>(cost, n, idx, val);
}

}  // namespace jb
