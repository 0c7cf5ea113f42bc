// Kernels of the action cost's pooling (the upper level's action encoder over whole chunks of the
// candidates' action embeddings; src/hjepa-plan.cpp:663-684 and its ops :478-619):
//
//   pool_chunks     e rows of the chunks (t-major, [Wa stride S][E]) <-> the 'mlp' encoder's concatenated
//                   input [Wa S][stride E] (op_concat_cols and its backward)
//   pool_tokens     step-linear outputs <-> the 'seq' encoder's token groups [Wa S][G = stride + 1][d]:
//                   a CLS row pos[0], then step l plus pos[l + 1] (op_tokens and its backward)
//   group_mha_fwd / _bwd
//                   multi-head self-attention inside each token group (op_mha): one CTA per group, the
//                   group's q / k / v rows in shared memory, one thread per (head, query row); the softmax
//                   probabilities are kept [row][head][key] for the backward
//
// Everything here is a few MB per solve iteration (a few hundred candidates x a handful of tokens):
// latency, not bandwidth or FLOPs, is what these kernels cost, so they are plain SIMT over shared memory.
#include "kernels.h"
#include "common.h"

#include <cmath>

namespace jb {

namespace {

// x[(j S + s)][i E + c] <-> e[((j stride + i) S + s)][c]
__global__ void k_pool_chunks(float * __restrict__ e, float * __restrict__ x, int Wa, int S, int stride, int E, int back) {
    const size_t n = (size_t) Wa * S * stride * E;
    for (size_t idx = (size_t) blockIdx.x * blockDim.x + threadIdx.x; idx < n; idx += (size_t) gridDim.x * blockDim.x) {
        const int c = (int) (idx % E);
        const size_t q = idx / E;                 // (j stride + i) S + s
        const int s = (int) (q % S);
        const int ji = (int) (q / S);
        const int j = ji / stride, i = ji % stride;
        const size_t xi = ((size_t) j * S + s) * ((size_t) stride * E) + (size_t) i * E + c;
        if (back) e[idx] = x[xi];
        else x[xi] = e[idx];
    }
}

// X[(g G + l)][c] = l == 0 ? pos[c] : z[((j stride + l - 1) S + s)][c] + pos[l][c],  g = j S + s
// back: gz[((j stride + l - 1) S + s)][c] = gX[(g G + l)][c]
__global__ void k_pool_tokens(float * __restrict__ z, const float * __restrict__ pos, float * __restrict__ X, int Wa, int S,
                              int stride, int d, int back) {
    const int G = stride + 1;
    const size_t n = (size_t) Wa * S * G * d;
    for (size_t idx = (size_t) blockIdx.x * blockDim.x + threadIdx.x; idx < n; idx += (size_t) gridDim.x * blockDim.x) {
        const int c = (int) (idx % d);
        const size_t q = idx / d;                 // g G + l
        const int l = (int) (q % G);
        const size_t g = q / G;
        const int s = (int) (g % S), j = (int) (g / S);
        if (l == 0) {
            if (!back) X[idx] = pos[c];
            continue;
        }
        const size_t zi = (((size_t) j * stride + (l - 1)) * S + s) * d + c;
        if (back) z[zi] = X[idx];
        else X[idx] = z[zi] + pos[(size_t) l * d + c];
    }
}

// One CTA per group of G token rows. qkv [rows][3 d] = [q | k | v]; o [rows][d]; probs [rows][H][G].
__global__ void k_group_mha_fwd(const float * __restrict__ qkv, float * __restrict__ o, float * __restrict__ probs, int G,
                                int d, int H, float scale, int causal) {
    extern __shared__ float sm[];
    float * sq = sm;                              // [G][3 d]
    float * sp = sm + (size_t) G * 3 * d;         // [G][H][G]
    const size_t g0 = (size_t) blockIdx.x * G;
    const int hd = d / H;
    for (int i = threadIdx.x; i < G * 3 * d; i += blockDim.x) sq[i] = qkv[g0 * 3 * d + i];
    __syncthreads();
    for (int pr = threadIdx.x; pr < H * G; pr += blockDim.x) {
        const int h = pr / G, i = pr % G;
        const float * q = sq + (size_t) i * 3 * d + h * hd;
        float * p = sp + ((size_t) i * H + h) * G;
        const int nk = causal ? i + 1 : G;   // causal: query i sees keys 0..i (a masked key has probability 0)
        float mx = -INFINITY;
        for (int j = 0; j < nk; j++) {
            const float * k = sq + (size_t) j * 3 * d + d + h * hd;
            float s = 0.0f;
            for (int c = 0; c < hd; c++) s += q[c] * k[c];
            p[j] = s * scale;
            mx = fmaxf(mx, p[j]);
        }
        float sum = 0.0f;
        for (int j = 0; j < nk; j++) { p[j] = expf(p[j] - mx); sum += p[j]; }
        for (int j = 0; j < nk; j++) p[j] = p[j] / sum;
        for (int j = nk; j < G; j++) p[j] = 0.0f;
        float * out = o + (g0 + i) * d + h * hd;
        for (int c = 0; c < hd; c++) {
            float acc = 0.0f;
            for (int j = 0; j < G; j++) acc += p[j] * sq[(size_t) j * 3 * d + 2 * d + h * hd + c];
            out[c] = acc;
        }
        float * pg = probs + ((g0 + i) * H + h) * G;
        for (int j = 0; j < G; j++) pg[j] = p[j];
    }
}

// gv_j = sum_i p_ij go_i ; gs_ij = p_ij (go_i . v_j - sum_j' p_ij' go_i . v_j') scale ; gq_i = sum_j gs_ij k_j ;
// gk_j = sum_i gs_ij q_i. Writes every element of gqkv (no accumulation).
__global__ void k_group_mha_bwd(const float * __restrict__ go, const float * __restrict__ qkv, const float * __restrict__ probs,
                                float * __restrict__ gqkv, int G, int d, int H, float scale) {
    extern __shared__ float sm[];
    float * sq = sm;                              // [G][3 d]
    float * sgo = sq + (size_t) G * 3 * d;        // [G][d]
    float * sp = sgo + (size_t) G * d;            // [G][H][G]
    float * sg = sp + (size_t) G * H * G;         // [G][H][G] d cost / d score
    const size_t g0 = (size_t) blockIdx.x * G;
    const int hd = d / H;
    for (int i = threadIdx.x; i < G * 3 * d; i += blockDim.x) sq[i] = qkv[g0 * 3 * d + i];
    for (int i = threadIdx.x; i < G * d; i += blockDim.x) sgo[i] = go[g0 * d + i];
    for (int i = threadIdx.x; i < G * H * G; i += blockDim.x) sp[i] = probs[g0 * H * G + i];
    __syncthreads();
    for (int pr = threadIdx.x; pr < H * G; pr += blockDim.x) {
        const int h = pr / G, i = pr % G;
        const float * goi = sgo + (size_t) i * d + h * hd;
        const float * p = sp + ((size_t) i * H + h) * G;
        float * gs = sg + ((size_t) i * H + h) * G;
        float dotp = 0.0f;
        for (int j = 0; j < G; j++) {
            const float * v = sq + (size_t) j * 3 * d + 2 * d + h * hd;
            float s = 0.0f;
            for (int c = 0; c < hd; c++) s += goi[c] * v[c];
            gs[j] = s;
            dotp += s * p[j];
        }
        for (int j = 0; j < G; j++) gs[j] = p[j] * (gs[j] - dotp) * scale;
        float * gq = gqkv + (g0 + i) * 3 * d + h * hd;
        for (int c = 0; c < hd; c++) {
            float acc = 0.0f;
            for (int j = 0; j < G; j++) acc += gs[j] * sq[(size_t) j * 3 * d + d + h * hd + c];
            gq[c] = acc;
        }
    }
    __syncthreads();
    for (int pr = threadIdx.x; pr < H * G; pr += blockDim.x) {
        const int h = pr / G, j = pr % G;
        float * gk = gqkv + (g0 + j) * 3 * d + d + h * hd;
        float * gv = gk + d;
        for (int c = 0; c < hd; c++) {
            float ak = 0.0f, av = 0.0f;
            for (int i = 0; i < G; i++) {
                ak += sg[((size_t) i * H + h) * G + j] * sq[(size_t) i * 3 * d + h * hd + c];
                av += sp[((size_t) i * H + h) * G + j] * sgo[(size_t) i * d + h * hd + c];
            }
            gk[c] = ak;
            gv[c] = av;
        }
    }
}

unsigned grid_for(size_t n) {
    const size_t b = (n + 255) / 256;
    return (unsigned) std::min<size_t>(std::max<size_t>(b, 1), (size_t) 148 * 16);
}

}  // namespace

void pool_chunks(float * e, float * x, int Wa, int S, int stride, int E, bool back, cudaStream_t st) {
    const size_t n = (size_t) Wa * S * stride * E;
    if (n) k_pool_chunks<<<grid_for(n), 256, 0, st>>>(e, x, Wa, S, stride, E, back ? 1 : 0);
}

void pool_tokens(float * z, const float * pos, float * X, int Wa, int S, int stride, int d, bool back, cudaStream_t st) {
    const size_t n = (size_t) Wa * S * (stride + 1) * d;
    if (n) k_pool_tokens<<<grid_for(n), 256, 0, st>>>(z, pos, X, Wa, S, stride, d, back ? 1 : 0);
}

size_t group_mha_smem(int G, int d, int H, bool backward) {
    return backward ? ((size_t) G * 4 * d + (size_t) 2 * G * H * G) * sizeof(float)
                    : ((size_t) G * 3 * d + (size_t) G * H * G) * sizeof(float);
}

bool group_mha_prepare(int G, int d, int H) {
    const size_t f = group_mha_smem(G, d, H, false), b = group_mha_smem(G, d, H, true);
    if (b > 227 * 1024) return false;
    // the opt-in limit only ever grows (per device), so a smaller group never lowers it under a larger one
    static size_t set_f[64] = {}, set_b[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return false;
    if (f > set_f[dev]) {
        if (cudaFuncSetAttribute(k_group_mha_fwd, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) f) != cudaSuccess) return false;
        set_f[dev] = f;
    }
    if (b > set_b[dev]) {
        if (cudaFuncSetAttribute(k_group_mha_bwd, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) b) != cudaSuccess) return false;
        set_b[dev] = b;
    }
    return true;
}

void group_mha_fwd(const float * qkv, float * o, float * probs, int n_groups, int G, int d, int H, cudaStream_t st, bool causal) {
    if (n_groups <= 0) return;
    const float scale = 1.0f / std::sqrt((float) (d / H));
    k_group_mha_fwd<<<n_groups, 128, group_mha_smem(G, d, H, false), st>>>(qkv, o, probs, G, d, H, scale, causal ? 1 : 0);
}

void group_mha_bwd(const float * go, const float * qkv, const float * probs, float * gqkv, int n_groups, int G, int d, int H,
                   cudaStream_t st) {
    if (n_groups <= 0) return;
    const float scale = 1.0f / std::sqrt((float) (d / H));
    k_group_mha_bwd<<<n_groups, 128, group_mha_smem(G, d, H, true), st>>>(go, qkv, probs, gqkv, G, d, H, scale);
}

}  // namespace jb
