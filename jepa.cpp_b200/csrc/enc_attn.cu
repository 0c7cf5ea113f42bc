// The encoders' token assembly, 3-D RoPE and attention (float32).
//
// Attention: one thread per query, 64 queries of one (item, head) per CTA; the item's keys and values
// stream through shared memory 32 at a time and every thread keeps its running maximum, normaliser and
// weighted sum in registers (the online softmax), so an item never materialises its score matrix. A
// block-causal item gives each query a contiguous key range (its temporal slot and the ones before it),
// so the mask is two bounds per query, not a table. Encoders run once per observation: latency-scale work.
#include "encoder.h"
#include "common.h"

#include <algorithm>
#include <cmath>

namespace jb {

namespace {

constexpr int QT = 64;   // queries (threads) per CTA
constexpr int KT = 32;   // keys per shared-memory tile

template <int HD>
__global__ void __launch_bounds__(QT) k_enc_attn(const float * __restrict__ qkv, float * __restrict__ o, int N, int D, float scale,
                                                 int n_prefix, int tpf) {
    __shared__ float sk[KT][HD];
    __shared__ float sv[KT][HD];
    const int item = blockIdx.z, h = blockIdx.y;
    const int qi = blockIdx.x * QT + threadIdx.x;
    const bool valid = qi < N;
    const size_t base = (size_t) item * N;
    const size_t ld = (size_t) 3 * D;
    float q[HD], acc[HD];
#pragma unroll
    for (int c = 0; c < HD; c++) {
        q[c] = valid ? qkv[(base + qi) * ld + (size_t) h * HD + c] : 0.0f;
        acc[c] = 0.0f;
    }
    // this query's keys [k_lo, k_hi): all of them, or (block-causal patch query) its slot and earlier ones
    int k_lo = 0, k_hi = N;
    if (tpf > 0 && qi >= n_prefix) {
        k_lo = n_prefix;
        k_hi = min(N, n_prefix + ((qi - n_prefix) / tpf + 1) * tpf);
    }
    float m = -INFINITY, l = 0.0f;
    for (int k0 = 0; k0 < N; k0 += KT) {
        for (int idx = threadIdx.x; idx < KT * HD; idx += QT) {
            const int j = idx / HD, c = idx % HD, key = k0 + j;
            const size_t r = (base + key) * ld + (size_t) h * HD + c;
            sk[j][c] = key < N ? qkv[r + D] : 0.0f;
            sv[j][c] = key < N ? qkv[r + 2 * (size_t) D] : 0.0f;
        }
        __syncthreads();
        const int nk = min(KT, N - k0);
        if (valid) {
            for (int j = 0; j < nk; j++) {
                if (k0 + j < k_lo || k0 + j >= k_hi) continue;
                float s = 0.0f;
#pragma unroll
                for (int c = 0; c < HD; c++) s += q[c] * sk[j][c];
                s = s * scale;
                if (s > m) {   // a new maximum: rescale what has been summed so far
                    const float corr = expf(m - s);
                    l = l * corr;
#pragma unroll
                    for (int c = 0; c < HD; c++) acc[c] = acc[c] * corr;
                    m = s;
                }
                const float p = expf(s - m);
                l = l + p;
#pragma unroll
                for (int c = 0; c < HD; c++) acc[c] = acc[c] + p * sv[j][c];
            }
        }
        __syncthreads();
    }
    if (valid) {
        float * out = o + (base + qi) * (size_t) D + (size_t) h * HD;
#pragma unroll
        for (int c = 0; c < HD; c++) out[c] = acc[c] / l;
    }
}

__global__ void k_enc_tokens(const float * __restrict__ patches, const float * __restrict__ cls, const float * __restrict__ reg,
                             const float * __restrict__ pos, float * __restrict__ X, int items, int N, int n_cls, int n_reg,
                             int D, const float * __restrict__ mod) {
    const size_t n = (size_t) items * N * D;
    const int P = N - n_cls - n_reg;
    for (size_t idx = (size_t) blockIdx.x * blockDim.x + threadIdx.x; idx < n; idx += (size_t) gridDim.x * blockDim.x) {
        const int d = (int) (idx % D);
        const size_t rt = idx / D;
        const int t = (int) (rt % N);
        const size_t i = rt / N;
        float v;
        if (t < n_cls) v = cls[d];
        else if (t < n_cls + n_reg) v = reg[(size_t) (t - n_cls) * D + d];
        else {
            v = patches[(i * P + (t - n_cls - n_reg)) * D + d];
            if (mod) v = v + mod[d];
        }
        X[idx] = pos ? v + pos[(size_t) t * D + d] : v;
    }
}

// one thread per (token, head, rotated pair); the last hd - 3 d lanes of a head have cos 1, sin 0 and are
// rotated as well (to themselves), which keeps the kernel to whole pairs
__global__ void k_enc_rope(float * __restrict__ qkv, const float * __restrict__ cos, const float * __restrict__ sin, int items,
                           int N, int D, int heads) {
    const int hd = D / heads, pairs = hd / 2;
    const size_t n = (size_t) items * N * heads * pairs;
    for (size_t idx = (size_t) blockIdx.x * blockDim.x + threadIdx.x; idx < n; idx += (size_t) gridDim.x * blockDim.x) {
        const int k = (int) (idx % pairs);
        const size_t th = idx / pairs;
        const int h = (int) (th % heads);
        const size_t row = th / heads;
        const int t = (int) (row % N);
        const float * c = cos + (size_t) t * hd + 2 * k;
        const float * s = sin + (size_t) t * hd + 2 * k;
        for (int part = 0; part < 2; part++) {   // q, then k
            float * x = qkv + row * (size_t) (3 * D) + (size_t) part * D + (size_t) h * hd + 2 * k;
            const float x0 = x[0], x1 = x[1];
            const float a0 = x0 * c[0], b0 = -x1 * s[0];
            const float a1 = x1 * c[1], b1 = x0 * s[1];
            x[0] = a0 + b0;
            x[1] = a1 + b1;
        }
    }
}

template <int HD>
void launch_attn(const float * qkv, float * o, int items, int N, int D, int heads, cudaStream_t st, int n_prefix, int tpf) {
    const dim3 grid((unsigned) ((N + QT - 1) / QT), (unsigned) heads, (unsigned) items);
    k_enc_attn<HD><<<grid, QT, 0, st>>>(qkv, o, N, D, 1.0f / std::sqrt((float) HD), n_prefix, tpf);
}

}  // namespace

bool enc_attention_supported(int D, int heads) {
    if (heads < 1 || D % heads) return false;
    const int hd = D / heads;
    return hd == 32 || hd == 48 || hd == 64 || hd == 80 || hd == 88 || hd == 96 || hd == 128;
}

bool enc_attention(const float * qkv, float * o, int items, int N, int D, int heads, cudaStream_t st, int n_prefix,
                   int block_causal_tpf) {
    if (items < 1 || N < 1) return true;
    if (heads < 1 || D % heads) return false;
    const int p = n_prefix, t = block_causal_tpf;
    switch (D / heads) {
        case 32: launch_attn<32>(qkv, o, items, N, D, heads, st, p, t); return true;
        case 48: launch_attn<48>(qkv, o, items, N, D, heads, st, p, t); return true;
        case 64: launch_attn<64>(qkv, o, items, N, D, heads, st, p, t); return true;
        case 80: launch_attn<80>(qkv, o, items, N, D, heads, st, p, t); return true;
        case 88: launch_attn<88>(qkv, o, items, N, D, heads, st, p, t); return true;
        case 96: launch_attn<96>(qkv, o, items, N, D, heads, st, p, t); return true;
        case 128: launch_attn<128>(qkv, o, items, N, D, heads, st, p, t); return true;
        default: return false;
    }
}

void enc_rope_qk(float * qkv, const float * cos, const float * sin, int items, int N, int D, int heads, cudaStream_t st) {
    const size_t n = (size_t) items * N * D / 2;
    if (!n) return;
    const unsigned blocks = (unsigned) std::min<size_t>((n + 255) / 256, (size_t) 148 * 16);
    k_enc_rope<<<blocks, 256, 0, st>>>(qkv, cos, sin, items, N, D, heads);
}

void enc_tokens(const float * patches, const float * cls, const float * reg, const float * pos, float * X, int items, int N,
                int n_cls, int n_reg, int D, cudaStream_t st, const float * mod) {
    const size_t n = (size_t) items * N * D;
    if (!n) return;
    const unsigned blocks = (unsigned) std::min<size_t>((n + 255) / 256, (size_t) 148 * 16);
    k_enc_tokens<<<blocks, 256, 0, st>>>(patches, cls, reg, pos, X, items, N, n_cls, n_reg, D, mod);
}

}  // namespace jb
