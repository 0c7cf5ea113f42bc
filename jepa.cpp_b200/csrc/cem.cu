// The CEM planner's sampling and elite refit on the device (jepa_ac_plan).
//
// k_cem_sample  the candidates' actions of one iteration from the sampling distribution kept on the
//               device: translation lanes 0..2 and the gripper (lane 6) drawn as z * std + mean and
//               clamped (+-maxnorm, +-gripper_clamp); the rotation lanes stay 0
// k_cem_refit   one CTA: the top-k LOWEST energies, ties to the lower candidate index (a stable sort's
//               first k), then per (horizon step, lane) the elites' mean and unbiased standard deviation,
//               summed in double in elite order, and the momentum update of the distribution
//
// The arithmetic is the reference's (src/vjepa2_ac.cpp:866-935): float sampling with two roundings, double
// elite statistics, float * float momentum terms added in double; with -fmad=false nothing is contracted,
// so the device refit gives the host loop's bits.
#include "kernels.h"
#include "common.h"

namespace jb {

namespace {

constexpr int REFIT_THREADS = 256;

__global__ void k_cem_sample(const float * __restrict__ noise, const float * __restrict__ mean, const float * __restrict__ sd,
                             int K, int H, int A, float maxnorm, float grip, float * __restrict__ acts) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;   // (candidate, horizon step)
    if (i >= K * H) return;
    const int c = i / H, h = i % H;
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const float z = noise[((size_t) h * K + c) * 4 + j];
        const float scaled = z * sd[h * 4 + j];
        v[j] = scaled + mean[h * 4 + j];
    }
#pragma unroll
    for (int j = 0; j < 3; j++) {
        if (v[j] < -maxnorm) v[j] = -maxnorm;
        if (v[j] > maxnorm) v[j] = maxnorm;
    }
    if (v[3] < -grip) v[3] = -grip;
    if (v[3] > grip) v[3] = grip;
    float * a = acts + ((size_t) c * H + h) * A;
    for (int j = 0; j < A; j++) a[j] = 0.0f;
    a[0] = v[0];
    a[1] = v[1];
    a[2] = v[2];
    a[6] = v[3];
}

// (energy, index) as one unsigned key ordered like (energy ascending, index ascending); -0 counts as +0
// (they compare equal) and NaN after every number
__device__ __forceinline__ unsigned long long order_key(float e, int c) {
    uint32_t u = __float_as_uint(e == 0.0f ? 0.0f : e);
    if (e != e) u = 0xFFFFFFFFu;
    else u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long) u << 32) | (uint32_t) c;
}

__device__ __forceinline__ unsigned long long warp_min_u64(unsigned long long v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
        v = w < v ? w : v;
    }
    return v;
}

struct RefitArgs {
    const float * energy;     // [K]
    const float * acts;       // [K][H][A] this iteration's samples
    float * mean, * sd;       // [H][4], updated in place
    float * best;             // the lowest energy of the iteration, written to best[0]
    int * elite;              // [topk] scratch: the elites' indices in rank order
    int K, H, A, topk;
    float m_mean, m_std, m_mean_grip, m_std_grip;
};

__global__ void __launch_bounds__(REFIT_THREADS) k_cem_refit(RefitArgs r) {
    __shared__ unsigned long long part[REFIT_THREADS / 32];
    __shared__ unsigned long long chosen;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    // k rounds of a block-wide minimum over the keys above the last one chosen
    unsigned long long floor_key = 0;
    bool first = true;
    for (int e = 0; e < r.topk; e++) {
        unsigned long long best = ~0ull;
        for (int c = t; c < r.K; c += REFIT_THREADS) {
            const unsigned long long k = order_key(r.energy[c], c);
            if ((first || k > floor_key) && k < best) best = k;
        }
        best = warp_min_u64(best);
        if (lane == 0) part[warp] = best;
        __syncthreads();
        if (warp == 0) {
            unsigned long long v = lane < REFIT_THREADS / 32 ? part[lane] : ~0ull;
            v = warp_min_u64(v);
            if (lane == 0) {
                chosen = v;
                r.elite[e] = (int) (uint32_t) v;
                if (e == 0) r.best[0] = r.energy[(uint32_t) v];
            }
        }
        __syncthreads();
        floor_key = chosen;
        first = false;
    }
    // per (horizon step, sampled lane): the elites' statistics and the momentum update
    for (int i = t; i < r.H * 4; i += REFIT_THREADS) {
        const int h = i >> 2, j = i & 3;
        const int col = j < 3 ? j : 6;
        double mu = 0.0;
        for (int e = 0; e < r.topk; e++) mu += r.acts[((size_t) r.elite[e] * r.H + h) * r.A + col];
        mu /= (double) r.topk;
        double ss = 0.0;
        for (int e = 0; e < r.topk; e++) {
            const double d = r.acts[((size_t) r.elite[e] * r.H + h) * r.A + col] - mu;
            ss += d * d;
        }
        const double dev = sqrt(ss / (r.topk > 1 ? (double) (r.topk - 1) : 1.0));   // unbiased (n - 1)
        const float mm = j < 3 ? r.m_mean : r.m_mean_grip, ms = j < 3 ? r.m_std : r.m_std_grip;
        const float keep_mean = r.mean[i] * mm, keep_sd = r.sd[i] * ms;       // float products
        r.mean[i] = (float) (mu * (1.0 - (double) mm) + (double) keep_mean);
        r.sd[i] = (float) (dev * (1.0 - (double) ms) + (double) keep_sd);
    }
}

}  // namespace

void cem_sample(const float * noise, const float * mean, const float * sd, int K, int H, int A, float maxnorm,
                float gripper_clamp, float * acts, cudaStream_t st) {
    const int n = K * H;
    k_cem_sample<<<(n + 255) / 256, 256, 0, st>>>(noise, mean, sd, K, H, A, maxnorm, gripper_clamp, acts);
}

void cem_refit(const float * energy, const float * acts, float * mean, float * sd, float * best, int * elite, int K, int H,
               int A, int topk, float m_mean, float m_std, float m_mean_grip, float m_std_grip, cudaStream_t st) {
    RefitArgs r{energy, acts, mean, sd, best, elite, K, H, A, topk, m_mean, m_std, m_mean_grip, m_std_grip};
    k_cem_refit<<<1, REFIT_THREADS, 0, st>>>(r);
}

}  // namespace jb
