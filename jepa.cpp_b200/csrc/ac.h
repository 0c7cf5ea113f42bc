// V-JEPA 2-AC engine of a context: the predictor's device weights (f16 operands, f32 norms / biases),
// the 3-D RoPE tables of every frame slot, and the rollout workspaces.
//
// The predictor is evaluated frame by frame with a key / value cache: under the block-causal frame mask
// (reference: src/vjepa2_ac.cpp:355-366) the hidden states of frame t depend only on frames 0..t, so a
// rollout step computes only its new frame's rows and attends to the cached keys and values of the
// frames before it. The reference recomputes the whole prefix every step (ac_rollout,
// src/vjepa2_ac.cpp:455-577); the results are the same rows. Frames every candidate shares (the observed
// frames before the last, when the caller gives their actions) are computed once, at candidate stride 0.
#pragma once

#include "common.h"
#include "kernels.h"

#include <cuda_fp16.h>

#include <cstdint>
#include <vector>

struct jepa_model;
struct jepa_context;

namespace jb {

struct ACLayer {
    const float * ln1_w = nullptr, * ln1_b = nullptr, * ln2_w = nullptr, * ln2_b = nullptr;
    const __half * wqkv = nullptr, * wout = nullptr, * wup = nullptr, * wdown = nullptr;
    const float * bqkv = nullptr, * bout = nullptr, * bup = nullptr, * bdown = nullptr;
};

// Keys / values of one frame: layer l at base + l * layer_stride, candidate c at + c * cand_stride
// (elements; cand_stride 0 = shared by every candidate). Rows [kv_rows][2 D], k then v.
struct KVRef {
    const __half * base = nullptr;
    long long layer_stride = 0, cand_stride = 0;
};

// One predictor evaluation over `nf` consecutive frames [f0, f0 + nf) of `n_cand` candidates.
struct PassSpec {
    int n_cand = 1, f0 = 0, nf = 1;
    const __half * lat[AC_MAX_FRAMES] = {};      // f16 latents [HW][E] of pass frame k, candidate c at lat[k] + c * lat_cand[k]
    long long lat_cand[AC_MAX_FRAMES] = {};      // 0 (shared: embedded once, broadcast) or HW * E
    const float * acts = nullptr, * sts = nullptr;   // frame k of candidate c: acts + c * act_cand + k * A
    long long act_cand = 0, st_cand = 0;
    __half * kv_out = nullptr;                   // this pass's cache block, rows [cand][nf][R][2 D] per layer
    long long kv_layer = 0;
    KVRef keys[AC_MAX_FRAMES];                   // key frames 0 .. f0-1 (the pass's own frames follow)
    bool full = false;                           // no frame mask: every query frame sees every frame of the pass
    int n_out = 0;                               // trailing frames projected to out [n_cand][n_out][HW][out_dim]
    float * out = nullptr;
    __half * out16 = nullptr;                    // optional f16 copy of out (the next step's embedding input)
    bool normalize = false;                      // jepa_ac_normalize on out (rollouts with normalize_reps)
};

struct ACEngine {
    int device = 0;
    int D = 0, E = 0, OUT = 0, F = 0, L = 0, NH = 0, HD = 0, A = 0, S = 0, HW = 0, R = 0, slots = 0;
    float ln_eps = 1e-6f, norm_eps = 1e-5f;
    bool normalize = false, causal = false;

    std::vector<void *> allocations;             // weights and tables
    std::vector<ACLayer> layers;
    const __half * wembed = nullptr, * wproj = nullptr;
    const float * bembed = nullptr, * bproj = nullptr, * wact = nullptr, * bact = nullptr, * wst = nullptr, * bst = nullptr;
    const float * norm_w = nullptr, * norm_b = nullptr;
    float * rope_cos = nullptr, * rope_sin = nullptr;   // [slots + 2 grid][rope_d] per-axis tables, sin sign-folded
    int rope_d = 0, grid = 1;

    // grow-only device buffers
    struct Buf {
        void * p = nullptr;
        size_t bytes = 0;
    };
    Buf ws, kv_shared, kv_cand, outs, io;
    // shared-prefix cache: the handle and its generation whose shared frames kv_shared holds
    const void * shared_owner = nullptr;
    uint64_t shared_gen = 0;
    int shared_frames = 0;
    long long launches = 0;                      // kernels launched (running count; callers take differences)

    ~ACEngine();
    bool init(const jepa_model & m, cudaStream_t st);
    bool grow(Buf & b, size_t bytes, const char * what);
    size_t ws_bytes(long long rows) const;
    int pass(const PassSpec & p, cudaStream_t st);
};

// The AC engine of a context, built on first use; nullptr (with the reason logged) when the model has no
// action-conditioned predictor or the engine cannot be built for it.
ACEngine * ac_engine_of(jepa_context * ctx, const char * fn);

}  // namespace jb
