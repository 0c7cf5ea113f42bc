// The encoders on the GPU (jepa_encode; reference: src/jepa.cpp:586-1000). Image families: patch embedding,
// CLS / register tokens, learned positions, pre-LN transformer blocks (optional layer scale), final norm;
// every (batch, frame) slice is one sequence. Video families (V-JEPA 2 / 2.1, LeVJEPA): tubelet patch
// embedding, optional modality vector, CLS / registers without positions, 3-D RoPE on the queries and keys
// of every block, full or block-causal attention; every clip is one sequence. A call's sequences run as
// one batch of rows.
#pragma once

#include "hplan.h"

#include <vector>

namespace jb {

struct EncLayer {
    DLin qkv, out, up, down;
    float * ln1_w = nullptr, * ln1_b = nullptr, * ln2_w = nullptr, * ln2_b = nullptr;
    float * ls1 = nullptr, * ls2 = nullptr;    // layer scale (a vector of ones when the model has none)
};

struct EncEngine {
    std::vector<void *> allocations;
    bool video = false;                        // a video family (3-D RoPE instead of learned positions)
    DLin patch;
    DLin patch_img;                            // V-JEPA 2.1's one-frame image tokenizer (when present)
    float * mod_video = nullptr, * mod_img = nullptr;   // modality vectors (jepa.enc.modality_embed)
    float * cls = nullptr, * reg = nullptr, * pos = nullptr, * norm_w = nullptr, * norm_b = nullptr;
    float * ones = nullptr;
    int64_t pos_rows = 0;
    std::vector<EncLayer> layers;
    ~EncEngine();
    bool build(const jepa_model & m, cudaStream_t st);
};

// the attention of the encoders: every (item, head) over the N tokens of the item, float32.
// qkv [items N][3 D] = [q | k | v], o [items N][D]. hd = D / heads; false = head width not supported.
// block_causal_tpf > 0: block-causal over temporal slots of that many tokens after n_prefix prefix rows -- a
// prefix query sees every key, a patch query the patch keys of its own slot and the slots before it (no
// prefix key).
bool enc_attention(const float * qkv, float * o, int items, int N, int D, int heads, cudaStream_t st,
                   int n_prefix = 0, int block_causal_tpf = 0);
// 3-D RoPE in place on the q and k columns of qkv [items N][3 D]: pair (2k, 2k + 1) of every head of token t
// becomes (x0 cos[t][2k] - x1 sin[t][2k], x1 cos[t][2k+1] + x0 sin[t][2k+1]); cos / sin [N][hd]
void enc_rope_qk(float * qkv, const float * cos, const float * sin, int items, int N, int D, int heads, cudaStream_t st);
bool enc_attention_supported(int D, int heads);
// X[i N + t] = (t < c ? cls : t < c + R ? reg[t - c] : patches[i P + t - c - R] + mod) + pos[t]
// (pos and mod may be null: no positions, no modality vector)
void enc_tokens(const float * patches, const float * cls, const float * reg, const float * pos, float * X, int items,
                int N, int n_cls, int n_reg, int D, cudaStream_t st, const float * mod = nullptr);

}  // namespace jb
