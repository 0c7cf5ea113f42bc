// The image encoder on the GPU (jepa_encode for the image families; reference: src/jepa.cpp:586-720):
// patch embedding, CLS / register tokens, learned positions, pre-LN transformer blocks (optional layer
// scale), final norm. Every (batch, frame) slice is one sequence; all of a call's slices run as one batch.
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
    DLin patch;
    float * cls = nullptr, * reg = nullptr, * pos = nullptr, * norm_w = nullptr, * norm_b = nullptr;
    float * ones = nullptr;
    int64_t pos_rows = 0;
    std::vector<EncLayer> layers;
    ~EncEngine();
    bool build(const jepa_model & m, cudaStream_t st);
};

// the attention of the image encoder: every (item, head) over all N tokens of the item, float32.
// qkv [items N][3 D] = [q | k | v], o [items N][D]. hd = D / heads; false = head width not supported
bool enc_attention(const float * qkv, float * o, int items, int N, int D, int heads, cudaStream_t st);
bool enc_attention_supported(int D, int heads);
// X[i N + t] = (t < c ? cls : t < c + R ? reg[t - c] : patches[i P + t - c - R]) + pos[t]
void enc_tokens(const float * patches, const float * cls, const float * reg, const float * pos, float * X, int items,
                int N, int n_cls, int n_reg, int D, cudaStream_t st);

}  // namespace jb
