// The engine's jepa_model / jepa_context: GGUF metadata parsed into the hyper-parameters the planners
// need, the file's tensors kept in host memory (uploaded and dequantised lazily by the planners), and the
// per-context GPU state.
#pragma once

#include "gguf.h"
#include "common.h"
#include "../../include/jepa.h"

#include <memory>
#include <string>
#include <vector>

namespace jb {

// one level of an H-JEPA hierarchy (the jepa.hjepa.* arrays; reference: src/jepa-internal.h:237-248)
struct HLevel {
    int embed_dim = 0, stride = 1, window = 1, target_length = 0, action_dim = 0, act_embed_dim = 0;
    std::string enc_kind, act_enc_kind, pred_kind;
    int act_enc_dim = 0, act_enc_n_layer = 0, act_enc_n_head = 0, act_enc_max_chunk = 0;
    int pred_dim = 0, pred_n_layer = 0, pred_n_head = 0, pred_head_dim = 0, pred_ffn_dim = 0, pred_n_frames = 0;
};

struct HParams {
    bool present = false;
    float ln_eps = 1e-5f, adaln_eps = 1e-6f;
    std::string proj_kind;
    int pixel_dim = 0, proprio_dim = 0, raw_action_dim = 0, frameskip = 0;
    std::vector<HLevel> levels;
};

// V-JEPA 2-AC predictor metadata (jepa.pred.*; reference: src/jepa-gguf.cpp:454-480)
struct ACParams {
    bool present = false;
    int embed_dim = 0, n_layer = 0, n_head = 0, ffn_dim = 0, head_dim = 0;
    int action_dim = 0, state_dim = 0, n_cond_tokens = 0, grid_size = 0, n_frames = 0;
    bool normalize_reps = false;
    float norm_reps_eps = 1e-5f, ln_eps = 1e-6f;
    bool frame_causal = false;          // block-causal mask over frames (jepa.pred.frame_causal)
    bool rope_interleaved = false;      // jepa.pred.rope_freq_layout == "interleaved" (else tiled)
    float rope_theta = 10000.0f;        // jepa.enc.rope_theta
    int out_dim = 0;                    // jepa.pred.out_dim (defaults to the encoder width)
    std::string act = "gelu_erf";       // jepa.pred.act
};

struct EncParams {
    int embed_dim = 0, n_layer = 0, n_head = 0, ffn_dim = 0, patch_size = 16, tubelet_size = 1, img_size = 224;
    int n_frames = 1, n_registers = 0, in_chans = 3;
    bool cls_token = false;
    float ln_eps = 1e-6f;               // jepa.enc.ln_eps
    std::string act = "gelu_erf";       // jepa.enc.act
    // video encoders (V-JEPA 2 / 2.1, LeVJEPA): 3-D RoPE on q / k, optional modality vectors, the 2.1 image
    // tokenizer, block-causal attention across temporal slots
    float rope_theta = 10000.0f;        // jepa.enc.rope_theta
    bool rope_interleaved = false;      // jepa.enc.rope_freq_layout == "interleaved" (else tiled)
    bool rope_interpolate = false;      // jepa.enc.rope_interpolate: positions rescaled to rope_ref_grid
    int rope_ref_grid = 0;              // jepa.enc.rope_ref_grid
    bool modality_embed = false;        // jepa.enc.modality_embed
    bool image_patch_embed = false;     // jepa.enc.image_patch_embed
    bool block_causal = false;          // jepa.enc.attn_mode == "block_causal"
};

}  // namespace jb

struct jepa_model {
    std::string path;
    std::unique_ptr<jb::gguf_file> file;
    std::string name, family, modality;
    uint32_t file_type = 0;
    jb::EncParams enc;
    jb::HParams hj;
    jb::ACParams ac;
    std::string pred_kind;       // jepa.pred.kind ("" = none)
    int device = 0;
    size_t n_bytes = 0;
    std::string device_name;

    const jb::gguf_tensor * get(const std::string & name) const { return file->tensor(name); }
};

namespace jb { struct HPlanner; struct Shard; struct ACEngine; }

namespace jb { struct EncEngine; }

struct jepa_context {
    jepa_model * model = nullptr;
    jepa_context_params params{};
    int n_threads = 1;
    int device = 0;
    cudaStream_t stream = nullptr;
    std::unique_ptr<jb::HPlanner> hplan;
    std::unique_ptr<jb::Shard> shard;
    std::unique_ptr<jb::ACEngine> ac;
    std::unique_ptr<jb::EncEngine> enc;   // the image encoder's weights on the device (jepa_encode), on first use
    double last_ms = 0.0;
    long long last_launches = 0;
    int max_batch = 32;
    bool prec_f32 = true;
    ~jepa_context();
};

namespace jb {
// load-time validation of the tensors the H-JEPA planner reads (reference: src/hjepa.cpp:96-241)
bool hjepa_bind(const jepa_model & m);
}
