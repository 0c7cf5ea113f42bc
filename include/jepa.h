// jepa-b200 -- the jepa.cpp C API, served by a B200-native planner engine.
//
// This header is the drop-in boundary: it declares exactly the functions and types of jepa.cpp's
// public header (reference: include/jepa.h, 114 functions), with the same signatures, struct layouts
// and return conventions, so that jepa-plan, jepa-worldmodel and the Python binding (which binds every
// one of these names at import, reference: python/src/jepa_cpp/_api.py:413-418) link against this
// library unchanged. Planner entry points run on the GPU; the encoder / preprocessing entry points,
// which lie outside the planning engine, are present and fail with a message.
//
// Conventions (as in the reference): opaque handles; caller-owned output buffers; int 0 = success,
// -1 = failure (or NULL), with the reason on stderr and in jepa_error_text(); NULL arguments are
// defined (an error or a no-op); no exception crosses this boundary.
#pragma once
#include <stddef.h>
#include <stdint.h>
#include <stdbool.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)   // every declaration below is exported
#endif

typedef struct jepa_model   jepa_model;
typedef struct jepa_context jepa_context;

enum { JEPA_KV_AUTO = 0, JEPA_KV_F16 = 1, JEPA_KV_F32 = 2 };

typedef struct {
    int   n_threads;      // host threads (0 = all); the planner itself runs on the GPU
    bool  use_flash_attn;
    bool  verbose;
    int   flash_kv;       // JEPA_KV_*
} jepa_context_params;

typedef struct {          // NCTHW float32 input of the encoders
    const float * data;
    int n_batch, n_chans, n_frames, height, width;
} jepa_input;

typedef struct {          // malloc'd result rows; free data with jepa_free
    float * data;
    int64_t n_tokens;
    int64_t dim;
} jepa_output;

enum { JEPA_RESAMPLE_BILINEAR = 0, JEPA_RESAMPLE_BICUBIC = 1 };
enum { JEPA_RESIZE_SHORTEST_EDGE = 0, JEPA_RESIZE_SQUASH = 1 };

typedef struct {
    float mean[3];
    float std[3];
    int   resize_short;
    int   crop;
    int   resample;
    int   resize_mode;
    float rescale;
    bool  fused_norm;
} jepa_preprocess_params;

enum { JEPA_MODALITY_AUTO = 0, JEPA_MODALITY_VIDEO = 1, JEPA_MODALITY_IMAGE = 2 };

#define JEPA_HJEPA_MAX_PLAN_LEVELS 8

// One level's solver and cost settings; field order and meaning as the reference (include/jepa.h:286-310).
typedef struct jepa_hjepa_level_plan {
    int   horizon;                 // planning horizon of this call, in the level's own steps
    int   pre_decay_horizon;       // jepa_hjepa_horizons only (0 = the stride of the level above)
    int   n_samples;               // candidates optimised together
    int   n_steps;                 // gradient iterations at most
    float lr, weight_decay;        // AdamW (betas 0.9 / 0.999, eps 1e-8)
    float var_scale;               // initial perturbation, in units of the action prior's std
    float action_noise;            // std of the noise added after each step (0 = none)
    float action_clip_sigma;       // > 0: clip to mean +- sigma * std; 0: the recorded 2..98 % range
    int   min_its;                 // iterations before early stopping may trigger
    int   early_stop_patience;     // 0 = never stop early
    float early_stop_rel_delta;
    int   cost_last_n;             // how many of the last predicted states are scored
    float intermediate_cost_weight;
    float action_cost_weight;      // pooled-action cost against the upper level's macro-actions (0 = off)
    int   num_subgoals;            // of this level's predicted states, how many the level below must reach
    int   horizon_one_goal_upper;
} jepa_hjepa_level_plan;

// Standard-normal draws, consumed in the reference's order.
typedef void (*jepa_randn_fn)(void * user, float * out, size_t n);

typedef struct jepa_hjepa_goal {
    const float * states;          // [n_states, embed_dim(level)]
    int           n_states;
    int           level;           // 0 = the planned level
    int           dense;
    const float * actions;         // [n_states, action_dim(level + 1)] or NULL
} jepa_hjepa_goal;

typedef struct jepa_hjepa_plan_info {   // sizeof == 128
    int   planned[JEPA_HJEPA_MAX_PLAN_LEVELS];
    int   goal_level[JEPA_HJEPA_MAX_PLAN_LEVELS];
    int   iters[JEPA_HJEPA_MAX_PLAN_LEVELS];
    float cost[JEPA_HJEPA_MAX_PLAN_LEVELS];
} jepa_hjepa_plan_info;

typedef struct jepa_ac_context jepa_ac_context;

typedef struct {
    int   samples;                 // candidates per iteration (K)
    int   topk;                    // elites kept per iteration
    int   cem_steps;               // iterations
    int   horizon;                 // H
    float maxnorm;                 // translation clamp and initial translation std
    float gripper_clamp;
    float momentum_mean, momentum_std;
    float momentum_mean_gripper, momentum_std_gripper;
    float round_gripper;
    uint32_t seed;                 // used only when noise is NULL
} jepa_ac_cem_params;

typedef struct {
    bool verbose;
    int  device;                   // CUDA device; -1 = CUDA device 0 (no CPU path here)
} jepa_model_params;

// Lifecycle and threading. A model is immutable once loaded; a context is used by one thread at a time
// (reference contract: include/jepa.h:612-647). In this engine a context owns one GPU's planner state.
jepa_context_params jepa_context_default_params(void);
jepa_model * jepa_model_load(const char * gguf_path, bool verbose);
void jepa_model_free(jepa_model * model);
jepa_context * jepa_context_new(jepa_model * model, jepa_context_params params);
void jepa_context_free(jepa_context * ctx);
int jepa_context_n_threads(const jepa_context * ctx);
double jepa_context_last_compute_ms(const jepa_context * ctx);

// Introspection (reference: include/jepa.h:45-68).
const char * jepa_model_family(const jepa_model * model);
const char * jepa_model_name(const jepa_model * model);
int jepa_model_embed_dim(const jepa_model * model);
int jepa_model_patch_size(const jepa_model * model);
int jepa_model_tubelet_size(const jepa_model * model);
int jepa_model_img_size(const jepa_model * model);
int jepa_model_n_frames(const jepa_model * model);
int jepa_model_n_layer(const jepa_model * model);
int jepa_model_n_head(const jepa_model * model);
bool jepa_model_has_cls(const jepa_model * model);
int jepa_model_n_registers(const jepa_model * model);
int jepa_model_n_prefix_tokens(const jepa_model * model);
bool jepa_model_has_predictor(const jepa_model * model);
bool jepa_model_has_head(const jepa_model * model);
bool jepa_model_has_projector(const jepa_model * model);
int jepa_model_n_classes(const jepa_model * model);
const char * jepa_model_label(const jepa_model * model, int idx);
int jepa_model_file_type(const jepa_model * model);
const char * jepa_model_file_type_name(const jepa_model * model);
size_t jepa_model_n_bytes(const jepa_model * model);

// Preprocessing and image input: outside the planner engine. The symbols exist so that every binding of
// the reference API loads; they return NULL / no-ops (reference: include/jepa.h:70-107).
jepa_preprocess_params jepa_preprocess_default_params(const jepa_model * model);
float * jepa_preprocess_image_file(const jepa_model * model, const char * path, int * out_h, int * out_w);
float * jepa_preprocess_image_rgb(const jepa_model * model, const uint8_t * rgb, int h, int w, int * out_h, int * out_w);
float * jepa_preprocess_frames_rgb(const jepa_model * model, const uint8_t * const * frames, int n_frames, int h, int w, int * out_h, int * out_w);
float * jepa_preprocess_image_rgb_ex(const jepa_preprocess_params * p, const uint8_t * rgb, int h, int w, int * out_h, int * out_w);
float * jepa_preprocess_frames_rgb_ex(const jepa_preprocess_params * p, const uint8_t * const * frames, int n_frames, int h, int w, int * out_h, int * out_w);
uint8_t * jepa_load_image_rgb(const char * path, int * h, int * w);
void jepa_resize_antialias_u8(const uint8_t * src, int h, int w, int c, uint8_t * dst, int out_h, int out_w, int resample);
void jepa_free(void * p);

// Encoders, heads and the masked / LeWM predictors: outside the planner engine, present for ABI
// completeness; they return -1 with a message in jepa_error_text() (reference: include/jepa.h:109-230).
int jepa_encode(jepa_context * ctx, const jepa_input * in, jepa_output * out);
int jepa_pool_mean(const jepa_model * model, const jepa_output * enc, jepa_output * out);
int jepa_pool_cls(const jepa_model * model, const jepa_output * enc, jepa_output * out);
int jepa_lewm_project(jepa_context * ctx, const jepa_output * enc, jepa_output * out);
int jepa_lewm_project_rows(jepa_context * ctx, const float * cls_rows, int n_rows, jepa_output * out);
int jepa_head(jepa_context * ctx, const jepa_output * enc, jepa_output * out);
int jepa_predict(jepa_context * ctx, const jepa_output * enc, const int32_t * context_idx, int n_context, const int32_t * target_idx, int n_target, jepa_output * out);
int64_t jepa_token_grid(const jepa_model * model, int n_frames, int height, int width, int * gt, int * gh, int * gw);
int jepa_head_ex(jepa_context * ctx, const jepa_output * enc, jepa_output * pooled, jepa_output * logits);
void jepa_softmax(const float * logits, int n, float * probs);
int jepa_top_k(const float * logits, int n, int k, int32_t * idx);
const char * jepa_version(void);
void jepa_print_system_info(void);
int jepa_predict_ex(jepa_context * ctx, const jepa_output * enc, const int32_t * context_idx, int n_context, const int32_t * target_idx, int n_target, int mask_index, jepa_output * out);
int jepa_predict_mod(jepa_context * ctx, const jepa_output * enc, const int32_t * context_idx, int n_context, const int32_t * target_idx, int n_target, int mask_index, int modality, jepa_output * out);
int jepa_lewm_n_frames(const jepa_model * model);
int jepa_lewm_action_dim(const jepa_model * model);
int jepa_lewm_predict(jepa_context * ctx, const float * embs, const float * actions, int n_frames, jepa_output * out);
int jepa_lewm_rollout(jepa_context * ctx, const float * embs, int n_seed, const float * actions, int n_steps, float * out);

// H-JEPA hierarchy introspection and single-shot graphs (reference: include/jepa.h:232-287).
int jepa_hjepa_n_levels(const jepa_model * model);
int jepa_hjepa_embed_dim(const jepa_model * model, int level);
int jepa_hjepa_action_dim(const jepa_model * model, int level);
int jepa_hjepa_action_embed_dim(const jepa_model * model, int level);
int jepa_hjepa_stride(const jepa_model * model, int level);
int jepa_hjepa_n_frames(const jepa_model * model, int level);
int jepa_hjepa_proprio_dim(const jepa_model * model);
int jepa_hjepa_raw_action_dim(const jepa_model * model);
int jepa_hjepa_frameskip(const jepa_model * model);
int jepa_hjepa_norm_stats(const jepa_model * model, const char * column, float * mean, float * std, int capacity);
int jepa_hjepa_action_prior(const jepa_model * model, int level, float * out, int capacity);
int jepa_hjepa_embed(jepa_context * ctx, const float * cls_rows, const float * proprio, int n_rows, jepa_output * out);
int jepa_hjepa_lift(jepa_context * ctx, int level, const float * below, int n_rows, jepa_output * out);
int jepa_hjepa_action_embed(jepa_context * ctx, int level, const float * actions, int n_rows, jepa_output * out);
int jepa_hjepa_action_encode(jepa_context * ctx, int level, const float * below_act_emb, int n_rows, jepa_output * out);
int jepa_hjepa_predict(jepa_context * ctx, int level, const float * states, const float * actions, int n_frames, jepa_output * out);
int jepa_hjepa_rollout(jepa_context * ctx, int level, const float * states, int n_seed, const float * actions, int n_steps, int history, float * out);

// H-JEPA top-down gradient planner -- the GPU hot path of this engine (reference: include/jepa.h:289-373,
// src/hjepa-plan.cpp:1066-1256). Same arguments, same error behaviour (0 / -1 + jepa_error_text()).
jepa_hjepa_level_plan jepa_hjepa_level_plan_default(void);
int jepa_hjepa_plan_cost(jepa_context * ctx, int level, const float * state, const jepa_hjepa_goal * goal, const jepa_hjepa_level_plan * plan, const float * actions, int n_samples, int horizon, float * costs, float * grad);
int jepa_hjepa_solve(jepa_context * ctx, int level, const float * state, const jepa_hjepa_goal * goal, const jepa_hjepa_level_plan * plan, jepa_randn_fn randn, void * randn_user, float * actions, float * states, float * cost, int * iters);
int jepa_hjepa_horizons(const jepa_model * model, const jepa_hjepa_level_plan * levels, int n_levels, int replanning_interval, int eval_budget, int steps_taken, int * horizons);
int jepa_hjepa_plan(jepa_context * ctx, const float * const * states, const float * const * goals, const jepa_hjepa_level_plan * levels, int n_levels, jepa_randn_fn randn, void * randn_user, float * actions, jepa_hjepa_plan_info * info);

// V-JEPA 2-AC world model and CEM planner (reference: include/jepa.h:375-523, src/vjepa2_ac.cpp).
int jepa_ac_tokens_per_frame(const jepa_model * model);
int jepa_ac_action_dim(const jepa_model * model);
int jepa_ac_state_dim(const jepa_model * model);
int jepa_ac_max_frames(const jepa_model * model);
bool jepa_ac_normalize_reps(const jepa_model * model);
void jepa_ac_normalize(const jepa_model * model, float * rows, int64_t n_rows, int64_t dim);
int jepa_ac_predict(jepa_context * ctx, const float * context, int n_frames, int n_batch, const float * actions, const float * states, jepa_output * out);
int jepa_ac_predict_all(jepa_context * ctx, const float * context, int n_frames, int n_batch, const float * actions, const float * states, jepa_output * out);
int jepa_ac_rollout(jepa_context * ctx, const float * context, int n_seed, const float * seed_states, const float * actions, const float * states, int n_cand, int horizon, float * out);
int jepa_ac_rollout_ex(jepa_context * ctx, const float * context, int n_seed, const float * seed_actions, const float * seed_states, const float * actions, const float * states, int n_cand, int horizon, float * out);
jepa_ac_context * jepa_ac_context_new(jepa_context * ctx, const float * latents, int n_frames, const float * actions, const float * states);
void jepa_ac_context_free(jepa_ac_context * handle);
int jepa_ac_context_n_frames(const jepa_ac_context * handle);
int jepa_ac_context_capacity(const jepa_ac_context * handle);
int jepa_ac_context_update(jepa_ac_context * handle, const float * latents, const float * action, const float * state);
int jepa_ac_context_trim(jepa_ac_context * handle, int n_keep);
int jepa_ac_rollout_cached(jepa_context * ctx, jepa_ac_context * handle, const float * actions, const float * states, int n_cand, int horizon, float * out);
jepa_ac_cem_params jepa_ac_cem_default_params(void);
int jepa_ac_plan(jepa_context * ctx, jepa_ac_context * handle, const float * goal, const jepa_ac_cem_params * params, const float * noise, float * out_actions, float * out_energy);
void jepa_ac_next_state(const jepa_model * model, const float * state, const float * action, float * out);
void jepa_ac_energy(const float * pred, const float * goal, int n_batch, int64_t n_rows, int64_t dim, float * out);

// Encoder batching knobs (reference: include/jepa.h:525-545); kept for ABI completeness.
void jepa_context_set_max_batch(jepa_context * ctx, int n);
int jepa_context_max_batch(const jepa_context * ctx);
int jepa_context_last_batch(const jepa_context * ctx);

// Devices. Device n is CUDA device n; -1 (the reference's CPU) selects CUDA device 0, because this engine
// has no CPU path (reference: include/jepa.h:547-596).
jepa_model_params jepa_model_default_params(void);
jepa_model * jepa_model_load_ex(const char * gguf_path, const jepa_model_params * params);
int jepa_device_count(void);
const char * jepa_device_name(int device);
const char * jepa_device_description(int device);
void jepa_device_memory(int device, size_t * free_bytes, size_t * total_bytes);
int jepa_model_device(const jepa_model * model);
const char * jepa_model_device_name(const jepa_model * model);
bool jepa_model_is_gpu(const jepa_model * model);
void jepa_context_set_mul_mat_prec_f32(jepa_context * ctx, bool on);
bool jepa_context_mul_mat_prec_f32(const jepa_context * ctx);

// Diagnostics capture: every message is written to stderr and to a thread-local buffer
// (reference: include/jepa.h:597-611).
void jepa_error_reset(void);
const char * jepa_error_text(void);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif
