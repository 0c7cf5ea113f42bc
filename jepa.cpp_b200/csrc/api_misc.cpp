// Entry points of include/jepa.h that lie outside the planning engine: the image / video encoders,
// preprocessing, the attentive-pool head, the masked and LeWM predictors, and the H-JEPA single-shot
// graphs that jepa-plan calls before planning. They exist so that every binding of the reference API
// (which resolves every symbol at load time, reference: python/src/jepa_cpp/_api.py:413-418) loads
// against this library; each returns its failure value with the reason in jepa_error_text().
// The small stateless host helpers (jepa_free, jepa_softmax, jepa_top_k) are implemented.
#include "model.h"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <numeric>
#include <vector>

using jb::log;

namespace {
int unsupported(const char * fn) {
    log("jepa: %s: outside this engine (it runs the H-JEPA and V-JEPA 2-AC planners on the GPU)\n", fn);
    return -1;
}
template <class T> T * unsupported_ptr(const char * fn) { unsupported(fn); return nullptr; }
}  // namespace

extern "C" {

void jepa_free(void * p) { free(p); }

// probs = softmax(logits) (reference semantics: include/jepa.h:180-181)
void jepa_softmax(const float * logits, int n, float * probs) {
    if (!logits || !probs || n <= 0) return;
    float mx = logits[0];
    for (int i = 1; i < n; i++) mx = std::max(mx, logits[i]);
    double sum = 0;
    for (int i = 0; i < n; i++) { probs[i] = std::exp(logits[i] - mx); sum += probs[i]; }
    for (int i = 0; i < n; i++) probs[i] = (float) (probs[i] / sum);
}

// indices of the k largest logits, descending, ties by smaller index
int jepa_top_k(const float * logits, int n, int k, int32_t * idx) {
    if (!logits || !idx || n <= 0 || k <= 0) return 0;
    std::vector<int32_t> order((size_t) n);
    std::iota(order.begin(), order.end(), 0);
    k = std::min(k, n);
    std::partial_sort(order.begin(), order.begin() + k, order.end(), [&](int32_t a, int32_t b) {
        return logits[a] > logits[b] || (logits[a] == logits[b] && a < b);
    });
    std::copy(order.begin(), order.begin() + k, idx);
    return k;
}

jepa_preprocess_params jepa_preprocess_default_params(const jepa_model * model) {
    (void) model;
    jepa_preprocess_params p{};
    const float mean[3] = {0.485f, 0.456f, 0.406f}, std[3] = {0.229f, 0.224f, 0.225f};
    for (int i = 0; i < 3; i++) { p.mean[i] = mean[i]; p.std[i] = std[i]; }
    p.resize_short = 224;
    p.crop = 224;
    p.resample = JEPA_RESAMPLE_BILINEAR;
    p.resize_mode = JEPA_RESIZE_SHORTEST_EDGE;
    p.rescale = 1.0f / 255.0f;
    p.fused_norm = true;
    return p;
}

float * jepa_preprocess_image_file(const jepa_model *, const char *, int *, int *) { return unsupported_ptr<float>("jepa_preprocess_image_file"); }
float * jepa_preprocess_image_rgb(const jepa_model *, const uint8_t *, int, int, int *, int *) { return unsupported_ptr<float>("jepa_preprocess_image_rgb"); }
float * jepa_preprocess_frames_rgb(const jepa_model *, const uint8_t * const *, int, int, int, int *, int *) { return unsupported_ptr<float>("jepa_preprocess_frames_rgb"); }
float * jepa_preprocess_image_rgb_ex(const jepa_preprocess_params *, const uint8_t *, int, int, int *, int *) { return unsupported_ptr<float>("jepa_preprocess_image_rgb_ex"); }
float * jepa_preprocess_frames_rgb_ex(const jepa_preprocess_params *, const uint8_t * const *, int, int, int, int *, int *) { return unsupported_ptr<float>("jepa_preprocess_frames_rgb_ex"); }
uint8_t * jepa_load_image_rgb(const char *, int *, int *) { return unsupported_ptr<uint8_t>("jepa_load_image_rgb"); }
void jepa_resize_antialias_u8(const uint8_t *, int, int, int, uint8_t *, int, int, int) { unsupported("jepa_resize_antialias_u8"); }

int jepa_lewm_project(jepa_context *, const jepa_output *, jepa_output *) { return unsupported("jepa_lewm_project"); }
int jepa_lewm_project_rows(jepa_context *, const float *, int, jepa_output *) { return unsupported("jepa_lewm_project_rows"); }
int jepa_head(jepa_context *, const jepa_output *, jepa_output *) { return unsupported("jepa_head"); }
int jepa_predict(jepa_context *, const jepa_output *, const int32_t *, int, const int32_t *, int, jepa_output *) { return unsupported("jepa_predict"); }
int64_t jepa_token_grid(const jepa_model *, int, int, int, int *, int *, int *) { unsupported("jepa_token_grid"); return 0; }
int jepa_head_ex(jepa_context *, const jepa_output *, jepa_output *, jepa_output *) { return unsupported("jepa_head_ex"); }
int jepa_predict_ex(jepa_context *, const jepa_output *, const int32_t *, int, const int32_t *, int, int, jepa_output *) { return unsupported("jepa_predict_ex"); }
int jepa_predict_mod(jepa_context *, const jepa_output *, const int32_t *, int, const int32_t *, int, int, int, jepa_output *) { return unsupported("jepa_predict_mod"); }
int jepa_lewm_n_frames(const jepa_model *) { return 0; }
int jepa_lewm_action_dim(const jepa_model *) { return 0; }
int jepa_lewm_predict(jepa_context *, const float *, const float *, int, jepa_output *) { return unsupported("jepa_lewm_predict"); }
int jepa_lewm_rollout(jepa_context *, const float *, int, const float *, int, float *) { return unsupported("jepa_lewm_rollout"); }


}  // extern "C"
