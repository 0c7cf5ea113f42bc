// V-JEPA 2-AC rollout and CEM entry points. The GPU engine for them is the next item of the build;
// until it lands these return their failure value with the reason in jepa_error_text().
#include "model.h"

using jb::log;

namespace {
int not_yet(const char * fn) {
    log("jepa: %s: the V-JEPA 2-AC GPU engine is not built into this library yet\n", fn);
    return -1;
}
}  // namespace

extern "C" {

int jepa_ac_predict(jepa_context *, const float *, int, int, const float *, const float *, jepa_output *) { return not_yet("jepa_ac_predict"); }
int jepa_ac_predict_all(jepa_context *, const float *, int, int, const float *, const float *, jepa_output *) { return not_yet("jepa_ac_predict_all"); }
int jepa_ac_rollout(jepa_context *, const float *, int, const float *, const float *, const float *, int, int, float *) { return not_yet("jepa_ac_rollout"); }
int jepa_ac_rollout_ex(jepa_context *, const float *, int, const float *, const float *, const float *, const float *, int, int, float *) { return not_yet("jepa_ac_rollout_ex"); }
jepa_ac_context * jepa_ac_context_new(jepa_context *, const float *, int, const float *, const float *) { not_yet("jepa_ac_context_new"); return nullptr; }
void jepa_ac_context_free(jepa_ac_context *) {}
int jepa_ac_context_n_frames(const jepa_ac_context *) { return 0; }
int jepa_ac_context_capacity(const jepa_ac_context *) { return 0; }
int jepa_ac_context_update(jepa_ac_context *, const float *, const float *, const float *) { return not_yet("jepa_ac_context_update"); }
int jepa_ac_context_trim(jepa_ac_context *, int) { return not_yet("jepa_ac_context_trim"); }
int jepa_ac_rollout_cached(jepa_context *, jepa_ac_context *, const float *, const float *, int, int, float *) { return not_yet("jepa_ac_rollout_cached"); }
int jepa_ac_plan(jepa_context *, jepa_ac_context *, const float *, const jepa_ac_cem_params *, const float *, float *, float *) { return not_yet("jepa_ac_plan"); }

}  // extern "C"
