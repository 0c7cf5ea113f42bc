// V-JEPA 2-AC entry points of the C API: introspection and the host utilities the reference exposes
// (the non-affine LayerNorm, the pose update, the L1 energy, the CEM defaults), with the reference's
// semantics (src/vjepa2_ac.cpp:161-263, :787-802). The GPU rollout and CEM live in ac_engine.cpp.
#include "model.h"

#include <cmath>
#include <cstring>

using jb::log;

namespace {
bool is_ac(const jepa_model * m) { return m && m->ac.present; }
}  // namespace

extern "C" {

int jepa_ac_tokens_per_frame(const jepa_model * m) { return is_ac(m) ? m->ac.grid_size * m->ac.grid_size : 0; }
int jepa_ac_action_dim(const jepa_model * m) { return is_ac(m) ? m->ac.action_dim : 0; }
int jepa_ac_state_dim(const jepa_model * m) { return is_ac(m) ? m->ac.state_dim : 0; }
int jepa_ac_max_frames(const jepa_model * m) { return is_ac(m) ? m->ac.n_frames : 0; }
bool jepa_ac_normalize_reps(const jepa_model * m) { return is_ac(m) && m->ac.normalize_reps; }

// non-affine LayerNorm per row: double mean / variance, float inverse std of (float) var + eps
void jepa_ac_normalize(const jepa_model * m, float * rows, int64_t n_rows, int64_t dim) {
    if (!rows || n_rows <= 0 || dim <= 0) return;
    const float eps = is_ac(m) ? m->ac.norm_reps_eps : 1e-5f;
    for (int64_t r = 0; r < n_rows; r++) {
        float * v = rows + r * dim;
        double mu = 0;
        for (int64_t i = 0; i < dim; i++) mu += v[i];
        mu /= (double) dim;
        double var = 0;
        for (int64_t i = 0; i < dim; i++) { const double d = v[i] - mu; var += d * d; }
        var /= (double) dim;
        const float inv = 1.0f / sqrtf((float) var + eps);
        const float muf = (float) mu;
        for (int64_t i = 0; i < dim; i++) v[i] = (float) ((v[i] - muf) * inv);
    }
}

// Pose update: translation added; rotation = R(action) R(pose) with extrinsic-xyz Euler angles
// (R = Rz(c) Ry(b) Rx(a)), decomposed back (b = asin(-R20), a = atan2(R21, R22), c = atan2(R10, R00),
// c = 0 at gimbal lock); gripper added and clipped to [0, 1].
void jepa_ac_next_state(const jepa_model * m, const float * state, const float * action, float * out) {
    const int dim = m ? jepa_ac_state_dim(m) : 7;
    if (!state || !action || !out || dim < 7) {
        if (out && state && dim > 0) memcpy(out, state, (size_t) dim * sizeof(float));
        return;
    }
    auto rot = [](const float * e, double R[3][3]) {
        // double-precision cos / sin of the float angles (the explicit casts keep the float overloads out)
        const double a = e[0], b = e[1], c = e[2];
        const double ca = cos(a), sa = sin(a), cb = cos(b), sb = sin(b), cc = cos(c), sc = sin(c);
        R[0][0] = cb * cc; R[0][1] = sa * sb * cc - ca * sc; R[0][2] = ca * sb * cc + sa * sc;
        R[1][0] = cb * sc; R[1][1] = sa * sb * sc + ca * cc; R[1][2] = ca * sb * sc - sa * cc;
        R[2][0] = -sb;     R[2][1] = sa * cb;                R[2][2] = ca * cb;
    };
    double P[3][3], Dm[3][3], R[3][3];
    rot(state + 3, P);
    rot(action + 3, Dm);
    for (int i = 0; i < 3; i++)
        for (int j = 0; j < 3; j++) R[i][j] = Dm[i][0] * P[0][j] + Dm[i][1] * P[1][j] + Dm[i][2] * P[2][j];
    const double s = std::fmax(-1.0, std::fmin(1.0, -R[2][0]));
    const double beta = asin(s);
    double alpha, gamma;
    if (fabs(s) < 1.0 - 1e-9) {
        alpha = atan2(R[2][1], R[2][2]);
        gamma = atan2(R[1][0], R[0][0]);
    } else {
        alpha = atan2(-R[1][2], R[1][1]);
        gamma = 0.0;
    }
    for (int i = 0; i < 3; i++) out[i] = state[i] + action[i];
    out[3] = (float) alpha;
    out[4] = (float) beta;
    out[5] = (float) gamma;
    float g = state[6] + action[6];
    out[6] = g < 0.0f ? 0.0f : (g > 1.0f ? 1.0f : g);
    for (int i = 7; i < dim; i++) out[i] = state[i];
}

// mean |pred - goal| over all rows and dims of each item, double accumulation
void jepa_ac_energy(const float * pred, const float * goal, int n_batch, int64_t n_rows, int64_t dim, float * out) {
    if (!pred || !goal || !out || n_batch <= 0 || n_rows <= 0 || dim <= 0) return;
    const int64_t per = n_rows * dim;
    for (int b = 0; b < n_batch; b++) {
        const float * a = pred + (int64_t) b * per;
        double acc = 0;
        for (int64_t i = 0; i < per; i++) acc += std::fabs((double) a[i] - (double) goal[i]);
        out[b] = (float) (acc / (double) per);
    }
}

jepa_ac_cem_params jepa_ac_cem_default_params(void) {
    jepa_ac_cem_params p;
    p.samples = 100;
    p.topk = 10;
    p.cem_steps = 100;
    p.horizon = 1;
    p.maxnorm = 0.05f;
    p.gripper_clamp = 0.75f;
    p.momentum_mean = 0.25f;
    p.momentum_std = 0.95f;
    p.momentum_mean_gripper = 0.15f;
    p.momentum_std_gripper = 0.15f;
    p.round_gripper = 0.25f;
    p.seed = 0;
    return p;
}

}  // extern "C"
