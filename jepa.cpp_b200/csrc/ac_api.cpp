// V-JEPA 2-AC entry points of the C API (reference interface: include/jepa.h:375-523): introspection and
// the host utilities the API exposes -- the non-affine LayerNorm, the pose update, the L1 energy, the CEM
// defaults. Their arithmetic (double statistics, double rotations) is fixed by parity with the reference;
// the GPU rollout and the CEM live in ac_engine.cpp and cem.cu.
#include "model.h"
#include "stats.h"

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

// Non-affine LayerNorm of each row in place: double mean and variance, a float inverse standard deviation
// of (float) variance + eps, each value moved and scaled in float.
void jepa_ac_normalize(const jepa_model * m, float * rows, int64_t n_rows, int64_t dim) {
    if (!rows || n_rows <= 0 || dim <= 0) return;
    const float eps = is_ac(m) ? m->ac.norm_reps_eps : 1e-5f;
    for (int64_t r = 0; r < n_rows; r++) {
        float * v = rows + r * dim;
        double mean = 0.0, var = 0.0;
        jb::two_pass_moments(dim, [v](int64_t i) { return v[i]; }, mean, var);
        const float centre = (float) mean, scale = 1.0f / sqrtf((float) var + eps);
        for (int64_t i = 0; i < dim; i++) v[i] = (v[i] - centre) * scale;
    }
}

namespace {

// 3 x 3 rotations in double for the pose update. Euler angles (a, b, c) are extrinsic x-y-z: first about x
// by a, then about the fixed y by b, then the fixed z by c, i.e. R = Rz(c) Ry(b) Rx(a).
struct Rot3 {
    double m[3][3];

    static Rot3 about(int axis, double angle) {
        const double c = cos(angle), s = sin(angle);
        Rot3 r{};
        const int i = (axis + 1) % 3, j = (axis + 2) % 3;   // the plane the rotation turns
        r.m[axis][axis] = 1.0;
        r.m[i][i] = c;
        r.m[j][j] = c;
        r.m[i][j] = -s;
        r.m[j][i] = s;
        return r;
    }
    Rot3 operator*(const Rot3 & o) const {
        Rot3 r{};
        for (int i = 0; i < 3; i++)
            for (int j = 0; j < 3; j++) r.m[i][j] = m[i][0] * o.m[0][j] + m[i][1] * o.m[1][j] + m[i][2] * o.m[2][j];
        return r;
    }
    static Rot3 from_extrinsic_xyz(const float * e) { return about(2, e[2]) * (about(1, e[1]) * about(0, e[0])); }
    // back to extrinsic x-y-z angles; on the gimbal-lock circle (|sin b| = 1) the z angle is reported as 0
    void to_extrinsic_xyz(double & a, double & b, double & c) const {
        const double sb = std::fmax(-1.0, std::fmin(1.0, -m[2][0]));
        b = asin(sb);
        if (fabs(sb) < 1.0 - 1e-9) {
            a = atan2(m[2][1], m[2][2]);
            c = atan2(m[1][0], m[0][0]);
        } else {
            a = atan2(-m[1][2], m[1][1]);
            c = 0.0;
        }
    }
};

}  // namespace

// The pose after one action: position + translation; orientation = R(action) R(pose) re-expressed as
// extrinsic x-y-z angles; gripper + command kept within [0, 1]; lanes after the seventh carried over.
void jepa_ac_next_state(const jepa_model * m, const float * state, const float * action, float * out) {
    const int dim = m ? jepa_ac_state_dim(m) : 7;
    if (!state || !action || !out || dim < 7) {
        if (out && state && dim > 0) memcpy(out, state, (size_t) dim * sizeof(float));
        return;
    }
    const Rot3 turned = Rot3::from_extrinsic_xyz(action + 3) * Rot3::from_extrinsic_xyz(state + 3);
    double a, b, c;
    turned.to_extrinsic_xyz(a, b, c);
    for (int i = 0; i < 3; i++) out[i] = state[i] + action[i];
    out[3] = (float) a;
    out[4] = (float) b;
    out[5] = (float) c;
    const float grip = state[6] + action[6];
    out[6] = std::fmin(1.0f, std::fmax(0.0f, grip));
    for (int i = 7; i < dim; i++) out[i] = state[i];
}

// Mean absolute difference between each item's n_rows x dim prediction and the goal, summed in double.
void jepa_ac_energy(const float * pred, const float * goal, int n_batch, int64_t n_rows, int64_t dim, float * out) {
    if (!pred || !goal || !out || n_batch <= 0 || n_rows <= 0 || dim <= 0) return;
    const int64_t n = n_rows * dim;
    for (int item = 0; item < n_batch; item++) {
        const float * p = pred + (int64_t) item * n;
        double l1 = 0.0;
        for (int64_t i = 0; i < n; i++) l1 += std::fabs((double) p[i] - (double) goal[i]);
        out[item] = (float) (l1 / (double) n);
    }
}

// The ABI's CEM defaults (values fixed by the reference's interface: those of Meta's planner).
jepa_ac_cem_params jepa_ac_cem_default_params(void) {
    jepa_ac_cem_params p{};
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
    return p;   // seed 0
}

}  // extern "C"
