// Host-side policies of the H-JEPA gradient planner (see plan_policy.h).
#include "plan_policy.h"

#include <algorithm>
#include <cmath>

namespace jb {

constexpr int MAX_HORIZON = 65536;   // the reference's frame limit (JEPA_LIMIT_N_FRAMES)

float interpolated_quantile(const std::vector<float> & ascending, double q) {
    const int64_t n = (int64_t) ascending.size();
    const double at = q * (double) (n - 1);
    const int64_t below = (int64_t) std::floor(at);
    const int64_t above = std::min(below + 1, n - 1);
    const double frac = at - (double) below;
    const double a = ascending[(size_t) below], b = ascending[(size_t) above];
    return (float) (a + (b - a) * frac);
}

ActionPrior ActionPrior::from_recorded(const std::vector<float> & recorded, int lanes, float clip_sigma) {
    ActionPrior p;
    const int64_t rows = lanes > 0 ? (int64_t) recorded.size() / lanes : 0;
    p.centre.assign((size_t) lanes, 0.0f);
    p.spread.assign((size_t) lanes, 1.0f);
    auto lane_value = [&](int lane) { return [&, lane](int64_t r) { return recorded[(size_t) (r * lanes + lane)]; }; };
    for (int a = 0; rows > 0 && a < lanes; a++) {
        double mean = 0.0, var = 0.0;
        two_pass_moments(rows, lane_value(a), mean, var);
        p.centre[(size_t) a] = (float) mean;
        p.spread[(size_t) a] = std::max((float) std::sqrt(var), 1e-4f);
    }
    if (clip_sigma > 0.0f) {
        for (int a = 0; a < lanes; a++) {
            const float c = p.centre[(size_t) a], w = clip_sigma * p.spread[(size_t) a];
            p.lo.push_back(c - w);
            p.hi.push_back(c + w);
        }
        return p;
    }
    if (rows == 0) return p;
    std::vector<float> lane((size_t) rows);
    for (int a = 0; a < lanes; a++) {
        const auto get = lane_value(a);
        for (int64_t r = 0; r < rows; r++) lane[(size_t) r] = get(r);
        std::sort(lane.begin(), lane.end());
        p.lo.push_back(interpolated_quantile(lane, 0.02));
        p.hi.push_back(interpolated_quantile(lane, 0.98));
    }
    return p;
}

std::vector<float> ActionPrior::seed(int S, size_t row, float var_scale, DrawSource & draws) const {
    const size_t lanes = centre.size(), total = (size_t) S * row;
    std::vector<float> x(total);
    for (size_t i = 0; i < total; i++) x[i] = centre[i % lanes];
    if (S > 1) {
        // candidate 0 stays at the centre; the draws cover candidates 1..S-1, sample-major
        std::vector<float> z(total - row);
        draws.take(z.data(), z.size());
        float * moved = x.data() + row;
        for (size_t i = 0; i < z.size(); i++) moved[i] += (z[i] * spread[i % lanes]) * var_scale;
    }
    return x;
}

DrawSource::DrawSource(jepa_randn_fn hook, void * user, int level)
    : hook_(hook), user_(user), engine_(0x4a455041ull + (uint64_t) level) {}

void DrawSource::take(float * out, size_t n) {
    if (hook_) {
        hook_(user_, out, n);
        return;
    }
    for (size_t i = 0; i < n; i++) out[i] = unit_(engine_);
}

AdamTable::AdamTable(int n_iters, float lr) : pairs((size_t) 2 * std::max(1, n_iters)) {
    for (int k = 0; k < n_iters; k++) {
        const float t = (float) (k + 1);
        const float first = 1.0f - std::pow(0.9f, t), second = 1.0f - std::pow(0.999f, t);
        pairs[(size_t) 2 * k] = lr / first;
        pairs[(size_t) 2 * k + 1] = std::sqrt(second);
    }
}

bool Patience::stop_after(float lowest, int iter) {
    const bool better = !std::isfinite(best_) || best_ - lowest > rel_ * std::max(std::fabs(best_), 1e-12f);
    if (better) {
        best_ = lowest;
        flat_ = 0;
        return false;
    }
    flat_++;
    return flat_ >= patience_ && iter + 1 >= min_its_;
}

// ---- horizon schedule --------------------------------------------------------------------------
int shrink_at(int i, int n, int h) {
    if (h == 1) return 1;
    if (n == 1) return h;
    if (n < h) {
        // fewer positions than values: evenly spaced samples of h .. 1, rounded up
        const double v = 1.0 + (double) (h - 1) * (double) (n - 1 - i) / (double) (n - 1);
        return std::max(1, (int) std::ceil(v));
    }
    // every value h .. 1 held for n / h positions, the last n % h values one position longer
    const int run = n / h, longer = n % h, shorter_span = (h - longer) * run;
    const int step = i < shorter_span ? i / run : (h - longer) + (i - shorter_span) / (run + 1);
    return h - step;
}

std::vector<int> horizons_at(const std::vector<int> & horizon, const std::vector<int> & hold, int calls, int call) {
    const int n = (int) horizon.size();
    std::vector<int> out((size_t) n);
    int onset = 0;   // the call at which the current level starts to shrink (the top: the first call)
    for (int lv = n; lv >= 1; lv--) {
        const int h = horizon[(size_t) lv - 1], keep = hold[(size_t) lv - 1];
        auto at = [&](int c) { return c < onset ? keep : shrink_at(c - onset, calls - onset, h); };
        out[(size_t) lv - 1] = at(call);
        // the level below starts to shrink where this one first plans a single step
        int first_one = calls;
        for (int c = 0; c < calls; c++) {
            if (at(c) == 1) { first_one = c; break; }
        }
        onset = first_one;
    }
    return out;
}

// ---- argument rules ----------------------------------------------------------------------------
int states_seen_by_goal(const HPlanner & pm, const CostSpec & cs) {
    // the goal's level keeps every stride-th prediction of the level below it, from the context state on
    int seen = cs.horizon;
    for (int lv = cs.level + 1; lv <= cs.goal_level; lv++) seen /= cs.dense ? 1 : pm.levels[(size_t) lv - 1].hp.stride;
    return seen;
}

namespace {

struct RuleInput {
    const HPlanner & pm;
    const CostSpec & cs;
    int n_levels;
};

bool action_encoder_complete(const HPlanner & pm, const CostSpec & cs) {
    const DLevel & L = pm.levels[(size_t) cs.level - 1];
    const DLevel & U = pm.levels[(size_t) cs.level];
    const DActEnc & ae = U.ae;
    const int width_in = L.act0 ? L.E : L.A, stride = U.hp.stride;
    if (ae.kind == 1) {
        return ae.fc1 && ae.fc2 && ae.fc1.in == stride * width_in && ae.fc2.in == ae.fc1.out && ae.fc2.out == U.A;
    }
    if (ae.kind != 2) return false;
    const int d = ae.d;
    bool ok = d > 0 && ae.n_head > 0 && d % ae.n_head == 0 && ae.step && ae.step.in == width_in && ae.step.out == d &&
              ae.pos && ae.pos_n >= (int64_t) (stride + 1) * d && !ae.blocks.empty() && ae.head0 && ae.head0.in == d &&
              ae.head2 && ae.head2.in == ae.head0.out && ae.head2.out == U.A;
    for (const DSeqBlock & B : ae.blocks) {
        ok = ok && B.qkv.in == d && B.qkv.out == 3 * d && B.out.in == d && B.out.out == d && B.up.in == d &&
             B.down.in == B.up.out && B.down.out == d && B.ln1_w && B.ln2_w;
    }
    return ok;
}

struct Rule {
    bool (*broken)(const RuleInput &);
    void (*explain)(const RuleInput &, const char * fn);
};

// in order: a rule may assume that the rules before it hold
const Rule GOAL_RULES[] = {
    {[](const RuleInput & r) { return r.cs.level < 1 || r.cs.level > r.n_levels; },
     [](const RuleInput & r, const char * fn) {
         log("jepa: %s: no level %d to plan (this model has %d)\n", fn, r.cs.level, r.n_levels);
     }},
    {[](const RuleInput & r) { return r.cs.goal_level < r.cs.level || r.cs.goal_level > r.n_levels; },
     [](const RuleInput & r, const char * fn) {
         log("jepa: %s: a goal at level %d cannot score level %d (goals live at the planned level or above, up to %d)\n",
             fn, r.cs.goal_level, r.cs.level, r.n_levels);
     }},
    {[](const RuleInput & r) { return r.cs.horizon < 1 || r.cs.horizon > MAX_HORIZON; },
     [](const RuleInput & r, const char * fn) {
         log("jepa: %s: horizon %d outside 1..%d\n", fn, r.cs.horizon, MAX_HORIZON);
     }},
    {[](const RuleInput & r) { return !r.cs.s0 || !r.cs.goal || r.cs.n_goal < 1; },
     [](const RuleInput &, const char * fn) { log("jepa: %s: a start state and at least one goal state are needed\n", fn); }},
    {[](const RuleInput & r) { return r.cs.dense && r.cs.goal_level == r.cs.level; },
     [](const RuleInput &, const char * fn) {
         log("jepa: %s: dense goal projection only applies to goals above the planned level\n", fn);
     }},
    {[](const RuleInput & r) { return states_seen_by_goal(r.pm, r.cs) < 1; },
     [](const RuleInput & r, const char * fn) {
         log("jepa: %s: level %d's %d-step horizon is shorter than one step of level %d\n", fn, r.cs.level, r.cs.horizon,
             r.cs.goal_level);
     }},
    {[](const RuleInput & r) {
         const int window = std::min(std::max(1, r.cs.cost_last_n), states_seen_by_goal(r.pm, r.cs));
         return r.cs.n_goal != 1 && r.cs.n_goal != window;
     },
     [](const RuleInput & r, const char * fn) {
         const int window = std::min(std::max(1, r.cs.cost_last_n), states_seen_by_goal(r.pm, r.cs));
         log("jepa: %s: %d goal states given, %d predictions are scored (horizon %d, cost_last_n %d); pass 1 goal or %d\n",
             fn, r.cs.n_goal, window, r.cs.horizon, r.cs.cost_last_n, window);
     }},
    {[](const RuleInput & r) { return r.pm.pooled_chunks(r.cs) > 0 && !action_encoder_complete(r.pm, r.cs); },
     [](const RuleInput & r, const char * fn) {
         log("jepa: %s: the action cost pools actions through level %d's action encoder, which is missing or incomplete "
             "(jepa.hjepa.act_enc_kind mlp or seq, with its weights)\n", fn, r.cs.level + 1);
     }},
};

}  // namespace

bool goal_rules_hold(const HPlanner & pm, const CostSpec & cs, const char * fn) {
    const RuleInput in{pm, cs, (int) pm.levels.size()};
    for (const Rule & rule : GOAL_RULES) {
        if (rule.broken(in)) {
            rule.explain(in, fn);
            return false;
        }
    }
    return true;
}

CostSpec cost_spec_of(int level, int horizon, const float * state, const jepa_hjepa_goal * goal,
                      const jepa_hjepa_level_plan * lp) {
    CostSpec cs;
    cs.level = level;
    cs.horizon = horizon;
    cs.s0 = state;
    cs.goal_level = level;
    if (goal) {
        cs.goal = goal->states;
        cs.n_goal = goal->n_states;
        if (goal->level > 0) cs.goal_level = goal->level;
        cs.dense = goal->dense != 0;
        cs.goal_action = goal->actions;
    }
    if (lp) {
        cs.cost_last_n = lp->cost_last_n;
        cs.intermediate_cost_weight = lp->intermediate_cost_weight;
        cs.action_cost_weight = lp->action_cost_weight;
    }
    return cs;
}

}  // namespace jb
