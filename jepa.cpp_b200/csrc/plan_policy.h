// Host-side policies of the H-JEPA gradient planner: everything that decides WHICH numbers the GPU
// sweep sees, but does no per-candidate arithmetic itself.
//
//   ActionPrior   where candidates start and the box they are kept in, from a level's recorded
//                 latent actions (reference behaviour: src/hjepa-plan.cpp:845-884)
//   DrawSource    the normal draws that perturb candidates (caller hook, else a seeded engine)
//   AdamTable     per-iteration AdamW step sizes, bias corrections computed on the host in float
//   Patience      early stopping on the best cost seen before each update
//   horizon_at    the receding-horizon schedule of every level (reference: :1042-1059, :1121-1162)
//   GoalRules     the argument rules a cost specification has to satisfy (reference: :974-1010)
//
// The arithmetic of each piece is fixed by parity with the reference (float vs double, the order of
// the reductions, interpolation between order statistics); the structure is this engine's own.
#pragma once

#include "hplan.h"
#include "stats.h"

#include <cstdint>
#include <random>
#include <string>
#include <vector>

namespace jb {

// ---- statistics --------------------------------------------------------------------------------
// The q-quantile of ascending values by linear interpolation between the two order statistics that
// bracket position q (n - 1), computed in double and rounded once to float.
float interpolated_quantile(const std::vector<float> & ascending, double q);

// ---- action prior ------------------------------------------------------------------------------
struct ActionPrior {
    std::vector<float> centre, spread;   // per action lane
    std::vector<float> lo, hi;           // per lane; empty when candidates are not boxed
    bool boxed() const { return !lo.empty(); }

    // From `rows` recorded actions of `lanes` values each (row-major; none recorded: centre 0, spread 1).
    // The spread is the population standard deviation, at least 1e-4. The box is centre +- clip_sigma
    // spread when clip_sigma > 0, otherwise the 2 % / 98 % quantiles of the recordings when there are
    // any, otherwise none.
    static ActionPrior from_recorded(const std::vector<float> & recorded, int lanes, float clip_sigma);

    // S candidates of `row` values (T steps of `lanes` lanes): every one at the centre, all but the first
    // moved by (z * spread) * var_scale with z from `draws`, drawn sample-major for candidates 1..S-1.
    std::vector<float> seed(int S, size_t row, float var_scale, class DrawSource & draws) const;
};

// ---- draws -------------------------------------------------------------------------------------
// N(0, 1) draws: the caller's jepa_randn_fn when there is one, else std::mt19937_64 seeded
// 0x4a455041 + level feeding std::normal_distribution<float> -- the reference's generator, so that
// default runs of the two planners perturb candidates identically.
class DrawSource {
  public:
    DrawSource(jepa_randn_fn hook, void * user, int level);
    void take(float * out, size_t n);

  private:
    jepa_randn_fn hook_;
    void * user_;
    std::mt19937_64 engine_;
    std::normal_distribution<float> unit_{0.0f, 1.0f};
};

// ---- optimiser ---------------------------------------------------------------------------------
// AdamW with beta1 0.9, beta2 0.999: iteration k's step size lr / (1 - 0.9^(k+1)) and the square root of
// the second-moment correction 1 - 0.999^(k+1), each in float as the host computes them.
struct AdamTable {
    std::vector<float> pairs;            // [n][2]: step size, sqrt(second-moment correction)
    AdamTable(int n_iters, float lr);
};

// Stops after `patience` iterations in a row that did not lower the best cost by more than
// rel_delta * |best| (and not before min_its iterations); the cost judged is the lowest over the
// candidates before the iteration's update.
class Patience {
  public:
    Patience(int patience, int min_its, float rel_delta) : patience_(patience), min_its_(min_its), rel_(rel_delta) {}
    bool active() const { return patience_ > 0; }
    // the lowest cost seen at iteration `iter` (0-based); true = stop after this iteration
    bool stop_after(float lowest, int iter);

  private:
    int patience_, min_its_;
    float rel_;
    float best_ = INFINITY;
    int flat_ = 0;
};

// ---- horizon schedule --------------------------------------------------------------------------
// Horizons of every level (1..n) at call `call` of `calls` replanning calls. The top level shrinks from
// its horizon to 1 over all calls; each level below keeps its pre-decay horizon (or, when that is 0,
// the stride of the level above) until the call at which the level above first reaches horizon 1, and
// from there shrinks from its own horizon to 1 over the calls that remain.
std::vector<int> horizons_at(const std::vector<int> & horizon, const std::vector<int> & hold, int calls, int call);
// value at position i of a shrink from h to 1 over n positions
int shrink_at(int i, int n, int h);

// ---- argument rules ----------------------------------------------------------------------------
// Checks a cost specification against the planner's levels; logs the first rule broken, naming `fn`.
bool goal_rules_hold(const HPlanner & pm, const CostSpec & cs, const char * fn);
// Predictions of level cs.level that the goal's level sees (strides of the levels in between divide
// the horizon; a dense projection keeps every one).
int states_seen_by_goal(const HPlanner & pm, const CostSpec & cs);
// A cost specification from the C API's goal and plan structs (fields left at their defaults when absent).
CostSpec cost_spec_of(int level, int horizon, const float * state, const jepa_hjepa_goal * goal,
                      const jepa_hjepa_level_plan * lp);

}  // namespace jb
