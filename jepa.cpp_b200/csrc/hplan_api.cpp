// The H-JEPA planner entry points of the C API (reference interface: include/jepa.h:289-373) and the
// level solve that drives the GPU sweep.
//
// A level's solve keeps everything per candidate on the device: the candidates, the AdamW moments, the
// clamp box, the iteration counter and the per-iteration step sizes. One CUDA graph -- forward, cost,
// backward and the AdamW update of every candidate chain -- is captured once and replayed per iteration,
// so the host only launches graphs (and, with early stopping, reads the lowest cost back). The host-side
// choices (prior, draws, step sizes, stopping, schedule, argument rules) live in plan_policy.*; the
// hierarchy that hands each level's plan down as the next level's goals is the Cascade below.
#include "hplan.h"
#include "plan_policy.h"
#include "shard.h"

#include "../../include/jepa_b200.h"

#include <algorithm>
#include <cmath>
#include <cstring>

namespace jb {

// the context's planner, built on first use (weights on the device)
HPlanner * hplanner_of(jepa_context * ctx, const char * fn) {
    if (!ctx->model->hj.present) {
        log("jepa: %s: '%s' is not an H-JEPA model (jepa.family = '%s')\n", fn, ctx->model->name.c_str(), ctx->model->family.c_str());
        return nullptr;
    }
    if (!ctx->hplan) {
        cudaSetDevice(ctx->device);
        auto p = std::make_unique<HPlanner>();
        p->ctx = ctx;
        if (!p->build(*ctx->model)) {
            log("jepa: %s: could not place the planner's weights on CUDA device %d\n", fn, ctx->device);
            return nullptr;
        }
        ctx->hplan = std::move(p);
    }
    cudaSetDevice(ctx->device);
    if (device_flags_clear(ctx->stream)) return nullptr;
    return ctx->hplan.get();
}

// ---------------------------------------------------------------------------------------------
// one level's solve
// ---------------------------------------------------------------------------------------------
namespace {

// The rank's candidates [r0, r1) of S, split into nc chains of consecutive rows.
struct Slice {
    int r0 = 0, r1 = 0, nc = 1;
    std::vector<int> edge;   // chain c holds local rows [edge[c], edge[c + 1])
    int rows() const { return r1 - r0; }
    int chain_of(int local) const {
        int c = 0;
        while (c + 1 < nc && local >= edge[(size_t) c + 1]) c++;
        return c;
    }
};

}  // namespace

int HPlanner::solve(const CostSpec & cs, const jepa_hjepa_level_plan & lp, DrawSource & draws, SolveOut & out) {
    cudaStream_t st = ctx->stream;
    const DLevel & L = levels[(size_t) cs.level - 1];
    const int A = L.A, T = cs.horizon, S = std::max(1, lp.n_samples), D = L.D;
    const size_t row = (size_t) T * A;
    const ActionPrior prior = ActionPrior::from_recorded(L.queue, A, lp.action_clip_sigma);
    Shard * sh = ctx->shard.get();
    const bool sharded = sh && sh->world > 1;
    const int world = sharded ? sh->world : 1, rank = sharded ? sh->rank : 0;

    // every rank draws the whole stream, so that its candidates are the ones a single GPU would have
    const std::vector<float> x0 = prior.seed(S, row, lp.var_scale, draws);
    out.iters = 0;
    Slice sl;
    sl.r0 = (int) ((int64_t) S * rank / world);
    sl.r1 = (int) ((int64_t) S * (rank + 1) / world);
    if (sl.rows() < 1) { log("jepa: hjepa solve: rank %d of %d has no candidates (%d in all)\n", rank, world, S); return -1; }
    sl.nc = streams_for(sl.rows(), L.P);
    sl.edge.resize((size_t) sl.nc + 1);
    for (int c = 0; c <= sl.nc; c++) sl.edge[(size_t) c] = (int) ((int64_t) sl.rows() * c / sl.nc);
    std::vector<Workspace *> chain((size_t) sl.nc);
    std::string gens;
    for (int c = 0; c < sl.nc; c++) {
        chain[(size_t) c] = workspace(cs.level, sl.edge[(size_t) c + 1] - sl.edge[(size_t) c], T, cs, c, sl.nc);
        if (!chain[(size_t) c] || !cost_tables(*chain[(size_t) c], cs)) return -1;
        gens += std::to_string(chain[(size_t) c]->gen) + ",";
    }
    Workspace * w0 = chain[0];
    launches = 0;
    cudaEvent_t t_begin, t_end;
    cudaEventCreate(&t_begin);
    cudaEventCreate(&t_end);
    cudaEventRecord(t_begin, st);

    // device state of every chain: candidates, zeroed moments, counters, the start state, the clamp box
    for (int c = 0; c < sl.nc; c++) {
        Workspace * w = chain[(size_t) c];
        const size_t first = (size_t) sl.r0 + (size_t) sl.edge[(size_t) c];
        const size_t n = (size_t) w->S * row;
        JB_CUDA(cudaMemcpyAsync(w->x, x0.data() + first * row, n * 4, cudaMemcpyHostToDevice, st));
        JB_CUDA(cudaMemsetAsync(w->m, 0, n * 4, st));
        JB_CUDA(cudaMemsetAsync(w->v, 0, n * 4, st));
        JB_CUDA(cudaMemsetAsync(w->step_ctr, 0, 4 * sizeof(int), st));
        if (w->fix_count) JB_CUDA(cudaMemsetAsync(w->fix_count, 0, w->fix_counters * sizeof(int), st));
        JB_CUDA(cudaMemcpyAsync(w->gtmp, cs.s0, (size_t) D * 4, cudaMemcpyHostToDevice, st));
        copy_rows(w->gtmp, 0, w->states, D, w->S, D, st);
        gather_actions(w->x, w->a_all, w->S, T, A, st);
        launches += 2;
        if (prior.boxed()) {
            JB_CUDA(cudaMemcpyAsync(w->lo, prior.lo.data(), (size_t) A * 4, cudaMemcpyHostToDevice, st));
            JB_CUDA(cudaMemcpyAsync(w->hi, prior.hi.data(), (size_t) A * 4, cudaMemcpyHostToDevice, st));
        }
    }
    const AdamTable adam(lp.n_steps, lp.lr);
    Patience patience(lp.early_stop_patience, lp.min_its, lp.early_stop_rel_delta);

    // Per-iteration action noise. With a fixed iteration count every iteration's draws are taken up front
    // (one slot per iteration, the rank's rows of each); with early stopping the count is not known, so
    // one slot is refilled before each iteration.
    const bool noisy = lp.action_noise > 0.0f;
    const size_t slot = (size_t) sl.rows() * row;
    std::vector<float> zbuf;
    float * zdev = nullptr;
    if (noisy) {
        const size_t slots = patience.active() ? 1 : (size_t) std::max(1, lp.n_steps);
        if (!cuda_ok(cudaMalloc(&zdev, slots * slot * 4), "noise buffer")) return -1;
        if (!patience.active()) {
            zbuf.resize((size_t) S * row);
            for (int k = 0; k < lp.n_steps; k++) {
                draws.take(zbuf.data(), zbuf.size());
                if (!cuda_ok(cudaMemcpy(zdev + (size_t) k * slot, zbuf.data() + (size_t) sl.r0 * row, slot * 4, cudaMemcpyHostToDevice),
                             "noise upload")) {
                    cudaFree(zdev);
                    return -1;
                }
            }
        }
    }
    const size_t zstride = (noisy && !patience.active()) ? slot : 0;
    constexpr int TABLE_ROWS = 4096;   // step sizes held on the device at a time

    // one graph over every chain: chain c on its own stream, forked from and joined into the context's
    auto capture = [&](bool with_grad, cudaGraphExec_t * exec, long long * nodes) -> int {
        cudaGraph_t g;
        JB_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        const long long before = launches;
        bool ok = sl.nc == 1 || cuda_ok(cudaEventRecord(ev[0], st), "fork");
        for (int c = 1; c < sl.nc && ok; c++) ok = cuda_ok(cudaStreamWaitEvent(chain[(size_t) c]->st, ev[0], 0), "fork");
        for (int c = 0; c < sl.nc && ok; c++) {
            Workspace * w = chain[(size_t) c];
            ok = forward(*w, cs, with_grad) == 0 && (!with_grad || backward(*w, cs) == 0);
            if (ok && with_grad) {
                adam_step(w->x, w->m, w->v, w->da_all, w->a_all, w->sched, w->step_ctr, lp.lr * lp.weight_decay,
                          zdev ? zdev + (size_t) sl.edge[(size_t) c] * row : nullptr, lp.action_noise, zstride,
                          prior.boxed() ? w->lo : nullptr, prior.boxed() ? w->hi : nullptr, w->S, T, A, w->st);
                launches++;
            }
        }
        for (int c = 1; c < sl.nc && ok; c++) {
            ok = cuda_ok(cudaEventRecord(ev[(size_t) c], chain[(size_t) c]->st), "join") &&
                 cuda_ok(cudaStreamWaitEvent(st, ev[(size_t) c], 0), "join");
        }
        const cudaError_t end = cudaStreamEndCapture(st, &g);
        if (!ok || end != cudaSuccess) { cudaGetLastError(); log("jepa: hjepa solve: capturing the iteration graph failed\n"); return -1; }
        *nodes = launches - before;
        const cudaError_t inst = cudaGraphInstantiate(exec, g, 0);
        cudaGraphDestroy(g);
        return cuda_ok(inst, "cudaGraphInstantiate") ? 0 : -1;
    };
    // lowest cost over the rank's chains, first one on ties (chains are in row order): value, local row
    auto lowest = [&](float & value, int & local) -> int {
        std::vector<float> v((size_t) sl.nc);
        std::vector<int> at((size_t) sl.nc);
        for (int c = 0; c < sl.nc; c++) {
            Workspace * w = chain[(size_t) c];
            argmin_first(w->cost, w->S, w->best_idx, w->best_val, st);
            launches++;
            JB_CUDA(cudaMemcpyAsync(&v[(size_t) c], w->best_val, 4, cudaMemcpyDeviceToHost, st));
            JB_CUDA(cudaMemcpyAsync(&at[(size_t) c], w->best_idx, 4, cudaMemcpyDeviceToHost, st));
        }
        JB_CUDA(cudaStreamSynchronize(st));
        int b = 0;
        for (int c = 1; c < sl.nc; c++) if (v[(size_t) c] < v[(size_t) b]) b = c;
        value = v[(size_t) b];
        local = sl.edge[(size_t) b] + at[(size_t) b];
        return 0;
    };
    auto iterate = [&]() -> int {
        const std::string key = std::to_string(lp.lr * lp.weight_decay) + "/" + std::to_string(lp.action_noise) + "/" +
                                std::to_string(prior.boxed()) + "/" + std::to_string((uintptr_t) zdev) + "/" +
                                std::to_string(zstride) + "/" + gens;
        if (!w0->g_iter || w0->iter_key != key) {
            if (w0->g_iter) { cudaGraphExecDestroy(w0->g_iter); w0->g_iter = nullptr; }
            if (capture(true, &w0->g_iter, &w0->iter_nodes)) return -1;
            w0->iter_key = key;
        }
        launches = 0;
        for (int k = 0; k < lp.n_steps; k++) {
            if (k % TABLE_ROWS == 0) {
                if (k > 0 && zstride) {
                    log("jepa: hjepa solve: action noise drawn up front covers at most %d iterations\n", TABLE_ROWS);
                    return -1;
                }
                const int n = std::min(TABLE_ROWS, lp.n_steps - k);
                for (Workspace * w : chain) {
                    JB_CUDA(cudaMemcpyAsync(w->sched, adam.pairs.data() + (size_t) 2 * k, (size_t) 2 * n * 4, cudaMemcpyHostToDevice, st));
                    JB_CUDA(cudaMemsetAsync(w->step_ctr, 0, 2 * sizeof(int), st));
                }
            }
            if (noisy && patience.active()) {
                zbuf.resize((size_t) S * row);
                draws.take(zbuf.data(), zbuf.size());
                JB_CUDA(cudaMemcpyAsync(zdev, zbuf.data() + (size_t) sl.r0 * row, slot * 4, cudaMemcpyHostToDevice, st));
            }
            JB_CUDA(cudaGraphLaunch(w0->g_iter, st));
            launches += w0->iter_nodes;
            out.iters = k + 1;
            if (patience.active()) {
                // the costs this iteration's gradient was taken at, i.e. before its update
                float low = 0.0f;
                int at = 0;
                if (lowest(low, at)) return -1;
                if (sharded && !sh->min_f32(low, &low, st)) return -1;
                if (patience.stop_after(low, k)) break;
            }
        }
        // a final evaluation without gradient picks the plan
        if (!w0->g_fwd || w0->fwd_key != gens) {
            if (w0->g_fwd) { cudaGraphExecDestroy(w0->g_fwd); w0->g_fwd = nullptr; }
            if (capture(false, &w0->g_fwd, &w0->fwd_nodes)) return -1;
            w0->fwd_key = gens;
        }
        JB_CUDA(cudaGraphLaunch(w0->g_fwd, st));
        launches += w0->fwd_nodes;
        float cost = 0.0f;
        int local = 0;
        if (lowest(cost, local)) return -1;
        int owner = rank;
        if (sharded) {
            // every rank's (cost, global row): the lowest cost wins, the lower row on ties
            int global = sl.r0 + local;
            if (!sh->argmin_global(cost, global, &cost, &global, &owner, st)) return -1;
            local = global - sl.r0;
        }
        out.actions.assign(row, 0.0f);
        out.states.assign((size_t) (T + 1) * D, 0.0f);
        if (owner == rank) {
            const int c = sl.chain_of(local);
            const Workspace * w = chain[(size_t) c];
            const int r = local - sl.edge[(size_t) c];
            JB_CUDA(cudaMemcpyAsync(out.actions.data(), w->x + (size_t) r * row, row * 4, cudaMemcpyDeviceToHost, st));
            JB_CUDA(cudaMemcpy2DAsync(out.states.data(), (size_t) D * 4, w->states + (size_t) r * D, (size_t) w->S * D * 4,
                                      (size_t) D * 4, (size_t) T + 1, cudaMemcpyDeviceToHost, st));
            JB_CUDA(cudaStreamSynchronize(st));
        }
        if (sharded && (!sh->bcast_host(out.actions.data(), row, owner, st) ||
                        !sh->bcast_host(out.states.data(), out.states.size(), owner, st))) {
            return -1;
        }
        out.cost = cost;
        return 0;
    };
    int rc = iterate();
    if (zdev) cudaFree(zdev);
    cudaEventRecord(t_end, st);
    cudaEventSynchronize(t_end);
    float ms = 0;
    cudaEventElapsedTime(&ms, t_begin, t_end);
    cudaEventDestroy(t_begin);
    cudaEventDestroy(t_end);
    ctx->last_ms += ms;
    ctx->last_launches += launches;
    if (rc == 0 && gemm_error_flag(st)) { log("jepa: a tensor-core kernel gave up waiting on its pipeline\n"); rc = -1; }
    return rc;
}

// ---------------------------------------------------------------------------------------------
// the hierarchy: levels planned from the top down
// ---------------------------------------------------------------------------------------------
namespace {

// Walks the levels from the top. A planned level hands the level below it its predicted states (after
// the current one) as subgoals and its actions as goal actions; a level above the first that plans a
// single step is skipped, and then the level below aims at the real goal -- in the skipped level's space
// when that level asks for it (horizon_one_goal_upper), else in its own.
class Cascade {
  public:
    Cascade(HPlanner & pm, const float * const * states, const float * const * goals, const jepa_hjepa_level_plan * plans,
            int n_levels, jepa_randn_fn randn, void * user)
        : pm_(pm), states_(states), goals_(goals), plans_(plans), n_(n_levels), randn_(randn), user_(user) {}

    int run(float * actions, jepa_hjepa_plan_info * info) {
        for (int lv = n_; lv >= 1; lv--) {
            const jepa_hjepa_level_plan & lp = plans_[lv - 1];
            if (lv > 1 && lp.horizon == 1) {
                skip(lv, lp);
                continue;
            }
            CostSpec cs;
            bool aims_at_goal = false;
            if (!target(lv, lp, cs, aims_at_goal) || !goal_rules_hold(pm_, cs, "jepa_hjepa_plan")) return -1;
            DrawSource draws(randn_, user_, lv);
            SolveOut result;
            if (pm_.solve(cs, lp, draws, result)) return -1;
            if (info && lv <= JEPA_HJEPA_MAX_PLAN_LEVELS) {
                info->planned[lv - 1] = 1;
                info->cost[lv - 1] = result.cost;
                info->iters[lv - 1] = result.iters;
                info->goal_level[lv - 1] = cs.goal_level;
            }
            above_ = std::move(result);
            have_above_ = true;
            above_aims_at_goal_ = aims_at_goal;
            skipped_space_ = 0;
        }
        // level 1 always plans
        memcpy(actions, above_.actions.data(), above_.actions.size() * sizeof(float));
        return 0;
    }

  private:
    void skip(int lv, const jepa_hjepa_level_plan & lp) {
        // the highest skipped level keeps the goal space when asked to; a level that does not ask resets it
        if (!lp.horizon_one_goal_upper) skipped_space_ = 0;
        else if (!skipped_space_) skipped_space_ = lv;
        have_above_ = false;
    }

    bool target(int lv, const jepa_hjepa_level_plan & lp, CostSpec & cs, bool & aims_at_goal) {
        cs.level = lv;
        cs.horizon = lp.horizon;
        cs.s0 = states_[lv - 1];
        cs.cost_last_n = lp.cost_last_n;
        cs.intermediate_cost_weight = lp.intermediate_cost_weight;
        cs.action_cost_weight = lp.action_cost_weight;
        if (!have_above_) {
            // no plan above: the real goal, in the space of the skipped level that asked for it or in this one
            cs.goal_level = skipped_space_ ? skipped_space_ : lv;
            cs.goal = goals_[cs.goal_level - 1];
            cs.n_goal = 1;
            cs.dense = cs.goal_level > lv;
            aims_at_goal = true;
            return true;
        }
        const DLevel & up = pm_.levels[(size_t) lv];
        const int width = up.D, lanes = up.A;
        const int predicted = (int) above_.states.size() / width - 1;   // the plan's states after its current one
        const int wanted = plans_[lv].num_subgoals;
        const int n_sub = std::min(wanted, predicted);
        subgoals_.assign(above_.states.begin() + width, above_.states.begin() + (std::ptrdiff_t) (1 + n_sub) * width);
        subgoal_actions_.assign(above_.actions.begin(), above_.actions.begin() + (std::ptrdiff_t) n_sub * lanes);
        // when the subgoals run to the end of a plan that itself aimed at the real goal, the last one is
        // replaced by that goal
        aims_at_goal = wanted >= predicted && above_aims_at_goal_;
        if (aims_at_goal) memcpy(subgoals_.data() + (size_t) (n_sub - 1) * width, goals_[lv], (size_t) width * sizeof(float));
        cs.goal_level = lv + 1;
        cs.goal = subgoals_.data();
        cs.n_goal = n_sub;
        cs.goal_action = subgoal_actions_.data();
        if (n_sub > 1) {
            const int reach = (lp.horizon + up.hp.stride) / up.hp.stride - 1;   // level-(lv+1) states the horizon spans
            if (n_sub != reach) {
                log("jepa: jepa_hjepa_plan: level %d gets %d subgoals, but its horizon %d spans %d states of level %d (stride %d)\n",
                    lv, n_sub, lp.horizon, reach, lv + 1, up.hp.stride);
                return false;
            }
        }
        return true;
    }

    HPlanner & pm_;
    const float * const * states_;
    const float * const * goals_;
    const jepa_hjepa_level_plan * plans_;
    const int n_;
    jepa_randn_fn randn_;
    void * user_;
    SolveOut above_;                 // the plan of the last level planned
    bool have_above_ = false;
    bool above_aims_at_goal_ = true;
    int skipped_space_ = 0;          // goal space chosen by a skipped level (0 = none)
    std::vector<float> subgoals_, subgoal_actions_;
};

}  // namespace
}  // namespace jb

// =============================================================================================
// C API
// =============================================================================================
using namespace jb;

extern "C" {

int jepa_b200_hjepa_set_streams(jepa_context * ctx, int n) {
    if (!ctx || n < 0 || n > 8) { log("jepa: jepa_b200_hjepa_set_streams: a context and 0..8 streams are required\n"); return -1; }
    HPlanner * pm = hplanner_of(ctx, "jepa_b200_hjepa_set_streams");
    if (!pm) return -1;
    pm->n_streams = n;
    return 0;
}

int jepa_b200_hjepa_set_step_modulation(jepa_context * ctx, int mode) {
    if (!ctx || mode < 0 || mode > 2) { log("jepa: jepa_b200_hjepa_set_step_modulation: a context and mode 0, 1 or 2 are required\n"); return -1; }
    HPlanner * pm = hplanner_of(ctx, "jepa_b200_hjepa_set_step_modulation");
    if (!pm) return -1;
    if (pm->force_mod_mode != mode) pm->ws.clear();   // workspaces are planned for one mode
    pm->force_mod_mode = mode;
    return 0;
}

// The ABI's defaults for one level's plan (values fixed by the reference's interface).
jepa_hjepa_level_plan jepa_hjepa_level_plan_default(void) {
    jepa_hjepa_level_plan p{};
    p.horizon = 1;
    p.n_samples = 100;
    p.n_steps = 90;
    p.lr = 0.1f;
    p.weight_decay = 0.01f;
    p.var_scale = 1.0f;
    p.min_its = 30;
    p.early_stop_patience = 5;
    p.early_stop_rel_delta = 1e-2f;
    p.cost_last_n = 1;
    p.intermediate_cost_weight = 1.0f;
    p.num_subgoals = 1;
    return p;   // pre_decay_horizon, action_noise, action_clip_sigma, action_cost_weight, horizon_one_goal_upper: 0
}

int jepa_hjepa_plan_cost(jepa_context * ctx, int level, const float * state, const jepa_hjepa_goal * goal,
                         const jepa_hjepa_level_plan * plan, const float * actions, int n_samples, int horizon,
                         float * costs, float * grad) {
    if (!ctx || !state || !goal || !actions || !costs || n_samples < 1) return -1;
    HPlanner * pm = hplanner_of(ctx, "jepa_hjepa_plan_cost");
    if (!pm) return -1;
    const CostSpec cs = cost_spec_of(level, horizon, state, goal, plan);
    if (!goal_rules_hold(*pm, cs, "jepa_hjepa_plan_cost")) return -1;
    return pm->plan_cost(cs, actions, n_samples, costs, grad);
}

int jepa_hjepa_solve(jepa_context * ctx, int level, const float * state, const jepa_hjepa_goal * goal,
                     const jepa_hjepa_level_plan * plan, jepa_randn_fn randn, void * randn_user, float * actions,
                     float * states, float * cost, int * iters) {
    if (!ctx || !state || !goal || !plan || !actions) return -1;
    HPlanner * pm = hplanner_of(ctx, "jepa_hjepa_solve");
    if (!pm) return -1;
    const CostSpec cs = cost_spec_of(level, plan->horizon, state, goal, plan);
    if (!goal_rules_hold(*pm, cs, "jepa_hjepa_solve")) return -1;
    if (plan->n_samples < 1 || plan->n_steps < 0) {
        log("jepa: jepa_hjepa_solve: need n_samples >= 1 and n_steps >= 0 (got %d, %d)\n", plan->n_samples, plan->n_steps);
        return -1;
    }
    DrawSource draws(randn, randn_user, level);
    SolveOut r;
    ctx->last_ms = 0;
    ctx->last_launches = 0;
    if (pm->solve(cs, *plan, draws, r)) return -1;
    memcpy(actions, r.actions.data(), r.actions.size() * sizeof(float));
    if (states) memcpy(states, r.states.data(), r.states.size() * sizeof(float));
    if (cost) *cost = r.cost;
    if (iters) *iters = r.iters;
    return 0;
}

int jepa_hjepa_horizons(const jepa_model * model, const jepa_hjepa_level_plan * levels, int n_levels,
                        int replanning_interval, int eval_budget, int steps_taken, int * horizons) {
    if (!model || !levels || !horizons || !model->hj.present) return -1;
    const int n = (int) model->hj.levels.size();
    if (n_levels != n || replanning_interval < 1 || eval_budget < 1 || steps_taken < 0) {
        log("jepa: jepa_hjepa_horizons: expected %d level plans, replanning_interval >= 1, eval_budget >= 1, steps_taken >= 0\n", n);
        return -1;
    }
    const int calls = (eval_budget + replanning_interval - 1) / replanning_interval;
    const int call = steps_taken / replanning_interval;
    if (call >= calls) {
        log("jepa: jepa_hjepa_horizons: step %d falls after the last replanning call of a %d-step budget\n", steps_taken, eval_budget);
        return -1;
    }
    std::vector<int> horizon((size_t) n), hold((size_t) n);
    for (int lv = n; lv >= 1; lv--) {
        const jepa_hjepa_level_plan & lp = levels[lv - 1];
        if (lp.horizon < 1) {
            log("jepa: jepa_hjepa_horizons: level %d's horizon %d is not positive\n", lv, lp.horizon);
            return -1;
        }
        horizon[(size_t) lv - 1] = lp.horizon;
        hold[(size_t) lv - 1] = lv < n ? (lp.pre_decay_horizon > 0 ? lp.pre_decay_horizon : model->hj.levels[(size_t) lv].stride) : 0;
    }
    const std::vector<int> h = horizons_at(horizon, hold, calls, call);
    std::copy(h.begin(), h.end(), horizons);
    return 0;
}

int jepa_hjepa_plan(jepa_context * ctx, const float * const * states, const float * const * goals,
                    const jepa_hjepa_level_plan * levels, int n_levels, jepa_randn_fn randn, void * randn_user,
                    float * actions, jepa_hjepa_plan_info * info) {
    if (!ctx || !states || !goals || !levels || !actions) return -1;
    HPlanner * pm = hplanner_of(ctx, "jepa_hjepa_plan");
    if (!pm) return -1;
    if (n_levels != (int) pm->levels.size()) {
        log("jepa: jepa_hjepa_plan: the model has %zu levels, %d plans were given\n", pm->levels.size(), n_levels);
        return -1;
    }
    for (int lv = 1; lv <= n_levels; lv++) {
        const jepa_hjepa_level_plan & lp = levels[lv - 1];
        if (!states[lv - 1] || !goals[lv - 1]) {
            log("jepa: jepa_hjepa_plan: level %d needs its current state and its goal\n", lv);
            return -1;
        }
        if (lp.n_samples < 1 || lp.n_steps < 0 || lp.num_subgoals < 1) {
            log("jepa: jepa_hjepa_plan: level %d needs n_samples >= 1, n_steps >= 0, num_subgoals >= 1 (got %d, %d, %d)\n", lv,
                lp.n_samples, lp.n_steps, lp.num_subgoals);
            return -1;
        }
    }
    if (info) *info = jepa_hjepa_plan_info{};
    ctx->last_ms = 0;
    ctx->last_launches = 0;
    Cascade cascade(*pm, states, goals, levels, n_levels, randn, randn_user);
    return cascade.run(actions, info);
}

}  // extern "C"
