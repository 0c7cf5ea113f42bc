// The H-JEPA planner entry points of the C API (reference: include/jepa.h:289-373,
// src/hjepa-plan.cpp:840-1256): argument checks and messages, the action prior, the noise source, the
// AdamW solve loop around the GPU sweep, the horizon schedule and the top-down hierarchy.
//
// Host-side semantics follow the reference step for step (they decide which numbers the GPU sees):
//   * candidates start at the prior mean, all but the first perturbed by noise drawn sample-major,
//     from the caller's jepa_randn_fn or from std::mt19937_64 + std::normal_distribution<float> seeded
//     0x4a455041 + level, the reference's own generator;
//   * AdamW with the bias corrections computed on the host in float as powf(beta, step + 1);
//   * early stopping on the minimum cost of the candidates BEFORE the update of that iteration;
//   * the lowest cost candidate (first one on ties) after a final evaluation without gradient.
#include "hplan.h"
#include "shard.h"

#include "../../include/jepa_b200.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <random>

namespace jb {

struct NoiseSource {
    jepa_randn_fn fn = nullptr;
    void * user = nullptr;
    std::mt19937_64 rng;
    std::normal_distribution<float> dist{0.0f, 1.0f};
    void fill(float * out, size_t n) {
        if (fn) { fn(user, out, n); return; }
        for (size_t i = 0; i < n; i++) out[i] = dist(rng);
    }
};

namespace {

constexpr int LIMIT_N_FRAMES = 65536;

struct Prior { std::vector<float> mean, std, lo, hi; };

// the action prior of a level (reference semantics: src/hjepa-plan.cpp:845-884)
Prior prior_of(const DLevel & L, float clip_sigma) {
    Prior p;
    const int A = L.A;
    const int64_t n = (int64_t) L.queue.size() / A;
    p.mean.assign((size_t) A, 0.0f);
    p.std.assign((size_t) A, 1.0f);
    if (n > 0) {
        for (int a = 0; a < A; a++) {
            double mu = 0, var = 0;
            for (int64_t i = 0; i < n; i++) mu += L.queue[(size_t) (i * A + a)];
            mu /= (double) n;
            for (int64_t i = 0; i < n; i++) { const double c = L.queue[(size_t) (i * A + a)] - mu; var += c * c; }
            p.mean[(size_t) a] = (float) mu;
            p.std[(size_t) a] = std::max((float) std::sqrt(var / (double) n), 1e-4f);
        }
    }
    if (clip_sigma > 0.0f) {
        for (int a = 0; a < A; a++) {
            p.lo.push_back(p.mean[(size_t) a] - clip_sigma * p.std[(size_t) a]);
            p.hi.push_back(p.mean[(size_t) a] + clip_sigma * p.std[(size_t) a]);
        }
    } else if (n > 0) {
        std::vector<float> col((size_t) n);
        for (int a = 0; a < A; a++) {
            for (int64_t i = 0; i < n; i++) col[(size_t) i] = L.queue[(size_t) (i * A + a)];
            std::sort(col.begin(), col.end());
            auto q = [&](double f) {
                const double pos = f * (double) (n - 1);
                const int64_t i0 = (int64_t) std::floor(pos), i1 = std::min(i0 + 1, n - 1);
                const double fr = pos - (double) i0;
                return (float) ((double) col[(size_t) i0] + ((double) col[(size_t) i1] - (double) col[(size_t) i0]) * fr);
            };
            p.lo.push_back(q(0.02));
            p.hi.push_back(q(0.98));
        }
    }
    return p;
}

int scored_states(const HPlanner & pm, const CostSpec & cs) {
    int len = cs.horizon + 1;
    for (int lv = cs.level + 1; lv <= cs.goal_level; lv++) {
        const int stride = cs.dense ? 1 : pm.levels[(size_t) lv - 1].hp.stride;
        len = (len - 1) / stride + 1;
    }
    return len - 1;
}

bool check_spec(const HPlanner & pm, const CostSpec & cs, const char * fn) {
    const int n_levels = (int) pm.levels.size();
    if (cs.level < 1 || cs.level > n_levels) {
        log("jepa: %s: level %d is out of range, the model has levels 1..%d\n", fn, cs.level, n_levels);
        return false;
    }
    if (cs.goal_level < cs.level || cs.goal_level > n_levels) {
        log("jepa: %s: the goal's level %d has to be in %d..%d (the planned level up to the top)\n", fn, cs.goal_level, cs.level, n_levels);
        return false;
    }
    if (cs.horizon < 1 || cs.horizon > LIMIT_N_FRAMES) {
        log("jepa: %s: horizon %d is out of range [1, %d]\n", fn, cs.horizon, LIMIT_N_FRAMES);
        return false;
    }
    if (!cs.s0 || !cs.goal || cs.n_goal < 1) {
        log("jepa: %s: the current state and at least one goal state are required\n", fn);
        return false;
    }
    if (cs.dense && cs.goal_level == cs.level) {
        log("jepa: %s: a dense goal projection needs a goal above the planned level\n", fn);
        return false;
    }
    const int scored = scored_states(pm, cs);
    if (scored < 1) {
        log("jepa: %s: horizon %d at level %d does not reach one state of level %d (strides multiply)\n", fn, cs.horizon, cs.level, cs.goal_level);
        return false;
    }
    const int W = std::min(std::max(1, cs.cost_last_n), scored);
    if (cs.n_goal != 1 && cs.n_goal != W) {
        log("jepa: %s: %d goal states for %d scored predictions (horizon %d, cost_last_n %d): give one goal, or exactly one per scored prediction\n",
            fn, cs.n_goal, W, cs.horizon, cs.cost_last_n);
        return false;
    }
    if (pm.pooled_chunks(cs) > 0) {
        const DLevel & L = pm.levels[(size_t) cs.level - 1];
        const DLevel & U = pm.levels[(size_t) cs.level];
        const DActEnc & ae = U.ae;
        const int Ein = L.act0 ? L.E : L.A, stride = U.hp.stride;
        bool complete = false;
        if (ae.kind == 1) {
            complete = ae.fc1 && ae.fc2 && ae.fc1.in == stride * Ein && ae.fc2.in == ae.fc1.out && ae.fc2.out == U.A;
        } else if (ae.kind == 2) {
            const int d = ae.d;
            complete = d > 0 && ae.n_head > 0 && d % ae.n_head == 0 && ae.step && ae.step.in == Ein && ae.step.out == d &&
                       ae.pos && ae.pos_n >= (int64_t) (stride + 1) * d && !ae.blocks.empty() && ae.head0 && ae.head0.in == d &&
                       ae.head2 && ae.head2.in == ae.head0.out && ae.head2.out == U.A;
            for (const DSeqBlock & B : ae.blocks)
                complete = complete && B.qkv.in == d && B.qkv.out == 3 * d && B.out.in == d && B.out.out == d && B.up.in == d &&
                           B.down.in == B.up.out && B.down.out == d && B.ln1_w && B.ln2_w;
        }
        if (!complete) {
            log("jepa: %s: the action cost needs level %d's action encoder (jepa.hjepa.act_enc_kind mlp | seq with its weights)\n",
                fn, cs.level + 1);
            return false;
        }
    }
    return true;
}

CostSpec spec_from(int level, int horizon, const float * state, const jepa_hjepa_goal * goal, const jepa_hjepa_level_plan * lp) {
    CostSpec cs;
    cs.level = level;
    cs.horizon = horizon;
    cs.s0 = state;
    if (goal) {
        cs.goal = goal->states;
        cs.n_goal = goal->n_states;
        cs.goal_level = goal->level > 0 ? goal->level : level;
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


// stable_worldmodel.solver.decreasing_horizon_schedule (reference: src/hjepa-plan.cpp:1042-1059)
std::vector<int> decreasing_schedule(int num_calls, int horizon) {
    if (horizon == 1) return std::vector<int>((size_t) num_calls, 1);
    if (num_calls == 1) return {horizon};
    std::vector<int> s;
    if (num_calls < horizon) {
        for (int idx = 0; idx < num_calls; idx++) {
            const double v = 1.0 + (double) (horizon - 1) * (double) (num_calls - 1 - idx) / (double) (num_calls - 1);
            s.push_back(std::max(1, (int) std::ceil(v)));
        }
        return s;
    }
    const int per = num_calls / horizon, extra = num_calls % horizon;
    for (int i = 0; i < horizon; i++) {
        const int count = per + (i >= horizon - extra ? 1 : 0);
        s.insert(s.end(), (size_t) count, horizon - i);
    }
    return s;
}

}  // namespace

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
    return ctx->hplan.get();
}

// ---------------------------------------------------------------------------------------------
// one level's solve
// ---------------------------------------------------------------------------------------------
int HPlanner::solve(const CostSpec & cs, const jepa_hjepa_level_plan & lp, NoiseSource & noise, SolveOut & out) {
    cudaStream_t st = ctx->stream;
    const DLevel & L = levels[(size_t) cs.level - 1];
    const int A = L.A, T = cs.horizon, S = std::max(1, lp.n_samples), D = L.D;
    const size_t row = (size_t) T * A, N = (size_t) S * row;
    const Prior prior = prior_of(L, lp.action_clip_sigma);
    Shard * sh = ctx->shard.get();
    const int world = sh ? sh->world : 1, rank = sh ? sh->rank : 0;
    const int r0 = (int) ((int64_t) S * rank / world), r1 = (int) ((int64_t) S * (rank + 1) / world);
    const int Sl = r1 - r0;   // this rank's candidates

    // candidates: prior mean, all but the first perturbed (the whole stream is drawn on every rank)
    std::vector<float> x(N), z(N);
    for (size_t i = 0; i < N; i++) x[i] = prior.mean[i % (size_t) A];
    if (S > 1) {
        noise.fill(z.data(), N - row);
        for (size_t i = 0; i < N - row; i++) x[row + i] += z[i] * prior.std[i % (size_t) A] * lp.var_scale;
    }
    out.iters = 0;
    if (Sl < 1) { log("jepa: hjepa solve: %d candidates over %d GPUs leaves rank %d without any\n", S, world, rank); return -1; }
    // the rank's candidates as nc streams of consecutive rows: stream c holds rows [cr[c], cr[c + 1])
    const int nc = streams_for(Sl, L.P);
    std::vector<int> cr((size_t) nc + 1);
    for (int c = 0; c <= nc; c++) cr[(size_t) c] = (int) ((int64_t) Sl * c / nc);
    std::vector<Workspace *> wc((size_t) nc);
    std::string gens;
    for (int c = 0; c < nc; c++) {
        wc[(size_t) c] = workspace(cs.level, cr[(size_t) c + 1] - cr[(size_t) c], T, cs, c, nc);
        if (!wc[(size_t) c] || !cost_tables(*wc[(size_t) c], cs)) return -1;
        gens += std::to_string(wc[(size_t) c]->gen) + ",";
    }
    Workspace * w0 = wc[0];
    launches = 0;
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventRecord(e0, st);
    const bool clamp = !prior.lo.empty();
    for (int c = 0; c < nc; c++) {
        Workspace * w = wc[(size_t) c];
        const int Sc = w->S;
        JB_CUDA(cudaMemcpyAsync(w->x, x.data() + (size_t) (r0 + cr[(size_t) c]) * row, (size_t) Sc * row * 4, cudaMemcpyHostToDevice, st));
        JB_CUDA(cudaMemsetAsync(w->m, 0, (size_t) Sc * row * 4, st));
        JB_CUDA(cudaMemsetAsync(w->v, 0, (size_t) Sc * row * 4, st));
        JB_CUDA(cudaMemsetAsync(w->step_ctr, 0, 4 * sizeof(int), st));
        JB_CUDA(cudaMemcpyAsync(w->gtmp, cs.s0, (size_t) D * 4, cudaMemcpyHostToDevice, st));
        copy_rows(w->gtmp, 0, w->states, D, Sc, D, st);
        gather_actions(w->x, w->a_all, Sc, T, A, st);
        launches += 2;
        if (clamp) {
            JB_CUDA(cudaMemcpyAsync(w->lo, prior.lo.data(), (size_t) A * 4, cudaMemcpyHostToDevice, st));
            JB_CUDA(cudaMemcpyAsync(w->hi, prior.hi.data(), (size_t) A * 4, cudaMemcpyHostToDevice, st));
        }
    }
    // AdamW bias corrections, per iteration, in float on the host as the reference computes them
    const float b1 = 0.9f, b2 = 0.999f;
    std::vector<float> sched((size_t) 2 * std::max(1, lp.n_steps));
    for (int k = 0; k < lp.n_steps; k++) {
        const float c1 = 1.0f - std::pow(b1, (float) (k + 1)), c2 = 1.0f - std::pow(b2, (float) (k + 1));
        sched[(size_t) 2 * k] = lp.lr / c1;
        sched[(size_t) 2 * k + 1] = std::sqrt(c2);
    }
    // action noise: drawn up front when the iteration count is fixed, per iteration otherwise
    const bool noisy = lp.action_noise > 0.0f;
    const bool early = lp.early_stop_patience > 0;
    std::vector<float> zall;
    float * zdev = nullptr;
    if (noisy) {
        const size_t slots = early ? 1 : (size_t) std::max(1, lp.n_steps);
        if (!cuda_ok(cudaMalloc(&zdev, slots * (size_t) Sl * row * 4), "noise buffer")) return -1;
        if (!early) {
            zall.resize(N);
            for (int k = 0; k < lp.n_steps; k++) {
                noise.fill(zall.data(), N);
                cudaMemcpy(zdev + (size_t) k * Sl * row, zall.data() + (size_t) r0 * row, (size_t) Sl * row * 4, cudaMemcpyHostToDevice);
            }
        }
    }
    const int sched_cap = 4096;
    // one graph over every candidate stream: stream c's kernels on its own CUDA stream, forked from and
    // joined back into the context's stream
    auto capture = [&](bool with_grad, cudaGraphExec_t * exec, long long * nodes, const size_t zstride) -> int {
        cudaGraph_t g;
        JB_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        const long long l0 = launches;
        int rc = 0;
        if (nc > 1) rc = cuda_ok(cudaEventRecord(ev[0], st), "fork") ? 0 : -1;
        for (int c = 1; c < nc && !rc; c++) rc = cuda_ok(cudaStreamWaitEvent(wc[(size_t) c]->st, ev[0], 0), "fork") ? 0 : -1;
        for (int c = 0; c < nc && !rc; c++) {
            Workspace * w = wc[(size_t) c];
            rc = forward(*w, cs, with_grad);
            if (!rc && with_grad) rc = backward(*w, cs);
            if (!rc && with_grad) {
                adam_step(w->x, w->m, w->v, w->da_all, w->a_all, w->sched, w->step_ctr, lp.lr * lp.weight_decay,
                          zdev ? zdev + (size_t) cr[(size_t) c] * row : nullptr, lp.action_noise, zstride,
                          clamp ? w->lo : nullptr, clamp ? w->hi : nullptr, w->S, T, A, w->st);
                launches++;
            }
        }
        for (int c = 1; c < nc && !rc; c++) {
            rc = cuda_ok(cudaEventRecord(ev[(size_t) c], wc[(size_t) c]->st), "join") &&
                 cuda_ok(cudaStreamWaitEvent(st, ev[(size_t) c], 0), "join") ? 0 : -1;
        }
        const cudaError_t ce = cudaStreamEndCapture(st, &g);
        if (rc || ce != cudaSuccess) { cudaGetLastError(); log("jepa: hjepa solve: graph capture failed\n"); return -1; }
        *nodes = launches - l0;
        const cudaError_t ie = cudaGraphInstantiate(exec, g, 0);
        cudaGraphDestroy(g);
        return cuda_ok(ie, "cudaGraphInstantiate") ? 0 : -1;
    };
    // the first lowest cost over the candidate streams (stream order = row order): (value, local row)
    auto best_of = [&](float * val, int * idx, int * which) -> int {
        std::vector<float> v((size_t) nc);
        std::vector<int> ix((size_t) nc);
        for (int c = 0; c < nc; c++) {
            Workspace * w = wc[(size_t) c];
            argmin_first(w->cost, w->S, w->best_idx, w->best_val, st);
            launches++;
            JB_CUDA(cudaMemcpyAsync(&v[(size_t) c], w->best_val, 4, cudaMemcpyDeviceToHost, st));
            JB_CUDA(cudaMemcpyAsync(&ix[(size_t) c], w->best_idx, 4, cudaMemcpyDeviceToHost, st));
        }
        JB_CUDA(cudaStreamSynchronize(st));
        int b = 0;
        for (int c = 1; c < nc; c++) if (v[(size_t) c] < v[(size_t) b]) b = c;
        *val = v[(size_t) b];
        *idx = cr[(size_t) b] + ix[(size_t) b];
        if (which) *which = b;
        return 0;
    };
    auto run = [&]() -> int {
        const size_t zstride = (noisy && !early) ? (size_t) Sl * row : 0;
        // capture one iteration (forward, backward, AdamW) as a graph, replayed every iteration
        const std::string key = std::to_string(lp.lr * lp.weight_decay) + "/" + std::to_string(lp.action_noise) + "/" +
                                std::to_string(clamp) + "/" + std::to_string((uintptr_t) zdev) + "/" + std::to_string(zstride) +
                                "/" + gens;
        if (!w0->g_iter || w0->iter_key != key) {
            if (w0->g_iter) { cudaGraphExecDestroy(w0->g_iter); w0->g_iter = nullptr; }
            if (capture(true, &w0->g_iter, &w0->iter_nodes, zstride)) return -1;
            w0->iter_key = key;
        }
        launches = 0;
        float best = INFINITY;
        int stalled = 0;
        for (int step = 0; step < lp.n_steps; step++) {
            if (step % sched_cap == 0) {
                const int n = std::min(sched_cap, lp.n_steps - step);
                for (Workspace * w : wc) {
                    JB_CUDA(cudaMemcpyAsync(w->sched, sched.data() + (size_t) 2 * step, (size_t) 2 * n * 4, cudaMemcpyHostToDevice, st));
                    JB_CUDA(cudaMemsetAsync(w->step_ctr, 0, 2 * sizeof(int), st));
                }
                if (step > 0 && noisy && !early) {
                    log("jepa: hjepa solve: more than %d iterations with pre-drawn action noise are not supported\n", sched_cap);
                    return -1;
                }
            }
            if (noisy && early) {
                z.resize(N);
                noise.fill(z.data(), N);
                JB_CUDA(cudaMemcpyAsync(zdev, z.data() + (size_t) r0 * row, (size_t) Sl * row * 4, cudaMemcpyHostToDevice, st));
            }
            JB_CUDA(cudaGraphLaunch(w0->g_iter, st));
            launches += w0->iter_nodes;
            out.iters = step + 1;
            if (early) {
                // on the costs of the candidates BEFORE this update, as the reference does
                float score = 0.0f;
                int bi = 0;
                if (best_of(&score, &bi, nullptr)) return -1;
                if (sh && world > 1) score = sh->min_f32(score, st);
                const bool improved = !std::isfinite(best) || best - score > lp.early_stop_rel_delta * std::max(std::fabs(best), 1e-12f);
                if (improved) { best = score; stalled = 0; }
                else if (++stalled >= lp.early_stop_patience && step + 1 >= lp.min_its) break;
            }
        }
        // final evaluation without gradient, then the first lowest-cost candidate
        if (!w0->g_fwd || w0->fwd_key != gens) {
            if (w0->g_fwd) { cudaGraphExecDestroy(w0->g_fwd); w0->g_fwd = nullptr; }
            if (capture(false, &w0->g_fwd, &w0->fwd_nodes, 0)) return -1;
            w0->fwd_key = gens;
        }
        JB_CUDA(cudaGraphLaunch(w0->g_fwd, st));
        launches += w0->fwd_nodes;
        int idx = 0, which = 0;
        float cost = 0.0f;
        if (best_of(&cost, &idx, &which)) return -1;
        out.actions.assign(row, 0.0f);
        out.states.assign((size_t) (T + 1) * D, 0.0f);
        int owner = rank;
        if (sh && world > 1) {
            // (cost, global index) of every rank; the lowest cost wins, the lowest index on ties
            int gidx = r0 + idx;
            sh->argmin_global(cost, gidx, &cost, &gidx, &owner, st);
            idx = gidx - r0;
        }
        if (owner == rank) {
            for (int c = 0; c < nc; c++) if (idx >= cr[(size_t) c]) which = c;
            const Workspace * w = wc[(size_t) which];
            const int li = idx - cr[(size_t) which];
            JB_CUDA(cudaMemcpyAsync(out.actions.data(), w->x + (size_t) li * row, row * 4, cudaMemcpyDeviceToHost, st));
            JB_CUDA(cudaMemcpy2DAsync(out.states.data(), (size_t) D * 4, w->states + (size_t) li * D, (size_t) w->S * D * 4,
                                      (size_t) D * 4, (size_t) T + 1, cudaMemcpyDeviceToHost, st));
            JB_CUDA(cudaStreamSynchronize(st));
        }
        if (sh && world > 1) {
            if (!sh->bcast_host(out.actions.data(), row, owner, st) || !sh->bcast_host(out.states.data(), out.states.size(), owner, st)) return -1;
        }
        out.cost = cost;
        return 0;
    };
    const int rc = run();
    if (zdev) cudaFree(zdev);
    cudaEventRecord(e1, st);
    cudaEventSynchronize(e1);
    float ms = 0;
    cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    ctx->last_ms += ms;
    ctx->last_launches += launches;
    if (rc == 0 && gemm_error_flag(st)) { log("jepa: a tensor-core kernel gave up waiting on its pipeline\n"); return -1; }
    return rc;
}

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
    if (!ctx || mode < 0 || mode > 1) { log("jepa: jepa_b200_hjepa_set_step_modulation: a context and mode 0 or 1 are required\n"); return -1; }
    HPlanner * pm = hplanner_of(ctx, "jepa_b200_hjepa_set_step_modulation");
    if (!pm) return -1;
    if (pm->force_step_mod != (mode == 1)) pm->ws.clear();   // workspaces are planned for one mode
    pm->force_step_mod = mode == 1;
    return 0;
}

jepa_hjepa_level_plan jepa_hjepa_level_plan_default(void) {
    jepa_hjepa_level_plan p;
    p.horizon = 1;
    p.pre_decay_horizon = 0;
    p.n_samples = 100;
    p.n_steps = 90;
    p.lr = 0.1f;
    p.weight_decay = 0.01f;
    p.var_scale = 1.0f;
    p.action_noise = 0.0f;
    p.action_clip_sigma = 0.0f;
    p.min_its = 30;
    p.early_stop_patience = 5;
    p.early_stop_rel_delta = 1e-2f;
    p.cost_last_n = 1;
    p.intermediate_cost_weight = 1.0f;
    p.action_cost_weight = 0.0f;
    p.num_subgoals = 1;
    p.horizon_one_goal_upper = 0;
    return p;
}

int jepa_hjepa_plan_cost(jepa_context * ctx, int level, const float * state, const jepa_hjepa_goal * goal,
                         const jepa_hjepa_level_plan * plan, const float * actions, int n_samples, int horizon,
                         float * costs, float * grad) {
    if (!ctx || !state || !goal || !actions || !costs || n_samples < 1) return -1;
    HPlanner * pm = hplanner_of(ctx, "jepa_hjepa_plan_cost");
    if (!pm) return -1;
    const CostSpec cs = spec_from(level, horizon, state, goal, plan);
    if (!check_spec(*pm, cs, "jepa_hjepa_plan_cost")) return -1;
    return pm->plan_cost(cs, actions, n_samples, costs, grad);
}

int jepa_hjepa_solve(jepa_context * ctx, int level, const float * state, const jepa_hjepa_goal * goal,
                     const jepa_hjepa_level_plan * plan, jepa_randn_fn randn, void * randn_user, float * actions,
                     float * states, float * cost, int * iters) {
    if (!ctx || !state || !goal || !plan || !actions) return -1;
    HPlanner * pm = hplanner_of(ctx, "jepa_hjepa_solve");
    if (!pm) return -1;
    const CostSpec cs = spec_from(level, plan->horizon, state, goal, plan);
    if (!check_spec(*pm, cs, "jepa_hjepa_solve")) return -1;
    if (plan->n_samples < 1 || plan->n_steps < 0) {
        log("jepa: jepa_hjepa_solve: n_samples %d and n_steps %d have to be >= 1 and >= 0\n", plan->n_samples, plan->n_steps);
        return -1;
    }
    NoiseSource ns;
    ns.fn = randn;
    ns.user = randn_user;
    ns.rng.seed(0x4a455041ull + (uint64_t) level);
    SolveOut r;
    ctx->last_ms = 0;
    ctx->last_launches = 0;
    if (pm->solve(cs, *plan, ns, r)) return -1;
    memcpy(actions, r.actions.data(), r.actions.size() * sizeof(float));
    if (states) memcpy(states, r.states.data(), r.states.size() * sizeof(float));
    if (cost) *cost = r.cost;
    if (iters) *iters = r.iters;
    return 0;
}

int jepa_hjepa_horizons(const jepa_model * model, const jepa_hjepa_level_plan * levels, int n_levels,
                        int replanning_interval, int eval_budget, int steps_taken, int * horizons) {
    if (!model || !levels || !horizons || !model->hj.present) return -1;
    if (n_levels != (int) model->hj.levels.size() || replanning_interval < 1 || eval_budget < 1 || steps_taken < 0) {
        log("jepa: jepa_hjepa_horizons: need one plan per level (%zu), a positive replanning interval and budget, and steps_taken >= 0\n",
            model->hj.levels.size());
        return -1;
    }
    const int calls = (eval_budget + replanning_interval - 1) / replanning_interval;
    const int call = steps_taken / replanning_interval;
    if (call >= calls) {
        log("jepa: jepa_hjepa_horizons: step %d is past the evaluation budget of %d\n", steps_taken, eval_budget);
        return -1;
    }
    std::vector<int> above;
    for (int lv = n_levels; lv >= 1; lv--) {
        const jepa_hjepa_level_plan & lp = levels[lv - 1];
        if (lp.horizon < 1) {
            log("jepa: jepa_hjepa_horizons: level %d has horizon %d\n", lv, lp.horizon);
            return -1;
        }
        std::vector<int> s;
        if (lv == n_levels) {
            s = decreasing_schedule(calls, lp.horizon);
        } else {
            // hold the pre-decay horizon until the level above is down to one step, then decay
            const int pre = lp.pre_decay_horizon > 0 ? lp.pre_decay_horizon : model->hj.levels[(size_t) lv].stride;
            const auto one = std::find(above.begin(), above.end(), 1);
            if (one == above.end()) {
                s.assign((size_t) calls, pre);
            } else {
                const int tail_start = (int) (one - above.begin());
                s.assign((size_t) tail_start, pre);
                const std::vector<int> tail = decreasing_schedule(calls - tail_start, lp.horizon);
                s.insert(s.end(), tail.begin(), tail.end());
            }
        }
        horizons[lv - 1] = s[(size_t) call];
        above = std::move(s);
    }
    return 0;
}

int jepa_hjepa_plan(jepa_context * ctx, const float * const * states, const float * const * goals,
                    const jepa_hjepa_level_plan * levels, int n_levels, jepa_randn_fn randn, void * randn_user,
                    float * actions, jepa_hjepa_plan_info * info) {
    if (!ctx || !states || !goals || !levels || !actions) return -1;
    HPlanner * pm = hplanner_of(ctx, "jepa_hjepa_plan");
    if (!pm) return -1;
    if (n_levels != (int) pm->levels.size()) {
        log("jepa: jepa_hjepa_plan: %d level plans for a model with %zu levels\n", n_levels, pm->levels.size());
        return -1;
    }
    for (int lv = 1; lv <= n_levels; lv++) {
        if (!states[lv - 1] || !goals[lv - 1]) {
            log("jepa: jepa_hjepa_plan: the current and goal state of level %d are missing\n", lv);
            return -1;
        }
        if (levels[lv - 1].n_samples < 1 || levels[lv - 1].n_steps < 0 || levels[lv - 1].num_subgoals < 1) {
            log("jepa: jepa_hjepa_plan: level %d: n_samples, n_steps and num_subgoals have to be >= 1, >= 0, >= 1\n", lv);
            return -1;
        }
    }
    if (info) *info = jepa_hjepa_plan_info{};
    ctx->last_ms = 0;
    ctx->last_launches = 0;
    SolveOut upper;
    bool have_upper = false;
    int skipped_goal_level = 0;
    bool upper_anchored = true;
    std::vector<float> goal_buf, goal_act;
    for (int lv = n_levels; lv >= 1; lv--) {
        const jepa_hjepa_level_plan & lp = levels[lv - 1];
        if (lv > 1 && lp.horizon == 1) {
            // a one-step plan up here gives the level below no waypoint: skip it and pass the real goal down
            skipped_goal_level = lp.horizon_one_goal_upper ? (skipped_goal_level ? skipped_goal_level : lv) : 0;
            have_upper = false;
            continue;
        }
        CostSpec cs;
        cs.level = lv;
        cs.horizon = lp.horizon;
        cs.s0 = states[lv - 1];
        cs.cost_last_n = lp.cost_last_n;
        cs.intermediate_cost_weight = lp.intermediate_cost_weight;
        cs.action_cost_weight = lp.action_cost_weight;
        bool anchored;
        if (!have_upper) {
            cs.goal_level = skipped_goal_level ? skipped_goal_level : lv;
            cs.goal = goals[cs.goal_level - 1];
            cs.n_goal = 1;
            cs.dense = cs.goal_level > lv;
            anchored = true;
        } else {
            const DLevel & up = pm->levels[(size_t) lv];
            const int Du = up.D, Au = up.A;
            const int n_up = (int) upper.states.size() / Du;
            const int n_sub = std::min(levels[lv].num_subgoals, n_up - 1);
            goal_buf.assign(upper.states.begin() + Du, upper.states.begin() + (std::ptrdiff_t) (1 + n_sub) * Du);
            goal_act.assign(upper.actions.begin(), upper.actions.begin() + (std::ptrdiff_t) n_sub * Au);
            anchored = false;
            if (1 + levels[lv].num_subgoals >= n_up && upper_anchored) {
                // the upper plan's last state should have reached its goal: aim at the goal itself
                memcpy(goal_buf.data() + (size_t) (n_sub - 1) * Du, goals[lv], (size_t) Du * sizeof(float));
                anchored = true;
            }
            cs.goal_level = lv + 1;
            cs.goal = goal_buf.data();
            cs.n_goal = n_sub;
            cs.goal_action = goal_act.data();
            if (n_sub > 1) {
                const int expected = (lp.horizon + up.hp.stride) / up.hp.stride - 1;
                if (n_sub != expected) {
                    log("jepa: jepa_hjepa_plan: level %d: %d subgoals from above, but horizon %d at stride %d reaches %d states of level %d\n",
                        lv, n_sub, lp.horizon, up.hp.stride, expected, lv + 1);
                    return -1;
                }
            }
        }
        if (!check_spec(*pm, cs, "jepa_hjepa_plan")) return -1;
        NoiseSource ns;
        ns.fn = randn;
        ns.user = randn_user;
        ns.rng.seed(0x4a455041ull + (uint64_t) lv);
        SolveOut r;
        if (pm->solve(cs, lp, ns, r)) return -1;
        upper = std::move(r);
        if (info && lv <= JEPA_HJEPA_MAX_PLAN_LEVELS) {
            info->planned[lv - 1] = 1;
            info->cost[lv - 1] = upper.cost;
            info->iters[lv - 1] = upper.iters;
            info->goal_level[lv - 1] = cs.goal_level;
        }
        upper_anchored = anchored;
        skipped_goal_level = 0;
        have_upper = true;
    }
    memcpy(actions, upper.actions.data(), upper.actions.size() * sizeof(float));
    return 0;
}

}  // extern "C"
