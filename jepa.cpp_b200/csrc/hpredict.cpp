// The H-JEPA multi-frame predictor on the GPU: jepa_hjepa_predict and jepa_hjepa_rollout (reference:
// src/hjepa.cpp:566-667 over the adaLN-zero transformer of src/lewm.cpp:33-95).
//
// The planner runs the predictor one frame at a time (a window of one, where attention reduces to the
// value projection). These entry points run it over T <= pred_n_frames frames of one sequence with causal
// softmax attention across frames: row t of the output is the state predicted after frames 0..t.
//
//   c  = [pred.act_embed](act_embed(a))                 x = states + pos_embed[:T] (-> in_proj)
//   cs = silu([cond_proj](c))
//   per block: mod = adaln(cs); h = ln1(LN0(x) (1 + sc_a) + sh_a); q, k, v = qkv(h)
//              x += g_a * out(causal_attention(q, k, v)); h = ln2(LN0(x) (1 + sc_m) + sh_m)
//              x += g_m * down(gelu(up(h)))
//   y  = norm(x) (-> out_proj) (-> proj.2(gelu(proj.0)))
//
// A call covers a handful of rows, so every product is a SIMT linear (float32, one output per thread) and
// the attention is the grouped kernel of pool.cu with its causal mask; the work is launch latency, not
// bandwidth or FLOPs. A rollout keeps its growing sequence on the device: one upload, n_steps predictor
// passes over the last `history` frames, one download.
#include "hplan.h"
#include "common.h"

#include "../../include/jepa.h"

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <vector>

namespace jb {

int HPlanner::predict_dev(int level, const float * states, const float * actions, int T, float * out, cudaStream_t st) {
    const DLevel & L = levels[(size_t) level - 1];
    const int D = L.D, P = L.P, I = L.I, F = L.F, A = L.A, H = L.hp.pred_n_head, ldm = 6 * P;
    PredWs & w = pred;
    if (!group_mha_prepare(T, I, H)) { log("jepa: hjepa predictor: %d frames of width %d do not fit one CTA\n", T, I); return -1; }
    // conditioning: act_embed (SiLU MLP, identity when absent), the predictor's own embedder, cond_proj, SiLU
    const float * c = actions;
    int cw = A;
    if (L.act0) {
        linear_simt(c, cw, L.act0.w, L.act0.b, w.t1, L.act0.out, T, L.act0.out, cw, st);
        act_fwd(w.t1, L.act0.out, w.t2, L.act0.out, T, L.act0.out, 2, st);
        linear_simt(w.t2, L.act0.out, L.act2.w, L.act2.b, w.c, L.E, T, L.E, L.act0.out, st);
        c = w.c; cw = L.E;
    }
    if (L.pact0) {
        linear_simt(c, cw, L.pact0.w, L.pact0.b, w.t1, L.pact0.out, T, L.pact0.out, cw, st);
        act_fwd(w.t1, L.pact0.out, w.t2, L.pact0.out, T, L.pact0.out, 2, st);
        linear_simt(w.t2, L.pact0.out, L.pact2.w, L.pact2.b, w.cc, L.C, T, L.C, L.pact0.out, st);
        c = w.cc; cw = L.C;
    }
    if (L.cond_proj) {
        linear_simt(c, cw, L.cond_proj.w, L.cond_proj.b, w.t1, P, T, P, cw, st);
        act_fwd(w.t1, P, w.cs, P, T, P, 2, st);
    } else {
        act_fwd(c, cw, w.cs, P, T, P, 2, st);
    }
    // x = states + pos_embed[:T] (-> in_proj)
    copy_rows(states, D, w.xa, D, T, D, st);
    add_inplace(w.xa, D, L.pos_all, D, T, D, st);
    if (L.in_proj) linear_simt(w.xa, D, L.in_proj.w, L.in_proj.b, w.x, P, T, P, D, st);
    else copy_rows(w.xa, D, w.x, P, T, P, st);
    for (int l = 0; l < L.L; l++) {
        const DBlock & B = L.blocks[(size_t) l];
        linear_simt(w.cs, P, L.adaln.w + (size_t) l * ldm * P, L.adaln.b + (size_t) l * ldm, w.mod, ldm, T, ldm, P, st);
        // attention half (the prologue writes hi / lo planes; their sum is the float32 value exactly)
        block_pre(w.x, P, w.mod, ldm, 0, P, B.ln1_w, B.ln1_b, adaln_eps, ln_eps, w.hhi, w.hlo, P, w.st0, w.st1, T, P, st);
        add_inplace(w.hhi, P, w.hlo, P, T, P, st);
        linear_simt(w.hhi, P, B.qk.w, B.qk.b, w.qkv, 3 * I, T, 2 * I, P, st);
        linear_simt(w.hhi, P, B.v.w, B.v.b, w.qkv + 2 * I, 3 * I, T, I, P, st);
        group_mha_fwd(w.qkv, w.o, w.probs, 1, T, I, H, st, true);
        linear_simt(w.o, I, B.out.w, B.out.b, w.a, P, T, P, I, st);
        gated_add(w.x, P, w.a, P, w.mod + 2 * P, ldm, w.xm, P, T, P, st);
        // MLP half
        block_pre(w.xm, P, w.mod, ldm, 3 * P, 4 * P, B.ln2_w, B.ln2_b, adaln_eps, ln_eps, w.hhi, w.hlo, P, w.st0, w.st1, T, P, st);
        add_inplace(w.hhi, P, w.hlo, P, T, P, st);
        linear_simt(w.hhi, P, B.up.w, B.up.b, w.u, F, T, F, P, st);
        act_fwd(w.u, F, w.g, F, T, F, 0, st);
        linear_simt(w.g, F, B.down.w, B.down.b, w.a, P, T, P, F, st);
        gated_add(w.xm, P, w.a, P, w.mod + 5 * P, ldm, w.x, P, T, P, st);
        launches += 19;
    }
    layer_norm(w.x, P, L.norm_w, L.norm_b, ln_eps, w.y, P, nullptr, nullptr, nullptr, T, P, st);
    const float * cur = w.y;
    int cwid = P;
    if (L.out_proj) {
        linear_simt(cur, cwid, L.out_proj.w, L.out_proj.b, w.t1, L.out_proj.out, T, L.out_proj.out, cwid, st);
        cur = w.t1; cwid = L.out_proj.out;
    }
    if (L.proj0) {
        linear_simt(cur, cwid, L.proj0.w, L.proj0.b, w.u, L.proj0.out, T, L.proj0.out, cwid, st);
        act_fwd(w.u, L.proj0.out, w.g, L.proj0.out, T, L.proj0.out, 0, st);
        linear_simt(w.g, L.proj0.out, L.proj2.w, L.proj2.b, w.t2, L.proj2.out, T, L.proj2.out, L.proj0.out, st);
        cur = w.t2; cwid = L.proj2.out;
    }
    copy_rows(cur, cwid, out, cwid, T, cwid, st);
    launches += 16;
    return 0;
}

// width of the predictor's output rows at a level
static int pred_out_dim(const DLevel & L) {
    if (L.proj2) return L.proj2.out;
    if (L.out_proj) return L.out_proj.out;
    return L.P;
}

namespace {

HPlanner * predictor_of(jepa_context * ctx, int level, const char * fn) {
    if (!ctx->model->hj.present) {
        log("jepa: %s: '%s' is not an H-JEPA model\n", fn, ctx->model->name.c_str());
        return nullptr;
    }
    const int n = (int) ctx->model->hj.levels.size();
    if (level < 1 || level > n) {
        log("jepa: %s: level %d is out of range, the model has levels 1..%d\n", fn, level, n);
        return nullptr;
    }
    HPlanner * pm = hplanner_of(ctx, fn);
    if (!pm || !pm->ensure_predict(level)) return nullptr;
    return pm;
}

struct DevBuf {
    void * p = nullptr;
    ~DevBuf() { if (p) cudaFree(p); }
    bool alloc(size_t bytes) { return cuda_ok(cudaMalloc(&p, std::max<size_t>(bytes, 4)), "predictor buffer"); }
    float * f() const { return (float *) p; }
};

}  // namespace

}  // namespace jb

using namespace jb;

extern "C" {

int jepa_hjepa_predict(jepa_context * ctx, int level, const float * states, const float * actions, int n_frames,
                       jepa_output * out) {
    if (!ctx || !states || !actions || !out || n_frames <= 0) return -1;
    HPlanner * pm = predictor_of(ctx, level, "jepa_hjepa_predict");
    if (!pm) return -1;
    const DLevel & L = pm->levels[(size_t) level - 1];
    if (n_frames > L.hp.pred_n_frames) {
        log("jepa: jepa_hjepa_predict: %d frames requested, the level-%d predictor has %d position slots\n", n_frames, level,
            L.hp.pred_n_frames);
        return -1;
    }
    const int T = n_frames, D = L.D, A = L.A, Do = pred_out_dim(L);
    cudaStream_t st = ctx->stream;
    DevBuf s, a, y;
    if (!s.alloc((size_t) T * D * 4) || !a.alloc((size_t) T * A * 4) || !y.alloc((size_t) T * Do * 4)) return -1;
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventRecord(e0, st);
    pm->launches = 0;
    JB_CUDA(cudaMemcpyAsync(s.p, states, (size_t) T * D * 4, cudaMemcpyHostToDevice, st));
    JB_CUDA(cudaMemcpyAsync(a.p, actions, (size_t) T * A * 4, cudaMemcpyHostToDevice, st));
    if (pm->predict_dev(level, s.f(), a.f(), T, y.f(), st)) return -1;
    float * data = (float *) malloc((size_t) T * Do * sizeof(float));
    if (!data) { log("jepa: jepa_hjepa_predict: out of host memory\n"); return -1; }
    if (!cuda_ok(cudaMemcpyAsync(data, y.p, (size_t) T * Do * 4, cudaMemcpyDeviceToHost, st), "predict output") ||
        !cuda_ok(cudaStreamSynchronize(st), "jepa_hjepa_predict")) {
        free(data);
        return -1;
    }
    cudaEventRecord(e1, st);
    cudaEventSynchronize(e1);
    float ms = 0;
    cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    ctx->last_ms = ms;
    ctx->last_launches = pm->launches;
    if (gemm_error_flag(st)) { free(data); log("jepa: jepa_hjepa_predict: a tensor-core kernel gave up waiting on its pipeline\n"); return -1; }
    out->data = data;
    out->n_tokens = T;
    out->dim = Do;
    return 0;
}

int jepa_hjepa_rollout(jepa_context * ctx, int level, const float * states, int n_seed, const float * actions, int n_steps,
                       int history, float * out) {
    if (!ctx || !states || !actions || !out || n_seed <= 0 || n_steps <= 0) return -1;
    HPlanner * pm = predictor_of(ctx, level, "jepa_hjepa_rollout");
    if (!pm) return -1;
    const DLevel & L = pm->levels[(size_t) level - 1];
    if (history < 1 || history > L.hp.pred_n_frames) {
        log("jepa: jepa_hjepa_rollout: history %d is outside 1..%d (the level-%d predictor's position slots)\n", history,
            L.hp.pred_n_frames, level);
        return -1;
    }
    const int D = L.D, A = L.A, Do = pred_out_dim(L);
    if (Do != D) {
        log("jepa: jepa_hjepa_rollout: the level-%d predictor writes %d-wide rows for %d-wide states\n", level, Do, D);
        return -1;
    }
    const int64_t n_seq = (int64_t) n_seed + n_steps;
    const int64_t n_act = n_seq - 1;   // row j of the sequence is conditioned on actions[j]
    cudaStream_t st = ctx->stream;
    DevBuf seq, act, y;
    if (!seq.alloc((size_t) n_seq * D * 4) || !act.alloc((size_t) n_act * A * 4) || !y.alloc((size_t) L.hp.pred_n_frames * Do * 4))
        return -1;
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventRecord(e0, st);
    pm->launches = 0;
    JB_CUDA(cudaMemcpyAsync(seq.p, states, (size_t) n_seed * D * 4, cudaMemcpyHostToDevice, st));
    JB_CUDA(cudaMemcpyAsync(act.p, actions, (size_t) n_act * A * 4, cudaMemcpyHostToDevice, st));
    for (int step = 0; step < n_steps; step++) {
        const int64_t have = (int64_t) n_seed + step;
        const int wlen = have < history ? (int) have : history;
        const int64_t first = have - wlen;
        if (pm->predict_dev(level, seq.f() + (size_t) first * D, act.f() + (size_t) first * A, wlen, y.f(), st)) return -1;
        // the window's last row is the next state
        JB_CUDA(cudaMemcpyAsync(seq.f() + (size_t) have * D, y.f() + (size_t) (wlen - 1) * D, (size_t) D * 4,
                                cudaMemcpyDeviceToDevice, st));
    }
    JB_CUDA(cudaMemcpyAsync(out, seq.f() + (size_t) n_seed * D, (size_t) n_steps * D * 4, cudaMemcpyDeviceToHost, st));
    cudaEventRecord(e1, st);
    if (!cuda_ok(cudaEventSynchronize(e1), "jepa_hjepa_rollout")) return -1;
    float ms = 0;
    cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    ctx->last_ms = ms;
    ctx->last_launches = pm->launches;
    if (gemm_error_flag(st)) { log("jepa: jepa_hjepa_rollout: a tensor-core kernel gave up waiting on its pipeline\n"); return -1; }
    return 0;
}

}  // extern "C"
