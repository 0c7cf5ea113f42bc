// H-JEPA gradient planner on the GPU: device weights, per-solve workspaces and the forward / backward
// sweep of the candidate rollout (the reference's host tape, src/hjepa-plan.cpp:208-810, re-planned as
// whole-batch kernels).
#pragma once

#include "kernels.h"
#include "model.h"

#include <map>
#include <memory>
#include <vector>

namespace jb {

// One linear layer on the device. w / wt are float32 [out][in] / [in][out]; the split planes are the
// tensor-core operands of the forward (y = x W^T, K = in) and backward (dx = dy W, K = out) products.
struct DLin {
    int in = 0, out = 0;
    float * w = nullptr, * wt = nullptr;
    float * w_hi = nullptr, * w_lo = nullptr, * wt_hi = nullptr, * wt_lo = nullptr;
    // the GGUF block planes the GEMM dequantises in its mainloop, per orientation (fmt QF_NONE: the hi / lo
    // planes above serve that orientation)
    QuantB fq, tq;
    float * b = nullptr;
    explicit operator bool() const { return in > 0; }
    // the B operand of y = x W^T (forward) and of dx = dy W (transposed)
    SplitMat fwd() const { SplitMat m{w_hi, w_lo, in}; m.q = fq; return m; }
    SplitMat bwd() const { SplitMat m{wt_hi, wt_lo, out}; m.q = tq; return m; }
    bool tc_fwd() const { return in >= 16 && (in % 4) == 0 && out >= 16; }
    bool tc_bwd() const { return out >= 16 && (out % 4) == 0 && in >= 16; }
};

struct DBlock {
    DLin v, out, up, down;
    DLin qk;    // the query and key rows of the fused qkv, f32 only: the multi-frame predictor (loaded on first use)
    DLin ov;    // out(V(h)) composed: W_out W_v, W_out b_v + b_out (one query over one key: attention is V)
    float * ln1_w = nullptr, * ln1_b = nullptr, * ln2_w = nullptr, * ln2_b = nullptr;
};

// One transformer block of a 'seq' action encoder (pre-norm, ReLU MLP).
struct DSeqBlock {
    DLin qkv, out, up, down;
    float * ln1_w = nullptr, * ln1_b = nullptr, * ln2_w = nullptr, * ln2_b = nullptr;
};

// A level's action encoder: `stride` action embeddings of the level below -> one latent action of this
// level (build_action_pool, src/hjepa-plan.cpp:663-684). 'mlp': concat -> fc1 -> ReLU -> fc2 (-> LN);
// 'seq': a CLS token plus one token per step through transformer blocks, CLS -> head -> LN(1e-6).
struct DActEnc {
    int kind = 0;                     // 0 none, 1 mlp, 2 seq
    DLin fc1, fc2;
    DLin step, head0, head2;
    std::vector<DSeqBlock> blocks;
    float * pos = nullptr;            // [max_chunk + 1][d]
    int64_t pos_n = 0;                // elements of pos
    float * headln_w = nullptr, * headln_b = nullptr, * out_w = nullptr, * out_b = nullptr;
    int d = 0, n_head = 0;
};

struct DLevel {
    HLevel hp;
    DActEnc ae;
    int D = 0, P = 0, F = 0, I = 0, L = 0, A = 0, E = 0, C = 0;   // state, predictor, ffn, inner, layers, action, act-embed, cond widths
    float * pos0 = nullptr;
    DLin act0, act2, pact0, pact2, in_proj, cond_proj, out_proj, proj0, proj2;
    float * norm_w = nullptr, * norm_b = nullptr;
    std::vector<DBlock> blocks;
    DLin adaln;                       // every block's adaLN linear stacked: [6 P L][P]
    // this level's state encoder (applied to states of the level below)
    float * enc_in_w = nullptr, * enc_in_b = nullptr, * enc_out_w = nullptr, * enc_out_b = nullptr;
    DLin enc_fc1, enc_fc2;
    std::vector<float> queue;         // host: recorded latent actions [n][A]
    float * pos_all = nullptr;        // every row of pred.pos_embed [n_frames][D] (multi-frame predictor, on first use)
};

// Device buffers of the multi-frame predictor (jepa_hjepa_predict / _rollout): T <= the largest
// pred_n_frames rows, each buffer as wide as the widest activation of any level.
struct PredWs {
    Arena arena;
    int rows = 0, heads = 0;
    size_t width = 0;
    float * xa = nullptr, * x = nullptr, * xm = nullptr, * c = nullptr, * cc = nullptr, * cs = nullptr;
    float * t1 = nullptr, * t2 = nullptr, * mod = nullptr, * hhi = nullptr, * hlo = nullptr, * qkv = nullptr;
    float * o = nullptr, * a = nullptr, * u = nullptr, * g = nullptr, * y = nullptr, * probs = nullptr;
    LnStats * st0 = nullptr, * st1 = nullptr;
};

// Device buffers of one encoder application in the goal-projection chain.
struct EncStage {
    int lv = 0;                       // level whose encoder runs
    std::vector<int> src_pos;         // positions (in the previous list) it reads
    int n = 0;                        // states encoded (excluding the context state)
    float * in = nullptr;             // gathered inputs [n S][Din]
    LnStats * st1 = nullptr, * st2 = nullptr;
    float * h_hi = nullptr, * h_lo = nullptr;   // in_norm output, split
    float * u = nullptr;              // fc1 pre-activation [n S][H]
    float * g_hi = nullptr, * g_lo = nullptr;   // gelu(u), split
    float * y = nullptr;              // fc2 output [n S][Dout]
    float * out = nullptr;            // after out_norm [n S][Dout] (= y when there is none)
    float * gout = nullptr, * gy = nullptr, * gin = nullptr;   // gradients
    float * d_hi = nullptr, * d_lo = nullptr;
};

// Device buffers of the action cost: the last Wa whole chunks of the candidates' action embeddings pooled
// by the upper level's action encoder, n = Wa S rows (chunk-major), G = stride + 1 tokens per row for 'seq'.
struct PoolWs {
    int Wa = 0, c0 = 0, stride = 0, G = 0;   // chunks scored, first chunk, steps per chunk, tokens per group
    float * x = nullptr;              // mlp: [n][stride E] concatenated chunk; seq: step-linear outputs [Wa stride S][d]
    std::vector<float *> xs, qkv, probs, xmid, u;   // seq: per block (xs: block inputs, one more for the output)
    std::vector<LnStats *> st1, st2;
    float * h = nullptr, * r = nullptr;             // mlp: fc1 pre-activation / ReLU; seq: LN / ReLU scratch
    float * z = nullptr, * zg = nullptr, * zl = nullptr;   // seq head: head0 output, GELU, head LN
    float * ypre = nullptr, * y = nullptr;          // before the output LN / pooled latent actions [n][Au]
    LnStats * sth = nullptr, * sto = nullptr;
    float * gy = nullptr;             // cost gradient wrt y
    float * ga = nullptr, * gb = nullptr, * gc = nullptr;   // backward scratch
    float * ge = nullptr;             // gradient wrt the embeddings, [R][E] t-major, zero outside the chunks
    const float ** ptrs = nullptr;
    float ** gptrs = nullptr;
    float * goals = nullptr, * weights = nullptr;
};

struct Workspace {
    int level = 0, S = 0, T = 0;
    long long gen = 0;                // creation number (keys the graphs that span several workspaces)
    // step-at-a-time modulation (when every step's [T S][6PL] modulation and its gradient do not fit): the
    // adaLN GEMM runs per step in the forward and again in the backward, dmod is folded into dcs per step.
    // Bit-identical to the all-steps mode while the step's rows and all steps' rows take the same GEMM kernel
    // (always below 768 wide; at 768 and wider, when a step has more than 256 rows), else equal to rounding.
    bool step_mod = false;
    // within step_mod: every step's forward modulation is still kept ([T S][6PL], one copy), so the backward
    // reads it instead of recomputing it; only the gradient is folded per step (dmod holds one step's rows)
    bool keep_mod = false;
    cudaStream_t st = nullptr;        // the stream its kernels are launched on
    PoolWs pool;
    Arena arena;
    // actions / optimiser
    float * x = nullptr, * m = nullptr, * v = nullptr, * grad = nullptr, * a_all = nullptr, * da_all = nullptr;
    float * sched = nullptr, * z = nullptr, * lo = nullptr, * hi = nullptr;
    int * step_ctr = nullptr;
    // conditioning path over R = T S rows
    float * ae_u = nullptr, * ae_s = nullptr, * e = nullptr, * pa_u = nullptr, * pa_s = nullptr, * c0 = nullptr;
    float * cpre = nullptr, * cs_hi = nullptr, * cs_lo = nullptr, * mod = nullptr, * dmod_hi = nullptr, * dmod_lo = nullptr;
    float * dcs = nullptr, * dc = nullptr, * tmpR = nullptr, * tmpR2 = nullptr;
    // rollout
    float * states = nullptr;         // [(T+1) S][D]
    float * gstate = nullptr;         // [(T+1) S][D] cost gradients wrt the states
    float * xs = nullptr;             // [T][L+1][S][P]
    float * xmid = nullptr, * o = nullptr, * dn = nullptr;   // [T][L][S][P]
    float * u = nullptr;              // [T][L][S][F] gelu' at the up projection's pre-activation
    LnStats * sta0 = nullptr, * sta1 = nullptr, * stm0 = nullptr, * stm1 = nullptr;   // [T][L][S]
    LnStats * stn = nullptr;          // [T][S]
    float * yn = nullptr;             // final-norm output when a projection follows [T][S][P]
    float * yo = nullptr, * pu = nullptr;   // out_proj output / proj0 pre-activation [T][S][*]
    // scratch
    float * h_hi = nullptr, * h_lo = nullptr, * v_hi = nullptr, * v_lo = nullptr, * g_hi = nullptr, * g_lo = nullptr;
    float * gx = nullptr, * gmid = nullptr, * gh = nullptr, * d_hi = nullptr, * d_lo = nullptr, * du_hi = nullptr, * du_lo = nullptr;
    float * dv_hi = nullptr, * dv_lo = nullptr, * gtmp = nullptr, * gtmp2 = nullptr, * sp_hi = nullptr, * sp_lo = nullptr;
    // cost
    float * cost = nullptr, * goals = nullptr, * weights = nullptr;
    const float ** pred_ptrs = nullptr;
    float ** gpred_ptrs = nullptr;
    int * best_idx = nullptr;
    float * best_val = nullptr;
    std::vector<EncStage> enc;
    // scratch of the GEMM's K-split fix-up (narrow, long products: every such product of this workspace
    // uses it, so the split never depends on a call's row count); counters zeroed before each call
    float * fix = nullptr; size_t fix_floats = 0;
    int * fix_count = nullptr; size_t fix_counters = 0;
    // captured graphs
    cudaGraphExec_t g_iter = nullptr, g_fwd = nullptr;
    std::string graph_key, iter_key, fwd_key;
    long long iter_nodes = 0, fwd_nodes = 0;
    ~Workspace();
};

// One cost evaluation: which level plans how far, scored against which goal (the reference's cost
// specification, src/hjepa-plan.cpp:689-701)
struct CostSpec {
    int level = 1, horizon = 1;
    const float * s0 = nullptr;
    const float * goal = nullptr;
    int n_goal = 1, goal_level = 1;
    bool dense = false;
    const float * goal_action = nullptr;
    int cost_last_n = 1;
    float intermediate_cost_weight = 1.0f, action_cost_weight = 0.0f;
};

struct SolveOut {
    std::vector<float> actions, states;
    float cost = 0.0f;
    int iters = 0;
};

class DrawSource;

struct HPlanner {
    jepa_context * ctx = nullptr;
    float ln_eps = 1e-5f, adaln_eps = 1e-6f;
    std::vector<DLevel> levels;
    std::vector<void *> allocations;
    std::map<int, std::unique_ptr<Workspace>> ws;   // per (level, candidate stream): key level * 16 + stream
    long long launches = 0, ws_gen = 0;
    // A level's candidates run as `n` independent streams of consecutive rows, each with its own workspace,
    // captured as parallel branches of one graph: every kernel is latency-bound at a few hundred rows, so
    // two chains side by side fill the SMs one chain leaves idle. Rows never interact, so the result is
    // the same for any stream count.
    int n_streams = 0;                // 0 = automatic
    int force_mod_mode = 0;           // 0 automatic, 1 step at a time (recomputed), 2 forward kept, gradient per step
    std::vector<cudaStream_t> side;   // streams of the candidate streams 1..n-1
    std::vector<cudaEvent_t> ev;      // fork / join events of the captures

    ~HPlanner();
    bool build(const jepa_model & m);
    // chunk c of n_chunks candidate streams of one level (created in order; n_chunks sizes the memory decision)
    Workspace * workspace(int level, int S, int T, const CostSpec & cs, int chunk = 0, int n_chunks = 1);
    int streams_for(int S, int width) const;   // candidate chains for S candidates of a level of this predictor width
    bool ensure_streams(int n);
    // costs [S] and (optionally) grad [S][T][A] of host actions; all host buffers
    int plan_cost(const CostSpec & cs, const float * actions, int S, float * costs, float * grad);
    int solve(const CostSpec & cs, const jepa_hjepa_level_plan & lp, DrawSource & draws, SolveOut & out);

    // pieces
    int forward(Workspace & w, const CostSpec & cs, bool want_grad);
    int backward(Workspace & w, const CostSpec & cs);
    bool cost_tables(Workspace & w, const CostSpec & cs);
    // the multi-frame predictor: causal attention over T <= pred_n_frames frames of one sequence
    PredWs pred;
    // the level-1 projector of the encoder's CLS row and the proprio stream (jepa_hjepa_embed), on first use
    struct EmbedW {
        bool loaded = false;
        DLin proj0, proj2, pro0, pro2;
        float * proj_ln_w = nullptr, * proj_ln_b = nullptr, * pro_ln_w = nullptr, * pro_ln_b = nullptr;
    } emb;
    bool ensure_embed();
    DLin upload_plain(const std::string & name, int64_t row0, int64_t rows);   // f32 weight (+ bias) only
    float * upload_vec(const std::string & name);
    bool ensure_predict(int level);
    int predict_dev(int level, const float * states, const float * actions, int T, float * out, cudaStream_t st);
    int step_modulation(Workspace & w, int t0, int nt);       // mod of steps [t0, t0 + nt)
    int step_modulation_bwd(Workspace & w, int t0, int nt);   // dcs of steps [t0, t0 + nt) from dmod
    int pooled_chunks(const CostSpec & cs) const;     // Wa: chunks the action cost compares (0 = no action cost)
    int pool_forward(Workspace & w, bool want_grad);   // action cost, added to the costs
    int pool_backward(Workspace & w);                  // its gradient into pool.ge
    int lin_fwd(const DLin & L, const float * x, int ldx, const float * x_hi, const float * x_lo, int M, float * y, int ldy,
                float * y_hi, float * y_lo, Workspace & w);
    int lin_bwd(const DLin & L, const float * dy, int lddy, const float * dy_hi, const float * dy_lo, int M, float * dx, int lddx,
                Workspace & w);
};

// the context's H-JEPA planner, built on first use (weights on the device); null after logging
HPlanner * hplanner_of(jepa_context * ctx, const char * fn);

}  // namespace jb
