// H-JEPA gradient planner on the GPU (the reference's src/hjepa-plan.cpp, re-designed for B200).
//
// The reference evaluates candidates in chunks of 8 on host threads, one reverse-mode tape each
// (src/hjepa-plan.cpp:208-838). Here every candidate of a level is one row of one batch and a solve is:
//
//   per Adam iteration (captured once as a CUDA graph and replayed):
//     conditioning path, all T steps at once (R = T S rows): act_embed / pred.act_embed / cond_proj,
//       SiLU, and ONE tcgen05 GEMM for every block's adaLN modulation of every step  [R x 6 P L]
//     rollout, t = 0..T-1, per block: prologue (LN + FiLM + ln1) -> V GEMM -> out GEMM with the gated
//       residual in its epilogue -> prologue (LN + FiLM + ln2) -> up GEMM with GELU in its epilogue ->
//       down GEMM with the gated residual in its epilogue; final norm (+ projections)
//     cost: squared L2 of the scored states (after the upper levels' state encoders when the goal lives
//       above), with its gradient
//     backward sweep, t = T-1..0, the same structure reversed: transposed GEMMs against the same
//       weights with GELU' in the epilogue, fused LayerNorm / FiLM / gated-residual backward kernels
//       writing the adaLN gradient [R x 6 P L]
//     ONE GEMM for the gradient of every step's conditioning through every adaLN linear, SiLU', the
//       small conditioning linears backward, and the AdamW step + clamp on the actions
//   final forward without gradient, first-minimum candidate, its states.
//
// Rows are independent end to end (no reduction crosses candidates), so a candidate's result does not
// depend on the batch it is in, which is what makes candidate sharding across GPUs exact.
#include "hplan.h"
#include "upload.h"

#include <algorithm>
#include <cmath>
#include <cstring>

namespace jb {

// ---------------------------------------------------------------------------------------------
// weights
// ---------------------------------------------------------------------------------------------

// Every product of the planner's sweep multiplies by a weight (B never comes from the kernel before), and
// its epilogue reads only biases and operands written at least two kernels earlier (the modulation, the
// block's input, the forward pre-activations): both are loaded before the dependency wait.
// The planner's GEMM call: operands not produced by the previous kernel are loaded ahead of the dependency
// wait, and the workspace's fix-up scratch lets narrow, long products split their K range.
static int wgemm(const Workspace & w, const SplitMat & A, const SplitMat & B, int M, int N, int K, GemmEpi ep, cudaStream_t st) {
    ep.pre_b = 1;
    ep.pre_epi = 1;
    ep.fix = w.fix;
    ep.fix_floats = w.fix_floats;
    ep.fix_count = w.fix_count;
    ep.fix_counters = w.fix_counters;
    if (gemm_fixup_floats(M, N, K) > w.fix_floats || gemm_fixup_counters(M, N, K) > w.fix_counters) {
        log("jepa: hjepa planner: the workspace's GEMM scratch does not cover %d x %d x %d\n", M, N, K);
        return -1;
    }
    return gemm_tc(A, B, M, N, K, ep, st);
}

HPlanner::~HPlanner() {
    ws.clear();
    for (void * p : allocations) cudaFree(p);
    for (cudaStream_t s : side) cudaStreamDestroy(s);
    for (cudaEvent_t e : ev) cudaEventDestroy(e);
}

// Automatic chain count (measured on one B200): the narrow predictors, whose per-step products split K
// over clusters, run best in chains of about 256 candidates (up to four side by side); the wide ones
// (width >= 768, one CTA per 128 x 128 tile) in two chains once there are 512 candidates.
int HPlanner::streams_for(int S, int width) const {
    const int n = n_streams > 0 ? n_streams : width >= 768 ? (S >= 512 ? 2 : 1) : std::min(4, S / 256);
    return std::max(1, std::min({n, S, 8}));
}

bool HPlanner::ensure_streams(int n) {
    while ((int) side.size() < n - 1) {
        cudaStream_t s;
        JB_CUDA_B(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
        side.push_back(s);
    }
    while ((int) ev.size() < 2 * n) {
        cudaEvent_t e;
        JB_CUDA_B(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        ev.push_back(e);
    }
    return true;
}

Workspace::~Workspace() {
    if (g_iter) cudaGraphExecDestroy(g_iter);
    if (g_fwd) cudaGraphExecDestroy(g_fwd);
}

DLin HPlanner::upload_plain(const std::string & name, int64_t row0, int64_t rows) {
    Uploader up{allocations, *ctx->model, ctx->stream};
    DLin L = up.lin_plain(name, row0, rows);
    return up.ok ? L : DLin();
}

float * HPlanner::upload_vec(const std::string & name) {
    Uploader up{allocations, *ctx->model, ctx->stream};
    float * v = up.vec(name);
    return up.ok ? v : nullptr;
}

// the multi-frame predictor's extra weights (the query / key rows of every block, every position row), and
// its buffers, on first use
bool HPlanner::ensure_predict(int level) {
    DLevel & L = levels[(size_t) level - 1];
    if (!L.pos_all) {
        Uploader up{allocations, *ctx->model, ctx->stream};
        const std::string p = "lvl." + std::to_string(level) + ".";
        L.pos_all = up.vec(p + "pred.pos_embed");
        for (int i = 0; i < L.L && up.ok; i++)
            L.blocks[(size_t) i].qk = up.lin_plain(p + "pred.blk." + std::to_string(i) + ".attn_qkv", 0, 2 * (int64_t) L.I);
        if (!up.ok || !L.pos_all) { L.pos_all = nullptr; log("jepa: hjepa predictor: could not place its weights on the device\n"); return false; }
    }
    int rows = 1, heads = 1;
    size_t width = 1;
    for (const DLevel & V : levels) {
        rows = std::max(rows, V.hp.pred_n_frames);
        heads = std::max(heads, V.hp.pred_n_head);
        width = std::max({width, (size_t) V.D, (size_t) V.P, (size_t) V.F, (size_t) 3 * V.I, (size_t) 6 * V.P,
                          (size_t) V.A, (size_t) V.E, (size_t) V.C});
        for (const DLin * l : {&V.act0, &V.pact0, &V.proj0, &V.out_proj}) if (*l) width = std::max(width, (size_t) l->out);
    }
    if (pred.rows >= rows && pred.width >= width && pred.heads >= heads) return true;
    ArenaPlan ap;
    for (int i = 0; i < 18; i++) ap.add<float>((size_t) rows * width);
    ap.add<float>((size_t) rows * rows * heads);   // attention probabilities [T][heads][T]
    ap.add<LnStats>((size_t) rows); ap.add<LnStats>((size_t) rows);
    if (!pred.arena.reserve(ap.bytes + 4096, ctx->device)) return false;
    float ** bufs[] = {&pred.xa, &pred.x, &pred.xm, &pred.c, &pred.cc, &pred.cs, &pred.t1, &pred.t2, &pred.mod,
                       &pred.hhi, &pred.hlo, &pred.qkv, &pred.o, &pred.a, &pred.u, &pred.g, &pred.y};
    for (float ** b : bufs) *b = pred.arena.take<float>((size_t) rows * width);
    (void) pred.arena.take<float>((size_t) rows * width);
    pred.probs = pred.arena.take<float>((size_t) rows * rows * heads);
    pred.st0 = pred.arena.take<LnStats>((size_t) rows);
    pred.st1 = pred.arena.take<LnStats>((size_t) rows);
    pred.rows = rows;
    pred.width = width;
    pred.heads = heads;
    return pred.st1 != nullptr;
}

bool HPlanner::build(const jepa_model & m) {
    cudaSetDevice(ctx->device);
    Uploader up{allocations, m, ctx->stream};
    ln_eps = m.hj.ln_eps;
    adaln_eps = m.hj.adaln_eps;
    for (size_t li = 0; li < m.hj.levels.size(); li++) {
        DLevel L;
        L.hp = m.hj.levels[li];
        const std::string p = "lvl." + std::to_string(li + 1) + ".";
        L.D = L.hp.embed_dim;
        L.P = L.hp.pred_dim;
        L.F = L.hp.pred_ffn_dim;
        L.I = L.hp.pred_n_head * L.hp.pred_head_dim;
        L.L = L.hp.pred_n_layer;
        L.A = L.hp.action_dim;
        L.E = L.hp.act_embed_dim;
        L.pos0 = up.vec(p + "pred.pos_embed", 0, L.D);
        L.act0 = up.lin(p + "act_embed.0");
        L.act2 = up.lin(p + "act_embed.2");
        L.pact0 = up.lin(p + "pred.act_embed.0");
        L.pact2 = up.lin(p + "pred.act_embed.2");
        L.in_proj = up.lin(p + "pred.in_proj");
        L.cond_proj = up.lin(p + "pred.cond_proj");
        L.out_proj = up.lin(p + "pred.out_proj");
        L.proj0 = up.lin(p + "pred.proj.0");
        L.proj2 = up.lin(p + "pred.proj.2");
        L.C = L.pact2 ? L.pact2.out : L.E;
        L.norm_w = up.vec(p + "pred.norm.weight");
        L.norm_b = up.vec(p + "pred.norm.bias");
        // every block's adaLN weight stacked into one [6 P L][P] operand
        L.adaln.in = L.P;
        L.adaln.out = 6 * L.P * L.L;
        L.adaln.w = up.alloc<float>((size_t) L.adaln.in * L.adaln.out);
        L.adaln.b = up.alloc<float>((size_t) L.adaln.out);
        if (L.adaln.b) cudaMemsetAsync(L.adaln.b, 0, (size_t) L.adaln.out * 4, ctx->stream);
        for (int i = 0; i < L.L && up.ok; i++) {
            const std::string q = p + "pred.blk." + std::to_string(i) + ".";
            DBlock B;
            B.v = up.lin(q + "attn_qkv", 2 * (int64_t) L.I, L.I);   // the value third: one query over one key (hjepa-plan.cpp:170-171)
            B.out = up.lin(q + "attn_out");
            B.ov = up.compose(B.v, B.out);
            B.up = up.lin(q + "ffn_up");
            B.down = up.lin(q + "ffn_down");
            B.ln1_w = up.vec(q + "ln1.weight"); B.ln1_b = up.vec(q + "ln1.bias");
            B.ln2_w = up.vec(q + "ln2.weight"); B.ln2_b = up.vec(q + "ln2.bias");
            const gguf_tensor * aw = m.get(q + "adaln.weight");
            up.dequant_into(aw, 0, 6 * (int64_t) L.P, L.adaln.w + (size_t) i * 6 * L.P * L.P);
            if (m.get(q + "adaln.bias")) {
                float * b = up.vec(q + "adaln.bias");
                if (b) cudaMemcpyAsync(L.adaln.b + (size_t) i * 6 * L.P, b, (size_t) 6 * L.P * 4, cudaMemcpyDeviceToDevice, ctx->stream);
            }
            L.blocks.push_back(B);
        }
        up.finish(L.adaln);
        L.enc_in_w = up.vec(p + "enc.in_norm.weight"); L.enc_in_b = up.vec(p + "enc.in_norm.bias");
        L.enc_out_w = up.vec(p + "enc.out_norm.weight"); L.enc_out_b = up.vec(p + "enc.out_norm.bias");
        L.enc_fc1 = up.lin(p + "enc.fc1");
        L.enc_fc2 = up.lin(p + "enc.fc2");
        // the action encoder (levels above the first; weights as the reference loads them, hjepa-plan.cpp:183-200)
        DActEnc & ae = L.ae;
        if (li > 0 && L.hp.act_enc_kind == "mlp") {
            ae.kind = 1;
            ae.fc1 = up.lin(p + "act_enc.fc1");
            ae.fc2 = up.lin(p + "act_enc.fc2");
        } else if (li > 0 && L.hp.act_enc_kind == "seq") {
            ae.kind = 2;
            ae.d = L.hp.act_enc_dim;
            ae.n_head = L.hp.act_enc_n_head;
            ae.step = up.lin(p + "act_enc.step");
            ae.pos = up.vec(p + "act_enc.pos");
            if (const gguf_tensor * t = m.get(p + "act_enc.pos")) ae.pos_n = t->nelements();
            for (int i = 0; i < L.hp.act_enc_n_layer && up.ok; i++) {
                const std::string q = p + "act_enc.blk." + std::to_string(i) + ".";
                DSeqBlock B;
                B.qkv = up.lin(q + "attn_qkv");
                B.out = up.lin(q + "attn_out");
                B.up = up.lin(q + "ffn_up");
                B.down = up.lin(q + "ffn_down");
                B.ln1_w = up.vec(q + "ln1.weight"); B.ln1_b = up.vec(q + "ln1.bias");
                B.ln2_w = up.vec(q + "ln2.weight"); B.ln2_b = up.vec(q + "ln2.bias");
                ae.blocks.push_back(B);
            }
            ae.head0 = up.lin(p + "act_enc.head.0");
            ae.head2 = up.lin(p + "act_enc.head.2");
            ae.headln_w = up.vec(p + "act_enc.head.ln.weight"); ae.headln_b = up.vec(p + "act_enc.head.ln.bias");
        }
        if (ae.kind) { ae.out_w = up.vec(p + "act_enc.out_norm.weight"); ae.out_b = up.vec(p + "act_enc.out_norm.bias"); }
        if (const gguf_tensor * q = m.get(p + "act_queue")) {
            L.queue.resize((size_t) q->nelements());
            dequant_row(q->type, q->data, L.queue.data(), q->nelements());
        }
        levels.push_back(std::move(L));
        if (!up.ok) break;
    }
    if (!up.ok) return false;
    return cuda_ok(cudaStreamSynchronize(ctx->stream), "planner weights");
}

// ---------------------------------------------------------------------------------------------
// workspace
// ---------------------------------------------------------------------------------------------
Workspace * HPlanner::workspace(int level, int S, int T, const CostSpec & cs, int chunk, int n_chunks) {
    const int Wa = pooled_chunks(cs);
    const std::string key = std::to_string(S) + "/" + std::to_string(T) + "/" + std::to_string(cs.goal_level) + "/" +
                            std::to_string(cs.dense) + "/" + std::to_string(cs.n_goal) + "/" + std::to_string(cs.cost_last_n) +
                            "/" + std::to_string(Wa);
    const int slot = level * 16 + chunk;
    if (chunk > 0 && !ensure_streams(chunk + 1)) return nullptr;
    auto it = ws.find(slot);
    if (it != ws.end() && it->second->graph_key == key) return it->second.get();
    ws.erase(slot);
    const DLevel & L = levels[(size_t) level - 1];
    const int D = L.D, P = L.P, F = L.F, I = L.I, NL = L.L, A = L.A;
    const size_t R = (size_t) T * S, ldm = (size_t) 6 * P * NL;
    auto w = std::make_unique<Workspace>();
    w->level = level; w->S = S; w->T = T; w->graph_key = key;
    w->gen = ++ws_gen;
    w->st = chunk == 0 ? ctx->stream : side[(size_t) chunk - 1];
    // encoder chain plan (goal above the planned level)
    std::vector<int> list;
    for (int t = 0; t <= T; t++) list.push_back(t);
    for (int lv = level + 1; lv <= cs.goal_level; lv++) {
        const int stride = cs.dense ? 1 : levels[(size_t) lv - 1].hp.stride;
        EncStage e;
        e.lv = lv;
        std::vector<int> keep;
        for (size_t i = 0; i < list.size(); i += (size_t) stride) keep.push_back((int) i);
        for (size_t j = 1; j < keep.size(); j++) e.src_pos.push_back(keep[j]);   // list position (0 = context state)
        e.n = (int) e.src_pos.size();
        list.assign(keep.size(), 0);
        w->enc.push_back(e);
    }
    int maxw = std::max({P, D, A, L.E, L.C, I});
    for (const DLin * l : {&L.act0, &L.pact0, &L.proj0}) if (*l) maxw = std::max(maxw, l->out);
    for (const EncStage & e : w->enc) {
        const DLevel & U = levels[(size_t) e.lv - 1];
        maxw = std::max({maxw, U.D, levels[(size_t) e.lv - 2].D, U.enc_fc1 ? U.enc_fc1.out : 0});
    }
    // action cost: the upper level's action encoder over the last Wa whole chunks
    PoolWs & pw = w->pool;
    const DActEnc * ae = Wa > 0 ? &levels[(size_t) level].ae : nullptr;
    const int Ein = L.act0 ? L.E : A, Au = Wa > 0 ? levels[(size_t) level].A : 0;
    size_t pool_scr = 0;
    if (ae) {
        pw.Wa = Wa;
        pw.stride = levels[(size_t) level].hp.stride;
        pw.c0 = T / pw.stride - Wa;
        pw.G = pw.stride + 1;
        const size_t n = (size_t) Wa * S, nG = n * (size_t) pw.G;
        const int NB = (int) ae->blocks.size();
        pw.xs.assign((size_t) NB + 1, nullptr);
        pw.qkv.assign((size_t) NB, nullptr); pw.probs.assign((size_t) NB, nullptr);
        pw.xmid.assign((size_t) NB, nullptr); pw.u.assign((size_t) NB, nullptr);
        int wide = std::max({Au, pw.stride * Ein});
        if (ae->kind == 1) wide = std::max(wide, ae->fc1.out);
        if (ae->kind == 2) {
            wide = std::max({wide, ae->head0.out, pw.stride * ae->d});
            int f = 3 * ae->d;
            for (const DSeqBlock & B : ae->blocks) f = std::max(f, B.up.out);
            pool_scr = nG * (size_t) f;
            if (!group_mha_prepare(pw.G, ae->d, ae->n_head)) {
                log("jepa: hjepa planner: a %d-token action-encoder group of width %d does not fit one CTA's shared memory\n", pw.G, ae->d);
                return nullptr;
            }
        }
        pool_scr = std::max(pool_scr, n * (size_t) wide);
    }
    // GEMM fix-up scratch: the largest any product of this workspace can ask for, at the largest row count it
    // runs (every step at once, the goal-projection encoders, the pooled action chunks)
    {
        const size_t rows = std::max({R + (size_t) S, ae ? (size_t) Wa * S * (size_t) pw.G : 0,
                                      ae ? (size_t) Wa * S * (size_t) pw.stride : 0});
        const int M_cap = (int) std::min<size_t>(rows, (size_t) INT32_MAX);
        auto cover = [&](int n_out, int n_in) {
            w->fix_floats = std::max({w->fix_floats, gemm_fixup_floats(M_cap, n_out, n_in), gemm_fixup_floats(M_cap, n_in, n_out)});
            w->fix_counters = std::max({w->fix_counters, gemm_fixup_counters(M_cap, n_out, n_in),
                                        gemm_fixup_counters(M_cap, n_in, n_out)});
        };
        auto cover_lin = [&](const DLin & l) { if (l) cover(l.out, l.in); };
        cover((int) ldm, P);
        for (const DLin * l : {&L.act0, &L.act2, &L.pact0, &L.pact2, &L.in_proj, &L.cond_proj, &L.out_proj, &L.proj0, &L.proj2})
            cover_lin(*l);
        for (const DBlock & B : L.blocks) { cover_lin(B.ov); cover_lin(B.up); cover_lin(B.down); }
        for (const EncStage & e : w->enc) {
            const DLevel & U = levels[(size_t) e.lv - 1];
            cover_lin(U.enc_fc1);
            cover_lin(U.enc_fc2);
        }
        if (ae) {
            for (const DLin * l : {&ae->fc1, &ae->fc2, &ae->step, &ae->head0, &ae->head2}) cover_lin(*l);
            for (const DSeqBlock & B : ae->blocks) { cover_lin(B.qkv); cover_lin(B.out); cover_lin(B.up); cover_lin(B.down); }
        }
    }
    ArenaPlan ap;
    // rows of mod and of dmod: every step's (R), or one step's (S) in the step-at-a-time modes (mod keeps R
    // rows when the forward modulation is kept)
    size_t mod_rows = R, dmod_rows = R;
    auto plan_all = [&](auto && add) {
        add((float **) &w->x, (size_t) S * T * A); add(&w->m, (size_t) S * T * A); add(&w->v, (size_t) S * T * A);
        add(&w->grad, (size_t) S * T * A); add(&w->a_all, R * A); add(&w->da_all, R * A);
        add(&w->lo, (size_t) A); add(&w->hi, (size_t) A);
        if (L.act0) { add(&w->ae_u, R * L.act0.out); add(&w->ae_s, R * L.act0.out); add(&w->e, R * L.E); }
        if (L.pact0) { add(&w->pa_u, R * L.pact0.out); add(&w->pa_s, R * L.pact0.out); add(&w->c0, R * L.C); }
        add(&w->cpre, R * P); add(&w->cs_hi, R * P); add(&w->cs_lo, R * P);
        add(&w->mod, mod_rows * ldm); add(&w->dmod_hi, dmod_rows * ldm); add(&w->dmod_lo, dmod_rows * ldm);
        add(&w->dcs, R * P); add(&w->dc, R * P); add(&w->tmpR, R * maxw); add(&w->tmpR2, R * maxw);
        add(&w->states, (size_t) (T + 1) * S * D); add(&w->gstate, (size_t) (T + 1) * S * D);
        add(&w->xs, (size_t) T * (NL + 1) * S * P);
        add(&w->xmid, (size_t) T * NL * S * P); add(&w->o, (size_t) T * NL * S * P); add(&w->dn, (size_t) T * NL * S * P);
        add(&w->u, (size_t) T * NL * S * F);
        if (L.out_proj || L.proj0) add(&w->yn, (size_t) T * S * P);
        if (L.out_proj && L.proj0) add(&w->yo, (size_t) T * S * L.out_proj.out);
        if (L.proj0) add(&w->pu, (size_t) T * S * L.proj0.out);
        const size_t sw = (size_t) S * std::max({P, F, I, D, maxw});
        add(&w->h_hi, sw); add(&w->h_lo, sw); add(&w->v_hi, sw); add(&w->v_lo, sw); add(&w->g_hi, sw); add(&w->g_lo, sw);
        add(&w->gx, sw); add(&w->gmid, sw); add(&w->gh, sw); add(&w->d_hi, sw); add(&w->d_lo, sw);
        add(&w->du_hi, sw); add(&w->du_lo, sw); add(&w->dv_hi, sw); add(&w->dv_lo, sw);
        add(&w->gtmp, sw); add(&w->gtmp2, sw);
        add(&w->sp_hi, std::max({sw, R * maxw, pool_scr})); add(&w->sp_lo, std::max({sw, R * maxw, pool_scr}));
        if (ae) {
            const size_t n = (size_t) Wa * S, nG = n * (size_t) pw.G;
            if (ae->kind == 1) {
                add(&pw.x, n * ae->fc1.in); add(&pw.h, n * ae->fc1.out); add(&pw.r, n * ae->fc1.out);
                if (ae->out_w) add(&pw.ypre, n * Au);
            } else {
                const int d = ae->d, H = ae->n_head;
                int fmax = 1;
                add(&pw.x, n * pw.stride * d);
                for (size_t b = 0; b < ae->blocks.size(); b++) {
                    const int f = ae->blocks[b].up.out;
                    fmax = std::max(fmax, f);
                    add(&pw.xs[b], nG * d); add(&pw.qkv[b], nG * 3 * d); add(&pw.probs[b], nG * H * pw.G);
                    add(&pw.xmid[b], nG * d); add(&pw.u[b], nG * f);
                }
                add(&pw.xs.back(), nG * d);
                add(&pw.h, nG * d); add(&pw.r, nG * fmax);
                add(&pw.z, n * ae->head0.out); add(&pw.zg, n * ae->head0.out); add(&pw.zl, n * ae->head0.out);
                add(&pw.ypre, n * Au);
            }
            add(&pw.y, n * Au); add(&pw.gy, n * Au);
            add(&pw.ga, pool_scr); add(&pw.gb, pool_scr); add(&pw.gc, pool_scr);
            add(&pw.ge, R * Ein);
            add(&pw.goals, (size_t) Wa * Au); add(&pw.weights, (size_t) Wa);
        }
        add(&w->cost, (size_t) S); add(&w->best_val, (size_t) 1);
        if (w->fix_floats) add(&w->fix, w->fix_floats);
        const int Dg = levels[(size_t) cs.goal_level - 1].D;
        // one goal row per scored prediction (W <= T + 1 of them; a single goal is repeated)
        add(&w->goals, (size_t) (T + 1) * Dg); add(&w->weights, (size_t) (T + 1));
        for (EncStage & e : w->enc) {
            const DLevel & U = levels[(size_t) e.lv - 1];
            const int Din = levels[(size_t) e.lv - 2].D, Dout = U.D;
            const int H = U.enc_fc1 ? U.enc_fc1.out : Din;
            const size_t n = (size_t) e.n * S;
            add(&e.in, n * Din); add(&e.h_hi, n * Din); add(&e.h_lo, n * Din); add(&e.u, n * H);
            add(&e.g_hi, n * H); add(&e.g_lo, n * H); add(&e.y, n * Dout); add(&e.out, n * Dout);
            add(&e.gout, n * Dout); add(&e.gy, n * std::max(Din, Dout)); add(&e.gin, n * std::max(Din, H));
            add(&e.d_hi, n * std::max(Dout, H)); add(&e.d_lo, n * std::max(Dout, H));
        }
    };
    auto count = [&](auto ** p, size_t n) { (void) p; ap.add<float>(n); };
    auto plan_total = [&]() -> size_t {   // bytes of the whole carve, in the order it is carved below
        ap = ArenaPlan();
        plan_all(count);
        ap.add<LnStats>((size_t) T * NL * S * 4 + (size_t) T * S);
        for (size_t i = 0; i < w->enc.size(); i++) ap.add<LnStats>((size_t) w->enc[i].n * S * 2);
        ap.add<float>((size_t) 2 * 4096);      // Adam schedule
        ap.add<int>(4);
        ap.add<int>(w->fix_counters);
        ap.add<void *>((size_t) 2 * (T + 1));  // cost pointer tables
        if (ae) {
            const size_t n = (size_t) Wa * S;
            ap.add<LnStats>(n);
            if (ae->kind == 2) {
                ap.add<LnStats>(n);
                for (size_t b = 0; b < 2 * ae->blocks.size(); b++) ap.add<LnStats>(n * (size_t) pw.G);
            }
            ap.add<void *>((size_t) Wa); ap.add<void *>((size_t) Wa);
        }
        return ap.bytes + 65536;
    };
    auto evict_other_levels = [&]() {   // a solve uses one level's workspaces at a time
        for (auto e = ws.begin(); e != ws.end();) e = e->first / 16 != level ? ws.erase(e) : std::next(e);
    };
    auto to_step_mod = [&](bool keep) {
        w->step_mod = true;
        w->keep_mod = keep;
        mod_rows = keep ? R : (size_t) S;
        dmod_rows = (size_t) S;
        return plan_total();
    };
    // Three memory modes, the first that fits this workspace and the ones of the level's candidate streams
    // still to be planned (about the same size each): every step's modulation and its gradient (one GEMM
    // each way); every step's modulation kept and the gradient folded per step; one step at a time (the
    // modulation recomputed in the backward). Other levels' cached workspaces are released first when
    // memory is short.
    const size_t left = (size_t) std::max(1, n_chunks - chunk);
    size_t need = plan_total();
    size_t free_b = 0, total_b = 0;
    cudaMemGetInfo(&free_b, &total_b);
    auto fits = [&](size_t n) { return n * left <= free_b / 10 * 9; };
    if (!fits(need)) {
        evict_other_levels();
        cudaMemGetInfo(&free_b, &total_b);
    }
    if (T > 1) {
        if (force_mod_mode == 1) need = to_step_mod(false);
        else if (force_mod_mode == 2) need = to_step_mod(true);
        else if (!fits(need)) {
            need = to_step_mod(true);
            if (!fits(need)) need = to_step_mod(false);
        }
    }
    bool got = w->arena.reserve(need, ctx->device);
    if (!got) {   // the free figure is not one allocatable block: release, then fall back to leaner modes
        evict_other_levels();
        got = w->arena.reserve(need, ctx->device);
        if (!got && T > 1 && !w->step_mod) got = w->arena.reserve(to_step_mod(true), ctx->device);
        if (!got && T > 1 && w->keep_mod) got = w->arena.reserve(to_step_mod(false), ctx->device);
    }
    if (!got) return nullptr;
    auto take = [&](auto ** p, size_t n) { *p = (std::remove_pointer_t<decltype(p)>) w->arena.take<float>(n); };
    plan_all(take);
    w->sta0 = w->arena.take<LnStats>((size_t) T * NL * S);
    w->sta1 = w->arena.take<LnStats>((size_t) T * NL * S);
    w->stm0 = w->arena.take<LnStats>((size_t) T * NL * S);
    w->stm1 = w->arena.take<LnStats>((size_t) T * NL * S);
    w->stn = w->arena.take<LnStats>((size_t) T * S);
    for (EncStage & e : w->enc) {
        e.st1 = w->arena.take<LnStats>((size_t) e.n * S);
        e.st2 = w->arena.take<LnStats>((size_t) e.n * S);
    }
    w->sched = w->arena.take<float>((size_t) 2 * 4096);
    w->step_ctr = w->arena.take<int>(4);
    if (w->fix_counters) {
        w->fix_count = w->arena.take<int>(w->fix_counters);
        if (!w->fix_count || !cuda_ok(cudaMemset(w->fix_count, 0, w->fix_counters * sizeof(int)), "GEMM fix-up counters")) return nullptr;
    }
    w->pred_ptrs = (const float **) w->arena.take<void *>((size_t) (T + 1));
    w->gpred_ptrs = (float **) w->arena.take<void *>((size_t) (T + 1));
    w->best_idx = w->arena.take<int>(1);
    if (ae) {
        const size_t n = (size_t) Wa * S, nG = n * (size_t) pw.G;
        pw.sto = w->arena.take<LnStats>(n);
        if (ae->kind == 2) {
            pw.sth = w->arena.take<LnStats>(n);
            pw.st1.assign(ae->blocks.size(), nullptr);
            pw.st2.assign(ae->blocks.size(), nullptr);
            for (size_t b = 0; b < ae->blocks.size(); b++) {
                pw.st1[b] = w->arena.take<LnStats>(nG);
                pw.st2[b] = w->arena.take<LnStats>(nG);
            }
        }
        pw.ptrs = (const float **) w->arena.take<void *>((size_t) Wa);
        pw.gptrs = (float **) w->arena.take<void *>((size_t) Wa);
        if (!pw.gptrs) { log("jepa: hjepa planner: workspace carve failed\n"); return nullptr; }
    }
    if (!w->pred_ptrs || !w->best_idx) { log("jepa: hjepa planner: workspace carve failed\n"); return nullptr; }
    Workspace * raw = w.get();
    ws[slot] = std::move(w);
    return raw;
}

// ---------------------------------------------------------------------------------------------
// linears: tensor cores when the shape allows, SIMT otherwise
// ---------------------------------------------------------------------------------------------
int HPlanner::lin_fwd(const DLin & L, const float * x, int ldx, const float * x_hi, const float * x_lo, int M, float * y, int ldy,
                      float * y_hi, float * y_lo, Workspace & w) {
    cudaStream_t st = w.st;
    if (L.tc_fwd()) {
        int ld = ldx;
        if (!x_hi) {
            split_f32(x, ldx, w.sp_hi, w.sp_lo, L.in, M, L.in, st);
            x_hi = w.sp_hi; x_lo = w.sp_lo; ld = L.in;
            launches++;
        }
        GemmEpi ep;
        ep.bias = L.b;
        ep.out0 = y; ep.ld0 = ldy;
        ep.out_hi = y_hi; ep.out_lo = y_lo; ep.ld_split = ldy;
        ep.mode = y_hi ? (y ? EPI_F32_SPLIT : EPI_SPLIT) : EPI_F32;
        launches++;
        return wgemm(w, {x_hi, x_lo, ld}, L.fwd(), M, L.out, L.in, ep, st);
    }
    linear_simt(x, ldx, L.w, L.b, y, ldy, M, L.out, L.in, st);
    launches++;
    if (y_hi) { split_f32(y, ldy, y_hi, y_lo, ldy, M, L.out, st); launches++; }
    return 0;
}

int HPlanner::lin_bwd(const DLin & L, const float * dy, int lddy, const float * dy_hi, const float * dy_lo, int M, float * dx,
                      int lddx, Workspace & w) {
    cudaStream_t st = w.st;
    if (L.tc_bwd()) {
        int ld = lddy;
        if (!dy_hi) {
            split_f32(dy, lddy, w.sp_hi, w.sp_lo, L.out, M, L.out, st);
            dy_hi = w.sp_hi; dy_lo = w.sp_lo; ld = L.out;
            launches++;
        }
        GemmEpi ep;
        ep.out0 = dx; ep.ld0 = lddx;
        launches++;
        return wgemm(w, {dy_hi, dy_lo, ld}, L.bwd(), M, L.in, L.out, ep, st);
    }
    linear_simt(dy, lddy, L.wt, nullptr, dx, lddx, M, L.in, L.out, st);
    launches++;
    return 0;
}

// ---------------------------------------------------------------------------------------------
// the adaLN modulation of steps [t0, t0 + nt): mod = adaln(silu(c)) for their rows, and its backward
// dcs = dmod adaln.W for the same rows (every step at once, or one step at a time: mod / dmod then hold
// one step's rows)
// ---------------------------------------------------------------------------------------------
static size_t mod_row0(const Workspace & w, int t) { return (w.step_mod && !w.keep_mod) ? 0 : (size_t) t * w.S; }
static size_t dmod_row0(const Workspace & w, int t) { return w.step_mod ? 0 : (size_t) t * w.S; }

int HPlanner::step_modulation(Workspace & w, int t0, int nt) {
    const DLevel & L = levels[(size_t) w.level - 1];
    const int P = L.P, ldm = 6 * P * L.L;
    GemmEpi ep;
    ep.bias = L.adaln.b;
    ep.out0 = w.mod + mod_row0(w, t0) * ldm; ep.ld0 = ldm;
    launches++;
    const size_t r0 = (size_t) t0 * w.S * P;
    return wgemm(w, {w.cs_hi + r0, w.cs_lo + r0, P}, L.adaln.fwd(), nt * w.S, ldm, P, ep, w.st);
}

int HPlanner::step_modulation_bwd(Workspace & w, int t0, int nt) {
    const DLevel & L = levels[(size_t) w.level - 1];
    const int P = L.P, ldm = 6 * P * L.L;
    GemmEpi ep;
    ep.out0 = w.dcs + (size_t) t0 * w.S * P; ep.ld0 = P;
    launches++;
    const size_t m0 = dmod_row0(w, t0) * ldm;
    return wgemm(w, {w.dmod_hi + m0, w.dmod_lo + m0, ldm}, L.adaln.bwd(), nt * w.S, P, ldm, ep, w.st);
}

// ---------------------------------------------------------------------------------------------
// forward: conditioning, adaLN modulation, rollout, cost
// ---------------------------------------------------------------------------------------------
int HPlanner::forward(Workspace & w, const CostSpec & cs, bool want_grad) {
    cudaStream_t st = w.st;
    const DLevel & L = levels[(size_t) w.level - 1];
    const int S = w.S, T = w.T, D = L.D, P = L.P, F = L.F, NL = L.L, A = L.A;
    const int R = S * T, ldm = 6 * P * NL;
    // ---- conditioning path over every step at once
    const float * cur = w.a_all;
    int cw = A;
    if (L.act0) {
        if (lin_fwd(L.act0, cur, cw, nullptr, nullptr, R, w.ae_u, L.act0.out, nullptr, nullptr, w)) return -1;
        act_fwd(w.ae_u, L.act0.out, w.ae_s, L.act0.out, R, L.act0.out, 2, st); launches++;
        if (lin_fwd(L.act2, w.ae_s, L.act0.out, nullptr, nullptr, R, w.e, L.E, nullptr, nullptr, w)) return -1;
        cur = w.e; cw = L.E;
    }
    if (L.pact0) {
        if (lin_fwd(L.pact0, cur, cw, nullptr, nullptr, R, w.pa_u, L.pact0.out, nullptr, nullptr, w)) return -1;
        act_fwd(w.pa_u, L.pact0.out, w.pa_s, L.pact0.out, R, L.pact0.out, 2, st); launches++;
        if (lin_fwd(L.pact2, w.pa_s, L.pact0.out, nullptr, nullptr, R, w.c0, L.C, nullptr, nullptr, w)) return -1;
        cur = w.c0; cw = L.C;
    }
    if (L.cond_proj) {
        if (lin_fwd(L.cond_proj, cur, cw, nullptr, nullptr, R, w.cpre, P, nullptr, nullptr, w)) return -1;
    } else {
        copy_rows(cur, cw, w.cpre, P, R, P, st); launches++;
    }
    act_fwd(w.cpre, P, w.tmpR, P, R, P, 2, st); launches++;
    split_f32(w.tmpR, P, w.cs_hi, w.cs_lo, P, R, P, st); launches++;
    if ((!w.step_mod || w.keep_mod) && step_modulation(w, 0, T)) return -1;
    // ---- rollout
    for (int t = 0; t < T; t++) {
        const float * s_t = w.states + (size_t) t * S * D;
        float * x0 = w.xs + (size_t) t * (NL + 1) * S * P;
        // (step-at-a-time modulation: step t's, at least one kernel ahead of its first reader)
        if (w.step_mod && !w.keep_mod && step_modulation(w, t, 1)) return -1;
        if (L.in_proj) {
            add_row_vec(s_t, D, L.pos0, w.gtmp, D, S, D, st); launches++;
            if (lin_fwd(L.in_proj, w.gtmp, D, nullptr, nullptr, S, x0, P, nullptr, nullptr, w)) return -1;
        } else {
            add_row_vec(s_t, D, L.pos0, x0, P, S, D, st); launches++;
        }
        for (int l = 0; l < NL; l++) {
            const DBlock & B = L.blocks[(size_t) l];
            const float * mod_l = w.mod + mod_row0(w, t) * ldm + (size_t) l * 6 * P;
            float * xin = x0 + (size_t) l * S * P;
            float * xout = xin + (size_t) S * P;
            const size_t tl = (size_t) t * NL + l;
            float * xm = w.xmid + tl * S * P, * o = w.o + tl * S * P, * dn = w.dn + tl * S * P, * u = w.u + tl * S * F;
            block_pre(xin, P, mod_l, ldm, 0, P, B.ln1_w, B.ln1_b, adaln_eps, ln_eps, w.h_hi, w.h_lo, P,
                      w.sta0 + tl * S, w.sta1 + tl * S, S, P, st);
            // attention half: o = out(V(h)) through the composed linear, xm = xin + gate * o
            GemmEpi e2;
            e2.mode = EPI_GATED; e2.bias = B.ov.b; e2.out0 = o; e2.ld0 = P; e2.aux = xin; e2.ld_aux = P;
            e2.gate = mod_l + 2 * P; e2.ld_gate = ldm; e2.out1 = xm; e2.ld1 = P;
            if (wgemm(w, {w.h_hi, w.h_lo, P}, B.ov.fwd(), S, P, P, e2, st)) return -1;
            block_pre(xm, P, mod_l, ldm, 3 * P, 4 * P, B.ln2_w, B.ln2_b, adaln_eps, ln_eps, w.h_hi, w.h_lo, P,
                      w.stm0 + tl * S, w.stm1 + tl * S, S, P, st);
            GemmEpi e3;
            // (u keeps gelu'(pre-activation) for the backward's EPI_MUL_SPLIT)
            e3.mode = EPI_GELU_D_SPLIT; e3.bias = B.up.b; e3.out0 = u; e3.ld0 = F; e3.out_hi = w.g_hi; e3.out_lo = w.g_lo; e3.ld_split = F;
            if (wgemm(w, {w.h_hi, w.h_lo, P}, B.up.fwd(), S, F, P, e3, st)) return -1;
            GemmEpi e4;
            e4.mode = EPI_GATED; e4.bias = B.down.b; e4.out0 = dn; e4.ld0 = P; e4.aux = xm; e4.ld_aux = P;
            e4.gate = mod_l + 5 * P; e4.ld_gate = ldm; e4.out1 = xout; e4.ld1 = P;
            if (wgemm(w, {w.g_hi, w.g_lo, F}, B.down.fwd(), S, P, F, e4, st)) return -1;
            launches += 5;
        }
        const float * xL = x0 + (size_t) NL * S * P;
        float * s_next = w.states + (size_t) (t + 1) * S * D;
        if (!L.out_proj && !L.proj0) {
            layer_norm(xL, P, L.norm_w, L.norm_b, ln_eps, s_next, D, nullptr, nullptr, w.stn + (size_t) t * S, S, P, st);
            launches++;
        } else {
            float * yn = w.yn + (size_t) t * S * P;
            layer_norm(xL, P, L.norm_w, L.norm_b, ln_eps, yn, P, nullptr, nullptr, w.stn + (size_t) t * S, S, P, st);
            launches++;
            const float * c = yn;
            int cwid = P;
            if (L.out_proj) {
                float * dst = L.proj0 ? w.yo + (size_t) t * S * L.out_proj.out : s_next;
                if (lin_fwd(L.out_proj, c, cwid, nullptr, nullptr, S, dst, L.out_proj.out, nullptr, nullptr, w)) return -1;
                c = dst; cwid = L.out_proj.out;
            }
            if (L.proj0) {
                float * pu = w.pu + (size_t) t * S * L.proj0.out;
                if (lin_fwd(L.proj0, c, cwid, nullptr, nullptr, S, pu, L.proj0.out, nullptr, nullptr, w)) return -1;
                act_fwd(pu, L.proj0.out, w.gtmp, L.proj0.out, S, L.proj0.out, 0, st); launches++;
                if (lin_fwd(L.proj2, w.gtmp, L.proj0.out, nullptr, nullptr, S, s_next, D, nullptr, nullptr, w)) return -1;
            }
        }
    }
    // ---- cost (and its gradient wrt the scored states)
    fill_f32(w.cost, 0.0f, (size_t) S, st); launches++;
    if (want_grad) { fill_f32(w.gstate, 0.0f, (size_t) (T + 1) * S * D, st); launches++; }
    int n_list = T;   // scored candidates: list positions 1..n_list
    const float * base = w.states + (size_t) S * D;   // position 1
    int Dl = D;
    for (size_t k = 0; k < w.enc.size(); k++) {
        EncStage & e = w.enc[k];
        const DLevel & U = levels[(size_t) e.lv - 1];
        const int Din = Dl, Dout = U.D, H = U.enc_fc1 ? U.enc_fc1.out : Din;
        const int n = e.n * S;
        for (int j = 0; j < e.n; j++) {
            const float * src = base + (size_t) (e.src_pos[(size_t) j] - 1) * S * Din;
            copy_rows(src, Din, e.in + (size_t) j * S * Din, Din, S, Din, st); launches++;
        }
        if (U.hp.enc_kind == "identity") {
            copy_rows(e.in, Din, e.out, Dout, n, Dout, st); launches++;
        } else {
            layer_norm(e.in, Din, U.enc_in_w, U.enc_in_b, ln_eps, nullptr, Din, e.h_hi, e.h_lo, e.st1, n, Din, st); launches++;
            if (U.enc_fc1.tc_fwd()) {
                GemmEpi ep;
                ep.mode = EPI_GELU_SPLIT; ep.bias = U.enc_fc1.b; ep.out0 = e.u; ep.ld0 = H; ep.out_hi = e.g_hi; ep.out_lo = e.g_lo; ep.ld_split = H;
                launches++;
                if (wgemm(w, {e.h_hi, e.h_lo, Din}, U.enc_fc1.fwd(), n, H, Din, ep, st)) return -1;
            } else {
                layer_norm(e.in, Din, U.enc_in_w, U.enc_in_b, ln_eps, w.tmpR2, Din, nullptr, nullptr, nullptr, n, Din, st);
                linear_simt(w.tmpR2, Din, U.enc_fc1.w, U.enc_fc1.b, e.u, H, n, H, Din, st);
                act_fwd(e.u, H, w.tmpR2, H, n, H, 0, st);
                split_f32(w.tmpR2, H, e.g_hi, e.g_lo, H, n, H, st);
                launches += 4;
            }
            float * yout = U.enc_out_w ? e.y : e.out;
            if (lin_fwd(U.enc_fc2, nullptr, H, e.g_hi, e.g_lo, n, yout, Dout, nullptr, nullptr, w)) return -1;
            if (U.enc_out_w) {
                layer_norm(e.y, Dout, U.enc_out_w, U.enc_out_b, ln_eps, e.out, Dout, nullptr, nullptr, e.st2, n, Dout, st);
                launches++;
            }
        }
        if (want_grad) { fill_f32(e.gout, 0.0f, (size_t) n * Dout, st); launches++; }
        base = e.out;
        n_list = e.n;
        Dl = Dout;
    }
    const int W = std::min(std::max(1, cs.cost_last_n), n_list);
    // pointer tables were written when the workspace's graph was planned (solve / plan_cost)
    cost_l2(w.pred_ptrs, w.goals, w.weights, w.gpred_ptrs, W, S, Dl, Dl, w.cost, want_grad, st);
    launches++;
    // the action cost comes after the state cost, as the reference adds them (hjepa-plan.cpp:769-791)
    if (w.pool.Wa > 0 && pool_forward(w, want_grad)) return -1;
    return 0;
}

// the cost's pointer tables (device) for the scored states of this workspace
bool HPlanner::cost_tables(Workspace & w, const CostSpec & cs) {
    cudaStream_t st = ctx->stream;
    const DLevel & L = levels[(size_t) w.level - 1];
    const int S = w.S, T = w.T;
    int n_list = T, Dl = L.D;
    const float * base = w.states + (size_t) S * L.D;
    float * gbase = w.gstate + (size_t) S * L.D;
    for (EncStage & e : w.enc) {
        base = e.out; gbase = e.gout; n_list = e.n; Dl = levels[(size_t) e.lv - 1].D;
    }
    const int W = std::min(std::max(1, cs.cost_last_n), n_list);
    std::vector<const float *> p((size_t) W);
    std::vector<float *> gp((size_t) W);
    std::vector<float> wt((size_t) W);
    for (int j = 0; j < W; j++) {
        const int k = n_list - W + j;
        p[(size_t) j] = base + (size_t) k * S * Dl;
        gp[(size_t) j] = gbase + (size_t) k * S * Dl;
        wt[(size_t) j] = (cs.intermediate_cost_weight != 1.0f && W > 1 && j < W - 1) ? cs.intermediate_cost_weight : 1.0f;
    }
    std::vector<float> goals((size_t) W * Dl);
    for (int j = 0; j < W; j++) memcpy(goals.data() + (size_t) j * Dl, cs.goal + (size_t) (cs.n_goal == 1 ? 0 : j) * Dl, (size_t) Dl * 4);
    // the action cost's tables: chunk j of the pooled rows against goal action n_goal - Wa + j, weight
    // action_cost_weight for every chunk
    PoolWs & pw = w.pool;
    std::vector<const float *> pp((size_t) pw.Wa);
    std::vector<float *> gpp((size_t) pw.Wa);
    std::vector<float> pwt((size_t) pw.Wa, cs.action_cost_weight), pgoals;
    if (pw.Wa > 0) {
        const int Au = levels[(size_t) w.level].A;
        for (int j = 0; j < pw.Wa; j++) {
            pp[(size_t) j] = pw.y + (size_t) j * S * Au;
            gpp[(size_t) j] = pw.gy + (size_t) j * S * Au;
        }
        pgoals.assign(cs.goal_action + (size_t) (cs.n_goal - pw.Wa) * Au, cs.goal_action + (size_t) cs.n_goal * Au);
        if (!cuda_ok(cudaMemcpyAsync(pw.ptrs, pp.data(), pp.size() * sizeof(void *), cudaMemcpyHostToDevice, st), "action cost tables") ||
            !cuda_ok(cudaMemcpyAsync(pw.gptrs, gpp.data(), gpp.size() * sizeof(void *), cudaMemcpyHostToDevice, st), "action cost tables") ||
            !cuda_ok(cudaMemcpyAsync(pw.weights, pwt.data(), pwt.size() * 4, cudaMemcpyHostToDevice, st), "action cost weights") ||
            !cuda_ok(cudaMemcpyAsync(pw.goals, pgoals.data(), pgoals.size() * 4, cudaMemcpyHostToDevice, st), "goal actions"))
            return false;
    }
    bool ok = cuda_ok(cudaMemcpyAsync(w.pred_ptrs, p.data(), (size_t) W * sizeof(void *), cudaMemcpyHostToDevice, st), "cost tables") &&
              cuda_ok(cudaMemcpyAsync(w.gpred_ptrs, gp.data(), (size_t) W * sizeof(void *), cudaMemcpyHostToDevice, st), "cost tables") &&
              cuda_ok(cudaMemcpyAsync(w.weights, wt.data(), (size_t) W * 4, cudaMemcpyHostToDevice, st), "cost weights") &&
              cuda_ok(cudaMemcpyAsync(w.goals, goals.data(), goals.size() * 4, cudaMemcpyHostToDevice, st), "goals") &&
              cuda_ok(cudaStreamSynchronize(st), "cost tables");
    return ok;
}

// ---------------------------------------------------------------------------------------------
// backward: encoders, rollout (reverse), conditioning path; leaves d actions (t-major) in da_all
// ---------------------------------------------------------------------------------------------
int HPlanner::backward(Workspace & w, const CostSpec & cs) {
    (void) cs;
    cudaStream_t st = w.st;
    const DLevel & L = levels[(size_t) w.level - 1];
    const int S = w.S, T = w.T, D = L.D, P = L.P, F = L.F, NL = L.L, A = L.A;
    const int R = S * T, ldm = 6 * P * NL;
    // ---- the action cost's encoder, into the gradient of the pooled action embeddings
    if (w.pool.Wa > 0 && pool_backward(w)) return -1;
    // ---- goal-projection encoders, top stage first, into the gradients of the states they read
    for (int k = (int) w.enc.size() - 1; k >= 0; k--) {
        EncStage & e = w.enc[(size_t) k];
        const DLevel & U = levels[(size_t) e.lv - 1];
        const int Din = k == 0 ? D : levels[(size_t) w.enc[(size_t) k - 1].lv - 1].D;
        const int Dout = U.D, H = U.enc_fc1 ? U.enc_fc1.out : Din;
        const int n = e.n * S;
        float * gsrc_base = k == 0 ? w.gstate + (size_t) S * D : w.enc[(size_t) k - 1].gout;
        if (U.hp.enc_kind == "identity") {
            for (int j = 0; j < e.n; j++) {
                add_inplace(gsrc_base + (size_t) (e.src_pos[(size_t) j] - 1) * S * Din, Din, e.gout + (size_t) j * S * Dout, Dout, S, Din, st);
                launches++;
            }
            continue;
        }
        const float * gy = e.gout;
        if (U.enc_out_w) {
            layer_norm_bwd(e.gout, Dout, e.y, Dout, e.st2, U.enc_out_w, nullptr, 0, e.gy, Dout, nullptr, 0, nullptr, 0,
                           nullptr, nullptr, 0, nullptr, nullptr, 0, n, Dout, st);
            launches++;
            gy = e.gy;
        }
        if (U.enc_fc2.tc_bwd() && U.enc_fc1.tc_bwd()) {
            split_f32(gy, Dout, e.d_hi, e.d_lo, Dout, n, Dout, st);
            GemmEpi ep;
            ep.mode = EPI_DGELU_SPLIT; ep.aux = e.u; ep.ld_aux = H; ep.out_hi = e.g_hi; ep.out_lo = e.g_lo; ep.ld_split = H;
            if (wgemm(w, {e.d_hi, e.d_lo, Dout}, U.enc_fc2.bwd(), n, H, Dout, ep, st)) return -1;
            GemmEpi ep2;
            ep2.out0 = e.gin; ep2.ld0 = Din;
            if (wgemm(w, {e.g_hi, e.g_lo, H}, U.enc_fc1.bwd(), n, Din, H, ep2, st)) return -1;
            launches += 3;
        } else {
            if (lin_bwd(U.enc_fc2, gy, Dout, nullptr, nullptr, n, w.tmpR2, H, w)) return -1;
            act_bwd(w.tmpR2, H, e.u, H, w.tmpR2, H, n, H, 0, false, st); launches++;
            if (lin_bwd(U.enc_fc1, w.tmpR2, H, nullptr, nullptr, n, e.gin, Din, w)) return -1;
        }
        // in_norm backward, then scatter-add into the sources
        layer_norm_bwd(e.gin, Din, e.in, Din, e.st1, U.enc_in_w, nullptr, 0, e.gy, Din, nullptr, 0, nullptr, 0,
                       nullptr, nullptr, 0, nullptr, nullptr, 0, n, Din, st);
        launches++;
        for (int j = 0; j < e.n; j++) {
            add_inplace(gsrc_base + (size_t) (e.src_pos[(size_t) j] - 1) * S * Din, Din, e.gy + (size_t) j * S * Din, Din, S, Din, st);
            launches++;
        }
    }
    // ---- rollout, reverse
    for (int t = T - 1; t >= 0; t--) {
        if (w.step_mod && !w.keep_mod && step_modulation(w, t, 1)) return -1;   // step t's modulation, recomputed
        const float * g_next = w.gstate + (size_t) (t + 1) * S * D;
        const float * x0 = w.xs + (size_t) t * (NL + 1) * S * P;
        const float * xL = x0 + (size_t) NL * S * P;
        const float * gy = g_next;
        int ldgy = D;
        if (L.proj0) {
            const int H = L.proj0.out;
            if (lin_bwd(L.proj2, gy, ldgy, nullptr, nullptr, S, w.gtmp, H, w)) return -1;
            act_bwd(w.gtmp, H, w.pu + (size_t) t * S * H, H, w.gtmp2, H, S, H, 0, false, st); launches++;
            float * dst = L.out_proj ? w.gtmp : w.gh;
            const int wdst = L.out_proj ? L.out_proj.out : P;
            if (lin_bwd(L.proj0, w.gtmp2, H, nullptr, nullptr, S, dst, wdst, w)) return -1;
            gy = dst; ldgy = wdst;
        }
        if (L.out_proj) {
            if (lin_bwd(L.out_proj, gy, ldgy, nullptr, nullptr, S, w.gh, P, w)) return -1;
            gy = w.gh; ldgy = P;
        }
        {
            const size_t tl = (size_t) t * NL + (NL - 1);
            const float * mod_l = w.mod + mod_row0(w, t) * ldm + (size_t) (NL - 1) * 6 * P;
            layer_norm_bwd(gy, ldgy, xL, P, w.stn + (size_t) t * S, L.norm_w, nullptr, 0, w.gx, P,
                           w.dn + tl * S * P, P, mod_l + 5 * P, ldm,
                           w.dmod_hi + dmod_row0(w, t) * ldm + (size_t) (NL - 1) * 6 * P + 5 * P,
                           w.dmod_lo + dmod_row0(w, t) * ldm + (size_t) (NL - 1) * 6 * P + 5 * P, ldm,
                           w.d_hi, w.d_lo, P, S, P, st);
            launches++;
        }
        for (int l = NL - 1; l >= 0; l--) {
            const DBlock & B = L.blocks[(size_t) l];
            const size_t tl = (size_t) t * NL + l;
            const float * mod_l = w.mod + mod_row0(w, t) * ldm + (size_t) l * 6 * P;
            float * dmh = w.dmod_hi + dmod_row0(w, t) * ldm + (size_t) l * 6 * P;
            float * dml = w.dmod_lo + dmod_row0(w, t) * ldm + (size_t) l * 6 * P;
            const float * xin = x0 + (size_t) l * S * P;
            // MLP half
            GemmEpi e1;
            e1.mode = EPI_MUL_SPLIT; e1.aux = w.u + tl * S * F; e1.ld_aux = F; e1.out_hi = w.du_hi; e1.out_lo = w.du_lo; e1.ld_split = F;
            if (wgemm(w, {w.d_hi, w.d_lo, P}, B.down.bwd(), S, F, P, e1, st)) return -1;
            GemmEpi e2;
            e2.out0 = w.gh; e2.ld0 = P;
            if (wgemm(w, {w.du_hi, w.du_lo, F}, B.up.bwd(), S, P, F, e2, st)) return -1;
            BlockBwdArgs a{};
            a.gh = w.gh; a.ldgh = P; a.gres = w.gx; a.ldres = P; a.x = w.xmid + tl * S * P; a.ldx = P;
            a.st0 = w.stm0 + tl * S; a.st1 = w.stm1 + tl * S; a.ln_w = B.ln2_w; a.ln_b = B.ln2_b;
            a.mod = mod_l; a.ld_mod = ldm; a.sh_off = 3 * P; a.sc_off = 4 * P;
            a.dmod_hi = dmh; a.dmod_lo = dml; a.ld_dmod = ldm; a.gx = w.gmid; a.ldgx = P;
            a.a2 = w.o + tl * S * P; a.lda2 = P; a.mod2 = mod_l; a.ld_mod2 = ldm; a.gate2_off = 2 * P;
            a.dmod2_hi = dmh; a.dmod2_lo = dml; a.ld_dmod2 = ldm; a.d_hi = w.d_hi; a.d_lo = w.d_lo; a.ldd = P;
            a.M = S; a.D = P; a.eps0 = adaln_eps; a.eps1 = ln_eps;
            block_bwd(a, st);
            // attention half (one query over one key: the value path, through the composed linear)
            GemmEpi e4;
            e4.out0 = w.gh; e4.ld0 = P;
            if (wgemm(w, {w.d_hi, w.d_lo, P}, B.ov.bwd(), S, P, P, e4, st)) return -1;
            BlockBwdArgs b{};
            b.gh = w.gh; b.ldgh = P; b.gres = w.gmid; b.ldres = P; b.x = xin; b.ldx = P;
            b.st0 = w.sta0 + tl * S; b.st1 = w.sta1 + tl * S; b.ln_w = B.ln1_w; b.ln_b = B.ln1_b;
            b.mod = mod_l; b.ld_mod = ldm; b.sh_off = 0; b.sc_off = P;
            b.dmod_hi = dmh; b.dmod_lo = dml; b.ld_dmod = ldm; b.gx = w.gx; b.ldgx = P;
            if (l > 0) {
                const size_t tl1 = tl - 1;
                b.a2 = w.dn + tl1 * S * P; b.lda2 = P; b.mod2 = mod_l - 6 * P; b.ld_mod2 = ldm; b.gate2_off = 5 * P;
                b.dmod2_hi = dmh - 6 * P; b.dmod2_lo = dml - 6 * P; b.ld_dmod2 = ldm; b.d_hi = w.d_hi; b.d_lo = w.d_lo; b.ldd = P;
            }
            b.M = S; b.D = P; b.eps0 = adaln_eps; b.eps1 = ln_eps;
            block_bwd(b, st);
            launches += 5;
        }
        // step-at-a-time modulation: this step's dmod into its rows of dcs now, before the next step reuses dmod
        if (w.step_mod && step_modulation_bwd(w, t, 1)) return -1;
        // gx = d (s_t + pos0 [-> in_proj]); pass it to the state the step read
        if (t > 0) {
            float * gs = w.gstate + (size_t) t * S * D;
            if (L.in_proj) {
                if (lin_bwd(L.in_proj, w.gx, P, nullptr, nullptr, S, w.gtmp, D, w)) return -1;
                add_inplace(gs, D, w.gtmp, D, S, D, st);
            } else {
                add_inplace(gs, D, w.gx, P, S, D, st);
            }
            launches++;
        }
    }
    // ---- conditioning path: every step's d(cs) through every adaLN linear in one GEMM
    if (!w.step_mod && step_modulation_bwd(w, 0, T)) return -1;
    act_bwd(w.dcs, P, w.cpre, P, w.dc, P, R, P, 2, false, st); launches++;
    float * g = w.dc;
    int gw = P;
    if (L.cond_proj) {
        if (lin_bwd(L.cond_proj, g, gw, nullptr, nullptr, R, w.tmpR, L.C, w)) return -1;
        g = w.tmpR; gw = L.C;
    }
    if (L.pact0) {
        const int H = L.pact0.out;
        if (lin_bwd(L.pact2, g, gw, nullptr, nullptr, R, w.tmpR2, H, w)) return -1;
        act_bwd(w.tmpR2, H, w.pa_u, H, w.tmpR2, H, R, H, 2, false, st); launches++;
        if (lin_bwd(L.pact0, w.tmpR2, H, nullptr, nullptr, R, w.tmpR, L.E, w)) return -1;
        g = w.tmpR; gw = L.E;
    }
    // g = d cost / d (action embeddings) through the predictor; the action cost's share joins it here
    if (L.act0) {
        const int H = L.act0.out;
        if (w.pool.Wa > 0) { add_inplace(g, gw, w.pool.ge, L.E, R, L.E, st); launches++; }
        if (lin_bwd(L.act2, g, gw, nullptr, nullptr, R, w.tmpR2, H, w)) return -1;
        act_bwd(w.tmpR2, H, w.ae_u, H, w.tmpR2, H, R, H, 2, false, st); launches++;
        if (lin_bwd(L.act0, w.tmpR2, H, nullptr, nullptr, R, w.da_all, A, w)) return -1;
    } else {
        copy_rows(g, gw, w.da_all, A, R, A, st); launches++;
        if (w.pool.Wa > 0) { add_inplace(w.da_all, A, w.pool.ge, A, R, A, st); launches++; }
    }
    return 0;
}

// ---------------------------------------------------------------------------------------------
// plan_cost: one evaluation of given candidates
// ---------------------------------------------------------------------------------------------
int HPlanner::plan_cost(const CostSpec & cs, const float * actions, int S, float * costs, float * grad) {
    cudaStream_t st = ctx->stream;
    const DLevel & L = levels[(size_t) cs.level - 1];
    const int T = cs.horizon, A = L.A, D = L.D;
    Workspace * w = workspace(cs.level, S, T, cs);
    if (!w) return -1;
    if (!cost_tables(*w, cs)) return -1;
    launches = 0;
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventRecord(e0, st);
    JB_CUDA(cudaMemcpyAsync(w->x, actions, (size_t) S * T * A * 4, cudaMemcpyHostToDevice, st));
    if (w->fix_count) JB_CUDA(cudaMemsetAsync(w->fix_count, 0, w->fix_counters * sizeof(int), st));
    JB_CUDA(cudaMemcpyAsync(w->gtmp, cs.s0, (size_t) D * 4, cudaMemcpyHostToDevice, st));
    copy_rows(w->gtmp, 0, w->states, D, S, D, st);
    gather_actions(w->x, w->a_all, S, T, A, st);
    launches += 2;
    if (forward(*w, cs, grad != nullptr)) return -1;
    if (grad) {
        if (backward(*w, cs)) return -1;
        scatter_actions(w->da_all, w->grad, S, T, A, st); launches++;
        JB_CUDA(cudaMemcpyAsync(grad, w->grad, (size_t) S * T * A * 4, cudaMemcpyDeviceToHost, st));
    }
    JB_CUDA(cudaMemcpyAsync(costs, w->cost, (size_t) S * 4, cudaMemcpyDeviceToHost, st));
    cudaEventRecord(e1, st);
    JB_CUDA(cudaStreamSynchronize(st));
    float ms = 0;
    cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    ctx->last_ms = ms;
    ctx->last_launches = launches;
    if (gemm_error_flag(st)) { log("jepa: a tensor-core kernel gave up waiting on its pipeline\n"); return -1; }
    return 0;
}

}  // namespace jb
