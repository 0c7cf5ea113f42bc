// The H-JEPA planner's action cost on the GPU: the candidates' action embeddings of the last Wa whole
// chunks pooled by the upper level's action encoder into latent actions, their squared L2 distance to the
// latent actions the upper level planned, weighted by action_cost_weight (src/hjepa-plan.cpp:769-791),
// and its gradient back into the embeddings.
//
// The Wa chunks are batched: n = Wa S rows, chunk-major (row j S + s is candidate s's chunk j). A chunk's
// steps are consecutive, so the Wa stride steps pooled are one contiguous block of the t-major embedding
// rows, starting at step c0 stride (c0 = T / stride - Wa). Linears go through the planner's lin_fwd /
// lin_bwd (3xTF32 tcgen05 GEMMs where the shape allows), row-wise kernels do the norms and activations, and
// pool.cu the concatenation, the token groups and the grouped attention.
#include "hplan.h"

#include <algorithm>

namespace jb {

int HPlanner::pooled_chunks(const CostSpec & cs) const {
    if (cs.action_cost_weight == 0.0f || !cs.goal_action || cs.goal_level != cs.level + 1 || cs.dense) return 0;
    if (cs.level < 1 || cs.level >= (int) levels.size()) return 0;
    const int n_pooled = cs.horizon / levels[(size_t) cs.level].hp.stride;   // whole chunks only
    return std::min({std::max(1, cs.cost_last_n), n_pooled, cs.n_goal});
}

int HPlanner::pool_forward(Workspace & w, bool want_grad) {
    cudaStream_t st = w.st;
    PoolWs & pw = w.pool;
    const DLevel & L = levels[(size_t) w.level - 1];
    const DLevel & U = levels[(size_t) w.level];
    const DActEnc & ae = U.ae;
    const int S = w.S, Au = U.A, stride = pw.stride, G = pw.G;
    const int Ein = L.act0 ? L.E : L.A;
    const int n = pw.Wa * S, nG = n * G;
    float * e = (L.act0 ? w.e : w.a_all) + (size_t) pw.c0 * stride * S * Ein;   // first pooled step's rows
    if (ae.kind == 1) {
        const int H1 = ae.fc1.out;
        pool_chunks(e, pw.x, pw.Wa, S, stride, Ein, false, st); launches++;
        if (lin_fwd(ae.fc1, pw.x, ae.fc1.in, nullptr, nullptr, n, pw.h, H1, nullptr, nullptr, w)) return -1;
        act_fwd(pw.h, H1, pw.r, H1, n, H1, 3, st); launches++;
        if (lin_fwd(ae.fc2, pw.r, H1, nullptr, nullptr, n, ae.out_w ? pw.ypre : pw.y, Au, nullptr, nullptr, w)) return -1;
        if (ae.out_w) { layer_norm(pw.ypre, Au, ae.out_w, ae.out_b, ln_eps, pw.y, Au, nullptr, nullptr, pw.sto, n, Au, st); launches++; }
    } else {
        const int d = ae.d, Dh = ae.head0.out;
        if (lin_fwd(ae.step, e, Ein, nullptr, nullptr, n * stride, pw.x, d, nullptr, nullptr, w)) return -1;
        pool_tokens(pw.x, ae.pos, pw.xs[0], pw.Wa, S, stride, d, false, st); launches++;
        for (size_t b = 0; b < ae.blocks.size(); b++) {
            const DSeqBlock & B = ae.blocks[b];
            const int F = B.up.out;
            // x = x + out(mha(qkv(LN1(x)))) ; x = x + down(relu(up(LN2(x))))
            layer_norm(pw.xs[b], d, B.ln1_w, B.ln1_b, ln_eps, pw.h, d, nullptr, nullptr, pw.st1[b], nG, d, st); launches++;
            if (lin_fwd(B.qkv, pw.h, d, nullptr, nullptr, nG, pw.qkv[b], 3 * d, nullptr, nullptr, w)) return -1;
            group_mha_fwd(pw.qkv[b], pw.h, pw.probs[b], n, G, d, ae.n_head, st); launches++;
            if (lin_fwd(B.out, pw.h, d, nullptr, nullptr, nG, pw.xmid[b], d, nullptr, nullptr, w)) return -1;
            add_inplace(pw.xmid[b], d, pw.xs[b], d, nG, d, st); launches++;
            layer_norm(pw.xmid[b], d, B.ln2_w, B.ln2_b, ln_eps, pw.h, d, nullptr, nullptr, pw.st2[b], nG, d, st); launches++;
            if (lin_fwd(B.up, pw.h, d, nullptr, nullptr, nG, pw.u[b], F, nullptr, nullptr, w)) return -1;
            act_fwd(pw.u[b], F, pw.r, F, nG, F, 3, st); launches++;
            if (lin_fwd(B.down, pw.r, F, nullptr, nullptr, nG, pw.xs[b + 1], d, nullptr, nullptr, w)) return -1;
            add_inplace(pw.xs[b + 1], d, pw.xmid[b], d, nG, d, st); launches++;
        }
        // the CLS row of every group -> head.0 -> GELU -> head LN -> head.2 -> LN(eps 1e-6)
        copy_rows(pw.xs.back(), G * d, pw.ga, d, n, d, st); launches++;
        if (lin_fwd(ae.head0, pw.ga, d, nullptr, nullptr, n, pw.z, Dh, nullptr, nullptr, w)) return -1;
        act_fwd(pw.z, Dh, pw.zg, Dh, n, Dh, 0, st); launches++;
        layer_norm(pw.zg, Dh, ae.headln_w, ae.headln_b, ln_eps, pw.zl, Dh, nullptr, nullptr, pw.sth, n, Dh, st); launches++;
        if (lin_fwd(ae.head2, pw.zl, Dh, nullptr, nullptr, n, pw.ypre, Au, nullptr, nullptr, w)) return -1;
        layer_norm(pw.ypre, Au, ae.out_w, ae.out_b, 1e-6f, pw.y, Au, nullptr, nullptr, pw.sto, n, Au, st); launches++;
    }
    if (want_grad) { fill_f32(pw.gy, 0.0f, (size_t) n * Au, st); launches++; }
    cost_l2(pw.ptrs, pw.goals, pw.weights, pw.gptrs, pw.Wa, S, Au, Au, w.cost, want_grad, st);
    launches++;
    return 0;
}

int HPlanner::pool_backward(Workspace & w) {
    cudaStream_t st = w.st;
    PoolWs & pw = w.pool;
    const DLevel & L = levels[(size_t) w.level - 1];
    const DLevel & U = levels[(size_t) w.level];
    const DActEnc & ae = U.ae;
    const int S = w.S, T = w.T, Au = U.A, stride = pw.stride, G = pw.G;
    const int Ein = L.act0 ? L.E : L.A;
    const int n = pw.Wa * S, nG = n * G;
    fill_f32(pw.ge, 0.0f, (size_t) T * S * Ein, st); launches++;
    float * ge = pw.ge + (size_t) pw.c0 * stride * S * Ein;
    if (ae.kind == 1) {
        const int H1 = ae.fc1.out;
        const float * g = pw.gy;
        if (ae.out_w) {
            layer_norm_bwd(pw.gy, Au, pw.ypre, Au, pw.sto, ae.out_w, nullptr, 0, pw.ga, Au, nullptr, 0, nullptr, 0,
                           nullptr, nullptr, 0, nullptr, nullptr, 0, n, Au, st);
            launches++;
            g = pw.ga;
        }
        if (lin_bwd(ae.fc2, g, Au, nullptr, nullptr, n, pw.gb, H1, w)) return -1;
        act_bwd(pw.gb, H1, pw.h, H1, pw.gc, H1, n, H1, 3, false, st); launches++;
        if (lin_bwd(ae.fc1, pw.gc, H1, nullptr, nullptr, n, pw.ga, ae.fc1.in, w)) return -1;
        pool_chunks(ge, pw.ga, pw.Wa, S, stride, Ein, true, st); launches++;
        return 0;
    }
    const int d = ae.d, Dh = ae.head0.out;
    layer_norm_bwd(pw.gy, Au, pw.ypre, Au, pw.sto, ae.out_w, nullptr, 0, pw.ga, Au, nullptr, 0, nullptr, 0,
                   nullptr, nullptr, 0, nullptr, nullptr, 0, n, Au, st);
    if (lin_bwd(ae.head2, pw.ga, Au, nullptr, nullptr, n, pw.gb, Dh, w)) return -1;
    layer_norm_bwd(pw.gb, Dh, pw.zg, Dh, pw.sth, ae.headln_w, nullptr, 0, pw.ga, Dh, nullptr, 0, nullptr, 0,
                   nullptr, nullptr, 0, nullptr, nullptr, 0, n, Dh, st);
    act_bwd(pw.ga, Dh, pw.z, Dh, pw.gb, Dh, n, Dh, 0, false, st);
    if (lin_bwd(ae.head0, pw.gb, Dh, nullptr, nullptr, n, pw.gc, d, w)) return -1;
    // only the CLS rows carry gradient into the last block's output
    fill_f32(pw.ga, 0.0f, (size_t) nG * d, st);
    copy_rows(pw.gc, d, pw.ga, G * d, n, d, st);
    launches += 5;
    for (int b = (int) ae.blocks.size() - 1; b >= 0; b--) {
        const DSeqBlock & B = ae.blocks[(size_t) b];
        const int F = B.up.out;
        // ga = d x_out ; MLP half: gb = d xmid = ga + LN2_bwd(up_bwd(relu'(down_bwd(ga))))
        if (lin_bwd(B.down, pw.ga, d, nullptr, nullptr, nG, pw.gb, F, w)) return -1;
        act_bwd(pw.gb, F, pw.u[(size_t) b], F, pw.gb, F, nG, F, 3, false, st);
        if (lin_bwd(B.up, pw.gb, F, nullptr, nullptr, nG, pw.gc, d, w)) return -1;
        layer_norm_bwd(pw.gc, d, pw.xmid[(size_t) b], d, pw.st2[(size_t) b], B.ln2_w, pw.ga, d, pw.gb, d, nullptr, 0, nullptr, 0,
                       nullptr, nullptr, 0, nullptr, nullptr, 0, nG, d, st);
        // attention half: ga = d x_in = gb + LN1_bwd(qkv_bwd(mha_bwd(out_bwd(gb))))
        if (lin_bwd(B.out, pw.gb, d, nullptr, nullptr, nG, pw.gc, d, w)) return -1;
        group_mha_bwd(pw.gc, pw.qkv[(size_t) b], pw.probs[(size_t) b], pw.ga, n, G, d, ae.n_head, st);
        if (lin_bwd(B.qkv, pw.ga, 3 * d, nullptr, nullptr, nG, pw.gc, d, w)) return -1;
        layer_norm_bwd(pw.gc, d, pw.xs[(size_t) b], d, pw.st1[(size_t) b], B.ln1_w, pw.gb, d, pw.ga, d, nullptr, 0, nullptr, 0,
                       nullptr, nullptr, 0, nullptr, nullptr, 0, nG, d, st);
        launches += 4;
    }
    // the step tokens' gradients -> the step linear -> the embeddings of the pooled steps
    pool_tokens(pw.gb, ae.pos, pw.ga, pw.Wa, S, stride, d, true, st); launches++;
    return lin_bwd(ae.step, pw.gb, d, nullptr, nullptr, n * stride, ge, Ein, w);
}

}  // namespace jb
