// The H-JEPA state and action encoders on the GPU: jepa_hjepa_embed, jepa_hjepa_lift,
// jepa_hjepa_action_embed, jepa_hjepa_action_encode (reference: src/hjepa.cpp:374-561). These turn the
// encoder's CLS rows and the recorded actions into the per-level states and latent actions the planners and
// predictors read, and back the subgoal / action hand-off between levels.
//
//   embed          level-1 state = projector(CLS) [ | proprio stream ]: mlp (GELU) / layernorm / identity
//   lift           level-k state t = enc(level k-1 state t stride): in_norm -> fc1 -> GELU -> fc2 (-> out_norm)
//   action_embed   the level's actions through act_embed (SiLU MLP; identity when absent)
//   action_encode  chunks of `stride` action embeddings of the level below -> the level's latent actions:
//                  'mlp' over the zero-padded flattened chunk, 'seq' a transformer over CLS + the chunk's
//                  steps (a short trailing chunk at its own length, which is what masking its padding as keys
//                  amounts to for the CLS row)
//
// A call covers a handful of rows: SIMT linears (float32) and the row-wise / grouped-attention kernels.
#include "hplan.h"
#include "common.h"

#include "../../include/jepa.h"

#include <algorithm>
#include <cstdlib>
#include <cstring>

namespace jb {

namespace {

struct DevBuf {
    void * p = nullptr;
    ~DevBuf() { if (p) cudaFree(p); }
    bool alloc(size_t floats) { return cuda_ok(cudaMalloc(&p, std::max<size_t>(floats, 1) * 4), "encoder buffer"); }
    float * f() const { return (float *) p; }
};

void lin(const DLin & L, const float * x, int ldx, int M, float * y, int ldy, cudaStream_t st) {
    linear_simt(x, ldx, L.w, L.b, y, ldy, M, L.out, L.in, st);
}

HPlanner * planner_for(jepa_context * ctx, int level, const char * fn) {
    if (!ctx->model->hj.present) {
        log("jepa: %s: '%s' is not an H-JEPA model\n", fn, ctx->model->name.c_str());
        return nullptr;
    }
    const int n = (int) ctx->model->hj.levels.size();
    if (level < 1 || level > n) {
        log("jepa: %s: level %d is out of range, the model has levels 1..%d\n", fn, level, n);
        return nullptr;
    }
    return hplanner_of(ctx, fn);
}

// device rows -> a malloc'd jepa_output (the caller frees data with jepa_free)
int emit(jepa_context * ctx, const float * dev, int64_t rows, int64_t dim, jepa_output * out) {
    float * data = (float *) malloc((size_t) std::max<int64_t>(rows * dim, 1) * sizeof(float));
    if (!data) { log("jepa: out of host memory\n"); return -1; }
    if (!cuda_ok(cudaMemcpyAsync(data, dev, (size_t) rows * dim * 4, cudaMemcpyDeviceToHost, ctx->stream), "encoder output") ||
        !cuda_ok(cudaStreamSynchronize(ctx->stream), "encoder")) {
        free(data);
        return -1;
    }
    out->data = data;
    out->n_tokens = rows;
    out->dim = dim;
    return 0;
}

}  // namespace

// the level-1 projector and proprio weights (float32, for SIMT products), on first use
bool HPlanner::ensure_embed() {
    if (emb.loaded) return true;
    const jepa_model & m = *ctx->model;
    auto load = [&](const std::string & name) -> DLin {
        const gguf_tensor * t = m.get(name + ".weight");
        return t ? upload_plain(name, 0, t->ne[1]) : DLin();
    };
    auto vec = [&](const std::string & name) -> float * { return m.get(name) ? upload_vec(name) : nullptr; };
    emb.proj0 = load("lvl.1.enc.proj.0");
    emb.proj2 = load("lvl.1.enc.proj.2");
    emb.proj_ln_w = vec("lvl.1.enc.proj_ln.weight");
    emb.proj_ln_b = vec("lvl.1.enc.proj_ln.bias");
    emb.pro0 = load("lvl.1.enc.proprio.0");
    emb.pro2 = load("lvl.1.enc.proprio.2");
    emb.pro_ln_w = vec("lvl.1.enc.proprio.ln.weight");
    emb.pro_ln_b = vec("lvl.1.enc.proprio.ln.bias");
    emb.loaded = true;
    return true;
}

}  // namespace jb

using namespace jb;

extern "C" {

int jepa_hjepa_embed(jepa_context * ctx, const float * cls_rows, const float * proprio, int n_rows, jepa_output * out) {
    if (!ctx || !cls_rows || !out || n_rows <= 0) return -1;
    HPlanner * pm = planner_for(ctx, 1, "jepa_hjepa_embed");
    if (!pm || !pm->ensure_embed()) return -1;
    const jepa_model & m = *ctx->model;
    const HParams & hj = m.hj;
    const DLevel & L = pm->levels[0];
    const bool fusion = L.hp.enc_kind == "vit_proprio";
    if (fusion && !proprio) {
        log("jepa: jepa_hjepa_embed: this model's state includes a %d-d proprio stream; pass it\n", hj.proprio_dim);
        return -1;
    }
    const gguf_tensor * cls_tok = m.get("enc.cls_token");
    const int Dv = cls_tok ? (int) cls_tok->nelements() : hj.pixel_dim;
    const HPlanner::EmbedW & E = pm->emb;
    if (hj.proj_kind == "mlp" && !(E.proj0 && E.proj2)) { log("jepa: jepa_hjepa_embed: the mlp projector's weights are missing\n"); return -1; }
    if (fusion && !(E.pro0 && E.pro2)) { log("jepa: jepa_hjepa_embed: the proprio stream's weights are missing\n"); return -1; }
    const int n = n_rows;
    const int pix = hj.proj_kind == "mlp" ? E.proj2.out : Dv;
    const int q = fusion ? E.pro2.out : 0;
    const int Do = pix + q;
    cudaStream_t st = ctx->stream;
    const size_t wmax = (size_t) std::max({Dv, Do, E.proj0 ? E.proj0.out : 0, E.pro0 ? E.pro0.out : 0, hj.proprio_dim, 1});
    DevBuf x, t1, t2, y, pr;
    if (!x.alloc((size_t) n * Dv) || !t1.alloc((size_t) n * wmax) || !t2.alloc((size_t) n * wmax) || !y.alloc((size_t) n * Do) ||
        !pr.alloc((size_t) n * std::max(hj.proprio_dim, 1)))
        return -1;
    JB_CUDA(cudaMemcpyAsync(x.p, cls_rows, (size_t) n * Dv * 4, cudaMemcpyHostToDevice, st));
    if (hj.proj_kind == "mlp") {
        lin(E.proj0, x.f(), Dv, n, t1.f(), E.proj0.out, st);
        act_fwd(t1.f(), E.proj0.out, t2.f(), E.proj0.out, n, E.proj0.out, 0, st);
        lin(E.proj2, t2.f(), E.proj0.out, n, y.f(), Do, st);
    } else if (hj.proj_kind == "layernorm") {
        layer_norm(x.f(), Dv, E.proj_ln_w, E.proj_ln_b, pm->ln_eps, y.f(), Do, nullptr, nullptr, nullptr, n, Dv, st);
    } else {
        copy_rows(x.f(), Dv, y.f(), Do, n, Dv, st);
    }
    if (fusion) {   // [pixel | proprio(linear -> LN -> GELU -> linear)]
        const int P = hj.proprio_dim, H = E.pro0.out;
        JB_CUDA(cudaMemcpyAsync(pr.p, proprio, (size_t) n * P * 4, cudaMemcpyHostToDevice, st));
        lin(E.pro0, pr.f(), P, n, t1.f(), H, st);
        layer_norm(t1.f(), H, E.pro_ln_w, E.pro_ln_b, pm->ln_eps, t2.f(), H, nullptr, nullptr, nullptr, n, H, st);
        act_fwd(t2.f(), H, t1.f(), H, n, H, 0, st);
        lin(E.pro2, t1.f(), H, n, y.f() + pix, Do, st);
    }
    return emit(ctx, y.f(), n, Do, out);
}

int jepa_hjepa_lift(jepa_context * ctx, int level, const float * below, int n_rows, jepa_output * out) {
    if (!ctx || !below || !out || n_rows <= 0) return -1;
    HPlanner * pm = planner_for(ctx, level, "jepa_hjepa_lift");
    if (!pm) return -1;
    if (level < 2) {
        log("jepa: jepa_hjepa_lift: level 1 states come from jepa_hjepa_embed; lift takes level >= 2\n");
        return -1;
    }
    const DLevel & U = pm->levels[(size_t) level - 1];
    const int Db = pm->levels[(size_t) level - 2].D, Du = U.D, stride = U.hp.stride;
    const int n_out = (n_rows - 1) / stride + 1;
    cudaStream_t st = ctx->stream;
    DevBuf b, x, h, g, y, z;
    const int H = U.enc_fc1 ? U.enc_fc1.out : 1;
    if (!b.alloc((size_t) n_rows * Db) || !x.alloc((size_t) n_out * Db) || !h.alloc((size_t) n_out * H) || !g.alloc((size_t) n_out * H) ||
        !y.alloc((size_t) n_out * Du) || !z.alloc((size_t) n_out * Du))
        return -1;
    JB_CUDA(cudaMemcpyAsync(b.p, below, (size_t) n_rows * Db * 4, cudaMemcpyHostToDevice, st));
    copy_rows(b.f(), stride * Db, x.f(), Db, n_out, Db, st);   // every stride-th row of the level below
    if (U.hp.enc_kind == "identity") return emit(ctx, x.f(), n_out, Db, out);
    layer_norm(x.f(), Db, U.enc_in_w, U.enc_in_b, pm->ln_eps, x.f(), Db, nullptr, nullptr, nullptr, n_out, Db, st);
    lin(U.enc_fc1, x.f(), Db, n_out, h.f(), H, st);
    act_fwd(h.f(), H, g.f(), H, n_out, H, 0, st);
    lin(U.enc_fc2, g.f(), H, n_out, y.f(), Du, st);
    if (!U.enc_out_w) return emit(ctx, y.f(), n_out, Du, out);
    layer_norm(y.f(), Du, U.enc_out_w, U.enc_out_b, pm->ln_eps, z.f(), Du, nullptr, nullptr, nullptr, n_out, Du, st);
    return emit(ctx, z.f(), n_out, Du, out);
}

int jepa_hjepa_action_embed(jepa_context * ctx, int level, const float * actions, int n_rows, jepa_output * out) {
    if (!ctx || !actions || !out || n_rows <= 0) return -1;
    HPlanner * pm = planner_for(ctx, level, "jepa_hjepa_action_embed");
    if (!pm) return -1;
    const DLevel & L = pm->levels[(size_t) level - 1];
    cudaStream_t st = ctx->stream;
    DevBuf a, h, g, e;
    const int A = L.A, H = L.act0 ? L.act0.out : 1;
    if (!a.alloc((size_t) n_rows * A) || !h.alloc((size_t) n_rows * H) || !g.alloc((size_t) n_rows * H) || !e.alloc((size_t) n_rows * L.E))
        return -1;
    JB_CUDA(cudaMemcpyAsync(a.p, actions, (size_t) n_rows * A * 4, cudaMemcpyHostToDevice, st));
    if (!L.act0) return emit(ctx, a.f(), n_rows, A, out);   // identity
    lin(L.act0, a.f(), A, n_rows, h.f(), H, st);
    act_fwd(h.f(), H, g.f(), H, n_rows, H, 2, st);
    lin(L.act2, g.f(), H, n_rows, e.f(), L.E, st);
    return emit(ctx, e.f(), n_rows, L.E, out);
}

int jepa_hjepa_action_encode(jepa_context * ctx, int level, const float * below_act_emb, int n_rows, jepa_output * out) {
    if (!ctx || !below_act_emb || !out || n_rows <= 0) return -1;
    HPlanner * pm = planner_for(ctx, level, "jepa_hjepa_action_encode");
    if (!pm) return -1;
    if (level < 2) {
        log("jepa: jepa_hjepa_action_encode: level 1 actions are given, not encoded; this takes level >= 2\n");
        return -1;
    }
    const DLevel & B = pm->levels[(size_t) level - 2];
    const DLevel & U = pm->levels[(size_t) level - 1];
    const DActEnc & ae = U.ae;
    const int E = B.act0 ? B.E : B.A, S = U.hp.stride, Au = U.A;
    const int n_full = n_rows / S, rem = n_rows % S, n_out = n_full + (rem ? 1 : 0);
    cudaStream_t st = ctx->stream;
    if (ae.kind == 1) {
        // each chunk flattened ([t][E] rows are already chunk-major), a short trailing chunk zero-padded
        DevBuf x, h, r, y, z;
        const int H1 = ae.fc1.out;
        if (!x.alloc((size_t) n_out * S * E) || !h.alloc((size_t) n_out * H1) || !r.alloc((size_t) n_out * H1) ||
            !y.alloc((size_t) n_out * Au) || !z.alloc((size_t) n_out * Au))
            return -1;
        JB_CUDA(cudaMemsetAsync(x.p, 0, (size_t) n_out * S * E * 4, st));
        JB_CUDA(cudaMemcpyAsync(x.p, below_act_emb, (size_t) n_rows * E * 4, cudaMemcpyHostToDevice, st));
        lin(ae.fc1, x.f(), S * E, n_out, h.f(), H1, st);
        act_fwd(h.f(), H1, r.f(), H1, n_out, H1, 3, st);
        lin(ae.fc2, r.f(), H1, n_out, y.f(), Au, st);
        if (!ae.out_w) return emit(ctx, y.f(), n_out, Au, out);
        layer_norm(y.f(), Au, ae.out_w, ae.out_b, pm->ln_eps, z.f(), Au, nullptr, nullptr, nullptr, n_out, Au, st);
        return emit(ctx, z.f(), n_out, Au, out);
    }
    if (ae.kind != 2) { log("jepa: jepa_hjepa_action_encode: level %d has no action encoder\n", level); return -1; }
    // 'seq': the full chunks as one batch of groups, a short trailing chunk as a group of its own length
    const int d = ae.d, Dh = ae.head0.out;
    int F = 1;
    for (const DSeqBlock & blk : ae.blocks) F = std::max(F, blk.up.out);
    const size_t nG = (size_t) n_out * (S + 1);
    DevBuf e, zs, X, Xm, h, qkv, o, u, r, probs, cls, zz, zg, zl, y2, y;
    if (!e.alloc((size_t) n_rows * E) || !zs.alloc((size_t) n_rows * d) || !X.alloc(nG * d) || !Xm.alloc(nG * d) || !h.alloc(nG * d) ||
        !qkv.alloc(nG * 3 * d) || !o.alloc(nG * d) || !u.alloc(nG * F) || !r.alloc(nG * F) ||
        !probs.alloc(nG * (S + 1) * std::max(ae.n_head, 1)) || !cls.alloc((size_t) n_out * d) || !zz.alloc((size_t) n_out * Dh) ||
        !zg.alloc((size_t) n_out * Dh) || !zl.alloc((size_t) n_out * Dh) || !y2.alloc((size_t) n_out * Au) || !y.alloc((size_t) n_out * Au))
        return -1;
    JB_CUDA(cudaMemcpyAsync(e.p, below_act_emb, (size_t) n_rows * E * 4, cudaMemcpyHostToDevice, st));
    lin(ae.step, e.f(), E, n_rows, zs.f(), d, st);
    struct Part { int chunks, steps, row0, out0; };
    const Part parts[2] = {{n_full, S, 0, 0}, {rem ? 1 : 0, rem, n_full * S, n_full}};
    for (const Part & pt : parts) {
        if (pt.chunks == 0) continue;
        const int G = pt.steps + 1, ng = pt.chunks * G;
        if (!group_mha_prepare(G, d, ae.n_head)) { log("jepa: jepa_hjepa_action_encode: the chunk does not fit one CTA\n"); return -1; }
        pool_tokens(zs.f() + (size_t) pt.row0 * d, ae.pos, X.f(), pt.chunks, 1, pt.steps, d, false, st);
        for (const DSeqBlock & blk : ae.blocks) {
            const int Fb = blk.up.out;
            layer_norm(X.f(), d, blk.ln1_w, blk.ln1_b, pm->ln_eps, h.f(), d, nullptr, nullptr, nullptr, ng, d, st);
            lin(blk.qkv, h.f(), d, ng, qkv.f(), 3 * d, st);
            group_mha_fwd(qkv.f(), o.f(), probs.f(), pt.chunks, G, d, ae.n_head, st);
            lin(blk.out, o.f(), d, ng, Xm.f(), d, st);
            add_inplace(Xm.f(), d, X.f(), d, ng, d, st);
            layer_norm(Xm.f(), d, blk.ln2_w, blk.ln2_b, pm->ln_eps, h.f(), d, nullptr, nullptr, nullptr, ng, d, st);
            lin(blk.up, h.f(), d, ng, u.f(), Fb, st);
            act_fwd(u.f(), Fb, r.f(), Fb, ng, Fb, 3, st);
            lin(blk.down, r.f(), Fb, ng, X.f(), d, st);
            add_inplace(X.f(), d, Xm.f(), d, ng, d, st);
        }
        copy_rows(X.f(), G * d, cls.f() + (size_t) pt.out0 * d, d, pt.chunks, d, st);   // the CLS rows
    }
    lin(ae.head0, cls.f(), d, n_out, zz.f(), Dh, st);
    act_fwd(zz.f(), Dh, zg.f(), Dh, n_out, Dh, 0, st);
    layer_norm(zg.f(), Dh, ae.headln_w, ae.headln_b, pm->ln_eps, zl.f(), Dh, nullptr, nullptr, nullptr, n_out, Dh, st);
    lin(ae.head2, zl.f(), Dh, n_out, y2.f(), Au, st);
    layer_norm(y2.f(), Au, ae.out_w, ae.out_b, 1e-6f, y.f(), Au, nullptr, nullptr, nullptr, n_out, Au, st);
    return emit(ctx, y.f(), n_out, Au, out);
}

}  // extern "C"
