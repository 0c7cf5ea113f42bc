// jepa_encode for the image families (hfvit, ijepa, lewm, and the encoder of an H-JEPA file) and the video
// families (vjepa2, vjepa2_1, levjepa), and the pooling helpers of the API (reference: src/jepa.cpp:586-1000,
// :1183-1270).
//
//   image: x = patch_embed(patches) ; tokens = [CLS][registers][patches] + pos_embed
//   video: x = patch_embed(tubelet patches) (+ modality vector) ; tokens = [CLS][registers][patches]
//   per block: x += ls1 * out(attention(qkv(LN1(x)))) ; x += ls2 * down(act(up(LN2(x))))
//              (video: 3-D RoPE on q and k before the attention, identity for the prefix rows; LeVJEPA's
//              block-causal attention across temporal slots)
//   y = LN(x)
//
// Every (batch, frame) slice (image) or clip (video) is one sequence; a call's sequences run as one batch of
// rows through the 3xTF32 tensor-core GEMMs of the planner (the residual add and the layer scale in the gated
// epilogue, GELU in the up product's epilogue) and a float32 attention kernel. Patchifying happens on the
// host as the reference does it.
#include "encoder.h"
#include "upload.h"
#include "common.h"

#include "../../include/jepa.h"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <vector>

namespace jb {

EncEngine::~EncEngine() {
    for (void * p : allocations) cudaFree(p);
}

bool EncEngine::build(const jepa_model & m, cudaStream_t st) {
    Uploader up{allocations, m, st};
    const EncParams & e = m.enc;
    const int D = e.embed_dim;
    video = m.family == "vjepa2" || m.family == "vjepa2_1" || m.family == "levjepa";
    patch = up.lin_fwd_only("enc.patch_embed");
    if (video && m.get("enc.patch_embed_img.weight")) patch_img = up.lin_fwd_only("enc.patch_embed_img");
    if (video && e.modality_embed) {
        if (m.get("enc.mod_embed_video")) mod_video = up.vec("enc.mod_embed_video");
        if (m.get("enc.mod_embed_img")) mod_img = up.vec("enc.mod_embed_img");
    }
    if (e.cls_token) cls = up.vec("enc.cls_token");
    if (e.n_registers > 0) reg = up.vec("enc.reg_tokens");
    if (!video) {
        pos = up.vec("enc.pos_embed");
        if (const gguf_tensor * t = m.get("enc.pos_embed")) pos_rows = t->nelements() / D;
    }
    norm_w = up.vec("enc.norm.weight");
    norm_b = up.vec("enc.norm.bias");
    std::vector<float> one((size_t) D, 1.0f);
    ones = up.alloc<float>((size_t) D);
    if (ones) up.ok = cuda_ok(cudaMemcpy(ones, one.data(), (size_t) D * 4, cudaMemcpyHostToDevice), "encoder") && up.ok;
    for (int i = 0; i < e.n_layer && up.ok; i++) {
        const std::string p = "enc.blk." + std::to_string(i) + ".";
        EncLayer L;
        // the fused q / k / v linear, or the three a file keeps apart stacked into one (src/jepa.cpp:399-412)
        L.qkv = m.get(p + "attn_qkv.weight") ? up.lin_fwd_only(p + "attn_qkv")
                                             : up.lin_fwd_only_stacked({p + "attn_q", p + "attn_k", p + "attn_v"});
        L.out = up.lin_fwd_only(p + "attn_out");
        L.up = up.lin_fwd_only(p + "ffn_up");
        L.down = up.lin_fwd_only(p + "ffn_down");
        L.ln1_w = up.vec(p + "ln1.weight"); L.ln1_b = up.vec(p + "ln1.bias");
        L.ln2_w = up.vec(p + "ln2.weight"); L.ln2_b = up.vec(p + "ln2.bias");
        L.ls1 = m.get(p + "ls1") ? up.vec(p + "ls1") : ones;
        L.ls2 = m.get(p + "ls2") ? up.vec(p + "ls2") : ones;
        if (!(L.qkv && L.out && L.up && L.down) || L.qkv.out != 3 * D || L.qkv.in != D || L.out.out != D || L.up.in != D ||
            L.down.out != D || L.down.in != L.up.out) {
            log("jepa: jepa_encode: block %d is not a pre-norm block of width %d with q, k and v of that width\n", i, D);
            return false;
        }
        layers.push_back(L);
    }
    if (!up.ok || !patch || (!video && !pos) || (e.cls_token && !cls) || (e.n_registers > 0 && !reg) ||
        (video && e.modality_embed && !mod_video)) {
        log("jepa: jepa_encode: the encoder's weights are incomplete or could not be placed on the device\n");
        return false;
    }
    return true;
}

namespace {

struct DevBuf {
    void * p = nullptr;
    ~DevBuf() { if (p) cudaFree(p); }
    bool alloc(size_t floats) { return cuda_ok(cudaMalloc(&p, std::max<size_t>(floats, 1) * 4), "encoder buffer"); }
    float * f() const { return (float *) p; }
};

int lin_tc(const DLin & L, const float * x_hi, const float * x_lo, int ldx, int M, GemmEpi ep, cudaStream_t st) {
    return gemm_tc({x_hi, x_lo, ldx}, L.fwd(), M, L.out, L.in, ep, st);
}

}  // namespace

namespace {

// What one jepa_encode call runs: `items` sequences of N tokens, [CLS][registers][patch rows], the patch rows
// prepared on the host.
struct EncCall {
    int items = 0, N = 0, n_cls = 0, n_reg = 0, n_patches = 0, K = 0;
    const DLin * patch = nullptr;
    const float * pos = nullptr, * mod = nullptr;        // learned positions (image) / modality vector (video)
    std::vector<float> rows;                             // [items n_patches][K]
    std::vector<float> rope_cos, rope_sin;               // [N][hd] (video)
    int block_tpf = 0;                                   // block-causal slot size (0 = full attention)
};

// image families: every (batch, frame) slice a sequence, patches h-major, C x P x P per row
bool plan_image(const jepa_model & m, const EncEngine & E, const jepa_input * in, EncCall & c) {
    const EncParams & e = m.enc;
    const int P = e.patch_size;
    const int gh = in->height / P, gw = in->width / P, C = in->n_chans;
    c.items = in->n_batch * in->n_frames;
    c.n_cls = e.cls_token ? 1 : 0;
    c.n_reg = e.n_registers;
    c.n_patches = gh * gw;
    c.N = c.n_patches + c.n_cls + c.n_reg;
    c.K = C * P * P;
    c.patch = &E.patch;
    c.pos = E.pos;
    if (E.pos_rows != c.N) {
        log("jepa: token grid %dx%d (+%d prefix) = %d tokens does not match enc.pos_embed (%lld rows); "
            "position-table interpolation is not implemented yet -- feed a %dx%d input\n",
            gh, gw, c.n_cls + c.n_reg, c.N, (long long) E.pos_rows, e.img_size, e.img_size);
        return false;
    }
    c.rows.resize((size_t) c.items * c.n_patches * c.K);
    const size_t plane = (size_t) in->height * in->width;
    for (int b = 0; b < in->n_batch; b++) {
        for (int t = 0; t < in->n_frames; t++) {
            const int item = b * in->n_frames + t;
            for (int ch = 0; ch < C; ch++) {
                const float * src = in->data + (((size_t) b * C + ch) * in->n_frames + t) * plane;
                for (int y = 0; y < gh; y++)
                    for (int x = 0; x < gw; x++) {
                        float * dst = c.rows.data() + ((size_t) item * c.n_patches + (size_t) y * gw + x) * c.K + (size_t) ch * P * P;
                        for (int py = 0; py < P; py++)
                            memcpy(dst + (size_t) py * P, src + (size_t) (y * P + py) * in->width + (size_t) x * P, (size_t) P * 4);
                    }
            }
        }
    }
    return true;
}

// The 3-D RoPE tables of a gt x gh x gw token grid (tokens t-major, then h, then w) for heads of width hd:
// lanes [0, d) turn with the temporal position, [d, 2d) with the row, [2d, 3d) with the column,
// d = 2 floor(floor(hd / 3) / 2), the rest stay (cos 1, sin 0); frequency k of an axis is theta^(-k / (d/2)).
// Tiled layout (V-JEPA 2): lane j of an axis uses frequency j mod d/2; interleaved (V-JEPA 2.1): lanes 2k and
// 2k + 1 use frequency k. Positions, frequencies and the trigonometry in double, stored as float; with
// interpolation the row and column positions are rescaled to a ref x ref training grid. n_prefix identity
// rows come first (prefix tokens are not on the grid).
void rope3d_tables(const EncParams & e, int hd, int gt, int gh, int gw, int n_prefix, std::vector<float> & cs,
                   std::vector<float> & sn) {
    const int d = 2 * ((hd / 3) / 2), half = d / 2;
    const int64_t n_grid = (int64_t) gt * gh * gw, rows = n_prefix + n_grid;
    cs.assign((size_t) rows * hd, 1.0f);
    sn.assign((size_t) rows * hd, 0.0f);
    std::vector<double> omega((size_t) half);
    for (int k = 0; k < half; k++) omega[(size_t) k] = 1.0 / std::pow((double) e.rope_theta, (double) k / (half * 1.0));
    const int64_t tpf = (int64_t) gh * gw;
    for (int64_t i = 0; i < n_grid; i++) {
        double pos[3] = {(double) (i / tpf), (double) ((i % tpf) / gw), (double) ((i % tpf) % gw)};
        if (e.rope_interpolate) {
            const double ref = (double) e.rope_ref_grid;
            if (gh > 1) pos[1] = pos[1] * (ref - 1.0) / (double) (gh - 1);
            if (gw > 1) pos[2] = pos[2] * (ref - 1.0) / (double) (gw - 1);
        }
        float * crow = cs.data() + (size_t) (n_prefix + i) * hd;
        float * srow = sn.data() + (size_t) (n_prefix + i) * hd;
        for (int ax = 0; ax < 3; ax++) {
            for (int j = 0; j < d; j++) {
                const int k = e.rope_interleaved ? j / 2 : j % half;
                const double f = pos[ax] * omega[(size_t) k];
                crow[ax * d + j] = (float) std::cos(f);
                srow[ax * d + j] = (float) std::sin(f);
            }
        }
    }
}

// video families: every clip a sequence; tubelet x P x P patches (C-T-H-W inside a row), tokens t-major then
// h then w; V-JEPA 2.1 takes a one-frame input through its image tokenizer (tubelet 1)
bool plan_video(const jepa_model & m, const EncEngine & E, const jepa_input * in, EncCall & c) {
    const EncParams & e = m.enc;
    const int P = e.patch_size, C = in->n_chans, T = in->n_frames;
    const bool image_path = T == 1 && e.image_patch_embed && E.patch_img;
    const int tub = image_path ? 1 : std::max(1, e.tubelet_size);
    if (T % tub != 0) {
        log("jepa: %d frames do not fill whole tubelets of %d frames (feed an image to this model as a %d-frame clip)\n", T, tub, tub);
        return false;
    }
    const int gt = T / tub, gh = in->height / P, gw = in->width / P;
    c.items = in->n_batch;
    c.n_cls = e.cls_token ? 1 : 0;
    c.n_reg = e.n_registers;
    c.n_patches = gt * gh * gw;
    c.N = c.n_patches + c.n_cls + c.n_reg;
    c.K = C * tub * P * P;
    c.patch = image_path ? &E.patch_img : &E.patch;
    c.mod = e.modality_embed ? (image_path ? E.mod_img : E.mod_video) : nullptr;
    if (e.modality_embed && !c.mod) {
        log("jepa: jepa.enc.modality_embed is set but the %s modality vector is missing\n", image_path ? "image" : "video");
        return false;
    }
    if (c.patch->in != c.K) {
        log("jepa: %s takes rows of %d values; a %d-channel input in %d-frame tubelets of %dx%d patches gives %d\n",
            image_path ? "enc.patch_embed_img" : "enc.patch_embed", c.patch->in, C, tub, P, P, c.K);
        return false;
    }
    c.block_tpf = e.block_causal ? gh * gw : 0;
    rope3d_tables(e, e.embed_dim / e.n_head, gt, gh, gw, c.n_cls + c.n_reg, c.rope_cos, c.rope_sin);
    c.rows.resize((size_t) c.items * c.n_patches * c.K);
    const size_t plane = (size_t) in->height * in->width;
    for (int b = 0; b < in->n_batch; b++) {
        for (int ts = 0; ts < gt; ts++)
            for (int y = 0; y < gh; y++)
                for (int x = 0; x < gw; x++) {
                    float * dst = c.rows.data() + ((size_t) b * c.n_patches + ((size_t) ts * gh + y) * gw + x) * c.K;
                    for (int ch = 0; ch < C; ch++)
                        for (int tt = 0; tt < tub; tt++) {
                            const float * src = in->data + (((size_t) b * C + ch) * T + (size_t) ts * tub + tt) * plane;
                            for (int py = 0; py < P; py++, dst += P)
                                memcpy(dst, src + (size_t) (y * P + py) * in->width + (size_t) x * P, (size_t) P * 4);
                        }
                }
    }
    return true;
}

}  // namespace

}  // namespace jb

using namespace jb;

extern "C" {

int jepa_encode(jepa_context * ctx, const jepa_input * in, jepa_output * out) {
    if (!ctx || !in || !out || !in->data) return -1;
    const jepa_model & m = *ctx->model;
    const EncParams & e = m.enc;
    static const char * families[] = {"hfvit", "ijepa", "lewm", "hjepa", "vjepa2", "vjepa2_1", "levjepa"};
    if (std::none_of(std::begin(families), std::end(families), [&](const char * f) { return m.family == f; })) {
        log("jepa: jepa_encode: family '%s' has no encoder in this engine (image: hfvit, ijepa, lewm, hjepa; video: vjepa2, "
            "vjepa2_1, levjepa)\n", m.family.c_str());
        return -1;
    }
    if (in->n_chans != e.in_chans) {
        log("jepa: input has %d channels, model expects %d\n", in->n_chans, e.in_chans);
        return -1;
    }
    if (in->n_batch < 1 || in->n_frames < 1 || in->height < 1 || in->width < 1) {
        log("jepa: bad input shape [%d, %d, %d, %d, %d]\n", in->n_batch, in->n_chans, in->n_frames, in->height, in->width);
        return -1;
    }
    const int P = e.patch_size;
    if (in->height % P != 0 || in->width % P != 0) {
        log("jepa: input %dx%d is not a multiple of the patch size %d\n", in->height, in->width, P);
        return -1;
    }
    if (e.act != "gelu_erf" && e.act != "gelu_tanh" && e.act != "silu" && e.act != "relu") {
        log("jepa: jepa_encode: encoder activation '%s' is not supported by this engine\n", e.act.c_str());
        return -1;
    }
    if (!enc_attention_supported(e.embed_dim, e.n_head)) {
        log("jepa: jepa_encode: head width %d is not supported by this engine (32, 48, 64, 80, 88, 96, 128)\n",
            e.n_head > 0 ? e.embed_dim / e.n_head : 0);
        return -1;
    }
    cudaSetDevice(ctx->device);
    if (!ctx->enc) {
        auto eng = std::make_unique<EncEngine>();
        if (!eng->build(m, ctx->stream)) return -1;
        ctx->enc = std::move(eng);
    }
    EncEngine & E = *ctx->enc;
    EncCall c;
    if (!(E.video ? plan_video(m, E, in, c) : plan_image(m, E, in, c))) return -1;
    const int D = e.embed_dim, N = c.N, K = c.K, items = c.items;
    const int64_t rows = (int64_t) items * N;
    if (rows * (int64_t) std::max(3 * D, e.ffn_dim) >= ((int64_t) 1 << 40) || (int64_t) items * c.n_patches * K >= ((int64_t) 1 << 40)) {
        log("jepa: jepa_encode: the input is too large\n");
        return -1;
    }
    int F = 1;
    for (const EncLayer & L : E.layers) F = std::max(F, L.up.out);
    cudaStream_t st = ctx->stream;
    if (device_flags_clear(st)) return -1;
    const size_t R = (size_t) rows, wide = (size_t) std::max({3 * D, F, K});
    const int hd = D / e.n_head;
    DevBuf patches, p_hi, p_lo, pe, X, X2, h_hi, h_lo, qkv, o, o_hi, o_lo, a, u, g_hi, g_lo, y, rc, rs;
    if (!patches.alloc(c.rows.size()) || !p_hi.alloc(c.rows.size()) || !p_lo.alloc(c.rows.size()) ||
        !pe.alloc((size_t) items * c.n_patches * D) || !X.alloc(R * D) || !X2.alloc(R * D) || !h_hi.alloc(R * D) ||
        !h_lo.alloc(R * D) || !qkv.alloc(R * 3 * D) || !o.alloc(R * D) || !o_hi.alloc(R * D) || !o_lo.alloc(R * D) ||
        !a.alloc(R * wide) || !u.alloc(R * F) || !g_hi.alloc(R * F) || !g_lo.alloc(R * F) || !y.alloc(R * D) ||
        (E.video && (!rc.alloc((size_t) N * hd) || !rs.alloc((size_t) N * hd))))
        return -1;
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventRecord(e0, st);
    JB_CUDA(cudaMemcpyAsync(patches.p, c.rows.data(), c.rows.size() * 4, cudaMemcpyHostToDevice, st));
    if (E.video) {
        JB_CUDA(cudaMemcpyAsync(rc.p, c.rope_cos.data(), c.rope_cos.size() * 4, cudaMemcpyHostToDevice, st));
        JB_CUDA(cudaMemcpyAsync(rs.p, c.rope_sin.data(), c.rope_sin.size() * 4, cudaMemcpyHostToDevice, st));
    }
    split_f32(patches.f(), K, p_hi.f(), p_lo.f(), K, items * c.n_patches, K, st);
    {
        GemmEpi ep;
        ep.bias = c.patch->b; ep.out0 = pe.f(); ep.ld0 = D;
        if (lin_tc(*c.patch, p_hi.f(), p_lo.f(), K, items * c.n_patches, ep, st)) return -1;
    }
    enc_tokens(pe.f(), E.cls, E.reg, c.pos, X.f(), items, N, c.n_cls, c.n_reg, D, st, c.mod);
    const int M = (int) rows;
    for (const EncLayer & L : E.layers) {
        // attention half: X2 = X + ls1 * out(attention(rope(qkv(LN1(X)))))
        layer_norm(X.f(), D, L.ln1_w, L.ln1_b, e.ln_eps, nullptr, D, h_hi.f(), h_lo.f(), nullptr, M, D, st);
        GemmEpi e1;
        e1.bias = L.qkv.b; e1.out0 = qkv.f(); e1.ld0 = 3 * D;
        if (lin_tc(L.qkv, h_hi.f(), h_lo.f(), D, M, e1, st)) return -1;
        if (E.video) enc_rope_qk(qkv.f(), rc.f(), rs.f(), items, N, D, e.n_head, st);
        enc_attention(qkv.f(), o.f(), items, N, D, e.n_head, st, c.n_cls + c.n_reg, c.block_tpf);
        split_f32(o.f(), D, o_hi.f(), o_lo.f(), D, M, D, st);
        GemmEpi e2;
        e2.mode = EPI_GATED; e2.bias = L.out.b; e2.out0 = a.f(); e2.ld0 = D; e2.aux = X.f(); e2.ld_aux = D;
        e2.gate = L.ls1; e2.ld_gate = 0; e2.out1 = X2.f(); e2.ld1 = D;
        if (lin_tc(L.out, o_hi.f(), o_lo.f(), D, M, e2, st)) return -1;
        // MLP half: X = X2 + ls2 * down(act(up(LN2(X2))))
        layer_norm(X2.f(), D, L.ln2_w, L.ln2_b, e.ln_eps, nullptr, D, h_hi.f(), h_lo.f(), nullptr, M, D, st);
        const int Fl = L.up.out;
        GemmEpi e3;
        e3.bias = L.up.b;
        if (e.act == "gelu_erf") {
            e3.mode = EPI_GELU_SPLIT; e3.out0 = u.f(); e3.ld0 = Fl; e3.out_hi = g_hi.f(); e3.out_lo = g_lo.f(); e3.ld_split = Fl;
            if (lin_tc(L.up, h_hi.f(), h_lo.f(), D, M, e3, st)) return -1;
        } else {
            e3.out0 = u.f(); e3.ld0 = Fl;
            if (lin_tc(L.up, h_hi.f(), h_lo.f(), D, M, e3, st)) return -1;
            act_fwd(u.f(), Fl, a.f(), Fl, M, Fl, e.act == "silu" ? 2 : e.act == "gelu_tanh" ? 4 : 3, st);
            split_f32(a.f(), Fl, g_hi.f(), g_lo.f(), Fl, M, Fl, st);
        }
        GemmEpi e4;
        e4.mode = EPI_GATED; e4.bias = L.down.b; e4.out0 = a.f(); e4.ld0 = D; e4.aux = X2.f(); e4.ld_aux = D;
        e4.gate = L.ls2; e4.ld_gate = 0; e4.out1 = X.f(); e4.ld1 = D;
        if (lin_tc(L.down, g_hi.f(), g_lo.f(), Fl, M, e4, st)) return -1;
    }
    layer_norm(X.f(), D, E.norm_w, E.norm_b, e.ln_eps, y.f(), D, nullptr, nullptr, nullptr, M, D, st);
    float * data = (float *) malloc(R * D * sizeof(float));
    if (!data) { log("jepa: jepa_encode: out of host memory for %lld rows\n", (long long) rows); return -1; }
    if (!cuda_ok(cudaMemcpyAsync(data, y.p, R * D * 4, cudaMemcpyDeviceToHost, st), "encoder output") ||
        !cuda_ok(cudaStreamSynchronize(st), "jepa_encode")) {
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
    if (gemm_error_flag(st)) { free(data); log("jepa: a tensor-core kernel gave up waiting on its pipeline\n"); return -1; }
    out->data = data;
    out->n_tokens = rows;
    out->dim = D;
    return 0;
}

// mean over the patch tokens (the prefix tokens excluded), double accumulation (src/jepa.cpp:1227-1252)
int jepa_pool_mean(const jepa_model * model, const jepa_output * enc, jepa_output * out) {
    if (!model || !enc || !out || !enc->data) return -1;
    const int64_t skip = (model->enc.cls_token ? 1 : 0) + model->enc.n_registers;
    const int64_t D = enc->dim, n = enc->n_tokens - skip;
    if (D <= 0 || enc->n_tokens <= 0) {
        log("jepa: jepa_pool_mean: encoder output is [%lld tokens, %lld dims]\n", (long long) enc->n_tokens, (long long) D);
        return -1;
    }
    if (n <= 0) return -1;
    out->n_tokens = 1;
    out->dim = D;
    out->data = (float *) calloc((size_t) D, sizeof(float));
    if (!out->data) return -1;
    std::vector<double> acc((size_t) D, 0.0);
    for (int64_t i = skip; i < enc->n_tokens; i++)
        for (int64_t d = 0; d < D; d++) acc[(size_t) d] += enc->data[i * D + d];
    for (int64_t d = 0; d < D; d++) out->data[d] = (float) (acc[(size_t) d] / (double) n);
    return 0;
}

// the CLS row (row 0, after the final norm) (src/jepa.cpp:1254-1270)
int jepa_pool_cls(const jepa_model * model, const jepa_output * enc, jepa_output * out) {
    if (!model || !enc || !out || !enc->data) return -1;
    if (!model->enc.cls_token) { log("jepa: jepa_pool_cls: model has no CLS token\n"); return -1; }
    if (enc->dim <= 0 || enc->n_tokens < 1) {
        log("jepa: jepa_pool_cls: encoder output is [%lld tokens, %lld dims]\n", (long long) enc->n_tokens, (long long) enc->dim);
        return -1;
    }
    out->n_tokens = 1;
    out->dim = enc->dim;
    out->data = (float *) malloc((size_t) enc->dim * sizeof(float));
    if (!out->data) return -1;
    memcpy(out->data, enc->data, (size_t) enc->dim * sizeof(float));
    return 0;
}

}  // extern "C"
