// V-JEPA 2-AC on the GPU: the predictor forward (jepa_build_ac, src/vjepa2_ac.cpp:86-156, over the pre-LN
// block of src/jepa.cpp:444-471), the rollout (ac_rollout, src/vjepa2_ac.cpp:455-577), the cached context
// handle (:604-747), the CEM planner (jepa_ac_plan, :829-946) and the predict entry points (:272-441).
//
// One predictor evaluation ("pass") runs over the rows of a run of consecutive frames for every candidate
// at once, rows laid out [candidate][frame][2 + HW] (action row, state row, patch rows -- the reference's
// interleave, :115-124). Per layer: LayerNorm -> f16, the fused q/k/v GEMM whose epilogue applies 3-D
// RoPE and writes k / v into the frame's cache block, attention over the cached frames, the output GEMM
// with the residual add, LayerNorm, the GELU MLP. A rollout step is one pass over its new frame (the
// frames before it are cached); see ac.h.
#include "ac.h"
#include "model.h"
#include "shard.h"
#include "kprof.h"

#include "../../include/jepa.h"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <memory>
#include <vector>

struct jepa_ac_context {
    jepa_context * owner = nullptr;
    float * slab = nullptr;            // device [cap][HW][E] f32: the observed frames' latents
    int n_frames = 0, cap = 0;
    std::vector<float> actions;        // [cap][A] the actions between the frames
    std::vector<float> states;         // [cap][S] the pose at each frame
    uint64_t gen = 0;                  // bumped whenever the frames, actions or states change
};

namespace jb {

namespace {

uint64_t next_generation() {
    static std::atomic<uint64_t> g{1};
    return g.fetch_add(1);
}

// ---- weights -----------------------------------------------------------------------------------
struct ACUpload {
    ACEngine & e;
    const jepa_model & m;
    cudaStream_t st;
    bool ok = true;
    float * tmp = nullptr;             // dequantised f32 rows of one weight
    size_t tmp_n = 0;
    void * raw = nullptr;
    size_t raw_n = 0;

    ~ACUpload() {
        if (tmp) cudaFree(tmp);
        if (raw) cudaFree(raw);
    }
    template <class T> T * alloc(size_t n) {
        void * p = nullptr;
        if (!ok) return nullptr;
        if (cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)) != cudaSuccess) {
            cudaGetLastError();
            log("jepa: ac predictor: out of device memory while uploading the weights\n");
            ok = false;
            return nullptr;
        }
        e.allocations.push_back(p);
        return (T *) p;
    }
    const gguf_tensor * need(const std::string & name, int64_t ne0, int64_t ne1, bool required) {
        const gguf_tensor * t = m.get(name);
        if (!t) {
            if (required) { log("jepa: ac predictor: tensor '%s' is missing\n", name.c_str()); ok = false; }
            return nullptr;
        }
        if (t->ne[0] != ne0 || t->nelements() != ne0 * ne1) {
            log("jepa: ac predictor: tensor '%s' has shape [%lld, %lld], expected [%lld, %lld]\n", name.c_str(),
                (long long) t->ne[0], (long long) (t->nelements() / std::max<int64_t>(t->ne[0], 1)), (long long) ne0, (long long) ne1);
            ok = false;
            return nullptr;
        }
        return t;
    }
    // a float32 vector (norm weights, biases); nullptr when absent and optional
    const float * vec(const std::string & name, int64_t n, bool required) {
        const gguf_tensor * t = need(name, n, 1, required);
        if (!t || !ok) return nullptr;
        std::vector<float> h((size_t) n);
        dequant_row(t->type, t->data, h.data(), n);
        float * d = alloc<float>((size_t) n);
        if (d) ok = cuda_ok(cudaMemcpyAsync(d, h.data(), (size_t) n * 4, cudaMemcpyHostToDevice, st), "upload") && ok;
        ok = cuda_ok(cudaStreamSynchronize(st), "upload") && ok;
        return d;
    }
    // a [rows][cols] weight dequantised on the device (bit-exact block formats) into f32
    bool dequant(const gguf_tensor * t, int64_t rows, int64_t cols) {
        const size_t rb = row_bytes(t->type, cols);
        const size_t need_raw = rb * (size_t) rows, need_tmp = (size_t) rows * cols;
        if (need_raw > raw_n) {
            if (raw) cudaFree(raw);
            raw = nullptr;
            if (!cuda_ok(cudaMalloc(&raw, need_raw), "weight staging")) { ok = false; return false; }
            raw_n = need_raw;
        }
        if (need_tmp > tmp_n) {
            if (tmp) cudaFree(tmp);
            tmp = nullptr;
            if (!cuda_ok(cudaMalloc(&tmp, need_tmp * 4), "weight staging")) { ok = false; return false; }
            tmp_n = need_tmp;
        }
        ok = cuda_ok(cudaMemcpyAsync(raw, t->data, need_raw, cudaMemcpyHostToDevice, st), "upload") &&
             dequant_rows(t->type, raw, tmp, rows, cols, st) == 0 && ok;
        return ok;
    }
    const __half * mat16(const std::string & name, int64_t rows, int64_t cols) {
        const gguf_tensor * t = need(name, cols, rows, true);
        if (!t || !ok) return nullptr;
        __half * d = alloc<__half>((size_t) rows * cols);
        if (!d || !dequant(t, rows, cols)) return nullptr;
        to_f16(tmp, (int) cols, d, (int) cols, (int) rows, (int) cols, RowMap{}, st);
        ok = cuda_ok(cudaStreamSynchronize(st), "weight conversion") && ok;
        return d;
    }
    const float * mat32(const std::string & name, int64_t rows, int64_t cols) {
        const gguf_tensor * t = need(name, cols, rows, true);
        if (!t || !ok) return nullptr;
        float * d = alloc<float>((size_t) rows * cols);
        if (!d || !dequant(t, rows, cols)) return nullptr;
        ok = cuda_ok(cudaMemcpyAsync(d, tmp, (size_t) rows * cols * 4, cudaMemcpyDeviceToDevice, st), "upload") &&
             cuda_ok(cudaStreamSynchronize(st), "upload") && ok;
        return d;
    }
};

// 3-D RoPE tables (src/rope3d.cpp:9-134 semantics), factorised per axis: per-axis width d = 2((hd/3)/2),
// omega_k = 1 / theta^(k / (d/2)) in float, angle = position * omega (float), tiled layout uses
// omega[j mod d/2] and the interleaved one omega[j / 2]; rows [0, slots) hold the frame axis at t = row,
// rows [slots, slots + grid) the grid-row axis, rows [slots + grid, slots + 2 grid) the grid-column axis.
// The rotation's sign is folded into the even lanes of sin (axis offsets are multiples of d, so a lane's
// parity inside its axis is its parity inside the head). Lanes past 3d keep the identity.
void rope_tables(const ACEngine & e, const ACParams & p, std::vector<float> & cosv, std::vector<float> & sinv) {
    const int d = e.rope_d, half = d / 2, grid = p.grid_size;
    const int n = e.slots + 2 * grid;
    cosv.assign((size_t) std::max(n * d, 1), 1.0f);
    sinv.assign((size_t) std::max(n * d, 1), 0.0f);
    if (d == 0) return;
    std::vector<float> omega((size_t) half);
    for (int k = 0; k < half; k++) omega[(size_t) k] = 1.0f / powf(p.rope_theta, (float) k / (float) half);
    for (int r = 0; r < n; r++) {
        const float pos = (float) (r < e.slots ? r : r < e.slots + grid ? r - e.slots : r - e.slots - grid);
        for (int j = 0; j < d; j++) {
            const int k = p.rope_interleaved ? j / 2 : j % half;
            const float ang = pos * omega[(size_t) k];
            cosv[(size_t) r * d + j] = cosf(ang);
            const float sv = sinf(ang);
            sinv[(size_t) r * d + j] = (j % 2 == 0) ? -sv : sv;
        }
    }
}

}  // namespace

ACEngine::~ACEngine() {
    cudaSetDevice(device);
    for (void * p : allocations) cudaFree(p);
    for (Buf * b : {&ws, &kv_shared, &kv_cand, &outs, &io}) {
        if (b->p) cudaFree(b->p);
    }
}

bool ACEngine::grow(Buf & b, size_t bytes, const char * what) {
    if (bytes <= b.bytes) return true;
    if (b.p) cudaFree(b.p);
    b.p = nullptr;
    b.bytes = 0;
    if (cudaMalloc(&b.p, bytes) != cudaSuccess) {
        cudaGetLastError();
        log("jepa: ac predictor: could not allocate %.1f MiB of device memory for %s\n", bytes / 1048576.0, what);
        b.p = nullptr;
        return false;
    }
    b.bytes = bytes;
    return true;
}

size_t ACEngine::ws_bytes(long long rows) const {
    // X f32 [rows][D]; LN out, q, attention out f16 [rows][D]; MLP hidden f16 [rows][F]
    return (size_t) rows * ((size_t) D * 4 + (size_t) D * 2 * 3 + (size_t) F * 2) + 5 * 256;
}

bool ACEngine::init(const jepa_model & m, cudaStream_t st) {
    const ACParams & p = m.ac;
    device = m.device;
    D = p.embed_dim; E = m.enc.embed_dim; OUT = p.out_dim; F = p.ffn_dim; L = p.n_layer; NH = p.n_head;
    HD = p.head_dim; A = p.action_dim; S = p.state_dim; HW = p.grid_size * p.grid_size; R = p.n_cond_tokens + HW;
    slots = p.n_frames;
    ln_eps = p.ln_eps; norm_eps = p.norm_reps_eps; normalize = p.normalize_reps; causal = p.frame_causal;
    if (p.n_cond_tokens != 2) {
        log("jepa: ac predictor: jepa.pred.n_cond_tokens is %d; the predictor builds exactly 2 conditioning rows per "
            "frame (action, state)\n", p.n_cond_tokens);
        return false;
    }
    if (p.act != "gelu_erf" && p.act != "gelu") {
        log("jepa: ac predictor: activation '%s' is not built into the GPU engine (gelu_erf)\n", p.act.c_str());
        return false;
    }
    if (HD != 16 && HD != 32 && HD != 64) { log("jepa: ac predictor: head width %d is not supported (16, 32, 64)\n", HD); return false; }
    if (NH * HD != D || D % 32 || E % 8 || F % 8 || OUT % 8) {
        log("jepa: ac predictor: widths D %d (heads %d x %d), E %d, F %d, out %d need D = heads x head width, D a multiple "
            "of 32 and the rest multiples of 8\n", D, NH, HD, E, F, OUT);
        return false;
    }
    if (slots < 1 || slots > AC_MAX_FRAMES) { log("jepa: ac predictor: %d frame slots, the engine holds up to %d\n", slots, AC_MAX_FRAMES); return false; }

    ACUpload up{*this, m, st};
    wembed = up.mat16("pred.embed.weight", D, E);
    bembed = up.vec("pred.embed.bias", D, false);
    wact = up.mat32("pred.action_embed.weight", D, A);
    bact = up.vec("pred.action_embed.bias", D, false);
    wst = up.mat32("pred.state_embed.weight", D, S);
    bst = up.vec("pred.state_embed.bias", D, false);
    for (int i = 0; i < L && up.ok; i++) {
        const std::string q = "pred.blk." + std::to_string(i) + ".";
        ACLayer l;
        l.ln1_w = up.vec(q + "ln1.weight", D, false); l.ln1_b = up.vec(q + "ln1.bias", D, false);
        l.ln2_w = up.vec(q + "ln2.weight", D, false); l.ln2_b = up.vec(q + "ln2.bias", D, false);
        l.wqkv = up.mat16(q + "attn_qkv.weight", 3 * (int64_t) D, D); l.bqkv = up.vec(q + "attn_qkv.bias", 3 * (int64_t) D, false);
        l.wout = up.mat16(q + "attn_out.weight", D, D); l.bout = up.vec(q + "attn_out.bias", D, false);
        l.wup = up.mat16(q + "ffn_up.weight", F, D); l.bup = up.vec(q + "ffn_up.bias", F, false);
        l.wdown = up.mat16(q + "ffn_down.weight", D, F); l.bdown = up.vec(q + "ffn_down.bias", D, false);
        layers.push_back(l);
    }
    norm_w = up.vec("pred.norm.weight", D, true);
    norm_b = up.vec("pred.norm.bias", D, false);
    wproj = up.mat16("pred.proj.weight", OUT, D);
    bproj = up.vec("pred.proj.bias", OUT, false);
    if (!up.ok) return false;

    rope_d = 2 * ((HD / 3) / 2);
    grid = p.grid_size;
    std::vector<float> cosv, sinv;
    rope_tables(*this, p, cosv, sinv);
    rope_cos = up.alloc<float>(cosv.size());
    rope_sin = up.alloc<float>(sinv.size());
    if (!up.ok) return false;
    return cuda_ok(cudaMemcpyAsync(rope_cos, cosv.data(), cosv.size() * 4, cudaMemcpyHostToDevice, st), "rope tables") &&
           cuda_ok(cudaMemcpyAsync(rope_sin, sinv.data(), sinv.size() * 4, cudaMemcpyHostToDevice, st), "rope tables") &&
           cuda_ok(cudaStreamSynchronize(st), "rope tables");
}

// One predictor evaluation (see PassSpec). Kernel launches: embed GEMM(s), conditioning rows, per layer
// LN / qkv / attention / out / LN / up / down, final LN / projection / normalisation.
int ACEngine::pass(const PassSpec & p, cudaStream_t st) {
    const long long rows = (long long) p.n_cand * p.nf * R;
    if (rows > 0x7fffffffLL / 4 || p.nf < 1 || p.f0 + p.nf > slots) {
        log("jepa: ac predictor: pass of %d candidates x %d frames from frame %d is out of range\n", p.n_cand, p.nf, p.f0);
        return -1;
    }
    if (!grow(ws, ws_bytes(rows), "the predictor activations")) return -1;
    char * w = (char *) ws.p;
    auto carve = [&](size_t bytes) { char * q = w; w += (bytes + 255) & ~(size_t) 255; return q; };
    float * X = (float *) carve((size_t) rows * D * 4);
    __half * Hn = (__half *) carve((size_t) rows * D * 2);
    __half * Q = (__half *) carve((size_t) rows * D * 2);
    __half * O = (__half *) carve((size_t) rows * D * 2);
    __half * U = (__half *) carve((size_t) rows * F * 2);
    const int M = (int) rows;

    // 1. patch rows: embed each frame's latents (once and broadcast when every candidate shares them)
    for (int k = 0; k < p.nf; k++) {
        AcGemmEpi ep;
        ep.mode = AEPI_F32; ep.bias = bembed; ep.out_f32 = X; ep.ld_f32 = D;
        ep.remap_g = HW; ep.remap_off = k * R + 2;
        if (p.lat_cand[k] == 0) {
            ep.remap_gout = R;
            if (gemm_f16(p.lat[k], E, wembed, E, HW, D, E, ep, st) != 0) return -1;
            KTimer kt("ac_broadcast", st, 0, 8.0 * HW * D * (p.n_cand - 1));
            ac_broadcast_rows(X, D, (long long) p.nf * R, k * R + 2, HW, p.n_cand, D, st);
        } else {
            if (p.lat_cand[k] != (long long) HW * E) { log("jepa: ac predictor: latent rows of a frame must be contiguous\n"); return -1; }
            ep.remap_gout = p.nf * R;
            if (gemm_f16(p.lat[k], E, wembed, E, p.n_cand * HW, D, E, ep, st) != 0) return -1;
        }
    }
    // 2. action / state rows
    {
        KTimer kt("ac_cond_rows", st, 4.0 * p.n_cand * p.nf * D * (A + S), 8.0 * p.n_cand * p.nf * D);
        ac_cond_rows(p.acts, p.act_cand, p.sts, p.st_cand, A, S, wact, bact, wst, bst, X, D, p.n_cand, p.nf, R, D, st);
    }

    // 3. blocks
    AttnArgs at;
    at.q = Q; at.ldq = D; at.q_cand = (long long) p.nf * R * D; at.nq = R; at.n_qframes = p.nf; at.q_frame = R;
    at.out = O; at.ldo = D; at.o_cand = at.q_cand;
    at.key_frames0 = p.full ? p.f0 + p.nf : p.f0 + 1;
    at.key_step = p.full ? 0 : 1;
    at.kv_rows = R; at.ld_kv = 2 * D; at.D = D; at.n_head = NH; at.hd = HD; at.n_cand = p.n_cand;
    at.scale = 1.0f / sqrtf((float) HD);
    for (int l = 0; l < L; l++) {
        const ACLayer & ly = layers[(size_t) l];
        __half * kv = p.kv_out + (size_t) l * p.kv_layer;
        {
            KTimer kt("layer_norm_f16", st, 0, 6.0 * M * D);
            ln_to_f16(X, D, ly.ln1_w, ly.ln1_b, ln_eps, Hn, D, M, D, RowMap{}, st);
        }
        AcGemmEpi eq;
        eq.mode = AEPI_QKV; eq.bias = ly.bqkv; eq.out_f16 = Q; eq.ld_f16 = D; eq.kv = kv; eq.ld_kv = 2 * D;
        eq.rope_cos = rope_cos; eq.rope_sin = rope_sin; eq.rope_d = rope_d; eq.rope_slots = slots; eq.rope_grid = grid;
        eq.rope_slot0 = p.f0; eq.rope_nf = p.nf; eq.rope_frame_rows = R; eq.rope_cond = 2; eq.D = D; eq.hd = HD;
        if (gemm_f16(Hn, D, ly.wqkv, D, M, 3 * D, D, eq, st) != 0) return -1;
        for (int f = 0; f < p.f0; f++) {
            at.kv[f] = p.keys[f].base + (size_t) l * p.keys[f].layer_stride;
            at.kv_cand_stride[f] = p.keys[f].cand_stride;
        }
        for (int k = 0; k < p.nf; k++) {
            at.kv[p.f0 + k] = kv + (size_t) k * R * 2 * D;
            at.kv_cand_stride[p.f0 + k] = (long long) p.nf * R * 2 * D;
        }
        if (attention_f16(at, st) != 0) return -1;
        AcGemmEpi eo;
        eo.mode = AEPI_ADD_F32; eo.bias = ly.bout; eo.out_f32 = X; eo.ld_f32 = D;
        if (gemm_f16(O, D, ly.wout, D, M, D, D, eo, st) != 0) return -1;
        {
            KTimer kt("layer_norm_f16", st, 0, 6.0 * M * D);
            ln_to_f16(X, D, ly.ln2_w, ly.ln2_b, ln_eps, Hn, D, M, D, RowMap{}, st);
        }
        AcGemmEpi eu;
        eu.mode = AEPI_GELU_F16; eu.bias = ly.bup; eu.out_f16 = U; eu.ld_f16 = F;
        if (gemm_f16(Hn, D, ly.wup, D, M, F, D, eu, st) != 0) return -1;
        AcGemmEpi ed;
        ed.mode = AEPI_ADD_F32; ed.bias = ly.bdown; ed.out_f32 = X; ed.ld_f32 = D;
        if (gemm_f16(U, F, ly.wdown, F, M, D, F, ed, st) != 0) return -1;
    }

    // 4. the trailing n_out frames' patch rows: final norm, projection back to the encoder width
    if (p.n_out > 0) {
        const int mo = p.n_cand * p.n_out * HW;
        RowMap g;
        g.g1 = HW; g.g2 = p.n_out; g.s1 = R; g.s2 = p.nf * R; g.off = (p.nf - p.n_out) * R + 2;
        {
            KTimer kt("layer_norm_f16", st, 0, 6.0 * mo * D);
            ln_to_f16(X, D, norm_w, norm_b, ln_eps, Hn, D, mo, D, g, st);
        }
        AcGemmEpi ep;
        ep.mode = AEPI_F32; ep.bias = bproj; ep.out_f32 = p.out; ep.ld_f32 = OUT;
        if (gemm_f16(Hn, D, wproj, D, mo, OUT, D, ep, st) != 0) return -1;
        KTimer kt("ac_normalize", st, 0, (double) mo * OUT * (8.0 + (p.out16 ? 2.0 : 0.0)));
        if (p.normalize) {
            ac_normalize_rows(p.out, OUT, p.out16, OUT, mo, OUT, norm_eps, st);
        } else if (p.out16) {
            to_f16(p.out, OUT, p.out16, OUT, mo, OUT, RowMap{}, st);
        }
    }
    long long n = 1 + 7LL * L;                                        // conditioning rows, 7 per layer
    for (int k = 0; k < p.nf; k++) n += (p.lat_cand[k] == 0 && p.n_cand > 1) ? 2 : 1;
    if (p.n_out > 0) n += 2 + ((p.normalize || p.out16) ? 1 : 0);
    launches += n;
    return cuda_ok(cudaGetLastError(), "ac predictor launch") ? 0 : -1;
}

ACEngine * ac_engine_of(jepa_context * ctx, const char * fn) {
    const jepa_model * m = ctx->model;
    if (!m->ac.present) {
        log("jepa: %s: '%s' has no action-conditioned predictor (jepa.pred.kind = '%s')\n", fn, m->name.c_str(), m->pred_kind.c_str());
        return nullptr;
    }
    cudaSetDevice(ctx->device);
    if (!ctx->ac) {
        auto e = std::make_unique<ACEngine>();
        if (!e->init(*m, ctx->stream)) {
            log("jepa: %s: could not build the ac predictor on CUDA device %d\n", fn, ctx->device);
            return nullptr;
        }
        ctx->ac = std::move(e);
    }
    if (device_flags_clear(ctx->stream)) return nullptr;
    return ctx->ac.get();
}

namespace {

// ---- rollout -------------------------------------------------------------------------------------
struct RolloutReq {
    const __half * seed16 = nullptr;      // device [n_seed][HW][E] f16
    int n_seed = 0;
    const float * seed_actions = nullptr; // host [n_seed-1][A] or nullptr
    const float * seed_states = nullptr;  // host [n_seed][S]
    const float * actions = nullptr;      // host [n_cand][H][A]
    const float * states = nullptr;       // host [n_cand][H][S] or nullptr
    int n_cand = 0, H = 0;
    float * out = nullptr;                // host [n_cand][H][HW][OUT] or nullptr
    const float * goal = nullptr;         // device [HW][OUT]: energies of the last step instead of / besides out
    float * energy = nullptr;             // device [n_cand]
    const void * cache_owner = nullptr;   // shared-prefix cache key (nullptr: no caching)
    uint64_t cache_gen = 0;
};

struct Events {
    cudaEvent_t a = nullptr, b = nullptr;
    Events() { cudaEventCreate(&a); cudaEventCreate(&b); }
    ~Events() { cudaEventDestroy(a); cudaEventDestroy(b); }
};

size_t round256(size_t b) { return (b + 255) & ~(size_t) 255; }

int rollout(ACEngine & e, jepa_context * ctx, const RolloutReq & q, const char * fn) {
    cudaStream_t st = ctx->stream;
    const int n_seq = q.n_seed + q.H - 1;
    const int A = e.A, S = e.S, HW = e.HW, E = e.E, OUT = e.OUT, R = e.R, L = e.L, D = e.D;
    if (q.n_seed <= 0 || q.n_cand <= 0 || q.H <= 0) {
        log("jepa: %s: need n_seed > 0, n_cand > 0 and horizon > 0 (got %d / %d / %d)\n", fn, q.n_seed, q.n_cand, q.H);
        return -1;
    }
    if (n_seq > e.slots) {
        log("jepa: %s: %d seed frames + %d steps reaches a %d-frame context, over the predictor's %d frame slots "
            "(jepa.pred.n_frames)\n", fn, q.n_seed, q.H, n_seq, e.slots);
        return -1;
    }
    if (q.H > 1 && OUT != E) {
        log("jepa: %s: the predictor's output width %d differs from its input width %d, so predictions cannot be fed back\n", fn, OUT, E);
        return -1;
    }
    // per-candidate actions / poses of every frame (identical for every step that sees the frame)
    std::vector<float> acts((size_t) q.n_cand * n_seq * A), sts((size_t) q.n_cand * n_seq * S);
    for (int c = 0; c < q.n_cand; c++) {
        float * ac = acts.data() + (size_t) c * n_seq * A;
        float * sc = sts.data() + (size_t) c * n_seq * S;
        memcpy(sc, q.seed_states, (size_t) q.n_seed * S * sizeof(float));
        for (int j = 0; j < n_seq; j++) {
            if (j < q.n_seed - 1) {
                memcpy(ac + (size_t) j * A, q.seed_actions ? q.seed_actions + (size_t) j * A : q.actions + (size_t) c * q.H * A,
                       (size_t) A * sizeof(float));
                continue;
            }
            const int k = j - (q.n_seed - 1);
            memcpy(ac + (size_t) j * A, q.actions + ((size_t) c * q.H + k) * A, (size_t) A * sizeof(float));
            if (j >= q.n_seed) {
                if (q.states) memcpy(sc + (size_t) j * S, q.states + ((size_t) c * q.H + (j - q.n_seed)) * S, (size_t) S * sizeof(float));
                else jepa_ac_next_state(ctx->model, sc + (size_t) (j - 1) * S, ac + (size_t) (j - 1) * A, sc + (size_t) j * S);
            }
        }
    }
    const bool full = !e.causal;
    const int n_shared = (!full && q.seed_actions) ? q.n_seed - 1 : 0;
    const int nf0 = q.n_seed - n_shared;                 // frames of the first step's pass (causal)
    const long long frame_kv = (long long) R * 2 * D;    // halves of one frame's keys / values

    // per-call inputs
    const size_t io_bytes = round256(acts.size() * 4) + round256(sts.size() * 4);
    if (!e.grow(e.io, io_bytes, "the rollout inputs")) return -1;
    float * acts_d = (float *) e.io.p;
    float * sts_d = (float *) ((char *) e.io.p + round256(acts.size() * 4));
    JB_CUDA(cudaMemcpyAsync(acts_d, acts.data(), acts.size() * 4, cudaMemcpyHostToDevice, st));
    JB_CUDA(cudaMemcpyAsync(sts_d, sts.data(), sts.size() * 4, cudaMemcpyHostToDevice, st));

    // shared frames: computed once per (handle, generation)
    if (n_shared > 0) {
        const size_t need = (size_t) L * n_shared * frame_kv * 2;
        const bool hit = q.cache_owner && e.shared_owner == q.cache_owner && e.shared_gen == q.cache_gen &&
                         e.shared_frames == n_shared && e.kv_shared.bytes >= need;
        if (!hit) {
            e.shared_owner = nullptr;
            if (!e.grow(e.kv_shared, need, "the shared frames' keys and values")) return -1;
            PassSpec p;
            p.n_cand = 1; p.f0 = 0; p.nf = n_shared;
            for (int k = 0; k < n_shared; k++) { p.lat[k] = q.seed16 + (size_t) k * HW * E; p.lat_cand[k] = 0; }
            p.acts = acts_d; p.sts = sts_d; p.act_cand = (long long) n_seq * A; p.st_cand = (long long) n_seq * S;
            p.kv_out = (__half *) e.kv_shared.p; p.kv_layer = (long long) n_shared * frame_kv;
            p.n_out = 0;
            if (e.pass(p, st) != 0) return -1;
            e.shared_owner = q.cache_owner;
            e.shared_gen = q.cache_gen;
            e.shared_frames = n_shared;
        }
    }

    // candidates per chunk: everything that scales with the candidate count has to fit in free memory
    const long long kv_frames = full ? n_seq : (long long) (n_seq - n_shared);
    const long long pass_rows = (long long) (full ? n_seq : nf0) * R;
    const size_t per_cand = (size_t) L * kv_frames * frame_kv * 2 + e.ws_bytes(pass_rows) +
                            (size_t) HW * OUT * 4 + (size_t) q.H * HW * E * 2;
    size_t free_b = 0, total_b = 0;
    JB_CUDA(cudaMemGetInfo(&free_b, &total_b));
    const size_t reusable = e.ws.bytes + e.kv_cand.bytes + e.outs.bytes;
    const size_t avail = free_b + reusable > ((size_t) 2 << 30) ? (free_b + reusable - ((size_t) 2 << 30)) : 0;
    long long kc_max = (long long) (avail * 0.9 / (double) per_cand);
    if (kc_max < 1) {
        log("jepa: %s: one candidate needs %.1f MiB of device memory and %.1f MiB are free\n", fn, per_cand / 1048576.0, free_b / 1048576.0);
        return -1;
    }
    const int Kc = (int) std::min<long long>(std::min<long long>(q.n_cand, kc_max), 65535);
    const size_t kv_bytes = (size_t) L * Kc * kv_frames * frame_kv * 2;
    if (kv_bytes > e.kv_cand.bytes || e.ws_bytes((long long) Kc * pass_rows) > e.ws.bytes) {
        // release before growing so the old buffers do not count against the new ones
        for (ACEngine::Buf * b : {&e.kv_cand, &e.ws}) { if (b->p) cudaFree(b->p); b->p = nullptr; b->bytes = 0; }
    }
    if (!e.grow(e.kv_cand, kv_bytes, "the candidates' keys and values")) return -1;
    const size_t p_bytes = round256((size_t) Kc * HW * OUT * 4);
    const size_t lat_bytes = round256((size_t) Kc * HW * E * 2);
    if (!e.grow(e.outs, p_bytes + (size_t) q.H * lat_bytes, "the rollout outputs")) return -1;
    float * P = (float *) e.outs.p;
    auto lat16 = [&](int s) { return (__half *) ((char *) e.outs.p + p_bytes + (size_t) s * lat_bytes); };
    __half * kvc = (__half *) e.kv_cand.p;

    for (int c0 = 0; c0 < q.n_cand; c0 += Kc) {
        const int kc = std::min(Kc, q.n_cand - c0);
        // cache block of step s (causal): block 0 holds frames n_shared .. n_seed-1, block s >= 1 frame n_seed-1+s
        auto block_off = [&](int s) -> size_t {
            return s == 0 ? 0 : (size_t) L * kc * frame_kv * (nf0 + (s - 1));
        };
        for (int s = 0; s < q.H; s++) {
            PassSpec p;
            p.n_cand = kc;
            if (!full) {
                p.f0 = s == 0 ? n_shared : q.n_seed - 1 + s;
                p.nf = s == 0 ? nf0 : 1;
                if (s == 0) {
                    for (int k = 0; k < p.nf; k++) { p.lat[k] = q.seed16 + (size_t) (p.f0 + k) * HW * E; p.lat_cand[k] = 0; }
                } else {
                    p.lat[0] = lat16(s - 1); p.lat_cand[0] = (long long) HW * E;
                }
                for (int f = 0; f < n_shared; f++) {
                    p.keys[f].base = (const __half *) e.kv_shared.p + (size_t) f * frame_kv;
                    p.keys[f].layer_stride = (long long) n_shared * frame_kv;
                    p.keys[f].cand_stride = 0;
                }
                for (int k = 0; k < nf0 && s > 0; k++) {
                    p.keys[n_shared + k].base = kvc + (size_t) k * frame_kv;
                    p.keys[n_shared + k].layer_stride = (long long) kc * nf0 * frame_kv;
                    p.keys[n_shared + k].cand_stride = (long long) nf0 * frame_kv;
                }
                for (int b = 1; b < s; b++) {
                    KVRef & r = p.keys[q.n_seed - 1 + b];
                    r.base = kvc + block_off(b);
                    r.layer_stride = (long long) kc * frame_kv;
                    r.cand_stride = frame_kv;
                }
                p.kv_out = kvc + block_off(s);
                p.kv_layer = (long long) kc * p.nf * frame_kv;
            } else {
                p.f0 = 0;
                p.nf = q.n_seed + s;
                p.full = true;
                for (int k = 0; k < p.nf; k++) {
                    if (k < q.n_seed) { p.lat[k] = q.seed16 + (size_t) k * HW * E; p.lat_cand[k] = 0; }
                    else { p.lat[k] = lat16(k - q.n_seed); p.lat_cand[k] = (long long) HW * E; }
                }
                p.kv_out = kvc;
                p.kv_layer = (long long) kc * p.nf * frame_kv;
            }
            p.acts = acts_d + ((size_t) c0 * n_seq + p.f0) * A; p.act_cand = (long long) n_seq * A;
            p.sts = sts_d + ((size_t) c0 * n_seq + p.f0) * S; p.st_cand = (long long) n_seq * S;
            p.n_out = 1;
            p.out = P;
            p.out16 = s + 1 < q.H ? lat16(s) : nullptr;
            p.normalize = e.normalize;
            if (e.pass(p, st) != 0) return -1;
            if (q.out) {
                JB_CUDA(cudaMemcpy2DAsync(q.out + ((size_t) c0 * q.H + s) * HW * OUT, (size_t) q.H * HW * OUT * 4, P,
                                          (size_t) HW * OUT * 4, (size_t) HW * OUT * 4, (size_t) kc, cudaMemcpyDeviceToHost, st));
            }
            if (s + 1 == q.H && q.energy) {
                KTimer kt("ac_energy", st, 3.0 * kc * HW * OUT, 4.0 * ((double) kc + 1) * HW * OUT);
                ac_energy(P, (long long) HW * OUT, q.goal, (long long) HW * OUT, kc, q.energy + c0, st);
                e.launches++;
            }
        }
    }
    JB_CUDA(cudaStreamSynchronize(st));
    if (gemm_f16_error_flag(st) != 0 || attention_tc_error_flag(st) != 0) {
        log("jepa: %s: a tensor-core kernel timed out waiting on its pipeline; results are invalid\n", fn);
        return -1;
    }
    return 0;
}

// seed latents: host f32 rows -> device f16
const __half * upload_seed16(ACEngine & e, jepa_context * ctx, const float * host, int n_frames, ACEngine::Buf & buf) {
    const size_t n = (size_t) n_frames * e.HW * e.E;
    if (!e.grow(buf, round256(n * 4) + round256(n * 2), "the context latents")) return nullptr;
    float * f = (float *) buf.p;
    __half * h = (__half *) ((char *) buf.p + round256(n * 4));
    if (!cuda_ok(cudaMemcpyAsync(f, host, n * 4, cudaMemcpyHostToDevice, ctx->stream), "context upload")) return nullptr;
    to_f16(f, e.E, h, e.E, n_frames * e.HW, e.E, RowMap{}, ctx->stream);
    e.launches++;
    return h;
}

struct ScratchBuf {
    ACEngine::Buf b;
    ~ScratchBuf() { if (b.p) cudaFree(b.p); }
};

bool ac_ok(jepa_context * ctx, const char * fn) {
    if (!ctx->model->ac.present) {
        log("jepa: %s: '%s' has no action-conditioned predictor (jepa.pred.kind = '%s')\n", fn, ctx->model->name.c_str(),
            ctx->model->pred_kind.c_str());
        return false;
    }
    return true;
}

// The draws a plan uses when the caller passes no noise: xorshift128+ (shifts 23, 17, 26) seeded from
// `seed` and advanced 8 outputs, the top 53 bits of an output scaled into (0, 1], and one normal from two
// such uniforms by Box-Muller's cosine branch -- the generator of the reference planner
// (src/vjepa2_ac.cpp:807-826), so that a seeded plan samples what the reference samples.
class CemDraws {
  public:
    explicit CemDraws(uint32_t seed) : s0_(0x9E3779B97F4A7C15ull ^ seed), s1_(0xBF58476D1CE4E5B9ull + seed) {
        for (int i = 0; i < 8; i++) advance();
    }
    void fill(float * out, size_t n) {
        for (size_t i = 0; i < n; i++) out[i] = normal();
    }

  private:
    uint64_t advance() {
        uint64_t t = s0_;
        const uint64_t u = s1_;
        s0_ = u;
        t ^= t << 23;
        s1_ = t ^ u ^ (t >> 17) ^ (u >> 26);
        return s1_ + u;
    }
    float unit() { return (float) (((advance() >> 11) + 1) * (1.0 / 9007199254740993.0)); }
    float normal() {
        const float r = unit(), phase = unit();
        return sqrtf(-2.0f * logf(r)) * cosf(6.2831853071795864769f * phase);
    }
    uint64_t s0_, s1_;
};

int predict(jepa_context * ctx, const float * context, int T, int B, const float * actions, const float * states, bool all,
            jepa_output * out, const char * fn) {
    if (!ctx || !context || !actions || !states || !out) return -1;
    if (!ac_ok(ctx, fn)) return -1;
    ACEngine * e = ac_engine_of(ctx, fn);
    if (!e) return -1;
    if (T <= 0 || B <= 0) { log("jepa: %s: need n_frames > 0 and n_batch > 0 (got %d / %d)\n", fn, T, B); return -1; }
    if (T > e->slots) {
        log("jepa: %s: %d context frames, but the predictor's block-causal mask was built for %d frame slots "
            "(jepa.pred.n_frames)\n", fn, T, e->slots);
        return -1;
    }
    cudaStream_t st = ctx->stream;
    const int HW = e->HW, E = e->E, OUT = e->OUT, R = e->R, A = e->A, S = e->S, L = e->L;
    const int n_out = all ? T : 1;
    const long long frame_kv = (long long) R * 2 * e->D;
    const size_t per_cand = (size_t) T * HW * E * 6 + (size_t) L * T * frame_kv * 2 + e->ws_bytes((long long) T * R) +
                            (size_t) n_out * HW * OUT * 4;
    size_t free_b = 0, total_b = 0;
    JB_CUDA(cudaMemGetInfo(&free_b, &total_b));
    const size_t reusable = e->ws.bytes + e->kv_cand.bytes + e->outs.bytes + e->io.bytes;
    const size_t avail = free_b + reusable > ((size_t) 2 << 30) ? (free_b + reusable - ((size_t) 2 << 30)) : 0;
    const long long kc_max = (long long) (avail * 0.9 / (double) per_cand);
    if (kc_max < 1) { log("jepa: %s: one batch item needs %.1f MiB of device memory\n", fn, per_cand / 1048576.0); return -1; }
    const int Kc = (int) std::min<long long>(std::min<long long>(B, kc_max), 65535);

    Events ev;
    const long long l0 = e->launches;
    cudaEventRecord(ev.a, st);
    out->n_tokens = (int64_t) n_out * HW * B;
    out->dim = OUT;
    out->data = (float *) malloc((size_t) out->n_tokens * OUT * sizeof(float));
    if (!out->data) return -1;
    auto fail = [&]() { free(out->data); out->data = nullptr; out->n_tokens = out->dim = 0; return -1; };
    for (ACEngine::Buf * b : {&e->kv_cand, &e->ws, &e->outs, &e->io}) {
        if (b->p) cudaFree(b->p);
        b->p = nullptr;
        b->bytes = 0;
    }
    const size_t ctx_f32 = round256((size_t) Kc * T * HW * E * 4), ctx_f16 = round256((size_t) Kc * T * HW * E * 2);
    const size_t as_bytes = round256((size_t) Kc * T * A * 4) + round256((size_t) Kc * T * S * 4);
    if (!e->grow(e->io, ctx_f32 + ctx_f16 + as_bytes, "the context") ||
        !e->grow(e->kv_cand, (size_t) L * Kc * T * frame_kv * 2, "the keys and values") ||
        !e->grow(e->outs, round256((size_t) Kc * n_out * HW * OUT * 4), "the predictions")) {
        return fail();
    }
    float * cf = (float *) e->io.p;
    __half * ch = (__half *) ((char *) e->io.p + ctx_f32);
    float * ad = (float *) ((char *) e->io.p + ctx_f32 + ctx_f16);
    float * sd = (float *) ((char *) ad + round256((size_t) Kc * T * A * 4));
    e->shared_owner = nullptr;
    for (int c0 = 0; c0 < B; c0 += Kc) {
        const int kc = std::min(Kc, B - c0);
        if (!cuda_ok(cudaMemcpyAsync(cf, context + (size_t) c0 * T * HW * E, (size_t) kc * T * HW * E * 4, cudaMemcpyHostToDevice, st), "upload") ||
            !cuda_ok(cudaMemcpyAsync(ad, actions + (size_t) c0 * T * A, (size_t) kc * T * A * 4, cudaMemcpyHostToDevice, st), "upload") ||
            !cuda_ok(cudaMemcpyAsync(sd, states + (size_t) c0 * T * S, (size_t) kc * T * S * 4, cudaMemcpyHostToDevice, st), "upload")) {
            return fail();
        }
        // frame-major f16 copy: frame k of item c at ch + (k kc + c) HW E
        for (int k = 0; k < T; k++) {
            RowMap m;
            m.g1 = HW; m.g2 = 1; m.s2 = T * HW; m.off = k * HW;
            to_f16(cf, E, ch + (size_t) k * kc * HW * E, E, kc * HW, E, m, st);
            e->launches++;
        }
        PassSpec p;
        p.n_cand = kc; p.f0 = 0; p.nf = T; p.full = !e->causal;
        for (int k = 0; k < T; k++) { p.lat[k] = ch + (size_t) k * kc * HW * E; p.lat_cand[k] = (long long) HW * E; }
        p.acts = ad; p.act_cand = (long long) T * A; p.sts = sd; p.st_cand = (long long) T * S;
        p.kv_out = (__half *) e->kv_cand.p; p.kv_layer = (long long) kc * T * frame_kv;
        p.n_out = n_out; p.out = (float *) e->outs.p;
        if (e->pass(p, st) != 0) return fail();
        if (!cuda_ok(cudaMemcpyAsync(out->data + (size_t) c0 * n_out * HW * OUT, e->outs.p, (size_t) kc * n_out * HW * OUT * 4,
                                     cudaMemcpyDeviceToHost, st), "download")) {
            return fail();
        }
    }
    cudaEventRecord(ev.b, st);
    if (!cuda_ok(cudaStreamSynchronize(st), fn)) return fail();
    if (gemm_f16_error_flag(st) != 0 || attention_tc_error_flag(st) != 0) {
        log("jepa: %s: a tensor-core kernel timed out waiting on its pipeline\n", fn);
        return fail();
    }
    float ms = 0;
    cudaEventElapsedTime(&ms, ev.a, ev.b);
    ctx->last_ms = ms;
    ctx->last_launches = e->launches - l0;
    return 0;
}

int rollout_host(jepa_context * ctx, const float * context, int n_seed, const float * seed_actions, const float * seed_states,
                 const float * actions, const float * states, int n_cand, int horizon, float * out, const char * fn) {
    if (!ctx || !context || !seed_states || !actions || !out) return -1;
    if (!ac_ok(ctx, fn)) return -1;
    ACEngine * e = ac_engine_of(ctx, fn);
    if (!e) return -1;
    if (n_seed <= 0 || n_seed > e->slots) {
        log("jepa: %s: need 0 < n_seed <= %d frame slots (got %d)\n", fn, e->slots, n_seed);
        return -1;
    }
    ScratchBuf seed;
    Events ev;
    const long long l0 = e->launches;
    cudaEventRecord(ev.a, ctx->stream);
    const __half * s16 = upload_seed16(*e, ctx, context, n_seed, seed.b);
    if (!s16) return -1;
    RolloutReq q;
    q.seed16 = s16; q.n_seed = n_seed; q.seed_actions = seed_actions; q.seed_states = seed_states;
    q.actions = actions; q.states = states; q.n_cand = n_cand; q.H = horizon; q.out = out;
    const int rc = rollout(*e, ctx, q, fn);
    cudaEventRecord(ev.b, ctx->stream);
    cudaStreamSynchronize(ctx->stream);
    float ms = 0;
    cudaEventElapsedTime(&ms, ev.a, ev.b);
    ctx->last_ms = ms;
    ctx->last_launches = e->launches - l0;
    return rc;
}

}  // namespace

}  // namespace jb

using namespace jb;

extern "C" {

int jepa_ac_predict(jepa_context * ctx, const float * context, int n_frames, int n_batch, const float * actions,
                    const float * states, jepa_output * out) {
    return predict(ctx, context, n_frames, n_batch, actions, states, false, out, "jepa_ac_predict");
}

int jepa_ac_predict_all(jepa_context * ctx, const float * context, int n_frames, int n_batch, const float * actions,
                        const float * states, jepa_output * out) {
    return predict(ctx, context, n_frames, n_batch, actions, states, true, out, "jepa_ac_predict_all");
}

int jepa_ac_rollout_ex(jepa_context * ctx, const float * context, int n_seed, const float * seed_actions,
                       const float * seed_states, const float * actions, const float * states, int n_cand, int horizon,
                       float * out) {
    return rollout_host(ctx, context, n_seed, seed_actions, seed_states, actions, states, n_cand, horizon, out,
                        "jepa_ac_rollout_ex");
}

int jepa_ac_rollout(jepa_context * ctx, const float * context, int n_seed, const float * seed_states, const float * actions,
                    const float * states, int n_cand, int horizon, float * out) {
    return rollout_host(ctx, context, n_seed, nullptr, seed_states, actions, states, n_cand, horizon, out, "jepa_ac_rollout");
}

jepa_ac_context * jepa_ac_context_new(jepa_context * ctx, const float * latents, int n_frames, const float * actions,
                                      const float * states) {
    if (!ctx || !latents || !states || n_frames <= 0) return nullptr;
    if (!ac_ok(ctx, "jepa_ac_context_new")) return nullptr;
    const ACParams & p = ctx->model->ac;
    const int HW = p.grid_size * p.grid_size, E = ctx->model->enc.embed_dim;
    const int cap = p.n_frames > 0 ? p.n_frames : n_frames;
    if (n_frames > cap) {
        log("jepa: jepa_ac_context_new: %d frames, but the predictor has %d frame slots (jepa.pred.n_frames)\n", n_frames, cap);
        return nullptr;
    }
    cudaSetDevice(ctx->device);
    auto h = std::make_unique<jepa_ac_context>();
    h->owner = ctx;
    h->cap = cap;
    h->n_frames = n_frames;
    const size_t bytes = (size_t) cap * HW * E * sizeof(float);
    if (cudaMalloc((void **) &h->slab, bytes) != cudaSuccess) {
        cudaGetLastError();
        log("jepa: jepa_ac_context_new: cannot allocate %.1f MiB on CUDA device %d\n", bytes / 1048576.0, ctx->device);
        return nullptr;
    }
    if (!cuda_ok(cudaMemcpy(h->slab, latents, (size_t) n_frames * HW * E * sizeof(float), cudaMemcpyHostToDevice), "context upload")) {
        cudaFree(h->slab);
        return nullptr;
    }
    h->actions.assign((size_t) cap * p.action_dim, 0.0f);
    h->states.assign((size_t) cap * p.state_dim, 0.0f);
    memcpy(h->states.data(), states, (size_t) n_frames * p.state_dim * sizeof(float));
    if (actions && n_frames > 1) memcpy(h->actions.data(), actions, (size_t) (n_frames - 1) * p.action_dim * sizeof(float));
    h->gen = next_generation();
    return h.release();
}

void jepa_ac_context_free(jepa_ac_context * h) {
    if (!h) return;
    if (h->slab) {
        cudaSetDevice(h->owner->device);
        cudaFree(h->slab);
    }
    delete h;
}

int jepa_ac_context_n_frames(const jepa_ac_context * h) { return h ? h->n_frames : 0; }
int jepa_ac_context_capacity(const jepa_ac_context * h) { return h ? h->cap : 0; }

int jepa_ac_context_update(jepa_ac_context * h, const float * latents, const float * action, const float * state) {
    if (!h || !latents || !action || !state) return -1;
    const ACParams & p = h->owner->model->ac;
    const int HW = p.grid_size * p.grid_size, E = h->owner->model->enc.embed_dim;
    if (h->n_frames >= h->cap) {
        log("jepa: jepa_ac_context_update: the handle holds %d frames, its capacity (and the predictor's frame slots) is %d "
            "-- call jepa_ac_context_trim first\n", h->n_frames, h->cap);
        return -1;
    }
    cudaSetDevice(h->owner->device);
    if (!cuda_ok(cudaMemcpy(h->slab + (size_t) h->n_frames * HW * E, latents, (size_t) HW * E * sizeof(float), cudaMemcpyHostToDevice),
                 "context update")) {
        return -1;
    }
    memcpy(h->actions.data() + (size_t) (h->n_frames - 1) * p.action_dim, action, (size_t) p.action_dim * sizeof(float));
    memcpy(h->states.data() + (size_t) h->n_frames * p.state_dim, state, (size_t) p.state_dim * sizeof(float));
    h->n_frames++;
    h->gen = next_generation();
    return 0;
}

int jepa_ac_context_trim(jepa_ac_context * h, int n_keep) {
    if (!h || n_keep <= 0) return -1;
    if (n_keep >= h->n_frames) return 0;
    const ACParams & p = h->owner->model->ac;
    const int HW = p.grid_size * p.grid_size, E = h->owner->model->enc.embed_dim;
    const int drop = h->n_frames - n_keep;
    cudaSetDevice(h->owner->device);
    // the kept frames move to the front; device-to-device through a temporary (the ranges may overlap)
    float * tmp = nullptr;
    const size_t bytes = (size_t) n_keep * HW * E * sizeof(float);
    if (!cuda_ok(cudaMalloc((void **) &tmp, bytes), "context trim")) return -1;
    const bool ok = cuda_ok(cudaMemcpy(tmp, h->slab + (size_t) drop * HW * E, bytes, cudaMemcpyDeviceToDevice), "context trim") &&
                    cuda_ok(cudaMemcpy(h->slab, tmp, bytes, cudaMemcpyDeviceToDevice), "context trim");
    cudaFree(tmp);
    if (!ok) return -1;
    memmove(h->actions.data(), h->actions.data() + (size_t) drop * p.action_dim, (size_t) (n_keep - 1) * p.action_dim * sizeof(float));
    memmove(h->states.data(), h->states.data() + (size_t) drop * p.state_dim, (size_t) n_keep * p.state_dim * sizeof(float));
    h->n_frames = n_keep;
    h->gen = next_generation();
    return 0;
}

int jepa_ac_rollout_cached(jepa_context * ctx, jepa_ac_context * h, const float * actions, const float * states, int n_cand,
                           int horizon, float * out) {
    if (!ctx || !h || !actions || !out) return -1;
    if (!ac_ok(ctx, "jepa_ac_rollout_cached")) return -1;
    if (h->owner != ctx) {
        log("jepa: jepa_ac_rollout_cached: the handle was built for a different jepa_context; its latents live on that "
            "context's device\n");
        return -1;
    }
    ACEngine * e = ac_engine_of(ctx, "jepa_ac_rollout_cached");
    if (!e) return -1;
    ScratchBuf seed;
    Events ev;
    const long long l0 = e->launches;
    cudaEventRecord(ev.a, ctx->stream);
    const size_t n = (size_t) h->n_frames * e->HW * e->E;
    if (!e->grow(seed.b, n * 2, "the context latents")) return -1;
    to_f16(h->slab, e->E, (__half *) seed.b.p, e->E, h->n_frames * e->HW, e->E, RowMap{}, ctx->stream);
    e->launches++;
    RolloutReq q;
    q.seed16 = (const __half *) seed.b.p; q.n_seed = h->n_frames;
    q.seed_actions = h->n_frames > 1 ? h->actions.data() : nullptr; q.seed_states = h->states.data();
    q.actions = actions; q.states = states; q.n_cand = n_cand; q.H = horizon; q.out = out;
    q.cache_owner = h; q.cache_gen = h->gen;
    const int rc = rollout(*e, ctx, q, "jepa_ac_rollout_cached");
    cudaEventRecord(ev.b, ctx->stream);
    cudaStreamSynchronize(ctx->stream);
    float ms = 0;
    cudaEventElapsedTime(&ms, ev.a, ev.b);
    ctx->last_ms = ms;
    ctx->last_launches = e->launches - l0;
    return rc;
}

// CEM planning (reference interface: include/jepa.h:471-510; the loop of Meta's mpc_utils.py::cem as the
// reference runs it). The sampling distribution (mean and std per horizon step over translation and the
// gripper) and the whole draw stream live on the device; per iteration:
//   k_cem_sample  -> every candidate's actions (all K on every rank, so all ranks hold the same elites)
//   rollout       -> the rank's candidates through the cached context, L1 energy of the final frame
//   ncclAllGather -> every rank's energies (sharded only)
//   k_cem_refit   -> stable top-k elites, their mean and unbiased std, the momentum update
// The host copies each iteration's actions back (the rollout derives the poses from them with the double
// precision pose update) and, at the end, the mean: the plan is the mean with the rotation lanes zero and
// gripper commands below round_gripper dropped.
int jepa_ac_plan(jepa_context * ctx, jepa_ac_context * handle, const float * goal, const jepa_ac_cem_params * params,
                 const float * noise, float * out_actions, float * out_energy) {
    if (!ctx || !handle || !goal || !params || !out_actions) return -1;
    if (!ac_ok(ctx, "jepa_ac_plan")) return -1;
    const jepa_ac_cem_params & q = *params;
    if (q.samples < 1 || q.topk < 1 || q.topk > q.samples || q.cem_steps < 1 || q.horizon < 1) {
        log("jepa: jepa_ac_plan: samples %d, topk %d, cem_steps %d, horizon %d: all must be positive and topk <= samples\n",
            q.samples, q.topk, q.cem_steps, q.horizon);
        return -1;
    }
    const int A = ctx->model->ac.action_dim;
    if (A < 7) {
        log("jepa: jepa_ac_plan: CEM moves action lanes 0-2 (translation) and 6 (gripper); this model's actions have %d lanes\n", A);
        return -1;
    }
    if (handle->owner != ctx) {
        log("jepa: jepa_ac_plan: this context handle belongs to another jepa_context\n");
        return -1;
    }
    ACEngine * e = ac_engine_of(ctx, "jepa_ac_plan");
    if (!e) return -1;
    cudaStream_t st = ctx->stream;
    const int K = q.samples, H = q.horizon, iters = q.cem_steps;
    Shard * sh = ctx->shard.get();
    const int world = sh ? sh->world : 1, rank = sh ? sh->rank : 0;
    const int Kr = (K + world - 1) / world;
    const int lo = std::min(K, rank * Kr), hi = std::min(K, lo + Kr);

    // the draws of every iteration, in the order (iteration, horizon step, candidate, lane)
    const size_t per_iter = (size_t) H * K * 4;
    std::vector<float> own;
    const float * draws = noise;
    if (!draws) {
        own.resize(per_iter * iters);
        CemDraws(q.seed).fill(own.data(), own.size());
        draws = own.data();
    }
    // the starting distribution: mean 0, std maxnorm on translation and 1 on the gripper
    std::vector<float> dist((size_t) 8 * H, 0.0f);
    for (int h = 0; h < H; h++) {
        float * sd = dist.data() + (size_t) 4 * H + (size_t) 4 * h;
        sd[0] = sd[1] = sd[2] = q.maxnorm;
        sd[3] = 1.0f;
    }
    // device: goal, draws, distribution, actions, energies (the rank's, padded to Kr; all ranks'), per-iteration
    // best energies, elite indices
    const size_t goal_n = (size_t) e->HW * e->OUT;
    const size_t sizes[] = {goal_n * 4, per_iter * iters * 4, dist.size() * 4, (size_t) K * H * A * 4, (size_t) Kr * 4,
                            (size_t) Kr * world * 4, (size_t) iters * 4, (size_t) q.topk * 4};
    size_t total = 0;
    for (size_t b : sizes) total += round256(b);
    ScratchBuf dev, seed;
    if (!e->grow(dev.b, total, "the plan buffers")) return -1;
    char * cur = (char *) dev.b.p;
    auto carve = [&](size_t b) { char * p = cur; cur += round256(b); return p; };
    float * goal_d = (float *) carve(sizes[0]);
    float * draws_d = (float *) carve(sizes[1]);
    float * dist_d = (float *) carve(sizes[2]);
    float * acts_d = (float *) carve(sizes[3]);
    float * en_d = (float *) carve(sizes[4]);
    float * all_d = (float *) carve(sizes[5]);
    float * best_d = (float *) carve(sizes[6]);
    int * elite_d = (int *) carve(sizes[7]);
    float * mean_d = dist_d, * sd_d = dist_d + (size_t) 4 * H;

    Events ev;
    const long long l0 = e->launches;
    cudaEventRecord(ev.a, st);
    JB_CUDA(cudaMemcpyAsync(goal_d, goal, goal_n * 4, cudaMemcpyHostToDevice, st));
    JB_CUDA(cudaMemcpyAsync(draws_d, draws, per_iter * iters * 4, cudaMemcpyHostToDevice, st));
    JB_CUDA(cudaMemcpyAsync(dist_d, dist.data(), dist.size() * 4, cudaMemcpyHostToDevice, st));
    JB_CUDA(cudaMemsetAsync(en_d, 0, (size_t) Kr * 4, st));
    const size_t n_seed_el = (size_t) handle->n_frames * e->HW * e->E;
    if (!e->grow(seed.b, n_seed_el * 2, "the context latents")) return -1;
    to_f16(handle->slab, e->E, (__half *) seed.b.p, e->E, handle->n_frames * e->HW, e->E, RowMap{}, st);
    e->launches++;
    auto wait = [&](const char * what) { return world > 1 ? sh->finish(st, what) : cuda_ok(cudaStreamSynchronize(st), what); };

    std::vector<float> acts((size_t) K * H * A);
    for (int it = 0; it < iters; it++) {
        cem_sample(draws_d + per_iter * it, mean_d, sd_d, K, H, A, q.maxnorm, q.gripper_clamp, acts_d, st);
        e->launches++;
        JB_CUDA(cudaMemcpyAsync(acts.data(), acts_d, acts.size() * 4, cudaMemcpyDeviceToHost, st));
        if (!wait("jepa_ac_plan")) return -1;
        if (hi > lo) {
            RolloutReq rq;
            rq.seed16 = (const __half *) seed.b.p; rq.n_seed = handle->n_frames;
            rq.seed_actions = handle->n_frames > 1 ? handle->actions.data() : nullptr; rq.seed_states = handle->states.data();
            rq.actions = acts.data() + (size_t) lo * H * A; rq.n_cand = hi - lo; rq.H = H;
            rq.goal = goal_d; rq.energy = en_d;
            rq.cache_owner = handle; rq.cache_gen = handle->gen;
            if (rollout(*e, ctx, rq, "jepa_ac_plan") != 0) return -1;
        }
        // all ranks' energies in candidate order: rank r's slots [r Kr, r Kr + Kr) hold candidates r Kr ..
        const float * energies = en_d;
        if (world > 1) {
            if (!sh->allgather_f32(en_d, all_d, (size_t) Kr, st)) return -1;
            energies = all_d;
        }
        cem_refit(energies, acts_d, mean_d, sd_d, best_d + it, elite_d, K, H, A, q.topk, q.momentum_mean, q.momentum_std,
                  q.momentum_mean_gripper, q.momentum_std_gripper, st);
        e->launches++;
    }
    std::vector<float> best((size_t) iters);
    JB_CUDA(cudaMemcpyAsync(dist.data(), dist_d, dist.size() * 4, cudaMemcpyDeviceToHost, st));
    JB_CUDA(cudaMemcpyAsync(best.data(), best_d, best.size() * 4, cudaMemcpyDeviceToHost, st));
    cudaEventRecord(ev.b, st);
    if (!wait("jepa_ac_plan")) return -1;
    if (out_energy) std::copy(best.begin(), best.end(), out_energy);
    for (int h = 0; h < H; h++) {
        const float * m = dist.data() + (size_t) 4 * h;
        float * a = out_actions + (size_t) h * A;
        std::fill(a, a + A, 0.0f);
        a[0] = m[0];
        a[1] = m[1];
        a[2] = m[2];
        a[6] = fabsf(m[3]) < q.round_gripper ? 0.0f : m[3];
    }
    float ms = 0;
    cudaEventElapsedTime(&ms, ev.a, ev.b);
    ctx->last_ms = ms;
    ctx->last_launches = e->launches - l0;
    return 0;
}

}  // extern "C"
