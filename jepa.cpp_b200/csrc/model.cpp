// Model loading (GGUF -> hyper-parameters + host tensors), load-time validation of the H-JEPA tensors,
// and the lifecycle / introspection / device entry points of the C API.
//
// The keys are the jepa.* GGUF schema (the reference's docs/gguf-schema.md): required encoder keys, a range
// on the integers a file supplies, the per-level jepa.hjepa.* arrays with one entry per level. A file that
// fails a check is refused with a message naming the key or tensor, never loaded half-way.
#include "model.h"
#include "hplan.h"
#include "shard.h"
#include "ac.h"
#include "encoder.h"

#include "../../include/jepa_b200.h"

#include <algorithm>
#include <cinttypes>
#include <climits>
#include <cmath>
#include <cstdlib>
#include <cstring>

namespace jb {

namespace {

// Reads jepa.* metadata into the hyper-parameter structs. Each call names a key, its destination, its
// default and, for integers, the range a file may hold; the first key that is missing (when required),
// out of range or, for a per-level array, not one value per level, is logged and makes ok() false --
// later calls then do nothing, so a file is refused at its first bad key.
class KeyReader {
  public:
    explicit KeyReader(const gguf_file & g) : g_(g) {}
    bool ok() const { return ok_; }

    KeyReader & need(std::initializer_list<const char *> keys) {
        for (const char * k : keys) {
            if (ok_ && !g_.has(k)) fail("the file lacks the key %s\n", k);
        }
        return *this;
    }
    KeyReader & num(const char * key, int & dst, int def, int64_t lo = INT32_MIN, int64_t hi = INT32_MAX) {
        if (!ok_) return *this;
        dst = g_.geti(key, def);
        if (dst < lo || dst > hi) fail("%s holds %d, outside %lld..%lld\n", key, dst, (long long) lo, (long long) hi);
        return *this;
    }
    KeyReader & real(const char * key, float & dst, float def, float lo = -INFINITY, float hi = INFINITY) {
        if (!ok_) return *this;
        dst = g_.getf(key, def);
        if (!(dst >= lo && dst <= hi)) fail("%s holds %g, outside [%g, %g]\n", key, (double) dst, (double) lo, (double) hi);
        return *this;
    }
    KeyReader & flag(const char * key, bool & dst, bool def) {
        if (ok_) dst = g_.getb(key, def);
        return *this;
    }
    KeyReader & text(const char * key, std::string & dst, const char * def) {
        if (ok_) dst = g_.gets(key, def);
        return *this;
    }
    // an integer array with one value per level, each in lo..hi, into member `field` of every level
    KeyReader & per_level(const char * key, std::vector<HLevel> & levels, int HLevel::* field, int lo, int hi) {
        if (!ok_) return *this;
        const std::vector<int> v = g_.get_iarr(key);
        if (!same_count(key, v.size(), levels.size())) return *this;
        for (size_t i = 0; i < v.size() && ok_; i++) {
            if (v[i] < lo || v[i] > hi) fail("%s[%zu] holds %d, outside %d..%d\n", key, i, v[i], lo, hi);
            else levels[i].*field = v[i];
        }
        return *this;
    }
    KeyReader & per_level(const char * key, std::vector<HLevel> & levels, std::string HLevel::* field) {
        if (!ok_) return *this;
        const std::vector<std::string> v = g_.get_sarr(key);
        if (!same_count(key, v.size(), levels.size())) return *this;
        for (size_t i = 0; i < v.size(); i++) levels[i].*field = v[i];
        return *this;
    }
    template <class... Args> void fail(const char * fmt, Args... args) {
        std::string f = std::string("jepa: ") + fmt;
        log(f.c_str(), args...);
        ok_ = false;
    }

  private:
    bool same_count(const char * key, size_t have, size_t levels) {
        if (have == levels) return true;
        fail("%s has %zu entries for %zu levels (one per level is required)\n", key, have, levels);
        return false;
    }
    const gguf_file & g_;
    bool ok_ = true;
};

constexpr int MAX_WIDTH = 65536, MAX_DEPTH = 1024, MAX_FFN = 1048576, MAX_FRAMES = 65536;

bool parse(jepa_model & m) {
    const gguf_file & g = *m.file;
    if (g.gets("general.architecture", "") != "jepa") {
        log("jepa: general.architecture is '%s'; this loader reads 'jepa' files only\n", g.gets("general.architecture", "").c_str());
        return false;
    }
    m.name = g.gets("general.name", "");
    m.family = g.gets("jepa.family", "");
    m.modality = g.gets("jepa.modality", "image");
    m.file_type = (uint32_t) g.geti("general.file_type", 0);
    static const char * const families[] = {"ijepa", "vjepa", "vjepa2", "vjepa2_1", "levjepa", "hfvit", "lewm", "hjepa"};
    if (std::none_of(std::begin(families), std::end(families), [&](const char * f) { return m.family == f; })) {
        log("jepa: jepa.family '%s' is not one this loader knows\n", m.family.c_str());
        return false;
    }
    KeyReader r(g);
    EncParams & e = m.enc;
    r.need({"jepa.enc.embed_dim", "jepa.enc.n_layer", "jepa.enc.n_head", "jepa.enc.ffn_dim", "jepa.enc.patch_size"})
        .num("jepa.enc.embed_dim", e.embed_dim, 0, 1, MAX_WIDTH)
        .num("jepa.enc.n_layer", e.n_layer, 0, 1, MAX_DEPTH)
        .num("jepa.enc.n_head", e.n_head, 0, 1, MAX_DEPTH)
        .num("jepa.enc.ffn_dim", e.ffn_dim, 0, 1, MAX_FFN)
        .num("jepa.enc.patch_size", e.patch_size, 16, 1, 1024)
        .num("jepa.enc.tubelet_size", e.tubelet_size, 1)
        .num("jepa.enc.img_size", e.img_size, 224)
        .num("jepa.enc.n_frames", e.n_frames, 1)
        .num("jepa.enc.n_registers", e.n_registers, 0)
        .num("jepa.enc.in_chans", e.in_chans, 3)
        .flag("jepa.enc.cls_token", e.cls_token, false)
        .real("jepa.enc.ln_eps", e.ln_eps, 1e-6f)
        .text("jepa.enc.act", e.act, "gelu_erf");
    std::string enc_layout, attn_mode;
    r.real("jepa.enc.rope_theta", e.rope_theta, 10000.0f, 1e-6f, 1e12f)
        .text("jepa.enc.rope_freq_layout", enc_layout, "tiled")
        .flag("jepa.enc.rope_interpolate", e.rope_interpolate, false)
        .num("jepa.enc.rope_ref_grid", e.rope_ref_grid, 0, 0, MAX_WIDTH)
        .flag("jepa.enc.modality_embed", e.modality_embed, false)
        .flag("jepa.enc.image_patch_embed", e.image_patch_embed, false)
        .text("jepa.enc.attn_mode", attn_mode, "full");
    if (!r.ok()) return false;
    e.rope_interleaved = enc_layout == "interleaved";
    e.block_causal = attn_mode == "block_causal";
    if (e.rope_interpolate && e.rope_ref_grid < 1) {
        log("jepa: jepa.enc.rope_interpolate asks for positions rescaled to jepa.enc.rope_ref_grid, which is %d\n", e.rope_ref_grid);
        return false;
    }

    m.pred_kind = g.has("jepa.pred.kind") ? g.gets("jepa.pred.kind", "none") : "";
    if (m.pred_kind == "none") m.pred_kind = "";
    if (m.pred_kind == "ac") {
        ACParams & a = m.ac;
        a.present = true;
        std::string layout;
        r.num("jepa.pred.embed_dim", a.embed_dim, 0, 1, MAX_WIDTH)
            .num("jepa.pred.n_layer", a.n_layer, 0, 1, MAX_DEPTH)
            .num("jepa.pred.n_head", a.n_head, 0, 1, MAX_DEPTH)
            .num("jepa.pred.ffn_dim", a.ffn_dim, 0, 1, MAX_FFN)
            .num("jepa.pred.head_dim", a.head_dim, 0)
            .num("jepa.pred.action_dim", a.action_dim, 0, 1, MAX_WIDTH)
            .num("jepa.pred.state_dim", a.state_dim, 0, 1, MAX_WIDTH)
            .num("jepa.pred.n_cond_tokens", a.n_cond_tokens, 0, 1, MAX_DEPTH)
            .num("jepa.pred.grid_size", a.grid_size, 0, 1, MAX_WIDTH)
            .num("jepa.pred.n_frames", a.n_frames, 0, 1, MAX_FRAMES)
            .num("jepa.pred.out_dim", a.out_dim, e.embed_dim)
            .flag("jepa.pred.normalize_reps", a.normalize_reps, false)
            .flag("jepa.pred.frame_causal", a.frame_causal, false)
            .real("jepa.pred.norm_reps_eps", a.norm_reps_eps, 1e-5f)
            .real("jepa.pred.ln_eps", a.ln_eps, 1e-6f)
            .real("jepa.enc.rope_theta", a.rope_theta, 10000.0f, 1e-6f, 1e12f)
            .text("jepa.pred.rope_freq_layout", layout, "")
            .text("jepa.pred.act", a.act, "gelu_erf");
        if (!r.ok()) return false;
        a.rope_interleaved = layout == "interleaved";
        if (a.head_dim == 0) {
            if (a.embed_dim % a.n_head) {
                log("jepa: jepa.pred.embed_dim %d does not split into %d heads\n", a.embed_dim, a.n_head);
                return false;
            }
            a.head_dim = a.embed_dim / a.n_head;
        }
        if (a.head_dim % 2) {
            log("jepa: the ac predictor's head width %d is odd; its 3-D RoPE rotates pairs of lanes\n", a.head_dim);
            return false;
        }
    }
    if (m.family == "hjepa") {
        HParams & hj = m.hj;
        int n = 0;
        r.num("jepa.hjepa.n_levels", n, 0, 1, 64);
        if (!r.ok()) return false;
        hj.present = true;
        hj.levels.resize((size_t) n);
        auto & lv = hj.levels;
        r.real("jepa.hjepa.ln_eps", hj.ln_eps, 1e-5f, 0.0f, 1.0f)
            .real("jepa.hjepa.adaln_eps", hj.adaln_eps, 1e-6f, 0.0f, 1.0f)
            .text("jepa.hjepa.proj_kind", hj.proj_kind, "identity")
            .num("jepa.hjepa.pixel_dim", hj.pixel_dim, 0)
            .num("jepa.hjepa.proprio_dim", hj.proprio_dim, 0)
            .num("jepa.hjepa.raw_action_dim", hj.raw_action_dim, 0)
            .num("jepa.hjepa.frameskip", hj.frameskip, 0)
            .per_level("jepa.hjepa.embed_dim", lv, &HLevel::embed_dim, 1, MAX_WIDTH)
            .per_level("jepa.hjepa.stride", lv, &HLevel::stride, 1, MAX_FRAMES)
            .per_level("jepa.hjepa.window", lv, &HLevel::window, 1, 1)
            .per_level("jepa.hjepa.target_length", lv, &HLevel::target_length, 0, MAX_FRAMES)
            .per_level("jepa.hjepa.action_dim", lv, &HLevel::action_dim, 1, MAX_WIDTH)
            .per_level("jepa.hjepa.act_embed_dim", lv, &HLevel::act_embed_dim, 1, MAX_WIDTH)
            .per_level("jepa.hjepa.act_enc_dim", lv, &HLevel::act_enc_dim, 0, MAX_WIDTH)
            .per_level("jepa.hjepa.act_enc_n_layer", lv, &HLevel::act_enc_n_layer, 0, MAX_DEPTH)
            .per_level("jepa.hjepa.act_enc_n_head", lv, &HLevel::act_enc_n_head, 0, MAX_DEPTH)
            .per_level("jepa.hjepa.act_enc_max_chunk", lv, &HLevel::act_enc_max_chunk, 0, MAX_FRAMES)
            .per_level("jepa.hjepa.pred_dim", lv, &HLevel::pred_dim, 1, MAX_WIDTH)
            .per_level("jepa.hjepa.pred_n_layer", lv, &HLevel::pred_n_layer, 1, MAX_DEPTH)
            .per_level("jepa.hjepa.pred_n_head", lv, &HLevel::pred_n_head, 1, MAX_DEPTH)
            .per_level("jepa.hjepa.pred_head_dim", lv, &HLevel::pred_head_dim, 1, MAX_WIDTH)
            .per_level("jepa.hjepa.pred_ffn_dim", lv, &HLevel::pred_ffn_dim, 1, MAX_FFN)
            .per_level("jepa.hjepa.pred_n_frames", lv, &HLevel::pred_n_frames, 1, MAX_FRAMES)
            .per_level("jepa.hjepa.enc_kind", lv, &HLevel::enc_kind)
            .per_level("jepa.hjepa.act_enc_kind", lv, &HLevel::act_enc_kind)
            .per_level("jepa.hjepa.pred_kind", lv, &HLevel::pred_kind);
        if (!r.ok()) return false;
    }
    return true;
}

// f32 vector of exactly n values (or absent when optional)
struct checker {
    const jepa_model & m;
    bool ok = true;
    void fail(const std::string & msg) { log("jepa: hjepa: %s\n", msg.c_str()); ok = false; }
    bool vec(const std::string & name, int64_t n, bool required) {
        const gguf_tensor * t = m.get(name);
        if (!t) { if (required) fail("required tensor " + name + " is missing"); return false; }
        if (t->type != T_F32) fail("tensor " + name + " has to be f32");
        if (t->nelements() != n) fail("tensor " + name + " holds " + std::to_string(t->nelements()) + " values, expected " + std::to_string(n));
        return true;
    }
    int64_t lin(const std::string & name, int64_t n_in, int64_t n_out, bool required) {
        const gguf_tensor * w = m.get(name + ".weight");
        if (!w) { if (required) fail("required tensor " + name + ".weight is missing"); return 0; }
        if (w->n_dims > 2 || (n_in > 0 && w->ne[0] != n_in) || (n_out > 0 && w->ne[1] != n_out)) {
            fail("tensor " + name + ".weight has shape [" + std::to_string(w->ne[0]) + ", " + std::to_string(w->ne[1]) +
                 "], expected [" + std::to_string(n_in > 0 ? n_in : w->ne[0]) + ", " + std::to_string(n_out > 0 ? n_out : w->ne[1]) + "]");
        }
        vec(name + ".bias", w->ne[1], false);
        return w->ne[1];
    }
    void table(const std::string & name, int64_t dim, int64_t min_rows, bool required) {
        const gguf_tensor * t = m.get(name);
        if (!t) { if (required) fail("required tensor " + name + " is missing"); return; }
        if (t->type != T_F32) fail("tensor " + name + " has to be f32");
        if (t->n_dims > 2 || t->ne[0] != dim || t->ne[1] < min_rows) {
            fail("tensor " + name + " needs width " + std::to_string(dim) + " and at least " + std::to_string(min_rows) + " rows");
        }
    }
    void want(bool c, const std::string & what, int level) { if (!c) fail("level " + std::to_string(level) + ": " + what); }
};

}  // namespace

bool hjepa_bind(const jepa_model & m) {
    const HParams & hj = m.hj;
    checker b{m};
    for (size_t li = 0; li < hj.levels.size() && b.ok; li++) {
        const int k = (int) li + 1;
        const HLevel & lv = hj.levels[li];
        const HLevel * below = li ? &hj.levels[li - 1] : nullptr;
        const std::string p = "lvl." + std::to_string(k) + ".";
        if (k == 1) {
            b.want(lv.stride == 1, "level 1 must have stride 1", k);
        } else {
            if (lv.enc_kind == "latent_mlp") {
                b.vec(p + "enc.in_norm.weight", below->embed_dim, true);
                b.vec(p + "enc.in_norm.bias", below->embed_dim, false);
                const int64_t h = b.lin(p + "enc.fc1", below->embed_dim, 0, true);
                b.lin(p + "enc.fc2", h, lv.embed_dim, true);
                if (b.vec(p + "enc.out_norm.weight", lv.embed_dim, false)) b.vec(p + "enc.out_norm.bias", lv.embed_dim, false);
            } else if (lv.enc_kind == "identity") {
                b.want(lv.embed_dim == below->embed_dim, "an identity encoder cannot change the width", k);
            } else {
                b.want(false, "jepa.hjepa.enc_kind must be latent_mlp | identity above level 1", k);
            }
        }
        if (const int64_t h = b.lin(p + "act_embed.0", lv.action_dim, 0, false)) {
            b.lin(p + "act_embed.2", h, lv.act_embed_dim, true);
        } else {
            b.want(lv.act_embed_dim == lv.action_dim, "no act_embed tensors, yet act_embed_dim differs from action_dim", k);
        }
        b.table(p + "act_queue", lv.action_dim, 1, false);
        const bool bare = lv.pred_kind == "adaln_bare";
        b.want(bare || lv.pred_kind == "adaln", "jepa.hjepa.pred_kind must be adaln | adaln_bare", k);
        const int64_t D = lv.pred_dim, inner = (int64_t) lv.pred_n_head * lv.pred_head_dim;
        b.table(p + "pred.pos_embed", lv.embed_dim, lv.pred_n_frames, true);
        int64_t cond = lv.act_embed_dim;
        if (bare) {
            const int64_t h = b.lin(p + "pred.act_embed.0", lv.act_embed_dim, 0, true);
            cond = b.lin(p + "pred.act_embed.2", h, 0, true);
        }
        if (!b.lin(p + "pred.in_proj", lv.embed_dim, D, false)) {
            b.want(lv.embed_dim == D, "pred.in_proj is missing but the predictor width differs from the state width", k);
        }
        if (!b.lin(p + "pred.cond_proj", cond, D, false)) {
            b.want(cond == D, "pred.cond_proj is missing but the predictor width differs from the conditioning width", k);
        }
        for (int i = 0; i < lv.pred_n_layer && b.ok; i++) {
            const std::string q = p + "pred.blk." + std::to_string(i) + ".";
            b.lin(q + "adaln", D, 6 * D, true);
            b.vec(q + "ln1.weight", D, !bare); b.vec(q + "ln1.bias", D, false);
            b.vec(q + "ln2.weight", D, !bare); b.vec(q + "ln2.bias", D, false);
            b.lin(q + "attn_qkv", D, 3 * inner, true);
            b.lin(q + "attn_out", inner, D, true);
            b.lin(q + "ffn_up", D, lv.pred_ffn_dim, true);
            b.lin(q + "ffn_down", lv.pred_ffn_dim, D, true);
        }
        b.vec(p + "pred.norm.weight", D, true);
        b.vec(p + "pred.norm.bias", D, false);
        int64_t out = D;
        if (const int64_t o = b.lin(p + "pred.out_proj", D, 0, false)) out = o;
        if (const int64_t h = b.lin(p + "pred.proj.0", out, 0, false)) out = b.lin(p + "pred.proj.2", h, 0, true);
        b.want(out == lv.embed_dim, "the predictor's output width differs from the level's state width", k);
    }
    return b.ok;
}

}  // namespace jb

// =============================================================================================
// C API: lifecycle, introspection, devices
// =============================================================================================
using jb::log;

extern "C" {

jepa_context_params jepa_context_default_params(void) {
    jepa_context_params p;
    p.n_threads = 0;
    p.use_flash_attn = true;
    p.verbose = false;
    p.flash_kv = JEPA_KV_AUTO;
    return p;
}

jepa_model_params jepa_model_default_params(void) {
    jepa_model_params p;
    p.verbose = false;
    p.device = -1;
    if (const char * e = getenv("JEPA_DEVICE")) {
        const char * s = e;
        if (!strncmp(s, "cuda:", 5)) s += 5;
        else if (!strncmp(s, "gpu:", 4)) s += 4;
        char * end = nullptr;
        const long v = strtol(s, &end, 10);
        if (!strcmp(e, "cpu")) p.device = -1;
        else if (end && *end == 0 && end != s && v >= 0) p.device = (int) v;
        else log("jepa: JEPA_DEVICE='%s' is not cpu | cuda:N | gpu:N | N; ignored\n", e);
    }
    return p;
}

jepa_model * jepa_model_load_ex(const char * gguf_path, const jepa_model_params * params) {
    if (!gguf_path) return nullptr;
    const jepa_model_params prm = params ? *params : jepa_model_default_params();
    // The metadata and the host copy of the tensors load anywhere; the planners need a CUDA device, which
    // jepa_context_new requires (a model loaded without one serves introspection and jepa_hjepa_horizons).
    int n_dev = 0;
    if (cudaGetDeviceCount(&n_dev) != cudaSuccess) { cudaGetLastError(); n_dev = 0; }
    const int dev = n_dev == 0 ? -1 : (prm.device >= 0 ? prm.device : 0);
    if (dev >= n_dev) { log("jepa: device %d requested, %d CUDA device(s) present\n", dev, n_dev); return nullptr; }
    std::string err;
    auto file = jb::gguf_read(gguf_path, &err);
    if (!file) { log("jepa: %s\n", err.c_str()); return nullptr; }
    auto m = std::make_unique<jepa_model>();
    m->path = gguf_path;
    m->file = std::move(file);
    m->device = dev;
    if (!jb::parse(*m)) return nullptr;
    if (m->hj.present && !jb::hjepa_bind(*m)) return nullptr;
    for (const auto & t : m->file->tensors) m->n_bytes += t.nbytes;
    m->device_name = dev >= 0 ? "CUDA" + std::to_string(dev) : "none";
    if (prm.verbose) {
        log("jepa: loaded %s (%s, %s, %zu tensors, %.1f MiB) for CUDA device %d\n", m->name.c_str(), m->family.c_str(),
            jb::type_name(m->file_type == 7 ? 8 : m->file_type == 2 ? 2 : m->file_type), m->file->tensors.size(),
            m->n_bytes / 1048576.0, dev);
    }
    return m.release();
}

jepa_model * jepa_model_load(const char * gguf_path, bool verbose) {
    jepa_model_params p = jepa_model_default_params();
    p.verbose = verbose;
    return jepa_model_load_ex(gguf_path, &p);
}

void jepa_model_free(jepa_model * model) { delete model; }

jepa_context * jepa_context_new(jepa_model * model, jepa_context_params params) {
    if (!model) return nullptr;
    if (model->device < 0) {
        log("jepa: jepa_context_new: no CUDA device is visible; this engine runs the planners on the GPU only\n");
        return nullptr;
    }
    auto ctx = std::make_unique<jepa_context>();
    ctx->model = model;
    ctx->params = params;
    ctx->n_threads = params.n_threads > 0 ? params.n_threads : 1;
    ctx->device = model->device;
    if (!jb::cuda_ok(cudaSetDevice(ctx->device), "cudaSetDevice")) return nullptr;
    if (!jb::cuda_ok(cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking), "cudaStreamCreate")) return nullptr;
    return ctx.release();
}

void jepa_context_free(jepa_context * ctx) { delete ctx; }
int jepa_context_n_threads(const jepa_context * ctx) { return ctx ? ctx->n_threads : 0; }
double jepa_context_last_compute_ms(const jepa_context * ctx) { return ctx ? ctx->last_ms : 0.0; }
double jepa_b200_last_plan_ms(const jepa_context * ctx) { return ctx ? ctx->last_ms : 0.0; }
long long jepa_b200_last_plan_launches(const jepa_context * ctx) { return ctx ? ctx->last_launches : 0; }

const char * jepa_model_family(const jepa_model * m) { return m ? m->family.c_str() : ""; }
const char * jepa_model_name(const jepa_model * m) { return m ? m->name.c_str() : ""; }
int jepa_model_embed_dim(const jepa_model * m) { return m ? m->enc.embed_dim : 0; }
int jepa_model_patch_size(const jepa_model * m) { return m ? m->enc.patch_size : 0; }
int jepa_model_tubelet_size(const jepa_model * m) { return m ? m->enc.tubelet_size : 0; }
int jepa_model_img_size(const jepa_model * m) { return m ? m->enc.img_size : 0; }
int jepa_model_n_frames(const jepa_model * m) { return m ? m->enc.n_frames : 0; }
int jepa_model_n_layer(const jepa_model * m) { return m ? m->enc.n_layer : 0; }
int jepa_model_n_head(const jepa_model * m) { return m ? m->enc.n_head : 0; }
bool jepa_model_has_cls(const jepa_model * m) { return m && m->enc.cls_token; }
int jepa_model_n_registers(const jepa_model * m) { return m ? m->enc.n_registers : 0; }
int jepa_model_n_prefix_tokens(const jepa_model * m) { return m ? (m->enc.cls_token ? 1 : 0) + m->enc.n_registers : 0; }
bool jepa_model_has_predictor(const jepa_model * m) { return m && (!m->pred_kind.empty() || m->hj.present); }
bool jepa_model_has_head(const jepa_model * m) { return m && m->file->has("jepa.head.kind") && m->file->gets("jepa.head.kind", "none") != "none"; }
bool jepa_model_has_projector(const jepa_model * m) { return m && m->get("enc.proj.0.weight") != nullptr; }
int jepa_model_n_classes(const jepa_model * m) { return m ? m->file->geti("jepa.head.n_classes", 0) : 0; }
const char * jepa_model_label(const jepa_model * m, int idx) {
    if (!m) return nullptr;
    const jb::gguf_value * v = m->file->find("jepa.head.labels");
    if (!v || idx < 0 || idx >= (int) v->as.size()) return nullptr;
    return v->as[(size_t) idx].c_str();
}
int jepa_model_file_type(const jepa_model * m) { return m ? (int) m->file_type : -1; }
const char * jepa_model_file_type_name(const jepa_model * m) {
    if (!m) return "unknown";
    switch (m->file_type) {
        case 0: return "f32"; case 1: return "f16"; case 2: return "q4_0"; case 3: return "q4_1";
        case 7: return "q8_0"; case 8: return "q5_0"; case 9: return "q5_1"; case 24: return "bf16";
        default: return "unknown";
    }
}
size_t jepa_model_n_bytes(const jepa_model * m) { return m ? m->n_bytes : 0; }

// ---- H-JEPA introspection (reference: include/jepa.h:232-247)
static const jb::HLevel * level_of(const jepa_model * m, int level) {
    if (!m || !m->hj.present || level < 1 || level > (int) m->hj.levels.size()) return nullptr;
    return &m->hj.levels[(size_t) level - 1];
}
int jepa_hjepa_n_levels(const jepa_model * m) { return m && m->hj.present ? (int) m->hj.levels.size() : 0; }
int jepa_hjepa_embed_dim(const jepa_model * m, int level) { const jb::HLevel * l = level_of(m, level); return l ? l->embed_dim : 0; }
int jepa_hjepa_action_dim(const jepa_model * m, int level) { const jb::HLevel * l = level_of(m, level); return l ? l->action_dim : 0; }
int jepa_hjepa_action_embed_dim(const jepa_model * m, int level) { const jb::HLevel * l = level_of(m, level); return l ? l->act_embed_dim : 0; }
int jepa_hjepa_stride(const jepa_model * m, int level) { const jb::HLevel * l = level_of(m, level); return l ? l->stride : 0; }
int jepa_hjepa_n_frames(const jepa_model * m, int level) { const jb::HLevel * l = level_of(m, level); return l ? l->pred_n_frames : 0; }
int jepa_hjepa_proprio_dim(const jepa_model * m) { return m && m->hj.present ? m->hj.proprio_dim : 0; }
int jepa_hjepa_raw_action_dim(const jepa_model * m) { return m && m->hj.present ? m->hj.raw_action_dim : 0; }
int jepa_hjepa_frameskip(const jepa_model * m) { return m && m->hj.present ? m->hj.frameskip : 0; }

int jepa_hjepa_norm_stats(const jepa_model * m, const char * column, float * mean, float * std, int capacity) {
    if (!m || !column) return 0;
    const std::string n = std::string("norm.") + column;
    const jb::gguf_tensor * tm = m->get(n + ".mean"), * ts = m->get(n + ".std");
    if (!tm || !ts || tm->type != jb::T_F32 || ts->type != jb::T_F32) return 0;
    const int k = (int) tm->nelements();
    if (capacity >= k && mean && std) {
        memcpy(mean, tm->data, (size_t) k * 4);
        memcpy(std, ts->data, (size_t) k * 4);
    }
    return k;
}

int jepa_hjepa_action_prior(const jepa_model * m, int level, float * out, int capacity) {
    const jb::HLevel * l = level_of(m, level);
    if (!l) return 0;
    const jb::gguf_tensor * t = m->get("lvl." + std::to_string(level) + ".act_queue");
    if (!t || t->type != jb::T_F32) return 0;
    const int rows = (int) (t->nelements() / l->action_dim);
    if (out && capacity >= rows) memcpy(out, t->data, (size_t) rows * l->action_dim * 4);
    return rows;
}

// ---- devices (reference: include/jepa.h:547-596)
int jepa_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) { cudaGetLastError(); return 0; }
    return n;
}

const char * jepa_device_name(int device) {
    static thread_local std::string s;
    if (device < 0 || device >= jepa_device_count()) return nullptr;
    s = "CUDA" + std::to_string(device);
    return s.c_str();
}

const char * jepa_device_description(int device) {
    static thread_local std::string s;
    cudaDeviceProp p;
    if (device < 0 || cudaGetDeviceProperties(&p, device) != cudaSuccess) { cudaGetLastError(); return nullptr; }
    s = p.name;
    return s.c_str();
}

void jepa_device_memory(int device, size_t * free_bytes, size_t * total_bytes) {
    size_t f = 0, t = 0;
    int prev = 0;
    cudaGetDevice(&prev);
    if (device >= 0 && cudaSetDevice(device) == cudaSuccess && cudaMemGetInfo(&f, &t) == cudaSuccess) {
        cudaSetDevice(prev);
    } else {
        cudaGetLastError();
    }
    if (free_bytes) *free_bytes = f;
    if (total_bytes) *total_bytes = t;
}

int jepa_model_device(const jepa_model * m) { return m ? m->device : -1; }
const char * jepa_model_device_name(const jepa_model * m) { return m ? m->device_name.c_str() : "CPU"; }
bool jepa_model_is_gpu(const jepa_model * m) { return m != nullptr && m->device >= 0; }
void jepa_context_set_mul_mat_prec_f32(jepa_context * ctx, bool on) { if (ctx) ctx->prec_f32 = on; }
bool jepa_context_mul_mat_prec_f32(const jepa_context * ctx) { return ctx && ctx->prec_f32; }
void jepa_context_set_max_batch(jepa_context * ctx, int n) { if (ctx) ctx->max_batch = n > 0 ? n : 32; }
int jepa_context_max_batch(const jepa_context * ctx) { return ctx ? ctx->max_batch : 0; }
int jepa_context_last_batch(const jepa_context * ctx) { return ctx ? 1 : 0; }

const char * jepa_version(void) { return "jepa-b200 0.1.0"; }
// the probe the reference's Python loader looks up (reference: python/shared.c:9)
__attribute__((visibility("default"))) const char * jepa_cpp_shared_abi(void) { return jepa_version(); }

void jepa_print_system_info(void) {
    const int n = jepa_device_count();
    fprintf(stderr, "jepa-b200: %d CUDA device(s)\n", n);
    for (int i = 0; i < n; i++) fprintf(stderr, "  CUDA%d: %s\n", i, jepa_device_description(i));
}

}  // extern "C"
