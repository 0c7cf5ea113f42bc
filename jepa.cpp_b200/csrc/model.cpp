// Model loading (GGUF -> hyper-parameters + host tensors), load-time validation of the H-JEPA tensors,
// and the lifecycle / introspection / device entry points of the C API.
//
// Key parsing follows the jepa.* schema the reference loader implements (src/jepa-gguf.cpp:254-550:
// required encoder keys, range checks on every integer taken from the file, the per-level jepa.hjepa.*
// arrays with one entry per level); a file that fails a check is refused with a message naming the key
// or tensor, never loaded half-way.
#include "model.h"
#include "hplan.h"
#include "shard.h"
#include "ac.h"
#include "encoder.h"

#include "../../include/jepa_b200.h"

#include <cinttypes>
#include <cstdlib>
#include <cstring>

namespace jb {

namespace {

bool in_range(const char * key, int64_t v, int64_t lo, int64_t hi) {
    if (v >= lo && v <= hi) return true;
    log("jepa: %s = %" PRId64 " is out of range [%" PRId64 ", %" PRId64 "]\n", key, v, lo, hi);
    return false;
}

bool parse(jepa_model & m) {
    const gguf_file & g = *m.file;
    if (g.gets("general.architecture", "") != "jepa") {
        log("jepa: general.architecture is '%s', expected 'jepa'\n", g.gets("general.architecture", "").c_str());
        return false;
    }
    m.name = g.gets("general.name", "");
    m.family = g.gets("jepa.family", "");
    m.modality = g.gets("jepa.modality", "image");
    m.file_type = (uint32_t) g.geti("general.file_type", 0);
    static const char * families[] = {"ijepa", "vjepa", "vjepa2", "vjepa2_1", "levjepa", "hfvit", "lewm", "hjepa"};
    bool known = false;
    for (const char * f : families) known = known || m.family == f;
    if (!known) { log("jepa: unknown jepa.family '%s'\n", m.family.c_str()); return false; }
    for (const char * k : {"jepa.enc.embed_dim", "jepa.enc.n_layer", "jepa.enc.n_head", "jepa.enc.ffn_dim", "jepa.enc.patch_size"}) {
        if (!g.has(k)) { log("jepa: missing required key %s\n", k); return false; }
    }
    EncParams & e = m.enc;
    e.embed_dim = g.geti("jepa.enc.embed_dim", 0);
    e.n_layer = g.geti("jepa.enc.n_layer", 0);
    e.n_head = g.geti("jepa.enc.n_head", 0);
    e.ffn_dim = g.geti("jepa.enc.ffn_dim", 0);
    e.patch_size = g.geti("jepa.enc.patch_size", 16);
    e.tubelet_size = g.geti("jepa.enc.tubelet_size", 1);
    e.img_size = g.geti("jepa.enc.img_size", 224);
    e.n_frames = g.geti("jepa.enc.n_frames", 1);
    e.n_registers = g.geti("jepa.enc.n_registers", 0);
    e.cls_token = g.getb("jepa.enc.cls_token", false);
    e.in_chans = g.geti("jepa.enc.in_chans", 3);
    e.ln_eps = g.getf("jepa.enc.ln_eps", 1e-6f);
    e.act = g.gets("jepa.enc.act", "gelu_erf");
    if (!in_range("jepa.enc.embed_dim", e.embed_dim, 1, 65536) || !in_range("jepa.enc.n_layer", e.n_layer, 1, 1024) ||
        !in_range("jepa.enc.n_head", e.n_head, 1, 1024) || !in_range("jepa.enc.ffn_dim", e.ffn_dim, 1, 1048576) ||
        !in_range("jepa.enc.patch_size", e.patch_size, 1, 1024)) {
        return false;
    }
    m.pred_kind = g.has("jepa.pred.kind") ? g.gets("jepa.pred.kind", "none") : "";
    if (m.pred_kind == "none") m.pred_kind = "";
    if (m.pred_kind == "ac") {
        ACParams & a = m.ac;
        a.present = true;
        a.embed_dim = g.geti("jepa.pred.embed_dim", 0);
        a.n_layer = g.geti("jepa.pred.n_layer", 0);
        a.n_head = g.geti("jepa.pred.n_head", 0);
        a.ffn_dim = g.geti("jepa.pred.ffn_dim", 0);
        a.head_dim = g.geti("jepa.pred.head_dim", 0);
        a.action_dim = g.geti("jepa.pred.action_dim", 0);
        a.state_dim = g.geti("jepa.pred.state_dim", 0);
        a.n_cond_tokens = g.geti("jepa.pred.n_cond_tokens", 0);
        a.grid_size = g.geti("jepa.pred.grid_size", 0);
        a.n_frames = g.geti("jepa.pred.n_frames", 0);
        a.normalize_reps = g.getb("jepa.pred.normalize_reps", false);
        a.norm_reps_eps = g.getf("jepa.pred.norm_reps_eps", 1e-5f);
        a.ln_eps = g.getf("jepa.pred.ln_eps", 1e-6f);
        a.frame_causal = g.getb("jepa.pred.frame_causal", false);
        a.rope_interleaved = g.gets("jepa.pred.rope_freq_layout", "") == "interleaved";
        a.rope_theta = g.getf("jepa.enc.rope_theta", 10000.0f);
        a.out_dim = g.geti("jepa.pred.out_dim", e.embed_dim);
        a.act = g.gets("jepa.pred.act", "gelu_erf");
        if (!(a.rope_theta >= 1e-6f && a.rope_theta <= 1e12f)) { log("jepa: jepa.enc.rope_theta is out of range\n"); return false; }
        if (!in_range("jepa.pred.embed_dim", a.embed_dim, 1, 65536) || !in_range("jepa.pred.n_layer", a.n_layer, 1, 1024) ||
            !in_range("jepa.pred.n_head", a.n_head, 1, 1024) || !in_range("jepa.pred.ffn_dim", a.ffn_dim, 1, 1048576) ||
            !in_range("jepa.pred.action_dim", a.action_dim, 1, 65536) || !in_range("jepa.pred.state_dim", a.state_dim, 1, 65536) ||
            !in_range("jepa.pred.n_cond_tokens", a.n_cond_tokens, 1, 1024) || !in_range("jepa.pred.grid_size", a.grid_size, 1, 65536) ||
            !in_range("jepa.pred.n_frames", a.n_frames, 1, 65536)) {
            return false;
        }
        if (a.head_dim == 0) {
            if (a.embed_dim % a.n_head) { log("jepa: jepa.pred.embed_dim %d is not divisible by n_head %d\n", a.embed_dim, a.n_head); return false; }
            a.head_dim = a.embed_dim / a.n_head;
        }
        if (a.head_dim % 2) { log("jepa: the ac predictor rotates pairs with 3-D RoPE, so its head width has to be even\n"); return false; }
    }
    if (m.family == "hjepa") {
        HParams & hj = m.hj;
        const int n = g.geti("jepa.hjepa.n_levels", 0);
        if (!in_range("jepa.hjepa.n_levels", n, 1, 64)) return false;
        hj.present = true;
        hj.ln_eps = g.getf("jepa.hjepa.ln_eps", 1e-5f);
        hj.adaln_eps = g.getf("jepa.hjepa.adaln_eps", 1e-6f);
        if (!(hj.ln_eps >= 0.0f && hj.ln_eps <= 1.0f) || !(hj.adaln_eps >= 0.0f && hj.adaln_eps <= 1.0f)) {
            log("jepa: jepa.hjepa.ln_eps / adaln_eps must be finite values in [0, 1]\n");
            return false;
        }
        hj.proj_kind = g.gets("jepa.hjepa.proj_kind", "identity");
        hj.pixel_dim = g.geti("jepa.hjepa.pixel_dim", 0);
        hj.proprio_dim = g.geti("jepa.hjepa.proprio_dim", 0);
        hj.raw_action_dim = g.geti("jepa.hjepa.raw_action_dim", 0);
        hj.frameskip = g.geti("jepa.hjepa.frameskip", 0);
        hj.levels.resize((size_t) n);
        struct ik { const char * key; int HLevel::* f; int lo, hi; };
        const ik ints[] = {
            {"jepa.hjepa.embed_dim", &HLevel::embed_dim, 1, 65536}, {"jepa.hjepa.stride", &HLevel::stride, 1, 65536},
            {"jepa.hjepa.window", &HLevel::window, 1, 1}, {"jepa.hjepa.target_length", &HLevel::target_length, 0, 65536},
            {"jepa.hjepa.action_dim", &HLevel::action_dim, 1, 65536}, {"jepa.hjepa.act_embed_dim", &HLevel::act_embed_dim, 1, 65536},
            {"jepa.hjepa.act_enc_dim", &HLevel::act_enc_dim, 0, 65536}, {"jepa.hjepa.act_enc_n_layer", &HLevel::act_enc_n_layer, 0, 1024},
            {"jepa.hjepa.act_enc_n_head", &HLevel::act_enc_n_head, 0, 1024}, {"jepa.hjepa.act_enc_max_chunk", &HLevel::act_enc_max_chunk, 0, 65536},
            {"jepa.hjepa.pred_dim", &HLevel::pred_dim, 1, 65536}, {"jepa.hjepa.pred_n_layer", &HLevel::pred_n_layer, 1, 1024},
            {"jepa.hjepa.pred_n_head", &HLevel::pred_n_head, 1, 1024}, {"jepa.hjepa.pred_head_dim", &HLevel::pred_head_dim, 1, 65536},
            {"jepa.hjepa.pred_ffn_dim", &HLevel::pred_ffn_dim, 1, 1048576}, {"jepa.hjepa.pred_n_frames", &HLevel::pred_n_frames, 1, 65536},
        };
        for (const ik & k : ints) {
            const std::vector<int> v = g.get_iarr(k.key);
            if ((int) v.size() != n) { log("jepa: %s holds %zu values, expected one per level (%d)\n", k.key, v.size(), n); return false; }
            for (int i = 0; i < n; i++) {
                if (!in_range(k.key, v[(size_t) i], k.lo, k.hi)) return false;
                hj.levels[(size_t) i].*k.f = v[(size_t) i];
            }
        }
        struct sk { const char * key; std::string HLevel::* f; };
        const sk strs[] = {{"jepa.hjepa.enc_kind", &HLevel::enc_kind}, {"jepa.hjepa.act_enc_kind", &HLevel::act_enc_kind},
                           {"jepa.hjepa.pred_kind", &HLevel::pred_kind}};
        for (const sk & k : strs) {
            const std::vector<std::string> v = g.get_sarr(k.key);
            if ((int) v.size() != n) { log("jepa: %s holds %zu values, expected one per level (%d)\n", k.key, v.size(), n); return false; }
            for (int i = 0; i < n; i++) hj.levels[(size_t) i].*k.f = v[(size_t) i];
        }
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
