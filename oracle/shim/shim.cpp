// Test-infrastructure shim (oracle only, never part of the product): lets the reference's own planner
// source, src/hjepa-plan.cpp, compile and run unmodified on the host as the parity oracle and as the
// timed CPU baseline.
//
// It supplies what that file and the headers it includes need from outside it:
//   * the ggml names of ggml.h / ggml-backend.h (element counts, f16 rows, q8_0 / q4_0 to_float,
//     tensor read-back), written from the call sites (src/hjepa-plan.cpp:61-79) and the published
//     block formats -- no ggml source exists here;
//   * jepa_log and jepa_model::get (declared in src/jepa-internal.h);
//   * a loader that fills jepa_model::hp.hjepa from the jepa.hjepa.* keys (the reference parses them
//     at src/jepa-gguf.cpp:490-550) and the name -> tensor map, using the project's GGUF reader;
//   * ref_context_new / ref_context_free, a jepa_context over that model with n_threads threads.
// The planner entry points themselves (jepa_hjepa_plan_cost / _solve / _plan / _horizons /
// _level_plan_default) are the reference's, exported from the same shared object.
#include "jepa-internal.h"
#include "gguf.h"          // the shim's (an opaque gguf_context)
#include "../../jepa.cpp_b200/csrc/gguf.h"

#include <cstdarg>
#include <cstring>
#include <memory>

// ---------------- ggml names ----------------
int64_t ggml_nelements(const ggml_tensor * t) { return t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3]; }
size_t ggml_nbytes(const ggml_tensor * t) { return t->nbytes; }
int ggml_n_dims(const ggml_tensor * t) { return t->n_dims; }
void ggml_fp16_to_fp32_row(const ggml_fp16_t * x, float * y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = jb::fp16_to_f32(x[i]);
}
static void q8_0_to_float(const void * x, float * y, int64_t k) { jb::dequant_row(jb::T_Q8_0, (const uint8_t *) x, y, k); }
static void q4_0_to_float(const void * x, float * y, int64_t k) { jb::dequant_row(jb::T_Q4_0, (const uint8_t *) x, y, k); }
static void bf16_to_float(const void * x, float * y, int64_t k) { jb::dequant_row(jb::T_BF16, (const uint8_t *) x, y, k); }
const ggml_type_traits * ggml_get_type_traits(ggml_type type) {
    static const ggml_type_traits q8 = {"q8_0", 32, 34, q8_0_to_float};
    static const ggml_type_traits q4 = {"q4_0", 32, 18, q4_0_to_float};
    static const ggml_type_traits b16 = {"bf16", 1, 2, bf16_to_float};
    switch (type) {
        case GGML_TYPE_Q8_0: return &q8;
        case GGML_TYPE_Q4_0: return &q4;
        case GGML_TYPE_BF16: return &b16;
        default: return nullptr;
    }
}
void ggml_backend_tensor_get(const ggml_tensor * t, void * data, size_t offset, size_t size) {
    memcpy(data, (const uint8_t *) t->data + offset, size);
}

// ---------------- jepa-internal.h names ----------------
void jepa_log(const char * fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vfprintf(stderr, fmt, ap);
    va_end(ap);
}
ggml_tensor * jepa_model::get(const std::string & name) const {
    auto it = tensors.find(name);
    return it == tensors.end() ? nullptr : it->second;
}

namespace {
struct shim_model {
    jepa_model m;
    std::unique_ptr<jb::gguf_file> file;
    std::vector<ggml_tensor> store;
};
}  // namespace

extern "C" {

// Load `path` as the reference planner sees a model: hparams + tensor map. NULL on failure.
void * ref_model_load(const char * path) {
    std::string err;
    auto sm = std::make_unique<shim_model>();
    sm->file = jb::gguf_read(path, &err);
    if (!sm->file) { fprintf(stderr, "ref shim: %s\n", err.c_str()); return nullptr; }
    const jb::gguf_file & g = *sm->file;
    jepa_hparams & hp = sm->m.hp;
    hp.name = g.gets("general.name", "");
    hp.family_str = g.gets("jepa.family", "");
    hp.family = hp.family_str == "hjepa" ? JEPA_FAMILY_HJEPA : JEPA_FAMILY_UNKNOWN;
    if (hp.family == JEPA_FAMILY_HJEPA) {
        jepa_hjepa_hparams & hj = hp.hjepa;
        const int n = g.geti("jepa.hjepa.n_levels", 0);
        hj.present = n > 0;
        hj.ln_eps = g.getf("jepa.hjepa.ln_eps", 1e-5f);
        hj.adaln_eps = g.getf("jepa.hjepa.adaln_eps", 1e-6f);
        hj.levels.resize((size_t) n);
        auto ia = [&](const char * k, int jepa_hjepa_level::* f) {
            std::vector<int> v = g.get_iarr(std::string("jepa.hjepa.") + k);
            for (int i = 0; i < n && i < (int) v.size(); i++) hj.levels[(size_t) i].*f = v[(size_t) i];
        };
        auto sa = [&](const char * k, std::string jepa_hjepa_level::* f) {
            std::vector<std::string> v = g.get_sarr(std::string("jepa.hjepa.") + k);
            for (int i = 0; i < n && i < (int) v.size(); i++) hj.levels[(size_t) i].*f = v[(size_t) i];
        };
        ia("embed_dim", &jepa_hjepa_level::embed_dim);       ia("stride", &jepa_hjepa_level::stride);
        ia("window", &jepa_hjepa_level::window);             ia("target_length", &jepa_hjepa_level::target_length);
        ia("action_dim", &jepa_hjepa_level::action_dim);     ia("act_embed_dim", &jepa_hjepa_level::act_embed_dim);
        ia("act_enc_dim", &jepa_hjepa_level::act_enc_dim);   ia("act_enc_n_layer", &jepa_hjepa_level::act_enc_n_layer);
        ia("act_enc_n_head", &jepa_hjepa_level::act_enc_n_head);
        ia("act_enc_max_chunk", &jepa_hjepa_level::act_enc_max_chunk);
        ia("pred_dim", &jepa_hjepa_level::pred_dim);         ia("pred_n_layer", &jepa_hjepa_level::pred_n_layer);
        ia("pred_n_head", &jepa_hjepa_level::pred_n_head);   ia("pred_head_dim", &jepa_hjepa_level::pred_head_dim);
        ia("pred_ffn_dim", &jepa_hjepa_level::pred_ffn_dim); ia("pred_n_frames", &jepa_hjepa_level::pred_n_frames);
        sa("enc_kind", &jepa_hjepa_level::enc_kind);
        sa("act_enc_kind", &jepa_hjepa_level::act_enc_kind);
        sa("pred_kind", &jepa_hjepa_level::pred_kind);
    }
    sm->store.resize(g.tensors.size());
    for (size_t i = 0; i < g.tensors.size(); i++) {
        const jb::gguf_tensor & t = g.tensors[i];
        ggml_tensor & x = sm->store[i];
        x.type = (ggml_type) t.type;
        for (int d = 0; d < 4; d++) x.ne[d] = t.ne[d];
        x.n_dims = t.n_dims;
        x.nbytes = t.nbytes;
        x.data = (void *) t.data;
        sm->m.tensors[t.name] = &x;
    }
    return sm.release();
}

void ref_model_free(void * model) { delete (shim_model *) model; }

void * ref_context_new(void * model, int n_threads) {
    jepa_context * ctx = new jepa_context();
    ctx->model = &((shim_model *) model)->m;
    ctx->n_threads = n_threads > 0 ? n_threads : 1;
    return ctx;
}

void ref_context_free(void * ctx) { delete (jepa_context *) ctx; }

}  // extern "C"
