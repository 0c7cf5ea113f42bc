// GGUF v2/v3 reader (header-only): metadata KV pairs, the tensor table, and the tensor bytes.
//
// Replaces the ggml `gguf.h` calls of the reference loader (src/jepa-gguf.cpp:788-907,
// gguf_init_from_file + gguf_get_* + the per-tensor fread) with a self-contained parser of the
// published container layout: magic "GGUF", version, tensor count, KV count, typed KV pairs, the
// tensor table (name, n_dims, ne[] in ggml order, ggml type, offset), then the data section aligned
// to general.alignment (default 32). Every length and offset read from the file is checked against
// the file size before it is used: a truncated or hostile file is refused with a message, never a
// crash (reference contract: src/jepa-gguf.cpp:821-852).
#pragma once

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace jb {

enum gguf_vtype : uint32_t {
    GV_U8 = 0, GV_I8 = 1, GV_U16 = 2, GV_I16 = 3, GV_U32 = 4, GV_I32 = 5, GV_F32 = 6, GV_BOOL = 7,
    GV_STR = 8, GV_ARR = 9, GV_U64 = 10, GV_I64 = 11, GV_F64 = 12,
};

// ggml tensor type ids used by jepa.cpp files (enum ggml_type)
enum ggml_tid : uint32_t { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q8_0 = 8, T_BF16 = 30 };

inline const char * type_name(uint32_t t) {
    switch (t) {
        case T_F32: return "f32"; case T_F16: return "f16"; case T_Q4_0: return "q4_0";
        case T_Q8_0: return "q8_0"; case T_BF16: return "bf16"; default: return "unsupported";
    }
}
// bytes of one row of n values (n a multiple of the block size for the block types); 0 = unknown type
inline size_t row_bytes(uint32_t t, int64_t n) {
    switch (t) {
        case T_F32: return (size_t) n * 4;
        case T_F16: case T_BF16: return (size_t) n * 2;
        case T_Q8_0: return (size_t) (n / 32) * 34;
        case T_Q4_0: return (size_t) (n / 32) * 18;
        default: return 0;
    }
}
inline int block_size(uint32_t t) { return (t == T_Q8_0 || t == T_Q4_0) ? 32 : 1; }

struct gguf_value {
    uint32_t type = 0;
    uint32_t arr_type = 0;
    int64_t i = 0;                    // any integer / bool
    double f = 0;                     // float / double
    std::string s;
    std::vector<int64_t> ai;          // integer arrays
    std::vector<double> af;           // float arrays
    std::vector<std::string> as;      // string arrays
};

struct gguf_tensor {
    std::string name;
    uint32_t type = 0;
    int n_dims = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    uint64_t offset = 0;              // relative to the data section
    size_t nbytes = 0;
    const uint8_t * data = nullptr;   // into gguf_file::bytes
    int64_t nelements() const { return ne[0] * ne[1] * ne[2] * ne[3]; }
};

struct gguf_file {
    std::vector<uint8_t> bytes;
    std::vector<std::pair<std::string, gguf_value>> kv;   // file order
    std::map<std::string, size_t> kv_index;
    std::vector<gguf_tensor> tensors;
    std::map<std::string, size_t> tensor_index;
    std::string error;

    const gguf_value * find(const std::string & key) const {
        auto it = kv_index.find(key);
        return it == kv_index.end() ? nullptr : &kv[it->second].second;
    }
    const gguf_tensor * tensor(const std::string & name) const {
        auto it = tensor_index.find(name);
        return it == tensor_index.end() ? nullptr : &tensors[it->second];
    }
    bool has(const std::string & key) const { return find(key) != nullptr; }
    bool get_int(const std::string & key, int64_t & out) const {
        const gguf_value * v = find(key);
        if (!v) return false;
        switch (v->type) {
            case GV_U8: case GV_I8: case GV_U16: case GV_I16: case GV_U32: case GV_I32:
            case GV_U64: case GV_I64: case GV_BOOL: out = v->i; return true;
            default: return false;
        }
    }
    int geti(const std::string & key, int def) const { int64_t v; return get_int(key, v) ? (int) v : def; }
    bool getb(const std::string & key, bool def) const { int64_t v; return get_int(key, v) ? v != 0 : def; }
    float getf(const std::string & key, float def) const {
        const gguf_value * v = find(key);
        if (!v) return def;
        if (v->type == GV_F32 || v->type == GV_F64) return (float) v->f;
        int64_t i; return get_int(key, i) ? (float) i : def;
    }
    std::string gets(const std::string & key, const std::string & def) const {
        const gguf_value * v = find(key);
        return (v && v->type == GV_STR) ? v->s : def;
    }
    std::vector<int> get_iarr(const std::string & key) const {
        std::vector<int> out;
        const gguf_value * v = find(key);
        if (v && v->type == GV_ARR) for (int64_t x : v->ai) out.push_back((int) x);
        return out;
    }
    std::vector<std::string> get_sarr(const std::string & key) const {
        const gguf_value * v = find(key);
        return (v && v->type == GV_ARR && v->arr_type == GV_STR) ? v->as : std::vector<std::string>();
    }
};

namespace detail {
struct cursor {
    const uint8_t * p; size_t n, pos = 0; bool ok = true;
    bool need(size_t k) { if (!ok || k > n - pos) { ok = false; return false; } return true; }
    template <class T> T get() { T v{}; if (need(sizeof(T))) { memcpy(&v, p + pos, sizeof(T)); pos += sizeof(T); } return v; }
    std::string str() {
        uint64_t len = get<uint64_t>();
        if (!ok || len > (uint64_t) (n - pos)) { ok = false; return std::string(); }
        std::string s((const char *) p + pos, (size_t) len); pos += (size_t) len; return s;
    }
};
inline bool scalar(cursor & c, uint32_t t, gguf_value & v) {
    switch (t) {
        case GV_U8:   v.i = c.get<uint8_t>(); break;
        case GV_I8:   v.i = c.get<int8_t>(); break;
        case GV_U16:  v.i = c.get<uint16_t>(); break;
        case GV_I16:  v.i = c.get<int16_t>(); break;
        case GV_U32:  v.i = c.get<uint32_t>(); break;
        case GV_I32:  v.i = c.get<int32_t>(); break;
        case GV_U64:  v.i = (int64_t) c.get<uint64_t>(); break;
        case GV_I64:  v.i = c.get<int64_t>(); break;
        case GV_BOOL: v.i = c.get<uint8_t>() ? 1 : 0; break;
        case GV_F32:  v.f = c.get<float>(); break;
        case GV_F64:  v.f = c.get<double>(); break;
        case GV_STR:  v.s = c.str(); break;
        default: return false;
    }
    return c.ok;
}
}  // namespace detail

// Parse `path` completely into memory. Returns nullptr and fills *err on failure.
inline std::unique_ptr<gguf_file> gguf_read(const std::string & path, std::string * err) {
    auto fail = [&](const std::string & why) -> std::unique_ptr<gguf_file> {
        if (err) *err = path + ": " + why;
        return nullptr;
    };
    FILE * f = fopen(path.c_str(), "rb");
    if (!f) return fail("cannot open");
    auto g = std::make_unique<gguf_file>();
    fseek(f, 0, SEEK_END);
    const long sz = ftell(f);
    fseek(f, 0, SEEK_SET);
    if (sz < 24) { fclose(f); return fail("too short to be a GGUF file"); }
    g->bytes.resize((size_t) sz);
    const size_t got = fread(g->bytes.data(), 1, (size_t) sz, f);
    fclose(f);
    if (got != (size_t) sz) return fail("short read");
    detail::cursor c{g->bytes.data(), g->bytes.size()};
    if (memcmp(g->bytes.data(), "GGUF", 4) != 0) return fail("bad magic (not a GGUF file)");
    c.pos = 4;
    const uint32_t version = c.get<uint32_t>();
    if (version < 2 || version > 3) return fail("unsupported GGUF version " + std::to_string(version));
    const uint64_t n_tensors = c.get<uint64_t>(), n_kv = c.get<uint64_t>();
    // every KV pair and tensor entry takes at least 8 bytes: a count above that is a corrupt header
    if (n_tensors > g->bytes.size() / 8 || n_kv > g->bytes.size() / 8) return fail("corrupt header counts");
    for (uint64_t i = 0; i < n_kv; i++) {
        std::string key = c.str();
        gguf_value v;
        v.type = c.get<uint32_t>();
        if (!c.ok) return fail("truncated metadata");
        if (v.type == GV_ARR) {
            v.arr_type = c.get<uint32_t>();
            const uint64_t n = c.get<uint64_t>();
            if (!c.ok || n > g->bytes.size()) return fail("corrupt array length for " + key);
            for (uint64_t j = 0; j < n; j++) {
                gguf_value e;
                if (!detail::scalar(c, v.arr_type, e)) return fail("bad array element in " + key);
                if (v.arr_type == GV_STR) v.as.push_back(e.s);
                else if (v.arr_type == GV_F32 || v.arr_type == GV_F64) v.af.push_back(e.f);
                else v.ai.push_back(e.i);
            }
        } else if (!detail::scalar(c, v.type, v)) {
            return fail("bad value for " + key);
        }
        g->kv_index[key] = g->kv.size();
        g->kv.emplace_back(std::move(key), std::move(v));
    }
    for (uint64_t i = 0; i < n_tensors; i++) {
        gguf_tensor t;
        t.name = c.str();
        t.n_dims = (int) c.get<uint32_t>();
        if (!c.ok || t.n_dims < 1 || t.n_dims > 4) return fail("bad tensor dims for " + t.name);
        for (int d = 0; d < t.n_dims; d++) {
            const uint64_t ne = c.get<uint64_t>();
            if (ne == 0 || ne > (1ull << 40)) return fail("bad extent in " + t.name);
            t.ne[d] = (int64_t) ne;
        }
        t.type = c.get<uint32_t>();
        t.offset = c.get<uint64_t>();
        if (!c.ok) return fail("truncated tensor table");
        const size_t rb = row_bytes(t.type, t.ne[0]);
        if (rb == 0) return fail("tensor " + t.name + " has unsupported type " + std::to_string(t.type));
        if (t.ne[0] % block_size(t.type) != 0) return fail("tensor " + t.name + " row is not a whole number of blocks");
        t.nbytes = rb * (size_t) (t.ne[1] * t.ne[2] * t.ne[3]);
        g->tensor_index[t.name] = g->tensors.size();
        g->tensors.push_back(std::move(t));
    }
    int64_t align = 32;
    g->get_int("general.alignment", align);
    if (align <= 0 || (align & (align - 1))) return fail("bad general.alignment");
    const size_t data0 = (c.pos + (size_t) align - 1) / (size_t) align * (size_t) align;
    for (gguf_tensor & t : g->tensors) {
        if (data0 > g->bytes.size() || t.offset > g->bytes.size() - data0 || t.nbytes > g->bytes.size() - data0 - t.offset) {
            return fail("tensor " + t.name + " extends past the end of the file");
        }
        t.data = g->bytes.data() + data0 + t.offset;
    }
    return g;
}

// ---------------------------------------------------------------------------------------------
// host dequantisation (the exact arithmetic of the block formats; the device kernels are checked
// against these bit for bit)
// ---------------------------------------------------------------------------------------------
inline float fp16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t) (h & 0x8000) << 16;
    uint32_t exp = (h >> 10) & 0x1f, man = h & 0x3ff, bits;
    if (exp == 0) {
        if (man == 0) bits = sign;
        else {                          // subnormal: renormalise
            exp = 127 - 15 + 1;
            while (!(man & 0x400)) { man <<= 1; exp--; }
            bits = sign | (exp << 23) | ((man & 0x3ff) << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f; memcpy(&f, &bits, 4); return f;
}

inline void dequant_row(uint32_t type, const uint8_t * src, float * dst, int64_t n) {
    switch (type) {
        case T_F32: memcpy(dst, src, (size_t) n * 4); break;
        case T_F16: for (int64_t i = 0; i < n; i++) { uint16_t h; memcpy(&h, src + 2 * i, 2); dst[i] = fp16_to_f32(h); } break;
        case T_BF16: for (int64_t i = 0; i < n; i++) { uint16_t h; memcpy(&h, src + 2 * i, 2); uint32_t b = (uint32_t) h << 16; memcpy(dst + i, &b, 4); } break;
        case T_Q8_0:
            for (int64_t b = 0; b < n / 32; b++) {
                const uint8_t * blk = src + b * 34;
                uint16_t h; memcpy(&h, blk, 2);
                const float d = fp16_to_f32(h);
                for (int j = 0; j < 32; j++) dst[b * 32 + j] = d * (float) (int8_t) blk[2 + j];
            }
            break;
        case T_Q4_0:
            for (int64_t b = 0; b < n / 32; b++) {
                const uint8_t * blk = src + b * 18;
                uint16_t h; memcpy(&h, blk, 2);
                const float d = fp16_to_f32(h);
                for (int j = 0; j < 16; j++) {
                    dst[b * 32 + j]      = (float) ((int) (blk[2 + j] & 0x0f) - 8) * d;
                    dst[b * 32 + j + 16] = (float) ((int) (blk[2 + j] >> 4) - 8) * d;
                }
            }
            break;
        default: break;
    }
}

}  // namespace jb
