// Weight upload from a GGUF model to the device: float32 planes, their transposes and, per orientation of
// each linear, the operand of its tensor-core products -- the 3xTF32 hi / lo planes (dequantised on the
// device, bit-exact with the block formats), or the GGUF block planes the GEMM dequantises in its mainloop
// (q8_0, q4_0, f16; 2.06 B per weight for both orientations of a q8_0 weight, against 16 for the planes).
// JEPA_B200_WEIGHT_LAYOUT chooses: "planes", "blocks" (every orientation the block planes serve), or "auto"
// (the default): hi / lo planes, the faster layout on every product measured (block planes cost 3-10 % of a
// plan on the 64-wide split-K products and 1.35-1.5x per launch on the persistent kernel's), unless the
// planes of the model's quantised weights would take more than a quarter of the device's free memory --
// then block planes everywhere they serve. Both layouts give the same bits. Every allocation goes into the
// owner's list, which frees them.
#pragma once

#include "hplan.h"
#include "kernels.h"
#include "model.h"
#include "gguf.h"
#include "common.h"

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

namespace jb {

enum WeightLayout : int { WL_AUTO = 0, WL_PLANES = 1, WL_BLOCKS = 2 };
inline int weight_layout() {
    const char * e = std::getenv("JEPA_B200_WEIGHT_LAYOUT");
    if (!e || !*e || !std::strcmp(e, "auto")) return WL_AUTO;
    if (!std::strcmp(e, "planes")) return WL_PLANES;
    if (!std::strcmp(e, "blocks")) return WL_BLOCKS;
    log("jepa: JEPA_B200_WEIGHT_LAYOUT=%s is not planes, blocks or auto: using auto\n", e);
    return WL_AUTO;
}

// The layout "auto" resolves to for a model on the current device: planes unless the hi / lo planes and f32
// copies of its quantised and f16 matrices (24 B per value) would take more than a quarter of the free memory.
inline int resolve_layout(int layout, const jepa_model & m) {
    if (layout != WL_AUTO) return layout;
    size_t values = 0;
    for (const gguf_tensor & t : m.file->tensors) {
        if ((t.type == 8 || t.type == 2 || t.type == 1) && t.n_dims == 2) values += (size_t) t.nelements();
    }
    size_t free_b = 0, total_b = 0;
    if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) { cudaGetLastError(); return WL_PLANES; }
    return 24 * values > free_b / 4 ? WL_BLOCKS : WL_PLANES;
}

struct Uploader {
    std::vector<void *> & allocs;   // every allocation, freed by the owner
    const jepa_model & m;
    cudaStream_t st;
    bool ok = true;
    std::vector<void *> temps;
    int layout = resolve_layout(weight_layout(), m);
    size_t block_bytes = 0, plane_bytes = 0;   // device bytes of the two operand layouts uploaded

    template <class T> T * alloc(size_t n) {
        void * p = nullptr;
        if (cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)) != cudaSuccess) {
            cudaGetLastError();
            log("jepa: hjepa planner: out of device memory while uploading the weights\n");
            ok = false;
            return nullptr;
        }
        allocs.push_back(p);
        return (T *) p;
    }
    // float32 vector (the validated norm / bias / table tensors are float32)
    float * vec(const std::string & name, int64_t offset = 0, int64_t n = -1) {
        const gguf_tensor * t = m.get(name);
        if (!t || !ok) return nullptr;
        if (n < 0) n = t->nelements() - offset;
        std::vector<float> host((size_t) n);
        std::vector<float> all((size_t) t->nelements());
        dequant_row(t->type, t->data, all.data(), t->nelements());
        std::copy(all.begin() + offset, all.begin() + offset + n, host.begin());
        float * d = alloc<float>((size_t) n);
        if (d) ok = cuda_ok(cudaMemcpyAsync(d, host.data(), (size_t) n * 4, cudaMemcpyHostToDevice, st), "upload") && ok;
        cudaStreamSynchronize(st);
        return d;
    }
    // dequantise rows [row0, row0 + rows) of a weight into dst (device, float32 [rows][in])
    bool dequant_into(const gguf_tensor * t, int64_t row0, int64_t rows, float * dst) {
        const size_t rb = row_bytes(t->type, t->ne[0]);
        void * raw = nullptr;
        if (cudaMalloc(&raw, rb * (size_t) rows) != cudaSuccess) { cudaGetLastError(); ok = false; return false; }
        bool good = cuda_ok(cudaMemcpyAsync(raw, t->data + rb * (size_t) row0, rb * (size_t) rows, cudaMemcpyHostToDevice, st), "upload") &&
                    dequant_rows(t->type, raw, dst, rows, t->ne[0], st) == 0;
        good = cuda_ok(cudaStreamSynchronize(st), "dequant") && good;
        cudaFree(raw);
        ok = ok && good;
        return good;
    }
    // the hi / lo planes of the orientations the block planes do not serve (and the f32 transpose, which the
    // SIMT backward of a small linear reads)
    void finish(DLin & L) {
        if (!ok) return;
        const size_t n = (size_t) L.in * L.out;
        if (!L.tq.fmt) {
            L.wt = alloc<float>(n);
            L.wt_hi = alloc<float>(n); L.wt_lo = alloc<float>(n);
            if (!ok) return;
            transpose_f32(L.w, L.wt, L.out, L.in, st);
            split_f32(L.wt, L.out, L.wt_hi, L.wt_lo, L.out, L.in, L.out, st);
            plane_bytes += 8 * n;
        }
        if (!L.fq.fmt) {
            L.w_hi = alloc<float>(n); L.w_lo = alloc<float>(n);
            if (!ok) return;
            split_f32(L.w, L.in, L.w_hi, L.w_lo, L.in, L.out, L.in, st);
            plane_bytes += 8 * n;
        }
        ok = cuda_ok(cudaStreamSynchronize(st), "weight layout") && ok;
    }
    // the block planes of rows [row0, row0 + rows) of t for the orientations chosen (fwd: y = x W^T, N = rows,
    // K = in; bwd: dx = dy W, N = in, K = rows)
    void blocks(DLin & L, const gguf_tensor * t, int64_t row0, int64_t rows, bool fwd, bool bwd) {
        if (!ok || (!fwd && !bwd)) return;
        const int64_t ne0 = t->ne[0];
        const size_t rb = row_bytes(t->type, ne0), nq = quant_plane_bytes(t->type, rows, ne0);
        const size_t nd = quant_scale_count(t->type, rows, ne0);
        // the orientation not kept is written to a temporary (quant_planes fills both)
        void * raw = nullptr, * spare = nullptr;
        if (cudaMalloc(&raw, rb * (size_t) rows) != cudaSuccess || (!(fwd && bwd) && cudaMalloc(&spare, nq) != cudaSuccess)) {
            cudaGetLastError();
            if (raw) cudaFree(raw);
            ok = false;
            log("jepa: hjepa planner: out of device memory while uploading the weights\n");
            return;
        }
        void * q = fwd ? alloc<uint8_t>(nq) : spare, * qt = bwd ? alloc<uint8_t>(nq) : spare;
        uint16_t * d = nd ? alloc<uint16_t>(nd) : nullptr;
        bool good = ok && cuda_ok(cudaMemcpyAsync(raw, t->data + rb * (size_t) row0, rb * (size_t) rows, cudaMemcpyHostToDevice, st), "upload") &&
                    quant_planes(t->type, raw, rows, ne0, q, qt, d, st) == 0;
        good = cuda_ok(cudaStreamSynchronize(st), "block planes") && good;
        cudaFree(raw);
        if (spare) cudaFree(spare);
        ok = ok && good;
        if (!ok) return;
        const int fmt = t->type == 8 ? QF_Q8 : t->type == 2 ? QF_Q4 : QF_F16;
        if (fwd) L.fq = QuantB{fmt, 0, q, d};
        if (bwd) L.tq = QuantB{fmt, 1, qt, d};
        block_bytes += (fwd ? nq : 0) + (bwd ? nq : 0) + 2 * nd;
    }
    // which orientations of a [rows][in] weight of this type take block planes
    void choose(uint32_t type, int64_t rows, int64_t in, bool & fwd, bool & bwd) const {
        fwd = bwd = layout == WL_BLOCKS && quant_ok(type, rows, in);
    }
    // out(V(h)) as one linear: W_ov = W_out W_v (a 3xTF32 product on the device), b_ov = W_out b_v + b_out
    DLin compose(const DLin & v, const DLin & out) {
        DLin L;
        if (!ok || !v || !out || out.in != v.out) return L;
        L.in = v.in;
        L.out = out.out;
        L.w = alloc<float>((size_t) L.in * L.out);
        if (!L.w) return DLin();
        GemmEpi ep;
        ep.out0 = L.w;
        ep.ld0 = L.in;
        // A: W_out's hi / lo planes (temporary ones when its forward product reads block planes)
        const float * a_hi = out.w_hi, * a_lo = out.w_lo;
        void * tmp = nullptr;
        if (!a_hi) {
            if (cudaMalloc(&tmp, (size_t) 8 * out.in * out.out) != cudaSuccess) { cudaGetLastError(); ok = false; return DLin(); }
            a_hi = (const float *) tmp;
            a_lo = a_hi + (size_t) out.in * out.out;
            split_f32(out.w, out.in, (float *) a_hi, (float *) a_lo, out.in, out.out, out.in, st);
        }
        const int rc = gemm_tc({a_hi, a_lo, out.in}, v.bwd(), out.out, v.in, v.out, ep, st);
        if (tmp) { cudaStreamSynchronize(st); cudaFree(tmp); }
        if (rc) { ok = false; return DLin(); }
        if (v.b || out.b) {
            L.b = alloc<float>((size_t) L.out);
            if (!L.b) return DLin();
            if (v.b) linear_simt(v.b, v.out, out.w, out.b, L.b, L.out, 1, out.out, out.in, st);
            else ok = cuda_ok(cudaMemcpyAsync(L.b, out.b, (size_t) L.out * 4, cudaMemcpyDeviceToDevice, st), "compose") && ok;
        }
        ok = cuda_ok(cudaStreamSynchronize(st), "compose") && ok;
        finish(L);
        return L;
    }
    // rows [row0, row0 + rows) of a linear as f32 w (+ bias) only, for the SIMT products of a handful of rows
    DLin lin_plain(const std::string & name, int64_t row0, int64_t rows) {
        DLin L;
        const gguf_tensor * t = m.get(name + ".weight");
        if (!t || !ok) return L;
        L.in = (int) t->ne[0];
        L.out = (int) rows;
        L.w = alloc<float>((size_t) L.in * L.out);
        if (!L.w || !dequant_into(t, row0, rows, L.w)) return DLin();
        if (m.get(name + ".bias")) L.b = vec(name + ".bias", row0, rows);
        return L;
    }
    // a forward-only linear: f32 w (+ bias) and the split planes of y = x W^T (no transposes)
    DLin lin_fwd_only(const std::string & name) {
        DLin L;
        const gguf_tensor * t = m.get(name + ".weight");
        if (!t || !ok) return L;
        L.in = (int) t->ne[0];
        L.out = (int) t->ne[1];
        L.w = alloc<float>((size_t) L.in * L.out);
        if (!L.w || !dequant_into(t, 0, L.out, L.w)) return DLin();
        if (m.get(name + ".bias")) L.b = vec(name + ".bias");
        L.w_hi = alloc<float>((size_t) L.in * L.out);
        L.w_lo = alloc<float>((size_t) L.in * L.out);
        if (!ok) return DLin();
        split_f32(L.w, L.in, L.w_hi, L.w_lo, L.in, L.out, L.in, st);
        ok = cuda_ok(cudaStreamSynchronize(st), "weight layout") && ok;
        return L;
    }
    // several forward-only linears of one input width stacked into one (their rows in order, a bias of zeros
    // where one has none): the attention's q, k and v when a file keeps them apart
    DLin lin_fwd_only_stacked(const std::vector<std::string> & names) {
        DLin L;
        std::vector<const gguf_tensor *> ts;
        for (const std::string & n : names) {
            const gguf_tensor * t = m.get(n + ".weight");
            if (!t || !ok || (!ts.empty() && t->ne[0] != ts[0]->ne[0])) return L;
            ts.push_back(t);
            L.out += (int) t->ne[1];
        }
        L.in = (int) ts[0]->ne[0];
        L.w = alloc<float>((size_t) L.in * L.out);
        bool any_bias = false;
        for (const std::string & n : names) any_bias = any_bias || m.get(n + ".bias");
        if (any_bias) L.b = alloc<float>((size_t) L.out);
        if (!ok) return DLin();
        if (L.b) cudaMemsetAsync(L.b, 0, (size_t) L.out * 4, st);
        int64_t r0 = 0;
        for (size_t i = 0; i < ts.size(); i++) {
            if (!dequant_into(ts[i], 0, ts[i]->ne[1], L.w + (size_t) r0 * L.in)) return DLin();
            if (m.get(names[i] + ".bias")) {
                float * b = vec(names[i] + ".bias");
                if (!b || !cuda_ok(cudaMemcpyAsync(L.b + r0, b, (size_t) ts[i]->ne[1] * 4, cudaMemcpyDeviceToDevice, st), "stack")) {
                    ok = false;
                    return DLin();
                }
            }
            r0 += ts[i]->ne[1];
        }
        L.w_hi = alloc<float>((size_t) L.in * L.out);
        L.w_lo = alloc<float>((size_t) L.in * L.out);
        if (!ok) return DLin();
        split_f32(L.w, L.in, L.w_hi, L.w_lo, L.in, L.out, L.in, st);
        ok = cuda_ok(cudaStreamSynchronize(st), "weight layout") && ok;
        return L;
    }
    DLin lin(const std::string & name, int64_t row0 = 0, int64_t rows = -1) {
        DLin L;
        const gguf_tensor * t = m.get(name + ".weight");
        if (!t || !ok) return L;
        if (rows < 0) rows = t->ne[1] - row0;
        L.in = (int) t->ne[0];
        L.out = (int) rows;
        L.w = alloc<float>((size_t) L.in * L.out);
        if (!L.w || !dequant_into(t, row0, rows, L.w)) return DLin();
        if (m.get(name + ".bias")) L.b = vec(name + ".bias", row0, rows);
        bool bf, bb;
        choose(t->type, rows, L.in, bf, bb);
        blocks(L, t, row0, rows, bf, bb);
        finish(L);
        return L;
    }
};


}  // namespace jb
