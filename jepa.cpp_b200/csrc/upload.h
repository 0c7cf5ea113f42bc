// Weight upload from a GGUF model to the device: float32 planes, their transposes and the 3xTF32 split
// planes of the tensor-core products (dequantised on the device, bit-exact with the block formats).
// Every allocation goes into the owner's list, which frees them.
#pragma once

#include "hplan.h"
#include "kernels.h"
#include "model.h"
#include "gguf.h"
#include "common.h"

#include <algorithm>
#include <string>
#include <vector>

namespace jb {

struct Uploader {
    std::vector<void *> & allocs;   // every allocation, freed by the owner
    const jepa_model & m;
    cudaStream_t st;
    bool ok = true;
    std::vector<void *> temps;

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
    void finish(DLin & L) {
        if (!ok) return;
        L.wt = alloc<float>((size_t) L.in * L.out);
        L.w_hi = alloc<float>((size_t) L.in * L.out); L.w_lo = alloc<float>((size_t) L.in * L.out);
        L.wt_hi = alloc<float>((size_t) L.in * L.out); L.wt_lo = alloc<float>((size_t) L.in * L.out);
        if (!ok) return;
        transpose_f32(L.w, L.wt, L.out, L.in, st);
        split_f32(L.w, L.in, L.w_hi, L.w_lo, L.in, L.out, L.in, st);
        split_f32(L.wt, L.out, L.wt_hi, L.wt_lo, L.out, L.in, L.out, st);
        ok = cuda_ok(cudaStreamSynchronize(st), "weight layout") && ok;
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
        if (gemm_tc({out.w_hi, out.w_lo, out.in}, {v.wt_hi, v.wt_lo, v.out}, out.out, v.in, v.out, ep, st)) { ok = false; return DLin(); }
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
        finish(L);
        return L;
    }
};


}  // namespace jb
