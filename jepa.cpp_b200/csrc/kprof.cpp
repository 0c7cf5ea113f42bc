// Per-kernel device timing (see kprof.h) and its C entry points.
#include "kprof.h"

#include "../../include/jepa_b200.h"

#include <cstdio>
#include <map>
#include <mutex>
#include <string>
#include <vector>

namespace jb {

bool g_kprof_on = false;

namespace {

struct Rec {
    std::string kind;
    cudaEvent_t e0, e1;
    double flops, bytes;
};

std::mutex g_mu;
std::vector<Rec> g_recs;

void clear_locked() {
    for (auto & r : g_recs) {
        cudaEventDestroy(r.e0);
        cudaEventDestroy(r.e1);
    }
    g_recs.clear();
}

}  // namespace

KTimer::KTimer(const char * k, cudaStream_t s, double f, double b) {
    if (!g_kprof_on) return;
    kind = k;
    st = s;
    flops = f;
    bytes = b;
    cudaEventCreate(&e0);
    cudaEventRecord(e0, st);
}

KTimer::~KTimer() {
    if (!e0) return;
    cudaEvent_t e1;
    cudaEventCreate(&e1);
    cudaEventRecord(e1, st);
    std::lock_guard<std::mutex> lk(g_mu);
    g_recs.push_back({kind, e0, e1, flops, bytes});
}

}  // namespace jb

extern "C" void jepa_b200_kprof_begin(void) {
    std::lock_guard<std::mutex> lk(jb::g_mu);
    jb::clear_locked();
    jb::g_kprof_on = true;
}

extern "C" int jepa_b200_kprof_end(char * out, size_t cap) {
    std::lock_guard<std::mutex> lk(jb::g_mu);
    jb::g_kprof_on = false;
    struct Agg { long long n = 0; double ms = 0, flops = 0, bytes = 0; };
    std::map<std::string, Agg> agg;
    bool ok = true;
    for (auto & r : jb::g_recs) {
        float t = 0;
        if (cudaEventSynchronize(r.e1) != cudaSuccess || cudaEventElapsedTime(&t, r.e0, r.e1) != cudaSuccess) ok = false;
        Agg & a = agg[r.kind];
        a.n++;
        a.ms += t;
        a.flops += r.flops;
        a.bytes += r.bytes;
    }
    jb::clear_locked();
    std::string s;
    char line[256];
    for (auto & kv : agg) {
        snprintf(line, sizeof(line), "%s %lld %.6f %.6e %.6e\n", kv.first.c_str(), kv.second.n, kv.second.ms, kv.second.flops,
                 kv.second.bytes);
        s += line;
    }
    if (out && cap > 0) {
        const size_t n = s.size() < cap - 1 ? s.size() : cap - 1;
        s.copy(out, n);
        out[n] = 0;
    }
    return ok ? (int) agg.size() : -1;
}
