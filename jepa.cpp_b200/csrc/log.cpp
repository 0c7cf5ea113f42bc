// Diagnostics: every message goes to stderr and to the calling thread's capture buffer, which
// jepa_error_text() returns (reference contract: include/jepa.h:597-611, src/jepa.cpp:16-36).
#include "common.h"
#include "../../include/jepa.h"

#include <string>

namespace jb {

namespace {
constexpr size_t CAPTURE_MAX = 8192;
thread_local std::string g_capture;
}  // namespace

void log(const char * fmt, ...) {
    char buf[2048];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    fputs(buf, stderr);
    g_capture += buf;
    if (g_capture.size() > CAPTURE_MAX) g_capture.erase(0, g_capture.size() - CAPTURE_MAX);
}

bool cuda_ok(cudaError_t e, const char * what) {
    if (e == cudaSuccess) return true;
    log("jepa: CUDA error in %s: %s\n", what, cudaGetErrorString(e));
    return false;
}

}  // namespace jb

extern "C" void jepa_error_reset(void) { jb::g_capture.clear(); }
extern "C" const char * jepa_error_text(void) { return jb::g_capture.c_str(); }
