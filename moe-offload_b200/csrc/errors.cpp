// Error reporting for the C ABI: every failing entry point records a per-thread message
// (moe_last_error) and returns a negative status code.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>

#include "../../include/moe_b200.h"

namespace {
thread_local char g_msg[512] = "";
}

int moe_set_error(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
    va_end(ap);
    return code;
}

int moe_set_cuda_error(cudaError_t e) {
    snprintf(g_msg, sizeof(g_msg), "CUDA error %d: %s", (int)e, cudaGetErrorString(e));
    return MOE_ECUDA;
}

extern "C" const char *moe_last_error(void) { return g_msg; }

extern "C" int moe_version(void) { return 100; }
