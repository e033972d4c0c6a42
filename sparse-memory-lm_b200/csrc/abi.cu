// Host-side plumbing shared by every entry point: thread-local error text, CUDA error mapping, SM counts.
#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"

namespace smlm {

static thread_local char g_error[512] = "";

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_error, sizeof(g_error), fmt, ap);
    va_end(ap);
}

int cuda_status(cudaError_t e, const char* what) {
    set_error("%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
    return SMLM_ERR_CUDA;
}

int sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 148;
    if (dev < 64 && cached[dev]) return cached[dev];
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    if (dev < 64) cached[dev] = n;
    return n;
}

}  // namespace smlm

extern "C" int smlm_version(void) { return 100; }

extern "C" const char* smlm_last_error(void) { return smlm::g_error; }
