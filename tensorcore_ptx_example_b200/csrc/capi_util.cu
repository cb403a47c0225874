// capi_util.cu -- host-side helpers every C-ABI library of this package compiles in once:
// the calling thread's last-error message, launch checks and the SM count of the device.
// Included by the library translation units (nvfp4_lib.cu, diag_lib.cu); each .so keeps its
// own copy, hidden behind -fvisibility=hidden.
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "capi_internal.h"

namespace nvfp4 {

static thread_local char t_err[1024] = "";

nvfp4_status_t fail(nvfp4_status_t code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_err, sizeof(t_err), fmt, ap);
    va_end(ap);
    return code;
}

void clear_error() { t_err[0] = 0; }

const char* last_error() { return t_err; }

nvfp4_status_t check_launch(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return NVFP4_OK;
}

int sm_count() {
    static std::mutex mu;
    static int cache[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> g(mu);
    if (dev < 0 || dev >= 64) return 148;
    if (cache[dev] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = n > 0 ? n : 148;
    }
    return cache[dev];
}

}  // namespace nvfp4
