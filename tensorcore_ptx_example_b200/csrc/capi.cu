// capi.cu -- library-wide C ABI: versions, errors, device status, layout helpers and the
// codec diagnostics that pin the hardware conversions against the CPU oracle.
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "capi_internal.h"
#include "nvfp4_common.cuh"

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

// Elementwise codec probes: one thread per value.
__global__ void diag_e2m1_kernel(const float* __restrict__ x, uint8_t* __restrict__ out, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float v[8] = {x[i], 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    out[i] = (uint8_t)(e2m1x8(v) & 0xFu);
}

__global__ void diag_e4m3_kernel(const float* __restrict__ x, uint8_t* __restrict__ out, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    out[i] = (uint8_t)e4m3_encode(x[i]);
}

}  // namespace nvfp4

using namespace nvfp4;

extern "C" {

int nvfp4_abi_version(void) { return NVFP4_ABI_VERSION; }

const char* nvfp4_last_error_string(void) { return t_err; }

nvfp4_status_t nvfp4_device_status(unsigned int* status_out, int clear) {
    clear_error();
    unsigned int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_status, sizeof(v));
    if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "reading device status: %s", cudaGetErrorString(e));
    if (clear) {
        const unsigned int zero = 0;
        e = cudaMemcpyToSymbol(g_status, &zero, sizeof(zero));
        if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "clearing device status: %s", cudaGetErrorString(e));
    }
    if (status_out) *status_out = v;
    return NVFP4_OK;
}

int64_t nvfp4_packed_bytes(int64_t rows, int64_t cols) { return rows * cols / 2; }

int64_t nvfp4_sf_bytes(int64_t rows, int64_t cols) {
    return ((rows + 127) / 128) * ((cols + 63) / 64) * 512;
}

int64_t nvfp4_sf_offset(int64_t row, int64_t kblock, int64_t cols) {
    const int64_t katoms = (cols + 63) / 64;
    const int64_t atom = (row / 128) * katoms + kblock / 4;
    return atom * 512 + (row % 32) * 16 + ((row % 128) / 32) * 4 + (kblock % 4);
}

nvfp4_status_t nvfp4_diag_e2m1_encode(const float* x, uint8_t* out, int64_t n, void* stream) {
    clear_error();
    if (n < 0 || (n > 0 && (!x || !out))) return fail(NVFP4_ERR_INVALID_ARG, "diag_e2m1: bad arguments");
    if (n == 0) return NVFP4_OK;
    const int tpb = 256;
    diag_e2m1_kernel<<<(unsigned)((n + tpb - 1) / tpb), tpb, 0, (cudaStream_t)stream>>>(x, out, n);
    return check_launch("diag_e2m1_kernel");
}

nvfp4_status_t nvfp4_diag_e4m3_encode(const float* x, uint8_t* out, int64_t n, void* stream) {
    clear_error();
    if (n < 0 || (n > 0 && (!x || !out))) return fail(NVFP4_ERR_INVALID_ARG, "diag_e4m3: bad arguments");
    if (n == 0) return NVFP4_OK;
    const int tpb = 256;
    diag_e4m3_kernel<<<(unsigned)((n + tpb - 1) / tpb), tpb, 0, (cudaStream_t)stream>>>(x, out, n);
    return check_launch("diag_e4m3_kernel");
}

}  // extern "C"
