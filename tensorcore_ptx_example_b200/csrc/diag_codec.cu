// diag_codec.cu -- elementwise probes of the hardware conversions the NVFP4 path depends on
// (diagnostics library): the E2M1 and E4M3 encoders (cvt.rn.satfinite), pinned against the CPU
// oracle's restatement, and the approximate reciprocal rcp.approx.ftz.f32 that the reference's
// quantizer uses (recip_ftz, nvfp4_allreduce.cuh:110-114), evaluated here so the tests can model
// the reference kernel's output exactly.  Also this library's error string and status word.
#include "capi_internal.h"
#include "nvfp4_common.cuh"
#include "nvfp4_diag.h"

namespace nvfp4 {
namespace diag {

__global__ void e2m1_kernel(const float* __restrict__ x, uint8_t* __restrict__ out, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float v[8] = {x[i], 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    out[i] = (uint8_t)(e2m1x8(v) & 0xFu);
}

__global__ void e4m3_kernel(const float* __restrict__ x, uint8_t* __restrict__ out, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    out[i] = (uint8_t)e4m3_encode(x[i]);
}

__global__ void rcp_approx_kernel(const float* __restrict__ x, float* __restrict__ out, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x[i]));
    out[i] = r;
}

template <typename In, typename Out>
static nvfp4_status_t launch_elementwise(void (*kernel)(const In*, Out*, int64_t), const char* who, const In* x,
                                         Out* out, int64_t n, void* stream) {
    clear_error();
    if (n < 0 || (n > 0 && (!x || !out))) return fail(NVFP4_ERR_INVALID_ARG, "%s: bad arguments", who);
    if (n == 0) return NVFP4_OK;
    const int tpb = 256;
    kernel<<<(unsigned)((n + tpb - 1) / tpb), tpb, 0, (cudaStream_t)stream>>>(x, out, n);
    return check_launch(who);
}

}  // namespace diag
}  // namespace nvfp4

using namespace nvfp4;

extern "C" {

const char* nvfp4_diag_last_error_string(void) { return last_error(); }

nvfp4_status_t nvfp4_diag_device_status(unsigned int* status_out, int clear) {
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

nvfp4_status_t nvfp4_diag_e2m1_encode(const float* x, uint8_t* out, int64_t n, void* stream) {
    return diag::launch_elementwise(diag::e2m1_kernel, "diag_e2m1_encode", x, out, n, stream);
}

nvfp4_status_t nvfp4_diag_e4m3_encode(const float* x, uint8_t* out, int64_t n, void* stream) {
    return diag::launch_elementwise(diag::e4m3_kernel, "diag_e4m3_encode", x, out, n, stream);
}

nvfp4_status_t nvfp4_diag_rcp_approx(const float* x, float* out, int64_t n, void* stream) {
    return diag::launch_elementwise(diag::rcp_approx_kernel, "diag_rcp_approx", x, out, n, stream);
}

}  // extern "C"
