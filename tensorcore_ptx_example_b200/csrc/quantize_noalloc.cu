// quantize_noalloc.cu -- the auto-scaled quantizer for callers that cannot allocate.
//
// nvfp4_quantize_bf16_auto hands the tensor amax from the reduction kernel to the quantize
// kernel through a caller-provided device workspace.  Some callers have no way to provide
// one: code that runs where cudaMalloc is forbidden or unsafe (inside a custom allocator's own
// callbacks, in a plugin whose host framework owns all device memory and exposes no scratch
// API, or on a path that must not synchronise the device, which cudaMalloc/cudaFree may do).
// nvfp4_quantize_bf16_auto_noalloc serves them: its scratch is a fixed file-scope device
// array that exists once per device for as long as the library stays loaded.
//
// Contract (repeated in include/nvfp4.h):
//   - scratch size: NOALLOC_SCRATCH_BYTES (256) bytes per device; the amax hand-off uses
//     nvfp4_quantize_workspace_bytes() of it.  The need does not grow with rows x cols; a
//     build whose workspace requirement exceeded the array would be rejected with
//     NVFP4_ERR_UNSUPPORTED.
//   - set-up: the first call on a device looks up the device address of the array with
//     cudaGetSymbolAddress while that device is current, and caches it for the life of the
//     process.  Make that first call before any stream capture.  Do not use the entry point on
//     a device after cudaDeviceReset: the reset reloads the module and the cached address
//     would be stale.
//   - no cudaMalloc, cudaFree or allocating library routine is called; the amax word is
//     cleared with cudaMemsetAsync on `stream` before every use.
//   - every call on a device shares the one array: calls that overlap on the GPU (different
//     streams without ordering between them) race on it and may produce wrong scales.
#include <mutex>

#include "capi_internal.h"

namespace nvfp4 {

constexpr size_t NOALLOC_SCRATCH_BYTES = 256;

// Device-side scratch.  In host code this name is only a host stand-in for the symbol, never
// a device address: the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

constexpr int NOALLOC_MAX_DEVICES = 64;

// Device address of g_noalloc_scratch on the current device, looked up once per device.
static nvfp4_status_t noalloc_scratch(void** out) {
    static std::mutex mu;
    static void* addr[NOALLOC_MAX_DEVICES] = {};
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "quantize_auto_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= NOALLOC_MAX_DEVICES)
        return fail(NVFP4_ERR_UNSUPPORTED, "quantize_auto_noalloc: device ordinal %d >= %d", dev, NOALLOC_MAX_DEVICES);
    std::lock_guard<std::mutex> g(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return fail(NVFP4_ERR_CUDA, "quantize_auto_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        addr[dev] = p;
    }
    *out = addr[dev];
    return NVFP4_OK;
}

}  // namespace nvfp4

using namespace nvfp4;

extern "C" {

nvfp4_status_t nvfp4_quantize_bf16_auto_noalloc(const void* x, int64_t rows, int64_t cols, void* packed, void* sf,
                                                float* global_scale_dev, void* stream) {
    clear_error();
    if (nvfp4_quantize_workspace_bytes() > NOALLOC_SCRATCH_BYTES)
        return fail(NVFP4_ERR_UNSUPPORTED, "quantize_auto_noalloc: needs %zu scratch bytes, the static array holds %zu",
                    nvfp4_quantize_workspace_bytes(), NOALLOC_SCRATCH_BYTES);
    void* ws = nullptr;
    const nvfp4_status_t st = noalloc_scratch(&ws);
    if (st != NVFP4_OK) return st;
    return nvfp4_quantize_bf16_auto(x, rows, cols, packed, sf, global_scale_dev, ws, stream);
}

}  // extern "C"
