// capi.cu -- library-wide C ABI: version, errors, device status and layout helpers.
#include "capi_internal.h"
#include "nvfp4_common.cuh"

using namespace nvfp4;

extern "C" {

int nvfp4_abi_version(void) { return NVFP4_ABI_VERSION; }

const char* nvfp4_last_error_string(void) { return last_error(); }

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

}  // extern "C"
