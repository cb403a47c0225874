// ref_ar_shim.cu -- exports the reference's NVFP4 all-reduce kernels as a C ABI.
//
// TEST / MEASUREMENT INFRASTRUCTURE ONLY.  #includes the UNMODIFIED reference header
// blackwell/allreduce_sm100_sm120/nvfp4_allreduce.cuh from the read-only reference tree
// (include path set by oracle/Makefile).  The built library (oracle/_ref/libref_ar.so) lets
// the GPU box run the reference's own quantize / fused one-shot / fused two-shot kernels
// beside this project's kernels for a same-box comparison (the quantizer parity test, and the
// benchmark's reference-kernel baselines).  Nothing in the product links against it.  The
// ref_ipc_* / ref_dev_* helpers at the end only allocate and share the buffers the reference
// launchers require (zeroed device memory, CUDA IPC handles, device arrays of peer pointers).
#include <cstdint>
#include <cstddef>
#include <cstring>

#include "nvfp4_allreduce.cuh"   // the reference header, found through -I

// Blocks of a fused kernel that can be resident at once on the current device (256 threads per
// block, the launchers' default).  The fused kernels wait in block_barrier for the same block
// index on every rank, so a grid no larger than this always makes progress.
template <typename K>
static int resident_blocks(K kernel) {
    int per_sm = 0, dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, 256, 0) != cudaSuccess) return -1;
    return per_sm * sms;
}

extern "C" {

// Host-side geometry helpers of the reference (nvfp4_allreduce.cuh:344-352, :398, :628-642).
size_t ref_column_bytes(size_t elts) { return nvfp4_ar::column_bytes(elts); }
size_t ref_fused_comm_bytes(size_t shard, int world) { return nvfp4_ar::fused_comm_bytes(shard, world); }
size_t ref_oneshot_comm_bytes(size_t numel, int world) { return nvfp4_ar::oneshot_comm_bytes(numel, world); }
size_t ref_fused_barrier_words(int world) { return nvfp4_ar::fused_barrier_words(world); }
int ref_default_fused_grid(size_t elts, int tpb) { return nvfp4_ar::default_fused_grid(elts, tpb); }
size_t ref_layout_total_bytes(size_t numel) { return nvfp4_ar::Layout::make(numel).total_bytes; }

// Reference quantize_kernel (linear scale layout, footer global scale), :427-454.
int ref_quantize(const void* in, void* out, size_t numel, float SFScaleVal, void* stream) {
    const nvfp4_ar::Layout L = nvfp4_ar::Layout::make(numel);
    const int tpb = 256;
    const int grid = int((numel / nvfp4_ar::ELTS_PER_THREAD + tpb - 1) / tpb);
    nvfp4_ar::quantize_kernel<<<grid, tpb, 0, (cudaStream_t)stream>>>(
        (const __nv_bfloat16*)in, (uint8_t*)out, L, SFScaleVal);
    return (int)cudaGetLastError();
}

// Reference fused two-shot / one-shot launchers (:650-682).  peer_comm / barrier arrays are
// DEVICE arrays of `world` pointers on the calling device, as the reference requires.
int ref_launch_twoshot(int world, const void* in, void* out, void* peer_comm, void* bar_in,
                       void* bar_out, int rank, size_t numel, float SF, uint32_t flag,
                       void* stream, int grid) {
    auto comm = (uint8_t**)peer_comm;
    auto bi = (uint32_t**)bar_in;
    auto bo = (uint32_t**)bar_out;
    auto s = (cudaStream_t)stream;
    auto x = (const __nv_bfloat16*)in;
    auto y = (__nv_bfloat16*)out;
    switch (world) {
        case 2: nvfp4_ar::launch_fused_rank<2>(x, y, comm, bi, bo, rank, numel, SF, flag, s, 256, grid); break;
        case 4: nvfp4_ar::launch_fused_rank<4>(x, y, comm, bi, bo, rank, numel, SF, flag, s, 256, grid); break;
        case 8: nvfp4_ar::launch_fused_rank<8>(x, y, comm, bi, bo, rank, numel, SF, flag, s, 256, grid); break;
        default: return -1;
    }
    return (int)cudaGetLastError();
}

int ref_launch_oneshot(int world, const void* in, void* out, void* peer_comm, void* bar,
                       int rank, size_t numel, float SF, uint32_t flag, void* stream, int grid) {
    auto comm = (uint8_t**)peer_comm;
    auto b = (uint32_t**)bar;
    auto s = (cudaStream_t)stream;
    auto x = (const __nv_bfloat16*)in;
    auto y = (__nv_bfloat16*)out;
    switch (world) {
        case 2: nvfp4_ar::launch_oneshot_fused_rank<2>(x, y, comm, b, rank, numel, SF, flag, s, 256, grid); break;
        case 4: nvfp4_ar::launch_oneshot_fused_rank<4>(x, y, comm, b, rank, numel, SF, flag, s, 256, grid); break;
        case 8: nvfp4_ar::launch_oneshot_fused_rank<8>(x, y, comm, b, rank, numel, SF, flag, s, 256, grid); break;
        default: return -1;
    }
    return (int)cudaGetLastError();
}

int ref_fused_resident_blocks(int world, int oneshot) {
    switch (world) {
        case 2: return oneshot ? resident_blocks(nvfp4_ar::oneshot_fused_kernel<2>) : resident_blocks(nvfp4_ar::twoshot_fused_kernel<2>);
        case 4: return oneshot ? resident_blocks(nvfp4_ar::oneshot_fused_kernel<4>) : resident_blocks(nvfp4_ar::twoshot_fused_kernel<4>);
        case 8: return oneshot ? resident_blocks(nvfp4_ar::oneshot_fused_kernel<8>) : resident_blocks(nvfp4_ar::twoshot_fused_kernel<8>);
        default: return -1;
    }
}

// ---- buffer plumbing for the reference launchers (not reference code) ----
// Zeroed device allocation of `bytes`.
int ref_dev_alloc_zero(size_t bytes, void** ptr) {
    *ptr = nullptr;
    cudaError_t e = cudaMalloc(ptr, bytes);
    if (e == cudaSuccess) e = cudaMemset(*ptr, 0, bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    return (int)e;
}
int ref_dev_free(void* ptr) { return (int)cudaFree(ptr); }
// Device array of n pointers (the peer tables the launchers take).
int ref_dev_ptr_array(void* const* host_ptrs, int n, void** dev_array) {
    cudaError_t e = cudaMalloc(dev_array, sizeof(void*) * (size_t)n);
    if (e == cudaSuccess) e = cudaMemcpy(*dev_array, host_ptrs, sizeof(void*) * (size_t)n, cudaMemcpyHostToDevice);
    return (int)e;
}
size_t ref_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }
int ref_ipc_get(void* ptr, void* handle_out) {
    return (int)cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(handle_out), ptr);
}
int ref_ipc_open(const void* handle, void** ptr) {
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    return (int)cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
}
int ref_ipc_close(void* ptr) { return (int)cudaIpcCloseMemHandle(ptr); }

}  // extern "C"
