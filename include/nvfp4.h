/*
 * nvfp4.h -- C ABI of the B200 (sm_100a) NVFP4 data path.
 *
 * Three subsystems, each hand-written CUDA for sm_100a, reached only through this header:
 *   1. bf16 -> NVFP4 quantizer (per-16 amax, UE4M3 block scale, fp32 global scale, E2M1
 *      packing; scale factors written directly in the tcgen05 scale-factor layout);
 *   2. block-scaled GEMM on tcgen05.mma kind::mxf4nvf4.block_scale.scale_vec::4X;
 *   3. NVFP4-compressed all-reduce over NVLink / NVSwitch peer memory, plus an in-house
 *      bf16 peer-to-peer all-reduce used as its baseline.
 *
 * Conventions
 *   - Every pointer argument named *_dev or a tensor buffer is DEVICE memory of the
 *     current device unless stated otherwise; `stream` is a cudaStream_t (NULL = legacy
 *     default stream).  Calls are asynchronous on `stream` and return after launch.
 *   - Host-side argument checks return NVFP4_ERR_INVALID_ARG and launch nothing.
 *     nvfp4_last_error_string() describes the last failure of the calling thread.
 *   - Device-side failures (a wait that ran out of time) are recorded in a per-device
 *     status word; read it with nvfp4_device_status() after synchronising.  No kernel of
 *     this library traps or waits without a time limit.
 *   - Tensors: bf16 activations / weights are row-major [rows][cols] with cols the
 *     reduction (K) dimension.  Packed NVFP4 data is row-major [rows][cols/2] bytes,
 *     element 2j in the low nibble of byte j.  Scale factors use the tcgen05 layout
 *     (nvfp4_sf_offset).  The global scale is gs = amax / (6 * 448); the reference's
 *     SFScaleVal is 1 / gs.
 *
 * Reference interfaces replaced (paths inside YijiaZhao/tensorcore_ptx_example):
 *   - blackwell/allreduce_sm100_sm120/nvfp4_allreduce.cuh:85-105   Layout        -> nvfp4_packed_bytes / nvfp4_sf_bytes
 *   - blackwell/allreduce_sm100_sm120/nvfp4_allreduce.cuh:427-454  quantize_kernel -> nvfp4_quantize_bf16
 *   - blackwell/allreduce_sm100_sm120/bench_ar.cu:760               host_global_scale -> nvfp4_amax_bf16
 *   - blackwell/allreduce_sm100_sm120/nvfp4_allreduce.cuh:305-317  dq32_acc      -> nvfp4_dequantize_bf16
 *   - blackwell/warp_specialization_sm100/sm100_tcgen05_nvfp4_tma_multistage_pipeline.cu:117
 *     ws_tcgen05_explicit_pipeline_kernel + p2::run() :336         -> nvfp4_gemm_bf16 / nvfp4_gemm_f32
 *   - blackwell/tcgen05_fp4_sm100/tcgen05_nvfp4_block16_ue4m3_maxtile_m128n256.cu:98,167
 *     (single M128xN256 tile + run())                               -> nvfp4_gemm_f32 (one tile)
 *   - blackwell/allreduce_sm100_sm120/nvfp4_allreduce.cuh:650-682  launch_fused_rank /
 *     launch_oneshot_fused_rank                                      -> nvfp4_ar_allreduce
 *   - blackwell/allreduce_sm100_sm120/nvfp4_allreduce.cuh:344-352,398  fused_comm_bytes /
 *     oneshot_comm_bytes / fused_barrier_words (caller-allocated)   -> nvfp4_ar_create (library-owned)
 *   - blackwell/allreduce_sm100_sm120/bench_ar.cu:770-772,833-850   peer pointer setup ->
 *     nvfp4_ar_set_peers_inprocess / nvfp4_ar_ipc_handle + nvfp4_ar_open_peers
 *   - blackwell/allreduce_sm100_sm120/bench_ar.cu:83,132 (third-party bf16 kernels used as
 *     the baseline)                                                  -> nvfp4_bf16_allreduce (own code)
 */
#ifndef NVFP4_B200_H
#define NVFP4_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NVFP4_ABI_VERSION 1

#if defined(__GNUC__)
#define NVFP4_API __attribute__((visibility("default")))
#else
#define NVFP4_API
#endif

typedef int nvfp4_status_t;
#define NVFP4_OK 0
#define NVFP4_ERR_INVALID_ARG 1
#define NVFP4_ERR_CUDA 2
#define NVFP4_ERR_TIMEOUT 3
#define NVFP4_ERR_UNSUPPORTED 4
#define NVFP4_ERR_NOT_READY 5

/* ------------------------------------------------------------- library ---- */
NVFP4_API int nvfp4_abi_version(void);
/* Human-readable description of the calling thread's last error ("" if none). */
NVFP4_API const char* nvfp4_last_error_string(void);
/* Reads (and, if clear != 0, resets) the device status word of the current device.
 * Synchronous.  0 = no device-side failure recorded; otherwise a DEV_* code (see
 * nvfp4_common.cuh).  Returns NVFP4_OK or NVFP4_ERR_CUDA. */
NVFP4_API nvfp4_status_t nvfp4_device_status(unsigned int* status_out, int clear);

/* -------------------------------------------------- layout (host only) ---- */
/* Bytes of packed E2M1 data for rows x cols (rows * cols / 2). */
NVFP4_API int64_t nvfp4_packed_bytes(int64_t rows, int64_t cols);
/* Bytes of the scale-factor buffer in the tcgen05 layout:
 * ceil(rows/128) * ceil(cols/64) * 512. */
NVFP4_API int64_t nvfp4_sf_bytes(int64_t rows, int64_t cols);
/* Byte offset of the block scale of (row, kblock = col / 16):
 *   atom = (row / 128) * ceil(cols / 64) + kblock / 4
 *   offset = atom * 512 + (row % 32) * 16 + ((row % 128) / 32) * 4 + kblock % 4 */
NVFP4_API int64_t nvfp4_sf_offset(int64_t row, int64_t kblock, int64_t cols);

/* ----------------------------------------------------------- quantizer ---- */
/* amax_dev[0] = max |x| over numel bf16 values (device float; overwritten).
 * numel % 8 == 0, x 16-byte aligned. */
NVFP4_API nvfp4_status_t nvfp4_amax_bf16(const void* x, int64_t numel, float* amax_dev, void* stream);

/* Quantize a rows x cols bf16 tensor with a given global scale gs (> 0).
 * cols % 64 == 0; x, packed and sf 16-byte aligned.  Writes rows*cols/2 bytes of packed
 * data and all nvfp4_sf_bytes(rows, cols) scale bytes (padding rows get scale 0). */
NVFP4_API nvfp4_status_t nvfp4_quantize_bf16(const void* x, int64_t rows, int64_t cols, float global_scale,
                                   void* packed, void* sf, void* stream);

/* Same, with the global scale computed on the device from the tensor's own amax
 * (gs = amax / 2688, amax 0 -> gs 1).  Writes gs to global_scale_dev[0].  Two kernels
 * (amax reduction, then quantize); no host synchronisation.  The amax travels between the
 * two kernels through `workspace`, a device scratch buffer of at least
 * nvfp4_quantize_workspace_bytes() bytes (its contents on entry do not matter). */
NVFP4_API size_t nvfp4_quantize_workspace_bytes(void);
NVFP4_API nvfp4_status_t nvfp4_quantize_bf16_auto(const void* x, int64_t rows, int64_t cols, void* packed,
                                        void* sf, float* global_scale_dev, void* workspace,
                                        void* stream);

/* nvfp4_quantize_bf16_auto for callers that cannot allocate device memory (no counterpart
 * in the reference).  Same arguments and results minus `workspace`: the amax hand-off uses a
 * fixed 256-byte file-scope device array of this library instead (one per device, held until
 * the process exits; the scratch it needs does not grow with rows x cols).  It calls no
 * cudaMalloc / cudaFree.  The first call on a device looks the array's address up with
 * cudaGetSymbolAddress: make that call before any stream capture.  All calls on a device share
 * the array and clear it on `stream` before use, so calls that overlap on the GPU race. */
NVFP4_API nvfp4_status_t nvfp4_quantize_bf16_auto_noalloc(const void* x, int64_t rows, int64_t cols, void* packed,
                                                void* sf, float* global_scale_dev, void* stream);

/* Dequantize to bf16: out = bf16(e2m1(code) * (ue4m3(scale) * gs)). */
NVFP4_API nvfp4_status_t nvfp4_dequantize_bf16(const void* packed, const void* sf, int64_t rows, int64_t cols,
                                     float global_scale, void* out, void* stream);

/* ---------------------------------------------------------------- GEMM ---- */
/* D[M][N] = bf16(alpha * sum_k A[m][k] B[n][k] sfa sfb), fp32 accumulation in TMEM.
 * A: packed M x K, sfa: nvfp4_sf_bytes(M, K); B: packed N x K (weights, K-major),
 * sfb: nvfp4_sf_bytes(N, K); D: bf16 row-major M x N.  alpha = gsA * gsB.
 * Requires M % 128 == 0, N % 256 == 0, K % 256 == 0, 16-byte aligned buffers. */
NVFP4_API nvfp4_status_t nvfp4_gemm_bf16(const void* A, const void* sfa, const void* B, const void* sfb,
                               float alpha, void* D, int64_t M, int64_t N, int64_t K, void* stream);
/* Same kernel, raw fp32 accumulators (no alpha) into D (fp32 row-major M x N). */
NVFP4_API nvfp4_status_t nvfp4_gemm_f32(const void* A, const void* sfa, const void* B, const void* sfb,
                              float* D, int64_t M, int64_t N, int64_t K, void* stream);

/* ----------------------------------------------------------- diagnostics ---- */
/* Device codec probes (used by the parity tests to pin the hardware conversions):
 * out[i] = E2M1 code of x[i] (RNE, satfinite) / E4M3 code of x[i]. */
NVFP4_API nvfp4_status_t nvfp4_diag_e2m1_encode(const float* x, uint8_t* out, int64_t n, void* stream);
NVFP4_API nvfp4_status_t nvfp4_diag_e4m3_encode(const float* x, uint8_t* out, int64_t n, void* stream);
/* FP4 tensor-core issue-rate microbenchmark: every SM (cta_group 1, M128 N256) or SM pair
 * (cta_group 2, M256 N256) issues `iters` K64 block-scaled MMAs from resident shared memory,
 * on sparse constant operands or (random_operands != 0) pseudo-random E2M1 codes.
 * FLOPs = 2 * 128 * 256 * 64 * iters * (number of SMs); time it with events around the call.
 * The measured rate is the roofline denominator of nvfp4_gemm_bf16. */
NVFP4_API nvfp4_status_t nvfp4_diag_mma_peak(int cta_group, int iters, int random_operands, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* NVFP4_B200_H */
