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
 *     nvfp4_ar_set_peers (one process) / nvfp4_ar_export_handle + nvfp4_ar_open_peers (IPC)
 *   - blackwell/allreduce_sm100_sm120/bench_ar.cu:83,132 (third-party bf16 kernels used as
 *     the baseline)                                                  -> nvfp4_ar_bf16_allreduce (own code)
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
/* amax_dev[0] = max |x| over the finite values among numel bf16 values (device float;
 * overwritten).  NaN and Inf are skipped and recorded as a device status (DEV_NONFINITE_INPUT,
 * 0x302, read with nvfp4_device_status).  numel % 8 == 0, x 16-byte aligned. */
NVFP4_API nvfp4_status_t nvfp4_amax_bf16(const void* x, int64_t numel, float* amax_dev, void* stream);

/* Quantize a rows x cols bf16 tensor with a given global scale gs (> 0).
 * cols % 64 == 0; x, packed and sf 16-byte aligned.  Writes rows*cols/2 bytes of packed
 * data and all nvfp4_sf_bytes(rows, cols) scale bytes (padding rows get scale 0).
 * Non-finite input: a 16-element block holding a NaN or an Inf gets scale byte 0x7F (the E4M3
 * NaN, so the block dequantizes to NaN; NVFP4 has no encoding for non-finite values) and zero
 * codes, and the device status DEV_NONFINITE_INPUT (0x302) is recorded. */
NVFP4_API nvfp4_status_t nvfp4_quantize_bf16(const void* x, int64_t rows, int64_t cols, float global_scale,
                                   void* packed, void* sf, void* stream);

/* Same, with the global scale computed on the device from the tensor's own amax over its finite
 * values (gs = amax / 2688, amax 0 -> gs 1; an empty tensor also gets gs 1).  Writes gs to
 * global_scale_dev[0].  Two kernels
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
 * cudaGetSymbolAddress and keeps it for the life of the process: make that call before any
 * stream capture, and do not use this entry point on a device after cudaDeviceReset (the reset
 * reloads the module, and the kept address would be stale).  All calls on a device share the
 * array and clear it on `stream` before use, so calls that overlap on the GPU race. */
NVFP4_API nvfp4_status_t nvfp4_quantize_bf16_auto_noalloc(const void* x, int64_t rows, int64_t cols, void* packed,
                                                void* sf, float* global_scale_dev, void* stream);

/* Dequantize to bf16: out = bf16(e2m1(code) * (ue4m3(scale) * gs)). */
NVFP4_API nvfp4_status_t nvfp4_dequantize_bf16(const void* packed, const void* sf, int64_t rows, int64_t cols,
                                     float global_scale, void* out, void* stream);

/* ---------------------------------------------------------------- GEMM ---- */
/* D[M][N] = bf16(alpha * sum_k A[m][k] B[n][k] sfa sfb), fp32 accumulation in TMEM.
 * A: packed M x K, sfa: nvfp4_sf_bytes(M, K); B: packed N x K (weights, K-major),
 * sfb: nvfp4_sf_bytes(N, K); D: bf16 row-major M x N.  alpha = gsA * gsB.
 * Requires K % 256 == 0, 16-byte aligned buffers, and either M % 128 == 0 with N % 256 == 0
 * (tiled kernels), or 0 < M < 128 with N % 128 == 0 (decode shapes: a split-K kernel over
 * 128-row tiles of B whose fp32 partials are summed in split order 0..S-1 before alpha and the
 * bf16 rounding -- inside thread-block clusters when the S <= 8 splits of a tile fit one, which
 * needs no workspace, else through a workspace: a buffer the library allocates once per device
 * for nvfp4_gemm_bf16, or the caller's for nvfp4_gemm_bf16_ws). */
NVFP4_API nvfp4_status_t nvfp4_gemm_bf16(const void* A, const void* sfa, const void* B, const void* sfb,
                               float alpha, void* D, int64_t M, int64_t N, int64_t K, void* stream);
/* Workspace bytes nvfp4_gemm_bf16_ws needs for this shape (0 for M % 128 == 0 and for decode
 * shapes reduced in-cluster; the workspace may then be NULL). */
NVFP4_API size_t nvfp4_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K);
NVFP4_API nvfp4_status_t nvfp4_gemm_bf16_ws(const void* A, const void* sfa, const void* B, const void* sfb,
                                  float alpha, void* D, int64_t M, int64_t N, int64_t K, void* workspace,
                                  size_t workspace_bytes, void* stream);
/* nvfp4_gemm_bf16 with flags (an extension of this library).  NVFP4_GEMM_WEIGHTS_CONST: B and
 * sfb are not written by work queued before this call on `stream` (model weights).  The decode
 * kernel (0 < M < 128) then starts streaming B before it waits for the preceding kernel
 * (programmatic dependent launch), overlapping that kernel's tail; A and sfa are still read only
 * after the wait.  The tiled kernels ignore the flag.  Results are identical with or without it. */
#define NVFP4_GEMM_WEIGHTS_CONST 1
NVFP4_API nvfp4_status_t nvfp4_gemm_bf16_flags(const void* A, const void* sfa, const void* B, const void* sfb,
                                     float alpha, void* D, int64_t M, int64_t N, int64_t K, int flags,
                                     void* stream);
/* Same kernel, raw fp32 accumulators (no alpha) into D (fp32 row-major M x N). */
NVFP4_API nvfp4_status_t nvfp4_gemm_f32(const void* A, const void* sfa, const void* B, const void* sfb,
                              float* D, int64_t M, int64_t N, int64_t K, void* stream);

/* GEMM with the quantizer fused into its epilogue, for back-to-back NVFP4 layers (no direct
 * counterpart in the reference: it composes the GEMM above with nvfp4_quantize_bf16).
 * Writes exactly the bytes of nvfp4_gemm_bf16 followed by nvfp4_quantize_bf16(D, gs_out):
 * D_packed (M x N/2 bytes, E2M1 codes) and D_sf (nvfp4_sf_bytes(M, N), tcgen05 layout), without
 * the bf16 D ever reaching memory.  gs_out is the global scale of D, given (finite, > 0).
 * Requires M % 256 == 0, N % 256 == 0, K % 256 == 0, 32-byte aligned D_packed. */
NVFP4_API nvfp4_status_t nvfp4_gemm_quantize(const void* A, const void* sfa, const void* B, const void* sfb,
                                   float alpha, float gs_out, void* D_packed, void* D_sf, int64_t M,
                                   int64_t N, int64_t K, void* stream);

/* ----------------------------------------------------------- all-reduce ---- */
/* NVFP4-compressed all-reduce of bf16 tensors across the GPUs of one node over NVLink /
 * NVSwitch peer memory, and the in-house bf16 peer-to-peer all-reduce it is measured
 * against.  One context per rank, created on that rank's GPU (current device); every rank
 * makes the same sequence of calls (same numel, algo, order) on its own stream.
 *
 * Reference: nvfp4_ar::launch_fused_rank / launch_oneshot_fused_rank
 * (blackwell/allreduce_sm100_sm120/nvfp4_allreduce.cuh:650-682) with caller-allocated comm
 * buffers (fused_comm_bytes / oneshot_comm_bytes / fused_barrier_words, :344-352, :398) and peer
 * pointer tables (bench_ar.cu:770-772, :833-850).  Here the context owns the buffers and the
 * barrier words; every wait is bounded; results do not depend on the number of ranks' launch
 * order: sums run in rank order 0..n-1.
 *
 * out = bf16(sum over ranks r = 0..n-1 of dequant(quant(in_r)))     (one-shot), or, two-shot,
 * each shard's fp32 sum requantized with global scale gs * n and dequantized.  Quantization is
 * NVFP4 with per-16 UE4M3 scales and the caller's global scale gs (same on every rank; the
 * reference's SFScaleVal is 1 / gs). */
typedef struct nvfp4_ar* nvfp4_ar_t;
#define NVFP4_AR_AUTO 0
#define NVFP4_AR_ONESHOT 1
#define NVFP4_AR_TWOSHOT 2
/* One-shot whose barrier is replaced by flags carried in the data (8-byte words: 7 bytes of
 * payload + a tag byte, as in NCCL's LL protocol): one fewer NVLink round trip, 1.33x the bytes
 * on the wire.  Same results as NVFP4_AR_ONESHOT.  NVFP4 only; at most
 * NVFP4_AR_LOWLAT_CAP_BYTES of bf16 per call. */
#define NVFP4_AR_LOWLAT 3
#define NVFP4_AR_LOWLAT_CAP_BYTES (1 << 20)
/* bf16 all-reduce whose sum is done inside the NVSwitch (NVLS): multimem.ld_reduce.add.acc::f32
 * through a multicast address returns the fp32 sum over every rank's buffer, multimem.st writes
 * it back to every rank (reference: the multimem reduction demo,
 * blackwell/comm_primitives_sm100_sm120/minimal_multimem_reduce.cu:68-80).  nvfp4_ar_bf16_allreduce
 * only, after nvfp4_ar_set_multicast; never chosen by NVFP4_AR_AUTO.  The switch orders the fp32
 * additions, so results equal the exact sum rounded once to bf16 except where fp32 rounding of
 * the partial sums moves a value across a bf16 rounding boundary (within 1 bf16 ulp). */
#define NVFP4_AR_NVLS 4
/* NVFP4_AR_AUTO picks the low-latency one-shot up to NVFP4_AR_LOWLAT_MAX_BYTES of bf16,
 * one-shot up to NVFP4_AR_ONESHOT_MAX_BYTES, two-shot above. */
#define NVFP4_AR_LOWLAT_MAX_BYTES (1 << 20)
#define NVFP4_AR_ONESHOT_MAX_BYTES (2 << 20)

/* Device bytes a context allocates (flags + two parities of comm buffers + two parities of the
 * low-latency area). */
NVFP4_API int64_t nvfp4_ar_buffer_bytes(int world, int64_t max_numel);
/* world 1..8, rank in [0, world); max_numel: largest numel any call will use. */
NVFP4_API nvfp4_status_t nvfp4_ar_create(int world, int rank, int64_t max_numel, nvfp4_ar_t* out);
NVFP4_API nvfp4_status_t nvfp4_ar_destroy(nvfp4_ar_t h);
/* Multi-process set-up: export this rank's buffer (nvfp4_ar_handle_bytes() bytes, a CUDA IPC
 * handle), gather every rank's export in rank order, then open the peers' buffers. */
NVFP4_API size_t nvfp4_ar_handle_bytes(void);
NVFP4_API nvfp4_status_t nvfp4_ar_export_handle(nvfp4_ar_t h, void* handle_out);
NVFP4_API nvfp4_status_t nvfp4_ar_open_peers(nvfp4_ar_t h, const void* handles);
/* Single-process set-up (one thread drives all GPUs, as the reference harness does): give every
 * context the device pointers of all ranks' buffers (nvfp4_ar_local_base); peer access is
 * enabled here. */
NVFP4_API nvfp4_status_t nvfp4_ar_local_base(nvfp4_ar_t h, void** base);
NVFP4_API nvfp4_status_t nvfp4_ar_set_peers(nvfp4_ar_t h, void* const* bases);
/* Registers the buffer NVFP4_AR_NVLS works in: `bytes` bytes that every rank has bound to the same
 * NVLink multicast object (e.g. torch symmetric memory with multicast support); mc_base is its
 * multicast address, uc_base this rank's unicast address of it.  Calls alternate between its two
 * halves, so one call may reduce at most bytes / 4 bf16 elements.  The buffer must outlive the
 * context's last NVLS call; every rank registers one of the same size. */
NVFP4_API nvfp4_status_t nvfp4_ar_set_multicast(nvfp4_ar_t h, void* mc_base, void* uc_base, int64_t bytes);
/* Time limit of each cross-GPU wait (default 5 s); a wait that runs out records a device status
 * (nvfp4_device_status) and the kernel returns. */
NVFP4_API nvfp4_status_t nvfp4_ar_set_timeout(nvfp4_ar_t h, uint64_t timeout_ns);
/* Recovery after a timed-out call: clears this rank's barrier and low-latency words and
 * restarts its epoch count.  Synchronises the device.  Every rank must call it, with no all-reduce of any rank in
 * flight (synchronise all ranks first, e.g. with a host barrier), before the next call. */
NVFP4_API nvfp4_status_t nvfp4_ar_reset(nvfp4_ar_t h);
/* The algorithm NVFP4_AR_AUTO resolves to: LOWLAT up to NVFP4_AR_LOWLAT_MAX_BYTES of bf16, then
 * ONESHOT (always with two ranks, up to NVFP4_AR_ONESHOT_MAX_BYTES with more), then TWOSHOT. */
NVFP4_API int nvfp4_ar_choose_algo(int world, int64_t numel);
/* NVFP4 all-reduce: numel % (32 * world) == 0, 16-byte aligned bf16 buffers on this rank's GPU;
 * in and out may not alias. */
NVFP4_API nvfp4_status_t nvfp4_ar_allreduce(nvfp4_ar_t h, const void* in, void* out, int64_t numel,
                                            float global_scale, int algo, void* stream);
/* bf16 all-reduce: peer-to-peer (ONESHOT / TWOSHOT / AUTO: fp32 sum in rank order, one bf16
 * rounding) or in the switch (NVFP4_AR_NVLS, see above): numel % (8 * world) == 0. */
NVFP4_API nvfp4_status_t nvfp4_ar_bf16_allreduce(nvfp4_ar_t h, const void* in, void* out, int64_t numel, int algo,
                                                 void* stream);
/* The same data path for `world` ranks that all live on ONE GPU (contexts created on it with
 * ranks 0..world-1 and joined with nvfp4_ar_set_peers): each phase is launched for every rank
 * in turn on `stream`, so no kernel waits for another.  bf16_payload != 0 runs the bf16
 * all-reduce.  For testing the arithmetic on a single GPU. */
NVFP4_API nvfp4_status_t nvfp4_ar_allreduce_emulated(nvfp4_ar_t const* handles, int world, const void* const* ins,
                                                     void* const* outs, int64_t numel, float global_scale, int algo,
                                                     int bf16_payload, void* stream);

/* Row-parallel GEMM fused with the NVFP4 two-shot all-reduce (no direct counterpart in the
 * reference; its oneshot_fused_kernel PUSH layout, nvfp4_allreduce.cuh:594-603, is the model).
 * Every rank r computes D_r = bf16(alpha * A_r B_r^T) for its K shard; the GEMM epilogue
 * quantizes each tile with global_scale into the per-owner payloads of the two-shot (in this
 * rank's all-reduce buffer), so the bf16 D_r never reaches memory; the all-reduce kernel then
 * pushes the payloads to their owners, which sum in rank order, requantize and all-gather as in
 * nvfp4_ar_allreduce.  `out` (bf16 M x N) is bit-identical to nvfp4_gemm_bf16 followed by
 * nvfp4_ar_allreduce(..., NVFP4_AR_TWOSHOT) with the same global_scale, on every rank.
 * Requires M % 256 == 0, N % 256 == 0, K % 256 == 0, M * N <= the context's max_numel,
 * M * N / world a multiple of 64.  global_scale bounds |D_r| for every rank (agree on it first). */
NVFP4_API nvfp4_status_t nvfp4_gemm_allreduce(nvfp4_ar_t h, const void* A, const void* sfa, const void* B,
                                              const void* sfb, float alpha, float global_scale, void* out,
                                              int64_t M, int64_t N, int64_t K, void* stream);
/* The same for `world` ranks on ONE GPU (see nvfp4_ar_allreduce_emulated): every rank's GEMM,
 * then the all-reduce phases rank by rank.  A, sfa, B, sfb, alpha and outs are per rank. */
NVFP4_API nvfp4_status_t nvfp4_gemm_allreduce_emulated(nvfp4_ar_t const* handles, int world, const void* const* A,
                                                       const void* const* sfa, const void* const* B,
                                                       const void* const* sfb, const float* alpha,
                                                       float global_scale, void* const* outs, int64_t M, int64_t N,
                                                       int64_t K, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* NVFP4_B200_H */
