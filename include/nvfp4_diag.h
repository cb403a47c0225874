/*
 * nvfp4_diag.h -- C ABI of the diagnostics library (libnvfp4_diag.so), built beside the product
 * library libnvfp4_b200.so from the same sources tree but shipped separately: nothing here is on
 * the data path.  The parity tests use these probes to pin hardware arithmetic (the E2M1 / E4M3
 * conversions, the approximate reciprocal that the reference's quantizer uses, and one block-
 * scaled tcgen05 MMA tile computed independently of the production GEMM) and the benchmark uses
 * the MMA issue-rate probe as the measured FP4 roofline.
 *
 * Reference interfaces these probes stand beside (paths inside YijiaZhao/tensorcore_ptx_example):
 *   - blackwell/allreduce_sm100_sm120/nvfp4_allreduce.cuh:110-114   recip_ftz -> nvfp4_diag_rcp_approx
 *   - blackwell/allreduce_sm100_sm120/nvfp4_allreduce.cuh:194-222,278  encode8_e2m1 / __nv_fp8_e4m3
 *                                                    -> nvfp4_diag_e2m1_encode / nvfp4_diag_e4m3_encode
 *   - blackwell/tcgen05_fp4_sm100/tcgen05_nvfp4_block16_ue4m3_maxtile_m128n256.cu:98-144 (one
 *     M128 N256 block-scaled MMA tile read back with tcgen05.ld)      -> nvfp4_diag_mma_tile
 *
 * Conventions as in nvfp4.h: device pointers, asynchronous on `stream`, status codes
 * NVFP4_OK / NVFP4_ERR_* (0 = OK); nvfp4_diag_last_error_string() describes the calling thread's
 * last failure of this library.
 */
#ifndef NVFP4_DIAG_H
#define NVFP4_DIAG_H

#include <stddef.h>
#include <stdint.h>

#include "nvfp4.h"

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define NVFP4_DIAG_API __attribute__((visibility("default")))
#else
#define NVFP4_DIAG_API
#endif

NVFP4_DIAG_API const char* nvfp4_diag_last_error_string(void);
/* Device status word of this library on the current device (see nvfp4_device_status). */
NVFP4_DIAG_API nvfp4_status_t nvfp4_diag_device_status(unsigned int* status_out, int clear);

/* out[i] = E2M1 code of x[i] (cvt.rn.satfinite, round to nearest even, saturate to +-6). */
NVFP4_DIAG_API nvfp4_status_t nvfp4_diag_e2m1_encode(const float* x, uint8_t* out, int64_t n, void* stream);
/* out[i] = E4M3 code of x[i] (cvt.rn.satfinite, saturate to +-448). */
NVFP4_DIAG_API nvfp4_status_t nvfp4_diag_e4m3_encode(const float* x, uint8_t* out, int64_t n, void* stream);
/* out[i] = rcp.approx.ftz.f32(x[i]): the approximate reciprocal of the reference's recip_ftz. */
NVFP4_DIAG_API nvfp4_status_t nvfp4_diag_rcp_approx(const float* x, float* out, int64_t n, void* stream);

/* One M128 N256 K256 block-scaled tile on one CTA (tcgen05.mma.cta_group::1
 * .kind::mxf4nvf4.block_scale.scale_vec::4X, four K64 MMAs into one TMEM accumulator), written
 * independently of the production GEMM: operands copied into shared memory with plain loads in
 * the no-swizzle K-major core-matrix layout, scales placed in TMEM with tcgen05.cp, the fp32
 * accumulator read back with tcgen05.ld.  A: packed [128][128] bytes, sfa: nvfp4_sf_bytes(128,
 * 256) bytes; B: packed [256][128] bytes, sfb: nvfp4_sf_bytes(256, 256) bytes (tcgen05 layout);
 * D: fp32 [128][256].  All 16-byte aligned. */
NVFP4_DIAG_API nvfp4_status_t nvfp4_diag_mma_tile(const void* A, const void* sfa, const void* B, const void* sfb,
                                                  float* D, void* stream);

/* FP4 tensor-core issue-rate microbenchmark: every SM (cta_group 1, M128 N256) or SM pair
 * (cta_group 2, M256 N256) issues `iters` K64 block-scaled MMAs from resident shared memory,
 * on sparse constant operands or (random_operands != 0) pseudo-random E2M1 codes.
 * FLOPs = 2 * 128 * 256 * 64 * iters * (number of SMs); time it with events around the call.
 * The measured rate is the roofline denominator of nvfp4_gemm_bf16. */
NVFP4_DIAG_API nvfp4_status_t nvfp4_diag_mma_peak(int cta_group, int iters, int random_operands, void* stream);
/* Effective SM clock (MHz: SM cycles / elapsed ns, summed over CTAs) of the nvfp4_diag_mma_peak
 * launches since the previous call (synchronises the device; resets the counters). */
NVFP4_DIAG_API nvfp4_status_t nvfp4_diag_mma_peak_clock(double* mhz);

#ifdef __cplusplus
}
#endif
#endif /* NVFP4_DIAG_H */
