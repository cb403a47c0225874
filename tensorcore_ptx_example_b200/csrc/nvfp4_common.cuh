// nvfp4_common.cuh -- device helpers shared by the NVFP4 kernels (sm_100a only).
//
// * NVFP4 codec: E2M1 / UE4M3 conversions through the hardware cvt instructions, and the
//   per-16-element block quantizer q16 with IEEE division (the reference's q16,
//   blackwell/allreduce_sm100_sm120/nvfp4_allreduce.cuh:272-290, uses rcp.approx.ftz;
//   here every reciprocal is a correctly rounded division so that a CPU reproduces the
//   result bit for bit).
// * Bounded waits: every spin in this library gives up after a time limit, records an
//   error code in a device-global status word and returns false.  Nothing traps.
// * Thin PTX wrappers for mbarrier, TMA and tcgen05.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "this library targets sm_100a only"
#endif

namespace nvfp4 {

// ------------------------------------------------------------ status word ----
// Device-global status of the library on this device (0 = OK).  Kernels write the first
// error they detect; the host reads and clears it with nvfp4_device_status().  The library
// is one translation unit (nvfp4_lib.cu), so this definition exists once per module.
__device__ unsigned int g_status = 0;

enum DeviceError : unsigned int {
    DEV_OK = 0,
    DEV_TIMEOUT_GEMM_PRODUCER = 0x101,
    DEV_TIMEOUT_GEMM_MMA = 0x102,
    DEV_TIMEOUT_GEMM_EPILOGUE = 0x103,
    DEV_TIMEOUT_GEMM_TEARDOWN = 0x104,
    DEV_TIMEOUT_GEMM_SF = 0x106,
    DEV_TMEM_BASE = 0x105,
    DEV_TIMEOUT_QUANT = 0x301,
    DEV_NONFINITE_INPUT = 0x302,      // a quantized block or an amax input held NaN or Inf
    DEV_TIMEOUT_AR_BARRIER = 0x201,
};

__device__ __forceinline__ void record_error(unsigned int code) {
    atomicCAS(&g_status, 0u, code);
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ------------------------------------------------------------------ codec ----
// Eight floats -> eight E2M1 nibbles, element i in bits [4i, 4i+4).  Hardware RNE with
// saturation to +-6; cvt packs its first source operand into the high nibble.
__device__ __forceinline__ uint32_t e2m1x8(const float* v) {
    uint32_t out;
    asm("{\n\t.reg .b8 q0, q1, q2, q3;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 q0, %2, %1;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 q1, %4, %3;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 q2, %6, %5;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 q3, %8, %7;\n\t"
        "mov.b32 %0, {q0, q1, q2, q3};\n\t}"
        : "=r"(out)
        : "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]));
    return out;
}

// One float -> E4M3 byte (RNE, saturating to +-448).
__device__ __forceinline__ uint32_t e4m3_encode(float x) {
    uint16_t pair;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(pair) : "f"(0.0f), "f"(x));
    return pair & 0xFFu;
}

// E4M3 byte -> float (exact).
__device__ __forceinline__ float e4m3_decode(uint32_t code) {
    uint32_t h2;
    const uint16_t in = (uint16_t)(code & 0xFFu);
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(in));
    return __half2float(__ushort_as_half((unsigned short)(h2 & 0xFFFFu)));
}

// Four E2M1 bytes (8 nibbles) -> 8 floats, nibble i -> out[i] (exact).
__device__ __forceinline__ void e2m1x8_decode(uint32_t w, float* out) {
    uint32_t h0, h1, h2, h3;
    asm("{\n\t.reg .b8 q0, q1, q2, q3;\n\t"
        "mov.b32 {q0, q1, q2, q3}, %4;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, q0;\n\t"
        "cvt.rn.f16x2.e2m1x2 %1, q1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %2, q2;\n\t"
        "cvt.rn.f16x2.e2m1x2 %3, q3;\n\t}"
        : "=r"(h0), "=r"(h1), "=r"(h2), "=r"(h3)
        : "r"(w));
    const uint32_t hs[4] = {h0, h1, h2, h3};
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hs[i]));
        out[2 * i] = f.x;
        out[2 * i + 1] = f.y;
    }
}

// Global scale pair from a tensor amax: gs = amax / (6 * 448), gs_inv = 1 / gs.
__device__ __forceinline__ void global_scale_from_amax(float amax, float& gs, float& gs_inv) {
    float g = (amax > 0.0f) ? __fdiv_rn(amax, 2688.0f) : 1.0f;
    if (g == 0.0f) g = 1.0f;
    gs = g;
    gs_inv = __fdiv_rn(1.0f, g);
}

// Block scale of one 16-element block from its amax:
//   s = (amax * RCP6) * gs_inv, stored as E4M3; inv = gs_inv * rcp(decode(stored)) (0 when the
//   stored scale is 0).  RCP6 is 1/6 rounded to fp32 and rcp is the correctly rounded
//   reciprocal, so every step is one IEEE operation a CPU reproduces bit for bit (the
//   reference, nvfp4_allreduce.cuh:272-290, uses rcp.approx.ftz for both reciprocals).
//   Returns the scale byte, writes inv.
constexpr uint32_t RCP6_BITS = 0x3E2AAAABu;    // fp32(1/6), round to nearest
__device__ __forceinline__ uint32_t block_scale(float amax, float gs_inv, float& inv) {
    const float t = __fmul_rn(amax, __uint_as_float(RCP6_BITS));
    const float s = __fmul_rn(t, gs_inv);
    const uint32_t code = e4m3_encode(s);
    const float sq = e4m3_decode(code);
    inv = (sq != 0.0f) ? __fmul_rn(gs_inv, __frcp_rn(sq)) : 0.0f;
    return code;
}

// (a * s, b * s), each rounded to nearest: one packed f32x2 multiply (sm_100).
__device__ __forceinline__ void mul2_rn(float a, float b, float s, float& ya, float& yb) {
    asm("{\n\t.reg .b64 x, y, z;\n\t"
        "mov.b64 x, {%2, %3};\n\t"
        "mov.b64 y, {%4, %4};\n\t"
        "mul.rn.f32x2 z, x, y;\n\t"
        "mov.b64 {%0, %1}, z;\n\t}"
        : "=f"(ya), "=f"(yb)
        : "f"(a), "f"(b), "f"(s));
}

// Scale byte of a block that holds a NaN or an Inf: the E4M3 NaN encoding, so the whole block
// dequantizes to NaN (NVFP4 has no encoding for non-finite values); its codes are 0.
constexpr uint32_t NONFINITE_SCALE = 0x7Fu;

// Quantize 16 floats: writes two 32-bit nibble words, returns the scale byte.  A block with a
// non-finite value gets NONFINITE_SCALE and zero codes, and records DEV_NONFINITE_INPUT.
__device__ __forceinline__ uint32_t q16(const float* v, float gs_inv, uint32_t& w0, uint32_t& w1) {
    // block amax with three-input max.NaN.abs: NaN propagates, so one compare finds NaN or Inf
    float m[6];
#pragma unroll
    for (int i = 0; i < 5; i++) asm("max.NaN.abs.f32 %0, %1, %2, %3;" : "=f"(m[i]) : "f"(v[3 * i]), "f"(v[3 * i + 1]), "f"(v[3 * i + 2]));
    m[5] = fabsf(v[15]);
    float amax, a2;
    asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(amax) : "f"(m[0]), "f"(m[1]), "f"(m[2]));
    asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(a2) : "f"(m[3]), "f"(m[4]), "f"(m[5]));
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(amax) : "f"(amax), "f"(a2));
    if (!(amax <= 3.402823466e38f)) {
        record_error(DEV_NONFINITE_INPUT);
        w0 = 0u;
        w1 = 0u;
        return NONFINITE_SCALE;
    }
    float inv;
    const uint32_t code = block_scale(amax, gs_inv, inv);
    float y[16];
#pragma unroll
    for (int i = 0; i < 8; i++) mul2_rn(v[2 * i], v[2 * i + 1], inv, y[2 * i], y[2 * i + 1]);
    w0 = e2m1x8(y);
    w1 = e2m1x8(y + 8);
    if (inv == 0.0f) { w0 = 0u; w1 = 0u; }
    return code;
}

// The same for 16 bf16 values packed two per word (element 2i in the low half of word i).
// The amax: max.NaN.xorsign.abs.bf16x2 keeps per lane the larger magnitude of two bf16 pairs
// (its sign is the xor of the signs, cleared afterwards) and propagates NaN, one instruction per
// word; for finite values that is exactly max |x| of each half, and a NaN or Inf anywhere in the
// block leaves a magnitude of at least 0x7F80 (the non-finite path above).
__device__ __forceinline__ uint32_t q16_bf16(const uint32_t* w, float gs_inv, uint32_t& w0, uint32_t& w1) {
    uint32_t m = w[0];
#pragma unroll
    for (int i = 1; i < 8; i++) asm("max.NaN.xorsign.abs.bf16x2 %0, %0, %1;" : "+r"(m) : "r"(w[i]));
    m &= 0x7FFF7FFFu;
    const uint32_t abits = (m >> 16) > (m & 0xFFFFu) ? (m >> 16) : (m & 0xFFFFu);
    if (abits >= 0x7F80u) {
        record_error(DEV_NONFINITE_INPUT);
        w0 = 0u;
        w1 = 0u;
        return NONFINITE_SCALE;
    }
    const float amax = __uint_as_float(abits << 16);
    float inv;
    const uint32_t code = block_scale(amax, gs_inv, inv);
    float y[16];
#pragma unroll
    for (int i = 0; i < 8; i++)
        mul2_rn(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xFFFF0000u), inv, y[2 * i], y[2 * i + 1]);
    w0 = e2m1x8(y);
    w1 = e2m1x8(y + 8);
    if (inv == 0.0f) { w0 = 0u; w1 = 0u; }
    return code;
}

// ------------------------------------------------------------- PTX basics ----
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// 32-byte load (sm_100 256-bit vector load); p must be 32-byte aligned.
__device__ __forceinline__ void ld_nc_v8(const void* p, uint32_t* r) {
    asm volatile("ld.global.nc.L1::no_allocate.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "l"(p));
}

__device__ __forceinline__ void st_v4(void* p, uint4 v) {
    asm volatile("st.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
}

// 32-byte global store (sm_100: .v8 of 32-bit elements); p must be 32-byte aligned.
__device__ __forceinline__ void st_global_v8(void* p, const uint32_t* v) {
    asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(v[0]), "r"(v[1]),
                 "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}

// --------------------------------------------------------------- mbarrier ----
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for the phase with the given parity to complete; false after `limit_ns`.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint64_t limit_ns,
                                          unsigned int err) {
#pragma unroll 1
    for (int i = 0; i < 256; i++)
        if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > limit_ns) {
            record_error(err);
            return false;
        }
    }
}

// Non-blocking probe of a phase (mbarrier.test_wait never suspends the thread).
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// mbar_wait for a thread that issues tcgen05.mma: polls with test_wait.  On B200 a try_wait in
// the MMA-issuing thread costs ~240 cycles of tensor-pipe time per call even when the phase has
// long completed, a test_wait ~110 (measured with 4 MMAs per wait).
__device__ __forceinline__ bool mbar_wait_spin(uint32_t bar, uint32_t parity, uint64_t limit_ns,
                                               unsigned int err) {
#pragma unroll 1
    for (int i = 0; i < 4096; i++)
        if (mbar_test_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
    while (true) {
#pragma unroll 1
        for (int i = 0; i < 64; i++)
            if (mbar_test_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > limit_ns) {
            record_error(err);
            return false;
        }
    }
}

// -------------------------------------------------------------------- TMA ----
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, int32_t x, int32_t y,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(tmap), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

// 2D TMA store from this CTA's shared memory (bulk-group completion).
__device__ __forceinline__ void tma_store_2d(const void* tmap, uint32_t src, int32_t x, int32_t y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tmap), "r"(src),
                 "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N committed bulk groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read_n() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ---------------------------------------------------------------- tcgen05 ----
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Commit all prior tcgen05 async operations of this thread to an mbarrier (one arrival).
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

}  // namespace nvfp4
