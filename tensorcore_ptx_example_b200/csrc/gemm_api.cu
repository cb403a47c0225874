// gemm_api.cu -- C ABI of the NVFP4 GEMM: shape checks and kernel choice.
//   0 < M < 128     : small-M split-K kernel (gemm_small.cu; decode shapes), N % 128 == 0; its
//                     partials are summed inside thread-block clusters when the splits of an
//                     n-tile fit one (no workspace), else through a workspace and a second kernel
//   M % 128 == 0    : CTA-pair kernel (gemm_2sm.cu, tcgen05 cta_group::2, 256x256 pair tiles; with
//                     M % 256 == 128 the last pair's second CTA covers zero-filled rows)
#include <cmath>
#include <cstdint>
#include <mutex>

#include "capi_internal.h"

namespace nvfp4 {
namespace gemm {

static bool small_m(int64_t M) { return M > 0 && M < 128; }

static nvfp4_status_t check_args(const void* A, const void* sfa, const void* B, const void* sfb, const void* D,
                                 int64_t M, int64_t N, int64_t K) {
    if (!A || !sfa || !B || !sfb || !D) return fail(NVFP4_ERR_INVALID_ARG, "gemm: null pointer");
    if (M <= 0 || N <= 0 || K <= 0 || K % 256 || (small_m(M) ? N % 128 : (M % 128 || N % 256)))
        return fail(NVFP4_ERR_INVALID_ARG,
                    "gemm: need K %% 256 == 0 and either M < 128 with N %% 128 == 0, or M %% 128 == 0 with "
                    "N %% 256 == 0 (got %lld %lld %lld)",
                    (long long)M, (long long)N, (long long)K);
    if (M > (1ll << 30) || N > (1ll << 30) || K > (1ll << 30)) return fail(NVFP4_ERR_INVALID_ARG, "gemm: dimension too large");
    if (!aligned16(A) || !aligned16(B) || !aligned16(sfa) || !aligned16(sfb) || !aligned16(D))
        return fail(NVFP4_ERR_INVALID_ARG, "gemm: buffers must be 16-byte aligned");
    return NVFP4_OK;
}

// Split-K workspace of the small-M path when the caller gives none: one buffer per device,
// allocated on first use and grown when a larger one is needed (cudaFree synchronises the device,
// so a buffer still in use by an earlier launch is never released under it).
static nvfp4_status_t internal_workspace(size_t need, void** out) {
    static std::mutex mu;
    static void* buf[64] = {};
    static size_t size[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return fail(NVFP4_ERR_UNSUPPORTED, "gemm: device ordinal %d", dev);
    std::lock_guard<std::mutex> g(mu);
    if (size[dev] < need) {
        if (buf[dev]) cudaFree(buf[dev]);
        buf[dev] = nullptr;
        size[dev] = 0;
        cudaError_t e = cudaMalloc(&buf[dev], need);
        if (e != cudaSuccess) {
            buf[dev] = nullptr;
            return fail(NVFP4_ERR_CUDA, "gemm: workspace of %zu bytes: %s", need, cudaGetErrorString(e));
        }
        size[dev] = need;
    }
    *out = buf[dev];
    return NVFP4_OK;
}

template <bool kOutF32>
static nvfp4_status_t dispatch(const void* A, const void* sfa, const void* B, const void* sfb, float alpha, void* D,
                               int64_t M, int64_t N, int64_t K, void* ws, size_t ws_bytes, cudaStream_t s,
                               int flags = 0) {
    nvfp4_status_t st = check_args(A, sfa, B, sfb, D, M, N, K);
    if (st != NVFP4_OK) return st;
    if (small_m(M)) {
        if (!ws) {
            ws_bytes = gsmall::workspace_bytes(M, N, K);
            if (ws_bytes && (st = internal_workspace(ws_bytes, &ws))) return st;
        } else if (!aligned16(ws)) {
            return fail(NVFP4_ERR_INVALID_ARG, "gemm: workspace must be 16-byte aligned");
        }
        return gsmall::launch<kOutF32>(A, sfa, B, sfb, alpha, D, M, N, K, ws, ws_bytes, s,
                                       (flags & NVFP4_GEMM_WEIGHTS_CONST) != 0);
    }
    return gemm2::launch<kOutF32 ? gemm2::OUT_F32 : gemm2::OUT_BF16>(A, sfa, B, sfb, alpha, D, M, N, K, s);
}

}  // namespace gemm
}  // namespace nvfp4

using namespace nvfp4;

extern "C" {

nvfp4_status_t nvfp4_gemm_bf16(const void* A, const void* sfa, const void* B, const void* sfb, float alpha, void* D,
                               int64_t M, int64_t N, int64_t K, void* stream) {
    clear_error();
    return gemm::dispatch<false>(A, sfa, B, sfb, alpha, D, M, N, K, nullptr, 0, (cudaStream_t)stream);
}

nvfp4_status_t nvfp4_gemm_bf16_flags(const void* A, const void* sfa, const void* B, const void* sfb, float alpha,
                                     void* D, int64_t M, int64_t N, int64_t K, int flags, void* stream) {
    clear_error();
    if (flags & ~NVFP4_GEMM_WEIGHTS_CONST) return fail(NVFP4_ERR_INVALID_ARG, "gemm_flags: unknown flag bits");
    return gemm::dispatch<false>(A, sfa, B, sfb, alpha, D, M, N, K, nullptr, 0, (cudaStream_t)stream, flags);
}

size_t nvfp4_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K) {
    return (M > 0 && M < 128) ? gsmall::workspace_bytes(M, N, K) : 0;
}

nvfp4_status_t nvfp4_gemm_bf16_ws(const void* A, const void* sfa, const void* B, const void* sfb, float alpha, void* D,
                                  int64_t M, int64_t N, int64_t K, void* workspace, size_t workspace_bytes,
                                  void* stream) {
    clear_error();
    if (M > 0 && M < 128 && !workspace && gsmall::workspace_bytes(M, N, K) > 0)
        return fail(NVFP4_ERR_INVALID_ARG, "gemm_ws: null workspace (this shape needs %zu bytes)",
                    gsmall::workspace_bytes(M, N, K));
    return gemm::dispatch<false>(A, sfa, B, sfb, alpha, D, M, N, K, workspace, workspace_bytes, (cudaStream_t)stream);
}

nvfp4_status_t nvfp4_gemm_quantize(const void* A, const void* sfa, const void* B, const void* sfb, float alpha,
                                   float gs_out, void* D_packed, void* D_sf, int64_t M, int64_t N, int64_t K,
                                   void* stream) {
    clear_error();
    if (!A || !sfa || !B || !sfb || !D_packed || !D_sf) return fail(NVFP4_ERR_INVALID_ARG, "gemm_quantize: null pointer");
    if (M == 0 || N == 0) return NVFP4_OK;
    if (M < 0 || N < 0 || K <= 0 || M % 256 || N % 256 || K % 256)
        return fail(NVFP4_ERR_INVALID_ARG, "gemm_quantize: need M %% 256 == 0, N %% 256 == 0, K %% 256 == 0 (got %lld %lld %lld)",
                    (long long)M, (long long)N, (long long)K);
    if (!(gs_out > 0.0f) || !std::isfinite(gs_out))
        return fail(NVFP4_ERR_INVALID_ARG, "gemm_quantize: global scale must be finite and > 0");
    if (((uintptr_t)D_packed & 31) || ((uintptr_t)D_sf & 3) || !aligned16(A) || !aligned16(B) || !aligned16(sfa) ||
        !aligned16(sfb))
        return fail(NVFP4_ERR_INVALID_ARG, "gemm_quantize: D_packed must be 32-byte aligned, operands 16-byte aligned");
    gemm2::EpiOut q{};
    q.packed = reinterpret_cast<uint8_t*>(D_packed);
    q.sf = reinterpret_cast<uint8_t*>(D_sf);
    q.gs_inv = 1.0f / gs_out;
    return gemm2::launch<gemm2::OUT_NVFP4>(A, sfa, B, sfb, alpha, nullptr, M, N, K, (cudaStream_t)stream, q);
}

nvfp4_status_t nvfp4_gemm_f32(const void* A, const void* sfa, const void* B, const void* sfb, float* D, int64_t M,
                              int64_t N, int64_t K, void* stream) {
    clear_error();
    return gemm::dispatch<true>(A, sfa, B, sfb, 1.0f, D, M, N, K, nullptr, 0, (cudaStream_t)stream);
}

}  // extern "C"
