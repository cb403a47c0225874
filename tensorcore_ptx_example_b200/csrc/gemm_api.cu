// gemm_api.cu -- C ABI of the NVFP4 GEMM: shape checks and kernel choice.
//   M % 256 == 0: CTA-pair kernel (gemm_2sm.cu, tcgen05 cta_group::2, 256x256 pair tiles)
//   otherwise   : single-CTA kernel (gemm.cu, 128x256 tiles)
#include "capi_internal.h"

namespace nvfp4 {
namespace gemm {

static nvfp4_status_t check_args(const void* A, const void* sfa, const void* B, const void* sfb, const void* D,
                                 int64_t M, int64_t N, int64_t K) {
    if (!A || !sfa || !B || !sfb || !D) return fail(NVFP4_ERR_INVALID_ARG, "gemm: null pointer");
    if (M <= 0 || N <= 0 || K <= 0 || M % 128 || N % 256 || K % 256)
        return fail(NVFP4_ERR_INVALID_ARG, "gemm: need M %% 128 == 0, N %% 256 == 0, K %% 256 == 0 (got %lld %lld %lld)",
                    (long long)M, (long long)N, (long long)K);
    if (M > (1ll << 30) || N > (1ll << 30) || K > (1ll << 30)) return fail(NVFP4_ERR_INVALID_ARG, "gemm: dimension too large");
    if (!aligned16(A) || !aligned16(B) || !aligned16(sfa) || !aligned16(sfb) || !aligned16(D))
        return fail(NVFP4_ERR_INVALID_ARG, "gemm: buffers must be 16-byte aligned");
    return NVFP4_OK;
}

template <bool kOutF32>
static nvfp4_status_t dispatch(const void* A, const void* sfa, const void* B, const void* sfb, float alpha, void* D,
                               int64_t M, int64_t N, int64_t K, cudaStream_t s) {
    nvfp4_status_t st = check_args(A, sfa, B, sfb, D, M, N, K);
    if (st != NVFP4_OK) return st;
    if (M % 256 == 0) return gemm2::launch<kOutF32>(A, sfa, B, sfb, alpha, D, M, N, K, s);
    return launch<kOutF32>(A, sfa, B, sfb, alpha, D, M, N, K, s);
}

}  // namespace gemm
}  // namespace nvfp4

using namespace nvfp4;

extern "C" {

nvfp4_status_t nvfp4_gemm_bf16(const void* A, const void* sfa, const void* B, const void* sfb, float alpha, void* D,
                               int64_t M, int64_t N, int64_t K, void* stream) {
    clear_error();
    return gemm::dispatch<false>(A, sfa, B, sfb, alpha, D, M, N, K, (cudaStream_t)stream);
}

nvfp4_status_t nvfp4_gemm_f32(const void* A, const void* sfa, const void* B, const void* sfb, float* D, int64_t M,
                              int64_t N, int64_t K, void* stream) {
    clear_error();
    return gemm::dispatch<true>(A, sfa, B, sfb, 1.0f, D, M, N, K, (cudaStream_t)stream);
}

}  // extern "C"
