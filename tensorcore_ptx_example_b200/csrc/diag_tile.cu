// diag_tile.cu -- one M128 N256 K256 NVFP4 block-scaled MMA tile, computed independently of the
// production GEMM (diagnostics library).  It pins the arithmetic of tcgen05.mma
// kind::mxf4nvf4.block_scale.scale_vec::4X for the CPU model of the tests: nothing here shares a
// data path with gemm2_kernel / gemm_small_kernel:
//   - operands: plain 16-byte global loads into shared memory in the no-swizzle K-major
//     core-matrix layout (8 rows x 16 bytes per core matrix; K-adjacent core matrices 128 bytes
//     apart, 8-row groups 256 bytes apart), the layout of the reference's single-tile tests
//     (blackwell/tcgen05_fp4_sm100/tcgen05_nvfp4_block16_ue4m3_maxtile_m128n256.cu:98-144,
//     LAYOUT.md:90-148) -- the production kernels use TMA with 128-byte swizzle;
//   - scales: one tcgen05.cp 32x128b.warpx4 per 512-byte scale atom -- the production kernels
//     store them with tcgen05.st from scale warps;
//   - one CTA (cta_group::1, M = 128) issuing four K64 MMAs into one accumulator -- the
//     production kernels run CTA pairs (M = 256) or swapped operands;
//   - accumulator read back with tcgen05.ld 32x32b and stored as fp32 without scaling.
#include "capi_internal.h"
#include "gemm.cu"
#include "nvfp4_common.cuh"
#include "nvfp4_diag.h"

namespace nvfp4 {
namespace diag {

constexpr int TILE_THREADS = 128;
constexpr int TILE_STEPS = 4;                          // K = 256 in four K64 MMAs
constexpr int TILE_A_STEP = 128 * 32;                  // one K step of A: 128 rows x 32 bytes
constexpr int TILE_B_STEP = 256 * 32;                  // one K step of B: 256 rows x 32 bytes
constexpr int TILE_OFF_A = 0;
constexpr int TILE_OFF_B = TILE_OFF_A + TILE_STEPS * TILE_A_STEP;
constexpr int TILE_OFF_SFA = TILE_OFF_B + TILE_STEPS * TILE_B_STEP;   // 4 atoms (rows 0-127)
constexpr int TILE_OFF_SFB = TILE_OFF_SFA + 4 * 512;                  // 8 atoms (2 row groups x 4)
constexpr int TILE_SMEM_USED = TILE_OFF_SFB + 8 * 512;
constexpr int TILE_SMEM = TILE_SMEM_USED + 128;                       // + alignment slack
constexpr uint32_t TILE_IDESC = (1u << 7) | (1u << 10) | ((256u >> 3) << 17) | ((128u >> 4) << 24);
constexpr int TILE_SF_COL = 256;                       // scale columns after the 256-column accumulator

// Offset of byte `kb` (0..31) of row `r` inside one K step of the no-swizzle K-major layout.
__device__ __forceinline__ int core_offset(int r, int kb) { return (r >> 3) * 256 + (kb >> 4) * 128 + (r & 7) * 16; }

// No-swizzle K-major shared-memory descriptor: LBO 128 bytes (K direction), SBO 256 bytes
// (8-row groups), version 1, swizzle mode 0.
__device__ __forceinline__ uint64_t desc_interleaved(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(256 >> 4) << 32) |
           (1ull << 46);
}

__global__ void __launch_bounds__(TILE_THREADS, 1)
mma_tile_kernel(const uint8_t* __restrict__ A, const uint8_t* __restrict__ sfa, const uint8_t* __restrict__ B,
                const uint8_t* __restrict__ sfb, float* __restrict__ D) {
    extern __shared__ uint8_t tile_raw[];
    __shared__ __align__(8) uint64_t done_bar;
    __shared__ uint32_t tmem_slot;
    const uint32_t raw = smem_u32(tile_raw);
    uint8_t* sm = tile_raw + (((raw + 127u) & ~127u) - raw);
    const uint32_t sbase = smem_u32(sm);
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;

    // operands: 16-byte chunks; chunk c16 (0..7) of a 128-byte row is K step c16 / 2, half c16 % 2
    for (int i = t; i < 128 * 8; i += TILE_THREADS) {
        const int r = i >> 3, c16 = i & 7;
        *reinterpret_cast<uint4*>(sm + TILE_OFF_A + (c16 >> 1) * TILE_A_STEP + core_offset(r, (c16 & 1) * 16)) =
            *reinterpret_cast<const uint4*>(A + r * 128 + c16 * 16);
    }
    for (int i = t; i < 256 * 8; i += TILE_THREADS) {
        const int r = i >> 3, c16 = i & 7;
        *reinterpret_cast<uint4*>(sm + TILE_OFF_B + (c16 >> 1) * TILE_B_STEP + core_offset(r, (c16 & 1) * 16)) =
            *reinterpret_cast<const uint4*>(B + r * 128 + c16 * 16);
    }
    // scale atoms as stored by the quantizer: A atom j = K step j; B atom g * 4 + j = rows
    // 128 g .. 128 g + 127 of K step j
    for (int i = t; i < 4 * 32; i += TILE_THREADS)
        *reinterpret_cast<uint4*>(sm + TILE_OFF_SFA + 16 * i) = *reinterpret_cast<const uint4*>(sfa + 16 * i);
    for (int i = t; i < 8 * 32; i += TILE_THREADS)
        *reinterpret_cast<uint4*>(sm + TILE_OFF_SFB + 16 * i) = *reinterpret_cast<const uint4*>(sfb + 16 * i);
    if (t == 0) {
        mbar_init(smem_u32(&done_bar), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // the MMA and tcgen05.cp read shared memory through the async proxy
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&tmem_slot)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    if (t == 0) {
        auto sfdesc = [](uint32_t s) { return (uint64_t)((s >> 4) & 0x3FFFu) | ((uint64_t)(128 >> 4) << 32) | (1ull << 46); };
        for (int j = 0; j < TILE_STEPS; j++) {
            const uint32_t col = tmem + TILE_SF_COL + 12 * j;
            asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(col),
                         "l"(sfdesc(sbase + TILE_OFF_SFA + 512 * j)));
            asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(col + 4),
                         "l"(sfdesc(sbase + TILE_OFF_SFB + 512 * j)));
            asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(col + 8),
                         "l"(sfdesc(sbase + TILE_OFF_SFB + 512 * (4 + j))));
        }
        for (int j = 0; j < TILE_STEPS; j++) {
            const uint64_t ad = desc_interleaved(sbase + TILE_OFF_A + j * TILE_A_STEP);
            const uint64_t bd = desc_interleaved(sbase + TILE_OFF_B + j * TILE_B_STEP);
            const uint32_t col = tmem + TILE_SF_COL + 12 * j;
            asm volatile(
                "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(tmem),
                "l"(ad), "l"(bd), "r"(TILE_IDESC), "r"((uint32_t)j), "r"(col), "r"(col + 4)
                : "memory");
        }
        tc_commit(smem_u32(&done_bar));
    }
    __syncwarp();
    // every thread waits for the MMAs (bounded); a run-out records an error and skips the read
    const bool ok = mbar_wait(smem_u32(&done_bar), 0, 2000000000ull, DEV_TIMEOUT_GEMM_MMA);
    tc_fence_after();
    if (__all_sync(0xFFFFFFFFu, ok)) {
        const int row = warp * 32 + lane;
#pragma unroll 1
        for (int c = 0; c < 256; c += 32) {
            uint32_t r[32];
            gemm::tc_ld32(tmem + ((uint32_t)(warp * 32) << 16) + c, r);
            gemm::tc_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; i += 4)
                *reinterpret_cast<uint4*>(D + row * 256 + c + i) = make_uint4(r[i], r[i + 1], r[i + 2], r[i + 3]);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
}

}  // namespace diag
}  // namespace nvfp4

using namespace nvfp4;

extern "C" {

nvfp4_status_t nvfp4_diag_mma_tile(const void* A, const void* sfa, const void* B, const void* sfb, float* D,
                                   void* stream) {
    clear_error();
    if (!A || !sfa || !B || !sfb || !D) return fail(NVFP4_ERR_INVALID_ARG, "diag_mma_tile: null pointer");
    if (!aligned16(A) || !aligned16(sfa) || !aligned16(B) || !aligned16(sfb) || !aligned16(D))
        return fail(NVFP4_ERR_INVALID_ARG, "diag_mma_tile: buffers must be 16-byte aligned");
    cudaError_t e = cudaFuncSetAttribute(diag::mma_tile_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         diag::TILE_SMEM);
    if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "diag_mma_tile: %s", cudaGetErrorString(e));
    diag::mma_tile_kernel<<<1, diag::TILE_THREADS, diag::TILE_SMEM, (cudaStream_t)stream>>>(
        reinterpret_cast<const uint8_t*>(A), reinterpret_cast<const uint8_t*>(sfa), reinterpret_cast<const uint8_t*>(B),
        reinterpret_cast<const uint8_t*>(sfb), D);
    return check_launch("mma_tile_kernel");
}

}  // extern "C"
