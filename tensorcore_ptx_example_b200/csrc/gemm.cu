// gemm.cu -- tcgen05 helpers shared by the NVFP4 GEMM kernels (gemm_2sm.cu: CTA-pair tiles for
// M % 128 == 0; gemm_small.cu: split-K decode shapes, M < 128).
//
// TMEM scale-factor layout used by both: lane = row % 32 (replicated in the four lane quadrants),
// column = row / 32, byte = 16-block index within the 64-wide K step -- what tcgen05.cp
// 32x128b.warpx4 would produce from one 512-byte atom of the tcgen05 SF layout; the kernels write
// it with tcgen05.st from their scale warps instead.
#include "capi_internal.h"
#include "nvfp4_common.cuh"

namespace nvfp4 {
namespace gemm {

// Shared-memory matrix descriptor, K-major, SWIZZLE_128B: rows of 128 bytes, 8-row groups
// 1024 bytes apart (SBO), version 1.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}

// 32 lanes x 32 columns of 32-bit accumulators; thread i receives row (quadrant base + i).
__device__ __forceinline__ void tc_ld32(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
        "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
        "%30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

}  // namespace gemm
}  // namespace nvfp4
