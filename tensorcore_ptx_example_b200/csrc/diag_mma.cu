// diag_mma.cu -- FP4 tensor-core issue-rate microbenchmark (the measured roofline of the GEMM).
// Part of the diagnostics library (diag_lib.cu -> libnvfp4_diag.so), not of the product library.
//
// Every CTA (or CTA pair) issues `iters` block-scaled MMAs back to back on operands that stay
// in shared memory and TMEM (no global traffic), committing every 32 MMAs and keeping at most
// two such groups in flight.  FLOPs = 2 * M * N * 64 * iters per CTA (pair).  The host times
// the launch with events; the rate is the ceiling a GEMM on this part can reach at the clock
// the run sees.
#include "capi_internal.h"
#include "nvfp4_common.cuh"
#include "nvfp4_diag.h"

namespace nvfp4 {
namespace diag {

constexpr int MMA_GROUP = 32;

// Effective SM clock of the launches since the last read: per CTA, thread 0 adds the SM cycles
// (clock64) and nanoseconds (globaltimer) between its start and its end.  Under a power limit the
// SM clock drops below the reported application clock while the tensor pipe is busy, so the
// rate is quoted together with the clock it ran at.
__device__ unsigned long long peak_clock[3];          // cycles, ns, CTAs

// Shared memory: A 16 KB (128 rows x 128 B) | B 32 KB (256 rows; a pair CTA reads 128) | one
// scale atom 512 B.  Every operand the MMAs read lies inside this buffer.
constexpr int PEAK_A = 16384, PEAK_B = 32768, PEAK_SF = 512;
constexpr int PEAK_SMEM_USED = 1024 + PEAK_A + PEAK_B + PEAK_SF;
// Requested dynamic shared memory: more than half an SM's capacity, so exactly one CTA runs per
// SM and every CTA's 512-column TMEM allocation is uncontended.
constexpr int PEAK_SMEM = 128 * 1024;
static_assert(PEAK_SMEM >= PEAK_SMEM_USED, "peak kernel buffer");

template <int kCtaGroup>
__global__ void __launch_bounds__(128, 1) mma_peak_kernel(int iters, int random_operands) {
    extern __shared__ uint8_t peak_raw[];
    const unsigned long long c_start = clock64(), t_start = globaltimer_ns();
    __shared__ __align__(8) uint64_t bars[2];
    __shared__ uint32_t tmem_slot;
    const uint32_t raw_addr = smem_u32(peak_raw);
    uint8_t* ops = peak_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Operands: sparse constant codes, or (random_operands) every nibble pseudo-random so the
    // multipliers toggle like they do on real data (power, and with it the clock, depends on it).
    for (int i = threadIdx.x; i < (PEAK_A + PEAK_B) / 4; i += blockDim.x) {
        uint32_t h = (uint32_t)i * 0x9E3779B1u + blockIdx.x * 0x85EBCA77u;
        h ^= h >> 15;
        h *= 0x2C1B3C6Du;
        h ^= h >> 13;
        reinterpret_cast<uint32_t*>(ops)[i] = random_operands ? h : ((i % 5 == 0) ? 0x22222222u : 0u);
    }
    for (int i = threadIdx.x; i < PEAK_SF / 4; i += blockDim.x)
        reinterpret_cast<uint32_t*>(ops + PEAK_A + PEAK_B)[i] = 0x38383838u;   // scale 1.0
    uint32_t rank = 0;
    if constexpr (kCtaGroup == 2) asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&bars[0]), 1);
        mbar_init(smem_u32(&bars[1]), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (warp == 0) {
        if constexpr (kCtaGroup == 2) {
            asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&tmem_slot)));
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
        } else {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&tmem_slot)));
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
        }
        tc_fence_before();
    }
    __syncthreads();
    if constexpr (kCtaGroup == 2) asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    constexpr uint32_t M = kCtaGroup == 2 ? 256 : 128;
    constexpr uint32_t IDESC = (1u << 7) | (1u << 10) | ((256u >> 3) << 17) | ((M >> 4) << 24);
    if (warp == 0 && lane == 0 && rank == 0) {
        const uint32_t a = smem_u32(ops), b = smem_u32(ops + PEAK_A), sf = smem_u32(ops + PEAK_A + PEAK_B);
        auto desc = [](uint32_t s) {
            return (uint64_t)((s >> 4) & 0x3FFFu) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
        };
        const uint64_t sfd = (uint64_t)((sf >> 4) & 0x3FFFu) | ((uint64_t)(128 >> 4) << 32) | (1ull << 46);
        const uint32_t sf_cols[3] = {448, 456, 460};   // SFA (4 columns), SFB (8 columns)
        for (int j = 0; j < 3; j++) {
            if constexpr (kCtaGroup == 2)
                asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(tmem + sf_cols[j]), "l"(sfd));
            else
                asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(tmem + sf_cols[j]), "l"(sfd));
        }
        uint32_t parity[2] = {0, 0};
        bool ok = true;
        for (int g = 0; g * MMA_GROUP < iters && ok; g++) {
            const int slot = g & 1;
            if (g >= 2) {   // keep at most two groups in flight
                ok = mbar_wait(smem_u32(&bars[slot]), parity[slot], 2000000000ull, DEV_TIMEOUT_GEMM_MMA);
                parity[slot] ^= 1u;
            }
            for (int i = 0; i < MMA_GROUP; i++) {
                const uint64_t ad = desc(a + 32 * (i & 3)), bd = desc(b + 32 * (i & 3));
                if constexpr (kCtaGroup == 2)
                    asm volatile(
                        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                        "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(tmem),
                        "l"(ad), "l"(bd), "r"(IDESC), "r"(1u), "r"(tmem + 448), "r"(tmem + 456)
                        : "memory");
                else
                    asm volatile(
                        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(tmem),
                        "l"(ad), "l"(bd), "r"(IDESC), "r"(1u), "r"(tmem + 448), "r"(tmem + 456)
                        : "memory");
            }
            if constexpr (kCtaGroup == 2)
                asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(&bars[slot])) : "memory");
            else
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(&bars[slot])) : "memory");
        }
        // drain both slots
        const int groups = (iters + MMA_GROUP - 1) / MMA_GROUP;
        for (int g = groups - 2 > 0 ? groups - 2 : 0; g < groups; g++) {
            const int slot = g & 1;
            mbar_wait(smem_u32(&bars[slot]), parity[slot], 2000000000ull, DEV_TIMEOUT_GEMM_TEARDOWN);
            parity[slot] ^= 1u;
        }
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if constexpr (kCtaGroup == 2) asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    tc_fence_after();
    if (threadIdx.x == 0) {
        atomicAdd(&peak_clock[0], clock64() - c_start);
        atomicAdd(&peak_clock[1], globaltimer_ns() - t_start);
        atomicAdd(&peak_clock[2], 1ull);
    }
    if (warp == 0) {
        if constexpr (kCtaGroup == 2) asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, 512;" ::"r"(tmem));
        else asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
    }
}

}  // namespace diag
}  // namespace nvfp4

using namespace nvfp4;

extern "C" {

nvfp4_status_t nvfp4_diag_mma_peak(int cta_group, int iters, int random_operands, void* stream) {
    clear_error();
    if ((cta_group != 1 && cta_group != 2) || iters < 64)
        return fail(NVFP4_ERR_INVALID_ARG, "diag_mma_peak: cta_group in {1,2}, iters >= 64");
    const int sms = sm_count();
    cudaError_t e = cudaFuncSetAttribute(cta_group == 1 ? diag::mma_peak_kernel<1> : diag::mma_peak_kernel<2>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, diag::PEAK_SMEM);
    if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "diag_mma_peak: %s", cudaGetErrorString(e));
    if (cta_group == 1) {
        diag::mma_peak_kernel<1><<<sms, 128, diag::PEAK_SMEM, (cudaStream_t)stream>>>(iters, random_operands);
    } else {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * (sms / 2), 1, 1);
        cfg.blockDim = dim3(128, 1, 1);
        cfg.dynamicSmemBytes = diag::PEAK_SMEM;
        cfg.stream = (cudaStream_t)stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, diag::mma_peak_kernel<2>, iters, random_operands);
        if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "diag_mma_peak: %s", cudaGetErrorString(e));
    }
    return check_launch("mma_peak_kernel");
}

nvfp4_status_t nvfp4_diag_mma_peak_clock(double* mhz) {
    clear_error();
    if (!mhz) return fail(NVFP4_ERR_INVALID_ARG, "diag_mma_peak_clock: null output");
    unsigned long long v[3] = {0, 0, 0};
    cudaError_t e = cudaMemcpyFromSymbol(v, diag::peak_clock, sizeof(v));
    const unsigned long long z[3] = {0, 0, 0};
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(diag::peak_clock, z, sizeof(z));
    if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "diag_mma_peak_clock: %s", cudaGetErrorString(e));
    *mhz = v[1] ? (double)v[0] / (double)v[1] * 1e3 : 0.0;
    return NVFP4_OK;
}

}  // extern "C"
