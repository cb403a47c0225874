// gemm.cu -- NVFP4 block-scaled GEMM on tcgen05 (sm_100a).
//
//   D[M][N] = alpha * sum_k A[m][k] * B[n][k] * sfa[m][k/16] * sfb[n][k/16]
//
// Persistent, warp-specialised kernel, one CTA per SM, 192 threads:
//   warp 0      TMA producer: per stage one 2D TMA for A (128 rows x 128 B, SWIZZLE_128B),
//               one for B (256 rows x 128 B) and three 1D bulk copies for the scale atoms
//               (SFA 2 KB, SFB 2 x 2 KB), all completing on the stage's "full" mbarrier.
//   warp 1      MMA issuer (one lane): per stage copies the 12 scale atoms smem -> TMEM with
//               tcgen05.cp.32x128b.warpx4, issues four
//               tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X
//               (M128 N256 K64 each) and commits to the stage's "empty" mbarrier.  It never
//               waits for its own MMAs; after a tile's last stage it commits to "tmem_full".
//   warps 2..5  epilogue: tcgen05.ld.32x32b of the fp32 accumulator (lane quadrant = warp % 4),
//               scale by alpha, round to bf16, 16-byte global stores; then arrive "tmem_empty".
//
// TMEM (512 columns): accumulator D in columns [0, 256); scale factors at [256, 304):
//   SFA for K step j at 256 + 4j (4 columns = 128 rows), SFB at 272 + 8j (8 columns = 256 rows).
//   Scale word layout in TMEM: lane = row % 32 (replicated in the four lane quadrants),
//   column = row / 32, byte = 16-block index within the 64-wide K step; this is what
//   tcgen05.cp 32x128b.warpx4 produces from one 512-byte atom of the tcgen05 SF layout.
//
// Reference: the single-CTA mainloop ws_tcgen05_explicit_pipeline_kernel
// (blackwell/warp_specialization_sm100/sm100_tcgen05_nvfp4_tma_multistage_pipeline.cu:117)
// waits for every MMA before releasing a stage, keeps scales fixed at 1.0 and runs one tile.
// Here the MMA warp only commits, scales are real per-16 UE4M3 factors, and the grid is
// persistent over all output tiles.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "capi_internal.h"
#include "nvfp4_common.cuh"

namespace nvfp4 {
namespace gemm {

constexpr int BM = 128, BN = 256, BK = 256;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK / 2;                        // 16 KB
constexpr int B_BYTES = BN * BK / 2;                        // 32 KB
constexpr int SFA_BYTES = (BM / 128) * (BK / 64) * 512;     // 2 KB
constexpr int SFB_BYTES = (BN / 128) * (BK / 64) * 512;     // 4 KB
constexpr int STAGE_TX = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
constexpr int NUM_THREADS = 192;
constexpr int TMEM_COLS = 512;
constexpr int TMEM_SFA = 256;
constexpr int TMEM_SFB = 272;

constexpr int OFF_A = 0;
constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
constexpr int OFF_SFA = OFF_B + STAGES * B_BYTES;
constexpr int OFF_SFB = OFF_SFA + STAGES * SFA_BYTES;
constexpr int OFF_BAR = OFF_SFB + STAGES * SFB_BYTES;
constexpr int NUM_BARS = 2 * STAGES + 3;                    // full, empty, tmem_full, tmem_empty, drain
constexpr int OFF_TMEM_PTR = OFF_BAR + NUM_BARS * 8;
constexpr int SMEM_BYTES = 1024 + OFF_TMEM_PTR + 16;
static_assert(SMEM_BYTES <= 232448, "shared memory budget");

constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;           // 2 s per wait

// Instruction descriptor: E2M1 x E2M1, UE4M3 scales, K-major A and B, M=128, N=256.
constexpr uint32_t IDESC = (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

// Shared-memory matrix descriptor, K-major, SWIZZLE_128B: rows of 128 bytes, 8-row groups
// 1024 bytes apart (SBO), version 1.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}
// Descriptor of one 512-byte scale atom for tcgen05.cp: 32 rows x 16 bytes, no swizzle,
// 8-row groups 128 bytes apart.
__device__ __forceinline__ uint64_t desc_sf(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(128 >> 4) << 32) | (1ull << 46);
}

__device__ __forceinline__ void tc_cp_sf(uint32_t taddr, uint64_t desc) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(desc) : "memory");
}

__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t sfa, uint32_t sfb,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(IDESC), "r"(accumulate), "r"(sfa), "r"(sfb)
        : "memory");
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

template <bool kOutF32>
__global__ void __launch_bounds__(NUM_THREADS, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
            const uint8_t* __restrict__ sfa, const uint8_t* __restrict__ sfb, void* __restrict__ out,
            int M, int N, int K, float alpha) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    const uint32_t base = (raw_addr + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (base - raw_addr);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t bar0 = base + OFF_BAR;
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
    const uint32_t tmem_full = bar0 + 8u * (2 * STAGES);
    const uint32_t tmem_empty = tmem_full + 8u;
    const uint32_t drain_bar = tmem_full + 16u;
    uint32_t* tmem_ptr = reinterpret_cast<uint32_t*>(smem + OFF_TMEM_PTR);

    const int num_m = M / BM, num_n = N / BN, tiles = num_m * num_n;
    const int nkb = K / BK;
    const int64_t katoms = K / 64;

    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmap_a);
        prefetch_tmap(&tmap_b);
        for (int s = 0; s < STAGES; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        mbar_init(tmem_full, 1);
        mbar_init(tmem_empty, 128);
        mbar_init(drain_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_ptr)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_ptr;
    // Self-check: a 512-column allocation owns all of TMEM and starts at lane 0, column 0.
    const int ntiles = (tmem == 0u) ? tiles : 0;
    if (tmem != 0u && threadIdx.x == 0) record_error(DEV_TMEM_BASE);

    if (warp == 0) {
        // ------------------------------------------------------------ producer ----
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            uint32_t pending = 0;   // stages with loads issued but not yet released by the MMA
            for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
                const int m_blk = tile % num_m, n_blk = tile / num_m;
                for (int kb = 0; kb < nkb; kb++) {
                    if (!mbar_wait(empty_bar(stage), phase ^ 1u, WAIT_LIMIT_NS, DEV_TIMEOUT_GEMM_PRODUCER)) {
                        ok = false;
                        break;
                    }
                    pending &= ~(1u << stage);
                    const uint32_t fb = full_bar(stage);
                    mbar_arrive_expect_tx(fb, STAGE_TX);
                    tma_load_2d(base + OFF_A + stage * A_BYTES, &tmap_a, kb * (BK / 2), m_blk * BM, fb);
                    tma_load_2d(base + OFF_B + stage * B_BYTES, &tmap_b, kb * (BK / 2), n_blk * BN, fb);
                    bulk_load(base + OFF_SFA + stage * SFA_BYTES,
                              sfa + ((int64_t)m_blk * katoms + kb * 4) * 512, SFA_BYTES, fb);
                    bulk_load(base + OFF_SFB + stage * SFB_BYTES,
                              sfb + ((int64_t)(2 * n_blk) * katoms + kb * 4) * 512, SFB_BYTES / 2, fb);
                    bulk_load(base + OFF_SFB + stage * SFB_BYTES + SFB_BYTES / 2,
                              sfb + ((int64_t)(2 * n_blk + 1) * katoms + kb * 4) * 512, SFB_BYTES / 2, fb);
                    pending |= 1u << stage;
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
            }
            for (int s = 0; s < STAGES; s++) {
                if (!(pending & (1u << s))) continue;
                const uint32_t par = (s < stage) ? phase : (phase ^ 1u);
                if (ok) {
                    // Tail: wait until the MMA released every filled stage, so no completion
                    // signal of the tensor pipe lands in shared memory after the CTA exits.
                    if (!mbar_wait(empty_bar(s), par, WAIT_LIMIT_NS, DEV_TIMEOUT_GEMM_TEARDOWN)) break;
                } else {
                    // Do not leave bulk copies in flight into shared memory that is about to be
                    // released: wait (bounded) for every stage that still has loads outstanding.
                    mbar_wait(full_bar(s), par, WAIT_LIMIT_NS, DEV_TIMEOUT_GEMM_TEARDOWN);
                }
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA issuer ----
        int stage = 0;
        uint32_t phase = 0, acc_phase = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
            if (!mbar_wait(tmem_empty, acc_phase ^ 1u, WAIT_LIMIT_NS, DEV_TIMEOUT_GEMM_MMA)) { ok = false; break; }
            tc_fence_after();
            for (int kb = 0; kb < nkb; kb++) {
                if (!mbar_wait(full_bar(stage), phase, WAIT_LIMIT_NS, DEV_TIMEOUT_GEMM_MMA)) { ok = false; break; }
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t sa = base + OFF_SFA + stage * SFA_BYTES;
                    const uint32_t sb = base + OFF_SFB + stage * SFB_BYTES;
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        tc_cp_sf(tmem + TMEM_SFA + 4 * j, desc_sf(sa + 512 * j));
                        tc_cp_sf(tmem + TMEM_SFB + 8 * j, desc_sf(sb + 512 * j));
                        tc_cp_sf(tmem + TMEM_SFB + 8 * j + 4, desc_sf(sb + SFB_BYTES / 2 + 512 * j));
                    }
                    const uint32_t a0 = base + OFF_A + stage * A_BYTES;
                    const uint32_t b0 = base + OFF_B + stage * B_BYTES;
#pragma unroll
                    for (int j = 0; j < 4; j++)
                        tc_mma(tmem, desc_sw128(a0 + 32 * j), desc_sw128(b0 + 32 * j), tmem + TMEM_SFA + 4 * j,
                               tmem + TMEM_SFB + 8 * j, (kb | j) != 0);
                    tc_commit(empty_bar(stage));
                }
                __syncwarp();
                if (++stage == STAGES) { stage = 0; phase ^= 1u; }
            }
            if (!ok) break;
            if (lane == 0) tc_commit(tmem_full);
            __syncwarp();
            acc_phase ^= 1u;
        }
        // Make sure no MMA or copy of this CTA is still running before TMEM is released.
        if (lane == 0) {
            tc_commit(drain_bar);
            mbar_wait(drain_bar, 0, WAIT_LIMIT_NS, DEV_TIMEOUT_GEMM_TEARDOWN);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------ epilogue ----
        const int quad = warp & 3;
        uint32_t acc_phase = 0;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
            const int m_blk = tile % num_m, n_blk = tile / num_m;
            if (!mbar_wait(tmem_full, acc_phase, WAIT_LIMIT_NS, DEV_TIMEOUT_GEMM_EPILOGUE)) break;
            tc_fence_after();
            const int64_t row = (int64_t)m_blk * BM + quad * 32 + lane;
#pragma unroll 1
            for (int c = 0; c < BN / 32; c++) {
                uint32_t r[32];
                tc_ld32(tmem + ((uint32_t)(quad * 32) << 16) + c * 32, r);
                tc_wait_ld();
                const int64_t col = (int64_t)n_blk * BN + c * 32;
                if constexpr (kOutF32) {
                    uint8_t* dst = reinterpret_cast<uint8_t*>(reinterpret_cast<float*>(out) + row * N + col);
#pragma unroll
                    for (int i = 0; i < 8; i++)
                        st_v4(dst + 16 * i, make_uint4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]));
                } else {
                    uint32_t o[16];
#pragma unroll
                    for (int i = 0; i < 16; i++) {
                        const __nv_bfloat162 p = __floats2bfloat162_rn(__fmul_rn(__uint_as_float(r[2 * i]), alpha),
                                                                       __fmul_rn(__uint_as_float(r[2 * i + 1]), alpha));
                        o[i] = *reinterpret_cast<const uint32_t*>(&p);
                    }
                    uint8_t* dst = reinterpret_cast<uint8_t*>(reinterpret_cast<__nv_bfloat16*>(out) + row * N + col);
#pragma unroll
                    for (int i = 0; i < 4; i++)
                        st_v4(dst + 16 * i, make_uint4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]));
                }
            }
            tc_fence_before();
            mbar_arrive(tmem_empty);
            acc_phase ^= 1u;
        }
    }

    // Reconverge every warp (the producer and MMA roles run on lane 0 only) before the
    // CTA-wide barrier, which is a warp-aligned instruction.
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
}

// ------------------------------------------------------------------ host ----
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 2D byte tensor [rows][row_bytes] with a box of box_rows x 128 bytes, SWIZZLE_128B.
static nvfp4_status_t make_tmap(CUtensorMap* m, const void* ptr, int64_t rows, int64_t row_bytes, int box_rows) {
    auto enc = get_encode();
    if (!enc) return fail(NVFP4_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    cuuint32_t box[2] = {128, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(NVFP4_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return NVFP4_OK;
}

template <bool kOutF32>
static nvfp4_status_t launch(const void* A, const void* sfa, const void* B, const void* sfb, float alpha, void* D,
                             int64_t M, int64_t N, int64_t K, cudaStream_t s) {
    if (!A || !sfa || !B || !sfb || !D) return fail(NVFP4_ERR_INVALID_ARG, "gemm: null pointer");
    if (M <= 0 || N <= 0 || K <= 0 || M % BM || N % BN || K % BK)
        return fail(NVFP4_ERR_INVALID_ARG, "gemm: need M %% 128 == 0, N %% 256 == 0, K %% 256 == 0 (got %lld %lld %lld)",
                    (long long)M, (long long)N, (long long)K);
    if (M > (1ll << 30) || N > (1ll << 30) || K > (1ll << 30))
        return fail(NVFP4_ERR_INVALID_ARG, "gemm: dimension too large");
    if (!aligned16(A) || !aligned16(B) || !aligned16(sfa) || !aligned16(sfb) || !aligned16(D))
        return fail(NVFP4_ERR_INVALID_ARG, "gemm: buffers must be 16-byte aligned");
    CUtensorMap ta, tb;
    nvfp4_status_t st = make_tmap(&ta, A, M, K / 2, BM);
    if (st != NVFP4_OK) return st;
    st = make_tmap(&tb, B, N, K / 2, BN);
    if (st != NVFP4_OK) return st;
    static bool attr_set[64] = {};   // per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemm_kernel<kOutF32>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
        if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "gemm: smem attribute: %s", cudaGetErrorString(e));
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    const int tiles = (int)((M / BM) * (N / BN));
    const int grid = tiles < sm_count() ? tiles : sm_count();
    gemm_kernel<kOutF32><<<grid, NUM_THREADS, SMEM_BYTES, s>>>(ta, tb, (const uint8_t*)sfa, (const uint8_t*)sfb, D,
                                                               (int)M, (int)N, (int)K, alpha);
    return check_launch("gemm_kernel");
}

}  // namespace gemm
}  // namespace nvfp4

