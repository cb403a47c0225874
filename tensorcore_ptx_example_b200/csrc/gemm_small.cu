// gemm_small.cu -- NVFP4 block-scaled GEMM for small M (decode shapes, M <= 128), sm_100a.
//
//   D[M][N] = alpha * sum_k A[m][k] B[n][k] sfa sfb      (same contract as nvfp4_gemm_bf16)
//
// With M = 16 the GEMM is a stream over B (N x K E2M1 + scales, 33 MB at N = 7168, K = 8192) and
// is HBM-bound.  The kernel swaps the operands so that the 128-row tensor-core tile runs over N:
// the MMA computes D^T tiles [128 n][Mp m] (Mp = M rounded up to 16) with B as the M-side operand
// and A as the N-side operand of tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X.
// Split-K gives enough work units to stream B from every SM: unit (n-tile, s) covers K range
// [s * Ks, (s + 1) * Ks).  The partial tiles are summed in split order 0..S-1 (fp32, round to
// nearest) and alpha -> bf16 is applied, in one of two ways:
//   in-cluster (one launch, no workspace; when S <= 8 divides 128): one CTA per unit, the S CTAs of
//     an n-tile form a thread-block cluster.  CTA r owns rows [r * 128 / S, (r + 1) * 128 / S) of the
//     tile: every CTA pushes its partial of those rows into CTA r's receive buffer (one-way
//     st.shared::cluster stores) and arrives on CTA r's "ready" mbarrier; CTA r then sums the S
//     partials in split order from its own shared memory and stores D.  (Reading the peers'
//     partials with ld.shared::cluster instead was measured slower: one round trip per load.)
//   workspace (otherwise): the partials go to a global workspace and a second kernel (four
//     outputs per thread, all S partial loads in flight) sums them.  Both kernels are
//     programmatic dependent launches.
// Both give the same bits.
//
// Persistent CTAs walk the work units (n-tile, split), split fastest so that the SMs stream
// neighbouring stretches of B.  For Mp <= 64 two CTAs share an SM (about 100 KB of shared memory
// and 256 TMEM columns each: two independent pipelines per SM); the grid is the largest one that
// divides the units evenly (cfg3 decode: 224 units on 224 CTAs).
//   warp 0      TMA producer: per 256-K stage the scale atoms of B and A (2 KB each, bulk copies)
//               on the stage's "sf_landed" barrier, then one box of B (128 rows x 128 B) and one
//               box of A (Mp rows x 128 B), both SWIZZLE_128B, on its "full" barrier;
//   warp 1      MMA issuer: per stage one wait on "full" (polled with test_wait), four
//               tcgen05.mma (M128 N=Mp K64), then one commit that releases the stage; after a
//               unit's last stage a commit to its accumulator buffer;
//   warps 2-5   epilogue: tcgen05.ld of a finished unit's D^T tile, fp32 partial -> workspace;
//   warps 6-9   scale warps: the stage's scale atoms shared memory -> registers -> TMEM slot of
//               the same index (tcgen05.st, lane quadrant warp % 4), then an arrival on the
//               stage's "full" barrier, which therefore completes only when the scales are in
//               TMEM too.  A slot is rewritten only after its stage was refilled, which the
//               producer does only after the MMAs that read the slot completed.
// TMEM: two accumulator buffers of Mp columns at [0, Mp) and [Mp, 2 Mp), then one 32-column scale
// slot per stage (B scales +0..15, A scales +16..31); the allocation is the next power of two.
//
// Timeline at cfg3 with the workspace reduction (M16 N7168 K8192, 224 CTAs, measured with global
// timestamps): CTA starts spread over 0.9 us, set-up 0.8 us, first stage lands 2 us later, the
// stream of B then runs at ~6.6 TB/s for ~5 us, the last CTA exits at ~8.5 us and the reduction
// kernel ends at ~11.5 us; the in-cluster reduction removes that second kernel.
#include "capi_internal.h"
#include "nvfp4_common.cuh"
#include "tma_host.h"

namespace nvfp4 {
namespace gsmall {

using gemm::desc_sw128;

constexpr int THREADS = 320;
constexpr int SF_SLOT_COLS = 32;
constexpr int MAX_STAGES = 8;
constexpr int B_BOX = 128 * 128;                      // 128 rows x 128 B (256 K)
constexpr int SF_STAGE = 2 * 4 * 512;                 // scale atoms of B and of A for 256 K
// Shared-memory budget of one CTA: 200 KB with one CTA per SM; ~100 KB when two CTAs share an SM
// (Mp <= 64, where the TMEM layout below fits in 256 columns), giving each SM two independent
// load/MMA pipelines.
#ifndef GSMALL_CTAS_PER_SM
#define GSMALL_CTAS_PER_SM 2
#endif
constexpr int SMEM_BUDGET_1 = 200 * 1024;
constexpr int SMEM_BUDGET_2 = 100 * 1024;
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;

__host__ __device__ constexpr int stage_bytes(int mp) { return B_BOX + mp * 128 + SF_STAGE; }
__host__ __device__ constexpr int ctas_per_sm(int mp) { return (GSMALL_CTAS_PER_SM == 2 && mp <= 64) ? 2 : 1; }
// In-cluster reduction: a receive buffer for the partial rows this CTA sums, [split][mp][rows]
// fp32 (128 x mp floats in all), after the stage ring.
__host__ __device__ constexpr int recv_bytes(int mp) { return 128 * mp * 4; }
__host__ __device__ constexpr int stage_budget(int mp, bool cl) {
    return (ctas_per_sm(mp) == 2 ? SMEM_BUDGET_2 : SMEM_BUDGET_1) - (cl ? recv_bytes(mp) : 0);
}
__host__ __device__ constexpr int num_stages(int mp, bool cl = false) {
    return stage_budget(mp, cl) / stage_bytes(mp) < MAX_STAGES ? stage_budget(mp, cl) / stage_bytes(mp) : MAX_STAGES;
}
// TMEM: accumulator buffers [0, mp) and [mp, 2 mp) (fp32 D^T tile, one column per output
// column), then one 32-column scale slot per stage; the allocation is the next power of two.
__host__ __device__ constexpr int sf_col0(int mp) { return (2 * mp + 31) / 32 * 32; }
__host__ __device__ constexpr int tmem_cols(int mp) {
    return sf_col0(mp) + SF_SLOT_COLS * num_stages(mp) <= 32    ? 32
           : sf_col0(mp) + SF_SLOT_COLS * num_stages(mp) <= 64  ? 64
           : sf_col0(mp) + SF_SLOT_COLS * num_stages(mp) <= 128 ? 128
           : sf_col0(mp) + SF_SLOT_COLS * num_stages(mp) <= 256 ? 256
                                                                 : 512;
}
static_assert(sf_col0(128) + SF_SLOT_COLS * MAX_STAGES <= 512, "scale slots fit in TMEM");
static_assert(ctas_per_sm(64) == 1 || (tmem_cols(64) <= 256 && tmem_cols(16) <= 256),
              "two CTAs per SM share the 512 TMEM columns");
// [stages][receive buffer (in-cluster)][full, empty, sf_landed per stage][acc_full 2][acc_empty 2]
// [drain][ready][tmem slot]
constexpr int NUM_BARS = 3 * MAX_STAGES + 6;
__host__ __device__ constexpr int smem_bytes(int mp, bool cl) {
    return 1024 + num_stages(mp, cl) * stage_bytes(mp) + (cl ? recv_bytes(mp) : 0) + NUM_BARS * 8 + 16;
}
static_assert(num_stages(16, true) >= 2 && num_stages(64, true) >= 2 && num_stages(128, true) >= 2,
              "stages left next to the receive buffer");
constexpr int MAX_CLUSTER_SPLITS = 8;

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t mapa_rank(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
// One arrival on the mbarrier at `addr` (this CTA's or a peer's, a shared::cluster address),
// ordered after this thread's earlier memory operations at cluster scope.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(addr) : "memory");
}
// Bounded wait whose completion acquires at cluster scope (the arrivals came from peer CTAs).
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t parity, uint64_t limit_ns, unsigned int err) {
    uint64_t t0 = 0;
#pragma unroll 1
    for (int i = 0;; i++) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(bar), "r"(parity)
            : "memory");
        if (ok) return true;
        if (i == 64) t0 = globaltimer_ns();
        if (i > 64 && globaltimer_ns() - t0 > limit_ns) {
            record_error(err);
            return false;
        }
    }
}

__device__ __forceinline__ void tc_st_x16(uint32_t taddr, const uint4* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16};" ::"r"(taddr),
        "r"(v[0].x), "r"(v[0].y), "r"(v[0].z), "r"(v[0].w), "r"(v[1].x), "r"(v[1].y), "r"(v[1].z), "r"(v[1].w),
        "r"(v[2].x), "r"(v[2].y), "r"(v[2].z), "r"(v[2].w), "r"(v[3].x), "r"(v[3].y), "r"(v[3].z), "r"(v[3].w)
        : "memory");
}
__device__ __forceinline__ void tc_ld_x16(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tc_mma_rt(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t sfa,
                                          uint32_t sfb, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
        : "memory");
}

// Workspace path (csplits == 0): ws[s][m][n] = partial of split s (fp32, the tensor core's
// accumulation over that K range).  In-cluster path (csplits = S, launched with cluster dims
// (S, 1, 1) and one CTA per unit): D (bf16, or fp32 for out_f32) is written directly.
__global__ void __launch_bounds__(THREADS, 1)
gemm_small_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                  const uint8_t* __restrict__ sfa, const uint8_t* __restrict__ sfb, float* __restrict__ ws, int M,
                  int N, int K, int ks, int mp, int b_const, int csplits, void* __restrict__ D, float alpha,
                  int out_f32) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    const uint32_t base = (raw_addr + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (base - raw_addr);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = num_stages(mp, csplits > 0), SB = stage_bytes(mp);
    const int n_tiles = N / 128, splits = K / ks, units = n_tiles * splits;
    const int katoms = K / 64, nbox = ks / 256;
    const uint32_t recv0 = base + S * SB;                 // in-cluster receive buffer
    const uint32_t bar0 = recv0 + (csplits > 0 ? recv_bytes(mp) : 0);
    auto full_bar = [&](int st) { return bar0 + 8u * st; };
    auto empty_bar = [&](int st) { return bar0 + 8u * (MAX_STAGES + st); };
    auto sf_landed = [&](int st) { return bar0 + 8u * (2 * MAX_STAGES + st); };
    const int acc_cols = mp, sf0 = sf_col0(mp), tcols = tmem_cols(mp);
    const uint32_t acc_full = bar0 + 8u * (3 * MAX_STAGES), acc_empty = acc_full + 16, drain = acc_full + 32;
    const uint32_t ready_bar = acc_full + 40;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + (bar0 - base) + NUM_BARS * 8);
    uint32_t* abort_flag = tmem_slot + 1;       // the epilogue warps give up together

    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmap_a);
        prefetch_tmap(&tmap_b);
        for (int st = 0; st < S; st++) {
            mbar_init(full_bar(st), 1 + 4);            // producer (B/A bytes) + the four scale warps
            mbar_init(empty_bar(st), 1);
            mbar_init(sf_landed(st), 1);               // producer (scale bytes)
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(acc_full + 8 * b, 1);
            mbar_init(acc_empty + 8 * b, 4);           // the four epilogue warps
        }
        mbar_init(drain, 1);
        mbar_init(ready_bar, csplits > 0 ? 4 * csplits : 1);   // each epilogue warp of every CTA
        *abort_flag = 0u;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(tcols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
        tc_fence_before();
    }
    __syncthreads();
    // Peers write into this CTA's receive buffer and arrive on its barrier only after it is
    // initialised: every thread arrives on the cluster barrier here and waits on it only before
    // its first access to a peer (the epilogue) or at exit.
    if (csplits > 0) asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // Programmatic dependent launch: the set-up above overlapped the previous kernel in the
    // stream; its results are visible after this wait.  The split-K reduction may launch now
    // (it waits for this grid in turn).  With b_const (B and its scales are not written by
    // earlier work in the stream, e.g. weights) the producer first issues the B loads of its
    // first stages and waits afterwards.
    if (!(b_const && warp == 0)) asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (warp == 0) {
        // ------------------------------------------------------------ producer ----
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            long fills = 0;
            // b_const: B and its scales of the first S stages (the ring's first use needs no
            // wait), issued before the dependency wait; their A halves follow it
            int pre = 0;
            if (b_const) {
                for (int u = blockIdx.x; u < units && pre < S; u += gridDim.x) {
                    const int sp = u % splits, nt = u / splits;
                    for (int b = 0; b < nbox && pre < S; b++, pre++) {
                        const int k = sp * ks + 256 * b;
                        const uint32_t sbase = base + pre * SB, fb = full_bar(pre), lb = sf_landed(pre);
                        mbar_arrive_expect_tx(lb, (uint32_t)SF_STAGE);
                        bulk_load(sbase + B_BOX + mp * 128, sfb + ((int64_t)nt * katoms + k / 64) * 512, 2048, lb);
                        mbar_arrive_expect_tx(fb, (uint32_t)(B_BOX + mp * 128));
                        tma_load_2d(sbase, &tmap_b, k / 2, nt * 128, fb);
                    }
                }
                asm volatile("griddepcontrol.wait;" ::: "memory");
            }
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
                const int sp = u % splits, nt = u / splits;
                for (int b = 0; b < nbox; b++) {
                    const int k = sp * ks + 256 * b;
                    const uint32_t sbase = base + stage * SB, fb = full_bar(stage), lb = sf_landed(stage);
                    if (fills < pre) {
                        // B already on its way: the A halves of the stage
                        bulk_load(sbase + B_BOX + mp * 128 + 2048, sfa + (int64_t)(k / 64) * 512, 2048, lb);
                        tma_load_2d(sbase + B_BOX, &tmap_a, k / 2, 0, fb);
                    } else {
                        if (!mbar_wait(empty_bar(stage), phase ^ 1u, WAIT_LIMIT_NS, DEV_TIMEOUT_GEMM_PRODUCER)) {
                            ok = false;
                            break;
                        }
                        // scales first (the scale warps move them on to TMEM), then B and A
                        mbar_arrive_expect_tx(lb, (uint32_t)SF_STAGE);
                        bulk_load(sbase + B_BOX + mp * 128, sfb + ((int64_t)nt * katoms + k / 64) * 512, 2048, lb);
                        bulk_load(sbase + B_BOX + mp * 128 + 2048, sfa + (int64_t)(k / 64) * 512, 2048, lb);
                        mbar_arrive_expect_tx(fb, (uint32_t)(B_BOX + mp * 128));
                        tma_load_2d(sbase, &tmap_b, k / 2, nt * 128, fb);
                        tma_load_2d(sbase + B_BOX, &tmap_a, k / 2, 0, fb);
                    }
                    fills++;
                    if (++stage == S) { stage = 0; phase ^= 1u; }
                }
            }
            // Tail: every filled stage is released by an MMA commit before the CTA exits.
            for (int st = 0; st < S && st < fills && ok; st++)
                if (!mbar_wait(empty_bar(st), st < stage ? phase : (phase ^ 1u), WAIT_LIMIT_NS, DEV_TIMEOUT_GEMM_TEARDOWN))
                    break;
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA issuer ----
        if (lane == 0) {
            const uint32_t idesc = (1u << 7) | (1u << 10) | ((uint32_t)(mp >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            int iter = 0;
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x, iter++) {
                const int buf = iter & 1;
                if (iter >= 2 &&
                    !mbar_wait(acc_empty + 8 * buf, (uint32_t)(((iter >> 1) - 1) & 1), WAIT_LIMIT_NS, DEV_TIMEOUT_GEMM_MMA)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + acc_cols * buf;
                for (int b = 0; b < nbox; b++) {
                    // B/A landed and the scale warps have put the stage's scales in TMEM
                    if (!mbar_wait_spin(full_bar(stage), phase, WAIT_LIMIT_NS, DEV_TIMEOUT_GEMM_MMA)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sbase = base + stage * SB;
                    const uint32_t slot = tmem + sf0 + SF_SLOT_COLS * stage;
#pragma unroll
                    for (int kk = 0; kk < 4; kk++)
                        tc_mma_rt(d, desc_sw128(sbase + 32 * kk), desc_sw128(sbase + B_BOX + 32 * kk), idesc,
                                  slot + 4 * kk, slot + 16 + 4 * kk, (b | kk) != 0);
                    tc_commit(empty_bar(stage));
                    if (++stage == S) { stage = 0; phase ^= 1u; }
                }
                if (!ok) break;
                tc_commit(acc_full + 8 * buf);
            }
            tc_commit(drain);
            mbar_wait(drain, 0, WAIT_LIMIT_NS, DEV_TIMEOUT_GEMM_TEARDOWN);
        }
        __syncwarp();
    } else if (warp >= 6) {
        // -------------------------------------------------------- scale warps ----
        const uint32_t lane_base = ((uint32_t)(warp & 3) * 32u) << 16;
        int stage = 0;
        uint32_t phase = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x) {
            bool ok = true;
            for (int b = 0; b < nbox; b++) {
                if (!__all_sync(0xFFFFFFFFu, mbar_wait(sf_landed(stage), phase, WAIT_LIMIT_NS, DEV_TIMEOUT_GEMM_SF))) {
                    ok = false;
                    break;
                }
                const uint8_t* sf = smem + stage * SB + B_BOX + mp * 128 + 16 * lane;
                uint4 vb[4], va[4];
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    vb[j] = *reinterpret_cast<const uint4*>(sf + 512 * j);
                    va[j] = *reinterpret_cast<const uint4*>(sf + 2048 + 512 * j);
                }
                const uint32_t slot = tmem + lane_base + sf0 + SF_SLOT_COLS * stage;
                tc_st_x16(slot, vb);
                tc_st_x16(slot + 16, va);
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(full_bar(stage));
                if (++stage == S) { stage = 0; phase ^= 1u; }
            }
            if (!ok) break;
        }
    } else if (csplits > 0) {
        // ------------------------------------------ epilogue, in-cluster reduction ----
        // One unit per CTA: split sp = this CTA's rank in the cluster, n-tile nt = cluster index.
        // CTA r of the cluster owns rows [r * rows, (r + 1) * rows) of the n-tile: every CTA
        // pushes its partial of those rows into CTA r's receive buffer (one-way stores to peer
        // shared memory) and arrives on CTA r's "ready" barrier; CTA r then sums the partials in
        // split order from its own shared memory and stores D.
        const uint32_t q = (uint32_t)(warp & 3);
        const int t = (int)threadIdx.x - 64;                  // 0..127 over the four epilogue warps
        const int sp = blockIdx.x % csplits, nt = blockIdx.x / csplits;
        const int rows = 128 / csplits;
        const bool ok = __all_sync(0xFFFFFFFFu, mbar_wait(acc_full, 0u, WAIT_LIMIT_NS, DEV_TIMEOUT_GEMM_EPILOGUE));
        tc_fence_after();
        asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");   // peers initialised
        const int n = (int)q * 32 + lane;                     // TMEM lane = row n of the D^T tile
        const int owner = n / rows, nn = n - owner * rows;
        const uint32_t dst = mapa_rank(recv0, (uint32_t)owner) + (uint32_t)((sp * mp * rows + nn) * 4);
        if (ok) {
            for (int c = 0; c < mp; c += 16) {
                uint32_t r[16];
                tc_ld_x16(tmem + ((q * 32u) << 16) + c, r);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int i = 0; i < 16; i++) st_cluster_f32(dst + (uint32_t)((c + i) * rows * 4), __uint_as_float(r[i]));
            }
        }
        __syncwarp();
        // (a warp that gave up arrives too, so no owner waits out its time limit; the status word
        // already records the failure)
        if (lane == 0)
            for (int r = 0; r < csplits; r++) mbar_arrive_cluster(mapa_rank(ready_bar, (uint32_t)r));
        if (mbar_wait_cluster(ready_bar, 0u, WAIT_LIMIT_NS, DEV_TIMEOUT_GEMM_EPILOGUE)) {
            const float* recv = reinterpret_cast<const float*>(smem + (recv0 - base));
            const int n0 = sp * rows;
            for (int i = t; i < rows * M; i += 128) {
                const int m = i / rows, r0 = i - m * rows;
                float acc = 0.0f;
                for (int s2 = 0; s2 < csplits; s2++) acc = __fadd_rn(acc, recv[(s2 * mp + m) * rows + r0]);
                const int64_t o = (int64_t)m * N + (int64_t)nt * 128 + n0 + r0;
                if (out_f32) reinterpret_cast<float*>(D)[o] = acc;
                else reinterpret_cast<__nv_bfloat16*>(D)[o] = __float2bfloat16_rn(__fmul_rn(acc, alpha));
            }
        }
    } else {
        // ------------------------------------------------ epilogue, workspace path ----
        const uint32_t q = (uint32_t)(warp & 3);
        const uint32_t lane_base = (q * 32u) << 16;
        int iter = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x, iter++) {
            const int buf = iter & 1;
            const bool ok = __all_sync(0xFFFFFFFFu, mbar_wait(acc_full + 8 * buf, (uint32_t)((iter >> 1) & 1),
                                                              WAIT_LIMIT_NS, DEV_TIMEOUT_GEMM_EPILOGUE));
            if (!ok && lane == 0) *abort_flag = 1u;
            tc_fence_after();
            const int sp = u % splits, nt = u / splits;
            const int n = nt * 128 + (int)q * 32 + lane;  // TMEM lane = row n of the D^T tile
            if (ok) {
                float* dst = ws + (int64_t)sp * M * N + n;
                for (int c = 0; c < mp; c += 16) {
                    uint32_t r[16];
                    tc_ld_x16(tmem + lane_base + acc_cols * buf + c, r);
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                    for (int i = 0; i < 16; i++)
                        if (c + i < M) dst[(int64_t)(c + i) * N] = __uint_as_float(r[i]);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(acc_empty + 8 * buf);
            }
            named_bar_sync(1, 128);
            if (*abort_flag) break;                         // every epilogue warp sees the same flag
        }
    }

    __syncwarp();
    // the threads that did not wait on the cluster barrier yet (all but the in-cluster epilogue)
    if (csplits > 0 && !(warp >= 2 && warp < 6)) asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tcols));
}

// out[m][n] = bf16(alpha * (((ws[0] + ws[1]) + ws[2]) + ...)) (or the fp32 sum for kOutF32); four
// consecutive outputs per thread (16-byte loads; M*N is a multiple of 128), the partial loads of
// up to 16 splits issued before the ordered adds.
template <bool kOutF32>
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* __restrict__ ws, void* __restrict__ out,
                                                            int64_t mn, int splits, float alpha) {
    // The next kernel in the stream may launch now and overlap its set-up with this one; the
    // partials of the GEMM kernel are visible after the wait.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int64_t mn4 = mn / 4;
    const float4* w4 = reinterpret_cast<const float4*>(ws);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < mn4; i += (int64_t)gridDim.x * blockDim.x) {
        float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
        for (int t0 = 0; t0 < splits; t0 += 16) {
            float4 v[16];
#pragma unroll
            for (int t = 0; t < 16; t++)
                v[t] = (t0 + t < splits) ? __ldcg(w4 + (int64_t)(t0 + t) * mn4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int t = 0; t < 16; t++)
                if (t0 + t < splits) {
                    a0 = __fadd_rn(a0, v[t].x);
                    a1 = __fadd_rn(a1, v[t].y);
                    a2 = __fadd_rn(a2, v[t].z);
                    a3 = __fadd_rn(a3, v[t].w);
                }
        }
        if constexpr (kOutF32) {
            reinterpret_cast<float4*>(out)[i] = make_float4(a0, a1, a2, a3);
        } else {
            const __nv_bfloat162 lo = __floats2bfloat162_rn(__fmul_rn(a0, alpha), __fmul_rn(a1, alpha));
            const __nv_bfloat162 hi = __floats2bfloat162_rn(__fmul_rn(a2, alpha), __fmul_rn(a3, alpha));
            uint2 o;
            o.x = *reinterpret_cast<const uint32_t*>(&lo);
            o.y = *reinterpret_cast<const uint32_t*>(&hi);
            reinterpret_cast<uint2*>(out)[i] = o;
        }
    }
}

// K per split: the largest of 2048, 1024, 512, 256 that divides K and still gives at least
// SPLIT_UNITS_TARGET work units (N/128 tiles x K/split), else the smallest that divides K.  A
// function of N and K only (the target is a constant, not the device's SM count), so results do
// not depend on the device.  cfg3 decode (N 7168, K 8192): 2048 -> 224 units.  (Measured there,
// back-to-back calls: 512-K splits 13.9 us, 1024 12.1 us, 2048 11.6 us -- fewer partials.)
constexpr int64_t SPLIT_UNITS_TARGET = 148;
inline int split_k(int64_t N, int64_t K) {
#ifdef GSMALL_SPLIT
    if (K % GSMALL_SPLIT == 0) return GSMALL_SPLIT;
#endif
    const int64_t tiles = N / 128;
    int best = 0;
    for (int ks : {2048, 1024, 512, 256}) {
        if (K % ks) continue;
        best = ks;
        if (tiles * (K / ks) >= SPLIT_UNITS_TARGET) return ks;
    }
    return best;
}

// Persistent grid for `units` equal work units over `slots` resident CTAs: all units at once
// when they fit; else the largest grid <= slots that divides them evenly, when that keeps at least
// 3/4 of the slots busy (e.g. 896 units on 148 slots: 128 CTAs x 7 units, no tail of a few CTAs
// with one unit more); otherwise one CTA per slot.
inline int persistent_grid(int units, int sms) {
    if (units <= sms) return units;
    for (int g = sms; g * 4 >= sms * 3; g--)
        if (units % g == 0) return g;
    return sms;
}

// The in-cluster reduction applies when the splits of an n-tile fit one cluster and divide its
// 128 rows; a function of N and K only.
inline bool in_cluster_reduce(int64_t N, int64_t K) {
    const int ks = split_k(N, K);
    return ks && K / ks <= MAX_CLUSTER_SPLITS && 128 % (K / ks) == 0;
}

// Workspace: the fp32 partials [splits][M][N] of the workspace path (none in-cluster).
inline size_t workspace_bytes(int64_t M, int64_t N, int64_t K) {
    const int ks = split_k(N, K);
    if (!ks || in_cluster_reduce(N, K)) return 0;
    return (size_t)(K / ks) * (size_t)M * (size_t)N * sizeof(float);
}

template <bool kOutF32>
nvfp4_status_t launch(const void* A, const void* sfa, const void* B, const void* sfb, float alpha, void* D,
                      int64_t M, int64_t N, int64_t K, void* ws, size_t ws_bytes, cudaStream_t s, bool b_const = false) {
    const int ks = split_k(N, K);
    if (ks == 0) return fail(NVFP4_ERR_INVALID_ARG, "gemm (small M): K %% 256 != 0");
    if (N % 128 != 0) return fail(NVFP4_ERR_INVALID_ARG, "gemm (small M): N %% 128 != 0");
    if (ws_bytes < workspace_bytes(M, N, K))
        return fail(NVFP4_ERR_INVALID_ARG, "gemm (small M): workspace of %zu bytes, need %zu", ws_bytes,
                    workspace_bytes(M, N, K));
    const int mp = (int)((M + 15) / 16 * 16);
    const int splits = (int)(K / ks);
    CUtensorMap ta, tb;
    nvfp4_status_t st;
    if ((st = make_tmap_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, K / 2, M, K / 2, 128, mp, CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    if ((st = make_tmap_2d(&tb, B, CU_TENSOR_MAP_DATA_TYPE_UINT8, K / 2, N, K / 2, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    const bool in_cluster = in_cluster_reduce(N, K);
    const int smem = smem_bytes(mp, in_cluster);
    // the attribute is set once per device, to the largest footprint of any Mp
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        int most = 0;
        for (int m = 16; m <= 128; m += 16)
            for (int cl = 0; cl < 2; cl++)
                if (smem_bytes(m, cl) > most) most = smem_bytes(m, cl);
        cudaError_t e = cudaFuncSetAttribute(gemm_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, most);
        if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "gemm (small M): smem attribute: %s", cudaGetErrorString(e));
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    const int units = (int)(N / 128) * splits;
    // in-cluster reduction: one CTA per unit, the S splits of an n-tile in one cluster
    const int grid = in_cluster ? units : persistent_grid(units, ctas_per_sm(mp) * sm_count());
    float* w = reinterpret_cast<float*>(ws);
    // Launched as a programmatic dependent of the previous work in the stream (and, in-cluster,
    // with cluster dims (S, 1, 1)).
    cudaLaunchAttribute attrs[2];
    attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[0].val.programmaticStreamSerializationAllowed = 1;
    attrs[1].id = cudaLaunchAttributeClusterDimension;
    attrs[1].val.clusterDim.x = (unsigned)splits;
    attrs[1].val.clusterDim.y = 1;
    attrs[1].val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(THREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attrs;
    cfg.numAttrs = in_cluster ? 2 : 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_small_kernel, ta, tb, reinterpret_cast<const uint8_t*>(sfa),
                                       reinterpret_cast<const uint8_t*>(sfb), w, (int)M, (int)N, (int)K, ks, mp,
                                       b_const ? 1 : 0, in_cluster ? splits : 0, D, alpha, kOutF32 ? 1 : 0);
    if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "gemm_small_kernel: %s", cudaGetErrorString(e));
    if ((st = check_launch("gemm_small_kernel")) || in_cluster) return st;
    const int64_t mn = M * N;
    int64_t rg = (mn / 4 + 255) / 256;
    const int64_t cap = (int64_t)sm_count() * 8;
    if (rg > cap) rg = cap;
    cfg.gridDim = dim3((unsigned)rg, 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.dynamicSmemBytes = 0;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, splitk_reduce_kernel<kOutF32>, (const float*)w, D, mn, splits, alpha);
    if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "splitk_reduce_kernel: %s", cudaGetErrorString(e));
    return check_launch("splitk_reduce_kernel");
}

}  // namespace gsmall
}  // namespace nvfp4
