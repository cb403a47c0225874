// quantize.cu -- bf16 -> NVFP4 quantizer, amax reduction and dequantizer (sm_100a).
//
// Data movement (HBM-bound; algorithmic bytes per element: read 2, write 0.5 packed +
// 0.0625 scale = 2.5625 B):
//   The unit of work is one scale-factor atom: 128 rows x 64 columns.  A persistent CTA
//   (two per SM) streams its atoms' bf16 tiles (128 rows x 128 bytes) into a 6-stage shared
//   memory ring with one 2D TMA load each (SWIZZLE_128B, so the per-row reads below are bank
//   conflict free); a producer warp issues the loads, four consumer warps quantize.
//   Consumer thread t handles row (t % 4) * 32 + t / 4 of the atom, so the 32-bit word of
//   four block scales it produces sits at word t of the 512-byte atom and the warps write
//   the atom with fully coalesced stores; each thread writes its 32 packed bytes with two
//   16-byte stores.  CTAs walk atoms in memory order (k-atom fastest).
//
// Arithmetic (per 16-element block; bit-exact against oracle/nvfp4_oracle.c orc_q16):
//   amax -> s = (amax / 6) * gs_inv -> e4m3(s) -> inv = gs_inv / e4m3(s) -> e2m1(v * inv).
//   Reference: nvfp4_allreduce.cuh:272-290 (q16) and :427-454 (quantize_kernel, which
//   writes a linear scale layout instead of the tcgen05 one).
#include "capi_internal.h"
#include "nvfp4_common.cuh"
#include "tma_host.h"

namespace nvfp4 {

constexpr int QTHREADS = 128;                 // dequantizer CTA
constexpr int QT_STAGES = 6;                  // quantizer ring depth
constexpr int QT_TILE = 128 * 128;            // 128 rows x 64 bf16
constexpr int QT_THREADS = 160;               // warps 0-3 consume, warp 4 loads
constexpr int QT_SMEM = 1024 + QT_STAGES * QT_TILE + 2 * QT_STAGES * 8;
constexpr uint64_t QT_WAIT_NS = 2000000000ull;

// Scale word for one (row, 64-column group): four block scales, kblock j in byte j.
template <bool kDevScale>
__global__ void __launch_bounds__(QT_THREADS)
quantize_kernel(const __grid_constant__ CUtensorMap tmap_x, int64_t rows, int64_t cols, float gs_host,
                const uint32_t* __restrict__ amax_word, float* __restrict__ gs_out,
                uint8_t* __restrict__ packed, uint32_t* __restrict__ sf_words, int64_t units) {
    extern __shared__ uint8_t qsmem_raw[];
    const uint32_t raw_addr = smem_u32(qsmem_raw);
    const uint32_t base = (raw_addr + 1023u) & ~1023u;
    const uint8_t* tiles = qsmem_raw + (base - raw_addr);
    const uint32_t bar0 = base + QT_STAGES * QT_TILE;
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (QT_STAGES + s); };
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t katoms = cols / 64;

    if (warp == 4 && lane == 0) {
        prefetch_tmap(&tmap_x);
        for (int s = 0; s < QT_STAGES; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 128);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    __syncthreads();

    if (warp == 4) {
        // ---------------------------------------------------------------- loads ----
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0, pending = 0;
            bool ok = true;
            for (int64_t u = blockIdx.x; u < units; u += gridDim.x) {
                if (!mbar_wait(empty_bar(stage), phase ^ 1u, QT_WAIT_NS, DEV_TIMEOUT_QUANT)) { ok = false; break; }
                pending &= ~(1u << stage);
                const int64_t rg = u / katoms, kg = u - rg * katoms;
                mbar_arrive_expect_tx(full_bar(stage), QT_TILE);
                tma_load_2d(base + stage * QT_TILE, &tmap_x, (int32_t)(kg * 64), (int32_t)(rg * 128), full_bar(stage));
                pending |= 1u << stage;
                if (++stage == QT_STAGES) { stage = 0; phase ^= 1u; }
            }
            if (!ok)   // never release shared memory with loads still landing in it
                for (int s = 0; s < QT_STAGES; s++)
                    if (pending & (1u << s))
                        mbar_wait(full_bar(s), s < stage ? phase : (phase ^ 1u), QT_WAIT_NS, DEV_TIMEOUT_QUANT);
        }
        __syncwarp();
        return;
    }

    // ------------------------------------------------------------------ consumers ----
    float gs = gs_host, gs_inv;
    if constexpr (kDevScale) {
        global_scale_from_amax(__uint_as_float(*amax_word), gs, gs_inv);
        if (blockIdx.x == 0 && threadIdx.x == 0 && gs_out) *gs_out = gs;
    } else {
        gs_inv = __fdiv_rn(1.0f, gs);
    }
    const int t = threadIdx.x;
    const int r_in_atom = (t & 3) * 32 + (t >> 2);
    int stage = 0;
    uint32_t phase = 0;
#pragma unroll 1
    for (int64_t u = blockIdx.x; u < units; u += gridDim.x) {
        if (!mbar_wait(full_bar(stage), phase, QT_WAIT_NS, DEV_TIMEOUT_QUANT)) break;
        // Row r_in_atom of the tile: 16-byte chunk c sits at chunk c ^ (row % 8) (SWIZZLE_128B).
        const uint8_t* srow = tiles + stage * QT_TILE + r_in_atom * 128;
        uint4 raw[8];
#pragma unroll
        for (int c = 0; c < 8; c++)
            raw[c] = *reinterpret_cast<const uint4*>(srow + ((c ^ (r_in_atom & 7)) << 4));
        // The stage is released only after the values read from it have been consumed (a
        // register dependency): an arrive issued right after the shared-memory loads let the
        // next TMA write overtake them (measured on B200 as rare corrupted rows).
        const uint32_t my_stage = stage;
        if (++stage == QT_STAGES) { stage = 0; phase ^= 1u; }

        const int64_t rg = u / katoms, kg = u - rg * katoms;
        const int64_t row = rg * 128 + r_in_atom;
        uint32_t word = 0;
        if (row < rows) {
            uint32_t nib[8];
#pragma unroll
            for (int b = 0; b < 4; b++) {
                float v[16];
#pragma unroll
                for (int i = 0; i < 2; i++) {
                    const uint32_t w[4] = {raw[2 * b + i].x, raw[2 * b + i].y, raw[2 * b + i].z,
                                           raw[2 * b + i].w};
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        v[i * 8 + 2 * j] = __uint_as_float(w[j] << 16);
                        v[i * 8 + 2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
                    }
                }
                const uint32_t code = q16(v, gs_inv, nib[2 * b], nib[2 * b + 1]);
                word |= code << (8 * b);
            }
            mbar_arrive(empty_bar(my_stage));
            uint8_t* dst = packed + row * (cols / 2) + kg * 32;
            st_v4(dst, make_uint4(nib[0], nib[1], nib[2], nib[3]));
            st_v4(dst + 16, make_uint4(nib[4], nib[5], nib[6], nib[7]));
        }
        else mbar_arrive(empty_bar(my_stage));
        sf_words[u * 128 + t] = word;
    }
}

// Dequantize: same ownership as the quantizer; 32 packed bytes + one scale word in,
// 64 bf16 out.  value = e2m1 * (e4m3(scale) * gs), one rounding for each product.
__global__ void __launch_bounds__(QTHREADS)
dequantize_kernel(const uint8_t* __restrict__ packed, const uint32_t* __restrict__ sf_words,
                  int64_t rows, int64_t cols, float gs, __nv_bfloat16* __restrict__ out,
                  int64_t units) {
    const int64_t katoms = cols / 64;
    const int t = threadIdx.x;
    const int r_in_atom = (t & 3) * 32 + (t >> 2);
#pragma unroll 1
    for (int64_t u = blockIdx.x; u < units; u += gridDim.x) {
        const int64_t rg = u / katoms, kg = u - rg * katoms;
        const int64_t row = rg * 128 + r_in_atom;
        if (row >= rows) continue;
        const uint32_t word = sf_words[u * 128 + t];
        const uint8_t* src = packed + row * (cols / 2) + kg * 32;
        const uint4 p0 = ld_nc_v4(src), p1 = ld_nc_v4(src + 16);
        const uint32_t nib[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
        uint8_t* dst = reinterpret_cast<uint8_t*>(out + row * cols + kg * 64);
#pragma unroll
        for (int b = 0; b < 4; b++) {
            const float bs = __fmul_rn(e4m3_decode((word >> (8 * b)) & 0xFFu), gs);
#pragma unroll
            for (int h = 0; h < 2; h++) {
                float v[8];
                e2m1x8_decode(nib[2 * b + h], v);
                uint32_t o[4];
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const __nv_bfloat162 pr =
                        __floats2bfloat162_rn(__fmul_rn(v[2 * j], bs), __fmul_rn(v[2 * j + 1], bs));
                    o[j] = *reinterpret_cast<const uint32_t*>(&pr);
                }
                st_v4(dst + (2 * b + h) * 16, make_uint4(o[0], o[1], o[2], o[3]));
            }
        }
    }
}

// max |x| of bf16 data, accumulated with atomicMax on the float bit pattern (non-negative
// floats order like their bit patterns).  *out must be zero before the launch.
__global__ void __launch_bounds__(256)
amax_kernel(const uint4* __restrict__ x, int64_t nvec, uint32_t* __restrict__ out) {
    uint32_t m = 0;
#pragma unroll 1
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec;
         i += (int64_t)gridDim.x * blockDim.x) {
        const uint4 v = ld_nc_v4(x + i);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; j++) {
            m = max(m, w[j] & 0x7FFFu);
            m = max(m, (w[j] >> 16) & 0x7FFFu);
        }
    }
    m = __reduce_max_sync(0xFFFFFFFFu, m);
    __shared__ uint32_t warp_max[8];
    if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        m = threadIdx.x < (blockDim.x >> 5) ? warp_max[threadIdx.x] : 0u;
        m = __reduce_max_sync(0xFFFFFFFFu, m);
        if (threadIdx.x == 0 && m != 0) atomicMax(out, m << 16);
    }
}

static int quant_grid(int64_t units) {
    const int64_t cap = (int64_t)sm_count() * 16;
    return (int)(units < cap ? units : cap);
}

// Launch the TMA quantizer (kDevScale: the global scale comes from *amax_word).
template <bool kDevScale>
static nvfp4_status_t launch_quantize(const void* x, int64_t rows, int64_t cols, float gs, const uint32_t* amax_word,
                                      float* gs_out, void* packed, void* sf, cudaStream_t s) {
    const int64_t units = ((rows + 127) / 128) * (cols / 64);
    if (units == 0) return NVFP4_OK;
    CUtensorMap tm;
    nvfp4_status_t st = make_tmap_2d(&tm, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, cols, rows, cols * 2, 64, 128,
                                     CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != NVFP4_OK) return st;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(quantize_kernel<kDevScale>, cudaFuncAttributeMaxDynamicSharedMemorySize, QT_SMEM);
        if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "quantize: smem attribute: %s", cudaGetErrorString(e));
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    const int64_t cap = (int64_t)sm_count() * 2;
    const int grid = (int)(units < cap ? units : cap);
    quantize_kernel<kDevScale><<<grid, QT_THREADS, QT_SMEM, s>>>(tm, rows, cols, gs, amax_word, gs_out,
                                                                reinterpret_cast<uint8_t*>(packed),
                                                                reinterpret_cast<uint32_t*>(sf), units);
    return check_launch("quantize_kernel");
}

static nvfp4_status_t launch_amax(const void* x, int64_t numel, uint32_t* word, cudaStream_t s) {
    cudaError_t e = cudaMemsetAsync(word, 0, sizeof(uint32_t), s);
    if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "amax memset: %s", cudaGetErrorString(e));
    const int64_t nvec = numel / 8;
    if (nvec == 0) return NVFP4_OK;
    int64_t grid = (nvec + 255) / 256;
    const int64_t cap = (int64_t)sm_count() * 8;
    if (grid > cap) grid = cap;
    amax_kernel<<<(unsigned)grid, 256, 0, s>>>(reinterpret_cast<const uint4*>(x), nvec, word);
    return check_launch("amax_kernel");
}

static nvfp4_status_t check_quant_args(const char* who, const void* x, int64_t rows, int64_t cols,
                                       const void* packed, const void* sf) {
    if (!x || !packed || !sf) return fail(NVFP4_ERR_INVALID_ARG, "%s: null pointer", who);
    if (rows < 0 || cols < 0) return fail(NVFP4_ERR_INVALID_ARG, "%s: negative shape", who);
    if (cols % 64 != 0)
        return fail(NVFP4_ERR_INVALID_ARG, "%s: cols=%lld must be a multiple of 64", who, (long long)cols);
    if (!aligned16(x) || !aligned16(packed) || !aligned16(sf))
        return fail(NVFP4_ERR_INVALID_ARG, "%s: buffers must be 16-byte aligned", who);
    return NVFP4_OK;
}

}  // namespace nvfp4

using namespace nvfp4;

extern "C" {

nvfp4_status_t nvfp4_amax_bf16(const void* x, int64_t numel, float* amax_dev, void* stream) {
    clear_error();
    if (!x || !amax_dev || numel < 0) return fail(NVFP4_ERR_INVALID_ARG, "amax: bad arguments");
    if (numel % 8 != 0 || !aligned16(x))
        return fail(NVFP4_ERR_INVALID_ARG, "amax: numel %% 8 == 0 and 16-byte alignment required");
    return launch_amax(x, numel, reinterpret_cast<uint32_t*>(amax_dev), (cudaStream_t)stream);
}

nvfp4_status_t nvfp4_quantize_bf16(const void* x, int64_t rows, int64_t cols, float global_scale,
                                   void* packed, void* sf, void* stream) {
    clear_error();
    nvfp4_status_t st = check_quant_args("quantize", x, rows, cols, packed, sf);
    if (st != NVFP4_OK) return st;
    if (!(global_scale > 0.0f) || !isfinite(global_scale))
        return fail(NVFP4_ERR_INVALID_ARG, "quantize: global_scale must be finite and > 0");
    return launch_quantize<false>(x, rows, cols, global_scale, nullptr, nullptr, packed, sf, (cudaStream_t)stream);
}

size_t nvfp4_quantize_workspace_bytes(void) { return 256; }

nvfp4_status_t nvfp4_quantize_bf16_auto(const void* x, int64_t rows, int64_t cols, void* packed,
                                        void* sf, float* global_scale_dev, void* workspace,
                                        void* stream) {
    clear_error();
    nvfp4_status_t st = check_quant_args("quantize_auto", x, rows, cols, packed, sf);
    if (st != NVFP4_OK) return st;
    if (!workspace || !aligned16(workspace))
        return fail(NVFP4_ERR_INVALID_ARG, "quantize_auto: workspace must be a 16-byte aligned device buffer");
    cudaStream_t s = (cudaStream_t)stream;
    uint32_t* word = reinterpret_cast<uint32_t*>(workspace);
    st = launch_amax(x, rows * cols, word, s);
    if (st != NVFP4_OK) return st;
    return launch_quantize<true>(x, rows, cols, 1.0f, word, global_scale_dev, packed, sf, s);
}

nvfp4_status_t nvfp4_dequantize_bf16(const void* packed, const void* sf, int64_t rows, int64_t cols,
                                     float global_scale, void* out, void* stream) {
    clear_error();
    nvfp4_status_t st = check_quant_args("dequantize", out, rows, cols, packed, sf);
    if (st != NVFP4_OK) return st;
    const int64_t units = ((rows + 127) / 128) * (cols / 64);
    if (units == 0) return NVFP4_OK;
    dequantize_kernel<<<quant_grid(units), QTHREADS, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<const uint8_t*>(packed), reinterpret_cast<const uint32_t*>(sf), rows, cols,
        global_scale, reinterpret_cast<__nv_bfloat16*>(out), units);
    return check_launch("dequantize_kernel");
}

}  // extern "C"
