// quantize.cu -- bf16 -> NVFP4 quantizer, amax reduction and dequantizer (sm_100a).
//
// Data movement (HBM-bound; algorithmic bytes per element: read 2, write 0.5 packed +
// 0.0625 scale = 2.5625 B):
//   The tensor is swept in flat element order, one 16-element block per thread: lane l of a
//   warp reads bytes [32 l, 32 l + 32) of a 1 KB stretch (one 32-byte load) and writes the
//   block's 8 packed bytes (a warp writes 256 contiguous bytes), so at any moment the grid
//   reads one contiguous stretch of memory.  Each thread has QR_UNROLL blocks (64 bytes) of
//   loads in flight before any arithmetic.  The 4 lanes of one row's 64-column group assemble
//   the 32-bit word of their four block scales and the first of them stores it at its place in
//   the tcgen05 layout; (row, column) are tracked incrementally, without divisions.
//   Measured against the alternatives on B200 (cfg2, 8192 x 7168): a 128 x 64 TMA-tile ring
//   read at ~4 TB/s even with the arithmetic and stores removed (38 us in all), 8 elements per
//   thread (a block split across a lane pair) doubled the per-element arithmetic (51-67 us);
//   this kernel: ~37 us with 2 blocks in flight per thread (4 or 8 were slower).
//
// Arithmetic (per 16-element block; bit-exact against oracle/nvfp4_oracle.c orc_q16):
//   amax -> s = (amax * fp32(1/6)) * gs_inv -> e4m3(s) -> inv = gs_inv * rcp(e4m3(s))
//   -> e2m1(v * inv), every step one correctly rounded IEEE operation.
//   Reference: nvfp4_allreduce.cuh:272-290 (q16) and :427-454 (quantize_kernel, which
//   writes a linear scale layout instead of the tcgen05 one).
#include "capi_internal.h"
#include "nvfp4_common.cuh"

namespace nvfp4 {

constexpr int QR_THREADS = 256;               // quantizer CTA
#ifndef QUANT_UNROLL
#define QUANT_UNROLL 2
#endif
#ifndef QUANT_CTAS_PER_SM
#define QUANT_CTAS_PER_SM 4
#endif
constexpr int QR_UNROLL = QUANT_UNROLL;       // 16-element blocks (32 bytes) in flight per thread

template <bool kDevScale, bool kLoad32>
__global__ void __launch_bounds__(QR_THREADS)
quantize_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows, int64_t cols, float gs_host,
                const uint32_t* __restrict__ amax_word, float* __restrict__ gs_out, uint8_t* __restrict__ packed,
                uint8_t* __restrict__ sf) {
    // Programmatic dependent launch.  Given scale: the input may come from the kernel before
    // this one, so wait for it first.  Device scale: this kernel follows the amax kernel, whose
    // input is the same x (complete before the amax kernel started); the first loads are issued
    // before the wait and only the amax word is read after it.
    float gs = gs_host, gs_inv = 0.0f;
    bool have_scale = !kDevScale;
    if constexpr (!kDevScale) {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        gs_inv = __fdiv_rn(1.0f, gs);
    }
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    auto fetch_scale = [&]() {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        global_scale_from_amax(__uint_as_float(*reinterpret_cast<const volatile uint32_t*>(amax_word)), gs, gs_inv);
        if (blockIdx.x == 0 && threadIdx.x == 0 && gs_out) *gs_out = gs;
        have_scale = true;
    };
    const int lane = threadIdx.x & 31;
    const int64_t katoms = cols / 64;
    const int64_t nblocks = rows * cols / 16;
    const int64_t step = (int64_t)gridDim.x * QR_THREADS;    // blocks between a thread's loads
    // (row, col) of this thread's block, tracked incrementally (no division in the loop)
    const int64_t e_step = step * 16;
    const int64_t dr = e_step / cols, dc = e_step - dr * cols;
    int64_t b0 = (int64_t)blockIdx.x * QR_THREADS + threadIdx.x;
    int64_t row = (b0 * 16) / cols, col = b0 * 16 - row * cols;
    const uint8_t* xb = reinterpret_cast<const uint8_t*>(x);
#pragma unroll 1
    for (; b0 - lane < nblocks; b0 += step * QR_UNROLL) {
        uint32_t raw[QR_UNROLL][8];
#pragma unroll
        for (int i = 0; i < QR_UNROLL; i++) {
            const int64_t b = b0 + i * step;
            if (b < nblocks) {
                if constexpr (kLoad32) {
                    ld_nc_v8(xb + b * 32, raw[i]);          // one 32-byte load per block
                } else {
                    const uint4 lo = ld_nc_v4(xb + b * 32), hi = ld_nc_v4(xb + b * 32 + 16);
                    raw[i][0] = lo.x; raw[i][1] = lo.y; raw[i][2] = lo.z; raw[i][3] = lo.w;
                    raw[i][4] = hi.x; raw[i][5] = hi.y; raw[i][6] = hi.z; raw[i][7] = hi.w;
                }
            } else {
#pragma unroll
                for (int j = 0; j < 8; j++) raw[i][j] = 0u;
            }
        }
        if constexpr (kDevScale)
            if (!have_scale) fetch_scale();
#pragma unroll
        for (int i = 0; i < QR_UNROLL; i++) {
            const int64_t b = b0 + i * step;
            uint32_t n0, n1;
            const uint32_t code = q16_bf16(raw[i], gs_inv, n0, n1);
            const uint32_t c1 = __shfl_down_sync(0xFFFFFFFFu, code, 1);
            const uint32_t c2 = __shfl_down_sync(0xFFFFFFFFu, code, 2);
            const uint32_t c3 = __shfl_down_sync(0xFFFFFFFFu, code, 3);
            if (b < nblocks) {
                *reinterpret_cast<uint2*>(packed + b * 8) = make_uint2(n0, n1);
                if ((lane & 3) == 0) {                // first block of a row's 64-column group
                    const int64_t off = ((row >> 7) * katoms + (col >> 6)) * 512 + (row & 31) * 16 + ((row >> 5) & 3) * 4;
                    *reinterpret_cast<uint32_t*>(sf + off) = code | (c1 << 8) | (c2 << 16) | (c3 << 24);
                }
            }
            row += dr;
            col += dc;
            if (col >= cols) { col -= cols; row++; }
        }
    }
    if constexpr (kDevScale)
        if (!have_scale) fetch_scale();
}

// Scale words of the padding rows of the last 128-row group (rows .. ceil(rows/128)*128 - 1):
// zero, as the layout requires for rows that do not exist.
__global__ void sf_pad_kernel(uint8_t* __restrict__ sf, int64_t rows, int64_t cols) {
    const int64_t katoms = cols / 64;
    const int64_t rg = rows >> 7;
    const int64_t pad = (rg + 1) * 128 - rows;   // 1..127 (only launched when rows % 128 != 0)
    const int64_t n = pad * katoms;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = rows + i / katoms, ka = i % katoms;
        const int64_t off = (rg * katoms + ka) * 512 + (row & 31) * 16 + ((row >> 5) & 3) * 4;
        *reinterpret_cast<uint32_t*>(sf + off) = 0u;
    }
}

// Dequantize (the cfg2 round trip): the quantizer's flat sweep in reverse, one 16-element block
// per thread and DQ_UNROLL blocks in flight: lane l of a warp reads bytes [8 l, 8 l + 8) of a
// 256-byte stretch of codes and writes 32 contiguous bytes of bf16, so a warp reads and writes
// contiguous memory; the four lanes of one row's 64-column group read the same scale word (one
// transaction) and take their byte of it.  HBM-bound: 0.5625 B/elt read, 2 B/elt written.
//   value = bf16(e2m1 * (e4m3(scale) * gs)), one rounding for each product.
constexpr int DQ_THREADS = 256;
constexpr int DQ_UNROLL = 8;

template <bool kStore32>
__global__ void __launch_bounds__(DQ_THREADS)
dequantize_kernel(const uint8_t* __restrict__ packed, const uint8_t* __restrict__ sf, int64_t rows, int64_t cols,
                  float gs, __nv_bfloat16* __restrict__ out) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int64_t katoms = cols / 64;
    const int64_t nblocks = rows * cols / 16;
    const int64_t step = (int64_t)gridDim.x * DQ_THREADS;
    const int64_t e_step = step * 16;
    const int64_t dr = e_step / cols, dc = e_step - dr * cols;
    int64_t b0 = (int64_t)blockIdx.x * DQ_THREADS + threadIdx.x;
    int64_t row = (b0 * 16) / cols, col = b0 * 16 - row * cols;
#pragma unroll 1
    for (; b0 < nblocks; b0 += step * DQ_UNROLL) {
        uint2 code[DQ_UNROLL];
        uint32_t word[DQ_UNROLL];
        int64_t c[DQ_UNROLL];
#pragma unroll
        for (int i = 0; i < DQ_UNROLL; i++) {
            const int64_t b = b0 + i * step;
            c[i] = col;
            if (b < nblocks) {
                asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];"
                             : "=r"(code[i].x), "=r"(code[i].y)
                             : "l"(packed + b * 8));
                const int64_t off = ((row >> 7) * katoms + (col >> 6)) * 512 + (row & 31) * 16 + ((row >> 5) & 3) * 4;
                word[i] = __ldg(reinterpret_cast<const uint32_t*>(sf + off));
            }
            row += dr;
            col += dc;
            if (col >= cols) { col -= cols; row++; }
        }
#pragma unroll
        for (int i = 0; i < DQ_UNROLL; i++) {
            const int64_t b = b0 + i * step;
            if (b >= nblocks) break;
            const uint32_t kb = (uint32_t)(c[i] >> 4) & 3u;
            const float bs = __fmul_rn(e4m3_decode((word[i] >> (8 * kb)) & 0xFFu), gs);
            uint32_t o[8];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                float v[8];
                e2m1x8_decode(h ? code[i].y : code[i].x, v);
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const __nv_bfloat162 pr = __floats2bfloat162_rn(__fmul_rn(v[2 * j], bs), __fmul_rn(v[2 * j + 1], bs));
                    o[4 * h + j] = *reinterpret_cast<const uint32_t*>(&pr);
                }
            }
            uint8_t* dst = reinterpret_cast<uint8_t*>(out) + b * 32;
            if constexpr (kStore32) {
                st_global_v8(dst, o);                       // one 32-byte store
            } else {
                st_v4(dst, make_uint4(o[0], o[1], o[2], o[3]));
                st_v4(dst + 16, make_uint4(o[4], o[5], o[6], o[7]));
            }
        }
    }
}

// max |x| over the finite bf16 values, accumulated with atomicMax on the bit pattern (non-negative
// floats order like their bit patterns).  *out must be zero before the launch.
//   HBM-bound: 2 bytes per element read once.  At B200 bandwidth an SM must retire ~5.6 32-bit
//   words per cycle, so the loop spends one instruction per word: max.NaN.xorsign.abs.bf16x2
//   folds a word into the running pair-maximum (magnitudes; NaN propagates), with 32-byte loads
//   (AMAX_UNROLL of them in flight per thread before any arithmetic).
//   Non-finite values: a NaN or Inf leaves a magnitude >= 0x7F80 in the running maximum; only
//   then does the thread walk its elements again, skipping NaN and Inf, and record
//   DEV_NONFINITE_INPUT, so the result is the amax of the finite values.
constexpr int AMAX_THREADS = 256;
constexpr int AMAX_UNROLL = 4;

__device__ __forceinline__ uint32_t amax_fold(uint32_t m, uint32_t w) {
    asm("max.NaN.xorsign.abs.bf16x2 %0, %0, %1;" : "+r"(m) : "r"(w));
    return m;
}
// larger of the two magnitudes of a pair, skipping NaN and Inf (>= 0x7F80)
__device__ __forceinline__ uint32_t finite_max2(uint32_t m, uint32_t w) {
    const uint32_t lo = w & 0x7FFFu, hi = (w >> 16) & 0x7FFFu;
    if (lo < 0x7F80u && lo > m) m = lo;
    if (hi < 0x7F80u && hi > m) m = hi;
    return m;
}

template <bool kLoad32>
__global__ void __launch_bounds__(AMAX_THREADS)
amax_kernel(const uint8_t* __restrict__ x, int64_t numel, uint32_t* __restrict__ out) {
    constexpr int VB = kLoad32 ? 32 : 16;                  // bytes per load
    constexpr int VW = VB / 4;                             // words per load
    // Launched as a programmatic dependent of amax_zero_kernel, which started only after all
    // earlier work in the stream completed: x is ready; the zeroed output is waited for below.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int64_t nvec = numel * 2 / VB;
    const int64_t stride = (int64_t)gridDim.x * AMAX_THREADS;
    const int64_t first = (int64_t)blockIdx.x * AMAX_THREADS + threadIdx.x;
    uint32_t m = 0;
#pragma unroll 1
    for (int64_t i = first; i < nvec; i += stride * AMAX_UNROLL) {
        uint32_t r[AMAX_UNROLL][VW];
#pragma unroll
        for (int u = 0; u < AMAX_UNROLL; u++) {
            const int64_t v = i + u * stride;
            if (v < nvec) {
                if constexpr (kLoad32) {
                    ld_nc_v8(x + v * VB, r[u]);
                } else {
                    const uint4 q = ld_nc_v4(x + v * VB);
                    r[u][0] = q.x; r[u][1] = q.y; r[u][2] = q.z; r[u][3] = q.w;
                }
            } else {
#pragma unroll
                for (int j = 0; j < VW; j++) r[u][j] = 0u;
            }
        }
#pragma unroll
        for (int u = 0; u < AMAX_UNROLL; u++)
#pragma unroll
            for (int j = 0; j < VW; j++) m = amax_fold(m, r[u][j]);
    }
    // a tail of 8 elements when numel is not a multiple of VB / 2
    const int64_t tail = nvec * VB;
    if (first == 0 && tail < numel * 2) {
        const uint4 q = ld_nc_v4(x + tail);
        m = amax_fold(amax_fold(amax_fold(amax_fold(m, q.x), q.y), q.z), q.w);
    }
    m &= 0x7FFF7FFFu;
    uint32_t a = max(m & 0xFFFFu, m >> 16);
    if (a >= 0x7F80u) {
        // rare path: this thread saw a NaN or Inf; walk its elements again without them
        record_error(DEV_NONFINITE_INPUT);
        a = 0;
#pragma unroll 1
        for (int64_t v = first; v < nvec; v += stride) {
            const uint32_t* p = reinterpret_cast<const uint32_t*>(x + v * VB);
#pragma unroll
            for (int j = 0; j < VW; j++) a = finite_max2(a, p[j]);
        }
        if (first == 0 && tail < numel * 2) {
            const uint32_t* p = reinterpret_cast<const uint32_t*>(x + tail);
            for (int j = 0; j < 4; j++) a = finite_max2(a, p[j]);
        }
    }
    a = __reduce_max_sync(0xFFFFFFFFu, a);
    __shared__ uint32_t warp_max[AMAX_THREADS / 32];
    if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = a;
    __syncthreads();
    if (threadIdx.x < 32) {
        a = threadIdx.x < AMAX_THREADS / 32 ? warp_max[threadIdx.x] : 0u;
        a = __reduce_max_sync(0xFFFFFFFFu, a);
        if (threadIdx.x == 0) {
            asm volatile("griddepcontrol.wait;" ::: "memory");      // the output word is zero
            if (a != 0) atomicMax(out, a << 16);
        }
    }
}

// Zeroes the amax word; the amax kernel is launched as its programmatic dependent, so its launch
// and loads overlap this one-thread kernel instead of queueing behind a memset.
__global__ void amax_zero_kernel(uint32_t* __restrict__ out) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (threadIdx.x == 0) *out = 0u;
}

// cudaLaunchKernelEx with programmatic stream serialization (no dynamic shared memory).
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kernel)(KArgs...), unsigned grid, unsigned block, cudaStream_t s, Args... args) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(block, 1, 1);
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Launch the quantizer (kDevScale: the global scale comes from *amax_word).
template <bool kDevScale>
static nvfp4_status_t launch_quantize(const void* x, int64_t rows, int64_t cols, float gs, const uint32_t* amax_word,
                                      float* gs_out, void* packed, void* sf, cudaStream_t s) {
    const int64_t nblocks = rows * cols / 16;
    // an empty tensor still gets its global scale written on the auto-scaled path (gs 1 from
    // amax 0): one block runs, with no element to quantize
    if (nblocks == 0 && !kDevScale) return NVFP4_OK;
    const int64_t per_cta = (int64_t)QR_THREADS * QR_UNROLL;
    const int64_t cap = (int64_t)sm_count() * QUANT_CTAS_PER_SM;
    int64_t grid = (nblocks + per_cta - 1) / per_cta;
    if (grid > cap) grid = cap;
    if (grid < 1) grid = 1;
    // 32-byte loads when the input allows them (16-byte alignment is the API's minimum); a
    // programmatic dependent launch (the kernel waits before it reads what earlier work wrote)
    const auto* xp = reinterpret_cast<const __nv_bfloat16*>(x);
    auto* pp = reinterpret_cast<uint8_t*>(packed);
    auto* sp = reinterpret_cast<uint8_t*>(sf);
    const cudaError_t e = ((reinterpret_cast<uintptr_t>(x) & 31) == 0)
        ? launch_pdl(quantize_kernel<kDevScale, true>, (unsigned)grid, QR_THREADS, s, xp, rows, cols, gs, amax_word, gs_out, pp, sp)
        : launch_pdl(quantize_kernel<kDevScale, false>, (unsigned)grid, QR_THREADS, s, xp, rows, cols, gs, amax_word, gs_out, pp, sp);
    if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "quantize_kernel: %s", cudaGetErrorString(e));
    nvfp4_status_t st = check_launch("quantize_kernel");
    if (st != NVFP4_OK || rows % 128 == 0) return st;
    sf_pad_kernel<<<64, 256, 0, s>>>(reinterpret_cast<uint8_t*>(sf), rows, cols);
    return check_launch("sf_pad_kernel");
}

static nvfp4_status_t launch_amax(const void* x, int64_t numel, uint32_t* word, cudaStream_t s) {
    amax_zero_kernel<<<1, 32, 0, s>>>(word);
    nvfp4_status_t st = check_launch("amax_zero_kernel");
    if (st != NVFP4_OK || numel == 0) return st;
    const bool load32 = (reinterpret_cast<uintptr_t>(x) & 31) == 0;
    const int64_t per_cta = (int64_t)AMAX_THREADS * AMAX_UNROLL * (load32 ? 16 : 8);   // elements
    int64_t grid = (numel + per_cta - 1) / per_cta;
    const int64_t cap = (int64_t)sm_count() * 8;
    if (grid > cap) grid = cap;
    if (grid < 1) grid = 1;
    const auto* xb = reinterpret_cast<const uint8_t*>(x);
    const cudaError_t e = load32 ? launch_pdl(amax_kernel<true>, (unsigned)grid, AMAX_THREADS, s, xb, numel, word)
                                 : launch_pdl(amax_kernel<false>, (unsigned)grid, AMAX_THREADS, s, xb, numel, word);
    if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "amax_kernel: %s", cudaGetErrorString(e));
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
    const int64_t nblocks = rows * cols / 16;
    if (nblocks == 0) return NVFP4_OK;
    int64_t grid = (nblocks + (int64_t)DQ_THREADS * DQ_UNROLL - 1) / ((int64_t)DQ_THREADS * DQ_UNROLL);
    const int64_t cap = (int64_t)sm_count() * 8;
    if (grid > cap) grid = cap;
    const auto* pk = reinterpret_cast<const uint8_t*>(packed);
    const auto* sp = reinterpret_cast<const uint8_t*>(sf);
    auto* op = reinterpret_cast<__nv_bfloat16*>(out);
    const cudaError_t e =
        ((reinterpret_cast<uintptr_t>(out) & 31) == 0)
            ? launch_pdl(dequantize_kernel<true>, (unsigned)grid, DQ_THREADS, (cudaStream_t)stream, pk, sp, rows, cols,
                         global_scale, op)
            : launch_pdl(dequantize_kernel<false>, (unsigned)grid, DQ_THREADS, (cudaStream_t)stream, pk, sp, rows, cols,
                         global_scale, op);
    if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "dequantize_kernel: %s", cudaGetErrorString(e));
    return check_launch("dequantize_kernel");
}

}  // extern "C"
