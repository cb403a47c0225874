// allreduce.cu -- NVFP4-compressed all-reduce over NVLink / NVSwitch peer memory (sm_100a), and
// the in-house bf16 peer-to-peer all-reduce it is measured against.
//
// One context per rank (one GPU each).  A context owns one device allocation, exported to the
// other ranks (CUDA IPC between processes, or plain peer pointers inside one process):
//   [flags: u32 [AR_MAX_BLOCKS][AR_MAX_WORLD]] [parity 0 region] [parity 1 region]
//   [low-latency area: parity 0, parity 1, each [world][ll_slot]]
//   region = IN [world][in_slot] + GATHER [world][gather_slot]
// Calls alternate parities, so back-to-back calls never write the region a slower rank may
// still be reading.  Every call carries an epoch; barrier flags only grow (2 per call), so they
// are never reset.
//
// NVFP4 payload of n elements: packed E2M1 (n/2 bytes, element 2j in the low nibble of byte j)
// followed, 16-byte aligned, by one UE4M3 scale per 16 elements.  One thread handles a chunk of
// 32 elements: 64 bytes of bf16 in, 16 bytes packed + 2 bytes of scales out; a warp stores 512
// contiguous packed bytes and 64 contiguous scale bytes per chunk row, to local or peer memory.
//
// Data flow (reference: twoshot_fused_kernel / oneshot_fused_kernel,
// blackwell/allreduce_sm100_sm120/nvfp4_allreduce.cuh:498-619):
//   one-shot  A: quantize the whole input once (gs), push the payload into IN[me] of every rank;
//             barrier; B: out = bf16(sum over ranks 0..n-1 of dequant(IN[s])).
//   two-shot  A: quantize shard o of the input, push it into IN[me] of owner o; barrier;
//             B: owner sums IN[0..n-1] of its shard in rank order, requantizes with gs * n and
//             pushes the result into GATHER[me] of every rank; barrier;
//             C: out = bf16(dequant(GATHER[o])) for every owner o.
//             Two kernels run it: a grid-stride one (a thread takes one chunk and all n shards of
//             it) and, for small shards, one whose threads split the (shard, chunk) pairs of their
//             block's chunk group; both give the same bits.
//   Sums are fp32 fma(code, scale * gs, acc) in rank order 0..n-1 (the reference sums in a
//   rank-rotated order, :515-518); only the order of the pushes is rotated (rank me+1 first) so
//   that the ranks do not all target the same peer at once.
//
// Low-latency one-shot (small messages): the barrier is replaced by flags carried in the data,
// as in NCCL's LL protocol.  Every 8-byte word a rank pushes holds 7 bytes of payload and a
// non-zero tag byte; 64-bit stores and loads are single-copy atomic, so a reader that sees the
// tag in a word also sees that word's payload, and no fence or barrier is needed.  A chunk of 32
// elements (16 code bytes + 2 scale bytes) is 3 words, stored word-major ([3][chunks] u64) so a
// warp's stores cover 256 contiguous bytes.  The reader zeroes each word after reading it, so
// between calls the area is all zero: the next write to a word comes from a call of the same
// parity, which no peer starts before this rank has finished the current call (it needs this
// rank's data of the call in between).  A word with a tag therefore always belongs to the
// current call.
//
// NVLS bf16 all-reduce (NVFP4_AR_NVLS, bf16 payloads only): the sum is done inside the NVSwitch.
// Every rank has bound one buffer to an NVLink multicast object (registered with
// nvfp4_ar_set_multicast: its multicast address and this rank's unicast address).  A: copy the
// input into this rank's buffer (unicast); barrier; B: for the chunks of this rank's shard,
// multimem.ld_reduce.add.acc::f32 through the multicast address returns the fp32 sum over every
// rank's buffer (rounded once to bf16) and multimem.st writes it back to every rank's buffer;
// barrier; C: copy the buffer to the output.  On the wire each GPU sends and receives about
// 2 (n-1)/n x 2 bytes per element.  The switch fixes the order of the fp32 additions, not this
// code, so results are checked against the exact sum within a tolerance, not bit for bit.
// The buffer has two parity halves, alternated per call like the P2P regions.
//
// Synchronisation: block b of every rank handles the same chunks in every phase, so a phase
// only needs block b of every rank to have finished the previous phase: after its pushes block
// b does __syncthreads and stores the barrier value into flag [b][me] of every rank with
// st.release.sys; then thread s waits (ld.acquire.sys, bounded by the context's time limit)
// for flag [b][s] of its own rank.  A wait that runs out records DEV_TIMEOUT_AR_BARRIER in the
// device status word and the block skips the rest of the call; nothing traps.  The grid never
// exceeds the number of blocks that are resident at once, so every block's peer blocks run.
#include <cmath>
#include <cstring>
#include <mutex>

#include "capi_internal.h"
#include "nvfp4_common.cuh"

namespace nvfp4 {
namespace ar {

constexpr int AR_MAX_WORLD = 8;
constexpr int AR_MAX_BLOCKS = 1024;
constexpr int AR_THREADS = 512;
constexpr size_t AR_FLAG_BYTES = sizeof(uint32_t) * AR_MAX_BLOCKS * AR_MAX_WORLD;
constexpr uint64_t AR_DEFAULT_TIMEOUT_NS = 5000000000ull;

__host__ __device__ constexpr int64_t align16(int64_t x) { return (x + 15) & ~(int64_t)15; }
// Bytes of the NVFP4 payload of n elements (packed, then scales).
__host__ __device__ constexpr int64_t payload_bytes(int64_t n) { return align16(n / 2) + align16(n / 16); }

struct Params {
    uint8_t* comm[AR_MAX_WORLD];     // every rank's allocation base (own included)
    const __nv_bfloat16* in;
    __nv_bfloat16* out;
    int64_t numel;
    int64_t in_slot;                 // bytes of one IN slot
    int64_t gather_slot;             // bytes of one GATHER slot
    int64_t region;                  // bytes of one parity region
    int world, rank;
    uint32_t epoch;
    float gs;                        // global scale of the inputs (gs = amax / (6 * 448))
    uint64_t timeout_ns;
    int phase;                       // -1: all phases with barriers; 0/1/2: that phase alone;
                                     // -3 / 3: two-shot with phase 0 pushing already quantized
                                     // data (all phases / that phase alone)
    const uint8_t* q_codes;          // phase 0 from quantized data: codes [numel / 2] and scales
    const uint8_t* q_scales;         // [numel / 16] of the whole input, flat
    int64_t ll_off;                  // byte offset of the low-latency area in every rank's buffer
    int64_t ll_slot;                 // bytes of one low-latency slot
    uint8_t* nvls_mc;                // NVLS: multicast address of this call's parity half
    uint8_t* nvls_uc;                // NVLS: this rank's unicast address of the same half
};

__device__ __forceinline__ uint32_t* flags_of(const Params& p, int r) {
    return reinterpret_cast<uint32_t*>(p.comm[r]);
}
__device__ __forceinline__ uint8_t* region_of(const Params& p, int r) {
    return p.comm[r] + AR_FLAG_BYTES + (int64_t)(p.epoch & 1u) * p.region;
}
__device__ __forceinline__ uint8_t* in_slot(const Params& p, int r, int s) {
    return region_of(p, r) + (int64_t)s * p.in_slot;
}
__device__ __forceinline__ uint8_t* gather_slot(const Params& p, int r, int o) {
    return region_of(p, r) + (int64_t)p.world * p.in_slot + (int64_t)o * p.gather_slot;
}

// Low-latency slot of source rank s in rank r's buffer, for this call's parity.
__device__ __forceinline__ uint64_t* ll_slot_of(const Params& p, int r, int s) {
    return reinterpret_cast<uint64_t*>(p.comm[r] + p.ll_off +
                                       ((int64_t)(p.epoch & 1u) * p.world + s) * p.ll_slot);
}
__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* ptr, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(ptr), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* ptr) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(ptr) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* ptr, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* ptr) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
    return v;
}
// 16-byte load that bypasses L1 (the data was written by other GPUs during this kernel).
__device__ __forceinline__ uint4 ld_cg_v4(const void* ptr) {
    uint4 r;
    asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(ptr));
    return r;
}
__device__ __forceinline__ uint16_t ld_cg_u16(const void* ptr) {
    uint16_t r;
    asm volatile("ld.global.cg.u16 %0, [%1];" : "=h"(r) : "l"(ptr));
    return r;
}

// Block b of this rank meets block b of every rank.  Returns false (for the whole block) if a
// wait ran out.
__device__ bool block_barrier(const Params& p, uint32_t value) {
    __syncthreads();
    const int t = threadIdx.x;
    const int64_t slot = (int64_t)blockIdx.x * AR_MAX_WORLD;
    if (t < p.world) st_release_sys(flags_of(p, t) + slot + p.rank, value);
    bool ok = true;
    if (t < p.world) {
        const uint32_t* f = flags_of(p, p.rank) + slot + t;
        int spins = 0;
        uint64_t t0 = 0;
        while ((int32_t)(ld_acquire_sys(f) - value) < 0) {
            if (++spins == 64) t0 = globaltimer_ns();
            if (spins > 64 && (spins & 63) == 0 && globaltimer_ns() - t0 > p.timeout_ns) {
                record_error(DEV_TIMEOUT_AR_BARRIER);
                ok = false;
                break;
            }
        }
    }
    return __syncthreads_and(ok) != 0;
}

// ---------------------------------------------------------------- NVFP4 codec ----
// 32 bf16 values at x (16-byte aligned) -> 16 packed bytes + 2 scale bytes (block 0 low byte); the
// four 16-byte loads are issued before any arithmetic.
__device__ __forceinline__ void quant32(const __nv_bfloat16* x, float gs_inv, uint4& packed, uint32_t& scales) {
    uint4 raw[4];
#pragma unroll
    for (int i = 0; i < 4; i++) raw[i] = ld_nc_v4(reinterpret_cast<const uint8_t*>(x) + 16 * i);
    uint32_t w[4];
    scales = 0;
#pragma unroll
    for (int b = 0; b < 2; b++) {
        const uint32_t q[8] = {raw[2 * b].x,     raw[2 * b].y,     raw[2 * b].z,     raw[2 * b].w,
                               raw[2 * b + 1].x, raw[2 * b + 1].y, raw[2 * b + 1].z, raw[2 * b + 1].w};
        scales |= q16_bf16(q, gs_inv, w[2 * b], w[2 * b + 1]) << (8 * b);
    }
    packed = make_uint4(w[0], w[1], w[2], w[3]);
}
// Same from 32 fp32 values.
__device__ __forceinline__ void quant32f(const float* v, float gs_inv, uint4& packed, uint32_t& scales) {
    uint32_t w[4];
    const uint32_t s0 = q16(v, gs_inv, w[0], w[1]);
    const uint32_t s1 = q16(v + 16, gs_inv, w[2], w[3]);
    packed = make_uint4(w[0], w[1], w[2], w[3]);
    scales = s0 | (s1 << 8);
}
// acc[i] = fma(e2m1(code_i), decode(scale) * gs, acc[i]) for one 32-element chunk.
__device__ __forceinline__ void dq32_acc(uint4 packed, uint32_t scales, float gs, float* acc) {
    const uint32_t w[4] = {packed.x, packed.y, packed.z, packed.w};
#pragma unroll
    for (int b = 0; b < 2; b++) {
        const float bs = __fmul_rn(e4m3_decode((scales >> (8 * b)) & 0xFFu), gs);
#pragma unroll
        for (int h = 0; h < 2; h++) {
            float c[8];
            e2m1x8_decode(w[2 * b + h], c);
#pragma unroll
            for (int i = 0; i < 8; i++) acc[16 * b + 8 * h + i] = __fmaf_rn(c[i], bs, acc[16 * b + 8 * h + i]);
        }
    }
}
__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* out, const float* acc) {
#pragma unroll
    for (int i = 0; i < 4; i++) {
        uint32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const __nv_bfloat162 pr = __floats2bfloat162_rn(acc[8 * i + 2 * k], acc[8 * i + 2 * k + 1]);
            o[k] = *reinterpret_cast<const uint32_t*>(&pr);
        }
        st_v4(reinterpret_cast<uint8_t*>(out) + 16 * i, make_uint4(o[0], o[1], o[2], o[3]));
    }
}
// Store one chunk's payload into a payload of `n` elements at `dst`, chunk index c.
__device__ __forceinline__ void put_chunk(uint8_t* dst, int64_t n, int64_t c, uint4 packed, uint32_t scales) {
    st_v4(dst + c * 16, packed);
    *reinterpret_cast<uint16_t*>(dst + align16(n / 2) + c * 2) = (uint16_t)scales;
}
__device__ __forceinline__ void get_chunk(const uint8_t* src, int64_t n, int64_t c, uint4& packed, uint32_t& scales) {
    packed = ld_cg_v4(src + c * 16);
    scales = ld_cg_u16(src + align16(n / 2) + c * 2);
}

// ---------------------------------------------------------------- NVFP4 kernels ----
// Every phase is a grid-stride loop over chunks of 32 elements (one chunk per thread per pass); a
// thread handles a chunk's every rank or shard in turn.  Measured on 2 x B200 against variants
// that prefetched the next rank's or shard's data, split (shard, chunk) pairs over a block's
// threads, or ran two 512-thread blocks per SM (cfg4, back-to-back calls): two-shot 58.9-59.5 us
// here against 61.0 and 66.2 us, and 22 against 27-28 us at 4 MB of bf16 (one-shot 15 vs 18 us);
// the prefetching one-shot was 2 % faster at cfg4 only.  (Emulated on one GPU, where every
// "remote" access is local, the other variants were faster: the NVLink round trips decide.)
template <bool kTwoShot>
__global__ void __launch_bounds__(AR_THREADS) ar_nvfp4_kernel(const Params p) {
    const int n = p.world, me = p.rank;
    const float gs_inv = __fdiv_rn(1.0f, p.gs);
    const uint32_t v1 = p.epoch * 2u + 1u, v2 = p.epoch * 2u + 2u;
    const bool fused = p.phase < 0;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t first = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;

    if (!kTwoShot) {
        const int64_t chunks = p.numel / 32;
        if (fused || p.phase == 0) {
            for (int64_t c = first; c < chunks; c += stride) {
                uint4 pk;
                uint32_t sc;
                quant32(p.in + c * 32, gs_inv, pk, sc);
                for (int k = 1; k <= n; k++) {                 // rank me+1 first, own last
                    const int r = (me + k) % n;
                    put_chunk(in_slot(p, r, me), p.numel, c, pk, sc);
                }
            }
        }
        if (fused && !block_barrier(p, v1)) return;
        if (fused || p.phase == 1) {
            for (int64_t c = first; c < chunks; c += stride) {
                // fixed sum order 0 .. n-1, the loads of two slots in flight (measured on 2 x B200:
                // 2-5 % faster below cfg4, equal at cfg4; the same in the two-shot's sum was not faster)
                float acc[32];
#pragma unroll
                for (int i = 0; i < 32; i++) acc[i] = 0.0f;
                for (int s = 0; s < n; s += 2) {
                    uint4 pk0, pk1;
                    uint32_t sc0, sc1 = 0;
                    get_chunk(in_slot(p, me, s), p.numel, c, pk0, sc0);
                    if (s + 1 < n) get_chunk(in_slot(p, me, s + 1), p.numel, c, pk1, sc1);
                    dq32_acc(pk0, sc0, p.gs, acc);
                    if (s + 1 < n) dq32_acc(pk1, sc1, p.gs, acc);
                }
                store_bf16x32(p.out + c * 32, acc);
            }
        }
        return;
    }

    const int64_t shard = p.numel / n;
    const int64_t schunks = shard / 32;
    if (p.phase == -3 || p.phase == 3) {
        // the shards were quantized by the producer of the data (a GEMM epilogue): push them
        for (int64_t c = first; c < schunks; c += stride) {
            for (int k = 1; k <= n; k++) {
                const int o = (me + k) % n;
                const int64_t e32 = (int64_t)o * schunks + c;     // chunk of 32 elements of the input
                const uint4 pk = ld_nc_v4(p.q_codes + e32 * 16);
                const uint32_t sc = *reinterpret_cast<const uint16_t*>(p.q_scales + e32 * 2);
                put_chunk(in_slot(p, o, me), shard, c, pk, sc);
            }
        }
    }
    if (p.phase == -1 || p.phase == 0) {
        for (int64_t c = first; c < schunks; c += stride) {
            for (int k = 1; k <= n; k++) {                     // owner me+1 first, own shard last
                const int o = (me + k) % n;
                uint4 pk;
                uint32_t sc;
                quant32(p.in + (int64_t)o * shard + c * 32, gs_inv, pk, sc);
                put_chunk(in_slot(p, o, me), shard, c, pk, sc);
            }
        }
    }
    if (fused && !block_barrier(p, v1)) return;
    const float gs_red = __fmul_rn(p.gs, (float)n);
    if (fused || p.phase == 1) {
        const float gs_red_inv = __fdiv_rn(1.0f, gs_red);
        for (int64_t c = first; c < schunks; c += stride) {
            float acc[32];
#pragma unroll
            for (int i = 0; i < 32; i++) acc[i] = 0.0f;
            for (int s = 0; s < n; s++) {                      // fixed sum order 0 .. n-1
                uint4 pk;
                uint32_t sc;
                get_chunk(in_slot(p, me, s), shard, c, pk, sc);
                dq32_acc(pk, sc, p.gs, acc);
            }
            uint4 pk;
            uint32_t sc;
            quant32f(acc, gs_red_inv, pk, sc);
            for (int k = 1; k <= n; k++) {
                const int r = (me + k) % n;
                put_chunk(gather_slot(p, r, me), shard, c, pk, sc);
            }
        }
    }
    if (fused && !block_barrier(p, v2)) return;
    if (fused || p.phase == 2) {
        for (int64_t c = first; c < schunks; c += stride) {
            for (int o = 0; o < n; o++) {
                uint4 pk;
                uint32_t sc;
                get_chunk(gather_slot(p, me, o), shard, c, pk, sc);
                float acc[32];
#pragma unroll
                for (int i = 0; i < 32; i++) acc[i] = 0.0f;
                dq32_acc(pk, sc, gs_red, acc);
                store_bf16x32(p.out + (int64_t)o * shard + c * 32, acc);
            }
        }
    }
}

// Two-shot for small shards (at most one group of chunks per resident block): the grid-stride
// kernel above gives a thread all n shards of its chunk in phases A and C, n dependent round
// trips per thread, and at 4 MB of bf16 on 8 ranks it ran 16 blocks (41.5 us).  Here block b owns
// the chunk group [b * per, (b + 1) * per) of every shard (per = AR_THREADS / n) and its threads
// split the group's (shard, chunk) pairs: thread o_idx * per + j takes shard o_idx's chunk j in
// phases A and C; in phase B threads j < per sum chunk j of this rank's shard.  The same chunks
// go to block b on every rank in every phase, so the per-block barrier suffices.  Arithmetic and
// order as in ar_nvfp4_kernel<true>: the same bits.
__global__ void __launch_bounds__(AR_THREADS, 2) ar_nvfp4_twoshot_split_kernel(const Params p) {
    const int n = p.world, me = p.rank;
    const int per = AR_THREADS / n;
    const int t = threadIdx.x, o_idx = t / per, j = t % per;
    const int64_t shard = p.numel / n;
    const int64_t schunks = shard / 32;
    const int64_t c = (int64_t)blockIdx.x * per + j;
    const bool pair_ok = o_idx < n && c < schunks;
    const uint32_t v1 = p.epoch * 2u + 1u, v2 = p.epoch * 2u + 2u;
    const bool fused = p.phase < 0;
    if ((p.phase == -3 || p.phase == 3) && pair_ok) {
        // the shards were quantized by the producer of the data (a GEMM epilogue): push them
        const int o = (me + 1 + o_idx) % n;
        const int64_t e32 = (int64_t)o * schunks + c;
        const uint4 pk = ld_nc_v4(p.q_codes + e32 * 16);
        const uint32_t sc = *reinterpret_cast<const uint16_t*>(p.q_scales + e32 * 2);
        put_chunk(in_slot(p, o, me), shard, c, pk, sc);
    }
    if ((p.phase == -1 || p.phase == 0) && pair_ok) {
        const int o = (me + 1 + o_idx) % n;                  // owner me+1 first, own shard last
        uint4 pk;
        uint32_t sc;
        quant32(p.in + (int64_t)o * shard + c * 32, __fdiv_rn(1.0f, p.gs), pk, sc);
        put_chunk(in_slot(p, o, me), shard, c, pk, sc);
    }
    if (fused && !block_barrier(p, v1)) return;
    const float gs_red = __fmul_rn(p.gs, (float)n);
    if ((fused || p.phase == 1) && t < per && c < schunks) {
        float acc[32];
#pragma unroll
        for (int i = 0; i < 32; i++) acc[i] = 0.0f;
        for (int s = 0; s < n; s++) {                          // fixed sum order 0 .. n-1
            uint4 pk;
            uint32_t sc;
            get_chunk(in_slot(p, me, s), shard, c, pk, sc);
            dq32_acc(pk, sc, p.gs, acc);
        }
        uint4 pk;
        uint32_t sc;
        quant32f(acc, __fdiv_rn(1.0f, gs_red), pk, sc);
        for (int k = 1; k <= n; k++) put_chunk(gather_slot(p, (me + k) % n, me), shard, c, pk, sc);
    }
    if (fused && !block_barrier(p, v2)) return;
    if ((fused || p.phase == 2) && pair_ok) {
        uint4 pk;
        uint32_t sc;
        get_chunk(gather_slot(p, me, o_idx), shard, c, pk, sc);
        float acc[32];
#pragma unroll
        for (int i = 0; i < 32; i++) acc[i] = 0.0f;
        dq32_acc(pk, sc, gs_red, acc);
        store_bf16x32(p.out + (int64_t)o_idx * shard + c * 32, acc);
    }
}

// ---------------------------------------------------------------- low-latency one-shot ----
constexpr int AR_LL_THREADS = 128;
constexpr int AR_LL_WORDS = 3;                 // u64 words per 32-element chunk
constexpr uint64_t AR_LL_TAG = 1ull << 56;     // top byte of a written word: never zero
constexpr uint64_t AR_LL_M56 = AR_LL_TAG - 1;  // its 7 payload bytes

// Chunk c of a slot of `chunks` chunks: the 144 payload bits (codes lo = bytes 0-7, hi = bytes
// 8-15, then the two scale bytes) as 56 + 56 + 32 bits, each word tagged.
__device__ __forceinline__ void ll_put(uint64_t* slot, int64_t chunks, int64_t c, uint4 pk, uint32_t sc) {
    const uint64_t lo = (uint64_t)pk.x | ((uint64_t)pk.y << 32), hi = (uint64_t)pk.z | ((uint64_t)pk.w << 32);
    const uint64_t w[AR_LL_WORDS] = {(lo & AR_LL_M56) | AR_LL_TAG,
                                     (((lo >> 56) | (hi << 8)) & AR_LL_M56) | AR_LL_TAG,
                                     (hi >> 48) | ((uint64_t)(sc & 0xFFFFu) << 16) | AR_LL_TAG};
#pragma unroll
    for (int i = 0; i < AR_LL_WORDS; i++) st_relaxed_sys_u64(slot + i * chunks + c, w[i]);
}
// The 144 payload bits of one chunk from its three tagged words (inverse of ll_put).
__device__ __forceinline__ void ll_unpack(uint64_t w0, uint64_t w1, uint64_t w2, uint4& pk, uint32_t& sc) {
    const uint64_t lo = (w0 & AR_LL_M56) | (w1 << 56);
    const uint64_t hi = ((w1 & AR_LL_M56) >> 8) | (w2 << 48);
    pk = make_uint4((uint32_t)lo, (uint32_t)(lo >> 32), (uint32_t)hi, (uint32_t)(hi >> 32));
    sc = (uint32_t)(w2 >> 16) & 0xFFFFu;
}

// One-shot with the data-carried flags: A: quantize each chunk and push it to every peer;
// B: sum the ranks' chunks in rank order 0..n-1 as each arrives (this rank's own chunk is
// quantized again: the same bits as the pushed one).  Results equal ar_nvfp4_kernel<false>.
// phase -1: A and B; 0: A alone; 1: B alone (single-GPU emulation).
__global__ void __launch_bounds__(AR_LL_THREADS) ar_nvfp4_ll_kernel(const Params p) {
    const int n = p.world, me = p.rank;
    const float gs_inv = __fdiv_rn(1.0f, p.gs);
    const int64_t chunks = p.numel / 32;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t first = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (p.phase == -1 || p.phase == 0) {
        for (int64_t c = first; c < chunks; c += stride) {
            uint4 pk;
            uint32_t sc;
            quant32(p.in + c * 32, gs_inv, pk, sc);
            for (int k = 1; k < n; k++) {                     // rank me+1 first
                const int r = (me + k) % n;
                ll_put(ll_slot_of(p, r, me), chunks, c, pk, sc);
            }
        }
    }
    if (p.phase == -1 || p.phase == 1) {
        for (int64_t c = first; c < chunks; c += stride) {
            // every peer's three words of chunk c are loaded before any is checked (one round
            // trip for all peers, not one per peer); only untagged words are loaded again
            uint64_t w[AR_MAX_WORLD][AR_LL_WORDS];
#pragma unroll
            for (int s = 0; s < AR_MAX_WORLD; s++)
#pragma unroll
                for (int i = 0; i < AR_LL_WORDS; i++)
                    w[s][i] = (s < n && s != me) ? ld_relaxed_sys_u64(ll_slot_of(p, me, s) + i * chunks + c) : AR_LL_TAG;
            int spins = 0;
            uint64_t t0 = 0;
            for (;;) {
                bool ready = true;
#pragma unroll
                for (int s = 0; s < AR_MAX_WORLD; s++)
#pragma unroll
                    for (int i = 0; i < AR_LL_WORDS; i++) ready &= w[s][i] >= AR_LL_TAG;
                if (ready) break;
                if (++spins == 64) t0 = globaltimer_ns();
                if (spins > 64 && (spins & 63) == 0 && globaltimer_ns() - t0 > p.timeout_ns) {
                    record_error(DEV_TIMEOUT_AR_BARRIER);
                    return;
                }
#pragma unroll
                for (int s = 0; s < AR_MAX_WORLD; s++)
#pragma unroll
                    for (int i = 0; i < AR_LL_WORDS; i++)
                        if (w[s][i] < AR_LL_TAG) w[s][i] = ld_relaxed_sys_u64(ll_slot_of(p, me, s) + i * chunks + c);
            }
            // consumed: zero the words, so the next call of this parity starts from an empty area
#pragma unroll
            for (int s = 0; s < AR_MAX_WORLD; s++)
                if (s < n && s != me)
#pragma unroll
                    for (int i = 0; i < AR_LL_WORDS; i++) ll_slot_of(p, me, s)[i * chunks + c] = 0;
            float acc[32];
#pragma unroll
            for (int i = 0; i < 32; i++) acc[i] = 0.0f;
#pragma unroll
            for (int s = 0; s < AR_MAX_WORLD; s++) {              // fixed sum order 0 .. n-1
                if (s >= n) break;
                uint4 pk;
                uint32_t sc;
                if (s == me) quant32(p.in + c * 32, gs_inv, pk, sc);   // the same bits as the pushed chunk
                else ll_unpack(w[s][0], w[s][1], w[s][2], pk, sc);
                dq32_acc(pk, sc, p.gs, acc);
            }
            store_bf16x32(p.out + c * 32, acc);
        }
    }
}

// ---------------------------------------------------------------- bf16 kernels ----
// Chunk = 8 bf16 (16 bytes).  Sum in fp32, rank order 0 .. n-1, round to bf16 once.
__device__ __forceinline__ void acc_bf16x8(uint4 v, float* acc) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; k++) {
        acc[2 * k] = __fadd_rn(acc[2 * k], __uint_as_float(w[k] << 16));
        acc[2 * k + 1] = __fadd_rn(acc[2 * k + 1], __uint_as_float(w[k] & 0xFFFF0000u));
    }
}
__device__ __forceinline__ uint4 pack_bf16x8(const float* acc) {
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const __nv_bfloat162 pr = __floats2bfloat162_rn(acc[2 * k], acc[2 * k + 1]);
        o[k] = *reinterpret_cast<const uint32_t*>(&pr);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// Loads of all ranks' chunks are issued before the first is used, so the baseline is not held back
// by one round trip per rank.
template <bool kTwoShot>
__global__ void __launch_bounds__(AR_THREADS, 2) ar_bf16_kernel(const Params p) {
    const int n = p.world, me = p.rank;
    const uint32_t v1 = p.epoch * 2u + 1u, v2 = p.epoch * 2u + 2u;
    const bool fused = p.phase < 0;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t first = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint8_t* in = reinterpret_cast<const uint8_t*>(p.in);
    uint8_t* out = reinterpret_cast<uint8_t*>(p.out);
    auto sum_ranks = [&](auto src, int64_t c, float* acc) {      // fp32 sum in rank order 0 .. n-1
        uint4 v[AR_MAX_WORLD];
#pragma unroll
        for (int s = 0; s < AR_MAX_WORLD; s++)
            if (s < n) v[s] = ld_cg_v4(src(s) + c * 16);
#pragma unroll
        for (int s = 0; s < AR_MAX_WORLD; s++)
            if (s < n) acc_bf16x8(v[s], acc);
    };

    if (!kTwoShot) {
        const int64_t chunks = p.numel / 8;
        if (fused || p.phase == 0) {
            for (int64_t c = first; c < chunks; c += stride) {
                const uint4 v = ld_nc_v4(in + c * 16);
                for (int k = 1; k <= n; k++) st_v4(in_slot(p, (me + k) % n, me) + c * 16, v);
            }
        }
        if (fused && !block_barrier(p, v1)) return;
        if (fused || p.phase == 1) {
            for (int64_t c = first; c < chunks; c += stride) {
                float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                sum_ranks([&](int s) { return in_slot(p, me, s); }, c, acc);
                st_v4(out + c * 16, pack_bf16x8(acc));
            }
        }
        return;
    }
    const int64_t shard = p.numel / n;
    const int64_t schunks = shard / 8;
    if (fused || p.phase == 0) {
        for (int64_t c = first; c < schunks; c += stride) {
            uint4 v[AR_MAX_WORLD];
#pragma unroll
            for (int k = 1; k <= AR_MAX_WORLD; k++)
                if (k <= n) v[k - 1] = ld_nc_v4(in + ((int64_t)((me + k) % n) * shard) * 2 + c * 16);
#pragma unroll
            for (int k = 1; k <= AR_MAX_WORLD; k++)
                if (k <= n) st_v4(in_slot(p, (me + k) % n, me) + c * 16, v[k - 1]);
        }
    }
    if (fused && !block_barrier(p, v1)) return;
    if (fused || p.phase == 1) {
        for (int64_t c = first; c < schunks; c += stride) {
            float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            sum_ranks([&](int s) { return in_slot(p, me, s); }, c, acc);
            const uint4 r = pack_bf16x8(acc);
            for (int k = 1; k <= n; k++) st_v4(gather_slot(p, (me + k) % n, me) + c * 16, r);
        }
    }
    if (fused && !block_barrier(p, v2)) return;
    if (fused || p.phase == 2) {
        for (int64_t c = first; c < schunks; c += stride) {
            uint4 v[AR_MAX_WORLD];
#pragma unroll
            for (int o = 0; o < AR_MAX_WORLD; o++)
                if (o < n) v[o] = ld_cg_v4(gather_slot(p, me, o) + c * 16);
#pragma unroll
            for (int o = 0; o < AR_MAX_WORLD; o++)
                if (o < n) st_v4(out + ((int64_t)o * shard) * 2 + c * 16, v[o]);
        }
    }
}

// ---------------------------------------------------------------- NVLS (in-switch) bf16 ----
// 8 bf16 per 16-byte vector: the in-switch sum of one chunk over every rank's buffer (fp32
// accumulation, one rounding to bf16), and its store back to every rank's buffer.
__device__ __forceinline__ uint4 multimem_ld_reduce_bf16x8(const uint8_t* mc) {
    uint4 r;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(mc)
                 : "memory");
    return r;
}
__device__ __forceinline__ void multimem_st_bf16x8(uint8_t* mc, uint4 v) {
    asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(mc), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
}
// The same memory is written through one address (unicast or multicast) and read through the
// other: order the accesses across the two aliases.
__device__ __forceinline__ void fence_alias() { asm volatile("fence.proxy.alias;" ::: "memory"); }

constexpr int NVLS_UNROLL = 3;               // chunks in flight per thread in every phase (no spills at 2 blocks per SM)

__global__ void __launch_bounds__(AR_THREADS, 2) ar_bf16_nvls_kernel(const Params p) {
    const int n = p.world, me = p.rank;
    const uint32_t v1 = p.epoch * 2u + 1u, v2 = p.epoch * 2u + 2u;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t first = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint8_t* in = reinterpret_cast<const uint8_t*>(p.in);
    uint8_t* out = reinterpret_cast<uint8_t*>(p.out);
    const int64_t shard = p.numel / n;                 // elements
    const int64_t schunks = shard / 8;                 // 16-byte chunks of one shard
    // Every phase walks this block's chunks of a shard (c = first, first + stride, ...) with
    // NVLS_UNROLL of them loaded before any is stored: a load through the switch takes
    // microseconds, and one at a time per thread would leave the links idle.
    // A: this rank's input into its buffer -- the chunks of every shard that block b of any rank
    // reduces in B, so that B only needs block b of every rank to have finished A
    for (int q = 0; q < n; q++) {
        const int64_t base = ((int64_t)q * shard) * 2;
        for (int64_t c0 = first; c0 < schunks; c0 += stride * NVLS_UNROLL) {
            uint4 v[NVLS_UNROLL];
#pragma unroll
            for (int u = 0; u < NVLS_UNROLL; u++) {
                const int64_t c = c0 + u * stride;
                if (c < schunks) v[u] = ld_nc_v4(in + base + c * 16);
            }
#pragma unroll
            for (int u = 0; u < NVLS_UNROLL; u++) {
                const int64_t c = c0 + u * stride;
                if (c < schunks) st_v4(p.nvls_uc + base + c * 16, v[u]);
            }
        }
    }
    fence_alias();
    if (!block_barrier(p, v1)) return;
    fence_alias();
    // B: the in-switch sum of this rank's shard, written back to every rank
    {
        uint8_t* mine = p.nvls_mc + ((int64_t)me * shard) * 2;
        for (int64_t c0 = first; c0 < schunks; c0 += stride * NVLS_UNROLL) {
            uint4 v[NVLS_UNROLL];
#pragma unroll
            for (int u = 0; u < NVLS_UNROLL; u++) {
                const int64_t c = c0 + u * stride;
                if (c < schunks) v[u] = multimem_ld_reduce_bf16x8(mine + c * 16);
            }
#pragma unroll
            for (int u = 0; u < NVLS_UNROLL; u++) {
                const int64_t c = c0 + u * stride;
                if (c < schunks) multimem_st_bf16x8(mine + c * 16, v[u]);
            }
        }
    }
    fence_alias();
    if (!block_barrier(p, v2)) return;
    fence_alias();
    // C: the reduced tensor out of this rank's buffer
    for (int q = 0; q < n; q++) {
        const int64_t base = ((int64_t)q * shard) * 2;
        for (int64_t c0 = first; c0 < schunks; c0 += stride * NVLS_UNROLL) {
            uint4 v[NVLS_UNROLL];
#pragma unroll
            for (int u = 0; u < NVLS_UNROLL; u++) {
                const int64_t c = c0 + u * stride;
                if (c < schunks) v[u] = ld_cg_v4(p.nvls_uc + base + c * 16);
            }
#pragma unroll
            for (int u = 0; u < NVLS_UNROLL; u++) {
                const int64_t c = c0 + u * stride;
                if (c < schunks) st_v4(out + base + c * 16, v[u]);
            }
        }
    }
}

}  // namespace ar
}  // namespace nvfp4

// ====================================================================== host ====
using namespace nvfp4;
using namespace nvfp4::ar;

struct nvfp4_ar {
    int world = 0, rank = 0, device = -1;
    int64_t max_numel = 0;
    int64_t in_slot = 0, gather_slot = 0, region = 0;
    int64_t ll_numel = 0, ll_slot = 0, ll_off = 0;   // low-latency area: capacity, slot bytes, offset
    size_t bytes = 0;
    uint8_t* base = nullptr;
    uint8_t* peer[AR_MAX_WORLD] = {};
    bool ipc_opened[AR_MAX_WORLD] = {};
    bool ready = false;
    uint32_t epoch = 0;
    uint64_t timeout_ns = AR_DEFAULT_TIMEOUT_NS;
    int max_grid = 0, ll_max_grid = 0;   // resident grids: bf16 / NVLS kernels, low-latency kernel
    int nvfp4_max_grid = 0;              // resident grid of the NVFP4 one- and two-shot kernels
    int split_max_grid = 0;              // resident grid of the small-shard two-shot kernel
    uint8_t* nvls_mc = nullptr;      // NVLS buffer (nvfp4_ar_set_multicast): multicast address,
    uint8_t* nvls_uc = nullptr;      // this rank's unicast address,
    int64_t nvls_half = 0;           // bytes of one parity half
};

namespace {

// Slot sizes for a context: large enough for every algorithm at max_numel.
void slot_sizes(int world, int64_t max_numel, int64_t& in_slot, int64_t& gather_slot) {
    const int64_t shard = max_numel / world;
    int64_t a = payload_bytes(max_numel);          // NVFP4 one-shot
    int64_t b = align16(max_numel * 2);            // bf16 one-shot
    in_slot = a > b ? a : b;
    a = payload_bytes(shard);
    b = align16(shard * 2);
    gather_slot = a > b ? a : b;
}

// Low-latency area: elements one call may use, and bytes of one slot (3 u64 words per 32 elements).
void ll_sizes(int64_t max_numel, int64_t& ll_numel, int64_t& ll_slot) {
    ll_numel = max_numel < NVFP4_AR_LOWLAT_CAP_BYTES / 2 ? max_numel : NVFP4_AR_LOWLAT_CAP_BYTES / 2;
    ll_numel -= ll_numel % 32;
    ll_slot = ll_numel / 32 * AR_LL_WORDS * 8;
}

nvfp4_status_t check_ctx(nvfp4_ar_t h, const char* who) {
    if (!h) return fail(NVFP4_ERR_INVALID_ARG, "%s: null context", who);
    int dev = -1;
    cudaGetDevice(&dev);
    if (dev != h->device)
        return fail(NVFP4_ERR_INVALID_ARG, "%s: context lives on device %d, current device is %d", who, h->device, dev);
    return NVFP4_OK;
}

int resident_grid(const void* fn, int threads = AR_THREADS) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, 0) != cudaSuccess || per_sm < 1) {
        cudaGetLastError();
        per_sm = 1;
    }
    int g = per_sm * sm_count();
    return g < AR_MAX_BLOCKS ? g : AR_MAX_BLOCKS;
}

// Blocks for `work` chunks of a phase: a quarter of a chunk per thread or more blocks, at most what
// is resident -- spreading the chunks over more SMs gives each SM fewer dependent round trips.
int grid_for(nvfp4_ar_t h, int64_t work) {
    int64_t g = (work + AR_THREADS / 4 - 1) / (AR_THREADS / 4);
    if (g < 1) g = 1;
    if (g > h->max_grid) g = h->max_grid;
    return (int)g;
}

nvfp4_status_t check_call(nvfp4_ar_t h, const char* who, const void* in, const void* out, int64_t numel, int algo,
                          int elems_per_chunk) {
    nvfp4_status_t st = check_ctx(h, who);
    if (st) return st;
    if (!h->ready) return fail(NVFP4_ERR_NOT_READY, "%s: peers not set (nvfp4_ar_open_peers / nvfp4_ar_set_peers)", who);
    if (numel < 0 || numel > h->max_numel)
        return fail(NVFP4_ERR_INVALID_ARG, "%s: numel %lld outside [0, max_numel=%lld]", who, (long long)numel,
                    (long long)h->max_numel);
    if (algo != NVFP4_AR_AUTO && algo != NVFP4_AR_ONESHOT && algo != NVFP4_AR_TWOSHOT && algo != NVFP4_AR_LOWLAT &&
        algo != NVFP4_AR_NVLS)
        return fail(NVFP4_ERR_INVALID_ARG, "%s: algo must be NVFP4_AR_AUTO, _ONESHOT, _TWOSHOT, _LOWLAT or _NVLS", who);
    if (algo == NVFP4_AR_NVLS && elems_per_chunk != 8)
        return fail(NVFP4_ERR_UNSUPPORTED, "%s: NVFP4_AR_NVLS sums bf16 in the switch; NVFP4 payloads cannot be summed there",
                    who);
    if (algo == NVFP4_AR_NVLS && !h->nvls_mc)
        return fail(NVFP4_ERR_NOT_READY, "%s: NVFP4_AR_NVLS needs a multicast buffer (nvfp4_ar_set_multicast)", who);
    if (algo == NVFP4_AR_NVLS && numel * 2 > h->nvls_half)
        return fail(NVFP4_ERR_INVALID_ARG, "%s: %lld bf16 elements exceed the multicast buffer's half of %lld bytes", who,
                    (long long)numel, (long long)h->nvls_half);
    if (algo == NVFP4_AR_LOWLAT && elems_per_chunk != 32)
        return fail(NVFP4_ERR_INVALID_ARG, "%s: NVFP4_AR_LOWLAT is an NVFP4 algorithm", who);
    if (algo == NVFP4_AR_LOWLAT && numel > h->ll_numel)
        return fail(NVFP4_ERR_INVALID_ARG, "%s: NVFP4_AR_LOWLAT takes at most %lld elements in this context", who,
                    (long long)h->ll_numel);
    if (numel == 0) return NVFP4_OK;
    if (!in || !out) return fail(NVFP4_ERR_INVALID_ARG, "%s: null buffer", who);
    if (!aligned16(in) || !aligned16(out)) return fail(NVFP4_ERR_INVALID_ARG, "%s: buffers must be 16-byte aligned", who);
    const int64_t unit = (int64_t)elems_per_chunk * h->world;
    if (numel % unit != 0)
        return fail(NVFP4_ERR_INVALID_ARG, "%s: numel %lld must be a multiple of %d x world = %lld", who,
                    (long long)numel, elems_per_chunk, (long long)unit);
    return NVFP4_OK;
}

}  // namespace

extern "C" {

int64_t nvfp4_ar_buffer_bytes(int world, int64_t max_numel) {
    if (world < 1 || world > AR_MAX_WORLD || max_numel < 0) return -1;
    int64_t in_slot, gather_slot;
    slot_sizes(world, max_numel, in_slot, gather_slot);
    int64_t ll_numel, ll_slot;
    ll_sizes(max_numel, ll_numel, ll_slot);
    return (int64_t)AR_FLAG_BYTES + 2 * ((int64_t)world * in_slot + (int64_t)world * gather_slot) +
           2 * (int64_t)world * ll_slot;
}

nvfp4_status_t nvfp4_ar_create(int world, int rank, int64_t max_numel, nvfp4_ar_t* out) {
    clear_error();
    if (!out) return fail(NVFP4_ERR_INVALID_ARG, "ar_create: null output");
    *out = nullptr;
    if (world < 1 || world > AR_MAX_WORLD) return fail(NVFP4_ERR_INVALID_ARG, "ar_create: world must be 1..%d", AR_MAX_WORLD);
    if (rank < 0 || rank >= world) return fail(NVFP4_ERR_INVALID_ARG, "ar_create: rank %d outside [0, %d)", rank, world);
    if (max_numel < 0 || max_numel > (int64_t(1) << 34)) return fail(NVFP4_ERR_INVALID_ARG, "ar_create: bad max_numel");
    nvfp4_ar* h = new nvfp4_ar();
    h->world = world;
    h->rank = rank;
    h->max_numel = max_numel;
    cudaGetDevice(&h->device);
    slot_sizes(world, max_numel, h->in_slot, h->gather_slot);
    h->region = (int64_t)world * h->in_slot + (int64_t)world * h->gather_slot;
    ll_sizes(max_numel, h->ll_numel, h->ll_slot);
    h->ll_off = (int64_t)AR_FLAG_BYTES + 2 * h->region;
    h->bytes = (size_t)h->ll_off + 2 * (size_t)world * (size_t)h->ll_slot;
    cudaError_t e = cudaMalloc(&h->base, h->bytes);
    if (e == cudaSuccess) e = cudaMemset(h->base, 0, h->bytes);
    if (e != cudaSuccess) {
        if (h->base) cudaFree(h->base);
        delete h;
        cudaGetLastError();
        return fail(NVFP4_ERR_CUDA, "ar_create: %s", cudaGetErrorString(e));
    }
    // every kernel that meets peers in block barriers keeps all its blocks resident: each family's
    // grid is capped at the smallest resident grid of its kernels
    const int g1 = resident_grid((const void*)ar_nvfp4_kernel<true>), g2 = resident_grid((const void*)ar_nvfp4_kernel<false>);
    h->nvfp4_max_grid = g1 < g2 ? g1 : g2;
    h->split_max_grid = resident_grid((const void*)ar_nvfp4_twoshot_split_kernel);
    int g3 = resident_grid((const void*)ar_bf16_kernel<true>), g4 = resident_grid((const void*)ar_bf16_kernel<false>);
    const int g5 = resident_grid((const void*)ar_bf16_nvls_kernel);
    int g = g3;
    if (g4 < g) g = g4;
    if (g5 < g) g = g5;
    h->max_grid = g;
    h->ll_max_grid = resident_grid((const void*)ar_nvfp4_ll_kernel, AR_LL_THREADS);
    h->peer[rank] = h->base;
    if (world == 1) h->ready = true;
    *out = h;
    return NVFP4_OK;
}

nvfp4_status_t nvfp4_ar_destroy(nvfp4_ar_t h) {
    clear_error();
    if (!h) return NVFP4_OK;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(h->device);
    for (int r = 0; r < h->world; r++)
        if (h->ipc_opened[r]) cudaIpcCloseMemHandle(h->peer[r]);
    if (h->base) cudaFree(h->base);
    if (prev >= 0) cudaSetDevice(prev);
    delete h;
    return NVFP4_OK;
}

size_t nvfp4_ar_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

nvfp4_status_t nvfp4_ar_export_handle(nvfp4_ar_t h, void* handle_out) {
    clear_error();
    nvfp4_status_t st = check_ctx(h, "ar_export_handle");
    if (st) return st;
    if (!handle_out) return fail(NVFP4_ERR_INVALID_ARG, "ar_export_handle: null output");
    cudaIpcMemHandle_t mh;
    cudaError_t e = cudaIpcGetMemHandle(&mh, h->base);
    if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "ar_export_handle: %s", cudaGetErrorString(e));
    memcpy(handle_out, &mh, sizeof(mh));
    return NVFP4_OK;
}

nvfp4_status_t nvfp4_ar_open_peers(nvfp4_ar_t h, const void* handles) {
    clear_error();
    nvfp4_status_t st = check_ctx(h, "ar_open_peers");
    if (st) return st;
    if (!handles) return fail(NVFP4_ERR_INVALID_ARG, "ar_open_peers: null handles");
    if (h->ready && h->world > 1) return fail(NVFP4_ERR_INVALID_ARG, "ar_open_peers: peers already set");
    const uint8_t* hs = reinterpret_cast<const uint8_t*>(handles);
    for (int r = 0; r < h->world; r++) {
        if (r == h->rank) continue;
        cudaIpcMemHandle_t mh;
        memcpy(&mh, hs + (size_t)r * sizeof(mh), sizeof(mh));
        void* p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, mh, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (int q = 0; q < r; q++)
                if (h->ipc_opened[q]) {
                    cudaIpcCloseMemHandle(h->peer[q]);
                    h->ipc_opened[q] = false;
                    h->peer[q] = nullptr;
                }
            cudaGetLastError();
            return fail(NVFP4_ERR_CUDA, "ar_open_peers: rank %d: %s", r, cudaGetErrorString(e));
        }
        h->peer[r] = reinterpret_cast<uint8_t*>(p);
        h->ipc_opened[r] = true;
    }
    h->ready = true;
    return NVFP4_OK;
}

nvfp4_status_t nvfp4_ar_local_base(nvfp4_ar_t h, void** base) {
    clear_error();
    if (!h || !base) return fail(NVFP4_ERR_INVALID_ARG, "ar_local_base: null argument");
    *base = h->base;
    return NVFP4_OK;
}

nvfp4_status_t nvfp4_ar_set_peers(nvfp4_ar_t h, void* const* bases) {
    clear_error();
    nvfp4_status_t st = check_ctx(h, "ar_set_peers");
    if (st) return st;
    if (!bases) return fail(NVFP4_ERR_INVALID_ARG, "ar_set_peers: null bases");
    if (bases[h->rank] != h->base) return fail(NVFP4_ERR_INVALID_ARG, "ar_set_peers: entry of this rank is not its own base");
    for (int r = 0; r < h->world; r++) {
        if (!bases[r]) return fail(NVFP4_ERR_INVALID_ARG, "ar_set_peers: null base of rank %d", r);
        if (r == h->rank) continue;
        cudaPointerAttributes a;
        cudaError_t e = cudaPointerGetAttributes(&a, bases[r]);
        if (e != cudaSuccess || a.type != cudaMemoryTypeDevice) {
            cudaGetLastError();
            return fail(NVFP4_ERR_INVALID_ARG, "ar_set_peers: base of rank %d is not device memory", r);
        }
        if (a.device != h->device) {
            e = cudaDeviceEnablePeerAccess(a.device, 0);
            if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
            else if (e != cudaSuccess) {
                cudaGetLastError();
                return fail(NVFP4_ERR_CUDA, "ar_set_peers: peer access %d -> %d: %s", h->device, a.device,
                            cudaGetErrorString(e));
            }
        }
    }
    for (int r = 0; r < h->world; r++) h->peer[r] = reinterpret_cast<uint8_t*>(bases[r]);
    h->ready = true;
    return NVFP4_OK;
}

nvfp4_status_t nvfp4_ar_set_multicast(nvfp4_ar_t h, void* mc_base, void* uc_base, int64_t bytes) {
    clear_error();
    nvfp4_status_t st = check_ctx(h, "ar_set_multicast");
    if (st) return st;
    if (!mc_base || !uc_base || bytes < 32)
        return fail(NVFP4_ERR_INVALID_ARG, "ar_set_multicast: need multicast and unicast addresses and >= 32 bytes");
    if (!aligned16(mc_base) || !aligned16(uc_base))
        return fail(NVFP4_ERR_INVALID_ARG, "ar_set_multicast: addresses must be 16-byte aligned");
    h->nvls_mc = reinterpret_cast<uint8_t*>(mc_base);
    h->nvls_uc = reinterpret_cast<uint8_t*>(uc_base);
    h->nvls_half = (bytes / 2) & ~(int64_t)15;
    return NVFP4_OK;
}

nvfp4_status_t nvfp4_ar_set_timeout(nvfp4_ar_t h, uint64_t timeout_ns) {
    clear_error();
    if (!h) return fail(NVFP4_ERR_INVALID_ARG, "ar_set_timeout: null context");
    if (timeout_ns < 1000000ull || timeout_ns > 600000000000ull)
        return fail(NVFP4_ERR_INVALID_ARG, "ar_set_timeout: limit must be 1 ms .. 600 s");
    h->timeout_ns = timeout_ns;
    return NVFP4_OK;
}

nvfp4_status_t nvfp4_ar_reset(nvfp4_ar_t h) {
    clear_error();
    nvfp4_status_t st = check_ctx(h, "ar_reset");
    if (st) return st;
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemset(h->base, 0, AR_FLAG_BYTES);
    // a timed-out call may have left low-latency words set: clear them too
    if (e == cudaSuccess) e = cudaMemset(h->base + h->ll_off, 0, h->bytes - (size_t)h->ll_off);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "ar_reset: %s", cudaGetErrorString(e));
    h->epoch = 0;
    return NVFP4_OK;
}

int nvfp4_ar_choose_algo(int world, int64_t numel) {
    if (world <= 1) return NVFP4_AR_ONESHOT;
    // the low-latency one-shot needs no barrier but sends 1.33x the payload (faster than one-shot
    // up to its 1 MB cap on 2 and 8 x B200); one-shot pushes the whole payload to every peer but
    // needs one barrier: better than two-shot while the call is latency-bound (on 8 x B200 the
    // small-shard two-shot is ahead from 4 MB of bf16: 25.8 vs 30.0 us)
    if (numel * 2 <= NVFP4_AR_LOWLAT_MAX_BYTES) return NVFP4_AR_LOWLAT;
    // with two ranks the two-shot sends as many bytes as the one-shot (half the payload, twice)
    // and adds a barrier and a pass over HBM: one-shot at every size (measured on 2 x B200 from
    // 4 MB to 256 MB of bf16: 17.5 vs 26.1 us ... 221 vs 254 us)
    if (world == 2) return NVFP4_AR_ONESHOT;
    return numel * 2 <= NVFP4_AR_ONESHOT_MAX_BYTES ? NVFP4_AR_ONESHOT : NVFP4_AR_TWOSHOT;
}

// The algorithm a call runs.  AUTO resolves by size (nvfp4_ar_choose_algo).  The low-latency
// one-shot exists only for NVFP4 payloads within the context's low-latency area, so a LOWLAT that
// AUTO picked for a bf16 payload or a larger call runs as ONESHOT; an explicit NVFP4_AR_LOWLAT
// outside those limits never gets here (check_call rejects it).  Every entry point resolves
// through this one rule.
static int resolve_algo(nvfp4_ar_t h, int algo, int64_t numel, bool nvfp4_payload) {
    if (algo == NVFP4_AR_AUTO) algo = nvfp4_ar_choose_algo(h->world, numel);
    if (algo == NVFP4_AR_LOWLAT && (!nvfp4_payload || numel > h->ll_numel)) algo = NVFP4_AR_ONESHOT;
    return algo;
}

static Params make_params(nvfp4_ar_t h, const void* in, void* out, int64_t numel, float gs, int phase) {
    Params p = {};
    for (int r = 0; r < h->world; r++) p.comm[r] = h->peer[r];
    p.in = reinterpret_cast<const __nv_bfloat16*>(in);
    p.out = reinterpret_cast<__nv_bfloat16*>(out);
    p.numel = numel;
    p.in_slot = h->in_slot;
    p.gather_slot = h->gather_slot;
    p.region = h->region;
    p.world = h->world;
    p.rank = h->rank;
    p.epoch = h->epoch;
    p.gs = gs;
    p.timeout_ns = h->timeout_ns;
    p.phase = phase;
    p.ll_off = h->ll_off;
    p.ll_slot = h->ll_slot;
    return p;
}

static nvfp4_status_t launch_nvfp4_ll(nvfp4_ar_t h, const Params& p, cudaStream_t s) {
    int64_t g = (p.numel / 32 + AR_LL_THREADS - 1) / AR_LL_THREADS;
    if (g > h->ll_max_grid) g = h->ll_max_grid;   // every block resident: blocks wait on peers
    ar_nvfp4_ll_kernel<<<(int)(g < 1 ? 1 : g), AR_LL_THREADS, 0, s>>>(p);
    return check_launch("ar_nvfp4_ll_kernel");
}
static nvfp4_status_t launch_nvfp4(nvfp4_ar_t h, const Params& p, bool twoshot, cudaStream_t s) {
    if (twoshot) {
        // small shards: one chunk group per block, the threads splitting (shard, chunk) pairs
        const int per = AR_THREADS / p.world;
        const int64_t groups = (p.numel / p.world / 32 + per - 1) / per;
        if (groups <= h->split_max_grid) {
            ar_nvfp4_twoshot_split_kernel<<<(int)(groups < 1 ? 1 : groups), AR_THREADS, 0, s>>>(p);
            return check_launch("ar_nvfp4_twoshot_split_kernel");
        }
    }
    // one chunk per thread and pass, at most the resident blocks
    const int64_t work = twoshot ? p.numel / p.world / 32 : p.numel / 32;
    int64_t g = (work + AR_THREADS - 1) / AR_THREADS;
    if (g > h->nvfp4_max_grid) g = h->nvfp4_max_grid;
    const int grid = g < 1 ? 1 : (int)g;
    if (twoshot) ar_nvfp4_kernel<true><<<grid, AR_THREADS, 0, s>>>(p);
    else ar_nvfp4_kernel<false><<<grid, AR_THREADS, 0, s>>>(p);
    return check_launch("ar_nvfp4_kernel");
}
static nvfp4_status_t launch_bf16_nvls(nvfp4_ar_t h, Params p, cudaStream_t s) {
    p.nvls_mc = h->nvls_mc + (int64_t)(p.epoch & 1u) * h->nvls_half;
    p.nvls_uc = h->nvls_uc + (int64_t)(p.epoch & 1u) * h->nvls_half;
    ar_bf16_nvls_kernel<<<grid_for(h, (p.numel / p.world / 8 + NVLS_UNROLL - 1) / NVLS_UNROLL), AR_THREADS, 0, s>>>(p);
    return check_launch("ar_bf16_nvls_kernel");
}
static nvfp4_status_t launch_bf16(nvfp4_ar_t h, const Params& p, bool twoshot, cudaStream_t s) {
    const int64_t work = twoshot ? p.numel / p.world / 8 : p.numel / 8;
    const int grid = grid_for(h, work);
    if (twoshot) ar_bf16_kernel<true><<<grid, AR_THREADS, 0, s>>>(p);
    else ar_bf16_kernel<false><<<grid, AR_THREADS, 0, s>>>(p);
    return check_launch("ar_bf16_kernel");
}

nvfp4_status_t nvfp4_ar_allreduce(nvfp4_ar_t h, const void* in, void* out, int64_t numel, float global_scale, int algo,
                                  void* stream) {
    clear_error();
    nvfp4_status_t st = check_call(h, "ar_allreduce", in, out, numel, algo, 32);
    if (st || numel == 0) return st;
    if (!(global_scale > 0.0f) || !isfinite(global_scale))
        return fail(NVFP4_ERR_INVALID_ARG, "ar_allreduce: global_scale must be finite and > 0");
    algo = resolve_algo(h, algo, numel, true);
    h->epoch++;
    const Params p = make_params(h, in, out, numel, global_scale, -1);
    if (algo == NVFP4_AR_LOWLAT) return launch_nvfp4_ll(h, p, (cudaStream_t)stream);
    return launch_nvfp4(h, p, algo == NVFP4_AR_TWOSHOT, (cudaStream_t)stream);
}

nvfp4_status_t nvfp4_ar_bf16_allreduce(nvfp4_ar_t h, const void* in, void* out, int64_t numel, int algo,
                                       void* stream) {
    clear_error();
    nvfp4_status_t st = check_call(h, "ar_bf16_allreduce", in, out, numel, algo, 8);
    if (st || numel == 0) return st;
    algo = resolve_algo(h, algo, numel, false);
    h->epoch++;
    if (algo == NVFP4_AR_NVLS) return launch_bf16_nvls(h, make_params(h, in, out, numel, 0.0f, -1), (cudaStream_t)stream);
    return launch_bf16(h, make_params(h, in, out, numel, 0.0f, -1), algo == NVFP4_AR_TWOSHOT, (cudaStream_t)stream);
}

// The GEMM of a fused call quantizes D (codes [M][N/2], flat scales) into this rank's own buffer,
// in the parity region the call does not use: peers write a rank's region of parity q only in
// calls of parity q, and the next such call cannot start its pushes before this rank has passed
// this call's second barrier, long after the quantized data was pushed.
static uint8_t* scratch_codes(nvfp4_ar_t h) {
    return h->base + AR_FLAG_BYTES + (int64_t)((h->epoch & 1u) ^ 1u) * h->region;
}
static uint8_t* scratch_scales(nvfp4_ar_t h, int64_t numel) { return scratch_codes(h) + align16(numel / 2); }

static nvfp4_status_t launch_gemm_payload(nvfp4_ar_t h, const void* A, const void* sfa, const void* B, const void* sfb,
                                          float alpha, float gs, int64_t M, int64_t N, int64_t K, cudaStream_t s) {
    gemm2::EpiOut q{};
    q.gs_inv = 1.0f / gs;
    q.sf = scratch_scales(h, M * N);
    return gemm2::launch<gemm2::OUT_PAYLOAD>(A, sfa, B, sfb, alpha, scratch_codes(h), M, N, K, s, q);
}

static Params gemm_ar_params(nvfp4_ar_t h, void* out, int64_t numel, float gs, int phase) {
    Params p = make_params(h, nullptr, out, numel, gs, phase);
    p.q_codes = scratch_codes(h);
    p.q_scales = scratch_scales(h, numel);
    return p;
}

static nvfp4_status_t check_gemm_ar(nvfp4_ar_t h, const char* who, const void* A, const void* sfa, const void* B,
                                    const void* sfb, const void* out, int64_t M, int64_t N, int64_t K, float gs) {
    if (!A || !sfa || !B || !sfb) return fail(NVFP4_ERR_INVALID_ARG, "%s: null operand", who);
    if (M <= 0 || N <= 0 || K <= 0 || M % 256 || N % 256 || K % 256)
        return fail(NVFP4_ERR_INVALID_ARG, "%s: need M %% 256 == 0, N %% 256 == 0, K %% 256 == 0", who);
    if (!aligned16(A) || !aligned16(B) || !aligned16(sfa) || !aligned16(sfb))
        return fail(NVFP4_ERR_INVALID_ARG, "%s: operands must be 16-byte aligned", who);
    nvfp4_status_t st = check_call(h, who, A, out, M * N, NVFP4_AR_TWOSHOT, 32);
    if (st) return st;
    if ((M * N / h->world) % 64 != 0)
        return fail(NVFP4_ERR_INVALID_ARG, "%s: M*N/world must be a multiple of 64", who);
    if (!(gs > 0.0f) || !isfinite(gs)) return fail(NVFP4_ERR_INVALID_ARG, "%s: global_scale must be finite and > 0", who);
    return NVFP4_OK;
}

nvfp4_status_t nvfp4_gemm_allreduce(nvfp4_ar_t h, const void* A, const void* sfa, const void* B, const void* sfb,
                                    float alpha, float global_scale, void* out, int64_t M, int64_t N, int64_t K,
                                    void* stream) {
    clear_error();
    nvfp4_status_t st = check_gemm_ar(h, "gemm_allreduce", A, sfa, B, sfb, out, M, N, K, global_scale);
    if (st) return st;
    h->epoch++;
    cudaStream_t s = (cudaStream_t)stream;
    if ((st = launch_gemm_payload(h, A, sfa, B, sfb, alpha, global_scale, M, N, K, s))) return st;
    return launch_nvfp4(h, gemm_ar_params(h, out, M * N, global_scale, -3), true, s);
}

nvfp4_status_t nvfp4_gemm_allreduce_emulated(nvfp4_ar_t const* handles, int world, const void* const* A,
                                             const void* const* sfa, const void* const* B, const void* const* sfb,
                                             const float* alpha, float global_scale, void* const* outs, int64_t M,
                                             int64_t N, int64_t K, void* stream) {
    clear_error();
    if (!handles || !A || !sfa || !B || !sfb || !alpha || !outs || world < 1 || world > AR_MAX_WORLD)
        return fail(NVFP4_ERR_INVALID_ARG, "gemm_allreduce_emulated: bad arguments");
    for (int r = 0; r < world; r++) {
        nvfp4_status_t st = check_gemm_ar(handles[r], "gemm_allreduce_emulated", A[r], sfa[r], B[r], sfb[r], outs[r],
                                          M, N, K, global_scale);
        if (st) return st;
        if (handles[r]->world != world || handles[r]->rank != r || handles[r]->device != handles[0]->device)
            return fail(NVFP4_ERR_INVALID_ARG, "gemm_allreduce_emulated: contexts must be ranks 0..%d of one device",
                        world - 1);
    }
    cudaStream_t s = (cudaStream_t)stream;
    for (int r = 0; r < world; r++) handles[r]->epoch++;
    // every rank's GEMM, then the push of the payloads, then phase 1, then phase 2 of every rank:
    // no kernel waits
    for (int r = 0; r < world; r++) {
        nvfp4_status_t st =
            launch_gemm_payload(handles[r], A[r], sfa[r], B[r], sfb[r], alpha[r], global_scale, M, N, K, s);
        if (st) return st;
    }
    const int phases[3] = {3, 1, 2};
    for (int ph : phases)
        for (int r = 0; r < world; r++) {
            nvfp4_status_t st =
                launch_nvfp4(handles[r], gemm_ar_params(handles[r], outs[r], M * N, global_scale, ph), true, s);
            if (st) return st;
        }
    return NVFP4_OK;
}

nvfp4_status_t nvfp4_ar_allreduce_emulated(nvfp4_ar_t const* handles, int world, const void* const* ins,
                                           void* const* outs, int64_t numel, float global_scale, int algo,
                                           int bf16_payload, void* stream) {
    clear_error();
    if (!handles || !ins || !outs || world < 1 || world > AR_MAX_WORLD)
        return fail(NVFP4_ERR_INVALID_ARG, "ar_allreduce_emulated: bad arguments");
    if (algo == NVFP4_AR_NVLS)
        return fail(NVFP4_ERR_UNSUPPORTED, "ar_allreduce_emulated: NVFP4_AR_NVLS needs a multicast object across GPUs");
    for (int r = 0; r < world; r++) {
        nvfp4_status_t st = check_call(handles[r], "ar_allreduce_emulated", ins[r], outs[r], numel,
                                       algo == NVFP4_AR_AUTO ? NVFP4_AR_AUTO : algo, bf16_payload ? 8 : 32);
        if (st) return st;
        if (handles[r]->world != world || handles[r]->rank != r || handles[r]->device != handles[0]->device)
            return fail(NVFP4_ERR_INVALID_ARG, "ar_allreduce_emulated: contexts must be ranks 0..%d of one device", world - 1);
    }
    if (numel == 0) return NVFP4_OK;
    if (!bf16_payload && (!(global_scale > 0.0f) || !isfinite(global_scale)))
        return fail(NVFP4_ERR_INVALID_ARG, "ar_allreduce_emulated: global_scale must be finite and > 0");
    algo = resolve_algo(handles[0], algo, numel, !bf16_payload);
    const bool two = algo == NVFP4_AR_TWOSHOT;
    for (int r = 0; r < world; r++) handles[r]->epoch++;
    if (algo == NVFP4_AR_LOWLAT) {
        for (int ph = 0; ph < 2; ph++)
            for (int r = 0; r < world; r++) {
                nvfp4_status_t st = launch_nvfp4_ll(handles[r], make_params(handles[r], ins[r], outs[r], numel,
                                                                            global_scale, ph), (cudaStream_t)stream);
                if (st) return st;
            }
        return NVFP4_OK;
    }
    // Phase by phase, rank by rank: the launches are ordered on one stream, so no kernel ever
    // waits for another one.
    const int phases = two ? 3 : 2;
    for (int ph = 0; ph < phases; ph++)
        for (int r = 0; r < world; r++) {
            const Params p = make_params(handles[r], ins[r], outs[r], numel, global_scale, ph);
            nvfp4_status_t st = bf16_payload ? launch_bf16(handles[r], p, two, (cudaStream_t)stream)
                                             : launch_nvfp4(handles[r], p, two, (cudaStream_t)stream);
            if (st) return st;
        }
    return NVFP4_OK;
}

}  // extern "C"
