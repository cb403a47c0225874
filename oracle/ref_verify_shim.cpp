// ref_verify_shim.cpp -- exports the reference's own CPU oracle as a C ABI.
//
// TEST INFRASTRUCTURE ONLY.  This translation unit #includes the UNMODIFIED reference header
// random_cpu_ref/verify_random.h from the read-only reference tree (include path given by
// oracle/Makefile) and wraps its functions so that Python tests can pin this project's
// oracle (oracle/nvfp4_oracle.c) and drop-in header (include/verify_random.h) against the
// reference itself.  The build output goes to oracle/_ref/ only and is never shipped as
// product code.  It also serves as the "reference CPU implementation" that
// bench.py --impl reference times.
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "verify_random.h"   // the reference header, found through -I

extern "C" {

// xorshift stream: out[i] = successive xorshift(&seed) values; returns the final state.
uint32_t ref_xorshift_stream(uint32_t seed, int n, uint32_t* out) {
    for (int i = 0; i < n; i++) out[i] = xorshift(&seed);
    return seed;
}

// fill_random over the E2M1 (ebits=4) or UE4M3/E4M3 value sets.  set_id: 0 = E2M1_SET,
// 1 = E4M3_SET (8-bit), 2 = UE4M3_SET (8-bit), 3 = BF16_SET (16-bit).
uint32_t ref_fill_random(int set_id, uint8_t* enc, float* ref, int rows, int K, uint32_t seed) {
    const EncVal* set = E2M1_SET; int n = SETN(E2M1_SET); int ebits = 4;
    if (set_id == 1) { set = E4M3_SET; n = SETN(E4M3_SET); ebits = 8; }
    if (set_id == 2) { set = UE4M3_SET; n = SETN(UE4M3_SET); ebits = 8; }
    if (set_id == 3) { set = BF16_SET; n = SETN(BF16_SET); ebits = 16; }
    fill_random(enc, ref, rows, K, set, n, ebits, &seed);
    return seed;
}

// Value-set tables (encoding, value) for pinning.
int ref_value_set(int set_id, uint32_t* enc, float* val) {
    const EncVal* set = E2M1_SET; int n = SETN(E2M1_SET);
    if (set_id == 1) { set = E4M3_SET; n = SETN(E4M3_SET); }
    if (set_id == 2) { set = UE4M3_SET; n = SETN(UE4M3_SET); }
    if (set_id == 3) { set = BF16_SET; n = SETN(BF16_SET); }
    if (set_id == 4) { set = UE8M0_SET; n = SETN(UE8M0_SET); }
    for (int i = 0; i < n; i++) { if (enc) enc[i] = set[i].enc; if (val) val[i] = set[i].val; }
    return n;
}

void ref_cpu_gemm_ref(const float* A, const float* B, float* D, int M, int N, int K) {
    cpu_gemm_ref(A, B, D, M, N, K);
}

void ref_cpu_gemm_ref_bs(const float* A, const float* B, float* D, int M, int N, int K,
                         const float* sfa, const float* sfb, int nseg) {
    cpu_gemm_ref_bs(A, B, D, M, N, K, sfa, sfb, nseg);
}

// The same function over row slices on `nthreads` host threads (the reference code itself
// is single-threaded; only the partition is added here, for the timed CPU baseline).
void ref_cpu_gemm_ref_bs_threads(const float* A, const float* B, float* D, int M, int N, int K,
                                 const float* sfa, const float* sfb, int nseg, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    std::vector<std::thread> th;
    for (int t = 0; t < nthreads; t++) {
        const int m0 = M * t / nthreads, m1 = M * (t + 1) / nthreads;
        if (m1 <= m0) continue;
        th.emplace_back([=] {
            cpu_gemm_ref_bs(A + (size_t)m0 * K, B, D + (size_t)m0 * N, m1 - m0, N, K, sfa, sfb, nseg);
        });
    }
    for (auto& x : th) x.join();
}

void ref_to_core_matrix(uint8_t* buf, int rows) { vr_to_core_matrix(buf, rows); }

int ref_check_exact(const float* got, const float* want, int n) {
    return check_exact(got, want, n, "ref");
}

// Runs the reference vr_verify driver with a CPU "device" that computes the right answer
// for a no-probe, linear-output spec (used to pin include/verify_random.h's driver).
static int g_M, g_N, g_K, g_nseg;
static void cpu_run(const uint8_t* hA, const uint8_t* hB, const uint32_t* sfa,
                    const uint32_t* sfb, void* out) {
    static float a[256 * 64], b[256 * 64], fa[8], fb[8];
    static const float mag[8] = {0.f, .5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
    for (int r = 0; r < g_M; r++)
        for (int k = 0; k < g_K; k++) {
            const int i = r * g_K + k; uint8_t c = (hA[i / 2] >> ((i & 1) * 4)) & 0xF;
            a[i] = (c & 8) ? -mag[c & 7] : mag[c & 7];
        }
    for (int r = 0; r < g_N; r++)
        for (int k = 0; k < g_K; k++) {
            const int i = r * g_K + k; uint8_t c = (hB[i / 2] >> ((i & 1) * 4)) & 0xF;
            b[i] = (c & 8) ? -mag[c & 7] : mag[c & 7];
        }
    for (int g = 0; g < g_nseg; g++) {
        for (int s = 0; s < SETN(UE4M3_SET); s++) {
            if (UE4M3_SET[s].enc == sfa[g]) fa[g] = UE4M3_SET[s].val;
            if (UE4M3_SET[s].enc == sfb[g]) fb[g] = UE4M3_SET[s].val;
        }
        if (sfa[g] == 0x38) fa[g] = 1.f;
        if (sfb[g] == 0x38) fb[g] = 1.f;
    }
    cpu_gemm_ref_bs(a, b, (float*)out, g_M, g_N, g_K, fa, fb, g_nseg);
}

int ref_vr_verify_cpu(int M, int N, int K, int nseg, uint32_t seed) {
    g_M = M; g_N = N; g_K = K; g_nseg = nseg;
    VrSpec sp{};
    sp.M = M; sp.N = N; sp.K = K; sp.ebits = 4; sp.is_int = 0;
    sp.dset = E2M1_SET; sp.dsetn = SETN(E2M1_SET);
    sp.sset = UE4M3_SET; sp.ssetn = SETN(UE4M3_SET); sp.nseg = nseg;
    sp.sf_one = 0x38; sp.core_matrix = 0; sp.probe = 0; sp.nslot = 0; sp.enc_tab = VR_ENC_E2M1;
    return vr_verify(sp, cpu_run, seed);
}

}  // extern "C"
