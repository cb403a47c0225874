// vr_header_shim.cpp -- exposes include/verify_random.h (this project's drop-in rewrite of
// the reference test driver) as a C ABI so tests/test_oracle_pins.py can compare it with
// the reference's own header (golden fixtures in tests/golden/).  Host-only, test-only.
#include <cstdint>

#include "verify_random.h"

extern "C" {

uint32_t vh_xorshift_stream(uint32_t seed, int n, uint32_t* out) {
    for (int i = 0; i < n; i++) out[i] = xorshift(&seed);
    return seed;
}

uint32_t vh_fill_random(int set_id, uint8_t* enc, float* ref, int rows, int K, uint32_t seed) {
    const EncVal* set = E2M1_SET; int n = SETN(E2M1_SET); int ebits = 4;
    if (set_id == 1) { set = E4M3_SET; n = SETN(E4M3_SET); ebits = 8; }
    if (set_id == 2) { set = UE4M3_SET; n = SETN(UE4M3_SET); ebits = 8; }
    if (set_id == 3) { set = BF16_SET; n = SETN(BF16_SET); ebits = 16; }
    fill_random(enc, ref, rows, K, set, n, ebits, &seed);
    return seed;
}

int vh_value_set(int set_id, uint32_t* enc, float* val) {
    const EncVal* set = E2M1_SET; int n = SETN(E2M1_SET);
    if (set_id == 1) { set = E4M3_SET; n = SETN(E4M3_SET); }
    if (set_id == 2) { set = UE4M3_SET; n = SETN(UE4M3_SET); }
    if (set_id == 3) { set = BF16_SET; n = SETN(BF16_SET); }
    if (set_id == 4) { set = UE8M0_SET; n = SETN(UE8M0_SET); }
    for (int i = 0; i < n; i++) { if (enc) enc[i] = set[i].enc; if (val) val[i] = set[i].val; }
    return n;
}

void vh_cpu_gemm_ref(const float* A, const float* B, float* D, int M, int N, int K) { cpu_gemm_ref(A, B, D, M, N, K); }

void vh_cpu_gemm_ref_bs(const float* A, const float* B, float* D, int M, int N, int K, const float* sfa,
                        const float* sfb, int nseg) {
    cpu_gemm_ref_bs(A, B, D, M, N, K, sfa, sfb, nseg);
}

void vh_to_core_matrix(uint8_t* buf, int rows) { vr_to_core_matrix(buf, rows); }

static int g_M, g_N, g_K, g_nseg;
static void cpu_run(const uint8_t* hA, const uint8_t* hB, const uint32_t* sfa, const uint32_t* sfb, void* out) {
    static float a[256 * 64], b[256 * 64], fa[8], fb[8];
    static const float mag[8] = {0.f, .5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
    for (int i = 0; i < g_M * g_K; i++) { uint8_t c = (hA[i / 2] >> ((i & 1) * 4)) & 0xF; a[i] = (c & 8) ? -mag[c & 7] : mag[c & 7]; }
    for (int i = 0; i < g_N * g_K; i++) { uint8_t c = (hB[i / 2] >> ((i & 1) * 4)) & 0xF; b[i] = (c & 8) ? -mag[c & 7] : mag[c & 7]; }
    for (int g = 0; g < g_nseg; g++) { fa[g] = vr_ue4m3((uint8_t)sfa[g]); fb[g] = vr_ue4m3((uint8_t)sfb[g]); }
    cpu_gemm_ref_bs(a, b, (float*)out, g_M, g_N, g_K, fa, fb, g_nseg);
}

int vh_vr_verify_cpu(int M, int N, int K, int nseg, uint32_t seed) {
    g_M = M; g_N = N; g_K = K; g_nseg = nseg;
    VrSpec sp{};
    sp.M = M; sp.N = N; sp.K = K; sp.ebits = 4; sp.is_int = 0;
    sp.dset = E2M1_SET; sp.dsetn = SETN(E2M1_SET);
    sp.sset = UE4M3_SET; sp.ssetn = SETN(UE4M3_SET); sp.nseg = nseg;
    sp.sf_one = 0x38; sp.core_matrix = 0; sp.probe = 0; sp.nslot = 0; sp.enc_tab = VR_ENC_E2M1;
    return vr_verify(sp, cpu_run, seed);
}

// A deliberately wrong device (off by one slot) must make vr_verify fail.
static void wrong_run(const uint8_t* hA, const uint8_t* hB, const uint32_t* sfa, const uint32_t* sfb, void* out) {
    cpu_run(hA, hB, sfa, sfb, out);
    ((float*)out)[5] += 0.5f;
}

int vh_vr_verify_wrong(int M, int N, int K, int nseg, uint32_t seed) {
    g_M = M; g_N = N; g_K = K; g_nseg = nseg;
    VrSpec sp{};
    sp.M = M; sp.N = N; sp.K = K; sp.ebits = 4; sp.is_int = 0;
    sp.dset = E2M1_SET; sp.dsetn = SETN(E2M1_SET);
    sp.sset = UE4M3_SET; sp.ssetn = SETN(UE4M3_SET); sp.nseg = nseg;
    sp.sf_one = 0x38; sp.core_matrix = 0; sp.probe = 0; sp.nslot = 0; sp.enc_tab = VR_ENC_E2M1;
    return vr_verify(sp, wrong_run, seed);
}

void vh_gemm_ref_blockscaled(const float* A, const float* B, const uint8_t* sfa, const uint8_t* sfb, float* D, int M,
                             int N, int K) {
    vr_gemm_ref_blockscaled(A, B, sfa, sfb, D, M, N, K);
}

}  // extern "C"
