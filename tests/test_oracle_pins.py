"""Pin the oracle and the drop-in test header against the reference itself.

The golden fixtures (tests/golden/*.npz) were produced by the reference's own
random_cpu_ref/verify_random.h compiled into oracle/_ref (script: tests/golden/make_golden.py).
When oracle/_ref is present (the build container), the same checks also run live against it.
CPU only.
"""
import ctypes
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
SHIM_SRC = os.path.join(ROOT, "tests", "host", "vr_header_shim.cpp")
SHIM_SO = os.path.join(ROOT, "tests", "host", "_build", "libvr_header_shim.so")


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def g(name):
    return np.load(os.path.join(GOLDEN, name))


@pytest.fixture(scope="module")
def vh():
    """include/verify_random.h compiled as a host shared library."""
    os.makedirs(os.path.dirname(SHIM_SO), exist_ok=True)
    if not os.path.exists(SHIM_SO) or os.path.getmtime(SHIM_SO) < max(
            os.path.getmtime(SHIM_SRC), os.path.getmtime(os.path.join(ROOT, "include", "verify_random.h"))):
        subprocess.run(["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-ffp-contract=off",
                        "-I", os.path.join(ROOT, "include"), "-o", SHIM_SO, SHIM_SRC], check=True)
    L = ctypes.CDLL(SHIM_SO)
    P = ctypes.c_void_p
    L.vh_xorshift_stream.restype = ctypes.c_uint32
    L.vh_xorshift_stream.argtypes = [ctypes.c_uint32, ctypes.c_int, P]
    L.vh_fill_random.restype = ctypes.c_uint32
    L.vh_fill_random.argtypes = [ctypes.c_int, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_uint32]
    L.vh_value_set.restype = ctypes.c_int
    L.vh_value_set.argtypes = [ctypes.c_int, P, P]
    L.vh_cpu_gemm_ref.argtypes = [P, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    L.vh_cpu_gemm_ref_bs.argtypes = [P, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, P, ctypes.c_int]
    L.vh_to_core_matrix.argtypes = [P, ctypes.c_int]
    L.vh_vr_verify_cpu.restype = ctypes.c_int
    L.vh_vr_verify_cpu.argtypes = [ctypes.c_int] * 4 + [ctypes.c_uint32]
    L.vh_vr_verify_wrong.restype = ctypes.c_int
    L.vh_vr_verify_wrong.argtypes = [ctypes.c_int] * 4 + [ctypes.c_uint32]
    L.vh_gemm_ref_blockscaled.argtypes = [P, P, P, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    return L


# ------------------------------------------------------------- xorshift ----
def test_oracle_xorshift_matches_reference_stream(oracle):
    d = g("xorshift.npz")
    L = oracle.lib()
    for seed, stream in zip(d["seeds"], d["streams"]):
        s = ctypes.c_uint32(int(seed))
        got = np.array([L.orc_xorshift(ctypes.byref(s)) for _ in range(stream.size)], dtype=np.uint32)
        assert np.array_equal(got, stream)


def test_header_xorshift_matches_reference_stream(vh):
    d = g("xorshift.npz")
    for seed, stream in zip(d["seeds"], d["streams"]):
        got = np.zeros(stream.size, dtype=np.uint32)
        vh.vh_xorshift_stream(int(seed), stream.size, _p(got))
        assert np.array_equal(got, stream)


# ---------------------------------------------------------- fill_random ----
@pytest.mark.parametrize("set_id,name,ebits", [(0, "e2m1", 4), (1, "e4m3", 8), (2, "ue4m3", 8), (3, "bf16", 16)])
def test_header_fill_random_matches_reference(vh, set_id, name, ebits):
    d = g("fill_random.npz")
    rows, K = 96, 64
    enc = np.zeros(rows * K * ebits // 8, dtype=np.uint8)
    ref = np.zeros(rows * K, dtype=np.float32)
    final = vh.vh_fill_random(set_id, _p(enc), _p(ref), rows, K, 1)
    assert np.array_equal(enc, d[f"{name}_enc"])
    assert np.array_equal(ref, d[f"{name}_ref"])
    assert final == int(d[f"{name}_final_seed"][0])


def test_value_sets_match_reference(vh, oracle):
    d = g("value_sets.npz")
    for set_id, name in [(0, "e2m1"), (1, "e4m3"), (2, "ue4m3"), (3, "bf16"), (4, "ue8m0")]:
        n = vh.vh_value_set(set_id, None, None)
        enc = np.zeros(n, dtype=np.uint32)
        val = np.zeros(n, dtype=np.float32)
        vh.vh_value_set(set_id, _p(enc), _p(val))
        assert np.array_equal(enc, d[f"{name}_enc"]) and np.array_equal(val, d[f"{name}_val"])
    # the oracle's codecs decode every reference table entry to the tabled value
    L = oracle.lib()
    for e, v in zip(d["e2m1_enc"], d["e2m1_val"]):
        assert L.orc_e2m1_decode(int(e)) == v and L.orc_e2m1_encode(float(v)) == e
    for e, v in zip(d["ue4m3_enc"], d["ue4m3_val"]):
        assert L.orc_e4m3_decode(int(e)) == v and L.orc_e4m3_encode(float(v)) == e
    for e, v in zip(d["e4m3_enc"], d["e4m3_val"]):
        if v != 0:
            assert L.orc_e4m3_decode(int(e)) == v and L.orc_e4m3_encode(float(v)) == e


# ------------------------------------------------------------- GEMM refs ----
def test_header_gemm_refs_match_reference(vh):
    d = g("gemm_ref.npz")
    A, B = d["A"], d["B"]
    M, K = A.shape
    N = B.shape[0]
    D = np.zeros((M, N), dtype=np.float32)
    vh.vh_cpu_gemm_ref(_p(A), _p(B), _p(D), M, N, K)
    assert np.array_equal(D, d["D"])
    vh.vh_cpu_gemm_ref_bs(_p(A), _p(B), _p(D), M, N, K, _p(d["sfa"]), _p(d["sfb"]), 4)
    assert np.array_equal(D, d["Dbs"])
    # order-sensitive case: identical fp32 summation order required for ==
    A2, B2 = d["A2"], d["B2"]
    D2 = np.zeros((M, N), dtype=np.float32)
    vh.vh_cpu_gemm_ref_bs(_p(A2), _p(B2), _p(D2), M, N, 256, _p(d["s2a"]), _p(d["s2b"]), 8)
    assert np.array_equal(D2, d["D2"])


def test_oracle_gemm_matches_reference_on_value_sets(oracle):
    """On the reference's restricted value sets every summation order is exact, so every
    accumulation model of the oracle must reproduce cpu_gemm_ref_bs bit for bit."""
    d = g("gemm_ref.npz")
    A, B, sfa, sfb = d["A"], d["B"], d["sfa"], d["sfb"]
    M, K = A.shape
    N = B.shape[0]
    codes_a = oracle.e2m1_encode(A).reshape(M, K)
    codes_b = oracle.e2m1_encode(B).reshape(N, K)
    pa = (codes_a[:, 0::2] | (codes_a[:, 1::2] << 4)).astype(np.uint8)
    pb = (codes_b[:, 0::2] | (codes_b[:, 1::2] << 4)).astype(np.uint8)
    Kp = 256  # pad K with zero data
    pa = np.concatenate([pa, np.zeros((M, (Kp - K) // 2), np.uint8)], axis=1)
    pb = np.concatenate([pb, np.zeros((N, (Kp - K) // 2), np.uint8)], axis=1)
    sa = np.full(oracle.sf_bytes(M, Kp), 0x38, np.uint8)
    sb = np.full(oracle.sf_bytes(N, Kp), 0x38, np.uint8)
    oa, ob = oracle.sf_offsets(M, Kp), oracle.sf_offsets(N, Kp)
    ea = oracle.e4m3_encode(sfa)
    eb = oracle.e4m3_encode(sfb)
    for kb in range(K // 16):
        sa[oa[:, kb]] = ea[kb]
        sb[ob[:, kb]] = eb[kb]
    for model in range(4):
        D = oracle.gemm_f32(pa, sa, pb, sb, M, N, Kp, model=model)
        assert np.array_equal(D, d["Dbs"]), model


# ---------------------------------------------------------- core matrix ----
def test_header_core_matrix_matches_reference(vh):
    d = g("core_matrix.npz")
    for inp, outp, rows in zip(d["inputs"], d["outputs"], d["rows"]):
        buf = np.ascontiguousarray(inp.copy())
        vh.vh_to_core_matrix(_p(buf), int(rows))
        assert np.array_equal(buf, outp)


# ------------------------------------------------------------- vr_verify ----
def test_header_vr_verify_driver(vh):
    d = g("vr_verify.npz")
    for case, rc in zip(d["cases"], d["rc"]):
        assert vh.vh_vr_verify_cpu(*[int(v) for v in case]) == rc == 0
    # a device that is wrong in one slot must be caught
    assert vh.vh_vr_verify_wrong(128, 256, 64, 4, 1) == 1


def test_header_blockscaled_ref_matches_oracle(vh, oracle):
    """vr_gemm_ref_blockscaled (header addition) == oracle hardware model on full-range
    codes and per-(row, block) power-of-two scales (the cfg1 tile data)."""
    rng = np.random.default_rng(3)
    M, N, K = 32, 48, 256
    ca = rng.integers(0, 16, size=(M, K)).astype(np.uint8)
    cb = rng.integers(0, 16, size=(N, K)).astype(np.uint8)
    va = oracle.E2M1_TABLE[ca]
    vb = oracle.E2M1_TABLE[cb]
    ua = rng.integers(-4, 5, size=(M, K // 16))
    ub = rng.integers(-4, 5, size=(N, K // 16))
    ea = oracle.e4m3_encode((2.0 ** ua).astype(np.float32)).reshape(M, K // 16)
    eb = oracle.e4m3_encode((2.0 ** ub).astype(np.float32)).reshape(N, K // 16)
    D = np.zeros((M, N), dtype=np.float32)
    vh.vh_gemm_ref_blockscaled(_p(np.ascontiguousarray(va)), _p(np.ascontiguousarray(vb)),
                               _p(np.ascontiguousarray(ea)), _p(np.ascontiguousarray(eb)), _p(D), M, N, K)
    pa = (ca[:, 0::2] | (ca[:, 1::2] << 4)).astype(np.uint8)
    pb = (cb[:, 0::2] | (cb[:, 1::2] << 4)).astype(np.uint8)
    sa = np.zeros(oracle.sf_bytes(M, K), np.uint8)
    sb = np.zeros(oracle.sf_bytes(N, K), np.uint8)
    sa[oracle.sf_offsets(M, K)] = ea
    sb[oracle.sf_offsets(N, K)] = eb
    Do = oracle.gemm_f32(pa, sa, pb, sb, M, N, K, model=oracle.ACC_TCGEN05)
    assert np.array_equal(D, Do)


# ------------------------------------------- live checks against oracle/_ref ----
ref_available = pytest.mark.skipif(not os.path.exists(os.path.join(ROOT, "oracle", "_ref", "libref_verify.so")),
                                   reason="oracle/_ref not built (reference tree absent)")


@ref_available
def test_live_reference_fill_and_gemm(oracle):
    R = oracle.ref_lib()
    rng = np.random.default_rng(11)
    for seed in rng.integers(1, 2**31, size=5):
        enc = np.zeros(128 * 64 // 2, np.uint8)
        ref = np.zeros(128 * 64, np.float32)
        R.ref_fill_random(0, _p(enc), _p(ref), 128, 64, int(seed))
        s = ctypes.c_uint32(int(seed))
        L = oracle.lib()
        draws = np.array([L.orc_xorshift(ctypes.byref(s)) for _ in range(128 * 64)], dtype=np.uint32)
        table = g("value_sets.npz")["e2m1_val"]
        assert np.array_equal(ref, table[draws % len(table)])


# --------------------------------------- tcgen05 arithmetic, pinned on B200 ----
def test_oracle_tcgen05_model_reproduces_b200_outputs(oracle):
    """tests/golden/tcgen05_b200_outputs.npz holds raw fp32 outputs of a stand-alone single-tile
    tcgen05 probe measured on a B200 (nvfp4_diag_mma_tile, independent of the production GEMM;
    script: tests/golden/make_tcgen05_fixture.py).  The oracle's hardware model must reproduce
    all of them bit for bit, and the simpler round-to-nearest models must not (they are what the
    hardware does NOT do)."""
    import sys
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from test_gemm_gpu import cfg1_tile
    d = np.load(os.path.join(GOLDEN, "tcgen05_b200_outputs.npz"))
    M, N, K = 128, 256, 256
    rne_mismatch = 0
    for name in ["P1", "P2", "P3", "P4", "P5", "P6", "P7", "P8", "X1", "X2", "X3", "X4"]:
        args = (d[name + "_pa"], d[name + "_sa"], d["pb_ones"], d[name + "_sb"], M, N, K)
        got = oracle.gemm_f32(*args, model=oracle.ACC_TCGEN05)
        assert np.array_equal(got, d[name]), name
        rne_mismatch += int(np.count_nonzero(oracle.gemm_f32(*args, model=oracle.ACC_EXACT_PER_MMA) != d[name]))
    for seed in range(1, 5):
        pa, sa, pb, sb = cfg1_tile(oracle, seed)
        assert np.array_equal(oracle.gemm_f32(pa, sa, pb, sb, M, N, K, model=oracle.ACC_TCGEN05), d[f"cfg1_{seed}"])
    assert rne_mismatch > 1000
