"""Generate the golden fixtures in this directory from the REFERENCE's own CPU oracle.

    make -C oracle ref && python tests/golden/make_golden.py

Loads oracle/_ref/libref_verify.so, which is the reference's unmodified
random_cpu_ref/verify_random.h compiled through oracle/ref_verify_shim.cpp, and records:

  xorshift.npz        xorshift streams for several seeds (verify_random.h:63)
  fill_random.npz     fill_random encodings / values for the E2M1, E4M3, UE4M3 and BF16
                      value sets (verify_random.h:79), plus the final RNG state
  value_sets.npz      the value-set tables (verify_random.h:50-59, :141-150)
  gemm_ref.npz        cpu_gemm_ref and cpu_gemm_ref_bs outputs on value-set data
                      (verify_random.h:101-110, :154-169)
  core_matrix.npz     vr_to_core_matrix input / output pairs (verify_random.h:175-181)
  vr_verify.npz       return code of vr_verify driven by a correct CPU "device"

The fixtures pin this project's oracle (oracle/nvfp4_oracle.c) and its drop-in header
(include/verify_random.h) on machines where the reference tree is absent.
"""
import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import py_oracle  # noqa: E402


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def main():
    L = py_oracle.ref_lib()
    out = {}

    seeds = np.array([1, 2, 12345, 0xDEADBEEF, 0x7FFFFFFF], dtype=np.uint32)
    streams = np.zeros((len(seeds), 4096), dtype=np.uint32)
    for i, s in enumerate(seeds):
        L.ref_xorshift_stream(int(s), 4096, _p(streams[i]))
    np.savez_compressed(os.path.join(HERE, "xorshift.npz"), seeds=seeds, streams=streams)

    fr = {}
    for set_id, name, ebits in [(0, "e2m1", 4), (1, "e4m3", 8), (2, "ue4m3", 8), (3, "bf16", 16)]:
        rows, K, seed = 96, 64, 1
        nbytes = rows * K * ebits // 8
        enc = np.zeros(nbytes, dtype=np.uint8)
        ref = np.zeros(rows * K, dtype=np.float32)
        final = L.ref_fill_random(set_id, _p(enc), _p(ref), rows, K, seed)
        fr[f"{name}_enc"] = enc
        fr[f"{name}_ref"] = ref
        fr[f"{name}_final_seed"] = np.array([final], dtype=np.uint32)
    np.savez_compressed(os.path.join(HERE, "fill_random.npz"), **fr)

    vs = {}
    for set_id, name in [(0, "e2m1"), (1, "e4m3"), (2, "ue4m3"), (3, "bf16"), (4, "ue8m0")]:
        n = L.ref_value_set(set_id, None, None)
        enc = np.zeros(n, dtype=np.uint32)
        val = np.zeros(n, dtype=np.float32)
        L.ref_value_set(set_id, _p(enc), _p(val))
        vs[f"{name}_enc"], vs[f"{name}_val"] = enc, val
    np.savez_compressed(os.path.join(HERE, "value_sets.npz"), **vs)

    rng = np.random.default_rng(7)
    e2m1_vals = vs["e2m1_val"]
    ue4m3_vals = vs["ue4m3_val"]
    M, N, K, nseg = 64, 48, 64, 4
    A = rng.choice(e2m1_vals, size=(M, K)).astype(np.float32)
    B = rng.choice(e2m1_vals, size=(N, K)).astype(np.float32)
    sfa = rng.choice(ue4m3_vals, size=nseg).astype(np.float32)
    sfb = rng.choice(ue4m3_vals, size=nseg).astype(np.float32)
    D = np.zeros((M, N), dtype=np.float32)
    Dbs = np.zeros((M, N), dtype=np.float32)
    L.ref_cpu_gemm_ref(_p(A), _p(B), _p(D), M, N, K)
    L.ref_cpu_gemm_ref_bs(_p(A), _p(B), _p(Dbs), M, N, K, _p(sfa), _p(sfb), nseg)
    # A wide-range case where fp32 summation order matters (normal data, K=256).
    A2 = rng.standard_normal((M, 256)).astype(np.float32)
    B2 = rng.standard_normal((N, 256)).astype(np.float32)
    s2a = (2.0 ** rng.integers(-4, 5, size=8)).astype(np.float32)
    s2b = (2.0 ** rng.integers(-4, 5, size=8)).astype(np.float32)
    D2 = np.zeros((M, N), dtype=np.float32)
    L.ref_cpu_gemm_ref_bs(_p(A2), _p(B2), _p(D2), M, N, 256, _p(s2a), _p(s2b), 8)
    np.savez_compressed(os.path.join(HERE, "gemm_ref.npz"), A=A, B=B, sfa=sfa, sfb=sfb, D=D, Dbs=Dbs,
                        A2=A2, B2=B2, s2a=s2a, s2b=s2b, D2=D2)

    cm_in = rng.integers(0, 256, size=(4, 256 * 32), dtype=np.uint8)
    cm_out = cm_in.copy()
    rows = np.array([256, 128, 64, 16], dtype=np.int32)
    for i in range(4):
        buf = np.ascontiguousarray(cm_out[i])
        L.ref_to_core_matrix(_p(buf), int(rows[i]))
        cm_out[i] = buf
    np.savez_compressed(os.path.join(HERE, "core_matrix.npz"), inputs=cm_in, outputs=cm_out, rows=rows)

    # vr_verify with a correct CPU device: return codes for a few shapes/seeds.
    cases = np.array([[128, 256, 64, 4, 1], [64, 64, 64, 2, 3], [128, 16, 64, 1, 9]], dtype=np.int64)
    rcs = np.array([L.ref_vr_verify_cpu(*[int(v) for v in c]) for c in cases], dtype=np.int32)
    np.savez_compressed(os.path.join(HERE, "vr_verify.npz"), cases=cases, rc=rcs)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
