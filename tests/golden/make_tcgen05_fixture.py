"""Regenerate tests/golden/tcgen05_b200_outputs.npz on a B200 (GPU needed).

    python tests/golden/make_tcgen05_fixture.py [out.npz]

Runs the stand-alone single-tile probe of the diagnostics library (nvfp4_diag_mma_tile: one CTA,
operands in the no-swizzle core-matrix layout loaded with plain loads, scales placed with
tcgen05.cp, four K64 MMAs, tcgen05.ld read-back) -- not the production GEMM, whose parity the
fixture is used to check -- on experiments that expose the arithmetic of tcgen05.mma
kind::mxf4nvf4.block_scale.scale_vec::4X, and stores the raw fp32 outputs:
  cfg1_<seed>      cfg1 tiles (M128 N256 K256, all 16 E2M1 codes, scales 2^[-4,4])
  P1..P4           one K step: +big, -big and a small term in varying block positions
                   (exactness of the in-step sum over >= 38 bits)
  P5..P8           one K step: big +- small (rounding direction of the step result)
  X1..X4           big and small in two different K steps (width of the accumulate step)
The oracle model ORC_ACC_TCGEN05 must reproduce every value (tests/test_oracle_pins.py); the
production GEMM is then checked against that model (tests/test_gemm_gpu.py).  As a consistency
check the script also runs the production kernel on every experiment and reports whether it
agrees with the probe (the fixture holds the probe's outputs either way).
"""
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path[:0] = [ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")]
import py_oracle as po  # noqa: E402
import tensorcore_ptx_example_b200 as nv  # noqa: E402
from tensorcore_ptx_example_b200 import diag  # noqa: E402
from test_gemm_gpu import cfg1_tile  # noqa: E402  (same generator as the GPU tests)

OUT_PATH = sys.argv[1] if len(sys.argv) > 1 else os.path.join(ROOT, "tests", "golden", "tcgen05_b200_outputs.npz")



PRODUCTION_AGREES = []


def run(pa, sa, pb, sb, M, N, K):
    assert (M, N, K) == (128, 256, 256)
    t = [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (pa, sa, pb, sb)]
    D = diag.mma_tile(t[0], t[1], t[2], t[3])
    P = nv.gemm_f32(t[0], t[1], t[2], t[3], M, N, K)
    torch.cuda.synchronize()
    assert diag.device_status() == 0 and nv.device_status() == 0
    D = D.cpu().numpy()
    PRODUCTION_AGREES.append(bool(np.array_equal(D, P.cpu().numpy())))
    return D


def pack(codes):
    return (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)


def sf_from(scales_rows):  # [rows, K/16] float -> tcgen05 layout bytes
    rows, nkb = scales_rows.shape
    K = nkb * 16
    enc = po.e4m3_encode(scales_rows.astype(np.float32)).reshape(rows, nkb)
    sf = np.zeros(po.sf_bytes(rows, K), np.uint8)
    sf[po.sf_offsets(rows, K)] = enc
    return sf


res = {}
# E1: cfg1 random tiles
for seed in range(1, 5):
    pa, sa, pb, sb = cfg1_tile(po, seed)
    res[f"cfg1_{seed}"] = run(pa, sa, pb, sb, 128, 256, 256)

# E2: structured single-MMA experiments.  B = 1.0 everywhere; D[m][n] = sum_kb SA[m][kb]*sfa[m][kb]*sfb[n][kb]
M, N, K = 128, 256, 256
e4 = po.e4m3_table()
pos_scales = np.sort(np.unique(e4[1:0x7F][~np.isnan(e4[1:0x7F])]))   # 125 positive finite values
code_of = {1.0: 2, 1.5: 3, 2.0: 4, 3.0: 5, 4.0: 6, 6.0: 7, 0.5: 1, -1.0: 10, -1.5: 11, -6.0: 15, 6.0: 7}


def a_codes(block_vals):
    """A rows: per (row, block) a single nonzero value at the block's first element."""
    rows, nkb = block_vals.shape
    codes = np.zeros((rows, nkb * 16), np.uint8)
    for r in range(rows):
        for b in range(nkb):
            v = float(block_vals[r, b])
            if v != 0:
                c = po.e2m1_encode(np.array([v], np.float32))[0]
                assert po.E2M1_TABLE[c] == v, v
                codes[r, b * 16] = c
    return codes


b_codes = np.full((N, K), 2, np.uint8)   # all 1.0
pb = pack(b_codes)
layouts = {
    "P1": ([6, -6, 1, 0], [0, 1, 2, 3]),
    "P2": ([6, 1, -6, 0], None),
    "P3": ([1, 6, 0, -6], None),
    "P4": ([1, 0, 6, -6], None),
    "P5": ([6, 0, 1, 0], None),   # no cancel: big + small, rounding direction
    "P6": ([6, 1.5, 0, 0], None),
    "P7": ([6, -1.5, 0, 0], None),
    "P8": ([-6, 1.5, 0, 0], None),
}
for name, (vals, _) in layouts.items():
    bv = np.zeros((M, K // 16), np.float32)
    bv[:, 0:4] = np.array(vals, np.float32)[None, :]
    pa = pack(a_codes(bv))
    # row m: small-term scale s_m (sweep over pos_scales); big blocks use 448
    sA = np.ones((M, K // 16), np.float32)
    for bi, v in enumerate(vals):
        if abs(v) == 6:
            sA[:, bi] = 448.0
    small_idx = [i for i, v in enumerate(vals) if v != 0 and abs(v) != 6][0]
    sA[:, small_idx] = pos_scales[np.linspace(0, len(pos_scales) - 1, M).astype(int)]
    sB = np.ones((N, K // 16), np.float32)
    for bi, v in enumerate(vals):
        if abs(v) == 6:
            sB[:, bi] = 448.0
    sB[:, small_idx] = pos_scales[np.arange(N) % len(pos_scales)]
    sa, sb = sf_from(sA), sf_from(sB)
    res[f"{name}_pa"], res[f"{name}_sa"], res[f"{name}_sb"] = pa, sa, sb
    res[name] = run(pa, sa, pb, sb, M, N, K)

# E3: cross-MMA accumulation: k-step 0 gives big, k-step 1 gives small (separate MMAs)
for name, (v0, v1) in {"X1": (6, 1), "X2": (6, 1.5), "X3": (-6, 1.5), "X4": (1, 6)}.items():
    bv = np.zeros((M, K // 16), np.float32)
    bv[:, 0] = v0
    bv[:, 4] = v1
    pa = pack(a_codes(bv))
    sA = np.ones((M, K // 16), np.float32)
    sB = np.ones((N, K // 16), np.float32)
    big_b, small_b = (0, 4) if abs(v0) == 6 else (4, 0)
    sA[:, big_b] = 448.0
    sB[:, big_b] = 448.0
    sA[:, small_b] = pos_scales[np.linspace(0, len(pos_scales) - 1, M).astype(int)]
    sB[:, small_b] = pos_scales[np.arange(N) % len(pos_scales)]
    sa, sb = sf_from(sA), sf_from(sB)
    res[f"{name}_pa"], res[f"{name}_sa"], res[f"{name}_sb"] = pa, sa, sb
    res[name] = run(pa, sa, pb, sb, M, N, K)
res["pb_ones"] = pb
res["source"] = np.array("nvfp4_diag_mma_tile (stand-alone single-CTA probe)")
np.savez_compressed(OUT_PATH, **res)
print("saved", len(res), "arrays; production GEMM agrees with the probe on",
      sum(PRODUCTION_AGREES), "of", len(PRODUCTION_AGREES), "experiments")
