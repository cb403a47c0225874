"""The reference's own quantizer kernel run beside this project's on the same GPU, and the
differences between the two accounted for block by block.

oracle/_ref/libref_ar.so is built by oracle/Makefile from the unmodified reference header
blackwell/allreduce_sm100_sm120/nvfp4_allreduce.cuh (test infrastructure; nothing in the product
links it).  Its quantize_kernel (:427-454) computes per 16-element block

    scale_f = SF * (amax * rcp(6)),  scale = e4m3(scale_f),  inv = rcp(float(scale) * rcp(SF)),
    codes = e2m1(v * inv)                                  with rcp = rcp.approx.ftz.f32,

and this project computes the same chain with correctly rounded reciprocals (RCP6 = rn(1/6),
inv = SF * rn(1 / float(scale))), so that a CPU reproduces it.  The tests show, on all of cfg2
(8192 x 7168, N(0,1) with 0.1 % x50 outliers):

1. a model of the reference kernel -- the same chain on the CPU with the rcp.approx.ftz results
   measured on this GPU (diagnostics probe) in place of the rounded reciprocals -- reproduces the
   reference kernel's codes and scale bytes bit for bit, in every block;
2. every block in which this project's output differs from the reference kernel's is a block in
   which the two reciprocal chains give a different inverse scale (or, for a scale byte, a
   different scale_f); the count of such blocks is reported.
"""
import os

import numpy as np
import pytest
import torch

from tensorcore_ptx_example_b200 import diag, workloads

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
RCP6 = np.float32(np.uint32(0x3E2AAAAB).view(np.float32))


def _ref_lib():
    import py_oracle
    if not py_oracle.ref_ar_available():
        pytest.skip("oracle/_ref/libref_ar.so not built (needs the reference tree at build time)")
    return py_oracle.ref_ar_lib()


def _u16(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1)


def _gpu_rcp(values):
    """rcp.approx.ftz.f32 of each value, evaluated on this GPU; returns a dict value -> result."""
    v = np.unique(np.asarray(values, dtype=np.float32))
    r = diag.rcp_approx(torch.from_numpy(v).cuda()).cpu().numpy()
    return dict(zip(v.view(np.uint32).tolist(), r.tolist())), v, r


def _pack(codes):
    c = codes.reshape(-1)
    return (c[0::2] | (c[1::2] << 4)).astype(np.uint8)


def test_reference_quantizer_classified_against_ours(nv, oracle):
    import ctypes
    L = _ref_lib()
    rows, cols = workloads.CFG2_SHAPE
    numel = rows * cols
    x = workloads.activations(rows, cols, seed=2)
    amax = float(nv.amax(x).item())
    gs = nv.global_scale_from_amax(amax)
    sf_val = np.float32(1.0) / np.float32(gs)          # the reference's SFScaleVal = 1 / gs (= our gs_inv)

    # the reference kernel (linear layout: packed, then one scale byte per 16 elements, then SF)
    out = torch.zeros(int(L.ref_layout_total_bytes(numel)), dtype=torch.uint8, device="cuda")
    rc = L.ref_quantize(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(out.data_ptr()), numel, float(sf_val),
                        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    # this project's kernel
    packed, sf, _ = nv.quantize(x, gs)
    torch.cuda.synchronize()
    assert nv.device_status() == 0
    ref = out.cpu().numpy()
    ref_packed, ref_scales = ref[: numel // 2], ref[numel // 2: numel // 2 + numel // 16]
    ours_packed = packed.cpu().numpy().reshape(-1)
    ours_scales = sf.cpu().numpy()[oracle.sf_offsets(rows, cols).reshape(-1)]

    # ---- model of the reference kernel on the CPU, with the GPU's rcp.approx.ftz values
    xu = _u16(x)
    xf = (xu.astype(np.uint32) << 16).view(np.float32).reshape(-1, 16)
    amax_b = np.abs(xf).max(axis=1)
    tab, _, _ = _gpu_rcp([6.0, sf_val])
    r6 = np.float32(tab[int(np.float32(6.0).view(np.uint32))])
    rsf = np.float32(tab[int(np.float32(sf_val).view(np.uint32))])
    scale_f_ref = (sf_val * (amax_b * r6).astype(np.float32)).astype(np.float32)
    code_ref = oracle.e4m3_encode(scale_f_ref)
    e4 = oracle.e4m3_table()
    sq_ref = e4[code_ref]
    t = (sq_ref * rsf).astype(np.float32)
    tab_t, tv, tr = _gpu_rcp(t)
    inv_ref = tr[np.searchsorted(tv, t)].astype(np.float32)
    inv_ref[amax_b == 0] = np.float32(0)
    assert np.all(np.isfinite(inv_ref)), "a non-zero block with a zero scale (rcp of 0) is outside the model"
    y = (xf * inv_ref[:, None]).astype(np.float32)
    model_packed = _pack(oracle.e2m1_encode(y).reshape(-1, 16))
    assert np.array_equal(code_ref.astype(np.uint8), ref_scales), \
        f"model scale bytes differ from the reference kernel in {int(np.count_nonzero(code_ref != ref_scales))} blocks"
    assert np.array_equal(model_packed, ref_packed), \
        f"model codes differ from the reference kernel in {int(np.count_nonzero(model_packed != ref_packed))} bytes"

    # ---- this project's chain (the oracle) and the classification of every difference
    scale_f_ours = ((amax_b * RCP6).astype(np.float32) * sf_val).astype(np.float32)
    code_ours = oracle.e4m3_encode(scale_f_ours)
    sq_ours = e4[code_ours]
    with np.errstate(divide="ignore"):
        inv_ours = np.where(sq_ours != 0, (sf_val * (np.float32(1) / sq_ours).astype(np.float32)), 0).astype(np.float32)
    nblocks = numel // 16
    diff_scale = ours_scales != ref_scales
    diff_codes = (ours_packed.reshape(nblocks, 8) != ref_packed.reshape(nblocks, 8)).any(axis=1)
    diff = diff_scale | diff_codes
    inv_differs = inv_ours.view(np.uint32) != inv_ref.view(np.uint32)
    scale_f_differs = scale_f_ours.view(np.uint32) != scale_f_ref.view(np.uint32)
    unexplained = diff & ~(inv_differs | (diff_scale & scale_f_differs))
    report = {"blocks": nblocks, "differing_blocks": int(diff.sum()), "differing_scale_bytes": int(diff_scale.sum()),
              "blocks_with_other_inverse_scale": int(inv_differs.sum()),
              "rcp_approx_6_equals_rn": bool(r6 == RCP6), "unexplained": int(unexplained.sum())}
    print("reference quantize_kernel vs this project on cfg2:", report)
    assert report["unexplained"] == 0, report
