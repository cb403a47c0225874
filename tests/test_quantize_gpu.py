"""Quantizer parity on the GPU: the CUDA kernels against the CPU oracle, bit for bit.

Covers the hardware codec conversions (E2M1 / E4M3 cvt) over threshold neighbourhoods and
wide sweeps, the quantizer at small / ragged / full cfg2 (8192 x 7168) shapes, the on-device
global-scale path, amax, dequantization and edge cases (zeros, subnormals, signed zeros,
saturation).  All comparisons are exact (integer and byte outputs)."""
import numpy as np
import pytest
import torch

from tensorcore_ptx_example_b200 import diag, workloads

pytestmark = pytest.mark.gpu


def to_np_u16(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def from_np_u16(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).cuda()


def neighbourhood(centres, ulps):
    c = np.asarray(centres, dtype=np.float32)
    u = c.view(np.int32).astype(np.int64)
    offs = np.arange(-ulps, ulps + 1, dtype=np.int64)
    v = (u[:, None] + offs[None, :]).ravel()
    v = v[(v >= 0) & (v < 0x7F800000)]
    return v.astype(np.int32).view(np.float32)


# ------------------------------------------------------------------ codecs ----
def test_e2m1_cvt_matches_oracle(nv, oracle):
    rng = np.random.default_rng(1)
    thresholds = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0]
    pos = np.concatenate([
        neighbourhood(thresholds, 4096),
        rng.uniform(0, 8, 2_000_000).astype(np.float32),
        (2.0 ** rng.uniform(-30, 20, 500_000)).astype(np.float32),
        np.array([0.0, 1e-45, 1e-38, 7.0, 100.0, 3e38], dtype=np.float32),
        # every bf16 bit pattern that is a finite non-negative float
        (np.arange(0, 0x7F80, dtype=np.uint32) << 16).view(np.float32),
    ])
    x = np.concatenate([pos, -pos]).astype(np.float32)
    got = diag.e2m1_encode(torch.from_numpy(x).cuda()).cpu().numpy()
    torch.cuda.synchronize()
    want = oracle.e2m1_encode(x)
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, f"{bad.size} mismatches, first: x={x[bad[:8]]} gpu={got[bad[:8]]} cpu={want[bad[:8]]}"


def test_e4m3_cvt_matches_oracle(nv, oracle):
    rng = np.random.default_rng(2)
    tab = oracle.e4m3_table()
    finite = tab[:0x7F][~np.isnan(tab[:0x7F])]
    mids = ((finite[1:].astype(np.float64) + finite[:-1]) / 2).astype(np.float32)
    # every 16th float between 2^-12 and 2^10 covers the whole rounding range densely
    lo, hi = np.float32(2.0 ** -12).view(np.int32), np.float32(2.0 ** 10).view(np.int32)
    sweep = np.arange(lo, hi, 16, dtype=np.int32).view(np.float32)
    pos = np.concatenate([
        neighbourhood(np.concatenate([finite[1:], mids, [448.0, 464.0, 480.0]]), 2048),
        sweep,
        rng.uniform(0, 500, 1_000_000).astype(np.float32),
        np.array([0.0, 1e-45, 2.0 ** -10, 2.0 ** -9, 3 * 2.0 ** -11, 1e6, 3e38], dtype=np.float32),
    ])
    x = np.concatenate([pos, -pos]).astype(np.float32)
    got = diag.e4m3_encode(torch.from_numpy(x).cuda()).cpu().numpy()
    want = oracle.e4m3_encode(x)
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, f"{bad.size} mismatches, first: x={x[bad[:8]]} gpu={got[bad[:8]]} cpu={want[bad[:8]]}"


# ---------------------------------------------------------------- quantize ----
def check_quantize(nv, oracle, x_bf16, gs):
    rows, cols = x_bf16.shape
    packed, sf, _ = nv.quantize(x_bf16, gs)
    torch.cuda.synchronize()
    assert nv.device_status() == 0
    xu = to_np_u16(x_bf16)
    p_ref, s_ref = oracle.quantize_bf16(xu, gs)
    p = packed.cpu().numpy()
    s = sf.cpu().numpy()
    nbad_p = int(np.count_nonzero(p != p_ref))
    nbad_s = int(np.count_nonzero(s != s_ref))
    assert nbad_p == 0 and nbad_s == 0, f"packed mismatches {nbad_p}, scale mismatches {nbad_s}"
    return packed, sf


@pytest.mark.parametrize("rows,cols", [(128, 64), (256, 512), (300, 1024), (16, 8192), (1, 64), (1000, 7168)])
def test_quantize_bitexact(nv, oracle, rows, cols):
    x = workloads.activations(rows, cols, seed=rows * 7 + cols)
    gs, _ = oracle.global_scale(oracle.amax_bf16(to_np_u16(x)))
    check_quantize(nv, oracle, x, gs)


def test_quantize_cfg2_full_size_bitexact(nv, oracle):
    rows, cols = workloads.CFG2_SHAPE
    x = workloads.activations(rows, cols, seed=2)
    xu = to_np_u16(x)
    amax = oracle.amax_bf16(xu)
    gs, _ = oracle.global_scale(amax)
    check_quantize(nv, oracle, x, gs)


def test_quantize_auto_scale(nv, oracle):
    rows, cols = 512, 2048
    x = workloads.activations(rows, cols, seed=5)
    packed, sf, gs_dev = nv.quantize(x, None)
    torch.cuda.synchronize()
    gs_ref, _ = oracle.global_scale(oracle.amax_bf16(to_np_u16(x)))
    assert np.float32(gs_dev.item()) == np.float32(gs_ref)
    p_ref, s_ref = oracle.quantize_bf16(to_np_u16(x), gs_ref)
    assert np.array_equal(packed.cpu().numpy(), p_ref) and np.array_equal(sf.cpu().numpy(), s_ref)
    # second call through the same path gives the same bytes
    packed2, sf2, gs2 = nv.quantize(x, None)
    assert torch.equal(packed, packed2) and torch.equal(sf, sf2) and torch.equal(gs_dev, gs2)


def test_amax_exact(nv, oracle):
    for n, seed in [(8, 1), (4096, 2), (7168 * 8192, 3)]:
        x = workloads.activations(1, n, seed=seed) if n < 1 << 20 else workloads.activations(8192, 7168, seed)
        a = nv.amax(x.view(-1)).item()
        assert np.float32(a) == np.float32(oracle.amax_bf16(to_np_u16(x)))


def test_dequantize_bitexact(nv, oracle):
    rows, cols = 384, 1024
    x = workloads.activations(rows, cols, seed=9)
    gs, _ = oracle.global_scale(oracle.amax_bf16(to_np_u16(x)))
    packed, sf = check_quantize(nv, oracle, x, gs)
    y = nv.dequantize(packed, sf, rows, cols, gs)
    torch.cuda.synchronize()
    want = oracle.dequantize_bf16(packed.cpu().numpy(), sf.cpu().numpy(), rows, cols, gs)
    assert np.array_equal(to_np_u16(y), want)
    # NVFP4 error on N(0,1) with outliers: relative RMSE well under 0.15
    xf = x.float()
    rel = ((y.float() - xf).pow(2).mean().sqrt() / xf.pow(2).mean().sqrt()).item()
    assert rel < 0.15


def test_quantize_edge_cases(nv, oracle):
    rows, cols = 128, 256
    rng = np.random.default_rng(4)
    x = oracle.f32_to_bf16(rng.standard_normal((rows, cols)).astype(np.float32))
    x[0, :] = 0                                  # whole row of zero blocks
    x[1, :16] = 0x8000                           # negative zeros
    x[2, :] = 0x0001                             # smallest bf16 subnormal
    x[3, :16] = 0x7F7F                           # largest finite bf16
    x[4, 16:32] = oracle.f32_to_bf16(np.full(16, -3.0, np.float32))
    x[5, :] = oracle.f32_to_bf16(np.linspace(-1e-3, 1e-3, cols).astype(np.float32))
    xt = from_np_u16(x)
    for gs in [oracle.global_scale(oracle.amax_bf16(x))[0], 1.0, 1e-6, 1e3]:
        check_quantize(nv, oracle, xt, gs)
    zeros = from_np_u16(np.zeros((rows, cols), np.uint16))
    packed, sf, gsd = nv.quantize(zeros, None)
    torch.cuda.synchronize()
    assert gsd.item() == 1.0 and int(packed.sum()) == 0 and int(sf.sum()) == 0


DEV_NONFINITE_INPUT = 0x302


def test_nonfinite_input_defined_behaviour(nv, oracle):
    """NaN and +-Inf inputs: amax skips them, a block holding one gets scale 0x7F (E4M3 NaN) and
    zero codes, every other block is quantized as usual (bit-exact against the oracle), and the
    device status records DEV_NONFINITE_INPUT."""
    rows, cols = 256, 1024
    x = workloads.activations(rows, cols, seed=77)
    xu = to_np_u16(x).copy()
    rng = np.random.default_rng(5)
    pos = rng.choice(rows * cols, size=40, replace=False)
    specials = np.array([0x7FC0, 0xFFC0, 0x7F80, 0xFF80, 0x7F81], dtype=np.uint16)   # NaN, -NaN, Inf, -Inf, sNaN
    xu.reshape(-1)[pos] = specials[np.arange(pos.size) % specials.size]
    xd = from_np_u16(xu)
    nv.device_status()                                   # clear
    am = float(nv.amax(xd).item())
    torch.cuda.synchronize()
    assert nv.device_status() == DEV_NONFINITE_INPUT
    assert am == oracle.amax_bf16(xu) and np.isfinite(am)
    gs, _ = oracle.global_scale(am)
    packed, sf, _ = nv.quantize(xd, gs)
    torch.cuda.synchronize()
    assert nv.device_status() == DEV_NONFINITE_INPUT
    p_ref, s_ref = oracle.quantize_bf16(xu, gs)
    assert np.array_equal(packed.cpu().numpy(), p_ref)
    assert np.array_equal(sf.cpu().numpy(), s_ref)
    blocks = np.unique(pos // 16)
    offs = oracle.sf_offsets(rows, cols).reshape(-1)
    assert np.all(s_ref[offs[blocks]] == 0x7F)
    # the auto-scaled path takes the finite amax
    packed2, sf2, gs_dev = nv.quantize(xd, None)
    torch.cuda.synchronize()
    assert nv.device_status() == DEV_NONFINITE_INPUT
    assert np.float32(gs_dev.item()) == np.float32(gs)
    assert torch.equal(packed2, packed) and torch.equal(sf2, sf)
    # finite input leaves the status clear
    nv.quantize(x, gs)
    nv.amax(x)
    torch.cuda.synchronize()
    assert nv.device_status() == 0
