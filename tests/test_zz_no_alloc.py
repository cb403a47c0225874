"""The allocation-free auto-scaled quantizer (nvfp4_quantize_bf16_auto_noalloc).

Callers that cannot allocate device memory (a plugin whose host framework owns every byte of
device memory, code running inside an allocator's own callbacks, or a path that must never
synchronise the device the way cudaMalloc/cudaFree can) cannot pass the workspace that
nvfp4_quantize_bf16_auto needs.  The no-alloc entry point keeps that scratch in a fixed
256-byte device array of the library instead.  This test calls it through the C ABI and
checks that it produces exactly the bytes of the workspace entry point, on two calls in a row
(the second with a smaller amax, so a scratch word left over from the first call would show).

The file is named so that pytest collects it last; it also passes on its own in a fresh
process (the first call on the device does the symbol-address set-up).
"""
import ctypes

import pytest

torch = pytest.importorskip("torch")

from tensorcore_ptx_example_b200 import workloads  # noqa: E402


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _run_workspace(nv, L, x, rows, cols):
    packed = torch.zeros((rows, cols // 2), dtype=torch.uint8, device="cuda")
    sf = torch.zeros(nv.sf_bytes(rows, cols), dtype=torch.uint8, device="cuda")
    gs = torch.zeros(1, dtype=torch.float32, device="cuda")
    ws = torch.empty(int(L.nvfp4_quantize_workspace_bytes()), dtype=torch.uint8, device="cuda")
    rc = L.nvfp4_quantize_bf16_auto(_p(x), rows, cols, _p(packed), _p(sf), _p(gs), _p(ws), None)
    assert rc == 0, L.nvfp4_last_error_string()
    return packed, sf, gs


def _run_noalloc(nv, L, x, rows, cols):
    # outputs pre-filled with garbage: the entry point must write every byte
    packed = torch.full((rows, cols // 2), 0xA5, dtype=torch.uint8, device="cuda")
    sf = torch.full((nv.sf_bytes(rows, cols),), 0x5A, dtype=torch.uint8, device="cuda")
    gs = torch.full((1,), -1.0, dtype=torch.float32, device="cuda")
    rc = L.nvfp4_quantize_bf16_auto_noalloc(_p(x), rows, cols, _p(packed), _p(sf), _p(gs), None)
    assert rc == 0, L.nvfp4_last_error_string()
    return packed, sf, gs


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point(nv):
    L = nv.lib()
    rows, cols = 1000, 7168
    big = workloads.activations(rows, cols, seed=41)            # N(0,1) with x50 outliers
    small = (workloads.gaussian(rows, cols, seed=42, std=0.02))  # much smaller amax
    for x in (big, small):                                       # two calls in a row
        want = _run_workspace(nv, L, x, rows, cols)
        got = _run_noalloc(nv, L, x, rows, cols)
        torch.cuda.synchronize()
        assert nv.device_status() == 0
        # bit-exact: the same kernels on the same inputs (tolerance 0)
        assert torch.equal(got[2], want[2]), (got[2].item(), want[2].item())
        assert torch.equal(got[0], want[0])
        assert torch.equal(got[1], want[1])


@pytest.mark.gpu
def test_noalloc_empty_tensor_writes_global_scale(nv):
    """rows = 0: nothing to quantize, but the global scale is still written (amax 0 -> gs 1)."""
    L = nv.lib()
    x = torch.zeros(64, dtype=torch.bfloat16, device="cuda")          # valid pointers, 0 rows used
    packed = torch.zeros(64, dtype=torch.uint8, device="cuda")
    sf = torch.zeros(64, dtype=torch.uint8, device="cuda")
    gs = torch.full((1,), -1.0, dtype=torch.float32, device="cuda")
    rc = L.nvfp4_quantize_bf16_auto_noalloc(_p(x), 0, 64, _p(packed), _p(sf), _p(gs), None)
    assert rc == 0, L.nvfp4_last_error_string()
    torch.cuda.synchronize()
    assert nv.device_status() == 0
    assert gs.item() == 1.0
