"""Hardware probes and the FP4 MMA issue-rate microbenchmark (libnvfp4_diag.so, include/nvfp4_diag.h).

Not part of the data path: the parity tests use the probes to pin the hardware arithmetic the
NVFP4 path depends on, and the benchmark uses the MMA peak as the measured FP4 roofline.
Raises if the library has not been built (no fallback).
"""
from __future__ import annotations

import ctypes
import os

from . import PKG_DIR, NVFP4Error, _ptr, _stream

DIAG_LIB_PATH = os.path.join(PKG_DIR, "libnvfp4_diag.so")

_P, _I64, _I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
SIGNATURES = {
    "nvfp4_diag_last_error_string": (ctypes.c_char_p, []),
    "nvfp4_diag_device_status": (_I, [ctypes.POINTER(ctypes.c_uint), _I]),
    "nvfp4_diag_e2m1_encode": (_I, [_P, _P, _I64, _P]),
    "nvfp4_diag_e4m3_encode": (_I, [_P, _P, _I64, _P]),
    "nvfp4_diag_rcp_approx": (_I, [_P, _P, _I64, _P]),
    "nvfp4_diag_mma_tile": (_I, [_P, _P, _P, _P, _P, _P]),
    "nvfp4_diag_mma_peak": (_I, [_I, _I, _I, _P]),
    "nvfp4_diag_mma_peak_clock": (_I, [ctypes.POINTER(ctypes.c_double)]),
}

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(DIAG_LIB_PATH):
            raise RuntimeError(f"{DIAG_LIB_PATH} is missing; build it with `python -m tensorcore_ptx_example_b200.build`")
        L = ctypes.CDLL(DIAG_LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(code: int):
    if code != 0:
        raise NVFP4Error(code, lib().nvfp4_diag_last_error_string().decode())


def device_status(clear: bool = True) -> int:
    v = ctypes.c_uint(0)
    check(lib().nvfp4_diag_device_status(ctypes.byref(v), 1 if clear else 0))
    return v.value


def e2m1_encode(x, stream=None):
    import torch
    out = torch.empty(x.numel(), dtype=torch.uint8, device=x.device)
    check(lib().nvfp4_diag_e2m1_encode(_ptr(x), _ptr(out), x.numel(), _stream(stream)))
    return out


def e4m3_encode(x, stream=None):
    import torch
    out = torch.empty(x.numel(), dtype=torch.uint8, device=x.device)
    check(lib().nvfp4_diag_e4m3_encode(_ptr(x), _ptr(out), x.numel(), _stream(stream)))
    return out


def rcp_approx(x, stream=None):
    """rcp.approx.ftz.f32 of every element of a float32 CUDA tensor."""
    import torch
    x = x.contiguous()
    out = torch.empty_like(x)
    check(lib().nvfp4_diag_rcp_approx(_ptr(x), _ptr(out), x.numel(), _stream(stream)))
    return out


def mma_tile(a_packed, sfa, b_packed, sfb, stream=None):
    """fp32 [128, 256] accumulators of one M128 N256 K256 block-scaled tile (see nvfp4_diag.h)."""
    import torch
    D = torch.empty((128, 256), dtype=torch.float32, device=a_packed.device)
    check(lib().nvfp4_diag_mma_tile(_ptr(a_packed), _ptr(sfa), _ptr(b_packed), _ptr(sfb), _ptr(D), _stream(stream)))
    return D


def mma_peak(cta_group: int = 2, iters: int = 4096, repeats: int = 3, random_operands: bool = True,
             stream=None) -> float:
    """Measured FP4 block-scaled MMA rate in TFLOP/s (best of `repeats` launches)."""
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    if cta_group == 2:
        sms = 2 * (sms // 2)
    flops = 2.0 * 128 * 256 * 64 * iters * sms
    ro = 1 if random_operands else 0
    check(lib().nvfp4_diag_mma_peak(cta_group, iters, ro, _stream(s)))     # warm-up
    best = 0.0
    for _ in range(repeats):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(s)
        check(lib().nvfp4_diag_mma_peak(cta_group, iters, ro, _stream(s)))
        b.record(s)
        b.synchronize()
        best = max(best, flops / (a.elapsed_time(b) * 1e-3) / 1e12)
    return best


def mma_peak_clock() -> float:
    """Effective SM clock (MHz) inside the mma_peak launches since the previous call."""
    v = ctypes.c_double()
    check(lib().nvfp4_diag_mma_peak_clock(ctypes.byref(v)))
    return float(v.value)
