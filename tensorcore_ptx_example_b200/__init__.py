"""B200-native (sm_100a) NVFP4 data path: quantizer, block-scaled tcgen05 GEMM and
NVFP4-compressed all-reduce, reached through the C ABI in include/nvfp4.h.

This module is the Python host mirror of that ABI: thin ctypes wrappers that take torch
CUDA tensors (PyTorch is only used for device memory and streams).  There is no CPU
fallback: every function raises if libnvfp4_b200.so is missing or a call fails.
"""
from __future__ import annotations

import ctypes
import os

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libnvfp4_b200.so")

NVFP4_OK = 0
NVFP4_ERR_INVALID_ARG = 1
NVFP4_ERR_CUDA = 2
NVFP4_ERR_TIMEOUT = 3
NVFP4_ERR_UNSUPPORTED = 4
NVFP4_ERR_NOT_READY = 5

_STATUS_NAMES = {0: "OK", 1: "INVALID_ARG", 2: "CUDA", 3: "TIMEOUT", 4: "UNSUPPORTED", 5: "NOT_READY"}

# Exported C symbols and their ctypes signatures (kept in step with include/nvfp4.h;
# tests/test_capi.py checks the two lists against each other).
_P, _I64, _F, _I, _U = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_int, ctypes.c_uint32
SIGNATURES = {
    "nvfp4_abi_version": (_I, []),
    "nvfp4_last_error_string": (ctypes.c_char_p, []),
    "nvfp4_device_status": (_I, [ctypes.POINTER(ctypes.c_uint), _I]),
    "nvfp4_packed_bytes": (_I64, [_I64, _I64]),
    "nvfp4_sf_bytes": (_I64, [_I64, _I64]),
    "nvfp4_sf_offset": (_I64, [_I64, _I64, _I64]),
    "nvfp4_amax_bf16": (_I, [_P, _I64, _P, _P]),
    "nvfp4_quantize_bf16": (_I, [_P, _I64, _I64, _F, _P, _P, _P]),
    "nvfp4_quantize_workspace_bytes": (ctypes.c_size_t, []),
    "nvfp4_quantize_bf16_auto": (_I, [_P, _I64, _I64, _P, _P, _P, _P, _P]),
    "nvfp4_quantize_bf16_auto_noalloc": (_I, [_P, _I64, _I64, _P, _P, _P, _P]),
    "nvfp4_dequantize_bf16": (_I, [_P, _P, _I64, _I64, _F, _P, _P]),
    "nvfp4_gemm_bf16": (_I, [_P, _P, _P, _P, _F, _P, _I64, _I64, _I64, _P]),
    "nvfp4_gemm_f32": (_I, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _P]),
    "nvfp4_gemm_workspace_bytes": (ctypes.c_size_t, [_I64, _I64, _I64]),
    "nvfp4_gemm_bf16_ws": (_I, [_P, _P, _P, _P, _F, _P, _I64, _I64, _I64, _P, ctypes.c_size_t, _P]),
    "nvfp4_gemm_quantize": (_I, [_P, _P, _P, _P, _F, _F, _P, _P, _I64, _I64, _I64, _P]),
    "nvfp4_gemm_bf16_flags": (_I, [_P, _P, _P, _P, _F, _P, _I64, _I64, _I64, _I, _P]),
    "nvfp4_ar_buffer_bytes": (_I64, [_I, _I64]),
    "nvfp4_ar_create": (_I, [_I, _I, _I64, ctypes.POINTER(ctypes.c_void_p)]),
    "nvfp4_ar_destroy": (_I, [_P]),
    "nvfp4_ar_handle_bytes": (ctypes.c_size_t, []),
    "nvfp4_ar_export_handle": (_I, [_P, _P]),
    "nvfp4_ar_open_peers": (_I, [_P, _P]),
    "nvfp4_ar_local_base": (_I, [_P, ctypes.POINTER(ctypes.c_void_p)]),
    "nvfp4_ar_set_peers": (_I, [_P, _P]),
    "nvfp4_ar_set_timeout": (_I, [_P, ctypes.c_uint64]),
    "nvfp4_ar_set_multicast": (_I, [_P, _P, _P, _I64]),
    "nvfp4_ar_reset": (_I, [_P]),
    "nvfp4_ar_choose_algo": (_I, [_I, _I64]),
    "nvfp4_ar_allreduce": (_I, [_P, _P, _P, _I64, _F, _I, _P]),
    "nvfp4_ar_bf16_allreduce": (_I, [_P, _P, _P, _I64, _I, _P]),
    "nvfp4_ar_allreduce_emulated": (_I, [_P, _I, _P, _P, _I64, _F, _I, _I, _P]),
    "nvfp4_gemm_allreduce": (_I, [_P, _P, _P, _P, _P, _F, _F, _P, _I64, _I64, _I64, _P]),
    "nvfp4_gemm_allreduce_emulated": (_I, [_P, _I, _P, _P, _P, _P, _P, _F, _P, _I64, _I64, _I64, _P]),
}


class NVFP4Error(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"nvfp4 error {_STATUS_NAMES.get(code, code)}: {msg}")
        self.code = code


_lib = None


def lib():
    """The loaded C library.  Raises if it has not been built: there is no fallback."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing; build it with `python -m tensorcore_ptx_example_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(code: int):
    if code != NVFP4_OK:
        raise NVFP4Error(code, lib().nvfp4_last_error_string().decode())


def _stream(stream=None):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _empty(shape, dtype, device, stream=None):
    """torch.empty for a buffer that kernels on `stream` will use.  Allocations come from torch's
    caching allocator on the current stream; when the caller names another stream, the buffer is
    also recorded on that one, so the allocator does not hand its memory out again (after this
    function drops it, or after the caller frees it) before the work queued on `stream` is done."""
    import torch
    t = torch.empty(shape, dtype=dtype, device=device)
    if stream is not None and stream != torch.cuda.current_stream(t.device):
        t.record_stream(stream)
    return t


def device_status(clear: bool = True) -> int:
    v = ctypes.c_uint(0)
    check(lib().nvfp4_device_status(ctypes.byref(v), 1 if clear else 0))
    return v.value


# ------------------------------------------------------------------ layout ----
def packed_bytes(rows: int, cols: int) -> int:
    return int(lib().nvfp4_packed_bytes(rows, cols))


def sf_bytes(rows: int, cols: int) -> int:
    return int(lib().nvfp4_sf_bytes(rows, cols))


def sf_offset(row: int, kblock: int, cols: int) -> int:
    return int(lib().nvfp4_sf_offset(row, kblock, cols))


# --------------------------------------------------------------- quantizer ----
def amax(x, out=None, stream=None):
    """max |x| of a bf16 CUDA tensor, as a 1-element float32 CUDA tensor."""
    import torch
    assert x.dtype == torch.bfloat16 and x.is_cuda and x.is_contiguous()
    if out is None:
        out = _empty(1, torch.float32, x.device, stream)
    check(lib().nvfp4_amax_bf16(_ptr(x), x.numel(), _ptr(out), _stream(stream)))
    return out


def global_scale_from_amax(amax_value: float) -> float:
    """gs = amax / (6 * 448) in fp32 (amax 0 -> 1.0), the convention of every call here."""
    import numpy as np
    a = np.float32(amax_value)
    if a <= 0:
        return 1.0
    g = np.float32(a / np.float32(2688.0))
    return float(g) if g != 0 else 1.0


def quantize(x, global_scale: float | None = None, packed=None, sf=None, stream=None):
    """bf16 [rows, cols] -> (packed uint8 [rows, cols/2], sf uint8 [sf_bytes], gs).

    With global_scale None the scale is computed on the device from x's amax
    (returned as a 1-element CUDA tensor); otherwise the given float is used."""
    import torch
    assert x.dtype == torch.bfloat16 and x.is_cuda and x.is_contiguous() and x.dim() == 2
    rows, cols = x.shape
    if packed is None:
        packed = _empty((rows, cols // 2), torch.uint8, x.device, stream)
    if sf is None:
        sf = _empty(sf_bytes(rows, cols), torch.uint8, x.device, stream)
    if global_scale is None:
        gs = _empty(1, torch.float32, x.device, stream)
        ws = _empty(int(lib().nvfp4_quantize_workspace_bytes()), torch.uint8, x.device, stream)
        check(lib().nvfp4_quantize_bf16_auto(_ptr(x), rows, cols, _ptr(packed), _ptr(sf), _ptr(gs),
                                             _ptr(ws), _stream(stream)))
        return packed, sf, gs
    check(lib().nvfp4_quantize_bf16(_ptr(x), rows, cols, ctypes.c_float(global_scale), _ptr(packed),
                                    _ptr(sf), _stream(stream)))
    return packed, sf, global_scale


def dequantize(packed, sf, rows: int, cols: int, global_scale: float, out=None, stream=None):
    import torch
    if out is None:
        out = _empty((rows, cols), torch.bfloat16, packed.device, stream)
    check(lib().nvfp4_dequantize_bf16(_ptr(packed), _ptr(sf), rows, cols, ctypes.c_float(global_scale),
                                      _ptr(out), _stream(stream)))
    return out


# -------------------------------------------------------------------- GEMM ----
NVFP4_GEMM_WEIGHTS_CONST = 1


def gemm(a_packed, sfa, b_packed, sfb, M: int, N: int, K: int, alpha: float = 1.0, out=None, stream=None,
         weights_const: bool = False):
    """D = bf16(alpha * A @ B^T) for NVFP4 A [M, K] and B [N, K].  weights_const: B and its
    scales are not written by earlier work on the stream (lets the decode kernel stream B
    before its dependency wait)."""
    import torch
    if out is None:
        out = _empty((M, N), torch.bfloat16, a_packed.device, stream)
    if weights_const:
        check(lib().nvfp4_gemm_bf16_flags(_ptr(a_packed), _ptr(sfa), _ptr(b_packed), _ptr(sfb), ctypes.c_float(alpha),
                                          _ptr(out), M, N, K, NVFP4_GEMM_WEIGHTS_CONST, _stream(stream)))
    else:
        check(lib().nvfp4_gemm_bf16(_ptr(a_packed), _ptr(sfa), _ptr(b_packed), _ptr(sfb), ctypes.c_float(alpha),
                                    _ptr(out), M, N, K, _stream(stream)))
    return out


def gemm_quantize(a_packed, sfa, b_packed, sfb, M: int, N: int, K: int, alpha: float, global_scale: float,
                  packed=None, sf=None, stream=None):
    """NVFP4 of D = bf16(alpha * A @ B^T) with the given global scale, quantized in the GEMM's
    epilogue: (packed [M, N/2] uint8, scales in the tcgen05 layout)."""
    import torch
    if packed is None:
        packed = _empty((M, N // 2), torch.uint8, a_packed.device, stream)
    if sf is None:
        sf = _empty(sf_bytes(M, N), torch.uint8, a_packed.device, stream)
    check(lib().nvfp4_gemm_quantize(_ptr(a_packed), _ptr(sfa), _ptr(b_packed), _ptr(sfb), ctypes.c_float(alpha),
                                    ctypes.c_float(global_scale), _ptr(packed), _ptr(sf), M, N, K, _stream(stream)))
    return packed, sf


def gemm_f32(a_packed, sfa, b_packed, sfb, M: int, N: int, K: int, out=None, stream=None):
    """Raw fp32 accumulators of the same kernel (tile checks)."""
    import torch
    if out is None:
        out = _empty((M, N), torch.float32, a_packed.device, stream)
    check(lib().nvfp4_gemm_f32(_ptr(a_packed), _ptr(sfa), _ptr(b_packed), _ptr(sfb), _ptr(out), M, N, K,
                               _stream(stream)))
    return out
