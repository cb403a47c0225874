"""ctypes/numpy front end of the C oracle (oracle/nvfp4_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() as the checker,
and by bench.py's cpu_baseline / --impl reference legs.  The product package never
imports this module.

Also loads the reference's own CPU oracle (oracle/_ref/libref_verify.so, built from the
reference's random_cpu_ref/verify_random.h) when it is present.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libnvfp4_oracle.so")
REF_VERIFY_PATH = os.path.join(HERE, "_ref", "libref_verify.so")
REF_AR_PATH = os.path.join(HERE, "_ref", "libref_ar.so")

ACC_EXACT_PER_MMA = 0
ACC_ROUND_PER_MMA = 1
ACC_PER_BLOCK = 2
ACC_EXACT_ALL = 3
ACC_TCGEN05 = 4   # measured tcgen05 block-scaled MMA arithmetic (the hardware model)

_lib = None


def build():
    """Compile the oracle with its Makefile (no-op when up to date)."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = _bind(ctypes.CDLL(LIB_PATH))
    return _lib


def _bind(L):
    P = ctypes.c_void_p
    I64 = ctypes.c_int64
    F = ctypes.c_float
    U8 = ctypes.c_uint8
    sigs = {
        "orc_xorshift": (ctypes.c_uint32, [ctypes.POINTER(ctypes.c_uint32)]),
        "orc_e2m1_encode": (U8, [F]),
        "orc_e2m1_decode": (F, [U8]),
        "orc_e4m3_encode": (U8, [F]),
        "orc_e4m3_decode": (F, [U8]),
        "orc_e2m1_encode_array": (None, [P, P, I64]),
        "orc_e4m3_encode_array": (None, [P, P, I64]),
        "orc_f32_to_bf16": (ctypes.c_uint16, [F]),
        "orc_bf16_to_f32": (F, [ctypes.c_uint16]),
        "orc_sf_offset": (I64, [I64, I64, I64]),
        "orc_sf_bytes": (I64, [I64, I64]),
        "orc_global_scale": (None, [F, P, P]),
        "orc_amax_bf16": (F, [P, I64]),
        "orc_amax_f32": (F, [P, I64]),
        "orc_q16": (None, [P, F, P, P]),
        "orc_quantize_bf16": (None, [P, I64, I64, F, P, P, ctypes.c_int]),
        "orc_quantize_f32": (None, [P, I64, I64, F, P, P, ctypes.c_int]),
        "orc_dequantize_f32": (None, [P, P, I64, I64, F, P]),
        "orc_dequantize_bf16": (None, [P, P, I64, I64, F, P]),
        "orc_gemm_f32": (None, [P, P, P, P, I64, I64, I64, ctypes.c_int, P, ctypes.c_int]),
        "orc_gemm_f32_points": (None, [P, P, P, P, I64, I64, I64, ctypes.c_int, P, P, I64, P]),
        "orc_gemm_splitk_f32": (None, [P, P, P, P, I64, I64, I64, I64, P, ctypes.c_int]),
        "orc_gemm_epilogue_bf16": (ctypes.c_uint16, [F, F]),
        "orc_ar_oneshot": (None, [P, ctypes.c_int, I64, F, P, ctypes.c_int]),
        "orc_ar_twoshot": (None, [P, ctypes.c_int, I64, F, P, ctypes.c_int]),
        "orc_ar_bf16": (None, [P, ctypes.c_int, I64, P, ctypes.c_int]),
        "orc_sum_f64": (None, [P, ctypes.c_int, I64, P]),
    }
    for name, (res, args) in sigs.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    return L


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.c_void_p)


def nthreads_default() -> int:
    return max(1, min(64, os.cpu_count() or 1))


# ---------------------------------------------------------------- codecs ----
def e2m1_encode(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.empty(x.size, dtype=np.uint8)
    lib().orc_e2m1_encode_array(_p(x), _p(out), x.size)
    return out


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.empty(x.size, dtype=np.uint8)
    lib().orc_e4m3_encode_array(_p(x), _p(out), x.size)
    return out


E2M1_TABLE = np.array([0, .5, 1, 1.5, 2, 3, 4, 6, -0.0, -.5, -1, -1.5, -2, -3, -4, -6],
                      dtype=np.float32)


def e4m3_table() -> np.ndarray:
    L = lib()
    return np.array([L.orc_e4m3_decode(i) for i in range(256)], dtype=np.float32)


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


# ---------------------------------------------------------------- layout ----
def sf_bytes(rows: int, cols: int) -> int:
    return int(lib().orc_sf_bytes(rows, cols))


def sf_offsets(rows: int, cols: int) -> np.ndarray:
    """offsets[r, kb] of every block scale in the tcgen05 layout (vectorised restatement,
    checked against orc_sf_offset in the tests)."""
    r = np.arange(rows, dtype=np.int64)[:, None]
    kb = np.arange(cols // 16, dtype=np.int64)[None, :]
    katoms = (cols + 63) // 64
    atom = (r // 128) * katoms + kb // 4
    return atom * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + (kb % 4)


# -------------------------------------------------------------- quantize ----
def global_scale(amax: float):
    gs = ctypes.c_float()
    gi = ctypes.c_float()
    lib().orc_global_scale(float(amax), ctypes.byref(gs), ctypes.byref(gi))
    return gs.value, gi.value


def amax_bf16(x_bf16: np.ndarray) -> float:
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    return float(lib().orc_amax_bf16(_p(x), x.size))


def quantize_bf16(x_bf16: np.ndarray, gs: float, nthreads: int | None = None):
    """x_bf16: uint16 array [rows, cols].  Returns (packed uint8 [rows, cols/2],
    sf uint8 [sf_bytes])."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    rows, cols = x.shape
    packed = np.zeros((rows, cols // 2), dtype=np.uint8)
    sf = np.zeros(sf_bytes(rows, cols), dtype=np.uint8)
    lib().orc_quantize_bf16(_p(x), rows, cols, float(gs), _p(packed), _p(sf),
                            nthreads or nthreads_default())
    return packed, sf


def quantize_f32(x: np.ndarray, gs: float, nthreads: int | None = None):
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    packed = np.zeros((rows, cols // 2), dtype=np.uint8)
    sf = np.zeros(sf_bytes(rows, cols), dtype=np.uint8)
    lib().orc_quantize_f32(_p(x), rows, cols, float(gs), _p(packed), _p(sf),
                           nthreads or nthreads_default())
    return packed, sf


def dequantize_bf16(packed: np.ndarray, sf: np.ndarray, rows: int, cols: int, gs: float):
    out = np.zeros((rows, cols), dtype=np.uint16)
    lib().orc_dequantize_bf16(_p(np.ascontiguousarray(packed)), _p(np.ascontiguousarray(sf)),
                              rows, cols, float(gs), _p(out))
    return out


def dequantize_f32(packed: np.ndarray, sf: np.ndarray, rows: int, cols: int, gs: float):
    out = np.zeros((rows, cols), dtype=np.float32)
    lib().orc_dequantize_f32(_p(np.ascontiguousarray(packed)), _p(np.ascontiguousarray(sf)),
                             rows, cols, float(gs), _p(out))
    return out


# ------------------------------------------------------------------ GEMM ----
def gemm_f32(A, sfa, B, sfb, M, N, K, model=ACC_EXACT_PER_MMA, nthreads=None):
    D = np.zeros((M, N), dtype=np.float32)
    lib().orc_gemm_f32(_p(np.ascontiguousarray(A)), _p(np.ascontiguousarray(sfa)),
                       _p(np.ascontiguousarray(B)), _p(np.ascontiguousarray(sfb)),
                       M, N, K, model, _p(D), nthreads or nthreads_default())
    return D


def gemm_splitk_f32(A, sfa, B, sfb, M, N, K, ks, nthreads=None):
    """Split-K tcgen05 model: per-split chains of ks elements summed in split order (fp32)."""
    D = np.zeros((M, N), dtype=np.float32)
    lib().orc_gemm_splitk_f32(_p(np.ascontiguousarray(A)), _p(np.ascontiguousarray(sfa)),
                              _p(np.ascontiguousarray(B)), _p(np.ascontiguousarray(sfb)),
                              M, N, K, ks, _p(D), nthreads or nthreads_default())
    return D


def gemm_f32_points(A, sfa, B, sfb, M, N, K, ms, ns, model=ACC_EXACT_PER_MMA):
    ms = np.ascontiguousarray(ms, dtype=np.int64)
    ns = np.ascontiguousarray(ns, dtype=np.int64)
    out = np.zeros(ms.size, dtype=np.float32)
    lib().orc_gemm_f32_points(_p(np.ascontiguousarray(A)), _p(np.ascontiguousarray(sfa)),
                              _p(np.ascontiguousarray(B)), _p(np.ascontiguousarray(sfb)),
                              M, N, K, model, _p(ms), _p(ns), ms.size, _p(out))
    return out


def gemm_epilogue_bf16(acc: np.ndarray, alpha: float) -> np.ndarray:
    y = (np.asarray(acc, dtype=np.float32) * np.float32(alpha)).astype(np.float32)
    return f32_to_bf16(y)


# ------------------------------------------------------------ all-reduce ----
def _ptr_array(arrs):
    arrs = [np.ascontiguousarray(a, dtype=np.uint16) for a in arrs]
    ptrs = (ctypes.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])
    return arrs, ptrs


def ar_oneshot(inputs, gs, nthreads=None):
    arrs, ptrs = _ptr_array(inputs)
    out = np.zeros(arrs[0].size, dtype=np.uint16)
    lib().orc_ar_oneshot(ptrs, len(arrs), arrs[0].size, float(gs), _p(out),
                         nthreads or nthreads_default())
    return out


def ar_twoshot(inputs, gs, nthreads=None):
    arrs, ptrs = _ptr_array(inputs)
    out = np.zeros(arrs[0].size, dtype=np.uint16)
    lib().orc_ar_twoshot(ptrs, len(arrs), arrs[0].size, float(gs), _p(out),
                         nthreads or nthreads_default())
    return out


def ar_bf16(inputs):
    arrs, ptrs = _ptr_array(inputs)
    out = np.zeros(arrs[0].size, dtype=np.uint16)
    lib().orc_ar_bf16(ptrs, len(arrs), arrs[0].size, _p(out), 1)
    return out


def sum_f64(inputs):
    arrs, ptrs = _ptr_array(inputs)
    out = np.zeros(arrs[0].size, dtype=np.float64)
    lib().orc_sum_f64(ptrs, len(arrs), arrs[0].size, _p(out))
    return out


# ------------------------------------------------------ reference shim ----
_ref = None


def ref_verify_available() -> bool:
    return os.path.exists(REF_VERIFY_PATH)


def ref_lib():
    """The reference's own verify_random.h compiled into oracle/_ref (may be absent)."""
    global _ref
    if _ref is None:
        L = ctypes.CDLL(REF_VERIFY_PATH)
        P = ctypes.c_void_p
        L.ref_xorshift_stream.restype = ctypes.c_uint32
        L.ref_xorshift_stream.argtypes = [ctypes.c_uint32, ctypes.c_int, P]
        L.ref_fill_random.restype = ctypes.c_uint32
        L.ref_fill_random.argtypes = [ctypes.c_int, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_uint32]
        L.ref_value_set.restype = ctypes.c_int
        L.ref_value_set.argtypes = [ctypes.c_int, P, P]
        L.ref_cpu_gemm_ref.argtypes = [P, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.ref_cpu_gemm_ref_bs.argtypes = [P, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, P,
                                          ctypes.c_int]
        L.ref_cpu_gemm_ref_bs_threads.argtypes = [P, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                  P, P, ctypes.c_int, ctypes.c_int]
        L.ref_to_core_matrix.argtypes = [P, ctypes.c_int]
        L.ref_vr_verify_cpu.restype = ctypes.c_int
        L.ref_vr_verify_cpu.argtypes = [ctypes.c_int] * 4 + [ctypes.c_uint32]
        _ref = L
    return _ref


_ref_ar = None


def ref_ar_available() -> bool:
    return os.path.exists(REF_AR_PATH)


def ref_ar_lib():
    """The reference's nvfp4_allreduce.cuh kernels compiled into oracle/_ref/libref_ar.so
    (oracle/ref_ar_shim.cu): the reference's own GPU quantizer and fused all-reduce launchers,
    run on the GPU box beside this project's kernels as a same-box comparator."""
    global _ref_ar
    if _ref_ar is None:
        L = ctypes.CDLL(REF_AR_PATH)
        P, I, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
        sigs = {
            "ref_column_bytes": (SZ, [SZ]),
            "ref_fused_comm_bytes": (SZ, [SZ, I]),
            "ref_oneshot_comm_bytes": (SZ, [SZ, I]),
            "ref_fused_barrier_words": (SZ, [I]),
            "ref_default_fused_grid": (I, [SZ, I]),
            "ref_layout_total_bytes": (SZ, [SZ]),
            "ref_quantize": (I, [P, P, SZ, ctypes.c_float, P]),
            "ref_launch_twoshot": (I, [I, P, P, P, P, P, I, SZ, ctypes.c_float, ctypes.c_uint32, P, I]),
            "ref_launch_oneshot": (I, [I, P, P, P, P, I, SZ, ctypes.c_float, ctypes.c_uint32, P, I]),
            "ref_fused_resident_blocks": (I, [I, I]),
            "ref_dev_alloc_zero": (I, [SZ, ctypes.POINTER(P)]),
            "ref_dev_free": (I, [P]),
            "ref_dev_ptr_array": (I, [P, I, ctypes.POINTER(P)]),
            "ref_ipc_handle_bytes": (SZ, []),
            "ref_ipc_get": (I, [P, P]),
            "ref_ipc_open": (I, [P, ctypes.POINTER(P)]),
            "ref_ipc_close": (I, [P]),
        }
        for name, (res, args) in sigs.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _ref_ar = L
    return _ref_ar
