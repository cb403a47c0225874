"""C-ABI checks that need no GPU: the library loads, exports every function declared in
include/nvfp4.h, and its host-side helpers and argument checks behave (no kernel is launched
by any call here)."""
import ctypes
import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions(macro="NVFP4_API"):
    names = []
    for hdr in os.listdir(os.path.join(ROOT, "include")):
        if not hdr.endswith(".h"):
            continue
        text = open(os.path.join(ROOT, "include", hdr)).read()
        names += re.findall(rf"^{macro} [^(]*?\b(nvfp4_\w+)\(", text, flags=re.M)
    return sorted(set(names))


def exported(path):
    """Dynamic symbols a shared library defines (nm -D --defined-only)."""
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", path], check=True, capture_output=True, text=True).stdout
    return {ln.split()[-1] for ln in out.splitlines() if " T " in ln}


def test_library_exports_every_declared_symbol(nv):
    names = declared_functions()
    assert len(names) >= 15
    L = nv.lib()
    for n in names:
        assert hasattr(L, n), n
    # the Python mirror binds exactly the declared set, and the library exports nothing else
    assert sorted(nv.SIGNATURES) == names
    assert sorted(exported(nv.LIB_PATH)) == names


def test_diag_library_exports_every_declared_symbol():
    from tensorcore_ptx_example_b200 import diag
    names = declared_functions("NVFP4_DIAG_API")
    assert len(names) >= 6
    L = diag.lib()
    for n in names:
        assert hasattr(L, n), n
    assert sorted(diag.SIGNATURES) == names
    assert sorted(exported(diag.DIAG_LIB_PATH)) == names
    # the probes are not part of the product library
    assert not any(n.startswith("nvfp4_diag") for n in exported(
        __import__("tensorcore_ptx_example_b200").LIB_PATH))


def test_abi_version(nv):
    assert nv.lib().nvfp4_abi_version() == 1


def test_layout_helpers_match_oracle(nv, oracle):
    rng = np.random.default_rng(0)
    for _ in range(2000):
        cols = int(rng.integers(1, 300)) * 64
        row = int(rng.integers(0, 100000))
        kb = int(rng.integers(0, cols // 16))
        assert nv.sf_offset(row, kb, cols) == int(oracle.lib().orc_sf_offset(row, kb, cols))
    for rows, cols in [(1, 64), (127, 64), (128, 64), (129, 128), (8192, 7168), (16, 8192)]:
        assert nv.sf_bytes(rows, cols) == oracle.sf_bytes(rows, cols)
        assert nv.packed_bytes(rows, cols) == rows * cols // 2


def test_sf_layout_is_a_bijection(oracle):
    for rows, cols in [(128, 64), (256, 512), (384, 192)]:
        off = oracle.sf_offsets(rows, cols).ravel()
        assert np.array_equal(np.sort(off), np.arange(oracle.sf_bytes(rows, cols)))
        # one 32-bit word holds the four scales of one row
        o = oracle.sf_offsets(rows, cols)
        words = o // 4
        assert np.all(words[:, 0::4] == words[:, 3::4])


def _err(nv, code):
    assert code == nv.NVFP4_ERR_INVALID_ARG, code
    return nv.lib().nvfp4_last_error_string().decode()


def test_argument_checks_reject_before_launch(nv):
    L = nv.lib()
    fake = ctypes.c_void_p(1 << 20)   # never dereferenced: checks fail first
    msg = _err(nv, L.nvfp4_quantize_bf16(fake, 128, 100, ctypes.c_float(1.0), fake, fake, None))
    assert "multiple of 64" in msg
    msg = _err(nv, L.nvfp4_quantize_bf16(fake, 128, 128, ctypes.c_float(0.0), fake, fake, None))
    assert "global_scale" in msg
    msg = _err(nv, L.nvfp4_quantize_bf16(None, 128, 128, ctypes.c_float(1.0), fake, fake, None))
    assert "null" in msg
    unaligned = ctypes.c_void_p((1 << 20) + 4)
    msg = _err(nv, L.nvfp4_quantize_bf16(unaligned, 128, 128, ctypes.c_float(1.0), fake, fake, None))
    assert "aligned" in msg
    msg = _err(nv, L.nvfp4_gemm_bf16(fake, fake, fake, fake, ctypes.c_float(1.0), fake, 200, 256, 256, None))
    assert "M % 128" in msg
    msg = _err(nv, L.nvfp4_gemm_bf16(fake, fake, fake, fake, ctypes.c_float(1.0), fake, 16, 200, 256, None))
    assert "N % 128" in msg
    # 16 splits of 256 K on one 128-row tile: more than a cluster holds, so a workspace is needed
    msg = _err(nv, L.nvfp4_gemm_bf16_ws(fake, fake, fake, fake, ctypes.c_float(1.0), fake, 16, 128, 4096, None, 0, None))
    assert "workspace" in msg
    assert L.nvfp4_gemm_workspace_bytes(16, 128, 4096) == 16 * 16 * 128 * 4
    assert L.nvfp4_gemm_workspace_bytes(16, 7168, 8192) == 0          # cfg3 decode: reduced in-cluster
    msg = _err(nv, L.nvfp4_gemm_f32(fake, fake, fake, fake, fake, 128, 256, 100, None))
    assert "K % 256" in msg
    f1 = ctypes.c_float(1.0)
    msg = _err(nv, L.nvfp4_gemm_bf16_flags(fake, fake, fake, fake, f1, fake, 16, 256, 256, 6, None))
    assert "flag" in msg
    msg = _err(nv, L.nvfp4_gemm_quantize(fake, fake, fake, fake, f1, f1, fake, fake, 128, 256, 256, None))
    assert "M % 256" in msg
    msg = _err(nv, L.nvfp4_gemm_quantize(fake, fake, fake, fake, f1, ctypes.c_float(0.0), fake, fake, 256, 256, 256,
                                         None))
    assert "global scale" in msg
    msg = _err(nv, L.nvfp4_gemm_quantize(fake, fake, fake, fake, f1, f1, None, fake, 256, 256, 256, None))
    assert "null" in msg
    msg = _err(nv, L.nvfp4_gemm_quantize(fake, fake, fake, fake, f1, f1, ctypes.c_void_p((1 << 20) + 16), fake, 256,
                                         256, 256, None))
    assert "32-byte" in msg
    msg = _err(nv, L.nvfp4_amax_bf16(fake, 7, fake, None))
    assert "numel" in msg
    msg = _err(nv, L.nvfp4_quantize_bf16_auto(fake, 128, 128, fake, fake, fake, None, None))
    assert "workspace" in msg


def test_zero_sized_calls_are_noops(nv):
    L = nv.lib()
    fake = ctypes.c_void_p(1 << 20)
    assert L.nvfp4_quantize_bf16(fake, 0, 64, ctypes.c_float(1.0), fake, fake, None) == 0
    from tensorcore_ptx_example_b200 import diag
    assert diag.lib().nvfp4_diag_e2m1_encode(fake, fake, 0, None) == 0
    assert diag.lib().nvfp4_diag_rcp_approx(fake, fake, 0, None) == 0
