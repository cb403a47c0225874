"""Build the sm_100a CUDA library in-tree.

    python -m tensorcore_ptx_example_b200.build

compiles csrc/nvfp4_lib.cu (the whole product library, one translation unit) into
tensorcore_ptx_example_b200/libnvfp4_b200.so and csrc/diag_lib.cu (hardware probes and the MMA
issue-rate microbenchmark, off the data path) into tensorcore_ptx_example_b200/libnvfp4_diag.so,
both with ``nvcc -gencode arch=compute_100a,code=sm_100a -lineinfo -O3``.  nvcc cross-compiles, so
this works on a machine without a GPU; the .so files then travel with the source tree.
"""
from __future__ import annotations

import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libnvfp4_b200.so")
DIAG_LIB = os.path.join(PKG, "libnvfp4_diag.so")
NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _sources():
    return [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC))
            if f.endswith((".cu", ".cuh", ".h"))] + [os.path.join(ROOT, "include", h)
                                                      for h in ("nvfp4.h", "nvfp4_diag.h")]


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _nvcc_shared(out: str, tu: str, verbose: bool) -> None:
    cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           "-Xcompiler", "-fvisibility=hidden", "-I", os.path.join(ROOT, "include"),
           "-o", out + ".tmp", os.path.join(CSRC, tu)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(out + ".tmp", out)


def build_library(force: bool = False, verbose: bool = False) -> str:
    """Both libraries; returns the product library's path."""
    srcs = _sources()
    if force or _stale(LIB, srcs):
        _nvcc_shared(LIB, "nvfp4_lib.cu", verbose)
    if force or _stale(DIAG_LIB, srcs):
        _nvcc_shared(DIAG_LIB, "diag_lib.cu", verbose)
    return LIB


def build_cpp_tests(force: bool = False) -> list[str]:
    """Compile the C++ drop-in tests (tests/cpp/*.cpp) against the C ABI."""
    src_dir = os.path.join(ROOT, "tests", "cpp")
    out_dir = os.path.join(src_dir, "_build")
    os.makedirs(out_dir, exist_ok=True)
    outs = []
    for f in sorted(os.listdir(src_dir)):
        if not f.endswith(".cpp"):
            continue
        exe = os.path.join(out_dir, f[:-4])
        deps = [os.path.join(src_dir, f), os.path.join(ROOT, "include", "nvfp4.h"),
                os.path.join(ROOT, "include", "verify_random.h")]
        if force or _stale(exe, deps):
            cmd = ["g++", "-O2", "-std=c++17", "-I", os.path.join(ROOT, "include"),
                   "-I", "/usr/local/cuda/include", "-o", exe, os.path.join(src_dir, f),
                   "-L", PKG, "-lnvfp4_b200", f"-Wl,-rpath,{PKG}",
                   "-L", "/usr/local/cuda/lib64", "-lcudart", "-Wl,-rpath,/usr/local/cuda/lib64"]
            subprocess.run(cmd, check=True)
        outs.append(exe)
    return outs


if __name__ == "__main__":
    build_library(force="--force" in sys.argv, verbose="-v" in sys.argv)
    build_cpp_tests(force="--force" in sys.argv)
    print(LIB)
