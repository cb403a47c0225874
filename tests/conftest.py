"""Shared pytest setup.

Markers:
  gpu  -- needs a B200 (sm_100a) GPU; run with `pytest -m gpu`.  Every other test runs on
          a CPU-only machine (`pytest -m "not gpu"`).
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test needs a B200 GPU (sm_100a)")


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _has_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA device on this machine")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def oracle():
    import py_oracle
    py_oracle.build()
    return py_oracle


@pytest.fixture(scope="session")
def nv():
    """The product package with its CUDA library loaded (fails loudly if missing)."""
    import tensorcore_ptx_example_b200 as nv
    nv.lib()
    return nv

