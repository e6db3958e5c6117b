"""Shared fixtures: the C-ABI library (libgen9blas.so), the NumPy module, and the CPU oracle (test infrastructure).

Markers: `gpu` = needs an sm_100 GPU (the driver runs `pytest -m gpu` on a B200); everything else runs on CPU.
"""
import ctypes
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "gen9-gpu-blas_b200")
sys.path.insert(0, PKG)
sys.path.insert(0, os.path.join(ROOT, "tests"))
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))

import abi  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU; run with -m gpu")


def _build_oracle():
    so = os.path.join(ROOT, "oracle", "liboracle.so")
    src = os.path.join(ROOT, "oracle", "gen9_oracle.c")
    if not os.path.exists(so) or os.path.getmtime(so) < os.path.getmtime(src):
        subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "all"], check=True, capture_output=True)
    return so


@pytest.fixture(scope="session")
def oracle():
    """The C restatement of the reference hot path (oracle/gen9_oracle.c), signatures as gen9blas.h."""
    return abi.bind(ctypes.CDLL(_build_oracle()), "oracle_")


@pytest.fixture(scope="session")
def lib():
    """libgen9blas.so through its C ABI (no GPU needed to load it)."""
    path = os.path.join(PKG, "libgen9blas.so")
    if not os.path.exists(path):
        pytest.fail("libgen9blas.so is not built: run python gen9-gpu-blas_b200/build.py (or __graft_entry__.build())")
    return abi.bind(ctypes.CDLL(path), "gen9blas_")


@pytest.fixture(scope="session")
def gpu_lib(lib):
    """The C ABI with an initialised GPU; a GPU test without a usable sm_100 device fails loudly."""
    if lib.init() != 0:
        pytest.fail("GPU test without a usable sm_100 device: " + lib.error().decode())
    return lib


@pytest.fixture(scope="session")
def g9(gpu_lib):
    """The NumPy module (drop-in surface of lib/gen9blas.py)."""
    import gen9blas
    gen9blas._init()
    return gen9blas


def gemm_error(W, ref, scale):
    """Element-wise error of the reference tests (lib/test_basic.py:4-8): |C − ref| / (|alpha|·|A||B| + |beta·C0|)."""
    e = np.abs(np.asarray(W, np.float64) - ref) / scale
    return float(e.mean()), float(e.max())
