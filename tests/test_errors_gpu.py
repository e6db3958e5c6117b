"""Status codes of the 0.2 API, one call per code (the reference's lib/test_errors.py), their propagation through the
NumPy module and the LD_PRELOAD library, host-side fault injection (GEN9BLAS_FAULT) and the bounded device-side wait
(a wait that can never complete gives up and reports GEN9BLAS_ERR; the device stays usable). No GPU fault is provoked."""
import ctypes
import os
import subprocess
import sys

import numpy as np
import pytest

import abi
from conftest import ROOT

pytestmark = pytest.mark.gpu
OK, ERR, UNSUPPORTED, INVALID, OOM = 0, -1, -2, -3, -4


def test_status_codes(gpu_lib):
    L = gpu_lib
    assert L.version() // 100 == 2
    assert L.init() == OK and L.init() == OK
    assert L.has(999) == 0 and L.has(0) == 1 and L.has(1) == 1 and L.has(2) == 1
    assert L.device_gen() == 100
    a, b, c = np.ones((8, 8), np.float32), np.ones((8, 8), np.float32), np.zeros((8, 8), np.float32)
    assert L.gemm(abi.S, 0, 0, 8, 8, 8, 1.0, a.ctypes.data, 8, b.ctypes.data, 8, 0.0, c.ctypes.data, 8) == OK
    assert L.last_status() == OK and (c == 8).all()
    assert L.gemm(7, 0, 0, 8, 8, 8, 1.0, a.ctypes.data, 8, b.ctypes.data, 8, 0.0, c.ctypes.data, 8) == UNSUPPORTED
    x, y = np.ones(8, np.float32), np.zeros(8, np.float32)
    assert L.gemv(abi.S, 0, 8, 8, 1.0, a.ctypes.data, 4, x.ctypes.data, 1, 0.0, y.ctypes.data, 1) == INVALID
    assert L.axpy(abi.S, 8, 1.0, x.ctypes.data, 0, y.ctypes.data, 1) == INVALID
    assert L.gemm(abi.S, 0, 0, 0, 8, 8, 1.0, a.ctypes.data, 8, b.ctypes.data, 8, 0.0, c.ctypes.data, 8) == OK  # empty
    # packed weights: lib/test_errors.py:47-59
    assert L.gemm_pb(0, 8, 1.0, a.ctypes.data, 8, None, 0.0, c.ctypes.data, 8) == INVALID
    assert L.pack_b(7, 0, 8, 8, b.ctypes.data, 8) is None and L.last_status() == UNSUPPORTED
    assert L.pack_b(abi.S, 0, 0, 8, b.ctypes.data, 8) is None and L.last_status() == INVALID
    w = np.ones((64, 64), np.float16)
    P = L.pack_b(abi.HS, 1, 64, 64, w.ctypes.data, 64)
    assert P
    A, C64, nf = np.ones((17, 64), np.float32), np.zeros((17, 64), np.float32), ctypes.c_int(0)
    assert L.gemm_pb_skinny(17, A.ctypes.data, 64, P, C64.ctypes.data, 64, ctypes.byref(nf)) == 1   # DECLINED
    assert not C64.any()
    Sp = L.pack_b(abi.S, 1, 64, 64, np.ones((64, 64), np.float32).ctypes.data, 64)
    assert L.gemm_pb_skinny(4, A.ctypes.data, 64, Sp, C64.ctypes.data, 64, ctypes.byref(nf)) == INVALID
    assert L.gemm_pb_skinny(4, A.ctypes.data, 64, P, C64.ctypes.data, 64, ctypes.byref(nf)) == OK
    assert (C64[:4] == 64).all() and nf.value == 0
    L.packed_b_free(P)
    L.packed_b_free(Sp)
    assert L.alloc(1 << 50) is None and L.last_status() == OOM
    p = L.alloc(4096)
    assert p and L.is_usm(p, 4096) == 1 and L.is_usm(p, 8192 * 1024 * 1024) == 0
    L.free(p)


def test_bounded_device_wait_reports_and_recovers(gpu_lib):
    L = gpu_lib
    assert L.selftest_wait(5.0) == ERR
    assert b"gave up" in L.error()
    a = np.full((64, 64), 2, np.float32)
    c = np.zeros((64, 64), np.float32)
    assert L.gemm(abi.S, 0, 0, 64, 64, 64, 1.0, a.ctypes.data, 64, a.ctypes.data, 64, 0.0, c.ctypes.data, 64) == OK
    assert (c == 256).all()       # the context is intact after the timeout


CHILD = r"""
import ctypes, os, sys
import numpy as np
sys.path.insert(0, os.path.join(sys.argv[1], "tests")); sys.path.insert(0, os.path.join(sys.argv[1], "gen9-gpu-blas_b200"))
import abi, gen9blas
L = abi.bind(gen9blas._lib, "gen9blas_")
a = np.ones((64, 64), np.float32); c = np.zeros((64, 64), np.float32)
r = L.gemm(abi.S, 0, 0, 64, 64, 64, 1.0, a.ctypes.data, 64, a.ctypes.data, 64, 0.0, c.ctypes.data, 64)
try:
    gen9blas.sgemm(a, a); py = "no error"
except RuntimeError as e:
    py = str(e)
print(r); print(py)
"""


@pytest.mark.parametrize("fault,code,text", [("alloc", OOM, "injected fault"), ("launch", ERR, "injected fault"),
                                             ("wait", ERR, "gave up")])
def test_injected_faults_propagate(fault, code, text):
    env = dict(os.environ, GEN9BLAS_FAULT=fault)
    r = subprocess.run([sys.executable, "-c", CHILD, ROOT], capture_output=True, text=True, env=env, timeout=300)
    lines = r.stdout.strip().splitlines()
    assert r.returncode == 0 and int(lines[0]) == code, r.stdout + r.stderr
    assert text in lines[1]      # the NumPy module raises RuntimeError with gen9blas_error()


def test_shim_aborts_on_gpu_error():
    """The CBLAS library does not fall back to the CPU after a GPU error: one message, then abort."""
    env = dict(os.environ, GEN9BLAS_FAULT="launch")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "tests", "shim_child.py"), "cblas_gemm"],
                       capture_output=True, text=True, env=env, timeout=300)
    assert r.returncode != 0 and "GPU error in sgemm" in r.stderr
