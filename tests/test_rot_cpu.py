"""The host-side Givens helpers gen9blas_rotg / gen9blas_rotmg (CPU functions of the C ABI, lib/gen9blas.h:127-128;
no GPU involved) against OpenBLAS's srotg / srotmg -- the CPU BLAS the reference's CBLAS layer forwards to -- on
random and edge-case inputs."""
import ctypes
import os
import sys

import numpy as np
import pytest

from conftest import PKG, ROOT

sys.path.insert(0, os.path.join(ROOT, "oracle"))
import cpu_blas  # noqa: E402


@pytest.fixture(scope="module")
def libs():
    ob = cpu_blas.load_openblas()
    if ob is None:
        pytest.skip("no OpenBLAS found (set GEN9BLAS_OPENBLAS)")
    g9 = ctypes.CDLL(os.path.join(PKG, "libgen9blas.so"))
    fp = ctypes.POINTER(ctypes.c_float)
    for lib, pre in ((ob, "cblas_s"), (g9, "gen9blas_")):
        getattr(lib, pre + "rotg").argtypes = [fp] * 4
        getattr(lib, pre + "rotg").restype = None
        getattr(lib, pre + "rotmg").argtypes = [fp, fp, fp, ctypes.c_float, fp]
        getattr(lib, pre + "rotmg").restype = None
    return ob, g9


def run_rotg(f, a, b):
    w = [ctypes.c_float(a), ctypes.c_float(b), ctypes.c_float(), ctypes.c_float()]
    f(*[ctypes.byref(v) for v in w])
    return np.array([v.value for v in w], np.float64)


def run_rotmg(f, d1, d2, x1, y1):
    w = [ctypes.c_float(d1), ctypes.c_float(d2), ctypes.c_float(x1)]
    p = (ctypes.c_float * 5)()
    f(*[ctypes.byref(v) for v in w], ctypes.c_float(y1), p)
    flag = p[0]
    # only the entries the flag defines are significant (BLAS)
    keep = {-1.0: [1, 2, 3, 4], 0.0: [2, 3], 1.0: [1, 4], -2.0: []}[flag]
    return np.array([v.value for v in w] + [flag] + [p[k] for k in keep], np.float64)


def close(u, v, tol=4e-6):
    return u.shape == v.shape and bool(np.all(np.abs(u - v) <= tol * np.maximum(1.0, np.abs(v))))


def test_rotg_matches_openblas(libs):
    ob, g9 = libs
    rng = np.random.default_rng(0)
    cases = [(3.0, 4.0), (4.0, 3.0), (-3.0, 4.0), (3.0, -4.0), (0.0, 2.0), (2.0, 0.0), (0.0, 0.0), (1e-30, 1e-30),
             (1e30, -1e30), (5.0, 5.0)]
    cases += [tuple(v) for v in rng.uniform(-10, 10, (200, 2))]
    for a, b in cases:
        u, v = run_rotg(g9.gen9blas_rotg, a, b), run_rotg(ob.cblas_srotg, a, b)
        assert close(u, v), (a, b, u, v)


def test_rotmg_matches_openblas(libs):
    ob, g9 = libs
    rng = np.random.default_rng(1)
    cases = [(1.0, 1.0, 3.0, 4.0), (1.0, 1.0, 4.0, 3.0), (-1.0, 1.0, 1.0, 1.0), (1.0, 0.0, 1.0, 1.0),
             (1.0, 1.0, 1.0, 0.0), (1e-9, 1.0, 1.0, 1.0), (1e9, 1.0, 1.0, 1.0), (1.0, 1e-9, 1e3, 1.0),
             (2.0, -3.0, 1.0, 1.0)]
    cases += [(float(d1), float(d2), float(x), float(y)) for d1, d2, x, y in
              zip(rng.uniform(0.1, 5, 100), rng.uniform(0.1, 5, 100), rng.uniform(-3, 3, 100), rng.uniform(-3, 3, 100))]
    for c in cases:
        u, v = run_rotmg(g9.gen9blas_rotmg, *c), run_rotmg(ob.cblas_srotmg, *c)
        assert close(u, v), (c, u, v)
