"""Pins the CPU oracle (oracle/gen9_oracle.c) before it is trusted:
1. it reproduces, bit for bit, the reference's own golden digests (tools/golden/expected/uhd620-whl/lib.txt of
   kprzybys/gen9-gpu-blas, copied into tests/golden/ref_golden_hashes.json) for every call whose bytes do not depend
   on the hardware's summation order, using the call recipe of tools/golden/blas_golden.py;
2. it agrees with outputs of the reference's own CBLAS layer (lib/src/cblas.c built in CPU mode over OpenBLAS,
   tests/golden/ref_cblas_outputs.npz) within the parity tolerances;
3. its edge rules (iamax ties / NaN / empty, increments 0, negative strides) are the reference's."""
import ctypes
import hashlib
import json
import os

import numpy as np
import pytest

import abi
from make_golden import GEMM_CASES, ColMajor, NoTrans, RowMajor, Trans, gemm_inputs, vec_inputs

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def data(seed, shape, dt):   # tools/golden/blas_golden.py:19-20
    return np.random.default_rng(seed).standard_normal(shape).astype(dt)


def digest(x):               # tools/golden/blas_golden.py:64-66
    a = np.ascontiguousarray(np.asarray(x))
    return hashlib.sha256(a.dtype.str.encode() + str(a.shape).encode() + a.tobytes()).hexdigest()[:16]


def golden_calls(L):
    """The pinned calls of tools/golden/blas_golden.py:50-62 (n = 4097), run through a gen9blas.h-shaped API."""
    out = {}
    n = 4097
    for dt, tag, t in ((np.float32, "s", abi.S), (np.float64, "d", abi.D)):
        x, y = data(20, n, dt), data(21, n, dt).copy()
        assert L.axpy(t, n, 0.7, x.ctypes.data, 1, y.ctypes.data, 1) == 0
        out[tag + "axpy"] = digest(y)
        r = ctypes.c_int64()
        assert L.iamax(t, n, x.ctypes.data, 1, ctypes.byref(r)) == 0
        out[tag + "iamax"] = digest(np.asarray(r.value))
        gx, gy, A = data(28, 600, dt), data(29, 500, dt), data(30, (600, 500), dt).copy()
        assert L.ger(t, 600, 500, 0.3, gx.ctypes.data, 1, gy.ctypes.data, 1, A.ctypes.data, 500) == 0
        out[tag + "ger"] = digest(A)
        w = ctypes.c_double()
        assert L.nrm2(t, n, x.ctypes.data, 1, ctypes.byref(w)) == 0
        out[tag + "nrm2"] = digest(np.asarray(w.value))
        assert L.asum(t, n, x.ctypes.data, 1, ctypes.byref(w)) == 0
        out[tag + "asum"] = digest(np.asarray(w.value))
    return out


def test_oracle_reproduces_reference_golden_hashes(oracle):
    gold = json.load(open(os.path.join(GOLD, "ref_golden_hashes.json")))
    got = golden_calls(oracle)
    for name, h in gold.items():
        assert got[name] == h, (name, got[name], h)


REF = np.load(os.path.join(GOLD, "ref_cblas_outputs.npz"))


@pytest.mark.parametrize("tag", ["s", "d"])
def test_oracle_gemm_matches_reference_cblas(oracle, tag):
    """All CBLAS orders and transposes: the reference layer's col-major calls become row-major calls of the
    transposed problem (lib/src/cblas.c:190-191); the oracle computes them the same way."""
    t = abi.S if tag == "s" else abi.D
    tol = 1e-6 if tag == "s" else 1e-13
    for order in (RowMajor, ColMajor):
        for (M, N, K, al, be) in GEMM_CASES:
            for ta in (NoTrans, Trans):
                for tb in (NoTrans, Trans):
                    A, B, C0 = gemm_inputs(tag, order, ta, tb, M, N, K)
                    want = REF[f"{tag}gemm_o{order}_t{ta}{tb}_{M}x{N}x{K}"]
                    C = C0.copy()
                    iA, iB = int(ta == Trans), int(tb == Trans)
                    if order == RowMajor:
                        assert oracle.gemm(t, iA, iB, M, N, K, al, A.ctypes.data, A.shape[1], B.ctypes.data, B.shape[1],
                                           be, C.ctypes.data, N) == 0
                    else:   # column-major C = op(A)·op(B)  <=>  row-major Cᵀ = op(B)ᵀ·op(A)ᵀ
                        Af, Bf = np.asfortranarray(A), np.asfortranarray(B)
                        Ct = np.ascontiguousarray(C0.T)
                        assert oracle.gemm(t, iB, iA, N, M, K, al, Bf.ctypes.data, B.shape[0], Af.ctypes.data, A.shape[0],
                                           be, Ct.ctypes.data, M) == 0
                        C = Ct.T
                    a64 = A.astype(np.float64) if ta == NoTrans else A.astype(np.float64).T
                    b64 = B.astype(np.float64) if tb == NoTrans else B.astype(np.float64).T
                    scale = abs(al) * np.abs(a64) @ np.abs(b64) + abs(be) * np.abs(C0.astype(np.float64))
                    e = np.abs(C.astype(np.float64) - want.astype(np.float64)) / scale
                    assert e.max() <= tol, (order, M, N, K, ta, tb, e.max())


@pytest.mark.parametrize("tag", ["s", "d"])
def test_oracle_level12_matches_reference_cblas(oracle, tag):
    t = abi.S if tag == "s" else abi.D
    tol = 1e-6 if tag == "s" else 1e-13
    M, N = 37, 29
    for tr, name in ((0, NoTrans), (1, Trans)):
        A = vec_inputs(tag, "gemvA", M, N)
        x = vec_inputs(tag, "gemvx", N if not tr else M)
        y = vec_inputs(tag, "gemvy", M if not tr else N)
        y0 = y.copy()
        assert oracle.gemv(t, tr, M, N, 0.75, A.ctypes.data, N, x.ctypes.data, 1, -1.25, y.ctypes.data, 1) == 0
        Ad = A.astype(np.float64)
        op = Ad.T if tr else Ad
        scale = 0.75 * np.abs(op) @ np.abs(x.astype(np.float64)) + 1.25 * np.abs(y0.astype(np.float64))
        assert (np.abs(y - REF[f"{tag}gemv_t{name}"]) / scale).max() <= tol
    A = vec_inputs(tag, "gerA", 23, 31)
    gx, gy = vec_inputs(tag, "gerx", 23), vec_inputs(tag, "gery", 31)
    assert oracle.ger(t, 23, 31, -0.5, gx.ctypes.data, 1, gy.ctypes.data, 1, A.ctypes.data, 31) == 0
    np.testing.assert_allclose(A, REF[f"{tag}ger"], rtol=tol, atol=tol)
    n = 1000
    x, y = vec_inputs(tag, "l1x", n), vec_inputs(tag, "l1y", n)
    yy = y.copy()
    assert oracle.axpy(t, n, 0.7, x.ctypes.data, 1, yy.ctypes.data, 1) == 0
    np.testing.assert_allclose(yy, REF[f"{tag}axpy"], rtol=tol, atol=tol)
    w = ctypes.c_double()
    assert oracle.dot(t, n, x.ctypes.data, 1, y.ctypes.data, 1, ctypes.byref(w)) == 0
    assert abs(w.value - float(REF[f"{tag}dot"])) <= tol * float(np.abs(x.astype(np.float64)) @ np.abs(y.astype(np.float64)))
    assert oracle.nrm2(t, n, x.ctypes.data, 1, ctypes.byref(w)) == 0
    assert abs(w.value - float(REF[f"{tag}nrm2"])) <= tol * w.value
    assert oracle.asum(t, n, x.ctypes.data, 1, ctypes.byref(w)) == 0
    assert abs(w.value - float(REF[f"{tag}asum"])) <= tol * w.value
    r = ctypes.c_int64()
    assert oracle.iamax(t, n, x.ctypes.data, 1, ctypes.byref(r)) == 0
    assert r.value == int(REF[f"i{tag}amax"])


def test_oracle_edge_rules(oracle):
    r = ctypes.c_int64()
    x = np.array([1.0, -3.0, 3.0, np.nan, -3.0], np.float32)
    assert oracle.iamax(abi.S, 5, x.ctypes.data, 1, ctypes.byref(r)) == 0 and r.value == 1   # tie -> first index
    nan = np.full(7, np.nan, np.float32)
    assert oracle.iamax(abi.S, 7, nan.ctypes.data, 1, ctypes.byref(r)) == 0 and r.value == 0   # all NaN -> 0
    assert oracle.iamax(abi.S, 0, nan.ctypes.data, 1, ctypes.byref(r)) == 0 and r.value == -1  # empty -> -1
    assert oracle.iamax(abi.S, 3, nan.ctypes.data, 0, ctypes.byref(r)) == -3                   # inc 0
    # negative stride: the pointer is the lowest address, element 0 is the last one in memory
    v = np.array([5.0, 0.0, 1.0, 0.0, 9.0], np.float32)
    assert oracle.iamax(abi.S, 3, v.ctypes.data, -2, ctypes.byref(r)) == 0 and r.value == 0
    y = np.zeros(5, np.float32)
    assert oracle.axpy(abi.S, 3, 2.0, v.ctypes.data, -2, y.ctypes.data, 2) == 0
    np.testing.assert_array_equal(y, [18.0, 0.0, 2.0, 0.0, 10.0])
