"""GPU parity of the level-1/2 kernels against the oracle and FP64 NumPy, with the cases and criteria of the
reference's lib/test_level12.py:20-97 (strides incl. negative, shifted starts, tails, shared pages, gemv/ger shapes,
transposed views, submatrices) plus the bit-exact rules: axpy/ger/iamax must equal the oracle bit for bit and
reproduce the reference's golden digests."""
import ctypes
import json
import os

import numpy as np
import pytest

import abi
from test_oracle_golden import GOLD, golden_calls

pytestmark = pytest.mark.gpu
rng = np.random.default_rng(11)
TOL = {np.float32: 1e-6, np.float16: 2e-3, np.float64: 1e-13}
DTYPES = (np.float32, np.float16, np.float64)


def check(name, W, ref, scale, tol):
    e = float(np.max(np.abs(np.asarray(W, np.float64) - ref) / np.maximum(scale, 6.2e-5 if tol > 1e-5 else 1e-30)))
    assert e <= tol, f"{name}: {e:.2e} > {tol:.0e}"


def vector(n, dt, step=1, shift=0):
    base = rng.uniform(-1, 1, n * abs(step) + shift + 3).astype(dt)
    v = base[shift:shift + n * abs(step):abs(step)]
    return v[::-1] if step < 0 else v


def test_golden_digests_on_gpu(gpu_lib):
    """The GPU kernels reproduce the reference's own golden digests (element-wise exact results)."""
    gold = json.load(open(os.path.join(GOLD, "ref_golden_hashes.json")))
    got = golden_calls(gpu_lib)
    for name in ("saxpy", "daxpy", "sger", "dger", "siamax", "diamax"):
        assert got[name] == gold[name], name


@pytest.mark.parametrize("dt", DTYPES)
def test_level1_reference_cases(g9, dt):
    tol = TOL[dt]
    for n in (1, 5, 255, 256, 1000, 100003):
        for kx, ky, px in ((1, 1, 0), (1, 1, 1), (3, -2, 5), (-1, 1, 2)):
            label = f"n={n} strides {kx},{ky} shift {px}"
            x, y = vector(n, dt, kx, px), vector(n, dt, ky, 1)
            X, Y = x.astype(np.float64), y.astype(np.float64)
            g9.axpy(0.75, x, y)
            check("axpy " + label, y, 0.75 * X + Y, 0.75 * abs(X) + abs(Y), tol)
            y[:] = Y
            check("dot " + label, g9.dot(x, y), X @ Y, abs(X) @ abs(Y), 1e-6)
            check("asum " + label, g9.asum(x), abs(X).sum(), abs(X).sum(), 1e-6)
            check("nrm2 " + label, g9.nrm2(x), np.linalg.norm(X), np.linalg.norm(X), 1e-6)
            assert g9.iamax(x) == int(np.argmax(abs(X))), label
    v = rng.uniform(-1, 1, 3000).astype(dt)
    V = v.astype(np.float64)
    g9.axpy(2.0, v[:1000], v[1000:2000])   # operands on shared pages
    check("axpy shared pages", v[1000:2000], 2 * V[:1000] + V[1000:2000], 3, tol)
    v[:] = V
    check("dot x·x", g9.dot(v, v), V @ V, V @ V, 1e-6)


@pytest.mark.parametrize("dt", DTYPES)
def test_level2_reference_cases(g9, dt):
    tol = TOL[dt]
    for M, N in ((1, 1), (7, 3), (64, 64), (257, 1031), (1000, 2), (3, 5000), (2048, 1536)):
        A = rng.uniform(-1, 1, (M, N)).astype(dt)
        Ad = A.astype(np.float64)
        x, xt = vector(N, dt), vector(M, dt, -2, 3)
        y0, yt0 = vector(M, dt, 2), vector(N, dt)
        Y0, YT0 = y0.astype(np.float64), yt0.astype(np.float64)
        y = g9.gemv(A, x, alpha=1.5)
        check(f"gemv N {M}x{N}", y, 1.5 * Ad @ x.astype(np.float64), 1.5 * abs(Ad) @ abs(x.astype(np.float64)), tol)
        g9.gemv(A, x, alpha=0.5, beta=-2.0, y=y0)
        check(f"gemv N beta {M}x{N}", y0, 0.5 * Ad @ x.astype(np.float64) - 2 * Y0,
              0.5 * abs(Ad) @ abs(x.astype(np.float64)) + 2 * abs(Y0), tol)
        g9.gemv(A, xt, alpha=0.5, beta=1.0, y=yt0, trans=True)
        Xt = xt.astype(np.float64)
        check(f"gemv T {M}x{N}", yt0, 0.5 * Ad.T @ Xt + YT0, 0.5 * abs(Ad.T) @ abs(Xt) + abs(YT0), tol)
        xv = vector(M, dt)
        Xv = xv.astype(np.float64)
        yv = g9.gemv(A.T, xv)
        check(f"gemv A.T {M}x{N}", yv, Ad.T @ Xv, abs(Ad.T) @ abs(Xv), tol)
        xg, yg = vector(M, dt, 1, 1), vector(N, dt, -3, 0)
        Xg, Yg = xg.astype(np.float64), yg.astype(np.float64)
        A2 = A.copy()
        g9.ger(-0.5, xg, yg, A2)
        check(f"ger {M}x{N}", A2, Ad - 0.5 * np.outer(Xg, Yg), abs(Ad) + 0.5 * np.outer(abs(Xg), abs(Yg)), tol)
    B = rng.uniform(-1, 1, (300, 400)).astype(dt)
    Bd = B.astype(np.float64)
    y = g9.gemv(B[10:200, 5:305], B[0, :300])
    check("gemv submatrix", y, Bd[10:200, 5:305] @ Bd[0, :300], abs(Bd[10:200, 5:305]) @ abs(Bd[0, :300]), tol)


@pytest.mark.parametrize("t,dt", [(abi.S, np.float32), (abi.D, np.float64), (abi.H, np.float16)])
def test_elementwise_bit_exact_vs_oracle(gpu_lib, oracle, t, dt):
    """axpy and ger are element-wise FMAs in R: the GPU result equals the oracle's bit for bit, strides included."""
    for n, ix, iy in ((100003, 1, 1), (5001, 3, -2), (777, -1, 1)):
        x = rng.uniform(-1, 1, n * abs(ix)).astype(dt)
        y = rng.uniform(-1, 1, n * abs(iy)).astype(dt)
        yg, yo = y.copy(), y.copy()
        assert gpu_lib.axpy(t, n, -1.3, x.ctypes.data, ix, yg.ctypes.data, iy) == 0
        assert oracle.axpy(t, n, -1.3, x.ctypes.data, ix, yo.ctypes.data, iy) == 0
        assert np.array_equal(yg.view(np.uint8), yo.view(np.uint8))
    for M, N, lda in ((257, 1031, 1031), (64, 100, 130), (1000, 3, 5)):
        x = rng.uniform(-1, 1, M).astype(dt)
        y = rng.uniform(-1, 1, 2 * N).astype(dt)
        A = rng.uniform(-1, 1, (M, lda)).astype(dt)
        Ag, Ao = A.copy(), A.copy()
        assert gpu_lib.ger(t, M, N, 0.3, x.ctypes.data, 1, y.ctypes.data, -2, Ag.ctypes.data, lda) == 0
        assert oracle.ger(t, M, N, 0.3, x.ctypes.data, 1, y.ctypes.data, -2, Ao.ctypes.data, lda) == 0
        assert np.array_equal(Ag.view(np.uint8), Ao.view(np.uint8))


@pytest.mark.parametrize("t,dt", [(abi.S, np.float32), (abi.D, np.float64), (abi.H, np.float16)])
def test_iamax_rules(gpu_lib, oracle, t, dt):
    r, ro = ctypes.c_int64(), ctypes.c_int64()
    cases = [np.array([1.0, -3.0, 3.0, np.nan, -3.0]), np.full(7, np.nan), np.array([np.nan, 0.0, -0.0]),
             np.array([-0.0, 0.0]), np.zeros(300000)]
    big = rng.uniform(-1, 1, 1 << 20)
    big[[7, 500000, 1048000]] = 2.0          # three ties: the first wins
    big[123] = np.nan
    cases.append(big)
    for c in cases:
        x = c.astype(dt)
        for inc in (1, -1, 2):
            n = len(x) // abs(inc)
            assert gpu_lib.iamax(t, n, x.ctypes.data, inc, ctypes.byref(r)) == 0
            assert oracle.iamax(t, n, x.ctypes.data, inc, ctypes.byref(ro)) == 0
            assert r.value == ro.value, (len(x), inc, r.value, ro.value)
    x = np.ones(4, dt)
    assert gpu_lib.iamax(t, 0, x.ctypes.data, 1, ctypes.byref(r)) == 0 and r.value == -1
    assert gpu_lib.iamax(t, 4, x.ctypes.data, 0, ctypes.byref(r)) == -3


def test_reductions_deterministic_and_fp64(gpu_lib):
    """FP64 accumulation: the dot of FP32 vectors equals the exactly rounded FP64 sum to 1e-12 relative, and two
    calls give the same bits (fixed grid, fixed combine order)."""
    n = 1 << 22
    x = rng.uniform(-1, 1, n).astype(np.float32)
    y = rng.uniform(-1, 1, n).astype(np.float32)
    w1, w2 = ctypes.c_double(), ctypes.c_double()
    assert gpu_lib.dot(abi.S, n, x.ctypes.data, 1, y.ctypes.data, 1, ctypes.byref(w1)) == 0
    assert gpu_lib.dot(abi.S, n, x.ctypes.data, 1, y.ctypes.data, 1, ctypes.byref(w2)) == 0
    assert w1.value == w2.value
    exact = float(np.sum(x.astype(np.float64) * y.astype(np.float64), dtype=np.float64))
    assert abs(w1.value - exact) <= 1e-12 * float(np.abs(x.astype(np.float64)) @ np.abs(y.astype(np.float64)))


def test_level12_full_size_properties(gpu_lib):
    """n = 2^28 (BASELINE level-1 size) checked through size-independent properties on device-resident data."""
    torch = pytest.importorskip("torch")
    n = 1 << 28
    x = torch.zeros(n, dtype=torch.float32, device="cuda")
    idx = 200_000_017
    x[idx] = -5.0
    x[idx + 7] = 5.0                 # a tie after the first maximum
    torch.cuda.synchronize()
    r = ctypes.c_int64()
    assert gpu_lib.iamax(abi.S, n, x.data_ptr(), 1, ctypes.byref(r)) == 0 and r.value == idx
    x.fill_(0.5)
    torch.cuda.synchronize()      # torch works on its own stream; the library on its own one
    w = ctypes.c_double()
    assert gpu_lib.asum(abi.S, n, x.data_ptr(), 1, ctypes.byref(w)) == 0 and w.value == 0.5 * n
    assert gpu_lib.dot(abi.S, n, x.data_ptr(), 1, x.data_ptr(), 1, ctypes.byref(w)) == 0 and w.value == 0.25 * n
    y = torch.full((n,), 2.0, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    assert gpu_lib.axpy(abi.S, n, 4.0, x.data_ptr(), 1, y.data_ptr(), 1) == 0
    assert float(y.min()) == 4.0 and float(y.max()) == 4.0
    del x, y
    torch.cuda.empty_cache()
