"""GPU parity of the rest of levels 1-2 (scal, copy, swap, rot, rotm; symv, trmv, trsv, syr, syr2; gbmv, sbmv, tbmv,
tbsv, spmv, tpmv, tpsv, spr, spr2) through the NumPy module, against FP64 NumPy on the same rounded inputs with the
error rules of the reference's lib/test_level12.py (elementwise |W - ref| / scale, scale = |alpha|·|A||x| + |beta||y|;
solves by the relative error of the solution) and the layouts of lib/gen9blas.h:151-154 (row-major band
A[i, KL + j - i], packed rows of the triangle). Strided and negative-stride vectors, both triangles, transposes and
unit diagonals; FP16 is computed in FP32."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TYPES = [(np.float32, 2e-6), (np.float64, 1e-13), (np.float16, 2e-3)]
SOLVE_TOL = {np.float32: 1e-4, np.float64: 1e-12, np.float16: 5e-3}


def f64(x):
    return np.asarray(x, np.float64)


FLOOR = 0.05   # FP16 only: results below this magnitude are judged by absolute error (FP16 subnormals start at 6e-5)


def emax(W, ref, scale, dt=None):
    floor = FLOOR if (dt or np.asarray(W).dtype) == np.float16 else 1e-30
    return float((np.abs(f64(W) - ref) / np.maximum(scale, floor)).max())


def rnd(rng, shape, dt):
    return rng.uniform(-1, 1, shape).astype(dt)


def band_dense(Ab, M, N, KL, KU):
    D = np.zeros((M, N))
    for i in range(M):
        for j in range(max(0, i - KL), min(N, i + KU + 1)):
            D[i, j] = Ab[i, KL + j - i]
    return D


def packed_dense(Ap, n, upper):
    D = np.zeros((n, n))
    p = 0
    for i in range(n):
        js = range(i, n) if upper else range(0, i + 1)
        for j in js:
            D[i, j] = Ap[p]
            p += 1
    return D


def tri(D, upper, unit):
    T = np.triu(D) if upper else np.tril(D)
    if unit:
        np.fill_diagonal(T, 1.0)
    return T


def sym_of(D, upper):
    T = np.triu(D) if upper else np.tril(D)
    return T + T.T - np.diag(np.diag(T))


@pytest.mark.parametrize("dt,tol", TYPES)
def test_level1_extras(g9, dt, tol):
    rng = np.random.default_rng(1)
    n = 3001
    for sx, sy in ((1, 1), (2, 3), (-1, 2), (3, -2)):
        x = rnd(rng, n * abs(sx), dt)[::sx]
        y = rnd(rng, n * abs(sy), dt)[::sy]
        x0, y0 = f64(x.copy()), f64(y.copy())
        g9.scal(0.75, x)
        assert emax(x, 0.75 * x0, np.abs(0.75 * x0)) <= tol
        x[...] = x0.astype(dt)
        g9.copy(x, y)
        assert np.array_equal(y, x)
        y[...] = y0.astype(dt)
        g9.swap(x, y)
        assert np.array_equal(f64(x), y0) and np.array_equal(f64(y), x0)
        x[...], y[...] = x0.astype(dt), y0.astype(dt)
        c, s = 0.6, 0.8
        g9.rot(x, y, c, s)
        sc = c * np.abs(x0) + s * np.abs(y0)
        assert emax(x, c * x0 + s * y0, sc) <= tol and emax(y, c * y0 - s * x0, sc) <= tol
        for flag, h in ((-1.0, (0.5, -0.25, 0.75, 1.5)), (0.0, (9.0, -0.25, 0.75, 9.0)), (1.0, (0.5, 9.0, 9.0, 1.5))):
            x[...], y[...] = x0.astype(dt), y0.astype(dt)
            h11, h21, h12, h22 = h
            if flag == 0.0:
                h11, h22 = 1.0, 1.0
            elif flag == 1.0:
                h21, h12 = -1.0, 1.0
            g9.rotm(x, y, (flag, h[0], h[1], h[2], h[3]))
            sc = np.abs(h11 * x0) + np.abs(h12 * y0) + np.abs(h21 * x0) + np.abs(h22 * y0)
            assert emax(x, h11 * x0 + h12 * y0, sc) <= tol and emax(y, h21 * x0 + h22 * y0, sc) <= tol
        x[...], y[...] = x0.astype(dt), y0.astype(dt)
        g9.rotm(x, y, (-2.0, 1, 2, 3, 4))   # identity
        assert np.array_equal(f64(x), x0) and np.array_equal(f64(y), y0)


@pytest.mark.parametrize("dt,tol", TYPES)
@pytest.mark.parametrize("n", [77, 600])
def test_dense_symmetric_triangular(g9, dt, tol, n):
    rng = np.random.default_rng(2)
    for uplo in "LU":
        up = uplo == "U"
        A = rnd(rng, (n, n), dt)
        x, y0 = rnd(rng, n, dt), rnd(rng, n, dt)
        S = sym_of(f64(A), up)
        W = g9.symv(A, x, uplo, 1.5, -0.5, y0.copy())
        assert emax(W, 1.5 * S @ f64(x) - 0.5 * f64(y0), 1.5 * np.abs(S) @ np.abs(f64(x)) + 0.5 * np.abs(f64(y0))) <= tol
        for trans in (False, True):
            for diag in (False, True):
                T = tri(f64(A), up, diag)
                T = T.T if trans else T
                W = g9.trmv(A, x.copy(), uplo, trans, diag)
                assert emax(W, T @ f64(x), np.abs(T) @ np.abs(f64(x))) <= tol, (uplo, trans, diag)
                Ad = A.copy()
                Ad[np.diag_indices(n)] = n if not diag else 0.5   # dominant diagonal (unit: the diagonal is not read)
                if diag:
                    Ad = (f64(Ad) / n).astype(dt)
                Td = tri(f64(Ad), up, diag)
                Td = Td.T if trans else Td
                z = np.linalg.solve(Td, f64(x))
                W = g9.trsv(Ad, x.copy(), uplo, trans, diag)
                assert np.abs(f64(W) - z).max() / np.abs(z).max() <= SOLVE_TOL[dt], (uplo, trans, diag)
        xx, yy = rnd(rng, n, dt), rnd(rng, n, dt)
        C0 = A.copy()
        mask = np.triu(np.ones((n, n), bool)) if up else np.tril(np.ones((n, n), bool))
        W = g9.syr(0.5, xx, C0.copy(), uplo)
        ref = f64(C0) + 0.5 * np.outer(f64(xx), f64(xx))
        assert emax(W[mask], ref[mask], (np.abs(f64(C0)) + 0.5 * np.abs(np.outer(f64(xx), f64(xx))))[mask]) <= tol
        assert np.array_equal(W[~mask], C0[~mask])
        W = g9.syr2(0.5, xx, yy, C0.copy(), uplo)
        o = np.outer(f64(xx), f64(yy))
        ref = f64(C0) + 0.5 * (o + o.T)
        sc = np.abs(f64(C0)) + 0.5 * (np.abs(o) + np.abs(o.T))
        assert emax(W[mask], ref[mask], sc[mask]) <= tol and np.array_equal(W[~mask], C0[~mask])


@pytest.mark.parametrize("dt,tol", TYPES)
def test_banded(g9, dt, tol):
    rng = np.random.default_rng(3)
    for (M, N, KL, KU) in ((70, 50, 3, 5), (600, 900, 17, 0), (300, 300, 0, 40)):
        Ab = rnd(rng, (M, KL + KU + 1), dt)
        D = band_dense(f64(Ab), M, N, KL, KU)
        for trans in (False, True):
            op = D.T if trans else D
            x = rnd(rng, op.shape[1], dt)
            y0 = rnd(rng, op.shape[0], dt)
            W = g9.gbmv(Ab, x, M, N, KL, KU, 0.75, 0.25, y0.copy(), trans)
            assert emax(W, 0.75 * op @ f64(x) + 0.25 * f64(y0),
                        0.75 * np.abs(op) @ np.abs(f64(x)) + 0.25 * np.abs(f64(y0))) <= tol, (M, N, KL, KU, trans)
    n = 400
    for K in (0, 7, 63):
        for uplo in "LU":
            up = uplo == "U"
            Ab = rnd(rng, (n, K + 1), dt)
            D = band_dense(f64(Ab), n, n, 0 if up else K, K if up else 0)
            S = sym_of(D, up)
            x, y0 = rnd(rng, n, dt), rnd(rng, n, dt)
            W = g9.sbmv(Ab, x, K, uplo, 1.25, -0.5, y0.copy())
            assert emax(W, 1.25 * S @ f64(x) - 0.5 * f64(y0),
                        1.25 * np.abs(S) @ np.abs(f64(x)) + 0.5 * np.abs(f64(y0))) <= tol, (K, uplo)
            for trans in (False, True):
                for diag in (False, True):
                    T = tri(D, up, diag)
                    T = T.T if trans else T
                    W = g9.tbmv(Ab, x.copy(), K, uplo, trans, diag)
                    assert emax(W, T @ f64(x), np.abs(T) @ np.abs(f64(x))) <= tol, (K, uplo, trans, diag)
                    Ad = Ab.copy()
                    dcol = 0 if up else K   # the diagonal's column in the band array
                    if diag:                # unit diagonal (not read): small off-diagonals keep the solve stable
                        Ad = (f64(Ad) / (2 * K + 2)).astype(dt)
                    Ad[:, dcol] = 4.0 + K   # dominant diagonal
                    Td = tri(band_dense(f64(Ad), n, n, 0 if up else K, K if up else 0), up, diag)
                    Td = Td.T if trans else Td
                    z = np.linalg.solve(Td, f64(x))
                    W = g9.tbsv(Ad, x.copy(), K, uplo, trans, diag)
                    assert np.abs(f64(W) - z).max() / np.abs(z).max() <= SOLVE_TOL[dt], (K, uplo, trans, diag)


@pytest.mark.parametrize("dt,tol", TYPES)
@pytest.mark.parametrize("n", [45, 300])
def test_packed(g9, dt, tol, n):
    rng = np.random.default_rng(4)
    for uplo in "LU":
        up = uplo == "U"
        Ap = rnd(rng, n * (n + 1) // 2, dt)
        D = packed_dense(f64(Ap), n, up)
        S = D + D.T - np.diag(np.diag(D))
        x, y0 = rnd(rng, n, dt), rnd(rng, n, dt)
        W = g9.spmv(Ap, x, uplo, 0.5, 1.5, y0.copy())
        assert emax(W, 0.5 * S @ f64(x) + 1.5 * f64(y0), 0.5 * np.abs(S) @ np.abs(f64(x)) + 1.5 * np.abs(f64(y0))) <= tol
        for trans in (False, True):
            for diag in (False, True):
                T = tri(D, up, diag)
                T = T.T if trans else T
                W = g9.tpmv(Ap, x.copy(), uplo, trans, diag)
                assert emax(W, T @ f64(x), np.abs(T) @ np.abs(f64(x))) <= tol, (uplo, trans, diag)
                Dd = D.copy() / (n if diag else 1)   # unit diagonal (not read): small off-diagonals keep it stable
                np.fill_diagonal(Dd, n)
                Apd = np.array([Dd[i, j] for i in range(n) for j in (range(i, n) if up else range(0, i + 1))]).astype(dt)
                Td = tri(packed_dense(f64(Apd), n, up), up, diag)
                Td = Td.T if trans else Td
                z = np.linalg.solve(Td, f64(x))
                W = g9.tpsv(Apd, x.copy(), uplo, trans, diag)
                assert np.abs(f64(W) - z).max() / np.abs(z).max() <= SOLVE_TOL[dt], (uplo, trans, diag)
        xx, yy = rnd(rng, n, dt), rnd(rng, n, dt)
        o = np.outer(f64(xx), f64(yy))
        W = g9.spr(0.5, xx, Ap.copy(), uplo)
        ref = packed_dense(f64(Ap), n, up) + 0.5 * tri(np.outer(f64(xx), f64(xx)), up, False)
        got = packed_dense(f64(W), n, up)
        m = np.triu(np.ones((n, n), bool)) if up else np.tril(np.ones((n, n), bool))
        assert emax(got[m], ref[m], (np.abs(D) + 0.5 * np.abs(np.outer(f64(xx), f64(xx))))[m], dt) <= tol
        W = g9.spr2(0.5, xx, yy, Ap.copy(), uplo)
        ref = D + 0.5 * (o + o.T)
        got = packed_dense(f64(W), n, up)
        assert emax(got[m], ref[m], (np.abs(D) + 0.5 * (np.abs(o) + np.abs(o.T)))[m], dt) <= tol


@pytest.mark.parametrize("dt", [np.float32, np.float64])
def test_solves_and_products_large_strided(g9, dt):
    """Sizes spanning many 64-row blocks of the look-back solve and many 128×128 tiles of the triangle products, with
    strided and negative-stride vectors: trsv (n = 2000), tpsv (n = 1500), tbsv (n = 3000, K = 150: three blocks
    back), symv / trmv / spmv on the same triangles."""
    rng = np.random.default_rng(9)
    tol = SOLVE_TOL[dt]
    for n, step in ((2000, 2), (1300, -3)):
        buf = rnd(rng, n * abs(step), dt)
        for uplo in "LU":
            up = uplo == "U"
            A = rnd(rng, (n, n), dt)
            A[np.diag_indices(n)] = 2.0 * np.sqrt(n)
            for trans in (False, True):
                for diag in (False, True):
                    Ad = (f64(A) / (n if diag else 1)).astype(dt) if diag else A
                    T = tri(f64(Ad), up, diag)
                    T = T.T if trans else T
                    x = buf.copy()[::step]
                    z = np.linalg.solve(T, f64(x))
                    W = g9.trsv(Ad, x, uplo, trans, diag)
                    assert np.abs(f64(W) - z).max() / np.abs(z).max() <= tol, (n, uplo, trans, diag)
                    x = buf.copy()[::step]
                    W = g9.trmv(Ad, x, uplo, trans, diag)
                    assert emax(W, T @ f64(buf[::step]), np.abs(T) @ np.abs(f64(buf[::step]))) <= 1e-5
            S = sym_of(f64(A), up)
            y = buf.copy()[::step]
            W = g9.symv(A, buf[::step], uplo, 0.5, 2.0, y)
            assert emax(W, 0.5 * S @ f64(buf[::step]) + 2.0 * f64(buf[::step]),
                        0.5 * np.abs(S) @ np.abs(f64(buf[::step])) + 2.0 * np.abs(f64(buf[::step]))) <= 1e-5
    n = 1500
    for uplo in "LU":
        up = uplo == "U"
        D = tri(rnd(rng, (n, n), np.float64), up, False)
        np.fill_diagonal(D, 2.0 * np.sqrt(n))
        Ap = np.array([D[i, j] for i in range(n) for j in (range(i, n) if up else range(0, i + 1))]).astype(dt)
        Dq = packed_dense(f64(Ap), n, up)
        for trans in (False, True):
            T = Dq.T if trans else Dq
            x = rnd(rng, 2 * n, dt)[::-2]   # a negative-stride view, solved in place
            z = np.linalg.solve(T, f64(x))
            W = g9.tpsv(Ap, x, uplo, trans, False)
            assert np.abs(f64(W) - z).max() / np.abs(z).max() <= tol, ("tpsv", uplo, trans)
        S = Dq + Dq.T - np.diag(np.diag(Dq))
        x = rnd(rng, n, dt)
        W = g9.spmv(Ap, x, uplo)
        assert emax(W, S @ f64(x), np.abs(S) @ np.abs(f64(x))) <= 1e-5
    n, K = 3000, 150
    for uplo in "LU":
        up = uplo == "U"
        Ab = rnd(rng, (n, K + 1), dt)
        Ab[:, 0 if up else K] = 4.0 * np.sqrt(K)
        Td0 = band_dense(f64(Ab), n, n, 0 if up else K, K if up else 0)
        for trans in (False, True):
            T = Td0.T if trans else Td0
            x = rnd(rng, 3 * n, dt)[::3]
            z = np.linalg.solve(T, f64(x))
            W = g9.tbsv(Ab, x, K, uplo, trans, False)
            assert np.abs(f64(W) - z).max() / np.abs(z).max() <= tol, ("tbsv", uplo, trans)
