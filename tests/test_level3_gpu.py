"""GPU parity of the level-3 set on GEMM (SYMM, SYRK, SYR2K, TRMM, TRSM) through the NumPy module, with the cases,
error metric and limits of the reference's lib/test_level3.py:4-140 against FP64 NumPy on the same rounded inputs:
elementwise |W - ref| / (|alpha|·|A||B| + |beta|·|C0|) with mean / max limits per type, the untouched triangle of
SYRK / SYR2K compared bit for bit, TRSM by the relative error of the solution. Plus sizes above one band (n >= 512:
four banded GEMMs) and above one TRSM block (128)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# (name, dtype, accurate, mean limit, max limit): lib/test_level3.py:17-19
TYPES = [("fp16", np.float16, False, 4.9e-4, 5e-3), ("fp16 acc.", np.float16, True, 4.9e-4, 5e-3),
         ("fp32", np.float32, False, 1e-6, 1e-5), ("fp64", np.float64, False, 1e-14, 1e-13)]
TRSM_TOL = {(np.float64, False): 1e-12, (np.float32, False): 1e-4, (np.float16, False): 5e-3, (np.float16, True): 5e-3}


def f64(x):
    return x.astype(np.float64)


def err(W, ref, scale, mask=None):
    e = np.abs(f64(W) - ref) / np.maximum(scale, 1e-30)
    if mask is not None:
        e = e[mask]
    return e.mean(), e.max()


def rnd(rng, shape, dt):
    return rng.uniform(-1, 1, shape).astype(dt)


@pytest.mark.parametrize("name,dt,acc,tol_avg,tol_max", TYPES)
@pytest.mark.parametrize("M,N", [(70, 45), (600, 130)])
def test_symm(g9, name, dt, acc, tol_avg, tol_max, M, N):
    rng = np.random.default_rng(1)
    for side in "LR":
        for uplo in "LU":
            n = M if side == "L" else N
            S = rnd(rng, (n, n), dt)
            Ssym = np.tril(f64(S)) + np.tril(f64(S), -1).T if uplo == "L" else np.triu(f64(S)) + np.triu(f64(S), 1).T
            B, C0 = rnd(rng, (M, N), dt), rnd(rng, (M, N), dt)
            W = g9.symm(S, B, side, uplo, 2.0, -1.0, C0.copy(), accurate=acc)
            P = Ssym @ f64(B) if side == "L" else f64(B) @ Ssym
            Pa = np.abs(Ssym) @ np.abs(f64(B)) if side == "L" else np.abs(f64(B)) @ np.abs(Ssym)
            a, m = err(W, 2.0 * P - f64(C0), 2.0 * Pa + np.abs(f64(C0)))
            assert a <= tol_avg and m <= tol_max, (name, side, uplo, a, m)


@pytest.mark.parametrize("name,dt,acc,tol_avg,tol_max", TYPES)
@pytest.mark.parametrize("N,K", [(60, 90), (700, 300)])
def test_syrk_syr2k(g9, name, dt, acc, tol_avg, tol_max, N, K):
    rng = np.random.default_rng(2)
    for uplo in "LU":
        for tr in (False, True):
            A, B, C0 = rnd(rng, (K, N) if tr else (N, K), dt), rnd(rng, (K, N) if tr else (N, K), dt), rnd(rng, (N, N), dt)
            oA, oB = (f64(A).T, f64(B).T) if tr else (f64(A), f64(B))
            mask = np.tril(np.ones((N, N), bool)) if uplo == "L" else np.triu(np.ones((N, N), bool))
            W = g9.syrk(A, uplo, tr, 0.7, 0.3, C0.copy(), accurate=acc)
            a, m = err(W, 0.7 * oA @ oA.T + 0.3 * f64(C0), 0.7 * np.abs(oA) @ np.abs(oA).T + 0.3 * np.abs(f64(C0)), mask)
            assert a <= tol_avg and m <= tol_max, ("syrk", name, uplo, tr, a, m)
            assert np.array_equal(W[~mask], C0[~mask])
            W = g9.syr2k(A, B, uplo, tr, 0.7, 0.3, C0.copy(), accurate=acc)
            a, m = err(W, 0.7 * (oA @ oB.T + oB @ oA.T) + 0.3 * f64(C0),
                       0.7 * (np.abs(oA) @ np.abs(oB).T + np.abs(oB) @ np.abs(oA).T) + 0.3 * np.abs(f64(C0)), mask)
            assert a <= tol_avg and m <= tol_max, ("syr2k", name, uplo, tr, a, m)
            assert np.array_equal(W[~mask], C0[~mask])


@pytest.mark.parametrize("name,dt,acc,tol_avg,tol_max", TYPES)
@pytest.mark.parametrize("M,N", [(50, 70), (530, 90)])
def test_trmm(g9, name, dt, acc, tol_avg, tol_max, M, N):
    rng = np.random.default_rng(3)
    for side in "LR":
        for uplo in "LU":
            for ta in (False, True):
                for dg in (False, True):
                    n = M if side == "L" else N
                    A, B = rnd(rng, (n, n), dt), rnd(rng, (M, N), dt)
                    T = np.tril(f64(A)) if uplo == "L" else np.triu(f64(A))
                    if dg:
                        np.fill_diagonal(T, 1.0)
                    T = T.T if ta else T
                    W = g9.trmm(A, B, side, uplo, ta, dg, 1.5, accurate=acc)
                    P = T @ f64(B) if side == "L" else f64(B) @ T
                    Pa = np.abs(T) @ np.abs(f64(B)) if side == "L" else np.abs(f64(B)) @ np.abs(T)
                    a, m = err(W, 1.5 * P, 1.5 * Pa)
                    assert a <= tol_avg and m <= tol_max, (name, side, uplo, ta, dg, a, m)


@pytest.mark.parametrize("dt,acc", [(np.float64, False), (np.float32, False), (np.float16, False), (np.float16, True)])
def test_trsm(g9, dt, acc):
    """lib/test_level3.py:103-131: A triangular with a dominant diagonal (diag=1: the diagonal is not read)."""
    rng = np.random.default_rng(4)
    tol = TRSM_TOL[(dt, acc)]
    for side in "LR":
        for uplo in "LU":
            for ta in (False, True):
                for dg in (False, True):
                    for (M, N) in [(40, 30), (300, 200)]:
                        n = M if side == "L" else N
                        A = rng.uniform(-1, 1, (n, n)).astype(np.float32)
                        A[np.diag_indices(n)] = n if not dg else 0.5
                        if dg:
                            A *= 1.0 / n
                            A[np.diag_indices(n)] = 123.0
                        B = rng.uniform(-1, 1, (M, N)).astype(np.float32)
                        A, B = A.astype(dt), B.astype(dt)
                        T = np.tril(f64(A)) if uplo == "L" else np.triu(f64(A))
                        if dg:
                            np.fill_diagonal(T, 1.0)
                        T = T.T if ta else T
                        Xr = (np.linalg.solve(T, 2.0 * f64(B)) if side == "L"
                              else np.linalg.solve(T.T, 2.0 * f64(B).T).T)
                        X = f64(g9.trsm(A, B, side, uplo, ta, dg, 2.0, accurate=acc))
                        e = np.abs(X - Xr).max() / np.abs(Xr).max()
                        assert e <= tol, (np.dtype(dt).name, acc, side, uplo, ta, dg, M, N, e)


@pytest.mark.parametrize("dt", [np.float64, np.float32])
def test_trsm_large_recursive(g9, dt):
    """Triangles large enough for the recursive solve with composed 256- and 512-row leaf inverses, at sizes that
    leave ragged tails (n = 1300: 512-row leaves, then a 256-row leaf and a 20-row one; n = 700: 256-row leaves),
    every side / triangle / transpose / diagonal combination."""
    rng = np.random.default_rng(9)
    tol = TRSM_TOL[(dt, False)]
    for side, (M, N) in (("L", (1300, 96)), ("R", (80, 700))):
        for uplo in "LU":
            for ta in (False, True):
                for dg in (False, True):
                    n = M if side == "L" else N
                    A = rng.uniform(-1, 1, (n, n))
                    if dg:
                        A *= 1.0 / n
                        A[np.diag_indices(n)] = 123.0
                    else:
                        A[np.diag_indices(n)] = n
                    A = A.astype(dt)
                    B = rng.uniform(-1, 1, (M, N)).astype(dt)
                    T = np.tril(f64(A)) if uplo == "L" else np.triu(f64(A))
                    if dg:
                        np.fill_diagonal(T, 1.0)
                    T = T.T if ta else T
                    Xr = (np.linalg.solve(T, 2.0 * f64(B)) if side == "L"
                          else np.linalg.solve(T.T, 2.0 * f64(B).T).T)
                    X = f64(g9.trsm(A, B, side, uplo, ta, dg, 2.0))
                    e = np.abs(X - Xr).max() / np.abs(Xr).max()
                    assert e <= tol, (np.dtype(dt).name, side, uplo, ta, dg, M, N, e)


def test_views_and_degenerate(g9):
    """Transposed views of A (triangle and transA flip without a copy), K = 0 SYRK (C = beta·C on the triangle),
    empty shapes."""
    rng = np.random.default_rng(5)
    A = rnd(rng, (64, 64), np.float32)
    B = rnd(rng, (64, 40), np.float32)
    At = A.T   # a view: the library reads the same memory with the triangle swapped
    ref = np.tril(f64(At)) + np.tril(f64(At), -1).T
    W = g9.symm(At, B, "L", "L")
    assert err(W, ref @ f64(B), np.abs(ref) @ np.abs(f64(B)))[1] <= 1e-5
    T = np.triu(f64(At))
    W = g9.trmm(At, B, "L", "U")
    assert err(W, T @ f64(B), np.abs(T) @ np.abs(f64(B)))[1] <= 1e-5
    C0 = rnd(rng, (16, 16), np.float32)
    W = g9.syrk(np.zeros((16, 0), np.float32), "L", False, 1.0, 0.5, C0.copy())
    low = np.tril(np.ones((16, 16), bool))
    assert np.allclose(W[low], 0.5 * C0[low]) and np.array_equal(W[~low], C0[~low])
