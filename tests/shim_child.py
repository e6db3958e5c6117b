"""Child process for the LD_PRELOAD-library tests: loads libgen9blas_blas.so the way a program linked against
libblas.so.3 would see it (its CPU BLAS, OpenBLAS, chosen by GEN9BLAS_BLAS_CPU), runs one group of CBLAS / Fortran BLAS
calls and prints a JSON report. The environment (GEN9BLAS_BLAS, GEN9BLAS_BLAS_INFO) is set by the parent test.

    python tests/shim_child.py <group>
"""
import ctypes
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(HERE, "golden"))
from make_golden import (GEMM_CASES, L3_SYMM, L3_SYRK, L3_TRXM, ColMajor, Left, NoTrans, RowMajor, Trans,  # noqa: E402
                         Unit, Upper, gemm_inputs, l3_cases, l3_inputs, l3_key, run_l3, vec_inputs)

sys.path.insert(0, os.path.join(ROOT, "oracle"))
import cpu_blas  # noqa: E402
_openblas = cpu_blas.preload_openblas_deps()
if _openblas is None:
    sys.exit("no OpenBLAS found: set GEN9BLAS_OPENBLAS to a libopenblas shared object with cblas_* names")
os.environ.setdefault("GEN9BLAS_BLAS_CPU", _openblas)
L = ctypes.CDLL(os.path.join(ROOT, "gen9-gpu-blas_b200", "libgen9blas_blas.so"))
I, P = ctypes.c_int, ctypes.c_void_p
REF = np.load(os.path.join(HERE, "golden", "ref_cblas_outputs.npz"))


def rel(got, want, scale):
    return float((np.abs(np.asarray(got, np.float64) - np.asarray(want, np.float64)) / scale).max())


def group_cblas_gemm():
    """Row/column-major, all transposes, alpha/beta: compared with the reference CBLAS layer's own outputs."""
    out = {}
    for tag, F in (("s", ctypes.c_float), ("d", ctypes.c_double)):
        f = getattr(L, f"cblas_{tag}gemm")
        f.argtypes = [I, I, I, I, I, I, F, P, I, P, I, F, P, I]
        worst = 0.0
        for order in (RowMajor, ColMajor):
            for (M, N, K, al, be) in GEMM_CASES:
                for ta in (NoTrans, Trans):
                    for tb in (NoTrans, Trans):
                        A, B, C0 = gemm_inputs(tag, order, ta, tb, M, N, K)
                        if order == RowMajor:
                            As, Bs, Cs = np.ascontiguousarray(A), np.ascontiguousarray(B), C0.copy()
                            lda, ldb, ldc = A.shape[1], B.shape[1], N
                        else:
                            As, Bs, Cs = np.asfortranarray(A), np.asfortranarray(B), np.asfortranarray(C0.copy())
                            lda, ldb, ldc = A.shape[0], B.shape[0], M
                        f(order, ta, tb, M, N, K, al, As.ctypes.data, lda, Bs.ctypes.data, ldb, be, Cs.ctypes.data, ldc)
                        a64 = A.astype(np.float64) if ta == NoTrans else A.astype(np.float64).T
                        b64 = B.astype(np.float64) if tb == NoTrans else B.astype(np.float64).T
                        scale = abs(al) * np.abs(a64) @ np.abs(b64) + abs(be) * np.abs(C0.astype(np.float64))
                        want = REF[f"{tag}gemm_o{order}_t{ta}{tb}_{M}x{N}x{K}"]
                        worst = max(worst, rel(np.ascontiguousarray(Cs), want, scale))
        out[f"{tag}gemm_vs_ref_cblas"] = worst
    return out


def l3_scale(tag, case):
    """Denominator of the elementwise metric of lib/test_level3.py for one level-3 case (logical matrices)."""
    op = case[0]
    f64 = lambda x: x.astype(np.float64)
    if op == "symm":
        side, uplo = case[2], case[3]
        M, N, al, be = L3_SYMM
        A, B, C0 = l3_inputs(tag, op, *case[1:])
        S = np.abs(f64(A))
        return abs(al) * (S @ np.abs(f64(B)) if side == Left else np.abs(f64(B)) @ S) + abs(be) * np.abs(f64(C0))
    if op in ("syrk", "syr2k"):
        trans = case[3]
        N, K, al, be = L3_SYRK
        A, B, C0 = l3_inputs(tag, op, *case[1:])
        oA, oB = (f64(A).T, f64(B).T) if trans == Trans else (f64(A), f64(B))
        P = np.abs(oA) @ np.abs(oA).T if op == "syrk" else np.abs(oA) @ np.abs(oB).T + np.abs(oB) @ np.abs(oA).T
        return abs(al) * P + abs(be) * np.abs(f64(C0))
    side = case[2]
    M, N, al = L3_TRXM
    A, B = l3_inputs(tag, op, *case[1:])
    return abs(al) * (np.abs(f64(A)) @ np.abs(f64(B)) if side == Left else np.abs(f64(B)) @ np.abs(f64(A)))


def group_level3():
    """SYMM / SYRK / SYR2K / TRMM / TRSM, row- and column-major, every option: compared with the reference CBLAS
    layer's own outputs. Metric of lib/test_level3.py: elementwise for the products (the untouched triangle of
    SYRK / SYR2K must match exactly), max|X - X_ref| / max|X_ref| for TRSM."""
    out = {}
    for tag in ("s", "d"):
        worst = {"symm": 0.0, "syrk": 0.0, "syr2k": 0.0, "trmm": 0.0, "trsm": 0.0}
        other_exact = True
        for case in l3_cases():
            got = run_l3(L, tag, case)
            want = REF[l3_key(tag, case)]
            op = case[0]
            if op == "trsm":
                e = float(np.abs(got.astype(np.float64) - want).max() / np.abs(want).max())
            else:
                e = rel(got, want, np.maximum(l3_scale(tag, case), 1e-30))
            worst[op] = max(worst[op], e)
            if op in ("syrk", "syr2k"):   # the triangle that is not uplo stays as C0
                order, uplo = case[1], case[2]
                lower_logical = (uplo != Upper)
                mask = np.triu(np.ones(got.shape, bool), 1) if lower_logical else np.tril(np.ones(got.shape, bool), -1)
                other_exact &= bool(np.array_equal(got[mask], want[mask]))
        for op, v in worst.items():
            out[f"{tag}{op}"] = v
        out[f"{tag}_other_triangle_exact"] = other_exact
    return out


def group_fortran_and_l12():
    out = {}
    rng = np.random.default_rng(3)
    for tag, F, dt in (("s", ctypes.c_float, np.float32), ("d", ctypes.c_double, np.float64)):
        # Fortran xGEMM_ (column-major), padded leading dimensions, all transposes
        g = getattr(L, f"{tag}gemm_")
        g.argtypes = [ctypes.c_char_p, ctypes.c_char_p] + [ctypes.POINTER(I)] * 3 + [ctypes.POINTER(F), P,
                      ctypes.POINTER(I), P, ctypes.POINTER(I), ctypes.POINTER(F), P, ctypes.POINTER(I)]
        worst = 0.0
        for ta in "NT":
            for tb in "nt":
                M, N, K = 45, 38, 70
                A = rng.uniform(-1, 1, (M, K) if ta == "N" else (K, M)).astype(dt)
                B = rng.uniform(-1, 1, (K, N) if tb == "n" else (N, K)).astype(dt)
                C0 = rng.uniform(-1, 1, (M, N)).astype(dt)
                Af = np.zeros((A.shape[0] + 3, A.shape[1]), dt, order="F"); Af[:A.shape[0]] = A
                Bf = np.zeros((B.shape[0] + 1, B.shape[1]), dt, order="F"); Bf[:B.shape[0]] = B
                Cf = np.zeros((M + 2, N), dt, order="F"); Cf[:M] = C0
                al, be = F(1.5), F(-0.5)
                g(ta.encode(), tb.encode(), I(M), I(N), I(K), al, Af.ctypes.data, I(Af.shape[0]), Bf.ctypes.data,
                  I(Bf.shape[0]), be, Cf.ctypes.data, I(Cf.shape[0]))
                a64 = A.astype(np.float64) if ta == "N" else A.astype(np.float64).T
                b64 = B.astype(np.float64) if tb == "n" else B.astype(np.float64).T
                ref = 1.5 * a64 @ b64 - 0.5 * C0
                scale = 1.5 * np.abs(a64) @ np.abs(b64) + 0.5 * np.abs(C0)
                worst = max(worst, rel(Cf[:M], ref, scale))
                assert not Cf[M:].any()
        out[f"{tag}gemm_fortran"] = worst
        # cblas gemv (both orders, negative increments), ger, level 1 against FP64 NumPy
        gv = getattr(L, f"cblas_{tag}gemv")
        gv.argtypes = [I, I, I, I, F, P, I, P, I, F, P, I]
        worst = 0.0
        for order in (RowMajor, ColMajor):
            for tr in (NoTrans, Trans):
                M, N = 301, 257
                A = rng.uniform(-1, 1, (M, N)).astype(dt)
                As = np.ascontiguousarray(A) if order == RowMajor else np.asfortranarray(A)
                lda = N if order == RowMajor else M
                nx, ny = (N, M) if tr == NoTrans else (M, N)
                x = rng.uniform(-1, 1, 2 * nx).astype(dt)
                y0 = rng.uniform(-1, 1, ny).astype(dt)
                y = y0.copy()
                gv(order, tr, M, N, 0.5, As.ctypes.data, lda, x.ctypes.data, -2, 2.0, y.ctypes.data, 1)
                xs = x[::2][::-1].astype(np.float64)   # incx = -2: element 0 is the last in memory
                op = A.astype(np.float64) if tr == NoTrans else A.astype(np.float64).T
                worst = max(worst, rel(y, 0.5 * op @ xs + 2 * y0, 0.5 * np.abs(op) @ np.abs(xs) + 2 * np.abs(y0)))
        out[f"{tag}gemv"] = worst
        gr = getattr(L, f"cblas_{tag}ger")
        gr.argtypes = [I, I, I, F, P, I, P, I, P, I]
        M, N = 123, 77
        A = rng.uniform(-1, 1, (M, N)).astype(dt)
        x = rng.uniform(-1, 1, M).astype(dt)
        y = rng.uniform(-1, 1, N).astype(dt)
        Ac = np.asfortranarray(A.copy())
        gr(ColMajor, M, N, -0.25, x.ctypes.data, 1, y.ctypes.data, 1, Ac.ctypes.data, M)
        ref = A.astype(np.float64) - 0.25 * np.outer(x, y)
        out[f"{tag}ger"] = rel(Ac, ref, np.abs(A) + 0.25 * np.abs(np.outer(x, y)))
        n = 100003
        x = vec_inputs(tag, "l1x", n)
        yv = vec_inputs(tag, "l1y", n)
        ax = getattr(L, f"cblas_{tag}axpy")
        ax.argtypes = [I, F, P, I, P, I]
        yy = yv.copy()
        ax(n, 0.7, x.ctypes.data, 1, yy.ctypes.data, 1)
        out[f"{tag}axpy"] = rel(yy, 0.7 * x.astype(np.float64) + yv, 0.7 * np.abs(x) + np.abs(yv))
        dot = getattr(L, f"cblas_{tag}dot")
        dot.argtypes, dot.restype = [I, P, I, P, I], F
        X, Y = x.astype(np.float64), yv.astype(np.float64)
        out[f"{tag}dot"] = abs(dot(n, x.ctypes.data, 1, yv.ctypes.data, 1) - X @ Y) / (np.abs(X) @ np.abs(Y))
        for nm, refv in (("nrm2", np.linalg.norm(X)), ("asum", np.abs(X).sum())):
            fn = getattr(L, f"cblas_{tag}{nm}")
            fn.argtypes, fn.restype = [I, P, I], F
            out[f"{tag}{nm}"] = abs(fn(n, x.ctypes.data, 1) - refv) / refv
        im = getattr(L, f"cblas_i{tag}amax")
        im.argtypes, im.restype = [I, P, I], ctypes.c_size_t
        out[f"i{tag}amax_exact"] = int(im(n, x.ctypes.data, 1)) == int(np.argmax(np.abs(X)))
    return out


def group_forwarded():
    """A symbol the shim does not own (complex GEMM) reaches the CPU BLAS through the jump table."""
    f = L.cblas_zgemm
    f.argtypes = [I] * 6 + [P, P, I, P, I, P, P, I]
    rng = np.random.default_rng(1)
    A = (rng.standard_normal((5, 7)) + 1j * rng.standard_normal((5, 7))).astype(np.complex128)
    B = (rng.standard_normal((7, 3)) + 1j * rng.standard_normal((7, 3))).astype(np.complex128)
    C = np.zeros((5, 3), np.complex128)
    one, zero = np.array(1 + 0j), np.array(0j)
    f(RowMajor, NoTrans, NoTrans, 5, 3, 7, one.ctypes.data, A.ctypes.data, 7, B.ctypes.data, 3, zero.ctypes.data,
      C.ctypes.data, 3)
    return {"zgemm_forwarded": float(np.abs(C - A @ B).max())}


def group_l2x():
    """The rest of levels 1-2 through the library (GPU) and straight through OpenBLAS (the CPU BLAS the reference's
    CBLAS layer forwards to) on the same data: RowMajor, ColMajor and Fortran calls, random data in the whole band
    array / packed vector (as the reference's lib/test_blas_banded.py). Reports max |diff| / scale per function."""
    ob = ctypes.CDLL(os.environ["GEN9BLAS_BLAS_CPU"])
    rng = np.random.default_rng(9)
    out = {}
    n, K, M, N, KL, KU = 37, 4, 29, 41, 3, 5
    UP, LO, NT, TR, NU, UN = 121, 122, 111, 112, 131, 132
    for tag, F, dt in (("s", ctypes.c_float, np.float32), ("d", ctypes.c_double, np.float64)):
        def ref(p):
            return np.ascontiguousarray(p).copy()

        def call(name, args_fn):
            """args_fn(lib) -> (output arrays); returns max relative difference (GPU vs OpenBLAS)."""
            a = args_fn(L)
            b = args_fn(ob)
            worst = 0.0
            for x, y in zip(a, b):
                scale = max(1.0, float(np.abs(y.astype(np.float64)).max()))
                worst = max(worst, float(np.abs(x.astype(np.float64) - y.astype(np.float64)).max()) / scale)
            out[tag + name] = max(out.get(tag + name, 0.0), worst)

        A = rng.uniform(-1, 1, (n, n)).astype(dt)
        Ad = A.copy()
        Ad[np.diag_indices(n)] = n
        Ab = rng.uniform(-1, 1, (n, K + 1)).astype(dt)
        Abd = Ab.copy()
        Ap = rng.uniform(-1, 1, n * (n + 1) // 2).astype(dt)
        G = rng.uniform(-1, 1, (max(M, N), KL + KU + 1)).astype(dt)
        x0 = rng.uniform(-1, 1, max(M, N) * 2).astype(dt)
        y0 = rng.uniform(-1, 1, max(M, N) * 2).astype(dt)
        P = ctypes.c_void_p
        for o in (101, 102):
            for u in (UP, LO):
                Abd[:, 0 if (u == UP) == (o == 101) else K] = 4 + K   # dominant band diagonal in either storage order
                # packed with a dominant diagonal: rebuild from a dense matrix in this order's packing
                for fn in ("symv",):
                    def f(lib, fn=fn):
                        y = y0[:n].copy()
                        g = getattr(lib, f"cblas_{tag}symv")
                        g.argtypes = [ctypes.c_int] * 3 + [F, P, ctypes.c_int, P, ctypes.c_int, F, P, ctypes.c_int]
                        g(o, u, n, 1.5, A.ctypes.data, n, x0.ctypes.data, 1, -0.5, y.ctypes.data, 1)
                        return (y,)
                    call("symv", f)
                for t in (NT, TR):
                    for d in (NU, UN):
                        for nm, mat, extra in (("trmv", A, None), ("trsv", Ad, None), ("tbmv", Ab, K), ("tbsv", Abd, K),
                                               ("tpmv", Ap, -1), ("tpsv", None, -1)):
                            if nm == "tpsv":   # packed triangle of Ad in this (order, uplo)
                                lower_rm = (u == LO) == (o == 101)
                                mat = np.array([Ad[i, j] for i in range(n) for j in
                                                (range(0, i + 1) if lower_rm else range(i, n))], dt)
                            def f(lib, nm=nm, mat=mat, extra=extra):
                                x = x0[:n].copy()
                                g = getattr(lib, f"cblas_{tag}{nm}")
                                if extra is None:
                                    g.argtypes = [ctypes.c_int] * 5 + [P, ctypes.c_int, P, ctypes.c_int]
                                    g(o, u, t, d, n, mat.ctypes.data, n, x.ctypes.data, 1)
                                elif extra == -1:
                                    g.argtypes = [ctypes.c_int] * 5 + [P, P, ctypes.c_int]
                                    g(o, u, t, d, n, mat.ctypes.data, x.ctypes.data, 1)
                                else:
                                    g.argtypes = [ctypes.c_int] * 6 + [P, ctypes.c_int, P, ctypes.c_int]
                                    g(o, u, t, d, n, extra, mat.ctypes.data, K + 1, x.ctypes.data, 1)
                                return (x,)
                            call(nm, f)

                def f(lib):
                    y = y0[:n].copy()
                    g = getattr(lib, f"cblas_{tag}sbmv")
                    g.argtypes = [ctypes.c_int] * 4 + [F, P, ctypes.c_int, P, ctypes.c_int, F, P, ctypes.c_int]
                    g(o, u, n, K, 0.75, Ab.ctypes.data, K + 1, x0.ctypes.data, 1, 0.25, y.ctypes.data, 1)
                    return (y,)
                call("sbmv", f)

                def f(lib):
                    y = y0[:n].copy()
                    g = getattr(lib, f"cblas_{tag}spmv")
                    g.argtypes = [ctypes.c_int] * 3 + [F, P, P, ctypes.c_int, F, P, ctypes.c_int]
                    g(o, u, n, 0.75, Ap.ctypes.data, x0.ctypes.data, 1, 0.25, y.ctypes.data, 1)
                    return (y,)
                call("spmv", f)
                for nm in ("syr", "syr2", "spr", "spr2"):
                    def f(lib, nm=nm):
                        Aout = (A.copy() if nm.startswith("sy") else Ap.copy())
                        g = getattr(lib, f"cblas_{tag}{nm}")
                        two = nm.endswith("2")
                        packed = nm.startswith("sp")
                        if two and packed:
                            g.argtypes = [ctypes.c_int] * 3 + [F, P, ctypes.c_int, P, ctypes.c_int, P]
                            g(o, u, n, 0.5, x0.ctypes.data, 1, y0.ctypes.data, 1, Aout.ctypes.data)
                        elif packed:
                            g.argtypes = [ctypes.c_int] * 3 + [F, P, ctypes.c_int, P]
                            g(o, u, n, 0.5, x0.ctypes.data, 1, Aout.ctypes.data)
                        elif two:
                            g.argtypes = [ctypes.c_int] * 3 + [F, P, ctypes.c_int, P, ctypes.c_int, P, ctypes.c_int]
                            g(o, u, n, 0.5, x0.ctypes.data, 1, y0.ctypes.data, 1, Aout.ctypes.data, n)
                        else:
                            g.argtypes = [ctypes.c_int] * 3 + [F, P, ctypes.c_int, P, ctypes.c_int]
                            g(o, u, n, 0.5, x0.ctypes.data, 1, Aout.ctypes.data, n)
                        return (Aout,)
                    call(nm, f)
            for t in (NT, TR):
                def f(lib, t=t):
                    rows = M if o == 101 else N     # band rows of the stored array
                    g = getattr(lib, f"cblas_{tag}gbmv")
                    g.argtypes = [ctypes.c_int] * 6 + [F, P, ctypes.c_int, P, ctypes.c_int, F, P, ctypes.c_int]
                    ny = (N if t == TR else M)
                    y = y0[:ny].copy()
                    Gm = np.ascontiguousarray(G[:rows])
                    g(o, t, M, N, KL, KU, 1.25, Gm.ctypes.data, KL + KU + 1, x0.ctypes.data, 1, -0.75, y.ctypes.data, 1)
                    return (y,)
                call("gbmv", f)
        # level 1 (no storage order)
        for nm in ("scal", "copy", "swap", "rot", "rotm"):
            def f(lib, nm=nm):
                x, y = x0[:N].copy(), y0[:N].copy()
                g = getattr(lib, f"cblas_{tag}{nm}")
                if nm == "scal":
                    g.argtypes = [ctypes.c_int, F, P, ctypes.c_int]
                    g(N, 0.7, x.ctypes.data, 1)
                elif nm == "rot":
                    g.argtypes = [ctypes.c_int, P, ctypes.c_int, P, ctypes.c_int, F, F]
                    g(N, x.ctypes.data, 1, y.ctypes.data, 1, 0.6, 0.8)
                elif nm == "rotm":
                    prm = np.array([-1.0, 0.5, -0.25, 0.75, 1.5], dt)
                    g.argtypes = [ctypes.c_int, P, ctypes.c_int, P, ctypes.c_int, P]
                    g(N, x.ctypes.data, 1, y.ctypes.data, 1, prm.ctypes.data)
                else:
                    g.argtypes = [ctypes.c_int, P, ctypes.c_int, P, ctypes.c_int]
                    g(N, x.ctypes.data, 1, y.ctypes.data, 1)
                return (x, y)
            call(nm, f)
    return out


def group_config():
    """BASELINE config sizes through the CBLAS entry points: cblas_sgemm configs[0] (n = 1024 row-major NN, alpha 1,
    beta 0) and cblas_dgemm configs[3] (n = 3000 column-major, all four transposes, alpha 1.5, beta 0.5, C prefilled),
    each against FP64 NumPy and against the reference layer's own rows (tests/golden/ref_config_rows.npz)."""
    import make_golden as mg
    fix = np.load(os.path.join(HERE, "golden", "ref_config_rows.npz"))
    out = {}
    f = L.cblas_sgemm
    f.argtypes = [I, I, I, I, I, I, ctypes.c_float, P, I, P, I, ctypes.c_float, P, I]
    A, B = mg.c0_inputs()
    n = mg.C0_N
    C = np.full((n, n), np.nan, np.float32)
    f(RowMajor, NoTrans, NoTrans, n, n, n, 1.0, A.ctypes.data, n, B.ctypes.data, n, 0.0, C.ctypes.data, n)
    a64, b64 = A.astype(np.float64), B.astype(np.float64)
    scale = np.abs(a64) @ np.abs(b64)
    out["sgemm_c0_vs_fp64"] = rel(C, a64 @ b64, scale)
    rows = mg.c0_rows()
    out["sgemm_c0_vs_ref_cblas"] = rel(C[rows], fix["sgemm_c0_rows"], scale[rows])
    f = L.cblas_dgemm
    f.argtypes = [I, I, I, I, I, I, ctypes.c_double, P, I, P, I, ctypes.c_double, P, I]
    n = mg.C3_N
    rows = mg.c3_rows()
    w64 = w_ref = 0.0
    for ta in (NoTrans, Trans):
        for tb in (NoTrans, Trans):
            A, B, C0 = mg.c3_inputs(ta, tb)
            As, Bs, Cs = np.asfortranarray(A), np.asfortranarray(B), np.asfortranarray(C0.copy())
            f(ColMajor, ta, tb, n, n, n, mg.C3_ALPHA, As.ctypes.data, A.shape[0], Bs.ctypes.data, B.shape[0],
              mg.C3_BETA, Cs.ctypes.data, n)
            opA = A if ta == NoTrans else A.T
            opB = B if tb == NoTrans else B.T
            ref = mg.C3_ALPHA * opA[rows] @ opB + mg.C3_BETA * C0[rows]
            scale = mg.C3_ALPHA * np.abs(opA[rows]) @ np.abs(opB) + mg.C3_BETA * np.abs(C0[rows])
            w64 = max(w64, rel(Cs[rows], ref, scale))
            w_ref = max(w_ref, rel(Cs[rows], fix[f"dgemm_c3_t{ta}{tb}_rows"], scale))
    out["dgemm_c3_vs_fp64"], out["dgemm_c3_vs_ref_cblas"] = w64, w_ref
    return out


def group_sharded():
    """Large GEMMs through the CBLAS entry points, for a run with GEN9BLAS_DEVICES set (column blocks per GPU):
    cblas_sgemm n = 8192 row-major and cblas_dgemm n = 4096 column-major with alpha 1.5, beta 0.5, against FP64 on
    sampled rows."""
    rng = np.random.default_rng(12)
    out = {}
    f = L.cblas_sgemm
    f.argtypes = [I, I, I, I, I, I, ctypes.c_float, P, I, P, I, ctypes.c_float, P, I]
    n = 8192
    A = rng.uniform(-1, 1, (n, n)).astype(np.float32)
    B = rng.uniform(-1, 1, (n, n)).astype(np.float32)
    C = np.zeros((n, n), np.float32)
    f(RowMajor, NoTrans, NoTrans, n, n, n, 1.0, A.ctypes.data, n, B.ctypes.data, n, 0.0, C.ctypes.data, n)
    rows = rng.choice(n, 32, replace=False)
    a64, b64 = A[rows].astype(np.float64), B.astype(np.float64)
    out["sgemm_8192"] = rel(C[rows], a64 @ b64, np.abs(a64) @ np.abs(b64))
    f = L.cblas_dgemm
    f.argtypes = [I, I, I, I, I, I, ctypes.c_double, P, I, P, I, ctypes.c_double, P, I]
    n = 4096
    A, B, C0 = (np.asfortranarray(rng.uniform(-1, 1, (n, n))) for _ in range(3))
    Cf = C0.copy(order="F")
    f(ColMajor, NoTrans, Trans, n, n, n, 1.5, A.ctypes.data, n, B.ctypes.data, n, 0.5, Cf.ctypes.data, n)
    rows = rng.choice(n, 16, replace=False)
    ref = 1.5 * A[rows] @ B.T + 0.5 * C0[rows]
    sc = 1.5 * np.abs(A[rows]) @ np.abs(B.T) + 0.5 * np.abs(C0[rows])
    out["dgemm_4096_col"] = rel(Cf[rows], ref, sc)
    return out


if __name__ == "__main__":
    groups = {"cblas_gemm": group_cblas_gemm, "fortran_l12": group_fortran_and_l12, "forwarded": group_forwarded,
              "level3": group_level3, "l2x": group_l2x, "config": group_config,
              "sharded": group_sharded}
    print(json.dumps(groups[sys.argv[1]]()))
