"""Generates the committed parity fixtures under tests/golden/ (run here, where the reference checkout exists).

    python tests/golden/make_golden.py [--reference DIR] [--only hashes,cblas,config]

The reference checkout is DIR, else GEN9BLAS_REFERENCE, else a checkout named "reference" beside this repository;
the script stops with a message when none exists. OpenBLAS: GEN9BLAS_OPENBLAS, else a wheel's bundled copy
(oracle/cpu_blas.py).

1. ref_golden_hashes.json: the reference's own golden digests of its BLAS layer (tools/golden/expected/uhd620-whl/
   lib.txt of kprzybys/gen9-gpu-blas) for the calls whose result bytes do not depend on the hardware's summation
   order (element-wise FMA results and iamax indices), with the call recipe of tools/golden/blas_golden.py:16-66.
2. ref_cblas_outputs.npz: outputs of the reference's CBLAS layer itself (oracle/_ref/libgen9blas_blas_ref.so, built
   from lib/src/cblas.c by oracle/Makefile, running on OpenBLAS) for small seeded calls: row- and column-major SGEMM /
   DGEMM with all transposes, alpha/beta, non-tile-multiple sizes, gemv N/T, ger, axpy, dot, nrm2, asum, iamax, and
   the level-3 set on GEMM (row- and column-major SYMM, SYRK, SYR2K, TRMM, TRSM over every side / triangle /
   transpose / diagonal option; inputs from l3_inputs).
3. ref_config_rows.npz: sampled rows of the reference layer's output at BASELINE config sizes: SGEMM n = 1024
   row-major NN, alpha = 1, beta = 0, A and B uniform[-1,1] from seeds 1 and 2 (the speed section of
   lib/test_basic.py); DGEMM n = 3000 column-major, every transA/transB pair, alpha = 1.5, beta = 0.5, C prefilled
   uniform[-1,1] (inputs from gemm_inputs). The tests regenerate the inputs from the same seeds.
The GPU box never reads the reference: the tests only read these files.
"""
import ctypes
import json
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import cpu_blas  # noqa: E402

REF = None   # reference checkout, set by main()

# Digests whose inputs and arithmetic are fully defined by element-wise rules (see tests/test_oracle_golden.py).
PINNED = ["saxpy", "daxpy", "sger", "dger", "siamax", "diamax", "snrm2", "sasum"]


def golden_hashes():
    path = os.path.join(REF, "tools", "golden", "expected", "uhd620-whl", "lib.txt")
    out = {}
    for line in open(path):
        parts = line.split()
        if len(parts) == 2 and parts[0] in PINNED:
            out[parts[0]] = parts[1]
    missing = set(PINNED) - set(out)
    if missing:
        sys.exit(f"missing golden entries: {sorted(missing)}")
    return out


GEMM_CASES = [(17, 33, 15, 1.0, 0.0), (40, 24, 48, 0.5, 1.0), (31, 29, 70, 1.5, 0.5)]
RowMajor, ColMajor, NoTrans, Trans = 101, 102, 111, 112


def gemm_inputs(tag, order, ta, tb, M, N, K):
    """Seeded inputs of one CBLAS GEMM case (logical op-shapes before the storage order is applied)."""
    dt = np.float32 if tag == "s" else np.float64
    seed = hash_seed(tag, order, ta, tb, M, N, K)
    rng = np.random.default_rng(seed)
    ar, ac = (M, K) if ta == NoTrans else (K, M)
    br, bc = (K, N) if tb == NoTrans else (N, K)
    A = rng.uniform(-1, 1, (ar, ac)).astype(dt)
    B = rng.uniform(-1, 1, (br, bc)).astype(dt)
    C0 = rng.uniform(-1, 1, (M, N)).astype(dt)
    return A, B, C0


def hash_seed(*parts):
    s = 0
    for ch in repr(parts):
        s = (s * 131 + ord(ch)) % (1 << 61)
    return s


Upper, Lower, NonUnit, Unit, Left, Right = 121, 122, 131, 132, 141, 142
L3_SYMM = (23, 17, 1.5, -0.5)          # M, N, alpha, beta
L3_SYRK = (19, 27, 0.7, 0.3)           # N, K, alpha, beta
L3_TRXM = (21, 13, 1.25)               # M, N, alpha


def l3_inputs(tag, op, *key):
    """Seeded logical inputs of one level-3 case: SYMM (A n×n, B, C0), SYRK/SYR2K (A, B as op-shapes N×K before the
    trans flag, C0), TRMM/TRSM (A n×n with a dominant diagonal so that the triangular solves are well conditioned,
    B)."""
    dt = np.float32 if tag == "s" else np.float64
    rng = np.random.default_rng(hash_seed(tag, op, key))
    if op == "symm":
        side = key[1]
        M, N = L3_SYMM[:2]
        n = M if side == Left else N
        return (rng.uniform(-1, 1, (n, n)).astype(dt), rng.uniform(-1, 1, (M, N)).astype(dt),
                rng.uniform(-1, 1, (M, N)).astype(dt))
    if op in ("syrk", "syr2k"):
        trans = key[2]
        N, K = L3_SYRK[:2]
        shape = (K, N) if trans == Trans else (N, K)
        return (rng.uniform(-1, 1, shape).astype(dt), rng.uniform(-1, 1, shape).astype(dt),
                rng.uniform(-1, 1, (N, N)).astype(dt))
    side = key[1]
    M, N = L3_TRXM[:2]
    n = M if side == Left else N
    A = rng.uniform(-1, 1, (n, n))
    A[np.diag_indices(n)] = n + rng.uniform(0, 1, n)
    return A.astype(dt), rng.uniform(-1, 1, (M, N)).astype(dt)


def store(X, order):
    """(storage array, leading dimension) of a logical matrix in the given CBLAS order."""
    if order == RowMajor:
        return np.ascontiguousarray(X), X.shape[1]
    return np.asfortranarray(X), X.shape[0]


def l3_cases():
    """Every (op, order, options) combination of the level-3 fixtures."""
    for order in (RowMajor, ColMajor):
        for side in (Left, Right):
            for uplo in (Upper, Lower):
                yield ("symm", order, side, uplo)
        for uplo in (Upper, Lower):
            for trans in (NoTrans, Trans):
                yield ("syrk", order, uplo, trans)
                yield ("syr2k", order, uplo, trans)
        for side in (Left, Right):
            for uplo in (Upper, Lower):
                for trans in (NoTrans, Trans):
                    for diag in (NonUnit, Unit):
                        yield ("trmm", order, side, uplo, trans, diag)
                        yield ("trsm", order, side, uplo, trans, diag)


def l3_key(tag, case):
    return tag + case[0] + "_" + "_".join(str(v) for v in case[1:])


def run_l3(L, tag, case):
    """Runs one level-3 case through CBLAS library L; returns the logical (row-major) result matrix."""
    F = ctypes.c_float if tag == "s" else ctypes.c_double
    I, P = ctypes.c_int, ctypes.c_void_p
    op, order = case[0], case[1]
    if op == "symm":
        side, uplo = case[2], case[3]
        M, N, al, be = L3_SYMM
        A, B, C0 = l3_inputs(tag, op, *case[1:])
        (As, lda), (Bs, ldb), (Cs, ldc) = store(A, order), store(B, order), store(C0.copy(), order)
        f = getattr(L, f"cblas_{tag}symm")
        f.argtypes = [I, I, I, I, I, F, P, I, P, I, F, P, I]
        f(order, side, uplo, M, N, al, As.ctypes.data, lda, Bs.ctypes.data, ldb, be, Cs.ctypes.data, ldc)
        return np.ascontiguousarray(Cs)
    if op in ("syrk", "syr2k"):
        uplo, trans = case[2], case[3]
        N, K, al, be = L3_SYRK
        A, B, C0 = l3_inputs(tag, op, *case[1:])
        (As, lda), (Bs, ldb), (Cs, ldc) = store(A, order), store(B, order), store(C0.copy(), order)
        if op == "syrk":
            f = getattr(L, f"cblas_{tag}syrk")
            f.argtypes = [I, I, I, I, I, F, P, I, F, P, I]
            f(order, uplo, trans, N, K, al, As.ctypes.data, lda, be, Cs.ctypes.data, ldc)
        else:
            f = getattr(L, f"cblas_{tag}syr2k")
            f.argtypes = [I, I, I, I, I, F, P, I, P, I, F, P, I]
            f(order, uplo, trans, N, K, al, As.ctypes.data, lda, Bs.ctypes.data, ldb, be, Cs.ctypes.data, ldc)
        return np.ascontiguousarray(Cs)
    side, uplo, trans, diag = case[2:]
    M, N, al = L3_TRXM
    A, B = l3_inputs(tag, op, *case[1:])
    (As, lda), (Bs, ldb) = store(A, order), store(B.copy(), order)
    f = getattr(L, f"cblas_{tag}{op}")
    f.argtypes = [I, I, I, I, I, I, I, F, P, I, P, I]
    f(order, side, uplo, trans, diag, M, N, al, As.ctypes.data, lda, Bs.ctypes.data, ldb)
    return np.ascontiguousarray(Bs)


def vec_inputs(tag, what, *shape):
    dt = np.float32 if tag == "s" else np.float64
    return np.random.default_rng(hash_seed(tag, what, shape)).uniform(-1, 1, shape).astype(dt)


def ref_layer():
    """The reference's CBLAS layer built from its sources (oracle/Makefile), in CPU mode over OpenBLAS."""
    subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "ref", f"REF={REF}"], check=True, capture_output=True)
    openblas = cpu_blas.preload_openblas_deps()   # its dependencies, which the wheel folder keeps off the loader path
    if openblas is None:
        sys.exit("no OpenBLAS found: set GEN9BLAS_OPENBLAS to a libopenblas shared object with cblas_* names")
    os.environ["GEN9BLAS_BLAS"] = "cpu"
    os.environ["GEN9BLAS_BLAS_CPU"] = openblas
    os.environ["OPENBLAS_NUM_THREADS"] = "1"
    return ctypes.CDLL(os.path.join(ROOT, "oracle", "_ref", "libgen9blas_blas_ref.so"))


# BASELINE config sizes of ref_config_rows.npz
C0_N = 1024
C3_N, C3_ALPHA, C3_BETA = 3000, 1.5, 0.5


def c0_inputs():
    """SGEMM n = 1024 inputs, A and B uniform[-1,1] FP32 from seeds 1 and 2 (lib/test_basic.py:86-87)."""
    n = C0_N
    A = np.random.default_rng(1).uniform(-1, 1, (n, n)).astype(np.float32)
    B = np.random.default_rng(2).uniform(-1, 1, (n, n)).astype(np.float32)
    return A, B


def c0_rows():
    return np.unique(np.concatenate([[0, C0_N - 1], np.random.default_rng(3).choice(C0_N, 32, replace=False)]))


def c3_inputs(ta, tb):
    """DGEMM n = 3000 column-major inputs (logical stored matrices, gemm_inputs' seeds)."""
    return gemm_inputs("d", ColMajor, ta, tb, C3_N, C3_N, C3_N)


def c3_rows():
    return np.unique(np.concatenate([[0, C3_N - 1], np.random.default_rng(4).choice(C3_N, 4, replace=False)]))


def config_outputs(L):
    I, P = ctypes.c_int, ctypes.c_void_p
    res = {}
    f = L.cblas_sgemm
    f.argtypes = [I, I, I, I, I, I, ctypes.c_float, P, I, P, I, ctypes.c_float, P, I]
    A, B = c0_inputs()
    n = C0_N
    C = np.zeros((n, n), np.float32)
    f(RowMajor, NoTrans, NoTrans, n, n, n, 1.0, A.ctypes.data, n, B.ctypes.data, n, 0.0, C.ctypes.data, n)
    res["sgemm_c0_rows"] = C[c0_rows()]
    f = L.cblas_dgemm
    f.argtypes = [I, I, I, I, I, I, ctypes.c_double, P, I, P, I, ctypes.c_double, P, I]
    n = C3_N
    for ta in (NoTrans, Trans):
        for tb in (NoTrans, Trans):
            A, B, C0 = c3_inputs(ta, tb)
            As, Bs, Cs = np.asfortranarray(A), np.asfortranarray(B), np.asfortranarray(C0.copy())
            f(ColMajor, ta, tb, n, n, n, C3_ALPHA, As.ctypes.data, A.shape[0], Bs.ctypes.data, B.shape[0], C3_BETA,
              Cs.ctypes.data, n)
            res[f"dgemm_c3_t{ta}{tb}_rows"] = np.ascontiguousarray(Cs[c3_rows()])
    return res


def ref_outputs():
    L = ref_layer()
    I, P = ctypes.c_int, ctypes.c_void_p
    res = {}
    for tag, F in (("s", ctypes.c_float), ("d", ctypes.c_double)):
        gemm = getattr(L, f"cblas_{tag}gemm")
        gemm.argtypes = [I, I, I, I, I, I, F, P, I, P, I, F, P, I]
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
                        gemm(order, ta, tb, M, N, K, al, As.ctypes.data, lda, Bs.ctypes.data, ldb, be, Cs.ctypes.data, ldc)
                        res[f"{tag}gemm_o{order}_t{ta}{tb}_{M}x{N}x{K}"] = np.ascontiguousarray(Cs)
        gemv = getattr(L, f"cblas_{tag}gemv")
        gemv.argtypes = [I, I, I, I, F, P, I, P, I, F, P, I]
        M, N = 37, 29
        for tr in (NoTrans, Trans):
            A = vec_inputs(tag, "gemvA", M, N)
            x = vec_inputs(tag, "gemvx", N if tr == NoTrans else M)
            y = vec_inputs(tag, "gemvy", M if tr == NoTrans else N)
            gemv(RowMajor, tr, M, N, 0.75, A.ctypes.data, N, x.ctypes.data, 1, -1.25, y.ctypes.data, 1)
            res[f"{tag}gemv_t{tr}"] = y
        ger = getattr(L, f"cblas_{tag}ger")
        ger.argtypes = [I, I, I, F, P, I, P, I, P, I]
        A = vec_inputs(tag, "gerA", 23, 31)
        x = vec_inputs(tag, "gerx", 23)
        y = vec_inputs(tag, "gery", 31)
        ger(RowMajor, 23, 31, -0.5, x.ctypes.data, 1, y.ctypes.data, 1, A.ctypes.data, 31)
        res[f"{tag}ger"] = A
        n = 1000
        x = vec_inputs(tag, "l1x", n)
        y = vec_inputs(tag, "l1y", n)
        axpy = getattr(L, f"cblas_{tag}axpy")
        axpy.argtypes = [I, F, P, I, P, I]
        yy = y.copy()
        axpy(n, 0.7, x.ctypes.data, 1, yy.ctypes.data, 1)
        res[f"{tag}axpy"] = yy
        for nm in ("dot", "nrm2", "asum"):
            f = getattr(L, f"cblas_{tag}{nm}")
            f.restype = F
            if nm == "dot":
                f.argtypes = [I, P, I, P, I]
                v = f(n, x.ctypes.data, 1, y.ctypes.data, 1)
            else:
                f.argtypes = [I, P, I]
                v = f(n, x.ctypes.data, 1)
            res[f"{tag}{nm}"] = np.array(v, np.float32 if tag == "s" else np.float64)
        iam = getattr(L, f"cblas_i{tag}amax")
        iam.argtypes = [I, P, I]
        iam.restype = ctypes.c_size_t
        res[f"i{tag}amax"] = np.array(iam(n, x.ctypes.data, 1), np.int64)
        for case in l3_cases():
            res[l3_key(tag, case)] = run_l3(L, tag, case)
    return res


def main():
    import argparse
    global REF
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None, help="reference checkout (default: GEN9BLAS_REFERENCE, else a "
                                                        "checkout named reference beside this repository)")
    ap.add_argument("--only", default="hashes,cblas,config")
    a = ap.parse_args()
    REF = a.reference or cpu_blas.reference_dir()
    if not REF or not os.path.exists(os.path.join(REF, "lib", "src", "cblas.c")):
        sys.exit("reference checkout not found: pass --reference DIR or set GEN9BLAS_REFERENCE")
    only = set(a.only.split(","))
    if "hashes" in only:
        h = golden_hashes()
        with open(os.path.join(HERE, "ref_golden_hashes.json"), "w") as f:
            json.dump(h, f, indent=1, sort_keys=True)
        print("wrote", len(h), "golden hashes")
    if "cblas" in only:
        np.savez_compressed(os.path.join(HERE, "ref_cblas_outputs.npz"), **ref_outputs())
        print("wrote ref_cblas_outputs.npz")
    if "config" in only:
        np.savez_compressed(os.path.join(HERE, "ref_config_rows.npz"), **config_outputs(ref_layer()))
        print("wrote ref_config_rows.npz")


if __name__ == "__main__":
    main()
