"""Generates the committed parity fixtures under tests/golden/ (run here, where the reference checkout exists).

    python tests/golden/make_golden.py [REF=/root/reference]

1. ref_golden_hashes.json: the reference's own golden digests of its BLAS layer (tools/golden/expected/uhd620-whl/
   lib.txt of kprzybys/gen9-gpu-blas) for the calls whose result bytes do not depend on the hardware's summation
   order (element-wise FMA results and iamax indices), with the call recipe of tools/golden/blas_golden.py:16-66.
2. ref_cblas_outputs.npz: outputs of the reference's CBLAS layer itself (oracle/_ref/libgen9blas_blas_ref.so, built
   from lib/src/cblas.c by oracle/Makefile, running on OpenBLAS) for small seeded calls: row- and column-major SGEMM /
   DGEMM with all transposes, alpha/beta, non-tile-multiple sizes, gemv N/T, ger, axpy, dot, nrm2, asum, iamax.
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
REF = sys.argv[1] if len(sys.argv) > 1 else "/root/reference"
OPENBLAS_DIR = "/opt/prime-rl/.venv/lib/python3.12/site-packages/opencv_python_headless.libs"
OPENBLAS = os.path.join(OPENBLAS_DIR, "libopenblasp-r0-59ffcd50.3.15.so")

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


def vec_inputs(tag, what, *shape):
    dt = np.float32 if tag == "s" else np.float64
    return np.random.default_rng(hash_seed(tag, what, shape)).uniform(-1, 1, shape).astype(dt)


def ref_outputs():
    subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "ref", f"REF={REF}"], check=True, capture_output=True)
    os.environ["GEN9BLAS_BLAS"] = "cpu"
    os.environ["GEN9BLAS_BLAS_CPU"] = OPENBLAS
    os.environ["OPENBLAS_NUM_THREADS"] = "1"
    # OpenBLAS's own dependencies, by full path and in dependency order (the wheel directory is not on the loader path)
    for dep in ("libquadmath-2284e583.so.0.0.0", "libgfortran-83c28eba.so.5.0.0"):
        ctypes.CDLL(os.path.join(OPENBLAS_DIR, dep), mode=ctypes.RTLD_GLOBAL)
    L = ctypes.CDLL(os.path.join(ROOT, "oracle", "_ref", "libgen9blas_blas_ref.so"))
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
    return res


if __name__ == "__main__":
    h = golden_hashes()
    with open(os.path.join(HERE, "ref_golden_hashes.json"), "w") as f:
        json.dump(h, f, indent=1, sort_keys=True)
    np.savez_compressed(os.path.join(HERE, "ref_cblas_outputs.npz"), **ref_outputs())
    print("wrote", len(h), "golden hashes and ref_cblas_outputs.npz")
