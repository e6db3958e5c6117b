"""gen9blas -- NumPy module over libgen9blas.so, the B200 (sm_100a) build of gen9blas.

    import numpy as np, gen9blas
    C = gen9blas.hgemm(A, B)                      # float16, FP16 accumulation; accurate=True: FP32 accumulation
    C = gen9blas.sgemm(A.T, B, alpha=2.0)         # float32; transposed views and row slices without a copy
    C = gen9blas.gemm_batched(A3, B3)             # (count, M, K) · (count, K, N) -> (count, M, N)
    X = gen9blas.empty((n, n), np.float16)        # managed memory: used in place by the GPU, writable by the CPU
    gen9blas.axpy(0.5, x, y); d = gen9blas.dot(x, y); i = gen9blas.iamax(x)
    y = gen9blas.gemv(A, x); gen9blas.ger(1.0, x, y, A)
    C = gen9blas.symm(S, B); C = gen9blas.syrk(A, "L"); X = gen9blas.trsm(T, B, "L", "U")   # level 3 on GEMM

Same function names, argument meaning and error behaviour as the reference module lib/gen9blas.py of
kprzybys/gen9-gpu-blas (gemm/hgemm/sgemm/gemm_batched 168-204, symm..trsm 207-272, empty/free_pool 60-115,
axpy..ger 335-419): the type
follows the dtype, views map to leading dimensions and transpose flags (lib/gen9blas.py:316-328), errors raise
RuntimeError with gen9blas_error(). Plain NumPy arrays are staged through device buffers by the library; arrays from
gen9blas.empty() live in CUDA managed memory and are used in place.
"""
import ctypes
import os
import weakref

import numpy as np

_HERE = os.path.dirname(os.path.realpath(__file__))


def _find(name):
    p = os.path.join(_HERE, name)
    return p if os.path.exists(p) else name


_lib = ctypes.CDLL(os.environ.get("GEN9BLAS_LIB") or _find("libgen9blas.so"))
_i, _f, _p, _l, _d = ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_int64, ctypes.c_double
_lib.gen9blas_init.argtypes = []
_lib.gen9blas_gemm.argtypes = [_i, _i, _i, _i, _i, _i, _d, _p, _i, _p, _i, _d, _p, _i]
_lib.gen9blas_gemm_batched.argtypes = [_i, _i, _i, _i, _i, _i, _d, _p, _i, _l, _p, _i, _l, _d, _p, _i, _l, _i]
_lib.gen9blas_last_time_ms.restype = ctypes.c_double
_lib.gen9blas_alloc.argtypes = [ctypes.c_size_t]
_lib.gen9blas_alloc.restype = ctypes.c_void_p
_lib.gen9blas_free.argtypes = [ctypes.c_void_p]
_lib.gen9blas_error.restype = ctypes.c_char_p
_lib.gen9blas_axpy.argtypes = [_i, _i, _d, _p, _i, _p, _i]
_lib.gen9blas_dot.argtypes = [_i, _i, _p, _i, _p, _i, ctypes.POINTER(_d)]
_lib.gen9blas_asum.argtypes = [_i, _i, _p, _i, ctypes.POINTER(_d)]
_lib.gen9blas_nrm2.argtypes = [_i, _i, _p, _i, ctypes.POINTER(_d)]
_lib.gen9blas_iamax.argtypes = [_i, _i, _p, _i, ctypes.POINTER(_l)]
_lib.gen9blas_gemv.argtypes = [_i, _i, _i, _i, _d, _p, _i, _p, _i, _d, _p, _i]
_lib.gen9blas_ger.argtypes = [_i, _i, _i, _d, _p, _i, _p, _i, _p, _i]
_lib.gen9blas_symm.argtypes = [_i, _i, _i, _i, _i, _d, _p, _i, _p, _i, _d, _p, _i]
_lib.gen9blas_syrk.argtypes = [_i, _i, _i, _i, _i, _d, _p, _i, _d, _p, _i]
_lib.gen9blas_syr2k.argtypes = [_i, _i, _i, _i, _i, _d, _p, _i, _p, _i, _d, _p, _i]
_lib.gen9blas_trmm.argtypes = [_i, _i, _i, _i, _i, _i, _i, _d, _p, _i, _p, _i]
_lib.gen9blas_trsm.argtypes = [_i, _i, _i, _i, _i, _i, _i, _d, _p, _i, _p, _i]
_lib.gen9blas_set_device.argtypes = [_i]
_lib.gen9blas_set_stream.argtypes = [_p]
_lib.gen9blas_set_nowait.argtypes = [_i]
_lib.gen9blas_kernel_launches.restype = ctypes.c_longlong
GEN9BLAS_H, GEN9BLAS_S, GEN9BLAS_HS, GEN9BLAS_D = 0, 1, 2, 3
FEAT_FP16, FEAT_FP32, FEAT_FP64 = 0, 1, 2
_lib.gen9blas_version.restype = ctypes.c_int
if _lib.gen9blas_version() // 100 != 2:   # 0.2.x: the API this module is written for
    raise ImportError(f"gen9blas.py expects libgen9blas 0.2.x, loaded {_lib.gen9blas_version()}")
_ready = False


def _init():
    global _ready
    if not _ready:
        if _lib.gen9blas_init() != 0:
            raise RuntimeError(_lib.gen9blas_error().decode())
        _ready = True


def _check(w):
    if w != 0:
        raise RuntimeError(_lib.gen9blas_error().decode())


# Managed-memory pool: released blocks wait for the next gen9blas.empty of the same rounded size.
_pool = {}
_pool_bytes = 0
POOL_MAX = 1 << 30


def _block_size(n):
    return max(4096, (n + 65535) // 65536 * 65536 if n > 65536 else (n + 4095) // 4096 * 4096)


def _release(p, n):
    global _pool_bytes
    if _pool_bytes + n <= POOL_MAX:
        _pool.setdefault(n, []).append(p)
        _pool_bytes += n
    else:
        _lib.gen9blas_free(p)


def free_pool():
    """Returns the blocks waiting in the pool (arrays still in use stay allocated)."""
    global _pool_bytes
    for blocks in _pool.values():
        for p in blocks:
            _lib.gen9blas_free(p)
    _pool.clear()
    _pool_bytes = 0


def empty(shape, dtype=np.float16):
    """C-contiguous array in CUDA managed memory: the GPU uses it in place (views and slices too), the CPU reads and
    writes it directly. When every view is gone the block returns to the pool (up to POOL_MAX bytes)."""
    global _pool_bytes
    _init()
    dtype = np.dtype(dtype)
    n = int(np.prod(shape)) * dtype.itemsize
    nb = _block_size(n)
    if _pool.get(nb):
        p = _pool[nb].pop()
        _pool_bytes -= nb
    else:
        p = _lib.gen9blas_alloc(nb)
        if not p:
            raise MemoryError(_lib.gen9blas_error().decode())
    raw = (ctypes.c_char * nb).from_address(p)
    f = weakref.finalize(raw, _release, p, nb)
    f.atexit = False
    return np.frombuffer(raw, dtype=np.uint8, count=n).view(dtype).reshape(shape)


def available(dt, accurate=False):
    """Whether the type can be used on this GPU."""
    _init()
    k = _kind(dt, accurate)
    return bool(_lib.gen9blas_has(FEAT_FP32 if k == GEN9BLAS_S else FEAT_FP64 if k == GEN9BLAS_D else FEAT_FP16))


def _kind(dt, accurate):
    if np.dtype(dt) == np.float32:
        return GEN9BLAS_S
    if np.dtype(dt) == np.float64:
        return GEN9BLAS_D
    if np.dtype(dt) == np.float16:
        return GEN9BLAS_HS if accurate else GEN9BLAS_H
    raise TypeError("supported types: float16, float32, float64")


def _mat(A, dt, write=False):
    """(array, pointer, rows, columns, ld, trans) for a row-major matrix with a leading dimension; a transposed
    view is used without a copy (trans = 1)."""
    if A.ndim != 2:
        raise ValueError("expected a 2-D matrix")
    e = A.itemsize
    if A.dtype == dt and A.strides[1] == e and A.strides[0] >= A.shape[1] * e and A.strides[0] % e == 0:
        return A, A.ctypes.data, A.shape[0], A.shape[1], A.strides[0] // e, 0
    if not write and A.dtype == dt and A.strides[0] == e and A.strides[1] >= A.shape[0] * e and A.strides[1] % e == 0:
        return A, A.ctypes.data, A.shape[1], A.shape[0], A.strides[1] // e, 1
    if write:
        raise TypeError(f"the result must be a {np.dtype(dt).name} matrix with contiguous rows")
    A = np.ascontiguousarray(A, dtype=dt)
    return A, A.ctypes.data, A.shape[0], A.shape[1], A.shape[1], 0


def _m3(X, dt, write=False):
    X, p, _, _, ld, tr = _mat(X, dt, write)
    return X, p, ld, tr


def _c(X, dt):
    return np.ascontiguousarray(X, dtype=dt)


def _output(C, shape, dt):
    """(C, given, ldc): a new C from gen9blas.empty or the supplied C with contiguous rows (any row stride)."""
    if C is None:
        return empty(shape, dt), False, shape[-1]
    if C.shape != tuple(shape) or C.dtype != dt or C.strides[-1] != C.itemsize:
        raise ValueError(f"C must have shape {tuple(shape)}, type {np.dtype(dt).name} and contiguous rows")
    if C.ndim == 2:
        return C, True, _mat(C, dt, True)[4]
    if not C.flags.c_contiguous:
        raise ValueError("C (batch) must be C-contiguous")
    return C, True, shape[-1]


def gemm(A, B, alpha=1.0, beta=0.0, C=None, accurate=False):
    """C = alpha·A·B + beta·C (type from A: float16, float32 or float64)."""
    _init()
    dt = A.dtype if A.dtype in (np.float16, np.float32, np.float64) else np.float32
    (M, K), (K2, N) = A.shape, B.shape
    if K != K2:
        raise ValueError(f"incompatible dimensions: {A.shape} · {B.shape}")
    a, pa, lda, ta = _m3(A, dt)
    b, pb, ldb, tb = _m3(B, dt)
    C, given, ldc = _output(C, (M, N), dt)
    _check(_lib.gen9blas_gemm(_kind(dt, accurate), ta, tb, M, N, K, alpha, pa, lda, pb, ldb,
                              beta if given else 0.0, C.ctypes.data, ldc))
    return C


def hgemm(A, B, alpha=1.0, beta=0.0, C=None, accurate=False):
    return gemm(A if A.dtype == np.float16 else A.astype(np.float16),
                B if B.dtype == np.float16 else B.astype(np.float16), alpha, beta, C, accurate)


def sgemm(A, B, alpha=1.0, beta=0.0, C=None):
    return gemm(A if A.dtype == np.float32 else A.astype(np.float32),
                B if B.dtype == np.float32 else B.astype(np.float32), alpha, beta, C)


def dgemm(A, B, alpha=1.0, beta=0.0, C=None):
    return gemm(A if A.dtype == np.float64 else A.astype(np.float64),
                B if B.dtype == np.float64 else B.astype(np.float64), alpha, beta, C)


def gemm_batched(A, B, alpha=1.0, beta=0.0, C=None, accurate=False):
    """Batch: A (count, M, K), B (count, K, N) -> C (count, M, N), one kernel launch."""
    _init()
    dt = A.dtype if A.dtype in (np.float16, np.float32, np.float64) else np.float32
    a, b = _c(A, dt), _c(B, dt)
    (cnt, M, K), (cnt2, K2, N) = a.shape, b.shape
    if K != K2 or cnt != cnt2:
        raise ValueError(f"incompatible dimensions: {a.shape} · {b.shape}")
    C, given, _ = _output(C, (cnt, M, N), dt)
    _check(_lib.gen9blas_gemm_batched(_kind(dt, accurate), 0, 0, M, N, K, alpha, a.ctypes.data, K, M * K,
                                      b.ctypes.data, N, K * N, beta if given else 0.0, C.ctypes.data, N, M * N, cnt))
    return C


# ---------------- level 3 on GEMM (lib/gen9blas.py:207-272 of the reference) ----------------
_SIDE = {"L": 0, "R": 1}
_TRI = {"L": 0, "U": 1}


def _square(A, dt, uplo):
    """(array, pointer, n, ld, trans, uplo) of a square operand; a transposed view is the same memory read with the
    triangle swapped (and, for triangular operands, transA flipped)."""
    if A.ndim != 2 or A.shape[0] != A.shape[1]:
        raise ValueError("expected a square matrix")
    a, pa, lda, ta = _m3(A, dt)
    if ta:
        uplo = "U" if uplo == "L" else "L"
    return a, pa, A.shape[0], lda, ta, uplo


def symm(A, B, side="L", uplo="L", alpha=1.0, beta=0.0, C=None, accurate=False):
    """C = alpha·A·B + beta·C (side="L") or alpha·B·A + beta·C (side="R"); A symmetric, its uplo triangle is read."""
    _init()
    dt = B.dtype if B.dtype in (np.float16, np.float32, np.float64) else np.float32
    a, pa, n, lda, _, uplo = _square(A, dt, uplo)
    b, pb, ldb, tb = _m3(B, dt)
    if tb:
        b, pb, ldb, tb = _m3(_c(B, dt), dt)
    M, N = b.shape
    if n != (M if side == "L" else N):
        raise ValueError(f"incompatible dimensions: {A.shape} and {B.shape} (side {side})")
    C, given, ldc = _output(C, (M, N), dt)
    _check(_lib.gen9blas_symm(_kind(dt, accurate), _SIDE[side], _TRI[uplo], M, N, alpha, pa, lda, pb, ldb,
                              beta if given else 0.0, C.ctypes.data, ldc))
    return C


def syrk(A, uplo="L", trans=False, alpha=1.0, beta=0.0, C=None, accurate=False):
    """C = alpha·op(A)·op(A)ᵀ + beta·C on the uplo triangle (the other triangle of C is not modified)."""
    _init()
    dt = A.dtype if A.dtype in (np.float16, np.float32, np.float64) else np.float32
    N, K = (A.shape[1], A.shape[0]) if trans else A.shape
    a, pa, lda, ta = _m3(A, dt)   # a transposed view flips trans
    C, given, ldc = _output(C, (N, N), dt)
    if not given:
        C[...] = 0
    _check(_lib.gen9blas_syrk(_kind(dt, accurate), _TRI[uplo], int(trans) ^ ta, N, K, alpha, pa, lda,
                              beta if given else 0.0, C.ctypes.data, ldc))
    return C


def syr2k(A, B, uplo="L", trans=False, alpha=1.0, beta=0.0, C=None, accurate=False):
    """C = alpha·(op(A)·op(B)ᵀ + op(B)·op(A)ᵀ) + beta·C on the uplo triangle."""
    _init()
    dt = A.dtype if A.dtype in (np.float16, np.float32, np.float64) else np.float32
    N, K = (A.shape[1], A.shape[0]) if trans else A.shape
    a, pa, lda, ta = _m3(A, dt)
    b, pb, ldb, tb = _m3(B, dt)
    if ta != tb:   # one trans flag for both operands: B is copied to A's layout
        b, pb, ldb, tb = _m3(np.ascontiguousarray(B.T, dtype=dt).T if ta else _c(B, dt), dt)
    C, given, ldc = _output(C, (N, N), dt)
    if not given:
        C[...] = 0
    _check(_lib.gen9blas_syr2k(_kind(dt, accurate), _TRI[uplo], int(trans) ^ ta, N, K, alpha, pa, lda, pb, ldb,
                               beta if given else 0.0, C.ctypes.data, ldc))
    return C


def trmm(A, B, side="L", uplo="L", transA=False, diag=False, alpha=1.0, accurate=False):
    """Returns alpha·op(A)·B (side="L") or alpha·B·op(A) (side="R"); A triangular. B is not modified."""
    _init()
    dt = B.dtype if B.dtype in (np.float16, np.float32, np.float64) else np.float32
    a, pa, _, lda, ta, uplo = _square(A, dt, uplo)
    b = np.array(B, dtype=dt, order="C", copy=True)
    M, N = b.shape
    _check(_lib.gen9blas_trmm(_kind(dt, accurate), _SIDE[side], _TRI[uplo], int(transA) ^ ta, int(diag), M, N,
                              alpha, pa, lda, b.ctypes.data, N))
    return b


def trsm(A, B, side="L", uplo="L", transA=False, diag=False, alpha=1.0, accurate=False):
    """Returns X with op(A)·X = alpha·B (side="L") or X·op(A) = alpha·B (side="R"); A triangular. B is not modified.
    Diagonal-block inverses in FP64 on the GPU; the block updates in the element type's GEMM."""
    _init()
    dt = B.dtype if B.dtype in (np.float16, np.float32, np.float64) else np.float32
    a, pa, _, lda, ta, uplo = _square(A, dt, uplo)
    b = np.array(B, dtype=dt, order="C", copy=True)
    M, N = b.shape
    _check(_lib.gen9blas_trsm(_kind(dt, accurate), _SIDE[side], _TRI[uplo], int(transA) ^ ta, int(diag), M, N,
                              alpha, pa, lda, b.ctypes.data, N))
    return b


def last_time_ms():
    """GEN9BLAS_PROFILE=1: kernel time of the last call; otherwise the whole call."""
    return _lib.gen9blas_last_time_ms()


def last_zero_copy():
    """Bits 1 = A, 2 = B, 4 = C used in place (device or managed memory) by the last call."""
    return _lib.gen9blas_last_zero_copy()


# ---------------- levels 1-2 ----------------

def _dtype_of(*X):
    """Compute type from the first array: float16, float64 or (anything else) float32."""
    return np.float16 if X[0].dtype == np.float16 else np.float64 if X[0].dtype == np.float64 else np.float32


def _vec(x, dt, write=False):
    """(array, pointer to the lowest address, n, inc) of a 1-D vector; inc < 0 as in BLAS."""
    if x.ndim != 1:
        raise ValueError("expected a 1-D vector")
    if x.dtype != dt or x.strides[0] % x.itemsize or x.strides[0] == 0:
        if write:
            raise TypeError(f"the result must be a {np.dtype(dt).name} vector with a stride that is a multiple of the "
                            "element size")
        x = np.ascontiguousarray(x, dtype=dt)
    n, inc = x.shape[0], x.strides[0] // x.itemsize
    return x, x.ctypes.data + (min(inc, 0) * (n - 1) * x.itemsize if n else 0), n, inc


def _kind_basic(dt):
    return GEN9BLAS_S if dt == np.float32 else GEN9BLAS_D if dt == np.float64 else GEN9BLAS_H


def axpy(a, x, y):
    """y = a·x + y (in place); returns y."""
    _init()
    t = _dtype_of(y)
    y, py, n, iy = _vec(y, t, True)
    x, px, nx, ix = _vec(x, t)
    if nx != n:
        raise ValueError("lengths differ")
    _check(_lib.gen9blas_axpy(_kind_basic(t), n, a, px, ix, py, iy))
    return y


def dot(x, y):
    _init()
    t = _dtype_of(x)
    x, px, n, ix = _vec(x, t)
    y, py, ny, iy = _vec(y, t)
    if ny != n:
        raise ValueError("lengths differ")
    w = _d()
    _check(_lib.gen9blas_dot(_kind_basic(t), n, px, ix, py, iy, ctypes.byref(w)))
    return w.value


def asum(x):
    _init()
    t = _dtype_of(x)
    x, px, n, ix = _vec(x, t)
    w = _d()
    _check(_lib.gen9blas_asum(_kind_basic(t), n, px, ix, ctypes.byref(w)))
    return w.value


def nrm2(x):
    _init()
    t = _dtype_of(x)
    x, px, n, ix = _vec(x, t)
    w = _d()
    _check(_lib.gen9blas_nrm2(_kind_basic(t), n, px, ix, ctypes.byref(w)))
    return w.value


def iamax(x):
    """Index (0-based) of the first largest |x|; -1 for an empty vector."""
    _init()
    t = _dtype_of(x)
    x, px, n, ix = _vec(x, t)
    w = _l()
    _check(_lib.gen9blas_iamax(_kind_basic(t), n, px, ix, ctypes.byref(w)))
    return w.value


def gemv(A, x, alpha=1.0, beta=0.0, y=None, trans=False):
    """y = alpha·op(A)·x + beta·y; without y a new array. An A.T view is used without a copy."""
    _init()
    t = _dtype_of(A)
    A, pa, M, N, lda, tr = _mat(A, t)
    tr ^= int(trans)
    x, px, nx, ix = _vec(x, t)
    ny = N if tr else M
    if nx != (M if tr else N):
        raise ValueError("length of x does not match A")
    if y is None:
        y, beta = empty((ny,), t), 0.0
    y, py, n, iy = _vec(y, t, True)
    if n != ny:
        raise ValueError("length of y does not match A")
    _check(_lib.gen9blas_gemv(_kind_basic(t), tr, M, N, alpha, pa, lda, px, ix, beta, py, iy))
    return y


def ger(alpha, x, y, A):
    """A = alpha·x·yᵀ + A (in place); returns A."""
    _init()
    t = _dtype_of(A)
    A, pa, M, N, lda, _ = _mat(A, t, True)
    x, px, nx, ix = _vec(x, t)
    y, py, ny, iy = _vec(y, t)
    if nx != M or ny != N:
        raise ValueError("lengths of x, y do not match A")
    _check(_lib.gen9blas_ger(_kind_basic(t), M, N, alpha, px, ix, py, iy, pa, lda))
    return A


# ---------------- rest of levels 1-2 (lib/gen9blas.py:343-373, 420-610 of the reference) ----------------
_lib.gen9blas_scal.argtypes = [_i, _i, _d, _p, _i]
_lib.gen9blas_copy.argtypes = [_i, _i, _p, _i, _p, _i]
_lib.gen9blas_swap.argtypes = [_i, _i, _p, _i, _p, _i]
_lib.gen9blas_rot.argtypes = [_i, _i, _p, _i, _p, _i, _d, _d]
_lib.gen9blas_rotm.argtypes = [_i, _i, _p, _i, _p, _i, ctypes.POINTER(_d)]
_fp = ctypes.POINTER(ctypes.c_float)
_lib.gen9blas_rotg.argtypes = [_fp, _fp, _fp, _fp]
_lib.gen9blas_rotg.restype = None
_lib.gen9blas_rotmg.argtypes = [_fp, _fp, _fp, ctypes.c_float, _fp]
_lib.gen9blas_rotmg.restype = None
_lib.gen9blas_symv.argtypes = [_i, _i, _i, _d, _p, _i, _p, _i, _d, _p, _i]
_lib.gen9blas_trmv.argtypes = [_i, _i, _i, _i, _i, _p, _i, _p, _i]
_lib.gen9blas_trsv.argtypes = [_i, _i, _i, _i, _i, _p, _i, _p, _i]
_lib.gen9blas_syr.argtypes = [_i, _i, _i, _d, _p, _i, _p, _i]
_lib.gen9blas_syr2.argtypes = [_i, _i, _i, _d, _p, _i, _p, _i, _p, _i]
_lib.gen9blas_gbmv.argtypes = [_i] * 6 + [_d, _p, _i, _p, _i, _d, _p, _i]
_lib.gen9blas_sbmv.argtypes = [_i] * 4 + [_d, _p, _i, _p, _i, _d, _p, _i]
_lib.gen9blas_tbmv.argtypes = [_i] * 6 + [_p, _i, _p, _i]
_lib.gen9blas_tbsv.argtypes = [_i] * 6 + [_p, _i, _p, _i]
_lib.gen9blas_spmv.argtypes = [_i] * 3 + [_d, _p, _p, _i, _d, _p, _i]
_lib.gen9blas_tpmv.argtypes = [_i] * 5 + [_p, _p, _i]
_lib.gen9blas_tpsv.argtypes = [_i] * 5 + [_p, _p, _i]
_lib.gen9blas_spr.argtypes = [_i] * 3 + [_d, _p, _i, _p]
_lib.gen9blas_spr2.argtypes = [_i] * 3 + [_d, _p, _i, _p, _i, _p]


def _pair(x, y, write_y=True):
    t = _dtype_of(x)
    x, px, n, ix = _vec(x, t, True)
    y, py, ny, iy = _vec(y, t, write_y)
    if ny != n:
        raise ValueError("lengths differ")
    return t, x, px, n, ix, y, py, iy


def scal(a, x):
    """x = a·x (in place); returns x."""
    _init()
    t = _dtype_of(x)
    x, px, n, ix = _vec(x, t, True)
    _check(_lib.gen9blas_scal(_kind_basic(t), n, a, px, ix))
    return x


def copy(x, y=None):
    """y = x; without y: a new array (gen9blas.empty) of the type of x."""
    _init()
    t = _dtype_of(y if y is not None else x)
    if y is None:
        y = empty(x.shape, t)
    y, py, n, iy = _vec(y, t, True)
    x, px, nx, ix = _vec(x, t)
    if nx != n:
        raise ValueError("lengths differ")
    _check(_lib.gen9blas_copy(_kind_basic(t), n, px, ix, py, iy))
    return y


def swap(x, y):
    _init()
    t, x, px, n, ix, y, py, iy = _pair(x, y)
    _check(_lib.gen9blas_swap(_kind_basic(t), n, px, ix, py, iy))
    return x, y


def rot(x, y, c, s):
    """x, y = c·x + s·y, c·y − s·x (in place)."""
    _init()
    t, x, px, n, ix, y, py, iy = _pair(x, y)
    _check(_lib.gen9blas_rot(_kind_basic(t), n, px, ix, py, iy, c, s))
    return x, y


def rotm(x, y, param):
    """x, y = h11·x + h12·y, h21·x + h22·y (in place); param: (flag, h11, h21, h12, h22) as in BLAS."""
    _init()
    t, x, px, n, ix, y, py, iy = _pair(x, y)
    pr = (_d * 5)(*[float(v) for v in param])
    _check(_lib.gen9blas_rotm(_kind_basic(t), n, px, ix, py, iy, pr))
    return x, y


def rotg(a, b):
    """(r, z, c, s): the Givens rotation that zeroes b (computed on the CPU)."""
    w = [ctypes.c_float(a), ctypes.c_float(b), ctypes.c_float(), ctypes.c_float()]
    _lib.gen9blas_rotg(*[ctypes.byref(v) for v in w])
    return tuple(v.value for v in w)


def rotmg(d1, d2, x1, y1):
    """(d1, d2, x1, param): modified Givens rotation (CPU); param as in BLAS (5 numbers)."""
    w = [ctypes.c_float(d1), ctypes.c_float(d2), ctypes.c_float(x1)]
    pr = (ctypes.c_float * 5)()
    _lib.gen9blas_rotmg(*[ctypes.byref(v) for v in w], ctypes.c_float(y1), pr)
    return w[0].value, w[1].value, w[2].value, np.array(pr[:], np.float32)


_FLIP = {"L": "U", "U": "L"}


def _sq(A, t, uplo):
    """(pointer, n, ld, transposed, uplo in memory): an A.T view is read in place with the triangle swapped."""
    A, pa, M, N, lda, tr = _mat(A, t)
    if M != N:
        raise ValueError("expected a square matrix")
    return A, pa, N, lda, tr, _FLIP[uplo] if tr else uplo


def _out_vec(y, n, t, beta):
    if y is None:
        return empty((n,), t), 0.0
    return y, beta


def symv(A, x, uplo="L", alpha=1.0, beta=0.0, y=None):
    """y = alpha·A·x + beta·y, A symmetric (its uplo triangle is read); without y: a new array."""
    _init()
    t = _dtype_of(A)
    A, pa, n, lda, _, u = _sq(A, t, uplo)
    x, px, nx, ix = _vec(x, t)
    y, beta = _out_vec(y, n, t, beta)
    y, py, ny, iy = _vec(y, t, True)
    if nx != n or ny != n:
        raise ValueError("lengths of x, y do not match A")
    _check(_lib.gen9blas_symv(_kind_basic(t), _TRI[u], n, alpha, pa, lda, px, ix, beta, py, iy))
    return y


def trmv(A, x, uplo="L", trans=False, diag=False):
    """x = op(A)·x (in place), A triangular; diag=True: unit diagonal. Returns x."""
    _init()
    t = _dtype_of(x)
    A, pa, n, lda, tr, u = _sq(A, t, uplo)
    x, px, nx, ix = _vec(x, t, True)
    if nx != n:
        raise ValueError("length of x does not match A")
    _check(_lib.gen9blas_trmv(_kind_basic(t), _TRI[u], int(trans) ^ tr, int(diag), n, pa, lda, px, ix))
    return x


def trsv(A, x, uplo="L", trans=False, diag=False):
    """Solves op(A)·z = x and stores z in x (in place); A triangular. Returns x."""
    _init()
    t = _dtype_of(x)
    A, pa, n, lda, tr, u = _sq(A, t, uplo)
    x, px, nx, ix = _vec(x, t, True)
    if nx != n:
        raise ValueError("length of x does not match A")
    _check(_lib.gen9blas_trsv(_kind_basic(t), _TRI[u], int(trans) ^ tr, int(diag), n, pa, lda, px, ix))
    return x


def syr(alpha, x, A, uplo="L"):
    """A = alpha·x·xᵀ + A on the uplo triangle (in place); returns A."""
    _init()
    t = _dtype_of(A)
    A, pa, M, N, lda, _ = _mat(A, t, True)
    x, px, n, ix = _vec(x, t)
    if not M == N == n:
        raise ValueError("dimensions do not match")
    _check(_lib.gen9blas_syr(_kind_basic(t), _TRI[uplo], n, alpha, px, ix, pa, lda))
    return A


def syr2(alpha, x, y, A, uplo="L"):
    """A = alpha·(x·yᵀ + y·xᵀ) + A on the uplo triangle (in place); returns A."""
    _init()
    t = _dtype_of(A)
    A, pa, M, N, lda, _ = _mat(A, t, True)
    x, px, n, ix = _vec(x, t)
    y, py, ny, iy = _vec(y, t)
    if not M == N == n == ny:
        raise ValueError("dimensions do not match")
    _check(_lib.gen9blas_syr2(_kind_basic(t), _TRI[uplo], n, alpha, px, ix, py, iy, pa, lda))
    return A


def _band(A, t, width, write=False):
    A, pa, M, W, lda, tr = _mat(A, t, write)
    if tr or W != width:
        raise ValueError(f"band: expected a row-major array with {width} columns")
    return A, pa, M, lda


def _packed(Ap, t, n, write=False):
    Ap, pp, m, inc = _vec(Ap, t, write)
    if inc != 1 or m != n * (n + 1) // 2:
        raise ValueError(f"packed: expected a contiguous vector of length {n * (n + 1) // 2}")
    return Ap, pp


def gbmv(A, x, M, N, KL, KU, alpha=1.0, beta=0.0, y=None, trans=False):
    """y = alpha·op(A)·x + beta·y, A: M×N banded (array (M, KL + KU + 1), A[i, KL + j − i] = A(i, j))."""
    _init()
    t = _dtype_of(A)
    A, pa, m, lda = _band(A, t, KL + KU + 1)
    if m != M:
        raise ValueError("number of band rows != M")
    x, px, nx, ix = _vec(x, t)
    y, beta = _out_vec(y, N if trans else M, t, beta)
    y, py, ny, iy = _vec(y, t, True)
    if nx != (M if trans else N) or ny != (N if trans else M):
        raise ValueError("lengths of x, y")
    _check(_lib.gen9blas_gbmv(_kind_basic(t), int(trans), M, N, KL, KU, alpha, pa, lda, px, ix, beta, py, iy))
    return y


def sbmv(A, x, K, uplo="L", alpha=1.0, beta=0.0, y=None):
    """y = alpha·A·x + beta·y, A symmetric banded (array (n, K + 1), the uplo triangle)."""
    _init()
    t = _dtype_of(A)
    A, pa, n, lda = _band(A, t, K + 1)
    x, px, nx, ix = _vec(x, t)
    y, beta = _out_vec(y, n, t, beta)
    y, py, ny, iy = _vec(y, t, True)
    if nx != n or ny != n:
        raise ValueError("lengths of x, y")
    _check(_lib.gen9blas_sbmv(_kind_basic(t), _TRI[uplo], n, K, alpha, pa, lda, px, ix, beta, py, iy))
    return y


def tbmv(A, x, K, uplo="L", trans=False, diag=False):
    """x = op(A)·x (in place), A triangular banded (array (n, K + 1))."""
    _init()
    t = _dtype_of(x)
    A, pa, n, lda = _band(A, t, K + 1)
    x, px, nx, ix = _vec(x, t, True)
    _check(_lib.gen9blas_tbmv(_kind_basic(t), _TRI[uplo], int(trans), int(diag), n, K, pa, lda, px, ix))
    return x


def tbsv(A, x, K, uplo="L", trans=False, diag=False):
    """Solves op(A)·z = x (in place), A triangular banded (array (n, K + 1))."""
    _init()
    t = _dtype_of(x)
    A, pa, n, lda = _band(A, t, K + 1)
    x, px, nx, ix = _vec(x, t, True)
    _check(_lib.gen9blas_tbsv(_kind_basic(t), _TRI[uplo], int(trans), int(diag), n, K, pa, lda, px, ix))
    return x


def spmv(Ap, x, uplo="L", alpha=1.0, beta=0.0, y=None):
    """y = alpha·A·x + beta·y, A symmetric packed (vector of n(n+1)/2)."""
    _init()
    t = _dtype_of(Ap)
    x, px, n, ix = _vec(x, t)
    Ap, pp = _packed(Ap, t, n)
    y, beta = _out_vec(y, n, t, beta)
    y, py, ny, iy = _vec(y, t, True)
    _check(_lib.gen9blas_spmv(_kind_basic(t), _TRI[uplo], n, alpha, pp, px, ix, beta, py, iy))
    return y


def tpmv(Ap, x, uplo="L", trans=False, diag=False):
    """x = op(A)·x (in place), A triangular packed."""
    _init()
    t = _dtype_of(x)
    x, px, n, ix = _vec(x, t, True)
    Ap, pp = _packed(Ap, t, n)
    _check(_lib.gen9blas_tpmv(_kind_basic(t), _TRI[uplo], int(trans), int(diag), n, pp, px, ix))
    return x


def tpsv(Ap, x, uplo="L", trans=False, diag=False):
    """Solves op(A)·z = x (in place), A triangular packed."""
    _init()
    t = _dtype_of(x)
    x, px, n, ix = _vec(x, t, True)
    Ap, pp = _packed(Ap, t, n)
    _check(_lib.gen9blas_tpsv(_kind_basic(t), _TRI[uplo], int(trans), int(diag), n, pp, px, ix))
    return x


def spr(alpha, x, Ap, uplo="L"):
    """A = alpha·x·xᵀ + A (packed, in place)."""
    _init()
    t = _dtype_of(Ap)
    x, px, n, ix = _vec(x, t)
    Ap, pp = _packed(Ap, t, n, True)
    _check(_lib.gen9blas_spr(_kind_basic(t), _TRI[uplo], n, alpha, px, ix, pp))
    return Ap


def spr2(alpha, x, y, Ap, uplo="L"):
    """A = alpha·(x·yᵀ + y·xᵀ) + A (packed, in place)."""
    _init()
    t = _dtype_of(Ap)
    x, px, n, ix = _vec(x, t)
    y, py, ny, iy = _vec(y, t)
    Ap, pp = _packed(Ap, t, n, True)
    _check(_lib.gen9blas_spr2(_kind_basic(t), _TRI[uplo], n, alpha, px, ix, py, iy, pp))
    return Ap


# ---------------- constant weights kept on the GPU (lib/gen9blas.h:89-97, lib/gen9blas_ml.h:25-28) ----------------
_lib.gen9blas_pack_b.argtypes = [_i, _i, _i, _i, _p, _i]
_lib.gen9blas_pack_b.restype = _p
_lib.gen9blas_gemm_pb.argtypes = [_i, _i, _d, _p, _i, _p, _d, _p, _i]
_lib.gen9blas_packed_b_free.argtypes = [_p]
_lib.gen9blas_packed_b_free.restype = None
_lib.gen9blas_gemm_pb_skinny.argtypes = [_i, _p, _i, _p, _p, _i, ctypes.POINTER(_i)]


class PackedB:
    """op(B) packed once into GPU memory (gen9blas_pack_b), multiplied many times. B: a (K, N) matrix, or with
    transB=True the (N, K) weight matrix (W[N][K] as ggml and most checkpoints store it); a transposed view is read in
    place. B may be changed or freed afterwards. The device memory is released by free() (or when the object is
    collected)."""

    def __init__(self, B, transB=False, accurate=False):
        _init()
        dt = B.dtype if B.dtype in (np.float16, np.float32, np.float64) else np.float32
        B, pb, R, Cn, ldb, tr = _mat(B, dt)
        tB = int(transB) ^ tr                 # stored R × Cn: op(B) is R × Cn (tB = 0) or Cn × R (tB = 1)
        self.K, self.N = (Cn, R) if tB else (R, Cn)
        self.dtype, self.type = np.dtype(dt), _kind(dt, accurate)
        p = _lib.gen9blas_pack_b(self.type, tB, self.K, self.N, pb, ldb)
        if not p:
            raise RuntimeError(_lib.gen9blas_error().decode())
        self._p = p

    def free(self):
        if getattr(self, "_p", None):
            _lib.gen9blas_packed_b_free(self._p)
            self._p = None

    def __del__(self):
        self.free()

    def gemm(self, A, alpha=1.0, beta=0.0, C=None):
        """C = alpha·A·op(B) + beta·C (A: M × K of the packed type; an A.T view is read in place)."""
        if not self._p:
            raise ValueError("packed B was freed")
        a, pa, M, K, lda, ta = _mat(A, self.dtype)
        if ta:
            M, K = K, M
        if K != self.K:
            raise ValueError(f"A has {K} columns, the packed B {self.K} rows")
        C, given, ldc = _output(C, (M, self.N), self.dtype)
        _check(_lib.gen9blas_gemm_pb(ta, M, alpha, pa, lda, self._p, beta if given else 0.0, C.ctypes.data, ldc))
        return C

    def skinny(self, A):
        """(C, nonfinite): C = A·op(B) in FP32 for FP32 activations A (1 to 16 rows) and FP16 weights packed with
        accurate=True (gen9blas_gemm_pb_skinny)."""
        if not self._p:
            raise ValueError("packed B was freed")
        A = np.ascontiguousarray(A, dtype=np.float32)
        M, K = A.shape
        if K != self.K:
            raise ValueError(f"A has {K} columns, the packed B {self.K} rows")
        C = np.empty((M, self.N), np.float32)
        nf = _i(0)
        r = _lib.gen9blas_gemm_pb_skinny(M, A.ctypes.data, K, self._p, C.ctypes.data, self.N, ctypes.byref(nf))
        if r == 1:
            raise ValueError("gemm_pb_skinny takes 1 to 16 rows")
        _check(r)
        return C, bool(nf.value)


def pack_b(B, transB=False, accurate=False):
    return PackedB(B, transB, accurate)
