"""gen9blas -- NumPy module over libgen9blas.so, the B200 (sm_100a) build of gen9blas.

    import numpy as np, gen9blas
    C = gen9blas.hgemm(A, B)                      # float16, FP16 accumulation; accurate=True: FP32 accumulation
    C = gen9blas.sgemm(A.T, B, alpha=2.0)         # float32; transposed views and row slices without a copy
    C = gen9blas.gemm_batched(A3, B3)             # (count, M, K) · (count, K, N) -> (count, M, N)
    X = gen9blas.empty((n, n), np.float16)        # managed memory: used in place by the GPU, writable by the CPU
    gen9blas.axpy(0.5, x, y); d = gen9blas.dot(x, y); i = gen9blas.iamax(x)
    y = gen9blas.gemv(A, x); gen9blas.ger(1.0, x, y, A)
    C = gen9blas.symm(S, B); C = gen9blas.syrk(A, "L"); X = gen9blas.trsm(T, B, "L", "U")   # level 3 on GEMM

The public functions keep the names, argument meaning and error behaviour of the reference module lib/gen9blas.py of
kprzybys/gen9-gpu-blas (gemm/hgemm/sgemm/gemm_batched 168-204, symm..trsm 207-272, empty/free_pool 60-115, axpy..ger
335-419, the rest of levels 1-2 343-373 and 420-610): the element type follows the dtype; a 2-D operand whose rows are
contiguous is passed in place with its row stride as the leading dimension, a transposed view of such an array is
passed in place with the transpose flag set (lib/gen9blas.py:316-328), anything else is copied first (a result that
cannot be addressed raises TypeError); a 1-D operand is passed with its element stride as the BLAS increment
(negative: pointer to the lowest address); library errors raise RuntimeError with gen9blas_error().

Memory: plain NumPy arrays are staged through device buffers by the library. gen9blas.empty() returns arrays in CUDA
managed memory, which the GPU reads and writes in place; released blocks are kept per power-of-two size class (up to
CACHE_LIMIT bytes in total) because cudaMallocManaged / cudaFree synchronise the device.
"""
import ctypes
import os
from typing import NamedTuple

import numpy as np

_HERE = os.path.dirname(os.path.realpath(__file__))

# ------------------------------------------------------------------------------------------------ the C library
_I, _D, _P, _L64 = ctypes.c_int, ctypes.c_double, ctypes.c_void_p, ctypes.c_int64
_F = ctypes.c_float
_FP = ctypes.POINTER(_F)
# name -> (argument types, result type); every entry point this module calls, as declared in include/gen9blas.h
_SIGNATURES = {
    "version": ([], _I), "init": ([], _I), "has": ([_I], _I), "error": ([], ctypes.c_char_p),
    "last_time_ms": ([], _D), "last_zero_copy": ([], _I), "kernel_launches": ([], ctypes.c_longlong),
    "alloc": ([ctypes.c_size_t], _P), "free": ([_P], None),
    "set_device": ([_I], _I), "set_stream": ([_P], _I), "set_nowait": ([_I], None), "flush": ([], _I),
    "gemm": ([_I] * 6 + [_D, _P, _I, _P, _I, _D, _P, _I], _I),
    "gemm_batched": ([_I] * 6 + [_D, _P, _I, _L64, _P, _I, _L64, _D, _P, _I, _L64, _I], _I),
    "symm": ([_I] * 5 + [_D, _P, _I, _P, _I, _D, _P, _I], _I),
    "syrk": ([_I] * 5 + [_D, _P, _I, _D, _P, _I], _I),
    "syr2k": ([_I] * 5 + [_D, _P, _I, _P, _I, _D, _P, _I], _I),
    "trmm": ([_I] * 7 + [_D, _P, _I, _P, _I], _I),
    "trsm": ([_I] * 7 + [_D, _P, _I, _P, _I], _I),
    "axpy": ([_I, _I, _D, _P, _I, _P, _I], _I),
    "dot": ([_I, _I, _P, _I, _P, _I, ctypes.POINTER(_D)], _I),
    "asum": ([_I, _I, _P, _I, ctypes.POINTER(_D)], _I),
    "nrm2": ([_I, _I, _P, _I, ctypes.POINTER(_D)], _I),
    "iamax": ([_I, _I, _P, _I, ctypes.POINTER(_L64)], _I),
    "gemv": ([_I] * 4 + [_D, _P, _I, _P, _I, _D, _P, _I], _I),
    "ger": ([_I] * 3 + [_D, _P, _I, _P, _I, _P, _I], _I),
    "scal": ([_I, _I, _D, _P, _I], _I),
    "copy": ([_I, _I, _P, _I, _P, _I], _I),
    "swap": ([_I, _I, _P, _I, _P, _I], _I),
    "rot": ([_I, _I, _P, _I, _P, _I, _D, _D], _I),
    "rotm": ([_I, _I, _P, _I, _P, _I, ctypes.POINTER(_D)], _I),
    "rotg": ([_FP] * 4, None),
    "rotmg": ([_FP, _FP, _FP, _F, _FP], None),
    "symv": ([_I] * 3 + [_D, _P, _I, _P, _I, _D, _P, _I], _I),
    "trmv": ([_I] * 5 + [_P, _I, _P, _I], _I),
    "trsv": ([_I] * 5 + [_P, _I, _P, _I], _I),
    "syr": ([_I] * 3 + [_D, _P, _I, _P, _I], _I),
    "syr2": ([_I] * 3 + [_D, _P, _I, _P, _I, _P, _I], _I),
    "gbmv": ([_I] * 6 + [_D, _P, _I, _P, _I, _D, _P, _I], _I),
    "sbmv": ([_I] * 4 + [_D, _P, _I, _P, _I, _D, _P, _I], _I),
    "tbmv": ([_I] * 6 + [_P, _I, _P, _I], _I),
    "tbsv": ([_I] * 6 + [_P, _I, _P, _I], _I),
    "spmv": ([_I] * 3 + [_D, _P, _P, _I, _D, _P, _I], _I),
    "tpmv": ([_I] * 5 + [_P, _P, _I], _I),
    "tpsv": ([_I] * 5 + [_P, _P, _I], _I),
    "spr": ([_I] * 3 + [_D, _P, _I, _P], _I),
    "spr2": ([_I] * 3 + [_D, _P, _I, _P, _I, _P], _I),
    "pack_b": ([_I] * 4 + [_P, _I], _P),
    "gemm_pb": ([_I, _I, _D, _P, _I, _P, _D, _P, _I], _I),
    "packed_b_free": ([_P], None),
    "gemm_pb_skinny": ([_I, _P, _I, _P, _P, _I, ctypes.POINTER(_I)], _I),
}

_lib = ctypes.CDLL(os.environ.get("GEN9BLAS_LIB") or os.path.join(_HERE, "libgen9blas.so"))
_fn = {}
for _name, (_args, _res) in _SIGNATURES.items():
    _f = getattr(_lib, "gen9blas_" + _name)
    _f.argtypes, _f.restype = _args, _res
    _fn[_name] = _f

GEN9BLAS_H, GEN9BLAS_S, GEN9BLAS_HS, GEN9BLAS_D = 0, 1, 2, 3
FEAT_FP16, FEAT_FP32, FEAT_FP64 = 0, 1, 2
if _fn["version"]() // 100 != 2:   # this module speaks the 0.2.x API
    raise ImportError(f"gen9blas.py expects libgen9blas 0.2.x, loaded {_fn['version']()}")

_state = {"up": False}


def _error_text():
    return _fn["error"]().decode(errors="replace")


def _session():
    """Initialises the library once (gen9blas_init); a failure raises RuntimeError with the library's message."""
    if not _state["up"]:
        if _fn["init"]() != 0:
            raise RuntimeError(_error_text())
        _state["up"] = True


_init = _session   # the reference module's name for it


def _call(name, *args):
    """Calls gen9blas_<name>; a non-zero status raises RuntimeError with the library's message."""
    status = _fn[name](*args)
    if status != 0:
        raise RuntimeError(_error_text())
    return status


# ------------------------------------------------------------------------------------------------ managed memory
CACHE_LIMIT = 1 << 30   # bytes of released managed blocks kept for reuse
_MIN_BLOCK = 1 << 16


class _ManagedCache:
    """Released managed blocks by size class (powers of two from 64 KiB). cudaMallocManaged and cudaFree both
    synchronise the device, so a block of the right class is handed out again instead; past CACHE_LIMIT the largest
    cached blocks go back to the driver first."""

    def __init__(self):
        self.free = {}
        self.bytes = 0

    @staticmethod
    def size_class(nbytes):
        return max(_MIN_BLOCK, 1 << max(0, int(nbytes) - 1).bit_length())

    def take(self, nbytes):
        cls = self.size_class(nbytes)
        blocks = self.free.get(cls)
        if blocks:
            self.bytes -= cls
            return blocks.pop(), cls
        ptr = _fn["alloc"](cls)
        if not ptr:
            raise MemoryError(_error_text())
        return ptr, cls

    def give_back(self, ptr, cls):
        self.free.setdefault(cls, []).append(ptr)
        self.bytes += cls
        while self.bytes > CACHE_LIMIT:
            big = max(c for c, b in self.free.items() if b)
            _fn["free"](self.free[big].pop())
            self.bytes -= big

    def drop_all(self):
        for blocks in self.free.values():
            for ptr in blocks:
                _fn["free"](ptr)
        self.free.clear()
        self.bytes = 0


_cache = _ManagedCache()


class _ManagedBlock:
    """Owner of one managed block, exposed to NumPy through the array interface; NumPy keeps it as the base of every
    view, so the block returns to the cache only when the last view is gone."""

    def __init__(self, ptr, cls, shape, dtype):
        self.ptr, self.cls = ptr, cls
        self.__array_interface__ = {"shape": tuple(shape), "typestr": np.dtype(dtype).str, "data": (ptr, False),
                                    "version": 3}

    def __del__(self):
        if self.ptr and _cache is not None:
            _cache.give_back(self.ptr, self.cls)
            self.ptr = None


def empty(shape, dtype=np.float16):
    """C-contiguous array in CUDA managed memory: the GPU uses it (and its views and slices) in place, the CPU reads
    and writes it directly. The block returns to the cache when the last view is gone."""
    _session()
    shape = (shape,) if np.isscalar(shape) else tuple(int(s) for s in shape)
    dtype = np.dtype(dtype)
    nbytes = int(np.prod(shape, dtype=np.int64)) * dtype.itemsize
    ptr, cls = _cache.take(max(nbytes, 1))
    return np.asarray(_ManagedBlock(ptr, cls, shape, dtype))


def free_pool():
    """Hands the cached managed blocks back to the driver (arrays still in use keep theirs)."""
    _cache.drop_all()


# ------------------------------------------------------------------------------------------------ operand mapping
class _Matrix(NamedTuple):
    array: np.ndarray   # the array whose memory is passed (the argument itself, or a copy)
    ptr: int
    rows: int           # stored rows (row-major, leading dimension ld)
    cols: int
    ld: int
    trans: int          # 1: the argument is the transpose of the stored matrix


class _Vector(NamedTuple):
    array: np.ndarray
    ptr: int            # lowest address of the n elements
    n: int
    inc: int


def _type_code(dt, accurate=False):
    dt = np.dtype(dt)
    if dt == np.float16:
        return GEN9BLAS_HS if accurate else GEN9BLAS_H
    if dt == np.float32:
        return GEN9BLAS_S
    if dt == np.float64:
        return GEN9BLAS_D
    raise TypeError("supported types: float16, float32, float64")


def _compute_type(x):
    """Element type of a call from its leading operand: float16 and float64 as given, anything else float32."""
    return np.dtype(x.dtype) if x.dtype in (np.float16, np.float64) else np.dtype(np.float32)


def _matrix(A, dt, out=False):
    """Row-major description of a 2-D operand. Rows contiguous (any row stride that is a whole number of elements):
    in place. The transpose of such an array: in place with trans = 1 (inputs only). Otherwise a C-contiguous copy
    in dt; for a result (out=True) that is an error."""
    if A.ndim != 2:
        raise ValueError("expected a 2-D matrix")
    if A.dtype == dt:
        e = A.itemsize
        s0, s1 = A.strides
        if s1 == e and s0 % e == 0 and s0 >= A.shape[1] * e:
            return _Matrix(A, A.ctypes.data, A.shape[0], A.shape[1], s0 // e, 0)
        if not out and s0 == e and s1 % e == 0 and s1 >= A.shape[0] * e:
            return _Matrix(A, A.ctypes.data, A.shape[1], A.shape[0], s1 // e, 1)
    if out:
        raise TypeError(f"the result must be a {np.dtype(dt).name} matrix with contiguous rows")
    C = np.ascontiguousarray(A, dtype=dt)
    return _Matrix(C, C.ctypes.data, C.shape[0], C.shape[1], C.shape[1], 0)


def _vector(x, dt, out=False):
    """BLAS description of a 1-D operand: stride in elements as the increment (non-zero), the pointer at the lowest
    address for a negative increment; other vectors are copied (a result: TypeError)."""
    if x.ndim != 1:
        raise ValueError("expected a 1-D vector")
    stride = x.strides[0]
    if x.dtype != dt or stride == 0 or stride % x.itemsize:
        if out:
            raise TypeError(f"the result must be a {np.dtype(dt).name} vector with a stride that is a multiple of the "
                            "element size")
        x = np.ascontiguousarray(x, dtype=dt)
        stride = x.itemsize
    n, inc = x.shape[0], stride // x.itemsize
    low = x.ctypes.data + (inc * (n - 1) * x.itemsize if inc < 0 and n else 0)
    return _Vector(x, low, n, inc)


_FLIP = {"L": "U", "U": "L"}
_SIDE = {"L": 0, "R": 1}
_UPLO = {"L": 0, "U": 1}


def _square(A, dt, uplo):
    """A square operand and the triangle to read in its stored form: a transposed view is the stored matrix with the
    other triangle (its trans flag set, for triangular operands)."""
    m = _matrix(A, dt)
    if m.rows != m.cols:
        raise ValueError("expected a square matrix")
    return m, _FLIP[uplo] if m.trans else uplo


def _result(C, shape, dt):
    """(C, given, ldc) of a result: a new array from empty() when C is None, else the supplied C, which must have the
    shape and type and contiguous rows (2-D: any row stride; a batch: C-contiguous)."""
    shape = tuple(shape)
    if C is None:
        return empty(shape, dt), False, shape[-1]
    if C.shape != shape or C.dtype != dt or C.strides[-1] != C.itemsize:
        raise ValueError(f"C must have shape {shape}, type {np.dtype(dt).name} and contiguous rows")
    if C.ndim == 2:
        return C, True, _matrix(C, dt, out=True).ld
    if not C.flags.c_contiguous:
        raise ValueError("C (batch) must be C-contiguous")
    return C, True, shape[-1]


def available(dt, accurate=False):
    """Whether this GPU runs the type."""
    _session()
    feature = {GEN9BLAS_S: FEAT_FP32, GEN9BLAS_D: FEAT_FP64}.get(_type_code(dt, accurate), FEAT_FP16)
    return bool(_fn["has"](feature))


def last_time_ms():
    """Kernel time of the last call with GEN9BLAS_PROFILE=1, else the time of the whole call."""
    return _fn["last_time_ms"]()


def last_zero_copy():
    """Bits of the last call's operands used in place (device or managed memory): 1 = A, 2 = B, 4 = C."""
    return _fn["last_zero_copy"]()


# ------------------------------------------------------------------------------------------------ level 3
def gemm(A, B, alpha=1.0, beta=0.0, C=None, accurate=False):
    """C = alpha·A·B + beta·C; the type is A's (float16, float32 or float64; others compute in float32)."""
    _session()
    dt = _compute_type(A)
    if A.shape[1] != B.shape[0]:
        raise ValueError(f"incompatible dimensions: {A.shape} · {B.shape}")
    M, K, N = A.shape[0], A.shape[1], B.shape[1]
    a, b = _matrix(A, dt), _matrix(B, dt)
    C, given, ldc = _result(C, (M, N), dt)
    _call("gemm", _type_code(dt, accurate), a.trans, b.trans, M, N, K, alpha, a.ptr, a.ld, b.ptr, b.ld,
          beta if given else 0.0, C.ctypes.data, ldc)
    return C


def _as(X, dt):
    return X if X.dtype == dt else X.astype(dt)


def hgemm(A, B, alpha=1.0, beta=0.0, C=None, accurate=False):
    return gemm(_as(A, np.float16), _as(B, np.float16), alpha, beta, C, accurate)


def sgemm(A, B, alpha=1.0, beta=0.0, C=None):
    return gemm(_as(A, np.float32), _as(B, np.float32), alpha, beta, C)


def dgemm(A, B, alpha=1.0, beta=0.0, C=None):
    return gemm(_as(A, np.float64), _as(B, np.float64), alpha, beta, C)


def gemm_batched(A, B, alpha=1.0, beta=0.0, C=None, accurate=False):
    """A (count, M, K), B (count, K, N) -> C (count, M, N) in one launch (operands made C-contiguous)."""
    _session()
    dt = _compute_type(A)
    a, b = np.ascontiguousarray(A, dtype=dt), np.ascontiguousarray(B, dtype=dt)
    if a.ndim != 3 or b.ndim != 3 or a.shape[0] != b.shape[0] or a.shape[2] != b.shape[1]:
        raise ValueError(f"incompatible dimensions: {a.shape} · {b.shape}")
    count, M, K = a.shape
    N = b.shape[2]
    C, given, _ = _result(C, (count, M, N), dt)
    _call("gemm_batched", _type_code(dt, accurate), 0, 0, M, N, K, alpha, a.ctypes.data, K, M * K, b.ctypes.data, N,
          K * N, beta if given else 0.0, C.ctypes.data, N, M * N, count)
    return C


def symm(A, B, side="L", uplo="L", alpha=1.0, beta=0.0, C=None, accurate=False):
    """C = alpha·A·B + beta·C (side="L") or alpha·B·A + beta·C (side="R"); A symmetric, its uplo triangle is read."""
    _session()
    dt = _compute_type(B)
    a, uplo = _square(A, dt, uplo)
    b = _matrix(B, dt)
    if b.trans:   # the library reads B row-major
        b = _matrix(np.ascontiguousarray(B, dtype=dt), dt)
    M, N = b.rows, b.cols
    if a.rows != (M if side == "L" else N):
        raise ValueError(f"incompatible dimensions: {A.shape} and {B.shape} (side {side})")
    C, given, ldc = _result(C, (M, N), dt)
    _call("symm", _type_code(dt, accurate), _SIDE[side], _UPLO[uplo], M, N, alpha, a.ptr, a.ld, b.ptr, b.ld,
          beta if given else 0.0, C.ctypes.data, ldc)
    return C


def syrk(A, uplo="L", trans=False, alpha=1.0, beta=0.0, C=None, accurate=False):
    """C = alpha·op(A)·op(A)ᵀ + beta·C on the uplo triangle (the other triangle of C is left as it is)."""
    _session()
    dt = _compute_type(A)
    N, K = (A.shape[1], A.shape[0]) if trans else A.shape
    a = _matrix(A, dt)
    C, given, ldc = _result(C, (N, N), dt)
    if not given:
        C[...] = 0
    _call("syrk", _type_code(dt, accurate), _UPLO[uplo], int(trans) ^ a.trans, N, K, alpha, a.ptr, a.ld,
          beta if given else 0.0, C.ctypes.data, ldc)
    return C


def syr2k(A, B, uplo="L", trans=False, alpha=1.0, beta=0.0, C=None, accurate=False):
    """C = alpha·(op(A)·op(B)ᵀ + op(B)·op(A)ᵀ) + beta·C on the uplo triangle."""
    _session()
    dt = _compute_type(A)
    N, K = (A.shape[1], A.shape[0]) if trans else A.shape
    a, b = _matrix(A, dt), _matrix(B, dt)
    if b.trans != a.trans:   # one transpose flag serves both: B is copied into A's storage order
        b = _matrix(np.ascontiguousarray(B.T, dtype=dt).T if a.trans else np.ascontiguousarray(B, dtype=dt), dt)
    C, given, ldc = _result(C, (N, N), dt)
    if not given:
        C[...] = 0
    _call("syr2k", _type_code(dt, accurate), _UPLO[uplo], int(trans) ^ a.trans, N, K, alpha, a.ptr, a.ld, b.ptr, b.ld,
          beta if given else 0.0, C.ctypes.data, ldc)
    return C


def _triangular_3(name, A, B, side, uplo, transA, diag, alpha, accurate):
    _session()
    dt = _compute_type(B)
    a, uplo = _square(A, dt, uplo)
    X = np.array(B, dtype=dt, order="C", copy=True)   # the result; B itself stays as it is
    M, N = X.shape
    _call(name, _type_code(dt, accurate), _SIDE[side], _UPLO[uplo], int(transA) ^ a.trans, int(diag), M, N, alpha,
          a.ptr, a.ld, X.ctypes.data, N)
    return X


def trmm(A, B, side="L", uplo="L", transA=False, diag=False, alpha=1.0, accurate=False):
    """Returns alpha·op(A)·B (side="L") or alpha·B·op(A) (side="R"); A triangular. B is not modified."""
    return _triangular_3("trmm", A, B, side, uplo, transA, diag, alpha, accurate)


def trsm(A, B, side="L", uplo="L", transA=False, diag=False, alpha=1.0, accurate=False):
    """Returns X with op(A)·X = alpha·B (side="L") or X·op(A) = alpha·B (side="R"); A triangular. B is not modified.
    Diagonal-block inverses in FP64 on the GPU; the block updates in the element type's GEMM."""
    return _triangular_3("trsm", A, B, side, uplo, transA, diag, alpha, accurate)


# ------------------------------------------------------------------------------------------------ levels 1-2
def _same_length(*vs):
    if len({v.n for v in vs}) != 1:
        raise ValueError("lengths differ")


def _scalar(name, t, x, y=None, out_type=_D):
    """A reduction returning one value through a pointer argument (dot, asum, nrm2, iamax)."""
    r = out_type()
    args = (x.n, x.ptr, x.inc) + ((y.ptr, y.inc) if y is not None else ())
    _call(name, _type_code(t), *args, ctypes.byref(r))
    return r.value


def axpy(a, x, y):
    """y = a·x + y (in place); returns y."""
    _session()
    t = _compute_type(y)
    vy, vx = _vector(y, t, out=True), _vector(x, t)
    _same_length(vx, vy)
    _call("axpy", _type_code(t), vy.n, a, vx.ptr, vx.inc, vy.ptr, vy.inc)
    return y


def dot(x, y):
    _session()
    t = _compute_type(x)
    vx, vy = _vector(x, t), _vector(y, t)
    _same_length(vx, vy)
    return _scalar("dot", t, vx, vy)


def asum(x):
    _session()
    t = _compute_type(x)
    return _scalar("asum", t, _vector(x, t))


def nrm2(x):
    _session()
    t = _compute_type(x)
    return _scalar("nrm2", t, _vector(x, t))


def iamax(x):
    """Index (0-based) of the first largest |x|; -1 for an empty vector."""
    _session()
    t = _compute_type(x)
    return _scalar("iamax", t, _vector(x, t), out_type=_L64)


def _new_or_given(y, n, t, beta):
    """The output vector of a product: a new array (beta = 0) or the given y with its beta."""
    return (empty((n,), t), 0.0) if y is None else (y, beta)


def gemv(A, x, alpha=1.0, beta=0.0, y=None, trans=False):
    """y = alpha·op(A)·x + beta·y; without y a new array. An A.T view is used without a copy."""
    _session()
    t = _compute_type(A)
    a = _matrix(A, t)
    tr = a.trans ^ int(trans)
    vx = _vector(x, t)
    n_in, n_out = (a.rows, a.cols) if tr else (a.cols, a.rows)
    if vx.n != n_in:
        raise ValueError("length of x does not match A")
    y, beta = _new_or_given(y, n_out, t, beta)
    vy = _vector(y, t, out=True)
    if vy.n != n_out:
        raise ValueError("length of y does not match A")
    _call("gemv", _type_code(t), tr, a.rows, a.cols, alpha, a.ptr, a.ld, vx.ptr, vx.inc, beta, vy.ptr, vy.inc)
    return y


def ger(alpha, x, y, A):
    """A = alpha·x·yᵀ + A (in place); returns A."""
    _session()
    t = _compute_type(A)
    a = _matrix(A, t, out=True)
    vx, vy = _vector(x, t), _vector(y, t)
    if vx.n != a.rows or vy.n != a.cols:
        raise ValueError("lengths of x, y do not match A")
    _call("ger", _type_code(t), a.rows, a.cols, alpha, vx.ptr, vx.inc, vy.ptr, vy.inc, a.ptr, a.ld)
    return A


def scal(a, x):
    """x = a·x (in place); returns x."""
    _session()
    t = _compute_type(x)
    v = _vector(x, t, out=True)
    _call("scal", _type_code(t), v.n, a, v.ptr, v.inc)
    return x


def copy(x, y=None):
    """y = x; without y: a new array (gen9blas.empty) of the type of x."""
    _session()
    t = _compute_type(x if y is None else y)
    if y is None:
        y = empty(x.shape, t)
    vy, vx = _vector(y, t, out=True), _vector(x, t)
    _same_length(vx, vy)
    _call("copy", _type_code(t), vy.n, vx.ptr, vx.inc, vy.ptr, vy.inc)
    return y


def _two_written(x, y):
    t = _compute_type(x)
    vx, vy = _vector(x, t, out=True), _vector(y, t, out=True)
    _same_length(vx, vy)
    return t, vx, vy


def swap(x, y):
    _session()
    t, vx, vy = _two_written(x, y)
    _call("swap", _type_code(t), vx.n, vx.ptr, vx.inc, vy.ptr, vy.inc)
    return x, y


def rot(x, y, c, s):
    """x, y = c·x + s·y, c·y − s·x (in place)."""
    _session()
    t, vx, vy = _two_written(x, y)
    _call("rot", _type_code(t), vx.n, vx.ptr, vx.inc, vy.ptr, vy.inc, c, s)
    return x, y


def rotm(x, y, param):
    """x, y = h11·x + h12·y, h21·x + h22·y (in place); param: (flag, h11, h21, h12, h22) as in BLAS."""
    _session()
    t, vx, vy = _two_written(x, y)
    h = (_D * 5)(*map(float, param))
    _call("rotm", _type_code(t), vx.n, vx.ptr, vx.inc, vy.ptr, vy.inc, h)
    return x, y


def rotg(a, b):
    """(r, z, c, s): the Givens rotation that zeroes b (computed on the CPU)."""
    vals = [_F(a), _F(b), _F(), _F()]
    _fn["rotg"](*map(ctypes.byref, vals))
    return tuple(v.value for v in vals)


def rotmg(d1, d2, x1, y1):
    """(d1, d2, x1, param): modified Givens rotation (CPU); param as in BLAS (5 numbers)."""
    vals = [_F(d1), _F(d2), _F(x1)]
    h = (_F * 5)()
    _fn["rotmg"](*map(ctypes.byref, vals), _F(y1), h)
    return vals[0].value, vals[1].value, vals[2].value, np.array(h[:], np.float32)


def symv(A, x, uplo="L", alpha=1.0, beta=0.0, y=None):
    """y = alpha·A·x + beta·y, A symmetric (its uplo triangle is read); without y: a new array."""
    _session()
    t = _compute_type(A)
    a, u = _square(A, t, uplo)
    vx = _vector(x, t)
    y, beta = _new_or_given(y, a.rows, t, beta)
    vy = _vector(y, t, out=True)
    if vx.n != a.rows or vy.n != a.rows:
        raise ValueError("lengths of x, y do not match A")
    _call("symv", _type_code(t), _UPLO[u], a.rows, alpha, a.ptr, a.ld, vx.ptr, vx.inc, beta, vy.ptr, vy.inc)
    return y


def _triangular_2(name, A, x, uplo, trans, diag):
    _session()
    t = _compute_type(x)
    a, u = _square(A, t, uplo)
    vx = _vector(x, t, out=True)
    if vx.n != a.rows:
        raise ValueError("length of x does not match A")
    _call(name, _type_code(t), _UPLO[u], int(trans) ^ a.trans, int(diag), a.rows, a.ptr, a.ld, vx.ptr, vx.inc)
    return x


def trmv(A, x, uplo="L", trans=False, diag=False):
    """x = op(A)·x (in place), A triangular; diag=True: unit diagonal. Returns x."""
    return _triangular_2("trmv", A, x, uplo, trans, diag)


def trsv(A, x, uplo="L", trans=False, diag=False):
    """Solves op(A)·z = x and stores z in x (in place); A triangular. Returns x."""
    return _triangular_2("trsv", A, x, uplo, trans, diag)


def syr(alpha, x, A, uplo="L"):
    """A = alpha·x·xᵀ + A on the uplo triangle (in place); returns A."""
    _session()
    t = _compute_type(A)
    a = _matrix(A, t, out=True)
    vx = _vector(x, t)
    if not a.rows == a.cols == vx.n:
        raise ValueError("dimensions do not match")
    _call("syr", _type_code(t), _UPLO[uplo], vx.n, alpha, vx.ptr, vx.inc, a.ptr, a.ld)
    return A


def syr2(alpha, x, y, A, uplo="L"):
    """A = alpha·(x·yᵀ + y·xᵀ) + A on the uplo triangle (in place); returns A."""
    _session()
    t = _compute_type(A)
    a = _matrix(A, t, out=True)
    vx, vy = _vector(x, t), _vector(y, t)
    if not a.rows == a.cols == vx.n == vy.n:
        raise ValueError("dimensions do not match")
    _call("syr2", _type_code(t), _UPLO[uplo], vx.n, alpha, vx.ptr, vx.inc, vy.ptr, vy.inc, a.ptr, a.ld)
    return A


def _band(A, t, width, out=False):
    """A banded matrix in the BLAS row-major band layout: an (n, width) array with contiguous rows."""
    a = _matrix(A, t, out)
    if a.trans or a.cols != width:
        raise ValueError(f"band: expected a row-major array with {width} columns")
    return a


def _packed_triangle(Ap, t, n, out=False):
    v = _vector(Ap, t, out)
    if v.inc != 1 or v.n != n * (n + 1) // 2:
        raise ValueError(f"packed: expected a contiguous vector of length {n * (n + 1) // 2}")
    return v


def gbmv(A, x, M, N, KL, KU, alpha=1.0, beta=0.0, y=None, trans=False):
    """y = alpha·op(A)·x + beta·y, A: M×N banded (array (M, KL + KU + 1), A[i, KL + j − i] = A(i, j))."""
    _session()
    t = _compute_type(A)
    a = _band(A, t, KL + KU + 1)
    if a.rows != M:
        raise ValueError("number of band rows != M")
    n_in, n_out = (M, N) if trans else (N, M)
    vx = _vector(x, t)
    y, beta = _new_or_given(y, n_out, t, beta)
    vy = _vector(y, t, out=True)
    if vx.n != n_in or vy.n != n_out:
        raise ValueError("lengths of x, y")
    _call("gbmv", _type_code(t), int(trans), M, N, KL, KU, alpha, a.ptr, a.ld, vx.ptr, vx.inc, beta, vy.ptr, vy.inc)
    return y


def sbmv(A, x, K, uplo="L", alpha=1.0, beta=0.0, y=None):
    """y = alpha·A·x + beta·y, A symmetric banded (array (n, K + 1), the uplo triangle)."""
    _session()
    t = _compute_type(A)
    a = _band(A, t, K + 1)
    vx = _vector(x, t)
    y, beta = _new_or_given(y, a.rows, t, beta)
    vy = _vector(y, t, out=True)
    if vx.n != a.rows or vy.n != a.rows:
        raise ValueError("lengths of x, y")
    _call("sbmv", _type_code(t), _UPLO[uplo], a.rows, K, alpha, a.ptr, a.ld, vx.ptr, vx.inc, beta, vy.ptr, vy.inc)
    return y


def _triangular_band(name, A, x, K, uplo, trans, diag):
    _session()
    t = _compute_type(x)
    a = _band(A, t, K + 1)
    vx = _vector(x, t, out=True)
    _call(name, _type_code(t), _UPLO[uplo], int(trans), int(diag), a.rows, K, a.ptr, a.ld, vx.ptr, vx.inc)
    return x


def tbmv(A, x, K, uplo="L", trans=False, diag=False):
    """x = op(A)·x (in place), A triangular banded (array (n, K + 1))."""
    return _triangular_band("tbmv", A, x, K, uplo, trans, diag)


def tbsv(A, x, K, uplo="L", trans=False, diag=False):
    """Solves op(A)·z = x (in place), A triangular banded (array (n, K + 1))."""
    return _triangular_band("tbsv", A, x, K, uplo, trans, diag)


def spmv(Ap, x, uplo="L", alpha=1.0, beta=0.0, y=None):
    """y = alpha·A·x + beta·y, A symmetric packed (vector of n(n+1)/2)."""
    _session()
    t = _compute_type(Ap)
    vx = _vector(x, t)
    ap = _packed_triangle(Ap, t, vx.n)
    y, beta = _new_or_given(y, vx.n, t, beta)
    vy = _vector(y, t, out=True)
    _call("spmv", _type_code(t), _UPLO[uplo], vx.n, alpha, ap.ptr, vx.ptr, vx.inc, beta, vy.ptr, vy.inc)
    return y


def _triangular_packed(name, Ap, x, uplo, trans, diag):
    _session()
    t = _compute_type(x)
    vx = _vector(x, t, out=True)
    ap = _packed_triangle(Ap, t, vx.n)
    _call(name, _type_code(t), _UPLO[uplo], int(trans), int(diag), vx.n, ap.ptr, vx.ptr, vx.inc)
    return x


def tpmv(Ap, x, uplo="L", trans=False, diag=False):
    """x = op(A)·x (in place), A triangular packed."""
    return _triangular_packed("tpmv", Ap, x, uplo, trans, diag)


def tpsv(Ap, x, uplo="L", trans=False, diag=False):
    """Solves op(A)·z = x (in place), A triangular packed."""
    return _triangular_packed("tpsv", Ap, x, uplo, trans, diag)


def spr(alpha, x, Ap, uplo="L"):
    """A = alpha·x·xᵀ + A (packed, in place)."""
    _session()
    t = _compute_type(Ap)
    vx = _vector(x, t)
    ap = _packed_triangle(Ap, t, vx.n, out=True)
    _call("spr", _type_code(t), _UPLO[uplo], vx.n, alpha, vx.ptr, vx.inc, ap.ptr)
    return Ap


def spr2(alpha, x, y, Ap, uplo="L"):
    """A = alpha·(x·yᵀ + y·xᵀ) + A (packed, in place)."""
    _session()
    t = _compute_type(Ap)
    vx, vy = _vector(x, t), _vector(y, t)
    ap = _packed_triangle(Ap, t, vx.n, out=True)
    _call("spr2", _type_code(t), _UPLO[uplo], vx.n, alpha, vx.ptr, vx.inc, vy.ptr, vy.inc, ap.ptr)
    return Ap


# ------------------------------------------------------------------------------------------------ constant weights
class PackedB:
    """op(B) packed once into GPU memory (gen9blas_pack_b, lib/gen9blas.h:89-97), multiplied many times. B: a (K, N)
    matrix, or with transB=True the (N, K) weight matrix (W[N][K] as ggml and most checkpoints store it); a transposed
    view is read in place. B may be changed or freed afterwards. The device memory is released by free() (or when the
    object is collected)."""

    def __init__(self, B, transB=False, accurate=False):
        _session()
        dt = _compute_type(B)
        b = _matrix(B, dt)
        tB = int(transB) ^ b.trans           # stored rows × cols: op(B) = stored (tB = 0) or its transpose (tB = 1)
        self.K, self.N = (b.cols, b.rows) if tB else (b.rows, b.cols)
        self.dtype, self.type = dt, _type_code(dt, accurate)
        self._p = _fn["pack_b"](self.type, tB, self.K, self.N, b.ptr, b.ld)
        if not self._p:
            raise RuntimeError(_error_text())

    def free(self):
        if getattr(self, "_p", None):
            _fn["packed_b_free"](self._p)
            self._p = None

    def __del__(self):
        self.free()

    def _live(self):
        if not self._p:
            raise ValueError("packed B was freed")

    def gemm(self, A, alpha=1.0, beta=0.0, C=None):
        """C = alpha·A·op(B) + beta·C (A: M × K of the packed type; an A.T view is read in place)."""
        self._live()
        a = _matrix(A, self.dtype)
        M, K = (a.cols, a.rows) if a.trans else (a.rows, a.cols)
        if K != self.K:
            raise ValueError(f"A has {K} columns, the packed B {self.K} rows")
        C, given, ldc = _result(C, (M, self.N), self.dtype)
        _call("gemm_pb", a.trans, M, alpha, a.ptr, a.ld, self._p, beta if given else 0.0, C.ctypes.data, ldc)
        return C

    def skinny(self, A):
        """(C, nonfinite): C = A·op(B) in FP32 for FP32 activations A (1 to 16 rows) and FP16 weights packed with
        accurate=True (gen9blas_gemm_pb_skinny, lib/gen9blas_ml.h:25-28)."""
        self._live()
        A = np.ascontiguousarray(A, dtype=np.float32)
        M, K = A.shape
        if K != self.K:
            raise ValueError(f"A has {K} columns, the packed B {self.K} rows")
        C = np.empty((M, self.N), np.float32)
        flag = _I(0)
        status = _fn["gemm_pb_skinny"](M, A.ctypes.data, K, self._p, C.ctypes.data, self.N, ctypes.byref(flag))
        if status == 1:
            raise ValueError("gemm_pb_skinny takes 1 to 16 rows")
        if status != 0:
            raise RuntimeError(_error_text())
        return C, bool(flag.value)


def pack_b(B, transB=False, accurate=False):
    return PackedB(B, transB, accurate)
