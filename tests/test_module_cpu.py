"""CPU checks of the NumPy module's operand mapping (no GPU call): how array views become (pointer, rows, columns,
ld, trans) for matrices and (pointer, n, inc) for vectors -- the rules of the reference module (lib/gen9blas.py:304-328
for vectors and matrices, 135-136 for the in-place rule of strided rows and transposed views, usage lines 5 and 13) --
and the size classes of the managed-memory cache."""
import numpy as np
import pytest

import gen9blas as g


def test_matrix_contiguous_padded_and_transposed_views():
    A = np.zeros((6, 10), np.float32)
    m = g._matrix(A, np.float32)
    assert m.array is A and m.ptr == A.ctypes.data and (m.rows, m.cols, m.ld, m.trans) == (6, 10, 10, 0)
    S = A[:, :7]                                   # strided rows: in place, ld from the row stride
    m = g._matrix(S, np.float32)
    assert m.array is S and m.ptr == A.ctypes.data and (m.rows, m.cols, m.ld, m.trans) == (6, 7, 10, 0)
    T = A.T                                        # transposed view: in place, trans = 1, stored shape 6 × 10
    m = g._matrix(T, np.float32)
    assert m.array is T and m.ptr == A.ctypes.data and (m.rows, m.cols, m.ld, m.trans) == (6, 10, 10, 1)
    R = A[::2]                                     # every other row: ld doubles
    m = g._matrix(R, np.float32)
    assert m.ptr == A.ctypes.data and (m.rows, m.cols, m.ld, m.trans) == (3, 10, 20, 0)


def test_matrix_copies_what_it_cannot_address():
    A = np.arange(60, dtype=np.float32).reshape(6, 10)
    m = g._matrix(A[:, ::2], np.float32)           # column stride 2: a contiguous copy
    assert m.array.flags.c_contiguous and (m.rows, m.cols, m.ld, m.trans) == (6, 5, 5, 0)
    assert np.array_equal(m.array, A[:, ::2])
    m = g._matrix(A, np.float64)                   # other type: converted copy
    assert m.array.dtype == np.float64 and (m.rows, m.cols, m.ld, m.trans) == (6, 10, 10, 0)
    with pytest.raises(TypeError):
        g._matrix(A.T, np.float32, out=True)       # a result must have contiguous rows
    with pytest.raises(TypeError):
        g._matrix(A, np.float16, out=True)
    with pytest.raises(ValueError):
        g._matrix(A[0], np.float32)


def test_vector_increments():
    x = np.arange(10, dtype=np.float64)
    v = g._vector(x, np.float64)
    assert v.array is x and v.ptr == x.ctypes.data and (v.n, v.inc) == (10, 1)
    v = g._vector(x[::3], np.float64)
    assert v.ptr == x.ctypes.data and (v.n, v.inc) == (4, 3)
    v = g._vector(x[::-2], np.float64)             # negative increment: pointer to the lowest address, as in BLAS
    assert (v.n, v.inc) == (5, -2) and v.ptr == x.ctypes.data + 1 * 8
    b = np.broadcast_to(np.float64(1.0), (4,))     # stride 0 is not a BLAS vector: copied
    v = g._vector(b, np.float64)
    assert v.array.flags.c_contiguous and (v.n, v.inc) == (4, 1)
    with pytest.raises(TypeError):
        g._vector(b, np.float64, out=True)
    with pytest.raises(TypeError):
        g._vector(x, np.float32, out=True)
    with pytest.raises(ValueError):
        g._vector(np.zeros((2, 2)), np.float64)


def test_square_transposed_view_flips_the_triangle():
    A = np.zeros((5, 8), np.float32)[:, :5]
    m, uplo = g._square(A, np.float32, "L")
    assert (m.rows, m.ld, m.trans, uplo) == (5, 8, 0, "L")
    m, uplo = g._square(A.T, np.float32, "L")
    assert (m.rows, m.ld, m.trans, uplo) == (5, 8, 1, "U")
    with pytest.raises(ValueError):
        g._square(np.zeros((3, 4), np.float32), np.float32, "L")


def test_type_codes_compute_types_and_supplied_results():
    assert g._type_code(np.float32) == g.GEN9BLAS_S and g._type_code(np.float64, True) == g.GEN9BLAS_D
    assert g._type_code(np.float16) == g.GEN9BLAS_H and g._type_code(np.float16, True) == g.GEN9BLAS_HS
    with pytest.raises(TypeError):
        g._type_code(np.int32)
    assert g._compute_type(np.zeros(2, np.int64)) == np.float32 and g._compute_type(np.zeros(2, np.float16)) == np.float16
    C = np.zeros((4, 9), np.float32)
    c, given, ldc = g._result(C[:, :6], (4, 6), np.float32)   # supplied C with padded rows: written in place
    assert given and ldc == 9
    with pytest.raises(ValueError):
        g._result(C, (4, 6), np.float32)
    with pytest.raises(ValueError):
        g._result(C.astype(np.float64), (4, 9), np.float32)
    with pytest.raises(ValueError):
        g._result(np.zeros((2, 4, 9), np.float32)[:, :, :6], (2, 4, 6), np.float32)   # a batch must be contiguous


def test_managed_cache_size_classes():
    sc = g._ManagedCache.size_class
    assert sc(1) == 1 << 16 and sc(65536) == 1 << 16 and sc(65537) == 1 << 17 and sc(3 << 20) == 4 << 20
