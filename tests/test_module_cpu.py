"""CPU checks of the NumPy module's operand mapping (no GPU call): how array views become (pointer, rows, columns,
ld, trans) for matrices and (pointer, n, inc) for vectors, as in the reference module (lib/gen9blas.py:304-328 for
_vec / _mat, 135-136 for the zero-copy rule of strided rows and transposed views, usage lines 5 and 13)."""
import numpy as np
import pytest

import gen9blas as g


def test_mat_contiguous_padded_and_transposed_views():
    A = np.zeros((6, 10), np.float32)
    a, p, r, c, ld, tr = g._mat(A, np.float32)
    assert a is A and p == A.ctypes.data and (r, c, ld, tr) == (6, 10, 10, 0)
    S = A[:, :7]                                   # strided rows: zero copy, ld from the row stride
    a, p, r, c, ld, tr = g._mat(S, np.float32)
    assert a is S and p == A.ctypes.data and (r, c, ld, tr) == (6, 7, 10, 0)
    T = A.T                                        # transposed view: zero copy, trans = 1, stored shape 6 × 10
    a, p, r, c, ld, tr = g._mat(T, np.float32)
    assert a is T and p == A.ctypes.data and (r, c, ld, tr) == (6, 10, 10, 1)
    R = A[::2]                                     # every other row: ld doubles
    a, p, r, c, ld, tr = g._mat(R, np.float32)
    assert p == A.ctypes.data and (r, c, ld, tr) == (3, 10, 20, 0)


def test_mat_copies_what_it_cannot_address():
    A = np.arange(60, dtype=np.float32).reshape(6, 10)
    a, p, r, c, ld, tr = g._mat(A[:, ::2], np.float32)      # column stride 2: a contiguous copy
    assert a.flags.c_contiguous and (r, c, ld, tr) == (6, 5, 5, 0)
    assert np.array_equal(a, A[:, ::2])
    a, p, r, c, ld, tr = g._mat(A, np.float64)              # other type: converted copy
    assert a.dtype == np.float64 and (r, c, ld, tr) == (6, 10, 10, 0)
    with pytest.raises(TypeError):
        g._mat(A.T, np.float32, write=True)                 # a result must have contiguous rows
    with pytest.raises(TypeError):
        g._mat(A, np.float16, write=True)
    with pytest.raises(ValueError):
        g._mat(A[0], np.float32)


def test_vec_increments():
    x = np.arange(10, dtype=np.float64)
    a, p, n, inc = g._vec(x, np.float64)
    assert a is x and p == x.ctypes.data and (n, inc) == (10, 1)
    a, p, n, inc = g._vec(x[::3], np.float64)
    assert p == x.ctypes.data and (n, inc) == (4, 3)
    r = x[::-2]                                    # negative increment: pointer to the lowest address, as in BLAS
    a, p, n, inc = g._vec(r, np.float64)
    assert (n, inc) == (5, -2) and p == x.ctypes.data + 1 * 8
    b = np.broadcast_to(np.float64(1.0), (4,))     # stride 0 is not a BLAS vector: copied
    a, p, n, inc = g._vec(b, np.float64)
    assert a.flags.c_contiguous and (n, inc) == (4, 1)
    with pytest.raises(TypeError):
        g._vec(b, np.float64, write=True)
    with pytest.raises(TypeError):
        g._vec(x, np.float32, write=True)


def test_square_transposed_view_flips_the_triangle():
    A = np.zeros((5, 8), np.float32)[:, :5]
    a, p, n, lda, ta, uplo = g._square(A, np.float32, "L")
    assert (n, lda, ta, uplo) == (5, 8, 0, "L")
    a, p, n, lda, ta, uplo = g._square(A.T, np.float32, "L")
    assert (n, lda, ta, uplo) == (5, 8, 1, "U")
    with pytest.raises(ValueError):
        g._square(np.zeros((3, 4), np.float32), np.float32, "L")


def test_kinds_and_supplied_outputs():
    assert g._kind(np.float32, False) == g.GEN9BLAS_S and g._kind(np.float64, True) == g.GEN9BLAS_D
    assert g._kind(np.float16, False) == g.GEN9BLAS_H and g._kind(np.float16, True) == g.GEN9BLAS_HS
    with pytest.raises(TypeError):
        g._kind(np.int32, False)
    C = np.zeros((4, 9), np.float32)
    c, given, ldc = g._output(C[:, :6], (4, 6), np.float32)   # supplied C with padded rows: written in place
    assert given and ldc == 9
    with pytest.raises(ValueError):
        g._output(C, (4, 6), np.float32)
    with pytest.raises(ValueError):
        g._output(C.astype(np.float64), (4, 9), np.float32)
