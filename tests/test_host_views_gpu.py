"""Plain NumPy arrays (host memory, staged through device buffers) in the cases of the reference's
lib/test_userptr.py:4-12: data changed by the CPU between calls, several views of one array as different operands
(two written vectors interleaved in the same memory: swap / rot of x[0::2] and x[1::2]), and in-place results on
strided views, whose neighbouring elements must stay untouched."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dt", [np.float32, np.float64])
def test_interleaved_written_views(g9, dt):
    rng = np.random.default_rng(5)
    n = 20001
    buf = rng.uniform(-1, 1, 2 * n).astype(dt)
    ev, od = buf[0::2].copy(), buf[1::2].copy()
    g9.swap(buf[0::2], buf[1::2])
    assert np.array_equal(buf[0::2], od) and np.array_equal(buf[1::2], ev)
    c, s = 0.6, 0.8
    x0, y0 = buf[0::2].astype(np.float64), buf[1::2].astype(np.float64)
    g9.rot(buf[0::2], buf[1::2], c, s)
    tol = 1e-6 if dt == np.float32 else 1e-14
    assert np.abs(buf[0::2] - (c * x0 + s * y0)).max() <= tol
    assert np.abs(buf[1::2] - (c * y0 - s * x0)).max() <= tol
    b3 = rng.uniform(-1, 1, 3 * n).astype(dt)       # interleaved with a gap: x[0::3], x[1::3] written, x[2::3] not
    keep = b3[2::3].copy()
    a0, a1 = b3[0::3].copy(), b3[1::3].copy()
    g9.swap(b3[0::3], b3[1::3])
    assert np.array_equal(b3[0::3], a1) and np.array_equal(b3[1::3], a0) and np.array_equal(b3[2::3], keep)


@pytest.mark.parametrize("dt", [np.float32, np.float64])
def test_in_place_strided_views_leave_neighbours(g9, dt):
    rng = np.random.default_rng(6)
    n = 30000
    buf = rng.uniform(-1, 1, 3 * n).astype(dt)
    before = buf.copy()
    g9.scal(2.0, buf[1::3])
    assert np.array_equal(buf[1::3], (2.0 * before[1::3].astype(np.float64)).astype(dt))
    assert np.array_equal(buf[0::3], before[0::3]) and np.array_equal(buf[2::3], before[2::3])
    before = buf.copy()
    g9.axpy(0.5, buf[0::3], buf[2::3])              # x read, y written, interleaved in the same array
    tol = 1e-6 if dt == np.float32 else 1e-14
    assert np.abs(buf[2::3] - (before[2::3].astype(np.float64) + 0.5 * before[0::3])).max() <= tol
    assert np.array_equal(buf[0::3], before[0::3]) and np.array_equal(buf[1::3], before[1::3])


def test_cpu_changes_between_calls(g9):
    rng = np.random.default_rng(7)
    A = rng.uniform(-1, 1, (300, 200)).astype(np.float32)
    B = rng.uniform(-1, 1, (200, 100)).astype(np.float32)
    C = np.zeros((300, 100), np.float32)
    for r in range(4):
        A[r::7] += 1.0
        B[:, r] *= -2
        g9.sgemm(A, B, C=C)
        ref = A.astype(np.float64) @ B.astype(np.float64)
        assert np.abs(C - ref).max() / np.abs(ref).max() <= 1e-5
    W = g9.sgemm(A, A.T)                              # one array as both operands (a transposed view)
    ref = A.astype(np.float64) @ A.T.astype(np.float64)
    assert np.abs(W - ref).max() / np.abs(ref).max() <= 1e-5
