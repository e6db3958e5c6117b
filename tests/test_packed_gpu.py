"""GPU parity of the constant-weight API through the C ABI: gen9blas_pack_b / gen9blas_gemm_pb / gen9blas_packed_b_free
and gen9blas_gemm_pb_skinny.

- The cases of the reference's lib/test_packed.py:64-111: transposed and plain B, padding shapes (K off the 16-byte
  vector), alpha / beta, H / HS / D, a weight of 151936 × 1536 FP32 (0.93 GB) with M = 512, and one packed B reused
  with several A after B was zeroed. Error metric and limits of that file (max over sampled rows of
  |C − ref| / (|alpha|·Σ|a·b| + |beta·c0|): H 3e-3, S 1e-6, HS 3e-4, D 1e-14), and the result compared bit for bit
  with gen9blas_gemm on the same data (the same kernels run; only B's pitch differs).
- Small batches through gemm_pb (M up to the skinny threshold), including K off the vector (zero-padded copy of A).
- gemm_pb_skinny on the shapes of lib/test_skinny_pb.py:51-72 (FP32 activations × FP16 weights W[N][K]; max error
  1e-5 of Σ|a·w|, no non-finite flag), rows of extreme magnitude, and the non-finite flag.
"""
import ctypes

import numpy as np
import pytest

import abi

pytestmark = pytest.mark.gpu
H, S, HS, D = abi.H, abi.S, abi.HS, abi.D
DT = {H: np.float16, S: np.float32, HS: np.float16, D: np.float64}
TOL = {H: 3e-3, S: 1e-6, HS: 3e-4, D: 1e-14}   # lib/test_packed.py:28
rng = np.random.default_rng(7)


def pack(L, t, B, transB):
    K, N = (B.shape[1], B.shape[0]) if transB else B.shape
    P = L.pack_b(t, int(transB), K, N, B.ctypes.data, B.shape[1])
    assert P, L.error().decode()
    return P


def gemm_pb(L, A, P, N, dt, alpha=1.0, beta=0.0, C=None, transA=False):
    M = A.shape[1] if transA else A.shape[0]
    if C is None:
        C = np.zeros((M, N), dt)
    rc = L.gemm_pb(int(transA), M, alpha, A.ctypes.data, A.shape[1], P, beta, C.ctypes.data, C.shape[1])
    assert rc == 0, L.error().decode()
    return C


def rel_err(C, A, Bkn, alpha=1.0, beta=0.0, C0=None, rows=None):
    """lib/test_packed.py:51-61: max over sampled rows of |C − ref| / (|alpha|·Σ|a·b| + |beta·c0|)."""
    M = A.shape[0]
    rows = rows if rows is not None else sorted({0, M // 2, M - 1})
    A64, B64 = A[rows].astype(np.float64), Bkn.astype(np.float64)
    ref = alpha * (A64 @ B64)
    mag = abs(alpha) * (np.abs(A64) @ np.abs(B64))
    if C0 is not None and beta != 0:
        ref += beta * C0[rows].astype(np.float64)
        mag += abs(beta) * np.abs(C0[rows].astype(np.float64))
    return float(np.max(np.abs(C[rows].astype(np.float64) - ref) / np.maximum(mag, 1e-30)))


CASES = [  # (name, type, M, N, K, transB, alpha, beta): lib/test_packed.py:88-97
    ("S 512x1536x1536 transB", S, 512, 1536, 1536, 1, 1.0, 0.0),
    ("S 512x256x1536 transB (K/V)", S, 512, 256, 1536, 1, 1.0, 0.0),
    ("S 512x8960x1536 transB (gate/up)", S, 512, 8960, 1536, 1, 1.0, 0.0),
    ("S 512x1536x8960 transB (down)", S, 512, 1536, 8960, 1, 1.0, 0.0),
    ("S 33x100x2051 transB (padding)", S, 33, 100, 2051, 1, 1.0, 0.0),
    ("S 37x1000x300 plain B", S, 37, 1000, 300, 0, 1.0, 0.0),
    ("S 64x1536x1536 alpha 0.5 beta -2", S, 64, 1536, 1536, 1, 0.5, -2.0),
    ("H 256x1024x1024 transB", H, 256, 1024, 1024, 1, 1.0, 0.0),
    ("HS 256x1024x2048 transB", HS, 256, 1024, 2048, 1, 1.0, 0.0),
    ("D 64x512x512 transB", D, 64, 512, 512, 1, 1.0, 0.0),
    # beyond the reference's list: plain B from host memory in several 64 MiB bands, FP16 / FP64 padding
    ("S 64x4096x8192 plain B (bands)", S, 64, 4096, 8192, 0, 1.0, 0.0),
    ("HS 200x300x1001 plain B (padding)", HS, 200, 300, 1001, 0, 1.5, 0.5),
    ("D 130x70x99 transB (padding)", D, 130, 70, 99, 1, 1.0, 1.0),
]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_reference_cases(gpu_lib, case):
    L = gpu_lib
    name, t, M, N, K, transB, alpha, beta = case
    dt = DT[t]
    A = rng.uniform(-1, 1, (M, K)).astype(dt)
    B = rng.uniform(-1, 1, (N, K) if transB else (K, N)).astype(dt)
    Bkn = B.T if transB else B
    C0 = rng.uniform(-1, 1, (M, N)).astype(dt)
    P = pack(L, t, B, transB)
    try:
        C = gemm_pb(L, A, P, N, dt, alpha, beta, C0.copy())
        e = rel_err(C, A, Bkn, alpha, beta, C0)
        assert e <= TOL[t] and np.all(np.isfinite(C)), (name, e)
        C2 = C0.copy()
        assert L.gemm(t, 0, transB, M, N, K, alpha, A.ctypes.data, K, B.ctypes.data, B.shape[1], beta,
                      C2.ctypes.data, N) == 0
        assert np.array_equal(C, C2), (name, "differs from gen9blas_gemm")
    finally:
        L.packed_b_free(P)


def test_reuse_after_b_changed(gpu_lib):
    """lib/test_packed.py:99-111: pack once, overwrite B, multiply with two different A (and the first again)."""
    L = gpu_lib
    A1 = rng.uniform(-1, 1, (128, 1536)).astype(np.float32)
    A2 = rng.uniform(-1, 1, (512, 1536)).astype(np.float32)
    B = rng.uniform(-1, 1, (1536, 1536)).astype(np.float32)
    Bkn = B.T.copy()
    P = pack(L, S, B, 1)
    B[:] = 0.0
    try:
        for A in (A1, A2, A1):
            assert rel_err(gemm_pb(L, A, P, 1536, np.float32), A, Bkn) <= TOL[S]
    finally:
        L.packed_b_free(P)


def test_large_output_projection(gpu_lib):
    """lib/test_packed.py: 151936 × 1536 FP32 weight (Qwen2.5-1.5B's output projection, 0.93 GB) with M = 512."""
    L = gpu_lib
    N, K, M = 151936, 1536, 512
    W = rng.uniform(-1, 1, (N, K)).astype(np.float32)
    A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    P = pack(L, S, W, 1)
    try:
        C = gemm_pb(L, A, P, N, np.float32)
        assert rel_err(C, A, W.T) <= TOL[S]
        assert np.all(np.isfinite(C[::97]))
    finally:
        L.packed_b_free(P)


@pytest.mark.parametrize("t", [H, HS, S, D])
def test_small_batches_and_transposed_a(gpu_lib, t):
    """M up to the skinny threshold through gemm_pb: K on and off the 16-byte vector (zero-padded A), op(A) = Aᵀ,
    and alpha / beta on a C with a wider pitch (the bytes outside the M × N block stay)."""
    L = gpu_lib
    dt = DT[t]
    tol = {H: 3e-3, HS: 3e-4, S: 2e-6, D: 1e-14}[t]
    for N, K in ((1000, 777), (4096, 4096), (37, 96), (300, 1001)):
        W = rng.uniform(-1, 1, (N, K)).astype(dt)
        P = pack(L, t, W, 1)
        try:
            for M in (1, 3, 8, 9, 16, 17):
                A = rng.uniform(-1, 1, (M, K)).astype(dt)
                C = gemm_pb(L, A, P, N, dt)
                assert rel_err(C, A, W.T, rows=list(range(M))) <= tol, (N, K, M)
                At = np.ascontiguousarray(A.T)
                C = gemm_pb(L, At, P, N, dt, transA=True)
                assert rel_err(C, A, W.T, rows=list(range(M))) <= tol, (N, K, M, "transA")
                big = rng.uniform(-1, 1, (M, N + 7)).astype(dt)
                keep = big.copy()
                rc = L.gemm_pb(0, M, 0.5, A.ctypes.data, K, P, -1.0, big.ctypes.data, N + 7)
                assert rc == 0, L.error().decode()
                assert rel_err(big[:, :N], A, W.T, 0.5, -1.0, keep[:, :N], rows=list(range(M))) <= tol
                assert np.array_equal(big[:, N:], keep[:, N:])
        finally:
            L.packed_b_free(P)


def test_device_resident_operands_and_nowait(gpu_lib, g9):
    """Managed (gen9blas.empty) B, A and C are used in place: plain B is transposed on the device; with no-wait on,
    gemm_pb only enqueues and gen9blas_flush waits."""
    L = gpu_lib
    K, N, M = 1000, 3000, 300
    B = g9.empty((K, N), np.float16)
    B[...] = rng.uniform(-1, 1, (K, N)).astype(np.float16)
    P = pack(L, HS, B, 0)
    try:
        A = g9.empty((M, K), np.float16)
        A[...] = rng.uniform(-1, 1, (M, K)).astype(np.float16)
        C = g9.empty((M, N), np.float16)
        C[...] = 0
        L.set_nowait(1)
        try:
            assert L.gemm_pb(0, M, 1.0, A.ctypes.data, K, P, 0.0, C.ctypes.data, N) == 0
            assert L.flush() == 0
        finally:
            L.set_nowait(0)
        assert L.last_zero_copy() == 7
        assert rel_err(C, A, B) <= TOL[HS]
    finally:
        L.packed_b_free(P)


def skinny_pb(L, M, A, P, N):
    C = np.full((M, N), np.nan, np.float32)
    nf = ctypes.c_int(0)
    rc = L.gemm_pb_skinny(M, A.ctypes.data, A.shape[1], P, C.ctypes.data, N, ctypes.byref(nf))
    assert rc == 0, f"rc {rc}: {L.error().decode()}"
    return C, nf.value


@pytest.mark.parametrize("N,K", [(1024, 1024), (256, 1024), (3072, 1024), (1024, 3072), (1000, 1000), (37, 96),
                                 (3072, 2048), (4100, 2600)])
def test_gemm_pb_skinny(gpu_lib, N, K):
    """lib/test_skinny_pb.py:51-66: W[N][K] FP16 (N(0, 0.05)) packed as HS with transB = 1, A F32 N(0, 1). The last two
    shapes (at least one 16-row block per SM, K of at least 2048) take the kernel with one row block per CTA."""
    L = gpu_lib
    rs = np.random.default_rng(11)
    W = (rs.standard_normal((N, K)) * 0.05).astype(np.float16)
    P = pack(L, HS, W, 1)
    W64 = W.astype(np.float64)
    try:
        for M in (1, 2, 3, 4, 5, 8, 9, 12, 16):
            A = rs.standard_normal((M, K)).astype(np.float32)
            C, nf = skinny_pb(L, M, A, P, N)
            ref = A.astype(np.float64) @ W64.T
            mag = np.abs(A.astype(np.float64)) @ np.abs(W64.T)
            e = float(np.max(np.abs(C - ref) / mag))
            assert e < 1e-5 and nf == 0 and np.isfinite(C).all(), (N, K, M, e, nf)
    finally:
        L.packed_b_free(P)


@pytest.mark.parametrize("N,K,M", [(512, 640, 6), (3000, 2048, 6), (3000, 2304, 12)])
def test_gemm_pb_skinny_scaling_and_nonfinite(gpu_lib, N, K, M):
    """Rows of 1e-30 and 1e30 magnitude keep full accuracy (per-row power-of-two scaling of the FP16 parts); an inf
    in one row flags the call and leaves the other rows exact (stream-K kernel, then the one-block-per-CTA kernel
    with paired and with split token parts)."""
    L = gpu_lib
    W = (rng.standard_normal((N, K)) * 0.05).astype(np.float16)
    P = pack(L, HS, W, 1)
    W64 = W.astype(np.float64)
    try:
        A = rng.standard_normal((M, K)).astype(np.float32)
        A[1] *= 1e-30
        A[2] *= 1e30
        A[3] *= 3e-3
        C, nf = skinny_pb(L, M, A, P, N)
        ref = A.astype(np.float64) @ W64.T
        mag = np.abs(A.astype(np.float64)) @ np.abs(W64.T)
        assert nf == 0 and float(np.max(np.abs(C - ref) / mag)) < 1e-5
        A[4, 17] = np.inf
        C, nf = skinny_pb(L, M, A, P, N)
        assert nf == 1
        assert not np.isfinite(C[4]).all()
        rows = [0, 1, 2, 3, 5]
        assert float(np.max(np.abs(C[rows] - ref[rows]) / mag[rows])) < 1e-5
    finally:
        L.packed_b_free(P)
