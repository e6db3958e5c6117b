"""GPU parity of the skinny GEMM (min(M, N) <= 16): the cases of the reference's lib/test_skinny.py:43-63 (both weight
layouts, transposes, small-N role swap, alpha/beta with C as a slice, M around the tiles, K tails) with its error
metric max|C − ref| / max|ref| (4e-3 FP16, 2e-6 FP32), plus the 7B decoder shapes of BASELINE configs[2]."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
TOL = {np.float16: 4e-3, np.float32: 2e-6}
rng = np.random.default_rng(7)


def tab(g9, shape, dt, usm):
    X = g9.empty(shape, dt) if usm else np.empty(shape, dt)
    X[...] = rng.uniform(-1, 1, shape).astype(dt)
    return X


def err(result, ref):
    return float(np.max(np.abs(result.astype(np.float64) - ref)) / max(1e-30, np.max(np.abs(ref))))


@pytest.mark.parametrize("dt", [np.float16, np.float32])
@pytest.mark.parametrize("usm", [True, False])
def test_reference_skinny_cases(g9, dt, usm):
    fn = g9.hgemm if dt == np.float16 else g9.sgemm
    for M, N, K in [(1, 1000, 777), (3, 517, 1029), (4, 2048, 128), (5, 64, 9), (8, 333, 4096), (9, 1500, 1500),
                    (16, 4096, 1000), (17, 130, 257), (1, 8, 3), (2, 7, 2000), (16, 16, 16)]:
        for tA in (False, True):
            for tB in (False, True):
                A = tab(g9, (K, M), dt, usm).T if tA else tab(g9, (M, K), dt, usm)
                B = tab(g9, (N, K), dt, usm).T if tB else tab(g9, (K, N), dt, usm)
                Ad, Bd = A.astype(np.float64), B.astype(np.float64)
                desc = f"M={M} N={N} K={K} tA={tA} tB={tB}"
                assert err(fn(A, B), Ad @ Bd) <= TOL[dt], desc
                assert err(fn(B.T, A.T), Bd.T @ Ad.T) <= TOL[dt], desc + " (small N)"
        A = tab(g9, (M, K), dt, usm)
        W = tab(g9, (N, K), dt, usm)
        big = tab(g9, (M + 2, N + 5), dt, usm)
        C = big[1:M + 1, 2:N + 2]
        C0 = C.astype(np.float64)
        D0 = big.copy()
        fn(A, W.T, alpha=0.75, beta=-1.5, C=C)
        assert err(C, 0.75 * A.astype(np.float64) @ W.astype(np.float64).T - 1.5 * C0) <= TOL[dt]
        mask = np.ones(big.shape, bool)
        mask[1:M + 1, 2:N + 2] = False
        assert np.array_equal(big[mask], D0[mask]), "change outside the slice of C"


@pytest.mark.parametrize("M,N,K", [(1, 3000, 2100), (3, 4100, 2056), (8, 2380, 4104), (5, 4736, 2048), (2, 4096, 8),
                                   (4, 9000, 3000), (7, 14000, 2304), (1, 6000, 5000), (9, 3000, 2100),
                                   (16, 4100, 2056), (12, 9000, 4096), (16, 5000, 4096), (9, 4800, 6144),
                                   (13, 11000, 4104)])
def test_whole_blocks_per_cta_plan(g9, M, N, K):
    """At least one 16-row block per SM and K of at least 8 chunks of 256 take the kernel with one row block per CTA
    (one or two token tiles, one or several waves): K off the chunk, edge rows past N, alpha/beta into a slice of C,
    both operand orders (K = 8 stays on the stream-K kernel). The last three leave a partly filled last wave of
    blocks."""
    A = tab(g9, (M, K), np.float16, True)
    W = tab(g9, (N, K), np.float16, True)
    ref = A.astype(np.float64) @ W.astype(np.float64).T
    assert err(g9.hgemm(A, W.T), ref) <= TOL[np.float16], (M, N, K)
    assert err(g9.hgemm(W, A.T), ref.T) <= TOL[np.float16], (M, N, K, "swapped")
    big = tab(g9, (M + 2, N + 5), np.float16, True)
    C = big[1:M + 1, 2:N + 2]
    C0 = C.astype(np.float64)
    g9.hgemm(A, W.T, alpha=0.75, beta=-1.5, C=C)
    assert err(C, 0.75 * ref - 1.5 * C0) <= TOL[np.float16]


@pytest.mark.parametrize("M", [1, 2, 4, 8, 16])
def test_decoder_shapes(g9, M):
    """W FP16 N(0,0.02) of the 7B shapes, A FP16 N(0,1); C = A·Wᵀ."""
    for N, K in ((4096, 4096), (12288, 4096), (11008, 4096), (4096, 11008)):
        W = (rng.standard_normal((N, K)) * 0.02).astype(np.float16)
        A = rng.standard_normal((M, K)).astype(np.float16)
        C = g9.hgemm(A, W.T)
        ref = A.astype(np.float64) @ W.astype(np.float64).T
        assert err(C, ref) <= 4e-3, (M, N, K)


def test_nowait_chain_weights_written_by_previous_call(gpu_lib):
    """No-wait mode: gen9blas_gemm writes W (N × K, FP16) and the next call, a skinny GEMM C = A·Wᵀ, uses W as its
    weights. The skinny kernel may load weights before waiting for the preceding kernel only when no queued call
    writes them, so every round must see the new W. Rounds of fresh data, then gen9blas_flush; FP64 reference."""
    torch = pytest.importorskip("torch")
    g = torch.Generator(device="cuda").manual_seed(17)
    N, K, R, M = 4096, 2048, 256, 4
    X = torch.randn(N, R, device="cuda", generator=g, dtype=torch.float32).mul_(0.1).half()
    Y = torch.randn(R, K, device="cuda", generator=g, dtype=torch.float32).mul_(0.1).half()
    A = torch.randn(M, K, device="cuda", generator=g, dtype=torch.float32).half()
    torch.cuda.synchronize()
    for rnd in range(4):
        W = torch.full((N, K), float("nan"), device="cuda", dtype=torch.float16)
        C = torch.full((M, N), float("nan"), device="cuda", dtype=torch.float16)
        X.mul_(-1.0)   # new weights every round
        torch.cuda.synchronize()
        gpu_lib.set_nowait(1)
        try:
            assert gpu_lib.gemm(0, 0, 0, N, K, R, 1.0, X.data_ptr(), R, Y.data_ptr(), K, 0.0, W.data_ptr(), K) == 0
            assert gpu_lib.gemm(0, 0, 1, M, N, K, 1.0, A.data_ptr(), K, W.data_ptr(), K, 0.0, C.data_ptr(), N) == 0
            assert gpu_lib.flush() == 0, gpu_lib.error()
        finally:
            gpu_lib.set_nowait(0)
        ref = A.double() @ W.double().t()
        assert bool(torch.isfinite(C).all()), rnd
        assert float((C.double() - ref).abs().max() / ref.abs().max()) <= 4e-3, rnd
