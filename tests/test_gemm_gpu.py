"""GPU parity of dense GEMM (tcgen05 HGEMM fast/accurate, FFMA SGEMM, FP64 DGEMM) with the cases and error metric of
the reference's lib/test_basic.py:4-79 (sizes, alpha/beta, all four transposes, managed vs plain unaligned memory),
lib/test_level3.py:48-53 (batched) and lib/test_long_launch.py (large sizes, sampled rows), against FP64 NumPy on the
same FP16/FP32/FP64-rounded inputs and against the CPU oracle."""
import ctypes

import numpy as np
import pytest

import abi
import make_golden as mg
from conftest import ROOT, gemm_error

pytestmark = pytest.mark.gpu

# (name, dtype, accurate, mean limit, max limit): reference limits (test_basic.py:5-8, test_level3.py:5) with the
# maximum tightened to the build's targets (HGEMM fast 1e-3).
KINDS = [("hgemm", np.float16, False, 4.9e-4, 1e-3), ("hgemm acc.", np.float16, True, 4.9e-4, 1e-3),
         ("sgemm", np.float32, False, 1e-6, 1e-5), ("dgemm", np.float64, False, 1e-14, 1e-13)]
SIZES = [(1, 1, 1, 1, 0), (17, 33, 15, 1, 0), (100, 70, 300, 2.0, 0), (64, 96, 48, 0.5, 1.0),
         (333, 129, 1000, 1, -1.0), (1000, 1024, 777, 1, 0.5)]


def new_array(g9, shape, dt, zc):
    """zc=1: gen9blas.empty (managed memory, used in place); zc=0: plain NumPy array, deliberately unaligned."""
    if zc:
        return g9.empty(shape, dt)
    t = np.zeros(shape[0] * shape[1] + 64, dt)
    off = 32 if (t.ctypes.data % 4096) == 0 else 0
    return t[off:off + shape[0] * shape[1]].reshape(shape)


def case(g9, dt, accurate, M, N, K, al, be, ta, tb, zc, seed=0):
    rng = np.random.default_rng(seed)
    a = new_array(g9, (K, M) if ta else (M, K), dt, zc)
    a[...] = rng.uniform(-1, 1, a.shape)
    b = new_array(g9, (N, K) if tb else (K, N), dt, zc)
    b[...] = rng.uniform(-1, 1, b.shape)
    A, B = (a.T if ta else a), (b.T if tb else b)
    C0 = rng.uniform(-1, 1, (M, N)).astype(dt)
    C = new_array(g9, (M, N), dt, zc)
    C[...] = C0 if be else 0
    W = g9.gemm(A, B, al, be, C, accurate=accurate)
    a64, b64 = A.astype(np.float64), B.astype(np.float64)
    ref = al * a64 @ b64 + (be * C0.astype(np.float64) if be else 0)
    scale = abs(al) * np.abs(a64) @ np.abs(b64) + (abs(be) * np.abs(C0.astype(np.float64)) if be else 0)
    return gemm_error(W, ref, scale) + (g9.last_zero_copy(),)


@pytest.mark.parametrize("M", [17, 64, 128])
@pytest.mark.parametrize("al,be,ta,tb", [(1.0, 0.0, 0, 0), (0.75, -0.5, 1, 1), (1.0, 0.0, 0, 1)])
def test_hgemm_accurate_small_m_split_k(g9, M, al, be, ta, tb):
    """FP32-accumulating HGEMM with M <= 128 and few column tiles (N = 4096: 16 tiles of 256) splits K over the idle
    SMs: FP32 parts summed in part order by a second kernel, which applies alpha / beta and the FP16 rounding. The
    reference's accurate-mode limits (mean 1e-4, max 1e-3 of the |A|·|B| scale)."""
    avg, mx, _ = case(g9, np.float16, True, M, 4096, 4096, al, be, ta, tb, 0, seed=M)
    assert avg <= 1e-4 and mx <= 1e-3, (M, al, be, ta, tb, avg, mx)
    avg, mx, _ = case(g9, np.float16, True, M, 1000, 2050, al, be, ta, tb, 1, seed=M + 1)   # ragged N and K
    assert avg <= 1e-4 and mx <= 1e-3, (M, al, be, ta, tb, avg, mx)


@pytest.mark.parametrize("name,dt,accurate,tol_avg,tol_max", KINDS)
def test_reference_cases(g9, name, dt, accurate, tol_avg, tol_max):
    worst = []
    for (M, N, K, al, be) in SIZES:
        for ta, tb in [(0, 0), (1, 0), (0, 1), (1, 1)]:
            for zc in (0, 1):
                avg, mx, z = case(g9, dt, accurate, M, N, K, al, be, ta, tb, zc)
                if accurate and K >= 256:
                    ok = avg <= 1e-4 and mx <= 1e-3
                else:
                    ok = avg <= tol_avg and mx <= tol_max
                assert ok, f"{name} M={M} N={N} K={K} a={al} b={be} tA={ta} tB={tb} zc={zc}: avg {avg:.2e} max {mx:.2e}"
                assert z == (7 if zc else 0), z
                worst.append(mx)
    print(f"{name}: worst max error {max(worst):.2e}")


@pytest.mark.parametrize("t,dt", [(abi.S, np.float32), (abi.D, np.float64)])
def test_close_to_oracle(gpu_lib, oracle, t, dt):
    """FP32/FP64 results next to the oracle's FMA chain (same products, different summation order)."""
    rng = np.random.default_rng(5)
    for (M, N, K, ta, tb) in ((131, 67, 200, 0, 0), (64, 160, 33, 1, 1), (250, 130, 129, 0, 1)):
        A = rng.uniform(-1, 1, (K, M) if ta else (M, K)).astype(dt)
        B = rng.uniform(-1, 1, (N, K) if tb else (K, N)).astype(dt)
        C0 = rng.uniform(-1, 1, (M, N)).astype(dt)
        Cg, Co = C0.copy(), C0.copy()
        args = (t, ta, tb, M, N, K, 0.75, A.ctypes.data, A.shape[1], B.ctypes.data, B.shape[1], -0.5)
        assert gpu_lib.gemm(*args, Cg.ctypes.data, N) == 0
        assert oracle.gemm(*args, Co.ctypes.data, N) == 0
        a64 = (A.T if ta else A).astype(np.float64)
        b64 = (B.T if tb else B).astype(np.float64)
        scale = 0.75 * np.abs(a64) @ np.abs(b64) + 0.5 * np.abs(C0.astype(np.float64))
        assert (np.abs(Cg.astype(np.float64) - Co) / scale).max() <= (2e-6 if t == abi.S else 2e-13)


@pytest.mark.parametrize("t,dt", [(abi.H, np.float16), (abi.HS, np.float16), (abi.S, np.float32), (abi.D, np.float64)])
def test_beta_zero_ignores_c_and_slice_untouched(gpu_lib, t, dt):
    """beta = 0 never reads C (NaN there stays out of the result, sgemm.cl:196 / level12.cl:280 semantics), and a C
    that is a slice of a larger array leaves everything outside the slice unchanged."""
    rng = np.random.default_rng(9)
    for (M, N, K) in ((5, 300, 70), (200, 300, 64), (129, 257, 40)):
        A = rng.uniform(-1, 1, (M, K)).astype(dt)
        B = rng.uniform(-1, 1, (K, N)).astype(dt)
        big = np.full((M + 3, N + 11), np.nan, dt)
        C = big[1:M + 1, 3:N + 3]
        outside = np.ones(big.shape, bool)
        outside[1:M + 1, 3:N + 3] = False
        assert gpu_lib.gemm(t, 0, 0, M, N, K, 1.0, A.ctypes.data, K, B.ctypes.data, N, 0.0,
                            C.ctypes.data, big.shape[1]) == 0
        assert np.isfinite(C).all()
        assert np.isnan(big[outside]).all()
        ref = A.astype(np.float64) @ B.astype(np.float64)
        scale = np.abs(A.astype(np.float64)) @ np.abs(B.astype(np.float64))
        assert gemm_error(C, ref, scale)[1] <= (1e-3 if dt == np.float16 else 1e-5)


@pytest.mark.parametrize("name,dt,accurate,tol_avg,tol_max", KINDS)
def test_batched(g9, name, dt, accurate, tol_avg, tol_max):
    rng = np.random.default_rng(3)
    for cnt, M, N, K in ((1, 96, 112, 80), (7, 64, 40, 100), (33, 17, 33, 65)):
        A = rng.uniform(-1, 1, (cnt, M, K)).astype(dt)
        B = rng.uniform(-1, 1, (cnt, K, N)).astype(dt)
        C0 = rng.uniform(-1, 1, (cnt, M, N)).astype(dt)
        C = C0.copy()
        g9.gemm_batched(A, B, 1.5, 0.5, C, accurate=accurate)
        a64, b64, c64 = A.astype(np.float64), B.astype(np.float64), C0.astype(np.float64)
        ref = 1.5 * a64 @ b64 + 0.5 * c64
        scale = 1.5 * np.abs(a64) @ np.abs(b64) + 0.5 * np.abs(c64)
        avg, mx = gemm_error(C, ref, scale)
        assert avg <= tol_avg and mx <= tol_max, (name, cnt, avg, mx)


def test_hgemm_unaligned_leading_dimensions(gpu_lib):
    """Leading dimensions that are not multiples of 8 FP16 elements (TMA needs 16-byte pitches): repack path."""
    rng = np.random.default_rng(4)
    for t in (abi.H, abi.HS):
        for (M, N, K, lda, ldb, ldc, ta, tb) in ((70, 90, 45, 47, 93, 91, 0, 0), (33, 40, 17, 35, 19, 41, 1, 1),
                                                  (129, 257, 65, 67, 261, 259, 0, 1)):
            A = rng.uniform(-1, 1, ((K if ta else M), lda)).astype(np.float16)
            B = rng.uniform(-1, 1, ((N if tb else K), ldb)).astype(np.float16)
            C = np.zeros((M, ldc), np.float16)
            assert gpu_lib.gemm(t, ta, tb, M, N, K, 1.0, A.ctypes.data, lda, B.ctypes.data, ldb, 0.0,
                                C.ctypes.data, ldc) == 0
            a64 = (A[:, :M].T if ta else A[:, :K]).astype(np.float64)
            b64 = (B[:, :K].T if tb else B[:, :N]).astype(np.float64)
            ref = a64 @ b64
            avg, mx = gemm_error(C[:, :N], ref, np.abs(a64) @ np.abs(b64))
            assert mx <= 1e-3, (t, M, N, K, mx)
            assert not C[:, N:].any()


@pytest.mark.parametrize("accurate,limit", [(False, 1e-3), (True, 1e-4)])
def test_hgemm_headline_config(g9, accurate, limit):
    """n = 4096, A, B iid N(0,1)/sqrt(n) in FP16, C = A·B; north-star limits on the max error
    (fast 1e-3, accurate 1e-4), checked on 256 sampled rows against FP64."""
    n = 4096
    rng = np.random.default_rng(1)
    A = (rng.standard_normal((n, n)) / np.sqrt(n)).astype(np.float16)
    B = (rng.standard_normal((n, n)) / np.sqrt(n)).astype(np.float16)
    C = g9.hgemm(A, B, accurate=accurate)
    rows = rng.choice(n, 256, replace=False)
    a64, b64 = A[rows].astype(np.float64), B.astype(np.float64)
    avg, mx = gemm_error(C[rows], a64 @ b64, np.abs(a64) @ np.abs(b64))
    print(f"hgemm n=4096 accurate={accurate}: mean {avg:.2e} max {mx:.2e}")
    assert mx <= limit


@pytest.mark.parametrize("name,dt,accurate,tol_avg,tol_max", KINDS)
def test_large_sampled_rows(g9, name, dt, accurate, tol_avg, tol_max):
    """Long launches (lib/test_long_launch.py): n = 8192 (FP64: 4096), rows sampled against FP64."""
    n = 4096 if dt == np.float64 else 8192
    rng = np.random.default_rng(2)
    A = rng.uniform(-1, 1, (n, n)).astype(dt)
    B = rng.uniform(-1, 1, (n, n)).astype(dt)
    C = g9.gemm(A, B, accurate=accurate)
    rows = rng.choice(n, 64, replace=False)
    a64, b64 = A[rows].astype(np.float64), B.astype(np.float64)
    avg, mx = gemm_error(C[rows], a64 @ b64, np.abs(a64) @ np.abs(b64))
    lim_max = 1e-3 if dt == np.float16 else tol_max
    assert mx <= lim_max and avg <= (1e-4 if accurate else tol_avg), (name, avg, mx)


@pytest.mark.parametrize("t", [abi.H, abi.HS])
def test_hgemm_split_k_tail(gpu_lib, t):
    """Shapes whose last wave of 256×256 tiles -- or only wave, for problems with fewer tiles than CTA pairs -- is
    split along K over idle CTA pairs (2, 3 or 4 parts, uneven K ranges, edge columns, alpha/beta): the finishing part
    adds the other parts' FP32 partial sums."""
    rng = np.random.default_rng(21)
    for (M, N, K, al, be) in ((3072, 1792, 1024, 1.0, 0.0), (2304, 2304, 520, 1.5, -0.5), (1000, 5000, 300, 1.0, 1.0),
                              (4096, 4096, 4096, 0.5, 0.25), (1024, 1024, 1024, 1.0, 0.0), (768, 1280, 2048, 1.5, 0.5),
                              (1536, 1536, 640, 1.0, -1.0)):
        A = (rng.standard_normal((M, K)) / np.sqrt(K)).astype(np.float16)
        B = (rng.standard_normal((K, N)) / np.sqrt(K)).astype(np.float16)
        C0 = rng.uniform(-1, 1, (M, N)).astype(np.float16)
        C = C0.copy()
        for _ in range(2):   # twice: the handoff flags carry a per-launch epoch
            C[...] = C0
            assert gpu_lib.gemm(t, 0, 0, M, N, K, al, A.ctypes.data, K, B.ctypes.data, N, be, C.ctypes.data, N) == 0
            rows = np.concatenate([np.arange(0, M, max(1, M // 97)), [M - 1]])
            a64, b64 = A[rows].astype(np.float64), B.astype(np.float64)
            ref = al * a64 @ b64 + be * C0[rows].astype(np.float64)
            scale = abs(al) * np.abs(a64) @ np.abs(b64) + abs(be) * np.abs(C0[rows].astype(np.float64))
            avg, mx = gemm_error(C[rows], ref, scale)
            assert mx <= 1e-3, (t, M, N, K, mx)


def test_sgemm_large_grid_all_layouts(gpu_lib):
    """SGEMM on a grid of more than two waves: all four transposes, pitches that are and are not multiples of 4 floats
    (16-byte and 4-byte copy paths), ragged M, N, K, alpha / beta, bytes past N untouched."""
    rng = np.random.default_rng(37)
    M, N, K = 2200, 4100, 333
    for ta in (0, 1):
        for tb in (0, 1):
            for pad in (0, 1):
                ra, ca = (K, M) if ta else (M, K)
                rb, cb = (N, K) if tb else (K, N)
                lda, ldb, ldc = ca + pad, cb + pad, N + 3
                A = rng.uniform(-1, 1, (ra, lda)).astype(np.float32)
                B = rng.uniform(-1, 1, (rb, ldb)).astype(np.float32)
                C0 = rng.uniform(-1, 1, (M, ldc)).astype(np.float32)
                C = C0.copy()
                assert gpu_lib.gemm(abi.S, ta, tb, M, N, K, 1.5, A.ctypes.data, lda, B.ctypes.data, ldb, 0.5,
                                    C.ctypes.data, ldc) == 0
                a64 = (A[:, :ca].T if ta else A[:, :ca]).astype(np.float64)
                b64 = (B[:, :cb].T if tb else B[:, :cb]).astype(np.float64)
                rows = np.concatenate([np.arange(0, M, 37), np.arange(M - 130, M)])
                c64 = C0[rows, :N].astype(np.float64)
                ref = 1.5 * a64[rows] @ b64 + 0.5 * c64
                scale = 1.5 * np.abs(a64[rows]) @ np.abs(b64) + 0.5 * np.abs(c64)
                avg, mx = gemm_error(C[rows, :N], ref, scale)
                assert avg <= 1e-6 and mx <= 1e-5, (ta, tb, pad, avg, mx)
                assert (C[:, N:] == C0[:, N:]).all()


def test_sgemm_stream_k_ragged_all_layouts(gpu_lib):
    """SGEMM grids of less than one wave with K >= 256 (the stream-K kernel: tile × K-chunk iterations spread over one
    wave, partial tiles handed over between CTAs): ragged M, N and K (K not a multiple of the chunk), all four
    transposes, pitches that are and are not multiples of 4 floats, alpha / beta, bytes past N untouched; each shape
    twice, so the hand-over flags of a later call carry a new epoch."""
    rng = np.random.default_rng(41)
    for (M, N, K) in ((1000, 900, 1000), (3000, 100, 2001)):
        for ta in (0, 1):
            for tb in (0, 1):
                for pad in (0, 1):
                    ra, ca = (K, M) if ta else (M, K)
                    rb, cb = (N, K) if tb else (K, N)
                    lda, ldb, ldc = ca + pad, cb + pad, N + 3
                    A = rng.uniform(-1, 1, (ra, lda)).astype(np.float32)
                    B = rng.uniform(-1, 1, (rb, ldb)).astype(np.float32)
                    C0 = rng.uniform(-1, 1, (M, ldc)).astype(np.float32)
                    a64 = (A[:, :ca].T if ta else A[:, :ca]).astype(np.float64)
                    b64 = (B[:, :cb].T if tb else B[:, :cb]).astype(np.float64)
                    c64 = C0[:, :N].astype(np.float64)
                    ref = 1.5 * a64 @ b64 + 0.5 * c64
                    scale = 1.5 * np.abs(a64) @ np.abs(b64) + 0.5 * np.abs(c64)
                    for _ in range(2):
                        C = C0.copy()
                        assert gpu_lib.gemm(abi.S, ta, tb, M, N, K, 1.5, A.ctypes.data, lda, B.ctypes.data, ldb, 0.5,
                                            C.ctypes.data, ldc) == 0
                        avg, mx = gemm_error(C[:, :N], ref, scale)
                        assert avg <= 1e-6 and mx <= 1e-5, (M, N, K, ta, tb, pad, avg, mx)
                        assert (C[:, N:] == C0[:, N:]).all()


@pytest.mark.parametrize("t,dt", [(abi.H, np.float16), (abi.S, np.float32)])
def test_host_operands_banded_pipeline(gpu_lib, t, dt):
    """Host A and C large enough for the banded pipeline (row bands of A cross to the device while earlier bands are
    multiplied and their C rows return): a ragged last band, leading dimensions that are not 16-byte multiples, beta
    != 0 (C bands copied in too), and canary bytes between the rows of C that must survive."""
    rng = np.random.default_rng(29)
    M, N, K = 2500, 2000, 1500
    lda, ldc = K + 5, N + 3
    A = rng.uniform(-1, 1, (M, lda)).astype(dt)
    B = (rng.uniform(-1, 1, (K, N)) / np.sqrt(K)).astype(dt)
    C0 = rng.uniform(-1, 1, (M, ldc)).astype(dt)
    C0[:, N:] = 7.0
    C = C0.copy()
    assert gpu_lib.gemm(t, 0, 0, M, N, K, 1.5, A.ctypes.data, lda, B.ctypes.data, N, 0.5, C.ctypes.data, ldc) == 0
    rows = np.concatenate([np.arange(0, M, 37), np.arange(M - 200, M)])
    a64, b64, c64 = A[rows, :K].astype(np.float64), B.astype(np.float64), C0[rows, :N].astype(np.float64)
    ref = 1.5 * a64 @ b64 + 0.5 * c64
    scale = 1.5 * np.abs(a64) @ np.abs(b64) + 0.5 * np.abs(c64)
    avg, mx = gemm_error(C[rows, :N], ref, scale)
    assert mx <= (1e-3 if dt == np.float16 else 1e-5), (t, mx)
    assert (C[:, N:] == 7.0).all()


@pytest.mark.parametrize("t", [abi.H, abi.HS])
def test_hgemm_both_transposed(gpu_lib, t):
    """C = Aᵀ·Bᵀ with alpha = 1, beta = 0 runs as Cᵀ = B·A with the epilogue writing transposed 32 × 32 blocks:
    ragged edges in M, N and K, a split-K tail, 256×128 tiles, and a batch with padded strides; every element of C
    (and nothing past it) is checked against FP64."""
    rng = np.random.default_rng(23)
    for (M, N, K) in ((129, 257, 65), (1000, 5000, 300), (3072, 1792, 1024), (300, 1100, 777), (2048, 2048, 2048)):
        A = (rng.standard_normal((K, M)) / np.sqrt(K)).astype(np.float16)   # stored K × M
        B = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float16)   # stored N × K
        ldc = N + 8
        C = np.full((M, ldc), 7.0, np.float16)
        for _ in range(2):
            assert gpu_lib.gemm(t, 1, 1, M, N, K, 1.0, A.ctypes.data, M, B.ctypes.data, K, 0.0, C.ctypes.data, ldc) == 0
            a64, b64 = A.T.astype(np.float64), B.T.astype(np.float64)
            avg, mx = gemm_error(C[:, :N], a64 @ b64, np.abs(a64) @ np.abs(b64))
            assert mx <= 1e-3, (t, M, N, K, mx)
            assert (C[:, N:] == 7.0).all()
    cnt, M, N, K = 3, 384, 320, 200
    sa, sb, sc = K * M + 64, N * K + 32, M * N + 128
    A = rng.uniform(-1, 1, cnt * sa).astype(np.float16)
    B = rng.uniform(-1, 1, cnt * sb).astype(np.float16)
    C = np.full(cnt * sc, 7.0, np.float16)
    assert gpu_lib.gemm_batched(t, 1, 1, M, N, K, 1.0, A.ctypes.data, M, sa, B.ctypes.data, K, sb, 0.0, C.ctypes.data,
                                N, sc, cnt) == 0
    for i in range(cnt):
        a64 = A[i * sa:i * sa + K * M].reshape(K, M).T.astype(np.float64)
        b64 = B[i * sb:i * sb + N * K].reshape(N, K).T.astype(np.float64)
        c = C[i * sc:i * sc + M * N].reshape(M, N)
        avg, mx = gemm_error(c, a64 @ b64, np.abs(a64) @ np.abs(b64))
        assert mx <= 1e-3, (t, i, mx)
        assert (C[i * sc + M * N:(i + 1) * sc] == 7.0).all()


def test_gemm_allgather_writes_every_destination(gpu_lib):
    """The fused GEMM + all-gather epilogue on one GPU: two local buffers stand in for two ranks' C; each receives
    this rank's column block at col_offset and nothing else changes."""
    torch = pytest.importorskip("torch")
    M, K, N, nb = 512, 384, 1024, 256
    g = torch.Generator(device="cuda").manual_seed(3)
    A = torch.randn(M, K, device="cuda", generator=g, dtype=torch.float16)
    B = torch.randn(K, nb, device="cuda", generator=g, dtype=torch.float16)
    C1 = torch.full((M, N), 7.0, device="cuda", dtype=torch.float16)
    C2 = torch.full((M, N), 7.0, device="cuda", dtype=torch.float16)
    torch.cuda.synchronize()
    arr = (ctypes.c_void_p * 2)(C1.data_ptr(), C2.data_ptr())
    f = gpu_lib.dll.gen9blas_gemm_allgather
    f.argtypes = [ctypes.c_int] * 6 + [ctypes.c_double, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                       ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int64]
    for t in (abi.H, abi.HS):
        assert f(t, 0, 0, M, nb, K, 1.0, A.data_ptr(), K, B.data_ptr(), nb, arr, 2, N, 512) == 0, gpu_lib.error()
        torch.cuda.synchronize()
        ref = A.double() @ B.double()
        scale = A.double().abs() @ B.double().abs()
        for C in (C1, C2):
            blk = C[:, 512:768].double()
            assert float(((blk - ref).abs() / scale).max()) <= 1e-3
            rest = torch.cat([C[:, :512], C[:, 768:]], 1)
            assert bool((rest == 7.0).all())


# ---------------------------------------------------------------------------------------- BASELINE config sizes
def config_fixture():
    import os
    return np.load(os.path.join(ROOT, "tests", "golden", "ref_config_rows.npz"))


def test_baseline_c0_sgemm(gpu_lib):
    """SGEMM n = 1024 row-major NN, alpha = 1, beta = 0, A and B uniform[-1,1] from seeds 1 and 2
    (lib/test_basic.py:86-87). North-star limit max <= 1e-6 on every element against FP64, and within 1e-6 (same
    metric) of the reference CBLAS layer's own output on the fixture rows; run twice (split-K partials are reused)."""
    n = mg.C0_N
    A, B = mg.c0_inputs()
    a64, b64 = A.astype(np.float64), B.astype(np.float64)
    ref, scale = a64 @ b64, np.abs(a64) @ np.abs(b64)
    rows = mg.c0_rows()
    want = config_fixture()["sgemm_c0_rows"]
    for _ in range(2):
        C = np.full((n, n), np.nan, np.float32)
        assert gpu_lib.gemm(abi.S, 0, 0, n, n, n, 1.0, A.ctypes.data, n, B.ctypes.data, n, 0.0, C.ctypes.data, n) == 0
        avg, mx = gemm_error(C, ref, scale)
        print(f"sgemm n=1024: mean {avg:.2e} max {mx:.2e}")
        assert mx <= 1e-6 and avg <= 1e-7, (avg, mx)
        assert gemm_error(C[rows], want, scale[rows])[1] <= 1e-6


@pytest.mark.parametrize("n", [1024, 2048, 3000, 8192])
@pytest.mark.parametrize("accurate,limit", [(False, 1e-3), (True, 1e-4)])
def test_baseline_c1_hgemm_sizes(gpu_lib, n, accurate, limit):
    """configs[1] at the tile-remainder sizes (n = 1024: 256x128 pair tiles, single wave; 2048; 3000: ragged edges and
    a split-K tail) and at the 70 % target size n = 8192: A, B iid N(0,1)/sqrt(n) in FP16, north-star max limits (fast
    1e-3, accurate 1e-4) against FP64 on the FP16 inputs -- every row up to n = 2048, else a sample plus the last
    rows (the ragged tile row)."""
    rng = np.random.default_rng(1)
    A = (rng.standard_normal((n, n)) / np.sqrt(n)).astype(np.float16)
    B = (rng.standard_normal((n, n)) / np.sqrt(n)).astype(np.float16)
    C = np.full((n, n), np.nan, np.float16)
    t = abi.HS if accurate else abi.H
    assert gpu_lib.gemm(t, 0, 0, n, n, n, 1.0, A.ctypes.data, n, B.ctypes.data, n, 0.0, C.ctypes.data, n) == 0
    if n <= 2048:
        rows = np.arange(n)
    else:
        rows = np.unique(np.concatenate([rng.choice(n, 384 if n < 8192 else 128, replace=False), np.arange(n - 64, n)]))
    a64, b64 = A[rows].astype(np.float64), B.astype(np.float64)
    avg, mx = gemm_error(C[rows], a64 @ b64, np.abs(a64) @ np.abs(b64))
    print(f"hgemm n={n} accurate={accurate}: mean {avg:.2e} max {mx:.2e}")
    assert mx <= limit, (n, accurate, avg, mx)


def c3_call(lib, ta, tb, n, A, B, C):
    """Column-major DGEMM through the row-major C ABI by the CBLAS swap identity: column-major C = op(A)·op(B) is
    row-major Cᵀ = op(B)ᵀ·op(A)ᵀ on the same memory (the path the LD_PRELOAD library takes, lib/src/cblas.c:190)."""
    As, Bs, Cs = np.asfortranarray(A), np.asfortranarray(B), np.asfortranarray(C)
    r = lib.gemm(abi.D, int(tb == mg.Trans), int(ta == mg.Trans), n, n, n, mg.C3_ALPHA, Bs.ctypes.data, B.shape[0],
                 As.ctypes.data, A.shape[0], mg.C3_BETA, Cs.ctypes.data, n)
    return r, Cs


@pytest.mark.parametrize("n", [3000, 4096])
@pytest.mark.parametrize("ta,tb", [(mg.NoTrans, mg.NoTrans), (mg.Trans, mg.NoTrans), (mg.NoTrans, mg.Trans),
                                   (mg.Trans, mg.Trans)])
def test_baseline_c3_dgemm(gpu_lib, n, ta, tb):
    """DGEMM n = 3000 and 4096, column-major, all four transposes, alpha = 1.5, beta = 0.5, C prefilled
    uniform[-1,1]: max <= 1e-13 against FP64 on sampled rows; at n = 3000 also against the reference CBLAS layer's
    own output rows (fixture)."""
    A, B, C0 = mg.gemm_inputs("d", mg.ColMajor, ta, tb, n, n, n)
    r, Cs = c3_call(gpu_lib, ta, tb, n, A, B, C0.copy())
    assert r == 0, gpu_lib.error()
    rng = np.random.default_rng(n)
    rows = mg.c3_rows() if n == mg.C3_N else np.unique(np.concatenate([rng.choice(n, 16, replace=False), [0, n - 1]]))
    opA = A if ta == mg.NoTrans else A.T
    opB = B if tb == mg.NoTrans else B.T
    ref = mg.C3_ALPHA * opA[rows] @ opB + mg.C3_BETA * C0[rows]
    scale = mg.C3_ALPHA * np.abs(opA[rows]) @ np.abs(opB) + mg.C3_BETA * np.abs(C0[rows])
    avg, mx = gemm_error(Cs[rows], ref, scale)
    assert mx <= 1e-13, (n, ta, tb, mx)
    if n == mg.C3_N:
        want = config_fixture()[f"dgemm_c3_t{ta}{tb}_rows"]
        assert gemm_error(Cs[rows], want, scale)[1] <= 1e-13
