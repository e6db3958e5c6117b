"""GPU parity of the neural-network entry points (include/gen9blas_ml.h, the reference's lib/gen9blas_ml.h) through the C
ABI, against the NumPy restatement in oracle/ml_ref.py. Bars: bit-exact for layout ops, dequantization and the fused
versus unfused epilogues; one FP16 ulp for the FP16-result GEMMs (FP32 versus FP64 accumulation before the single FP16
rounding); float32 rounding-level tolerances for the norms, RoPE, interpolation and attention, written in each test."""
import ctypes
import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
import ml_ref  # noqa: E402

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
HS = 2
rng = np.random.default_rng(23)


def dev(a):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    torch.cuda.synchronize()
    return t


def ptr(x):
    if x is None:
        return None
    return x.data_ptr() if isinstance(x, torch.Tensor) else x.ctypes.data


def host(t, lib):
    assert lib.flush() == 0, lib.error()
    torch.cuda.synchronize()
    return t.cpu().numpy()


def ulps16(got, want):
    """Distance in FP16 ulps of want's magnitude (the results are FP16 values widened to float32)."""
    sp = np.spacing(np.abs(want).astype(np.float16)).astype(np.float64)
    return np.abs(got.astype(np.float64) - want.astype(np.float64)) / np.maximum(sp, 2.0 ** -24)


def f16w_close(got, A, W16, want):
    """The FP16-result GEMM bound: one FP16 ulp of the result plus FP32 accumulation error K·2^-23·(|A|·|W|) (the GPU sums
    in FP32, the oracle in float64; near-zero results of cancelling sums can round to different FP16 neighbours)."""
    K = A.shape[1]
    scale = np.abs(ml_ref.to_f16(A)).astype(np.float64) @ np.abs(W16.astype(np.float64)).T
    sp = np.spacing(np.abs(want).astype(np.float16)).astype(np.float64)
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    return bool(np.all(err <= sp + K * 2.0 ** -23 * scale + 2.0 ** -24)), float(np.max(err / (sp + K * 2.0 ** -23 * scale)))


def pack_hs(lib, W16):
    N, K = W16.shape
    P = lib.pack_b(HS, 1, K, N, ptr(np.ascontiguousarray(W16)), K)
    assert P, lib.error()
    return P


def nf_ptr():
    c = ctypes.c_int(-1)
    return c, ctypes.addressof(c)


# ------------------------------------------------------------------------------------------- FP16-weight GEMMs
@pytest.mark.parametrize("M,N,K", [(1, 300, 520), (7, 257, 333), (64, 1000, 512), (200, 96, 1024)])
def test_gemm_pb_f16w_against_oracle(gpu_lib, M, N, K):
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = (rng.standard_normal((N, K)) * 0.05).astype(np.float16)
    P = pack_hs(gpu_lib, W)
    try:
        want, _ = ml_ref.gemm_f16w(A, W)
        for on_dev in (False, True):
            C = dev(np.full((M, N), np.nan, np.float32)) if on_dev else np.full((M, N), np.nan, np.float32)
            Ax = dev(A) if on_dev else A
            nf, nfp = nf_ptr()
            assert gpu_lib.gemm_pb_f16w(M, ptr(Ax), K, P, ptr(C), N, nfp) == 0, gpu_lib.error()
            got = host(C, gpu_lib) if on_dev else C
            ok, worst = f16w_close(got, A, W, want)
            assert nf.value == 0 and ok and np.mean(ulps16(got, want) > 0) < 0.01, (on_dev, worst)
        # FP16 activations give the same bits: the F32 path rounds A to FP16 first
        A16 = A.astype(np.float16)
        C2 = np.full((M, N), np.nan, np.float32)
        nf, nfp = nf_ptr()
        assert gpu_lib.gemm_pb_f16w_h(M, ptr(A16), K, P, ptr(C2), N, nfp) == 0, gpu_lib.error()
        assert np.array_equal(C2, got)
    finally:
        gpu_lib.packed_b_free(P)


def test_gemm_pb_f16w_ex_equals_unfused_ops(gpu_lib):
    """C = gelu(A·Bp + bias) + R fused equals gemm_pb_f16w, binop_rows(+bias), gelu, binop_rows(+R) bit for bit; R may
    be C itself."""
    M, N, K = 37, 400, 256
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = (rng.standard_normal((N, K)) * 0.1).astype(np.float16)
    bias = rng.standard_normal(N).astype(np.float32)
    R = rng.standard_normal((M, N)).astype(np.float32)
    P = pack_hs(gpu_lib, W)
    try:
        nf, nfp = nf_ptr()
        C = np.zeros((M, N), np.float32)
        assert gpu_lib.gemm_pb_f16w_ex(M, ptr(A), K, P, ptr(C), N, ptr(bias), 1, ptr(R), N, nfp) == 0, gpu_lib.error()
        U = np.zeros((M, N), np.float32)
        assert gpu_lib.gemm_pb_f16w(M, ptr(A), K, P, ptr(U), N, nfp) == 0
        assert gpu_lib.binop_rows(0, M, N, ptr(U), N, ptr(bias), 0, 1, ptr(U), N, 1) == 0, gpu_lib.error()
        assert gpu_lib.gelu(M * N, ptr(U), ptr(U), 1) == 0
        assert gpu_lib.binop_rows(0, M, N, ptr(U), N, ptr(R), N, 1, ptr(U), N, 1) == 0
        assert np.array_equal(C, U)
        want, _ = ml_ref.gemm_f16w(A, W, bias, True, R)
        assert np.max(np.abs(C - want)) <= 4 * np.max(np.spacing(np.abs(want).astype(np.float16)).astype(np.float32))
        # in-place residual on device memory: R is C
        Cd = dev(R)
        assert gpu_lib.gemm_pb_f16w_ex(M, ptr(dev(A)), K, P, ptr(Cd), N, ptr(dev(bias)), 1, ptr(Cd), N, nfp) == 0
        assert np.array_equal(host(Cd, gpu_lib), C)
    finally:
        gpu_lib.packed_b_free(P)


@pytest.mark.parametrize("M,N,K", [(1, 4096, 2048), (5, 3000, 2304), (16, 2500, 4104), (9, 4096, 2048),
                                   (16, 11008, 4096), (12, 5000, 4096)])
def test_gemm_pb_f16w_single_kernel_shapes(gpu_lib, M, N, K):
    """Shapes that run the FP16-weight product as one kernel (M <= 16, at least 16 weight rows per SM, K >= 2048; the
    last two over several waves, the F32 activations rounded ahead of the kernel for the wider one): the same bits as
    the FP16-accumulating-in-FP32 GEMM (gen9blas_gemm, GEN9BLAS_HS) of the FP16-rounded activations,
    as the FP16-activation entry point, and as the unfused bias / GELU / residual chain; the oracle's bound; a
    non-finite result flagged."""
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = (rng.standard_normal((N, K)) * 0.05).astype(np.float16)
    bias = rng.standard_normal(N).astype(np.float32)
    R = rng.standard_normal((M, N)).astype(np.float32)
    P = pack_hs(gpu_lib, W)
    try:
        nf, nfp = nf_ptr()
        C = np.full((M, N), np.nan, np.float32)
        assert gpu_lib.gemm_pb_f16w(M, ptr(A), K, P, ptr(C), N, nfp) == 0, gpu_lib.error()
        A16 = A.astype(np.float16)
        G16 = np.zeros((M, N), np.float16)
        assert gpu_lib.gemm(HS, 0, 1, M, N, K, 1.0, ptr(A16), K, ptr(W), K, 0.0, ptr(G16), N) == 0, gpu_lib.error()
        assert nf.value == 0 and np.array_equal(C, G16.astype(np.float32))
        want, _ = ml_ref.gemm_f16w(A, W)
        ok, worst = f16w_close(C, A, W, want)
        assert ok, worst
        C2 = np.full((M, N), np.nan, np.float32)
        assert gpu_lib.gemm_pb_f16w_h(M, ptr(A16), K, P, ptr(C2), N, nfp) == 0
        assert np.array_equal(C2, C)
        Cx = dev(R)                                   # fused bias + GELU + in-place residual on device memory
        assert gpu_lib.gemm_pb_f16w_ex(M, ptr(dev(A)), K, P, ptr(Cx), N, ptr(dev(bias)), 1, ptr(Cx), N, nfp) == 0
        U = C.copy()
        assert gpu_lib.binop_rows(0, M, N, ptr(U), N, ptr(bias), 0, 1, ptr(U), N, 1) == 0
        assert gpu_lib.gelu(M * N, ptr(U), ptr(U), 1) == 0
        assert gpu_lib.binop_rows(0, M, N, ptr(U), N, ptr(R), N, 1, ptr(U), N, 1) == 0
        assert np.array_equal(host(Cx, gpu_lib), U)
        A[0, :] = 3000.0 * np.sign(W[0].astype(np.float32))   # C[0, 0] = 3000 · Σ|w|: beyond FP16
        assert gpu_lib.gemm_pb_f16w(M, ptr(A), K, P, ptr(C), N, nfp) == 0
        assert nf.value == 1
    finally:
        gpu_lib.packed_b_free(P)


def test_gemm_pb_f16w_overflow_sets_nonfinite(gpu_lib):
    M, N, K = 4, 64, 256
    A = np.full((M, K), 200.0, np.float32)
    W = np.full((N, K), 4.0, np.float16)              # 256 · 800 = 204800 > 65504: inf in FP16
    P = pack_hs(gpu_lib, W)
    try:
        C = np.zeros((M, N), np.float32)
        nf, nfp = nf_ptr()
        assert gpu_lib.gemm_pb_f16w(M, ptr(A), K, P, ptr(C), N, nfp) == 0
        assert nf.value == 1 and np.all(np.isinf(C))
    finally:
        gpu_lib.packed_b_free(P)


def test_nowait_pending_counts_overflowing_calls(gpu_lib):
    M, N, K = 2, 128, 256
    W = np.full((N, K), 4.0, np.float16)
    P = pack_hs(gpu_lib, W)
    A_big, A_ok = dev(np.full((M, K), 200.0, np.float32)), dev(np.full((M, K), 0.01, np.float32))
    C = dev(np.zeros((M, N), np.float32))
    gpu_lib.set_nowait(1)
    try:
        assert gpu_lib.flush() == 0
        gpu_lib.nowait_pending()                       # clears the flags of earlier queued calls
        for A in (A_ok, A_big, A_ok, A_big, A_big):
            nf, nfp = nf_ptr()
            assert gpu_lib.gemm_pb_f16w(M, ptr(A), K, P, ptr(C), N, nfp) == 0, gpu_lib.error()
            assert nf.value == 0                      # queued: not reported per call
        assert gpu_lib.flush() == 0
        assert gpu_lib.nowait_pending() == 3
        assert gpu_lib.nowait_pending() == 0
    finally:
        gpu_lib.set_nowait(0)
        gpu_lib.packed_b_free(P)


def test_gemm_multi_f16w(gpu_lib):
    M, K = 9, 384
    Ns = [128, 64, 200]
    A = rng.standard_normal((M, K)).astype(np.float32)
    Ws = [(rng.standard_normal((n, K)) * 0.05).astype(np.float16) for n in Ns]
    Ps = [pack_hs(gpu_lib, W) for W in Ws]
    try:
        outs = [dev(np.full((M, n + 3), np.nan, np.float32)) for n in Ns]   # padded rows: ldc = n + 3
        Parr = (ctypes.c_void_p * 3)(*Ps)
        Carr = (ctypes.c_void_p * 3)(*[ptr(o) for o in outs])
        ldc = (ctypes.c_int * 3)(*[n + 3 for n in Ns])
        nf = (ctypes.c_int * 3)(-1, -1, -1)
        assert gpu_lib.gemm_multi_f16w(M, ptr(A), K, 3, ctypes.addressof(Parr), ctypes.addressof(Carr),
                                       ctypes.addressof(ldc), ctypes.addressof(nf)) == 0, gpu_lib.error()
        assert list(nf) == [0, 0, 0]
        for i, n in enumerate(Ns):
            one = np.zeros((M, n), np.float32)
            c, cp = nf_ptr()
            assert gpu_lib.gemm_pb_f16w(M, ptr(A), K, Ps[i], ptr(one), n, cp) == 0
            got = host(outs[i], gpu_lib)
            assert np.array_equal(got[:, :n], one) and np.all(np.isnan(got[:, n:]))
        # a host output: not handled, nothing written
        hostC = np.zeros((M, Ns[0]), np.float32)
        Carr[0] = hostC.ctypes.data
        assert gpu_lib.gemm_multi_f16w(M, ptr(A), K, 3, ctypes.addressof(Parr), ctypes.addressof(Carr),
                                       ctypes.addressof(ldc), ctypes.addressof(nf)) == 1
        assert not hostC.any()
    finally:
        for P in Ps:
            gpu_lib.packed_b_free(P)


@pytest.mark.parametrize("M", [1, 5, 48])
def test_ffn_f16w(gpu_lib, M):
    K, N, Nd = 256, 688, 256
    X = rng.standard_normal((M, K)).astype(np.float32)
    Wg, Wu = [(rng.standard_normal((N, K)) * 0.06).astype(np.float16) for _ in range(2)]
    Wd = (rng.standard_normal((Nd, N)) * 0.04).astype(np.float16)
    Pg, Pu, Pd = pack_hs(gpu_lib, Wg), pack_hs(gpu_lib, Wu), pack_hs(gpu_lib, Wd)
    try:
        Y = np.zeros((M, Nd), np.float32)
        nf, nfp = nf_ptr()
        assert gpu_lib.ffn_f16w(M, ptr(X), K, Pg, Pu, Pd, ptr(Y), Nd, nfp) == 0, gpu_lib.error()
        want = ml_ref.ffn_f16w(X, Wg, Wu, Wd)
        assert nf.value == 0
        # the intermediates are FP16 roundings of FP32 (GPU) or FP64 (oracle) sums: a few FP16 ulps of the output scale
        assert np.max(np.abs(Y - want)) <= 4e-3 * np.max(np.abs(want)), np.max(np.abs(Y - want))
    finally:
        for P in (Pg, Pu, Pd):
            gpu_lib.packed_b_free(P)


@pytest.fixture(scope="module")
def ffn_7b(gpu_lib):
    """Gate, up (11008 x 4096) and down (4096 x 11008) FP16 weights of a 7B layer, packed once for the module."""
    K, N, Nd = 4096, 11008, 4096
    r = np.random.default_rng(77)
    Wg, Wu = [(r.standard_normal((N, K), np.float32) * 0.02).astype(np.float16) for _ in range(2)]
    Wd = (r.standard_normal((Nd, N), np.float32) * 0.02).astype(np.float16)
    Ps = [pack_hs(gpu_lib, W) for W in (Wg, Wu, Wd)]
    yield (K, N, Nd), Ps
    for P in Ps:
        gpu_lib.packed_b_free(P)


@pytest.mark.parametrize("M", [1, 5, 16])
@pytest.mark.parametrize("scale", [1.0, 300.0])
def test_ffn_f16w_decode_fused_equals_chain(gpu_lib, ffn_7b, M, scale):
    """At decode sizes (M <= 16, 16-byte aligned activation rows) ffn_f16w runs gate and up in one launch whose CTA
    pairs apply SWIGLU, then the down GEMM with its epilogue in the kernel; an activation pitch that is not a multiple
    of four floats takes the general six-kernel chain. Both give the same bits and the same non-finite flag (scale
    300 drives |silu(g)·u| past FP16)."""
    (K, N, Nd), (Pg, Pu, Pd) = ffn_7b
    X = (rng.standard_normal((M, K)) * scale).astype(np.float32)
    Xp = np.zeros((M, K + 1), np.float32)
    Xp[:, :K] = X
    Yf, Yc = np.zeros((M, Nd), np.float32), np.zeros((M, Nd), np.float32)
    nf1, nfp1 = nf_ptr()
    nf2, nfp2 = nf_ptr()
    assert gpu_lib.ffn_f16w(M, ptr(X), K, Pg, Pu, Pd, ptr(Yf), Nd, nfp1) == 0, gpu_lib.error()
    assert gpu_lib.ffn_f16w(M, ptr(Xp), K + 1, Pg, Pu, Pd, ptr(Yc), Nd, nfp2) == 0, gpu_lib.error()
    assert np.array_equal(Yf.view(np.uint32), Yc.view(np.uint32))
    assert nf1.value == nf2.value == (1 if scale > 1 else 0)
    for _ in range(2):   # repeated calls: the pairs' arrival counters return to zero
        Yr = np.zeros((M, Nd), np.float32)
        assert gpu_lib.ffn_f16w(M, ptr(X), K, Pg, Pu, Pd, ptr(Yr), Nd, None) == 0, gpu_lib.error()
        assert np.array_equal(Yr.view(np.uint32), Yf.view(np.uint32))


@pytest.mark.parametrize("qtype", [0, 1, 2])
def test_pack_b_q_dequantizes_bit_exactly(gpu_lib, qtype):
    """The packed FP16 weights equal ggml's dequantize_row_* + FP16 rounding: read back through an identity product
    (C = I · Wᵀ, one non-zero product per element: exact) and compared bit for bit."""
    K, N = (512, 96) if qtype else (96, 80)
    W = ml_ref.random_blocks(rng, qtype, N, K)
    row_bytes = W.shape[1]
    oor = ctypes.c_int(-1)
    P = gpu_lib.pack_b_q(qtype, K, N, ptr(W), row_bytes, ctypes.addressof(oor))
    assert P, gpu_lib.error()
    try:
        assert oor.value == 0
        I16 = np.eye(K, dtype=np.float16)
        C = np.zeros((K, N), np.float32)
        nf, nfp = nf_ptr()
        assert gpu_lib.gemm_pb_f16w_h(K, ptr(I16), K, P, ptr(C), N, nfp) == 0, gpu_lib.error()
        want = ml_ref.to_f16(ml_ref.dequant_rows(W, qtype, K))
        assert np.array_equal(C.T, want)
    finally:
        gpu_lib.packed_b_free(P)


def test_pack_b_q_out_of_range_and_bad_shapes(gpu_lib):
    K, N = 64, 8
    W = np.zeros((N, 2 * 34), np.uint8)
    W[:, 0:2] = np.array([60000.0], np.float16).view(np.uint8)
    W[:, 2:34] = np.int8(127).view(np.uint8)          # 127 · 60000 beyond FP16
    oor = ctypes.c_int(-1)
    P = gpu_lib.pack_b_q(0, K, N, ptr(W), W.shape[1], ctypes.addressof(oor))
    assert P and oor.value == 1
    gpu_lib.packed_b_free(P)
    assert not gpu_lib.pack_b_q(0, 48, N, ptr(W), W.shape[1], None)      # K not a multiple of 32
    assert not gpu_lib.pack_b_q(1, 128, N, ptr(W), 144, None)            # Q4_K needs K % 256 == 0
    assert not gpu_lib.pack_b_q(7, 256, N, ptr(W), 1024, None)           # unknown type


def test_layer_norm_pack_feeds_gemm_pa(gpu_lib):
    """layer_norm_pack writes the same Y as layer_norm, and gemm_pa_f16w_ex on its packed rows equals gemm_pb_f16w_ex
    on Y bit for bit."""
    M, K, N = 23, 200, 300
    X = rng.standard_normal((M, K + 5)).astype(np.float32)
    w, b = rng.standard_normal(K).astype(np.float32), rng.standard_normal(K).astype(np.float32)
    W = (rng.standard_normal((N, K)) * 0.05).astype(np.float16)
    bias = rng.standard_normal(N).astype(np.float32)
    P = pack_hs(gpu_lib, W)
    pa = gpu_lib.packed_a_create()
    assert pa
    try:
        Y1, Y2 = np.zeros((M, K), np.float32), np.zeros((M, K), np.float32)
        assert gpu_lib.layer_norm(M, K, ptr(X), K + 5, ptr(w), ptr(b), 1e-5, ptr(Y1), K, 1) == 0, gpu_lib.error()
        assert gpu_lib.layer_norm_pack(M, K, ptr(X), K + 5, ptr(w), ptr(b), 1e-5, ptr(Y2), K, pa, 1) == 0, gpu_lib.error()
        assert np.array_equal(Y1, Y2)
        C1, C2 = np.zeros((M, N), np.float32), np.zeros((M, N), np.float32)
        nf, nfp = nf_ptr()
        assert gpu_lib.gemm_pb_f16w_ex(M, ptr(Y1), K, P, ptr(C1), N, ptr(bias), 1, None, 0, nfp) == 0
        assert gpu_lib.gemm_pa_f16w_ex(pa, P, ptr(C2), N, ptr(bias), 1, None, 0, nfp) == 0, gpu_lib.error()
        assert np.array_equal(C1, C2)
        W2 = (rng.standard_normal((N, K + 8)) * 0.05).astype(np.float16)   # K mismatch: rejected
        P2 = pack_hs(gpu_lib, W2)
        assert gpu_lib.gemm_pa_f16w_ex(pa, P2, ptr(C2), N, None, 0, None, 0, nfp) < 0
        gpu_lib.packed_b_free(P2)
    finally:
        gpu_lib.flush()
        gpu_lib.packed_a_free(pa)
        gpu_lib.packed_b_free(P)


# ------------------------------------------------------------------------------------------- elementwise ops
@pytest.mark.parametrize("K,ld", [(4099, 4100), (4096, 4100)])   # scalar rows; 16-byte rows (vector kernels)
@pytest.mark.parametrize("on_dev", [False, True])
def test_norms(gpu_lib, on_dev, K, ld):
    M = 33
    Xf = rng.standard_normal((M, ld)).astype(np.float32) * 3
    w, b = rng.standard_normal(K).astype(np.float32), rng.standard_normal(K).astype(np.float32)
    for fn in ("rms", "ln"):
        for use_w in (False, True):
            Y = np.full((M, K), np.nan, np.float32)
            Xa, Ya = (dev(Xf), dev(Y)) if on_dev else (Xf, Y)
            if fn == "rms":
                r = gpu_lib.rms_norm(M, K, ptr(Xa), ld, ptr(w) if use_w else None, 1e-6, ptr(Ya), K, 1)
                want = ml_ref.rms_norm(Xf[:, :K], w if use_w else None, 1e-6)
            else:
                r = gpu_lib.layer_norm(M, K, ptr(Xa), ld, ptr(w) if use_w else None, ptr(b) if use_w else None, 1e-5,
                                       ptr(Ya), K, 1)
                want = ml_ref.layer_norm(Xf[:, :K], w if use_w else None, b if use_w else None, 1e-5)
            assert r == 0, gpu_lib.error()
            got = host(Ya, gpu_lib) if on_dev else Ya
            # FP64 sums in both: the float32 scale may differ by the last bit of the mean's rounding
            assert np.allclose(got, want, rtol=4e-7, atol=1e-7), (fn, use_w, np.max(np.abs(got - want)))


def test_binop_rows_broadcasts(gpu_lib):
    M, K = 17, 130
    A = rng.standard_normal((M, K + 2)).astype(np.float32)
    Brows = rng.standard_normal((M, K)).astype(np.float32)
    for op in (0, 1):
        f = np.add if op == 0 else np.multiply
        for ldb, bs0, B, want_b in ((K, 1, Brows, Brows), (0, 1, Brows[0], Brows[:1]),
                                    (1, 0, Brows[:, 0].copy(), Brows[:, :1])):
            C = np.zeros((M, K), np.float32)
            assert gpu_lib.binop_rows(op, M, K, ptr(A), K + 2, ptr(np.ascontiguousarray(B)), ldb, bs0, ptr(C), K, 1) == 0
            assert np.array_equal(C, f(A[:, :K], want_b)), (op, ldb, bs0)


def test_activations(gpu_lib):
    x = np.concatenate([np.linspace(-12, 12, 100001, dtype=np.float32),
                        rng.standard_normal(50000).astype(np.float32) * 4])
    n = x.size
    y = np.zeros_like(x)
    assert gpu_lib.gelu(n, ptr(x), ptr(y), 1) == 0
    want = ml_ref.gelu(x)
    # CUDA's tanhf and NumPy's tanh may differ in the last float32 bit; where 1 + tanh cancels (x around -4) that bit
    # is several FP16 ulps of the small result, so the bound is one FP16 ulp plus |x|·2^-22 (0.5·|x|·4 ulps of 1)
    sp = np.spacing(np.abs(want).astype(np.float16)).astype(np.float64)
    assert np.all(np.abs(y.astype(np.float64) - want) <= sp + np.abs(x) * 2.0 ** -22)
    assert np.mean(ulps16(y, want) > 0) < 1e-3
    xd = dev(x)
    assert gpu_lib.gelu(n, ptr(xd), ptr(xd), 1) == 0          # in place
    assert np.array_equal(host(xd, gpu_lib), y)
    assert gpu_lib.gelu_erf(n, ptr(x), ptr(y), 1) == 0
    want = ml_ref.gelu_erf(x)   # 1 + erf cancels below x ~ -3 as 1 + tanh does: the same |x|·2^-22 allowance
    assert np.all(np.abs(y.astype(np.float64) - want) <= 4 * np.spacing(np.abs(want)) + np.abs(x) * 2.0 ** -22)
    assert gpu_lib.relu(n, ptr(x), ptr(y), 1) == 0
    assert np.array_equal(y, ml_ref.relu(x))


@pytest.mark.parametrize("n", [4500000, 11009])
def test_gelu_table_equals_computed(gpu_lib, n):
    """16-byte aligned operands take the table kernel from 2^22 elements on (fp16(x) indexes a 64K-entry table built
    on the device from the same GELU function) and a vectorised computing kernel below; unaligned ones the scalar
    computing kernel. All agree bit for bit on every FP16 value, NaN and the infinities included, and on random
    floats around the ±10 cut."""
    x = np.concatenate([np.arange(65536, dtype=np.uint16).view(np.float16).astype(np.float32),
                        np.array([-10.0, 10.0, np.nextafter(-10.0, 0, dtype=np.float32),
                                  np.nextafter(10.0, 0, dtype=np.float32), np.inf, -np.inf, np.nan], np.float32),
                        (rng.standard_normal(max(n, 65543) - 65543) * 6).astype(np.float32)])
    x = np.ascontiguousarray(x[-n:] if n < x.size else x)
    buf = dev(np.concatenate([np.zeros(1, np.float32), x]))   # x at a 4-byte offset: not 16-byte aligned
    out = dev(np.zeros(n + 1, np.float32))
    xa = dev(x)
    ya = dev(np.zeros(n, np.float32))
    assert gpu_lib.gelu(n, ptr(xa), ptr(ya), 1) == 0
    assert gpu_lib.gelu(n, buf.data_ptr() + 4, out.data_ptr() + 4, 1) == 0
    a, m = host(ya, gpu_lib), host(out, gpu_lib)[1:]
    assert np.array_equal(a.view(np.uint32), m.view(np.uint32)) or np.array_equal(a, m, equal_nan=True)


def test_cvt_f16_heads(gpu_lib):
    rows, H, D = 11, 6, 40
    X = (rng.standard_normal((rows, H * 64 + 7)) * 3e4).astype(np.float32)   # beyond FP16: saturated
    Y = np.zeros((rows, H, D), np.float16)
    assert gpu_lib.cvt_f16_heads(rows, H, D, ptr(X), H * 64 + 7, 64, ptr(Y), 1) == 0
    want = np.clip(np.stack([X[:, h * 64:h * 64 + D] for h in range(H)], 1), -65504, 65504).astype(np.float16)
    assert np.array_equal(Y.view(np.uint16), want.view(np.uint16))


@pytest.mark.parametrize("f16", [0, 1])
def test_im2col(gpu_lib, f16):
    N, IC, IH, IW, KH, KW = 2, 3, 9, 11, 3, 2
    s0, s1, p0, p1, d0, d1 = 2, 1, 1, 2, 1, 2
    OW = (IW + 2 * p0 - d0 * (KW - 1) - 1) // s0 + 1
    OH = (IH + 2 * p1 - d1 * (KH - 1) - 1) // s1 + 1
    X = rng.standard_normal((N, IC, IH, IW)).astype(np.float32)
    Y = np.zeros((N, OH, OW, IC * KH * KW), np.float16 if f16 else np.float32)
    assert gpu_lib.im2col(N, IC, IH, IW, ptr(X), IC * IH * IW, IH * IW, KH, KW, OH, OW, s0, s1, p0, p1, d0, d1,
                          ptr(Y), f16, 1) == 0, gpu_lib.error()
    want = ml_ref.im2col(X, KH, KW, OH, OW, s0, s1, p0, p1, d0, d1)
    assert np.array_equal(Y.astype(np.float32), want.astype(np.float16).astype(np.float32) if f16 else want)


ROPE_CASES = [  # neox, ff, ext_factor, freq_scale
    (0, False, 0.0, 1.0), (1, False, 0.0, 1.0), (1, True, 0.0, 1.0), (0, True, 1.0, 0.25), (1, False, 0.5, 0.5)]


@pytest.mark.parametrize("neox,use_ff,ext,fs", ROPE_CASES)
def test_rope(gpu_lib, neox, use_ff, ext, fs):
    n_tok, nh, n_dims = 7, 5, 64
    X = rng.standard_normal((n_tok, nh, n_dims)).astype(np.float32)
    pos = np.array([0, 1, 5, 100, 511, 2047, 3000], np.int32)
    ff = rng.uniform(1.0, 4.0, n_dims // 2).astype(np.float32) if use_ff else None
    corr = np.array([3.5, 21.25], np.float32)
    Y = np.zeros_like(X)
    assert gpu_lib.rope(n_dims, nh, n_tok, ptr(X), n_dims, nh * n_dims, ptr(Y), n_dims, nh * n_dims, ptr(pos), ptr(ff),
                        neox, 10000.0, fs, ext, 1.0, ptr(corr), 1) == 0, gpu_lib.error()
    want = ml_ref.rope(X, pos, ff, neox, 10000.0, fs, ext, 1.0, corr)
    # cosf / sinf of angles up to ~3000 rad: a few float32 ulps of the argument reduction
    assert np.max(np.abs(Y - want)) < 2e-5, np.max(np.abs(Y - want))
    Xd = dev(X)   # in place on the device
    assert gpu_lib.rope(n_dims, nh, n_tok, ptr(Xd), n_dims, nh * n_dims, ptr(Xd), n_dims, nh * n_dims, ptr(pos),
                        ptr(ff), neox, 10000.0, fs, ext, 1.0, ptr(corr), 0) == 0
    assert np.array_equal(host(Xd, gpu_lib), Y)
    # overlapping heads: the reference's layout rule
    assert gpu_lib.rope(n_dims, nh, n_tok, ptr(X), n_dims - 2, nh * n_dims, ptr(Y), n_dims, nh * n_dims, ptr(pos),
                        None, neox, 10000.0, fs, ext, 1.0, ptr(corr), 1) == -2


@pytest.mark.parametrize("vision,sections", [(0, (16, 8, 8, 0)), (0, (11, 5, 0, 3)), (1, (16, 16, 0, 0)),
                                             (1, (8, 0, 12, 12))])
@pytest.mark.parametrize("nh", [3, 9])   # 9: groups of four heads and a remainder
def test_rope_multi(gpu_lib, vision, sections, nh):
    n_tok, n_dims = 6, 64
    ne0 = 2 * n_dims if vision else n_dims
    X = rng.standard_normal((n_tok, nh, ne0)).astype(np.float32)
    pos = rng.integers(0, 600, 4 * n_tok).astype(np.int32)
    corr = np.array([0.0, 0.0], np.float32)
    sec = np.array(sections, np.int32)
    Y = np.zeros_like(X)
    assert gpu_lib.rope_multi(n_dims, nh, n_tok, ptr(X), ne0, nh * ne0, ptr(Y), ne0, nh * ne0, ptr(pos), None,
                              ptr(sec), 10000.0, 1.0, 0.0, 1.0, ptr(corr), vision, 1) == 0, gpu_lib.error()
    want = ml_ref.rope_multi(X, pos, None, sections, vision, 10000.0, 1.0, 0.0, 1.0, corr)
    assert np.max(np.abs(Y - want)) < 2e-5


def test_cpy_any(gpu_lib):
    S = rng.standard_normal((3, 4, 5, 6)).astype(np.float32)        # ggml ne = (6, 5, 4, 3)
    P = S.transpose(0, 2, 1, 3)                                       # a permuted view, as ggml_permute makes
    sne = (ctypes.c_int64 * 4)(*P.shape[::-1])
    snb = (ctypes.c_int64 * 4)(*P.strides[::-1])
    D = np.zeros(P.shape, np.float16)
    dne = (ctypes.c_int64 * 4)(*D.shape[::-1])
    dnb = (ctypes.c_int64 * 4)(*D.strides[::-1])
    assert gpu_lib.cpy_any(ptr(S), 1, ctypes.addressof(sne), ctypes.addressof(snb), ptr(D), 0, ctypes.addressof(dne),
                           ctypes.addressof(dnb), 1) == 0, gpu_lib.error()
    assert np.array_equal(D.view(np.uint16), P.astype(np.float16).view(np.uint16))
    R = np.zeros((12, 30), np.float32)                               # F16 -> F32 into another shape (CONT + reshape)
    rne = (ctypes.c_int64 * 4)(30, 12, 1, 1)
    rnb = (ctypes.c_int64 * 4)(4, 120, 1440, 1440)
    assert gpu_lib.cpy_any(ptr(D), 0, ctypes.addressof(dne), ctypes.addressof(dnb), ptr(R), 1, ctypes.addressof(rne),
                           ctypes.addressof(rnb), 1) == 0, gpu_lib.error()
    assert np.array_equal(R.ravel(), D.astype(np.float32).ravel())
    bad = (ctypes.c_int64 * 4)(30, 12, 2, 1)
    assert gpu_lib.cpy_any(ptr(D), 0, ctypes.addressof(dne), ctypes.addressof(dnb), ptr(R), 1, ctypes.addressof(bad),
                           ctypes.addressof(rnb), 1) == -2     # element counts differ


@pytest.mark.parametrize("mode", [0, 1, 1 | 256, 1 | 512])
@pytest.mark.parametrize("dshape", [(2, 3, 10, 14), (2, 3, 3, 2)])
def test_upscale(gpu_lib, mode, dshape):
    S = rng.standard_normal((2, 3, 5, 7)).astype(np.float32)
    D = np.zeros(dshape, np.float32)
    sne, snb = (ctypes.c_int64 * 4)(*S.shape[::-1]), (ctypes.c_int64 * 4)(*S.strides[::-1])
    dne, dnb = (ctypes.c_int64 * 4)(*D.shape[::-1]), (ctypes.c_int64 * 4)(*D.strides[::-1])
    assert gpu_lib.upscale_f32(ptr(S), ctypes.addressof(sne), ctypes.addressof(snb), ptr(D), ctypes.addressof(dne),
                               ctypes.addressof(dnb), mode, 1) == 0, gpu_lib.error()
    want = ml_ref.upscale(S, dshape, mode)
    assert np.allclose(D, want, rtol=1e-6, atol=1e-6), np.max(np.abs(D - want))


@pytest.mark.parametrize("idx64", [0, 1])
def test_set_rows_f16(gpu_lib, idx64):
    nc, nr, ne02, ne03, ne1 = 64, 5, 4, 2, 32
    src = rng.standard_normal((ne03, ne02, nr, nc)).astype(np.float32)
    idx = np.stack([rng.permutation(ne1)[:nr] for _ in range(2)]).astype(np.int64 if idx64 else np.int32)  # [ne11=2]
    dst = dev(np.zeros((ne03, ne02, ne1, nc), np.float16))
    es = idx.itemsize
    bad = ctypes.c_int(-1)
    assert gpu_lib.set_rows_f16(nc, nr, ne02, ne03, ptr(src), nc, nr * nc, ne02 * nr * nc, ptr(idx), idx.nbytes, es,
                                nr * es, 0, idx64, 2, 1, ptr(dst), dst.numel() * 2, nc, ne1 * nc, ne02 * ne1 * nc, ne1, 1,
                                ctypes.addressof(bad)) == 0, gpu_lib.error()
    def expected():
        want = np.zeros((ne03, ne02, ne1, nc), np.float16)
        for i3 in range(ne03):
            for i2 in range(ne02):
                for i in range(nr):
                    if 0 <= idx[i2 % 2, i] < ne1:
                        want[i3, i2, idx[i2 % 2, i]] = src[i3, i2, i].astype(np.float16)
        return want

    got = host(dst, gpu_lib)
    assert bad.value == 0 and np.array_equal(got.view(np.uint16), expected().view(np.uint16))
    idx[0, 1] = ne1                                                    # out of range: reported, that row not written
    dst.zero_()
    torch.cuda.synchronize()
    assert gpu_lib.set_rows_f16(nc, nr, ne02, ne03, ptr(src), nc, nr * nc, ne02 * nr * nc, ptr(idx), idx.nbytes, es,
                                nr * es, 0, idx64, 2, 1, ptr(dst), dst.numel() * 2, nc, ne1 * nc, ne02 * ne1 * nc, ne1, 1,
                                ctypes.addressof(bad)) == 0
    assert bad.value == 1
    assert np.array_equal(host(dst, gpu_lib).view(np.uint16), expected().view(np.uint16))


# ------------------------------------------------------------------------------------------- attention
def _close_attn(got, want):
    # FP32 scores and sums over up to ~1000 keys against float64
    return np.max(np.abs(got - want)) <= 2e-5 * max(1.0, np.max(np.abs(want)))


@pytest.mark.parametrize("pad", [5, 8])
@pytest.mark.parametrize("D,H,HKV", [(128, 32, 8), (128, 8, 8), (64, 12, 2), (96, 16, 2), (128, 36, 4), (80, 32, 32),
                                     (112, 16, 2), (16, 8, 1)])
def test_attn_dec_streams(gpu_lib, D, H, HKV, pad):
    """Row padding 8 (16-byte rows, D a multiple of 16, at most 8 query heads per KV head) takes the tensor-core
    kernel, padding 5 and the 9-heads-per-KV-head case the per-head one."""
    ns, nq, nk = 3, 2, 700
    Q = dev(rng.standard_normal((ns, nq, H, D)).astype(np.float32))
    # llama.cpp cache layout with padding: [s][key][g][D + pad]
    Kc = rng.standard_normal((ns, nk + 9, HKV, D + pad)).astype(np.float16)
    Vc = rng.standard_normal((ns, nk + 9, HKV, D + pad)).astype(np.float16)
    Kd, Vd = dev(Kc), dev(Vc)
    O = dev(np.full((ns, nq, H, D), np.nan, np.float32))
    vis = np.array([1, 300, 699], np.int32)
    kk, kh, ks = HKV * (D + pad), D + pad, (nk + 9) * HKV * (D + pad)
    scale = 1.0 / np.sqrt(D)
    assert gpu_lib.attn_dec_supported(D, H, HKV) == 1
    assert gpu_lib.attn_dec(D, H, HKV, ns, nq, nk, ptr(Q), H * D, D, nq * H * D, ptr(Kd), kk, kh, ks, Kd.numel() * 2,
                            ptr(Vd), kk, kh, ks, Vd.numel() * 2, ptr(O), scale, ptr(vis), 1, 64, 1) == 0, gpu_lib.error()
    got = host(O, gpu_lib)
    Qh = Q.cpu().numpy()
    for s in range(ns):
        want = ml_ref.attention(Qh[s], Kc[s, :nk, :, :D], Vc[s, :nk, :, :D], scale,
                                [min(vis[s] + t, nk) for t in range(nq)])
        assert _close_attn(got[s], want), s


@pytest.mark.parametrize("qmul", [1e-6, 1.0, 3e3])
def test_attn_dec_query_scales(gpu_lib, qmul):
    """Tiny and huge queries: the tensor-core kernel splits each head's scaled query into two FP16 parts after a
    power-of-two normalisation, so neither underflows nor overflows; 3e3 makes the softmax nearly one-hot."""
    D, H, HKV, ns, nq, nk = 64, 8, 2, 2, 1, 300
    Q = dev((rng.standard_normal((ns, nq, H, D)) * qmul).astype(np.float32))
    Kc = rng.standard_normal((ns, nk, HKV, D)).astype(np.float16)
    Vc = rng.standard_normal((ns, nk, HKV, D)).astype(np.float16)
    Kd, Vd = dev(Kc), dev(Vc)
    O = dev(np.full((ns, nq, H, D), np.nan, np.float32))
    vis = np.array([77, 300], np.int32)
    kk, kh, ks, scale = HKV * D, D, nk * HKV * D, 0.125
    assert gpu_lib.attn_dec(D, H, HKV, ns, nq, nk, ptr(Q), H * D, D, nq * H * D, ptr(Kd), kk, kh, ks, Kd.numel() * 2,
                            ptr(Vd), kk, kh, ks, Vd.numel() * 2, ptr(O), scale, ptr(vis), 0, 64, 1) == 0, gpu_lib.error()
    got = host(O, gpu_lib)
    Qh = Q.cpu().numpy()
    for s in range(ns):
        want = ml_ref.attention(Qh[s], Kc[s], Vc[s], scale, [int(vis[s])])
        assert _close_attn(got[s], want), (s, np.max(np.abs(got[s] - want)))


def test_attn_dec_nan_past_visible(gpu_lib):
    """Cache rows past each stream's visible count hold NaN (an unwritten llama.cpp cache may): the tensor-core kernel
    may copy them (its first step is requested before the count is read) but masks their scores and zeroes their
    values, so the outputs stay finite and equal the oracle's over the visible rows."""
    D, H, HKV, ns, nq, nk = 128, 32, 8, 4, 1, 200
    Q = dev(rng.standard_normal((ns, nq, H, D)).astype(np.float32))
    Kc = rng.standard_normal((ns, nk, HKV, D)).astype(np.float16)
    Vc = rng.standard_normal((ns, nk, HKV, D)).astype(np.float16)
    vis = np.array([1, 37, 200, 96], np.int32)
    Kn, Vn = Kc.copy(), Vc.copy()
    for s_ in range(ns):
        Kn[s_, vis[s_]:] = np.nan
        Vn[s_, vis[s_]:] = np.nan
    Kd, Vd = dev(Kn), dev(Vn)
    O = dev(np.full((ns, nq, H, D), np.nan, np.float32))
    kk, kh, ks, scale = HKV * D, D, nk * HKV * D, D ** -0.5
    for _ in range(2):   # twice: the per-row arrival counters are back at zero after a call
        assert gpu_lib.attn_dec(D, H, HKV, ns, nq, nk, ptr(Q), H * D, D, nq * H * D, ptr(Kd), kk, kh, ks,
                                Kd.numel() * 2, ptr(Vd), kk, kh, ks, Vd.numel() * 2, ptr(O), scale, ptr(vis), 0, 64,
                                1) == 0, gpu_lib.error()
        got = host(O, gpu_lib)
        assert np.all(np.isfinite(got))
        Qh = Q.cpu().numpy()
        for s_ in range(ns):
            want = ml_ref.attention(Qh[s_], Kc[s_], Vc[s_], scale, [int(vis[s_])])
            assert _close_attn(got[s_], want), (s_, np.max(np.abs(got[s_] - want)))


@pytest.mark.parametrize("nk,vis", [(20000, 19999), (20000, 12345)])
def test_attn_dec_one_row_many_slots(gpu_lib, nk, vis):
    """One (stream, KV head) row split over the whole grid: the merging CTA combines hundreds of slots, more than a
    warp's 32 lanes take in one pass (the weights of earlier passes are rescaled to the running maximum)."""
    D, H, HKV, ns, nq = 64, 8, 1, 1, 1
    Q = dev(rng.standard_normal((ns, nq, H, D)).astype(np.float32))
    Kc = rng.standard_normal((ns, nk, HKV, D)).astype(np.float16)
    Vc = rng.standard_normal((ns, nk, HKV, D)).astype(np.float16)
    Kc[0, 7777] *= 3   # a few keys far above the rest: the running maximum moves between passes
    Kd, Vd = dev(Kc), dev(Vc)
    O = dev(np.full((ns, nq, H, D), np.nan, np.float32))
    vv = np.array([vis], np.int32)
    kk, kh, ks, scale = HKV * D, D, nk * HKV * D, 0.125
    assert gpu_lib.attn_dec(D, H, HKV, ns, nq, nk, ptr(Q), H * D, D, nq * H * D, ptr(Kd), kk, kh, ks, Kd.numel() * 2,
                            ptr(Vd), kk, kh, ks, Vd.numel() * 2, ptr(O), scale, ptr(vv), 0, 64, 1) == 0, gpu_lib.error()
    got = host(O, gpu_lib)
    want = ml_ref.attention(Q.cpu().numpy()[0], Kc[0], Vc[0], scale, [vis])
    assert _close_attn(got[0], want), np.max(np.abs(got[0] - want))


def test_attn_dec_long_chunks(gpu_lib):
    """Enough (stream, KV head) rows that the planner gives each warp several 32-key steps (the copy of the next
    step's rows overlapping this step's MMAs), with visible counts that end inside a step, a warp and a chunk."""
    D, H, HKV, ns, nq, nk = 128, 32, 8, 16, 1, 8192
    g = torch.Generator(device="cuda")
    g.manual_seed(21)
    Kd = torch.randn(ns, nk, HKV, D, device="cuda", generator=g).half()
    Vd = torch.randn(ns, nk, HKV, D, device="cuda", generator=g).half()
    Q = torch.randn(ns, nq, H, D, device="cuda", generator=g)
    O = torch.full((ns, nq, H, D), float("nan"), device="cuda")
    vis = np.array([8192, 1, 31, 33, 127, 129, 640, 641, 1000, 2047, 4097, 5000, 6143, 7777, 8191, 3], np.int32)
    kk, kh, ks, scale = HKV * D, D, nk * HKV * D, D ** -0.5
    torch.cuda.synchronize()   # the tensors are written by torch's stream; the library runs on its own
    assert gpu_lib.attn_dec(D, H, HKV, ns, nq, nk, Q.data_ptr(), H * D, D, nq * H * D, Kd.data_ptr(), kk, kh, ks,
                            Kd.numel() * 2, Vd.data_ptr(), kk, kh, ks, Vd.numel() * 2, O.data_ptr(), scale, ptr(vis),
                            0, 64, 1) == 0, gpu_lib.error()
    got = O.cpu().numpy()
    Qh, Kh, Vh = Q.cpu().numpy(), Kd.cpu().numpy(), Vd.cpu().numpy()
    for s in range(ns):
        want = ml_ref.attention(Qh[s], Kh[s], Vh[s], scale, [int(vis[s])])
        assert _close_attn(got[s], want), (s, int(vis[s]), np.max(np.abs(got[s] - want)))


def test_attn_f16kv_prefill_causal_and_streams(gpu_lib):
    D, H, HKV, nq, nk = 128, 16, 4, 37, 300
    Q = dev(rng.standard_normal((nq, H, D)).astype(np.float32))
    Kh = rng.standard_normal((nk, HKV, D)).astype(np.float16)
    Vh = rng.standard_normal((nk, HKV, D)).astype(np.float16)
    Kd, Vd = dev(Kh), dev(Vh)
    O = dev(np.zeros((nq, H, D), np.float32))
    vis0, scale = nk - nq + 1, 0.088
    launches = ctypes.c_int(-1)
    assert gpu_lib.attn_supported(D, H, HKV) == 1
    assert gpu_lib.attn_f16kv(D, H, HKV, nq, nk, ptr(Q), ptr(Kd), Kd.numel() * 2, ptr(Vd), Vd.numel() * 2, ptr(O), scale,
                              vis0, 1, ctypes.addressof(launches)) == 0, gpu_lib.error()
    assert launches.value == 1
    want = ml_ref.attention(Q.cpu().numpy(), Kh, Vh, scale, [min(vis0 + t, nk) for t in range(nq)])
    assert _close_attn(host(O, gpu_lib), want)
    # unsupported shape: declined, nothing written
    assert gpu_lib.attn_supported(256, H, HKV) == 0
    assert gpu_lib.attn_f16kv(256, H, HKV, nq, nk, ptr(Q), ptr(Kd), 0, ptr(Vd), 0, ptr(O), scale, vis0, 1, None) == 1
    # two streams in one call
    ns = 2
    Q2 = dev(rng.standard_normal((ns, nq, H, D)).astype(np.float32))
    K2 = rng.standard_normal((ns, nk, HKV, D)).astype(np.float16)
    V2 = rng.standard_normal((ns, nk, HKV, D)).astype(np.float16)
    K2d, V2d = dev(K2), dev(V2)
    O2 = dev(np.zeros((ns, nq, H, D), np.float32))
    v0 = np.array([5, nk - nq + 1], np.int32)
    assert gpu_lib.attn_streams_supported(D, H, HKV) == 1
    assert gpu_lib.attn_f16kv_streams(D, H, HKV, ns, nq, nk, ptr(Q2), nq * H * D, ptr(K2d), nk * HKV * D,
                                      K2d.numel() * 2, ptr(V2d), nk * HKV * D, V2d.numel() * 2, ptr(O2), scale, ptr(v0),
                                      1, ctypes.addressof(launches)) == 0, gpu_lib.error()
    got = host(O2, gpu_lib)
    Qn = Q2.cpu().numpy()
    for s in range(ns):
        want = ml_ref.attention(Qn[s], K2[s], V2[s], scale, [min(v0[s] + t, nk) for t in range(nq)])
        assert _close_attn(got[s], want), s
