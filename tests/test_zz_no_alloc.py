"""gen9blas_gemv_noalloc: the gemv entry point for callers that must not allocate GPU memory (loops that cannot take
the device-wide synchronisation of cudaMalloc/cudaFree, processes that hand all device memory to their own pool).
Its transposed product keeps the split-row partial sums in a fixed 8 MiB array of the library's device image
instead of the grow-only scratch buffer that gen9blas_gemv uses.

Checked through the C ABI on device-resident operands: two calls in a row, each equal (within the level-2
tolerances) to the output of the existing gen9blas_gemv and to alpha·op(A)·x + beta·y in FP64 NumPy; in no-wait
mode, ordered after a gen9blas_gemm that writes its A and waited for by gen9blas_flush; no growth of device memory
use across calls that would need more scratch; oversize N rejected with a clear error before any launch. This file
sorts last so that a run that stops at the first failure has already run every other test; it also passes alone in
a fresh process."""
import ctypes

import numpy as np
import pytest

import abi

pytestmark = pytest.mark.gpu
TOL = {abi.S: 1e-6, abi.H: 2e-3, abi.D: 1e-13}


@pytest.fixture(scope="module")
def torch():
    return pytest.importorskip("torch")


def scaled_error(got, ref, scale):
    return float((np.abs(got.astype(np.float64) - ref.astype(np.float64)) / np.maximum(scale, 1e-30)).max())


@pytest.mark.parametrize("t,dtname", [(abi.S, "float32"), (abi.H, "float16"), (abi.D, "float64")])
def test_noalloc_matches_gemv_twice(gpu_lib, torch, t, dtname):
    dt = getattr(torch, dtname)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(31)
    for (M, N, trans, incx, incy, beta) in ((1000, 3000, 1, 1, 1, 0.0), (3001, 513, 1, 2, -1, 0.5),
                                            (700, 900, 0, 1, 1, -1.0), (32768, 4096, 1, 1, 1, 0.0)):
        lda = N + 3
        A = torch.empty(M, lda, device="cuda", dtype=torch.float64).uniform_(-1, 1, generator=gen).to(dt)
        nx, ny = (M, N) if trans else (N, M)
        x = torch.empty(nx * incx, device="cuda", dtype=torch.float64).uniform_(-1, 1, generator=gen).to(dt)
        y0 = torch.empty(ny * abs(incy), device="cuda", dtype=torch.float64).uniform_(-1, 1, generator=gen).to(dt)
        y_ref, y1, y2 = y0.clone(), y0.clone(), y0.clone()
        torch.cuda.synchronize()
        args = (t, trans, M, N, 0.75, A.data_ptr(), lda, x.data_ptr(), incx, beta)
        assert gpu_lib.gemv(*args, y_ref.data_ptr(), incy) == 0, gpu_lib.error()
        assert gpu_lib.gemv_noalloc(*args, y1.data_ptr(), incy) == 0, gpu_lib.error()
        assert gpu_lib.gemv_noalloc(*args, y2.data_ptr(), incy) == 0, gpu_lib.error()
        torch.cuda.synchronize()
        Ad = A[:, :N].double().cpu().numpy()
        xs = x.double().cpu().numpy()[::incx]
        opA = Ad.T if trans else Ad
        y0m = y0.double().cpu().numpy()[::abs(incy)]                     # memory order (incy < 0: element 0 is last)
        y0l = y0m[::-1] if incy < 0 else y0m                              # logical order
        ref64 = 0.75 * (opA @ xs) + beta * y0l
        scale = 0.75 * (np.abs(opA) @ np.abs(xs))
        if incy < 0:
            ref64, scale = ref64[::-1], scale[::-1]
        scale = scale + abs(beta) * np.abs(y0m)
        ref = y_ref.cpu().numpy()[::abs(incy)]
        for got in (y1, y2):
            g = got.cpu().numpy()[::abs(incy)]
            assert scaled_error(g, ref, scale) <= TOL[t], (t, M, N, trans)      # same as gen9blas_gemv
            assert scaled_error(g, ref64, scale) <= TOL[t], (t, M, N, trans)    # and as FP64 NumPy


def test_noalloc_nowait_orders_after_gemm_and_flush_waits(gpu_lib, torch):
    """No-wait mode: a gen9blas_gemm writes the matrix that gen9blas_gemv_noalloc then reads; neither call waits, and
    gen9blas_flush must cover both (the noalloc call runs on the library's stream once the device is set up)."""
    gen = torch.Generator(device="cuda")
    gen.manual_seed(11)
    M, N, K = 2048, 3072, 256
    P = torch.empty(M, K, device="cuda", dtype=torch.float32).uniform_(-1, 1, generator=gen)
    Q = torch.empty(K, N, device="cuda", dtype=torch.float32).uniform_(-1, 1, generator=gen)
    x = torch.empty(M, device="cuda", dtype=torch.float32).uniform_(-1, 1, generator=gen)
    torch.cuda.synchronize()
    for rep in range(2):
        A = torch.full((M, N), float("nan"), device="cuda", dtype=torch.float32)
        y = torch.full((N,), float("nan"), device="cuda", dtype=torch.float32)
        torch.cuda.synchronize()
        gpu_lib.set_nowait(1)
        try:
            assert gpu_lib.gemm(abi.S, 0, 0, M, N, K, 1.0, P.data_ptr(), K, Q.data_ptr(), N, 0.0, A.data_ptr(), N) == 0
            assert gpu_lib.gemv_noalloc(abi.S, 1, M, N, 1.0, A.data_ptr(), N, x.data_ptr(), 1, 0.0, y.data_ptr(), 1) == 0
            assert gpu_lib.flush() == 0, gpu_lib.error()
        finally:
            gpu_lib.set_nowait(0)
        Ad = P.double().cpu().numpy() @ Q.double().cpu().numpy()
        xs = x.double().cpu().numpy()
        ref = Ad.T @ xs
        scale = np.abs(Ad.T) @ np.abs(xs)
        assert scaled_error(y.cpu().numpy(), ref, scale) <= 1e-5, rep


def test_noalloc_records_into_a_cuda_graph(gpu_lib, torch):
    """Called on a stream that is being captured (set with gen9blas_set_stream, no-wait mode off), the call records
    its launches and returns without waiting; each replay of the graph then computes y from the buffers' contents
    at replay time."""
    gen = torch.Generator(device="cuda")
    gen.manual_seed(17)
    M, N = 3000, 2000
    A = torch.empty(M, N, device="cuda", dtype=torch.float32).uniform_(-1, 1, generator=gen)
    x = torch.empty(M, device="cuda", dtype=torch.float32).uniform_(-1, 1, generator=gen)
    y = torch.zeros(N, device="cuda", dtype=torch.float32)
    torch.cuda.synchronize()
    # the first call looks up the fixed scratch array's address, which must happen before any capture
    assert gpu_lib.gemv_noalloc(abi.S, 1, M, N, 1.0, A.data_ptr(), N, x.data_ptr(), 1, 0.0, y.data_ptr(), 1) == 0
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, capture_error_mode="relaxed"):
        assert gpu_lib.set_stream(torch.cuda.current_stream().cuda_stream) == 0
        try:
            r = gpu_lib.gemv_noalloc(abi.S, 1, M, N, 0.5, A.data_ptr(), N, x.data_ptr(), 1, 0.0, y.data_ptr(), 1)
        finally:
            gpu_lib.set_stream(None)
    assert r == 0, gpu_lib.error()
    for rep in range(2):
        A.uniform_(-1, 1, generator=gen)
        x.uniform_(-1, 1, generator=gen)
        y.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        Ad, xs = A.double().cpu().numpy(), x.double().cpu().numpy()
        ref = 0.5 * (Ad.T @ xs)
        scale = 0.5 * (np.abs(Ad.T) @ np.abs(xs))
        assert scaled_error(y.cpu().numpy(), ref, scale) <= TOL[abi.S], rep
    del g


def test_noalloc_uses_no_new_device_memory(gpu_lib, torch):
    """After the first call (which loads the library's device image, fixed array included) larger transposed
    problems, which would grow gen9blas_gemv's scratch, leave the free device memory unchanged."""
    gen = torch.Generator(device="cuda")
    gen.manual_seed(5)
    A = torch.empty(8192, 60000, device="cuda", dtype=torch.float32).uniform_(-1, 1, generator=gen)
    x = torch.empty(8192, device="cuda", dtype=torch.float32).uniform_(-1, 1, generator=gen)
    y = torch.zeros(60000, device="cuda", dtype=torch.float32)
    torch.cuda.synchronize()
    assert gpu_lib.gemv_noalloc(abi.S, 1, 64, 1000, 1.0, A.data_ptr(), 60000, x.data_ptr(), 1, 0.0, y.data_ptr(), 1) == 0
    free0 = torch.cuda.mem_get_info()[0]
    for N in (30000, 60000):
        assert gpu_lib.gemv_noalloc(abi.S, 1, 8192, N, 1.0, A.data_ptr(), 60000, x.data_ptr(), 1, 0.0, y.data_ptr(), 1) == 0
    assert torch.cuda.mem_get_info()[0] == free0


def test_noalloc_rejects_oversize_and_host_memory(gpu_lib, torch):
    A = torch.zeros(2, 3_000_000, device="cuda", dtype=torch.float32)
    x = torch.zeros(2, device="cuda", dtype=torch.float32)
    y = torch.zeros(3_000_000, device="cuda", dtype=torch.float32)
    torch.cuda.synchronize()
    launches = gpu_lib.kernel_launches()
    r = gpu_lib.gemv_noalloc(abi.S, 1, 2, 3_000_000, 1.0, A.data_ptr(), 3_000_000, x.data_ptr(), 1, 0.0, y.data_ptr(), 1)
    assert r == -3 and b"scratch" in gpu_lib.error()
    assert gpu_lib.kernel_launches() == launches           # rejected before any launch
    h = np.zeros(16, np.float32)
    r = gpu_lib.gemv_noalloc(abi.S, 0, 4, 4, 1.0, h.ctypes.data, 4, h.ctypes.data, 1, 0.0, h.ctypes.data, 1)
    assert r == -3 and b"device" in gpu_lib.error()
