"""One-GPU checks of the multi-GPU building blocks: the fused skinny GEMM + all-gather (tensor-parallel decode) stores
its block into every destination buffer, and the NVLink rank barrier (gen9blas_peer_barrier) passes when every flag
is raised and gives up cleanly -- GEN9BLAS_ERR, device still usable -- when a flag never comes (a rank that did not
arrive). Two local buffers stand in for two ranks; nothing here faults or hangs a GPU."""
import ctypes

import pytest

import abi

pytestmark = pytest.mark.gpu
ERR = -1


def _allgather_fn(gpu_lib):
    f = gpu_lib.dll.gen9blas_gemm_allgather
    f.argtypes = [ctypes.c_int] * 6 + [ctypes.c_double, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                       ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int64]
    return f


@pytest.mark.parametrize("M", [1, 8, 16])
def test_skinny_allgather_writes_every_destination(gpu_lib, M):
    torch = pytest.importorskip("torch")
    K, N, nr, off = 1024, 2048, 512, 1024
    g = torch.Generator(device="cuda").manual_seed(M)
    X = torch.randn(M, K, device="cuda", generator=g, dtype=torch.float16)
    W = (torch.randn(nr, K, device="cuda", generator=g) * 0.02).half()     # this rank's weight rows
    C1 = torch.full((M, N), 7.0, device="cuda", dtype=torch.float16)
    C2 = torch.full((M, N), 7.0, device="cuda", dtype=torch.float16)
    torch.cuda.synchronize()
    gpu_lib.set_nowait(0)
    arr = (ctypes.c_void_p * 2)(C1.data_ptr(), C2.data_ptr())
    f = _allgather_fn(gpu_lib)
    for t in (abi.H, abi.HS):
        assert f(t, 0, 1, M, nr, K, 1.0, X.data_ptr(), K, W.data_ptr(), K, arr, 2, N, off) == 0, gpu_lib.error()
        torch.cuda.synchronize()
        ref = X.double() @ W.double().t()
        scale = X.double().abs() @ W.double().abs().t()
        for C in (C1, C2):
            blk = C[:, off:off + nr].double()
            assert float(((blk - ref).abs() / scale).max()) <= 1e-3
            rest = torch.cat([C[:, :off], C[:, off + nr:]], 1)
            assert bool((rest == 7.0).all())


def test_peer_barrier_single_rank_and_timeout(gpu_lib):
    torch = pytest.importorskip("torch")
    gpu_lib.set_nowait(0)
    one_flags = torch.zeros(2, dtype=torch.int32, device="cuda")   # 1 rank: flag + counter
    torch.cuda.synchronize()
    one = (ctypes.c_void_p * 1)(one_flags.data_ptr())
    for _ in range(3):
        assert gpu_lib.peer_barrier(one, 1, 0, 1000.0) == 0, gpu_lib.error()
    assert one_flags.tolist() == [3, 3]                                # epochs 1, 2, 3 counted on the device
    # Two ranks, but rank 1 never arrives: rank 0 raises its flag in both arrays, then gives up after 50 ms.
    mine = torch.zeros(3, dtype=torch.int32, device="cuda")
    other = torch.zeros(3, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    two = (ctypes.c_void_p * 2)(mine.data_ptr(), other.data_ptr())
    assert gpu_lib.peer_barrier(two, 2, 0, 50.0) == ERR
    assert b"gave up" in gpu_lib.error()
    assert mine.tolist() == [1, 0, 1] and other.tolist() == [1, 0, 0]
    # The device is intact, and the next barrier (epoch 2) passes once rank 1's flag shows epoch 2.
    mine[1] = 2
    torch.cuda.synchronize()
    assert gpu_lib.peer_barrier(two, 2, 0, 1000.0) == 0, gpu_lib.error()
    assert mine.tolist() == [2, 2, 2]
    a = torch.ones(64, 64, device="cuda")
    c = torch.zeros(64, 64, device="cuda")
    torch.cuda.synchronize()
    assert gpu_lib.gemm(abi.S, 0, 0, 64, 64, 64, 1.0, a.data_ptr(), 64, a.data_ptr(), 64, 0.0, c.data_ptr(), 64) == 0
    assert bool((c == 64).all())


def test_peer_barrier_rejects_bad_arguments(gpu_lib):
    torch = pytest.importorskip("torch")
    f = torch.zeros(2, dtype=torch.int32, device="cuda")
    arr = (ctypes.c_void_p * 2)(f.data_ptr(), None)
    assert gpu_lib.peer_barrier(arr, 2, 0, 10.0) == -3           # NULL flag array
    assert gpu_lib.peer_barrier(arr, 2, 2, 10.0) == -3           # rank out of range
    assert gpu_lib.peer_barrier(arr, 9, 0, 10.0) == -3           # too many ranks
