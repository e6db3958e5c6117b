"""The multi-GPU partitioning logic (gen9-gpu-blas_b200/g9dist.py) with world_size-2 gloo ranks on the CPU: shard
bounds cover every column once, the chunked column-sharded GEMM with its all-gather and re-layout reproduces the full
product, and so does the row-sharded (tensor-parallel) skinny GEMM. The local products use a CPU stand-in (torch
matmul in FP64) so that only the distribution is under test; the GPU kernels are covered by the -m gpu tests."""
import os
import socket
import time

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import g9dist


def test_shard_bounds():
    for n, world, align in ((32768, 8, 256), (1000, 3, 1), (7, 4, 1), (4096, 2, 128)):
        b = g9dist.shard_bounds(n, world, align)
        covered = [i for a, z in b for i in range(a, z)]
        assert covered == list(range(n))
        assert all(a % align == 0 for a, z in b if z > a)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(5)
        M, K, N = 24, 40, 64
        A = torch.randn(M, K, generator=g, dtype=torch.float64)
        B = torch.randn(K, N, generator=g, dtype=torch.float64)
        nb = N // world
        B_shard = B[:, rank * nb:(rank + 1) * nb].contiguous()
        C = torch.zeros(M, N, dtype=torch.float64)

        def local(Ap, Bp, Cp):
            Cp.copy_(Ap @ Bp)

        g9dist.column_sharded_gemm(A, B_shard, C, rank, world, local, chunks=4)
        ok1 = torch.allclose(C, A @ B, rtol=0, atol=1e-12)
        # tensor-parallel skinny: W rows split over the ranks
        W = torch.randn(N, K, generator=g, dtype=torch.float64)
        Ws = W[rank * nb:(rank + 1) * nb].contiguous()
        A2 = torch.randn(3, K, generator=g, dtype=torch.float64)
        C2 = torch.zeros(3, N, dtype=torch.float64)

        def local_skinny(Ap, Wp, Cp):
            Cp.copy_(Ap @ Wp.T)

        g9dist.row_sharded_skinny(A2, Ws, C2, rank, world, local_skinny)
        ok2 = torch.allclose(C2, A2 @ W.T, rtol=0, atol=1e-12)
        out[rank] = (bool(ok1), bool(ok2))
    finally:
        dist.destroy_process_group()


def test_sharded_gemm_and_skinny_two_gloo_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert dict(out) == {0: (True, True), 1: (True, True)}


def _fault_worker(rank, world, port, fault_rank, fault, out):
    """One gloo rank of a 2-rank job in which rank fault_rank fails on purpose (GEN9BLAS_FAULT on that rank only);
    records (stage, status) of the CommError each rank sees, then leaves without touching the broken group."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    if rank == fault_rank and fault != "absent":
        os.environ["GEN9BLAS_FAULT"] = fault
    else:
        os.environ.pop("GEN9BLAS_FAULT", None)
    try:
        g9dist.init_comm("gloo", timeout_s=4.0, rank=rank, world_size=world)
        if rank == fault_rank and fault == "absent":   # alive, but never takes part in the collective
            time.sleep(8.0)
            out[rank] = ("absent", 0)
            return
        M, K, N = 8, 16, 32
        A = torch.ones(M, K, dtype=torch.float64)
        B_shard = torch.ones(K, N // world, dtype=torch.float64)
        C = torch.zeros(M, N, dtype=torch.float64)
        g9dist.column_sharded_gemm(A, B_shard, C, rank, world, lambda a, b, c: c.copy_(a @ b), chunks=2, timeout_s=3.0)
        out[rank] = ("ok", 0)
    except g9dist.CommError as e:
        out[rank] = (e.stage, e.status)
    finally:
        os._exit(0)   # the group may hold a collective that will never complete: no orderly teardown


def _run_fault(fault):
    world = 2
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_fault_worker, args=(r, world, port, 1, fault, out)) for r in range(world)]
    # (fault "absent": rank 1 joins the group but skips the collective)
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return dict(out)


def test_injected_collective_failure_reaches_every_rank_as_a_status():
    """GEN9BLAS_FAULT=nccl_op on rank 1: rank 1 fails at its first collective (stage "collective"), rank 0's gather
    never completes and its host deadline turns that into stage "timeout"; both report GEN9BLAS_ERR (-1)."""
    res = _run_fault("nccl_op")
    assert res[1] == ("collective", g9dist.GEN9BLAS_ERR), res
    # rank 0 learns it from the backend (the peer's connection closed) or, failing that, from its deadline
    assert res[0] in (("collective", g9dist.GEN9BLAS_ERR), ("timeout", g9dist.GEN9BLAS_ERR)), res


def test_rank_that_never_joins_is_a_timeout():
    """Rank 1 stays alive but never takes part: rank 0's all-gather misses its host deadline (stage "timeout",
    GEN9BLAS_ERR) instead of waiting for the process group's long timeout."""
    t0 = time.monotonic()
    res = _run_fault("absent")
    assert res[0] == ("timeout", g9dist.GEN9BLAS_ERR) and res[1] == ("absent", 0), res
    assert time.monotonic() - t0 < 40


def test_injected_init_failure_reaches_every_rank_as_a_status():
    """GEN9BLAS_FAULT=nccl_init on rank 1: rank 1 never joins; rank 0's rendezvous times out; both raise CommError
    with stage "init" and GEN9BLAS_ERR."""
    res = _run_fault("nccl_init")
    assert res == {0: ("init", g9dist.GEN9BLAS_ERR), 1: ("init", g9dist.GEN9BLAS_ERR)}, res
