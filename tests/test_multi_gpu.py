"""Multi-GPU paths on real GPUs (skipped with fewer than 2): the fused GEMM + all-gather kernel writing into the
other rank's C over NVLink through CUDA IPC (ranks met by an NCCL all-reduce, then by the NVLink flag barrier), the
NCCL column-sharded GEMM, and the tensor-parallel skinny GEMM whose outputs go straight into every rank's C, all
against the full product."""
import os
import socket
import subprocess
import sys

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

CHILD = r'''
import ctypes, os, sys
import torch, torch.distributed as dist
sys.path.insert(0, os.path.join(sys.argv[1], "gen9-gpu-blas_b200"))
import g9dist
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
import datetime
dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
lib = ctypes.CDLL(os.path.join(sys.argv[1], "gen9-gpu-blas_b200", "libgen9blas.so"))
lib.gen9blas_error.restype = ctypes.c_char_p
assert lib.gen9blas_set_device(rank) == 0
M, K, N = 1024, 512, 2048
g = torch.Generator(device="cuda").manual_seed(11)
A = torch.randn(M, K, device="cuda", generator=g, dtype=torch.float16)
B = torch.randn(K, N, device="cuda", generator=g, dtype=torch.float16)
nb = N // world
Bs = B[:, rank * nb:(rank + 1) * nb].contiguous()
C = torch.zeros(M, N, device="cuda", dtype=torch.float16)
peers = g9dist.PeerView(lib, C, rank, world)
torch.cuda.synchronize()
g9dist.fused_column_sharded_gemm(lib, A, Bs, C, peers, rank, world)
torch.cuda.synchronize()
ref = A.double() @ B.double()
scale = A.double().abs() @ B.double().abs()
e1 = float(((C.double() - ref).abs() / scale).max())
C2 = torch.zeros(M, N, device="cuda", dtype=torch.float16)
g9dist.column_sharded_gemm(A, Bs, C2, rank, world, lambda a, b, c: g9dist.gemm_local(lib, a, b, c), chunks=4,
                           comm_stream=torch.cuda.Stream())
torch.cuda.synchronize()
e2 = float(((C2.double() - ref).abs() / scale).max())
# the same fused GEMM with the NVLink rank barrier instead of the NCCL all-reduce
bar = g9dist.PeerBarrier(lib, rank, world)
C.zero_()
torch.cuda.synchronize()
dist.barrier()   # every rank's C is zeroed before any rank stores into it
g9dist.fused_column_sharded_gemm(lib, A, Bs, C, peers, rank, world, barrier=bar)
torch.cuda.synchronize()
e3 = float(((C.double() - ref).abs() / scale).max())
# tensor-parallel decode: weight rows split over the ranks, outputs stored into every rank's C, barrier; three rounds
Mw, Kw, Nw = 8, 1024, 4096
W = (torch.randn(Nw, Kw, device="cuda", generator=g) * 0.02).half()
nr = Nw // world
Ws = W[rank * nr:(rank + 1) * nr].contiguous()
Cs = torch.zeros(Mw, Nw, device="cuda", dtype=torch.float16)
pv = g9dist.PeerView(lib, Cs, rank, world)
e4 = 0.0
for it in range(3):
    X = torch.randn(Mw, Kw, device="cuda", generator=g, dtype=torch.float16)
    torch.cuda.synchronize()
    g9dist.fused_row_sharded_skinny(lib, X, Ws, Cs, pv, rank, world, barrier=bar)
    torch.cuda.synchronize()
    r4 = X.double() @ W.double().t()
    s4 = X.double().abs() @ W.double().abs().t()
    e4 = max(e4, float(((Cs.double() - r4).abs() / s4).max()))
    dist.barrier()   # nobody overwrites Cs for the next round before every rank has checked this one
dist.barrier()
pv.close()
bar.close()
peers.close()
dist.destroy_process_group()
print("ERR", rank, e1, e2, e3, e4)
'''


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_fused_and_nccl_allgather_two_ranks():
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    port = _port()
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE="2", MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                   LOCAL_RANK=str(r), NCCL_NVLS_ENABLE="0")
        procs.append(subprocess.Popen([sys.executable, "-c", CHILD, ROOT], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.PIPE, text=True))
    outs = [p.communicate(timeout=300) for p in procs]
    for p, (o, e) in zip(procs, outs):
        assert p.returncode == 0, e[-2000:]
        line = [ln for ln in o.splitlines() if ln.startswith("ERR")][0].split()
        assert all(float(v) <= 1e-3 for v in line[2:6]), line


SWITCH_CHILD = r'''
import ctypes, os, sys
import numpy as np
sys.path.insert(0, os.path.join(sys.argv[1], "tests"))
import abi
L = abi.bind(ctypes.CDLL(os.path.join(sys.argv[1], "gen9-gpu-blas_b200", "libgen9blas.so")), "gen9blas_")
assert L.init() == 0, L.error()
rng = np.random.default_rng(5)
worst = 0.0
for dev in (0, 1, 0, 1):
    assert L.set_device(dev) == 0, L.error()
    for t, (M, N, K) in ((abi.H, (1024, 1024, 512)), (abi.HS, (96, 640, 256)), (abi.S, (512, 384, 256)),
                         (abi.D, (256, 320, 200))):
        dt = np.float16 if t in (abi.H, abi.HS) else np.float32 if t == abi.S else np.float64
        A = rng.uniform(-1, 1, (M, K)).astype(dt)
        B = rng.uniform(-1, 1, (K, N)).astype(dt)
        C = np.zeros((M, N), dt)
        r = L.gemm(t, 0, 0, M, N, K, 1.0, A.ctypes.data, K, B.ctypes.data, N, 0.0, C.ctypes.data, N)
        assert r == 0, (dev, t, L.error())
        a64, b64 = A.astype(np.float64), B.astype(np.float64)
        worst = max(worst, float((np.abs(C - a64 @ b64) / (np.abs(a64) @ np.abs(b64))).max()))
print("WORST", worst)
'''


def test_one_process_switches_devices():
    """One process runs the large-shared-memory kernels (tcgen05 HGEMM pair and 1-CTA kernels, SGEMM, DGEMM) on device
    0, then device 1, then both again through gen9blas_set_device: each kernel's shared-memory limit is raised on
    every device it runs on."""
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    r = subprocess.run([sys.executable, "-c", SWITCH_CHILD, ROOT], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    worst = float([ln for ln in r.stdout.splitlines() if ln.startswith("WORST")][0].split()[1])
    assert worst <= 1e-3, worst
