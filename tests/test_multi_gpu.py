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
# per shape (2048 rows and K = 1024 per rank: the stream-K kernel; 4096 rows and K = 2048: one row block per CTA)
e4 = 0.0
for Mw, Kw, Nw in ((8, 1024, 4096), (8, 2048, 4096 * world)):
    W = (torch.randn(Nw, Kw, device="cuda", generator=g) * 0.02).half()
    nr = Nw // world
    Ws = W[rank * nr:(rank + 1) * nr].contiguous()
    Cs = torch.zeros(Mw, Nw, device="cuda", dtype=torch.float16)
    pv = g9dist.PeerView(lib, Cs, rank, world)
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
dist.barrier()
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


SHARD_CHILD = r'''
import ctypes, os, sys
import numpy as np
import torch
sys.path.insert(0, os.path.join(sys.argv[1], "tests"))
sys.path.insert(0, os.path.join(sys.argv[1], "gen9-gpu-blas_b200"))
import abi
L = abi.bind(ctypes.CDLL(os.path.join(sys.argv[1], "gen9-gpu-blas_b200", "libgen9blas.so")), "gen9blas_")
assert L.init() == 0, L.error()
ids = (ctypes.c_int * 8)()
assert L.get_devices(ids, 8) == 2 and list(ids[:2]) == [0, 1]       # from GEN9BLAS_DEVICES
free1 = torch.cuda.mem_get_info(1)[0]
rng = np.random.default_rng(3)
out = {}
def err(C, A64, B64, rows, alpha=1.0, beta=0.0, C0=None):
    ref = alpha * A64[rows] @ B64 + (beta * C0[rows] if C0 is not None else 0)
    sc = abs(alpha) * np.abs(A64[rows]) @ np.abs(B64) + (abs(beta) * np.abs(C0[rows]) if C0 is not None else 0)
    return float((np.abs(C[rows].astype(np.float64) - ref) / sc).max())
# FP16, host operands, n = 8192 (two 4096-column blocks)
n = 8192
A = (rng.standard_normal((n, n)) / np.sqrt(n)).astype(np.float16)
B = (rng.standard_normal((n, n)) / np.sqrt(n)).astype(np.float16)
C = np.zeros((n, n), np.float16)
assert L.gemm(0, 0, 0, n, n, n, 1.0, A.ctypes.data, n, B.ctypes.data, n, 0.0, C.ctypes.data, n) == 0, L.error()
rows = np.concatenate([rng.choice(n, 48, replace=False), [0, n - 1]])
out["h_host"] = err(C, A.astype(np.float64), B.astype(np.float64), rows)
out["dev1_used_mb"] = (free1 - torch.cuda.mem_get_info(1)[0]) / 2**20
# FP32, ragged N (blocks of 4096 and 3904), transposed A, beta != 0 on a padded C, operands on device 0 (torch)
M, N, K = 4100, 8000, 3000
At = torch.rand(K, M, device="cuda:0", dtype=torch.float32) * 2 - 1      # stored K x M: op(A) = At^T
Bd = torch.rand(K, N, device="cuda:0", dtype=torch.float32) * 2 - 1
C0 = torch.rand(M, N + 5, device="cuda:0", dtype=torch.float32) * 2 - 1
Cd = C0.clone()
torch.cuda.synchronize()
assert L.gemm(1, 1, 0, M, N, K, 1.5, At.data_ptr(), M, Bd.data_ptr(), N, 0.5, Cd.data_ptr(), N + 5) == 0, L.error()
r2 = np.concatenate([rng.choice(M, 40, replace=False), [M - 1]])
out["s_dev_ragged"] = err(Cd[:, :N].cpu().numpy(), At.t().double().cpu().numpy(), Bd.double().cpu().numpy(), r2,
                          1.5, 0.5, C0[:, :N].double().cpu().numpy())
out["s_padding_kept"] = bool((Cd[:, N:] == C0[:, N:]).all())
# FP64 with B on device 1 (read there in place, copied to device 0 for the other block), transposed B
Kd, Nd, Md = 2048, 4608, 4096
Bt1 = torch.rand(Nd, Kd, device="cuda:1", dtype=torch.float64) * 2 - 1   # stored N x K: op(B) = Bt1^T
A0 = torch.rand(Md, Kd, device="cuda:0", dtype=torch.float64) * 2 - 1
C1 = torch.zeros(Md, Nd, device="cuda:0", dtype=torch.float64)
torch.cuda.synchronize(0); torch.cuda.synchronize(1)
assert L.gemm(3, 0, 1, Md, Nd, Kd, 1.0, A0.data_ptr(), Kd, Bt1.data_ptr(), Kd, 0.0, C1.data_ptr(), Nd) == 0, L.error()
r3 = np.concatenate([rng.choice(Md, 32, replace=False), [Md - 1]])
out["d_b_on_dev1"] = err(C1.cpu().numpy(), A0.cpu().numpy(), Bt1.t().cpu().numpy(), r3)
# the NumPy module: hgemm on managed arrays (gen9blas.empty) at n = 8192
import gen9blas
Am = gen9blas.empty((n, n), np.float16); Am[...] = A
Bm = gen9blas.empty((n, n), np.float16); Bm[...] = B
Cm = gen9blas.hgemm(Am, Bm)
out["h_module_managed"] = err(Cm, A.astype(np.float64), B.astype(np.float64), rows)
# turning sharding off through the API
assert L.set_devices(1, None) == 0 and L.get_devices(ids, 8) == 0
bad = (ctypes.c_int * 2)(0, 0)
assert L.set_devices(2, bad) == -3 and b"twice" in L.error()
print("OUT", repr(out))
'''


def test_sharded_gemm_two_devices_one_process():
    """GEN9BLAS_DEVICES=0,1 in one process: gen9blas_gemm splits large GEMMs by column blocks over both GPUs --
    FP16 n = 8192 from host memory, FP32 with a ragged last block, transposed A, beta on a padded C, FP64 with B owned
    by the second GPU, and the NumPy module on managed arrays -- each against FP64 with the north-star limits."""
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, GEN9BLAS_DEVICES="0,1", GEN9BLAS_SHARD_MIN_FLOP="1e10")
    r = subprocess.run([sys.executable, "-c", SHARD_CHILD, ROOT], capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stderr[-3000:]
    import ast
    out = ast.literal_eval([ln for ln in r.stdout.splitlines() if ln.startswith("OUT")][0][4:])
    assert out["h_host"] <= 1e-3 and out["h_module_managed"] <= 1e-3, out
    assert out["s_dev_ragged"] <= 1e-6 and out["s_padding_kept"], out
    assert out["d_b_on_dev1"] <= 1e-13, out
    assert out["dev1_used_mb"] > 100, out      # the second GPU held its operand copies


def test_sharded_gemm_through_cblas_two_devices():
    """The LD_PRELOAD library with GEN9BLAS_DEVICES=0,1: cblas_sgemm n = 8192 (row-major) and cblas_dgemm n = 4096
    (column-major, alpha 1.5, beta 0.5) split over two GPUs, against FP64."""
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, GEN9BLAS_DEVICES="0,1", GEN9BLAS_BLAS="gpu")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "tests", "shim_child.py"), "sharded"], capture_output=True,
                       text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stderr[-3000:]
    import json
    res = json.loads(r.stdout.strip().splitlines()[-1])
    assert res["sgemm_8192"] <= 1e-6 and res["dgemm_4096_col"] <= 1e-13, res
