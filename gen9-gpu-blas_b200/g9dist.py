"""Multi-GPU partitioning of the gen9blas hot path: one process per GPU, torch.distributed for the plumbing.

The reference is single-device (README.md:176-178); this module adds the scale-out of BASELINE configs[4]:
- column_sharded_gemm: C = alpha·A·B with A replicated and B / C split into column blocks; rank g computes
  C[:, cols_g] = A·B[:, cols_g] with the rank's own GPU kernels (libgen9blas.so), then the column blocks are
  all-gathered (NCCL over NVLink) in `chunks` pieces, each gather overlapping the GEMM of the next piece, and laid out
  into the row-major C;
- row_sharded_skinny: C = A·Wᵀ with the weight rows split over the ranks (tensor parallel decode): rank g computes
  C[:, rows_g] with the skinny kernel, then one all-gather of the small M × N/g outputs.
The partition arithmetic (shard bounds, gather layout, re-layout) is plain Python/torch so that it can be tested with
gloo ranks on the CPU (tests/test_dist_cpu.py) with a CPU stand-in for the local product.

Failure detection (the analogue of the reference's bounded GPU wait, lib/kcl.c:361-372): init_comm starts the process
group with a finite timeout, and every collective of these paths is waited for on the host with a deadline, polling the
backend's completion (an error the backend records -- NCCL's asynchronous error, a failed peer -- surfaces there). A
failure or a missed deadline raises CommError, whose `status` is the library's GEN9BLAS_ERR and `stage` says where
("init", "collective" or "timeout"). GEN9BLAS_FAULT=nccl_init or nccl_op makes this rank fail there on purpose (host
side only; the other ranks then see their deadline pass).
"""
import ctypes
import datetime
import os
import time

import torch

GEN9BLAS_H, GEN9BLAS_S, GEN9BLAS_HS, GEN9BLAS_D = 0, 1, 2, 3
GEN9BLAS_ERR = -1   # status of a failed or timed-out collective (the 0.2 API's execution-error code)
_KIND = {torch.float16: GEN9BLAS_H, torch.float32: GEN9BLAS_S, torch.float64: GEN9BLAS_D}
DEFAULT_TIMEOUT_S = 60.0


class CommError(RuntimeError):
    """A collective of the multi-GPU path failed or missed its deadline. status: the gen9blas status code;
    stage: "init", "collective" or "timeout"."""

    def __init__(self, stage, message, status=GEN9BLAS_ERR):
        super().__init__(f"{stage}: {message}")
        self.stage, self.status = stage, status


def _fault():
    v = os.environ.get("GEN9BLAS_FAULT", "")
    return v if v in ("nccl_init", "nccl_op") else ""


def init_comm(backend="nccl", timeout_s=DEFAULT_TIMEOUT_S, **kwargs):
    """torch.distributed.init_process_group(backend) with a finite timeout (rendezvous and collectives); a failure,
    or GEN9BLAS_FAULT=nccl_init, raises CommError(stage "init")."""
    if _fault() == "nccl_init":
        raise CommError("init", "communicator initialisation failed (injected: GEN9BLAS_FAULT=nccl_init)")
    try:
        torch.distributed.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kwargs)
    except Exception as e:   # rendezvous timeout, backend error
        raise CommError("init", f"init_process_group({backend}) failed: {e}") from e


def _issue(fn, what):
    """Starts one asynchronous collective; GEN9BLAS_FAULT=nccl_op makes this rank fail instead of taking part."""
    if _fault() == "nccl_op":
        raise CommError("collective", f"{what} failed (injected: GEN9BLAS_FAULT=nccl_op)")
    try:
        return fn()
    except Exception as e:
        raise CommError("collective", f"{what}: {e}") from e


def _finish(works, timeout_s, what):
    """Waits on the host for the given collectives until timeout_s (None: no deadline, stream-ordered wait only);
    backend errors and a missed deadline raise CommError."""
    if timeout_s is None:
        for w in works:
            w.wait()
        return
    deadline = time.monotonic() + timeout_s
    for w in works:
        while True:
            try:
                done = w.is_completed()
            except Exception as e:
                raise CommError("collective", f"{what}: {e}") from e
            if done:
                break
            if time.monotonic() > deadline:
                raise CommError("timeout", f"{what} did not complete within {timeout_s:g} s (a rank failed, left or "
                                           "never joined)")
            time.sleep(0.0002)
        try:
            w.wait()   # raises what the backend recorded for a failed collective
        except Exception as e:
            raise CommError("collective", f"{what}: {e}") from e


def shard_bounds(n, world, align=1):
    """[start, stop) of each rank's block of n items, blocks as equal as possible and multiples of `align` except the
    last. Every item belongs to exactly one rank."""
    per = -(-n // world)
    per = -(-per // align) * align
    out = []
    for g in range(world):
        a = min(n, g * per)
        out.append((a, min(n, a + per)))
    return out


def chunk_bounds(width, chunks):
    """Sub-blocks of a column block used to overlap the gather of one piece with the GEMM of the next."""
    return shard_bounds(width, chunks)


def gemm_local(lib, A, B, C, alpha=1.0, beta=0.0, accurate=False):
    """C = alpha·A·B + beta·C on this rank's GPU through the C ABI (row-major views with unit column stride)."""
    kind = GEN9BLAS_HS if (accurate and A.dtype == torch.float16) else _KIND[A.dtype]
    M, K = A.shape
    N = B.shape[1]
    r = lib.gen9blas_gemm(kind, 0, 0, M, N, K, ctypes.c_double(alpha), ctypes.c_void_p(A.data_ptr()), A.stride(0),
                          ctypes.c_void_p(B.data_ptr()), B.stride(0), ctypes.c_double(beta),
                          ctypes.c_void_p(C.data_ptr()), C.stride(0))
    if r != 0:
        raise RuntimeError(lib.gen9blas_error().decode())


def column_sharded_gemm(A, B_shard, C, rank, world, local_gemm, group=None, chunks=4, comm_stream=None,
                        timeout_s=DEFAULT_TIMEOUT_S):
    """C (M × N, row-major, every rank) = A (M × K) · B, where this rank holds B_shard = B[:, cols_rank].

    All ranks hold equal-width shards (N divisible by world). The shard is computed in `chunks` column pieces into a
    chunk-major buffer; after each piece its all-gather starts on `comm_stream` while the next piece computes. The
    gathered pieces are then copied into C's row-major layout. local_gemm(A, B_piece, C_piece) computes one piece.
    The gathers are waited for on the host (deadline timeout_s; None: stream-ordered only); a failure raises
    CommError. Returns C."""
    M = A.shape[0]
    nb = B_shard.shape[1]
    N = nb * world
    assert C.shape == (M, N)
    bounds = chunk_bounds(nb, chunks)
    widths = {b - a for a, b in bounds if b > a}
    assert len(widths) == 1, "column pieces must have equal widths"
    cw = widths.pop()
    nchunks = len([1 for a, b in bounds if b > a])
    if world == 1:
        for a, b in bounds:
            if b > a:
                local_gemm(A, B_shard[:, a:b], C[:, a:b])
        return C
    Cs = torch.empty((nchunks, M, cw), dtype=C.dtype, device=C.device)
    Cg = torch.empty((nchunks, world, M, cw), dtype=C.dtype, device=C.device)
    use_streams = C.is_cuda and comm_stream is not None
    main = torch.cuda.current_stream() if use_streams else None
    works = []
    for c, (a, b) in enumerate([ab for ab in bounds if ab[1] > ab[0]]):
        local_gemm(A, B_shard[:, a:b], Cs[c])
        gather = (lambda c=c: torch.distributed.all_gather_into_tensor(Cg[c].view(world * M, cw), Cs[c], group=group,
                                                                       async_op=True))
        if use_streams:
            ev = torch.cuda.Event()
            ev.record(main)
            comm_stream.wait_event(ev)
            with torch.cuda.stream(comm_stream):
                works.append(_issue(gather, f"all-gather of column piece {c}"))
        else:
            works.append(_issue(gather, f"all-gather of column piece {c}"))
    _finish(works, timeout_s, "column all-gather")
    if use_streams:
        main.wait_stream(comm_stream)
    # gathered piece (chunk c, rank q) holds C[:, q*nb + c*cw : + cw]
    C.view(M, world, nchunks, cw).copy_(Cg.permute(2, 1, 0, 3))
    return C


def row_sharded_skinny(A, W_shard, C, rank, world, local_skinny, group=None, timeout_s=DEFAULT_TIMEOUT_S):
    """C (M × N) = A (M × K) · Wᵀ with W (N × K) split into row blocks: this rank holds W_shard = W[rows_rank] and
    computes C[:, rows_rank]; one all-gather of the M × N/world outputs (host deadline timeout_s, CommError on
    failure), then a re-layout. Returns C."""
    M = A.shape[0]
    nr = W_shard.shape[0]
    N = nr * world
    assert C.shape == (M, N)
    if world == 1:
        local_skinny(A, W_shard, C)
        return C
    Cs = torch.empty((M, nr), dtype=C.dtype, device=C.device)
    local_skinny(A, W_shard, Cs)
    Cg = torch.empty((world, M, nr), dtype=C.dtype, device=C.device)
    w = _issue(lambda: torch.distributed.all_gather_into_tensor(Cg.view(world * M, nr), Cs, group=group,
                                                                async_op=True), "all-gather of the output rows")
    _finish([w], timeout_s, "output all-gather")
    C.view(M, world, nr).copy_(Cg.permute(1, 0, 2))
    return C


class PeerView:
    """Device pointers of one tensor's counterpart on every rank (CUDA IPC over NVLink), for kernels that write into
    the other ranks' memory. Collective: every rank constructs it with its own tensor of the same shape."""

    def __init__(self, lib, tensor, rank, world, group=None):
        self.lib = lib
        self.opened = []
        h = (ctypes.c_char * 64)()
        off = ctypes.c_int64()
        lib.gen9blas_ipc_handle.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64)]
        lib.gen9blas_ipc_open.argtypes = [ctypes.c_void_p]
        lib.gen9blas_ipc_open.restype = ctypes.c_void_p
        lib.gen9blas_ipc_close.argtypes = [ctypes.c_void_p]
        if lib.gen9blas_ipc_handle(ctypes.c_void_p(tensor.data_ptr()), h, ctypes.byref(off)) != 0:
            raise RuntimeError(lib.gen9blas_error().decode())
        mine = (bytes(h), off.value)
        allh = [None] * world
        torch.distributed.all_gather_object(allh, mine, group=group)
        self.ptrs = []
        for q in range(world):
            if q == rank:
                self.ptrs.append(tensor.data_ptr())
                continue
            hb = (ctypes.c_char * 64).from_buffer_copy(allh[q][0])
            base = lib.gen9blas_ipc_open(hb)
            if not base:
                raise RuntimeError(lib.gen9blas_error().decode())
            self.opened.append(base)
            self.ptrs.append(base + allh[q][1])

    def close(self):
        for b in self.opened:
            self.lib.gen9blas_ipc_close(ctypes.c_void_p(b))
        self.opened = []


class PeerBarrier:
    """Rank barrier over NVLink peer memory (gen9blas_peer_barrier): every rank owns a zeroed array of world + 1
    32-bit words (one flag per rank and the device-side epoch counter) mapped into the other ranks. wait() is enqueued
    on the library's stream and can be captured in a CUDA graph; all ranks must call it the same number of times.
    Collective construction."""

    def __init__(self, lib, rank, world, device=None, timeout_ms=5000.0, group=None):
        import torch
        self.lib, self.rank, self.world, self.timeout_ms = lib, rank, world, timeout_ms
        self.flags = torch.zeros(world + 1, dtype=torch.int32, device=device or torch.cuda.current_device())
        torch.cuda.synchronize()
        self.view = PeerView(lib, self.flags, rank, world, group=group)
        self.arr = (ctypes.c_void_p * world)(*self.view.ptrs)
        lib.gen9blas_peer_barrier.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_double]

    def wait(self):
        r = self.lib.gen9blas_peer_barrier(self.arr, self.world, self.rank, self.timeout_ms)
        if r != 0:   # e.g. the device-side wait gave up: a rank never arrived
            raise CommError("collective", "peer barrier: " + self.lib.gen9blas_error().decode(), status=r)

    def close(self):
        self.view.close()


def fused_column_sharded_gemm(lib, A, B_shard, C, peers, rank, world, accurate=False, group=None, barrier=None):
    """C (M × N on every rank) = A · B with B column-sharded, in one kernel per rank: the HGEMM epilogue writes each
    finished tile of this rank's block into every rank's C (peers: PeerView of C) over NVLink; then the ranks meet in
    a barrier (barrier: PeerBarrier, else a stream-ordered NCCL all-reduce of one element) before C is used. FP16."""
    M, K = A.shape
    nb = B_shard.shape[1]
    _allgather(lib, A, B_shard, 0, C, peers, rank * nb, accurate)
    _meet(C, world, group, barrier)
    return C


def fused_row_sharded_skinny(lib, A, W_shard, C, peers, rank, world, accurate=False, group=None, barrier=None):
    """Tensor-parallel decode: C (M × N on every rank, M <= 16) = A · Wᵀ with the weight rows split over the ranks
    (W_shard = W[rows_rank], N/world × K). The skinny kernel stores this rank's M × N/world block into every rank's C
    over NVLink; then the ranks meet as in fused_column_sharded_gemm. FP16."""
    _allgather(lib, A, W_shard, 1, C, peers, rank * W_shard.shape[0], accurate)
    _meet(C, world, group, barrier)
    return C


def _allgather(lib, A, B, transB, C, peers, col_off, accurate):
    M, K = A.shape
    nb = B.shape[0] if transB else B.shape[1]
    world = len(peers.ptrs)
    arr = (ctypes.c_void_p * world)(*peers.ptrs)
    lib.gen9blas_gemm_allgather.argtypes = [ctypes.c_int] * 6 + [ctypes.c_double, ctypes.c_void_p, ctypes.c_int,
                                                                  ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                                                  ctypes.c_int, ctypes.c_int, ctypes.c_int64]
    r = lib.gen9blas_gemm_allgather(GEN9BLAS_HS if accurate else GEN9BLAS_H, 0, transB, M, nb, K, 1.0,
                                    A.data_ptr(), A.stride(0), B.data_ptr(), B.stride(0), arr, world,
                                    C.stride(0), col_off)
    if r != 0:
        raise CommError("collective", "gen9blas_gemm_allgather: " + lib.gen9blas_error().decode(), status=r)


def _meet(C, world, group, barrier):
    import torch
    if world == 1:
        return
    if barrier is not None:
        barrier.wait()   # bounded on the device: a rank that never arrives makes the call return GEN9BLAS_ERR
    else:
        flag = torch.ones(1, device=C.device)
        w = _issue(lambda: torch.distributed.all_reduce(flag, group=group, async_op=True), "rank meeting")
        _finish([w], DEFAULT_TIMEOUT_S, "rank meeting")
