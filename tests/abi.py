"""ctypes signatures of the gen9blas.h entry points, shared by the library and the oracle (same signatures)."""
import ctypes

_i, _p, _d, _l = ctypes.c_int, ctypes.c_void_p, ctypes.c_double, ctypes.c_int64

SIGNATURES = {
    "version": ([], _i), "init": ([], _i), "device_gen": ([], _i), "has": ([_i], _i),
    "error": ([], ctypes.c_char_p), "last_status": ([], _i), "last_time_ms": ([], _d), "last_zero_copy": ([], _i),
    "alloc": ([ctypes.c_size_t], _p), "free": ([_p], None), "is_usm": ([_p, ctypes.c_size_t], _i),
    "gemm": ([_i, _i, _i, _i, _i, _i, _d, _p, _i, _p, _i, _d, _p, _i], _i),
    "gemm_batched": ([_i, _i, _i, _i, _i, _i, _d, _p, _i, _l, _p, _i, _l, _d, _p, _i, _l, _i], _i),
    "hgemm": ([_i, _i, _i, _d, _p, _i, _p, _i, _d, _p, _i], _i),
    "sgemm": ([_i, _i, _i, _d, _p, _i, _p, _i, _d, _p, _i], _i),
    "axpy": ([_i, _i, _d, _p, _i, _p, _i], _i),
    "dot": ([_i, _i, _p, _i, _p, _i, ctypes.POINTER(_d)], _i),
    "asum": ([_i, _i, _p, _i, ctypes.POINTER(_d)], _i),
    "nrm2": ([_i, _i, _p, _i, ctypes.POINTER(_d)], _i),
    "iamax": ([_i, _i, _p, _i, ctypes.POINTER(_l)], _i),
    "gemv": ([_i, _i, _i, _i, _d, _p, _i, _p, _i, _d, _p, _i], _i),
    "ger": ([_i, _i, _i, _d, _p, _i, _p, _i, _p, _i], _i),
    "set_device": ([_i], _i), "get_device": ([], _i), "set_stream": ([_p], _i), "set_nowait": ([_i], None),
    "flush": ([], _i), "kernel_launches": ([], ctypes.c_longlong),
    "set_devices": ([_i, ctypes.POINTER(_i)], _i), "get_devices": ([ctypes.POINTER(_i), _i], _i),
    "selftest_wait": ([_d], _i),
    "gemv_noalloc": ([_i, _i, _i, _i, _d, _p, _i, _p, _i, _d, _p, _i], _i),
    "peer_barrier": ([_p, _i, _i, _d], _i),
    "pack_b": ([_i, _i, _i, _i, _p, _i], _p),
    "gemm_pb": ([_i, _i, _d, _p, _i, _p, _d, _p, _i], _i),
    "packed_b_free": ([_p], None),
    "gemm_pb_skinny": ([_i, _p, _i, _p, _p, _i, ctypes.POINTER(_i)], _i),
}


class Bound:
    """Attribute access by short name: lib.gemm(...) calls <prefix>gemm with the signature above."""

    def __init__(self, dll, prefix):
        self.dll, self.prefix = dll, prefix
        for name, (args, res) in SIGNATURES.items():
            f = getattr(dll, prefix + name, None)
            if f is None:
                continue
            f.argtypes, f.restype = args, res
            setattr(self, name, f)


def bind(dll, prefix):
    return Bound(dll, prefix)


H, S, HS, D = 0, 1, 2, 3
