"""ctypes signatures of the gen9blas.h entry points, shared by the library and the oracle (same signatures)."""
import ctypes

_i, _p, _d, _l, _f = ctypes.c_int, ctypes.c_void_p, ctypes.c_double, ctypes.c_int64, ctypes.c_float

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
    # gen9blas_ml.h
    "gemm_pb_f16w": ([_i, _p, _i, _p, _p, _i, _p], _i),
    "gemm_pb_f16w_h": ([_i, _p, _i, _p, _p, _i, _p], _i),
    "gemm_pb_f16w_ex": ([_i, _p, _i, _p, _p, _i, _p, _i, _p, _i, _p], _i),
    "gemm_multi_f16w": ([_i, _p, _i, _i, _p, _p, _p, _p], _i),
    "ffn_f16w": ([_i, _p, _i, _p, _p, _p, _p, _i, _p], _i),
    "pack_b_q": ([_i, _i, _i, _p, ctypes.c_size_t, _p], _p),
    "packed_a_create": ([], _p), "packed_a_free": ([_p], None),
    "layer_norm_pack": ([_i, _i, _p, _i, _p, _p, _f, _p, _i, _p, _i], _i),
    "gemm_pa_f16w_ex": ([_p, _p, _p, _i, _p, _i, _p, _i, _p], _i),
    "nowait_pending": ([], _i),
    "span": ([_p, ctypes.c_size_t, _i], _i), "span_clear": ([], None),
    "rms_norm": ([_i, _i, _p, _i, _p, _f, _p, _i, _i], _i),
    "layer_norm": ([_i, _i, _p, _i, _p, _p, _f, _p, _i, _i], _i),
    "binop_rows": ([_i, _i, _i, _p, _i, _p, _i, _i, _p, _i, _i], _i),
    "gelu": ([ctypes.c_size_t, _p, _p, _i], _i), "gelu_erf": ([ctypes.c_size_t, _p, _p, _i], _i),
    "relu": ([ctypes.c_size_t, _p, _p, _i], _i),
    "im2col": ([_i, _i, _i, _i, _p, _l, _l] + [_i] * 10 + [_p, _i, _i], _i),
    "cvt_f16_heads": ([_i, _i, _i, _p, _l, _l, _p, _i], _i),
    "rope": ([_i, _i, _i, _p, _l, _l, _p, _l, _l, _p, _p, _i, _f, _f, _f, _f, _p, _i], _i),
    "rope_multi": ([_i, _i, _i, _p, _l, _l, _p, _l, _l, _p, _p, _p, _f, _f, _f, _f, _p, _i, _i], _i),
    "cpy_any": ([_p, _i, _p, _p, _p, _i, _p, _p, _i], _i),
    "upscale_f32": ([_p, _p, _p, _p, _p, _p, _i, _i], _i),
    "set_rows_f16": ([_i, _i, _i, _i, _p, _l, _l, _l, _p, ctypes.c_size_t, _l, _l, _l, _i, _i, _i, _p,
                      ctypes.c_size_t, _l, _l, _l, _l, _i, _p], _i),
    "attn_dec_supported": ([_i, _i, _i], _i), "attn_supported": ([_i, _i, _i], _i),
    "attn_streams_supported": ([_i, _i, _i], _i),
    "attn_dec": ([_i, _i, _i, _i, _i, _i, _p, _l, _l, _l, _p, _l, _l, _l, ctypes.c_size_t, _p, _l, _l, _l,
                  ctypes.c_size_t, _p, _f, _p, _i, _i, _i], _i),
    "attn_f16kv": ([_i, _i, _i, _i, _i, _p, _p, ctypes.c_size_t, _p, ctypes.c_size_t, _p, _f, _i, _i, _p], _i),
    "attn_f16kv_streams": ([_i, _i, _i, _i, _i, _i, _p, _l, _p, _l, ctypes.c_size_t, _p, _l, ctypes.c_size_t, _p,
                            _f, _p, _i, _p], _i),
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
