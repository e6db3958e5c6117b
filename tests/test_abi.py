"""CPU checks of the drop-in boundary: libgen9blas.so loads without a GPU, exports every function that
include/gen9blas.h declares (the reference's lib/gen9blas.h set plus the B200 additions), keeps the 0.2.x version
gate of the NumPy module, and fails initialisation cleanly (GEN9BLAS_ERR_NO_DEVICE) where there is no GPU."""
import ctypes
import os
import re
import subprocess

import pytest

from conftest import PKG, ROOT

HEADERS = [os.path.join(ROOT, "include", h) for h in ("gen9blas.h", "gen9blas_ml.h")]
LIB = os.path.join(PKG, "libgen9blas.so")


def declared_functions():
    text = "".join(open(h).read() for h in HEADERS)
    return sorted(set(re.findall(r"GEN9BLAS_API\s+[^;(]*?\b(gen9blas_\w+)\s*\(", text)))


def exported(path):
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


def test_header_declares_reference_surface():
    names = declared_functions()
    # the 51 entry points of the reference's lib/gen9blas.h plus the additions of this build
    for must in ("gen9blas_gemm", "gen9blas_gemm_batched", "gen9blas_hgemm", "gen9blas_sgemm", "gen9blas_axpy",
                 "gen9blas_dot", "gen9blas_nrm2", "gen9blas_asum", "gen9blas_iamax", "gen9blas_gemv", "gen9blas_ger",
                 "gen9blas_init", "gen9blas_error", "gen9blas_alloc", "gen9blas_spr2", "gen9blas_set_device",
                 "gen9blas_pack_b", "gen9blas_gemm_pb", "gen9blas_packed_b_free", "gen9blas_gemm_pb_skinny"):
        assert must in names
    assert len(names) == 101   # 67 + set_devices / get_devices + the 32 other entry points of lib/gen9blas_ml.h


def test_ml_header_matches_the_reference_list():
    """Every function of the reference's lib/gen9blas_ml.h (its 33 declarations; set_nowait and flush are declared in
    gen9blas.h) is declared here, with the same parameter count."""
    ml = open(HEADERS[1]).read()
    expected = {   # name: parameters, from lib/gen9blas_ml.h:14-149
        "gemm_pb_f16w": 7, "gemm_pb_f16w_h": 7, "gemm_pb_f16w_ex": 11, "gemm_pb_skinny": 7, "gemm_multi_f16w": 8,
        "ffn_f16w": 9, "pack_b_q": 6, "packed_a_create": 0, "packed_a_free": 1, "layer_norm_pack": 11,
        "gemm_pa_f16w_ex": 9, "nowait_pending": 0, "span": 3, "span_clear": 0, "rms_norm": 9, "layer_norm": 10,
        "binop_rows": 11, "gelu": 4, "gelu_erf": 4, "relu": 4, "im2col": 20, "cvt_f16_heads": 8, "rope": 18,
        "rope_multi": 19, "cpy_any": 9, "upscale_f32": 8, "set_rows_f16": 24, "attn_dec_supported": 3,
        "attn_dec": 26, "attn_supported": 3, "attn_f16kv": 15, "attn_streams_supported": 3, "attn_f16kv_streams": 19,
    }
    for name, nparams in expected.items():
        m = re.search(r"GEN9BLAS_API[^;(]*\bgen9blas_" + name + r"\s*\(([^)]*)\)", ml)
        assert m, name
        params = m.group(1).strip()
        count = 0 if params in ("", "void") else params.count(",") + 1
        assert count == nparams, (name, count)


def test_library_exports_every_declared_function():
    syms = exported(LIB)
    missing = [n for n in declared_functions() if n not in syms]
    assert not missing, missing
    # nothing else leaks: hidden visibility for the internals
    extra = sorted(s for s in syms if not s.startswith("gen9blas_"))
    assert not extra, extra[:10]


def test_version_gate(lib):
    assert lib.version() // 100 == 2   # lib/gen9blas.py:48-49 accepts 0.2.x


def test_build_recipe_targets_only_sm100a():
    """The recipe compiles every kernel for sm_100a alone (no PTX for other targets, no older architectures)."""
    import build
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]
    assert all("sm_" not in f and "compute_" not in f for f in build.NVFLAGS if f not in build.ARCH)


def test_init_without_gpu_is_clean(lib):
    if lib.init() == 0:
        pytest.skip("a GPU is present")
    assert lib.init() == -5                       # GEN9BLAS_ERR_NO_DEVICE, final for the process
    assert lib.last_status() == -5
    assert lib.error()                            # an explanation is set
    assert lib.has(0) == 0 and lib.device_gen() == 0
    x = (ctypes.c_float * 4)()
    assert lib.axpy(1, 4, 1.0, ctypes.addressof(x), 1, ctypes.addressof(x), 1) == -5
