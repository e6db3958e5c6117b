"""The LD_PRELOAD CBLAS/BLAS library libgen9blas_blas.so (drop-in for the reference's libgen9blas_blas.so,
lib/src/cblas.c): symbol surface and forwarding on CPU; GPU routing and parity against the reference's own CBLAS
outputs (GEN9BLAS_BLAS_INFO log, tolerances of lib/test_blas.py / test_blas_d.py) on a GPU."""
import json
import os
import subprocess
import sys

import pytest

from conftest import PKG, ROOT

SHIM = os.path.join(PKG, "libgen9blas_blas.so")
CHILD = os.path.join(ROOT, "tests", "shim_child.py")


def child(group, **env):
    e = dict(os.environ)
    e.update(env)
    r = subprocess.run([sys.executable, CHILD, group], capture_output=True, text=True, env=e, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return json.loads(r.stdout.strip().splitlines()[-1]), r.stderr


def test_exports_exactly_the_blas_surface():
    syms = [s.strip() for s in open(os.path.join(PKG, "shim", "blas_symbols.txt")) if s.strip()]
    assert len(syms) == 393
    out = subprocess.run(["nm", "-D", "--defined-only", SHIM], capture_output=True, text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert exported == set(syms)


def test_cpu_mode_routes_everything_to_the_cpu_blas():
    res, err = child("forwarded", GEN9BLAS_BLAS="cpu", GEN9BLAS_BLAS_INFO="1")
    assert res["zgemm_forwarded"] < 1e-12
    res, err = child("cblas_gemm", GEN9BLAS_BLAS="cpu", GEN9BLAS_BLAS_INFO="1")
    assert res["sgemm_vs_ref_cblas"] <= 1e-6 and res["dgemm_vs_ref_cblas"] <= 1e-13
    assert "-> GPU" not in err and "sgemm -> CPU" in err


def test_cpu_mode_level3_is_the_reference_cblas():
    """GEN9BLAS_BLAS=cpu: the level-3 symbols go to the CPU BLAS and reproduce the reference layer's outputs."""
    res, err = child("level3", GEN9BLAS_BLAS="cpu", GEN9BLAS_BLAS_INFO="1")
    for tag in ("s", "d"):
        for op in ("symm", "syrk", "syr2k", "trmm", "trsm"):
            assert res[tag + op] <= (1e-6 if tag == "s" else 1e-13), (tag + op, res[tag + op])
        assert res[tag + "_other_triangle_exact"]
    assert "-> GPU" not in err and "strsm -> CPU" in err


@pytest.mark.gpu
def test_gpu_level3_matches_reference_cblas():
    """SYMM, SYRK, SYR2K, TRMM, TRSM (S and D, row- and column-major, every side / triangle / transpose / diagonal)
    on the GPU against the reference CBLAS layer's outputs, with lib/test_level3.py's limits."""
    res, err = child("level3", GEN9BLAS_BLAS="gpu", GEN9BLAS_BLAS_INFO="1")
    for op in ("symm", "syrk", "syr2k", "trmm"):
        assert res["s" + op] <= 1e-5 and res["d" + op] <= 1e-13, (op, res)
    assert res["strsm"] <= 1e-4 and res["dtrsm"] <= 1e-12, res
    assert res["s_other_triangle_exact"] and res["d_other_triangle_exact"]
    for f in ("ssymm", "dsyrk", "ssyr2k", "dtrmm", "strsm", "dtrsm"):
        assert f"{f} -> GPU" in err, f
    assert "-> CPU" not in err


L2X = ("symv", "trmv", "trsv", "tbmv", "tbsv", "tpmv", "tpsv", "sbmv", "spmv", "syr", "syr2", "spr", "spr2", "gbmv",
       "scal", "copy", "swap", "rot", "rotm")


def test_cpu_mode_level12_extras_are_the_cpu_blas():
    res, err = child("l2x", GEN9BLAS_BLAS="cpu", GEN9BLAS_BLAS_INFO="1")
    for tag in ("s", "d"):
        for f in L2X:
            assert res[tag + f] <= 1e-12, (tag + f, res[tag + f])
    assert "-> GPU" not in err


@pytest.mark.gpu
def test_gpu_level12_extras_match_openblas():
    """lib/test_blas_banded.py's differential check (RowMajor and ColMajor, every triangle / transpose / diagonal)
    for the rest of levels 1-2 on the GPU: max |diff| / scale <= 1e-5 (FP32; solves 1e-4), 1e-12 (FP64)."""
    res, err = child("l2x", GEN9BLAS_BLAS="gpu", GEN9BLAS_BLAS_INFO="1")
    for f in L2X:
        tol = 1e-4 if f in ("trsv", "tbsv", "tpsv") else 1e-5
        assert res["s" + f] <= tol and res["d" + f] <= 1e-12, (f, res["s" + f], res["d" + f])
    for f in ("ssymv", "dtrsv", "stbsv", "dtpsv", "sgbmv", "dspr2", "sscal", "drotm"):
        assert f"{f} -> GPU" in err, f
    assert "-> CPU" not in err


@pytest.mark.gpu
def test_gpu_gemm_matches_reference_cblas():
    res, err = child("cblas_gemm", GEN9BLAS_BLAS="gpu", GEN9BLAS_BLAS_INFO="1")
    assert res["sgemm_vs_ref_cblas"] <= 2e-6, res
    assert res["dgemm_vs_ref_cblas"] <= 1e-13, res
    assert "sgemm -> GPU" in err and "dgemm -> GPU" in err and "-> CPU" not in err


def test_cpu_mode_config_sizes_are_the_reference_cblas():
    """GEN9BLAS_BLAS=cpu: configs[0] / configs[3] through cblas_sgemm / cblas_dgemm reproduce the fixture rows."""
    res, err = child("config", GEN9BLAS_BLAS="cpu", GEN9BLAS_BLAS_INFO="1")
    assert res["sgemm_c0_vs_ref_cblas"] <= 1e-6 and res["dgemm_c3_vs_ref_cblas"] <= 1e-13, res
    assert "-> GPU" not in err


@pytest.mark.gpu
def test_gpu_config_sizes_through_cblas():
    """BASELINE configs[0] (cblas_sgemm n = 1024 row-major) and configs[3] (cblas_dgemm n = 3000 column-major, all
    four transposes, alpha 1.5, beta 0.5, C prefilled) through the LD_PRELOAD library on the GPU: north-star limits
    (SGEMM max 1e-6, DGEMM 1e-13) against FP64 and against the reference CBLAS layer's own output rows."""
    res, err = child("config", GEN9BLAS_BLAS="gpu", GEN9BLAS_BLAS_INFO="1")
    assert res["sgemm_c0_vs_fp64"] <= 1e-6 and res["sgemm_c0_vs_ref_cblas"] <= 1e-6, res
    assert res["dgemm_c3_vs_fp64"] <= 1e-13 and res["dgemm_c3_vs_ref_cblas"] <= 1e-13, res
    assert "sgemm -> GPU" in err and "dgemm -> GPU" in err and "-> CPU" not in err


@pytest.mark.gpu
def test_gpu_fortran_and_level12():
    res, err = child("fortran_l12", GEN9BLAS_BLAS_INFO="1")
    for tag, tol in (("s", 1e-5), ("d", 1e-12)):   # lib/test_blas.py:55-60, lib/test_blas_d.py:1-7
        for k in ("gemm_fortran", "gemv", "ger", "axpy", "dot", "nrm2", "asum"):
            assert res[tag + k] <= tol, (tag + k, res[tag + k])
        assert res[f"i{tag}amax_exact"]
    for f in ("sgemm_", "dgemm_", "sgemv", "dger", "saxpy", "ddot", "snrm2", "dasum", "isamax"):
        assert f"{f} -> GPU" in err, f
    assert "-> CPU" not in err
    res, err = child("forwarded")
    assert res["zgemm_forwarded"] < 1e-12
