"""The config-size fixtures (tests/golden/ref_config_rows.npz: rows of the reference CBLAS layer's own output at
BASELINE configs[0] SGEMM n = 1024 and configs[3] DGEMM n = 3000 column-major) against FP64 NumPy on the CPU, with
the north-star limits and the elementwise metric of lib/test_basic.py:4-8. This pins what the fixtures hold before
the GPU tests compare the library with them."""
import os

import numpy as np
import pytest

from conftest import ROOT, gemm_error
import make_golden as mg

FIX = os.path.join(ROOT, "tests", "golden", "ref_config_rows.npz")


@pytest.fixture(scope="module")
def fix():
    return np.load(FIX)


def test_c0_sgemm_rows_of_the_reference(fix):
    A, B = mg.c0_inputs()
    rows = mg.c0_rows()
    a64, b64 = A[rows].astype(np.float64), B.astype(np.float64)
    avg, mx = gemm_error(fix["sgemm_c0_rows"], a64 @ b64, np.abs(a64) @ np.abs(b64))
    assert mx <= 1e-6 and avg <= 1e-7, (avg, mx)


@pytest.mark.parametrize("ta", [mg.NoTrans, mg.Trans])
@pytest.mark.parametrize("tb", [mg.NoTrans, mg.Trans])
def test_c3_dgemm_rows_of_the_reference(fix, ta, tb):
    A, B, C0 = mg.c3_inputs(ta, tb)
    rows = mg.c3_rows()
    opA = A if ta == mg.NoTrans else A.T
    opB = B if tb == mg.NoTrans else B.T
    ref = mg.C3_ALPHA * opA[rows] @ opB + mg.C3_BETA * C0[rows]
    scale = mg.C3_ALPHA * np.abs(opA[rows]) @ np.abs(opB) + mg.C3_BETA * np.abs(C0[rows])
    avg, mx = gemm_error(fix[f"dgemm_c3_t{ta}{tb}_rows"], ref, scale)
    assert mx <= 1e-13, (ta, tb, mx)
