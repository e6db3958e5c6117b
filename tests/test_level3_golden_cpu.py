"""Pins the level-3 oracle on the CPU: an FP64 NumPy restatement of SYMM, SYRK, SYR2K, TRMM and TRSM (the semantics of
the reference's lib/src/level3.c and CBLAS layer lib/src/cblas.c:194-228) reproduces the outputs of the reference's
own CBLAS layer, run here in CPU mode over OpenBLAS and committed as tests/golden/ref_cblas_outputs.npz, for every
order / side / triangle / transpose / diagonal combination; the triangle of C that SYRK / SYR2K must not touch is
compared bit for bit. The GPU level-3 tests (test_level3_gpu.py) compare against the same restatement."""
import os

import numpy as np
import pytest

from make_golden import L3_SYMM, L3_SYRK, L3_TRXM, Left, Trans, Unit, Upper, l3_cases, l3_inputs, l3_key

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
REF = np.load(os.path.join(GOLD, "ref_cblas_outputs.npz"))
TOL = {"s": 2e-6, "d": 1e-14}


def restated(tag, case):
    """(result, scale, untouched mask or None) of one level-3 case on the logical matrices, in FP64."""
    op = case[0]
    if op == "symm":
        side, uplo = case[2], case[3]
        M, N, al, be = L3_SYMM
        A, B, C0 = (x.astype(np.float64) for x in l3_inputs(tag, op, *case[1:]))
        T = np.triu(A) if uplo == Upper else np.tril(A)
        S = T + T.T - np.diag(np.diag(T))
        P, Pa = (S @ B, np.abs(S) @ np.abs(B)) if side == Left else (B @ S, np.abs(B) @ np.abs(S))
        return al * P + be * C0, abs(al) * Pa + abs(be) * np.abs(C0), None
    if op in ("syrk", "syr2k"):
        uplo, trans = case[2], case[3]
        N, K, al, be = L3_SYRK
        A, B, C0 = (x.astype(np.float64) for x in l3_inputs(tag, op, *case[1:]))
        oA, oB = (A.T, B.T) if trans == Trans else (A, B)
        if op == "syrk":
            P, Pa = oA @ oA.T, np.abs(oA) @ np.abs(oA).T
        else:
            P = oA @ oB.T + oB @ oA.T
            Pa = np.abs(oA) @ np.abs(oB).T + np.abs(oB) @ np.abs(oA).T
        keep = np.triu(np.ones((N, N), bool)) if uplo == Upper else np.tril(np.ones((N, N), bool))
        out = np.where(keep, al * P + be * C0, C0)
        return out, np.where(keep, abs(al) * Pa + abs(be) * np.abs(C0), 1.0), ~keep
    side, uplo, trans, diag = case[2:]
    M, N, al = L3_TRXM
    A, B = (x.astype(np.float64) for x in l3_inputs(tag, op, *case[1:]))
    T = np.triu(A) if uplo == Upper else np.tril(A)
    if diag == Unit:
        np.fill_diagonal(T, 1.0)
    if trans == Trans:
        T = T.T
    if op == "trmm":
        P, Pa = (T @ B, np.abs(T) @ np.abs(B)) if side == Left else (B @ T, np.abs(B) @ np.abs(T))
        return al * P, abs(al) * Pa, None
    X = np.linalg.solve(T, al * B) if side == Left else np.linalg.solve(T.T, al * B.T).T
    return X, np.full(X.shape, np.abs(X).max()), None


CASES = [(tag, case) for tag in "sd" for case in l3_cases()]


@pytest.mark.parametrize("tag,case", CASES, ids=[l3_key(t, c) for t, c in CASES])
def test_restated_level3_matches_reference_cblas(tag, case):
    ref = REF[l3_key(tag, case)].astype(np.float64)
    want, scale, untouched = restated(tag, case)
    assert ref.shape == want.shape
    if untouched is not None:   # SYRK / SYR2K: the other triangle is C0, bit for bit
        C0 = l3_inputs(tag, case[0], *case[1:])[2].astype(np.float64)
        assert np.array_equal(ref[untouched], C0[untouched])
    err = np.abs(ref - want) / np.maximum(scale, 1e-300)
    assert err.max() <= TOL[tag] * (50 if case[0] == "trsm" else 1), (case, err.max())
