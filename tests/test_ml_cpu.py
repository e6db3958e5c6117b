"""CPU checks of the ML-operation oracle (oracle/ml_ref.py): the ggml block formats through an independent packer
(values chosen first, packed into the published bit layout, then dequantized back), the closed forms of the
activations, and invariants of RoPE, interpolation and attention. No GPU."""
import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
import ml_ref  # noqa: E402

rng = np.random.default_rng(11)


def _f16_bytes(v):
    return np.array([v], np.float16).view(np.uint8)


def test_q8_0_round_trip():
    q = rng.integers(-128, 128, size=(3, 64)).astype(np.int8)
    d = np.float16(0.0371)
    W = np.zeros((3, 2 * 34), np.uint8)
    for j in range(2):
        W[:, 34 * j:34 * j + 2] = _f16_bytes(d)
        W[:, 34 * j + 2:34 * j + 34] = q[:, 32 * j:32 * j + 32].view(np.uint8)
    out = ml_ref.dequant_rows(W, 0, 64)
    assert np.array_equal(out, q.astype(np.float32) * np.float32(d))


def _pack_q4k_scales(sc, mn):
    """ggml Q4_K: 8 six-bit (scale, min) pairs in 12 bytes -- scales 0..3 and mins 0..3 in the low 6 bits of bytes 0..7,
    scales / mins 4..7 as low / high nibbles of bytes 8..11 with their top 2 bits in the top bits of bytes 0..7."""
    b = np.zeros(12, np.int64)
    for i in range(4):
        b[i] = sc[i] & 63 | ((sc[i + 4] >> 4) << 6)
        b[i + 4] = mn[i] & 63 | ((mn[i + 4] >> 4) << 6)
        b[i + 8] = (sc[i + 4] & 0xF) | ((mn[i + 4] & 0xF) << 4)
    return b.astype(np.uint8)


def test_q4_k_round_trip():
    K = 512
    W = np.zeros((2, K // 256 * 144), np.uint8)
    want = np.zeros((2, K), np.float32)
    for n in range(2):
        for j in range(K // 256):
            d, dmin = np.float16(0.0123), np.float16(0.0045)
            sc, mn = rng.integers(0, 64, 8), rng.integers(0, 64, 8)
            q = rng.integers(0, 16, 256)
            o = 144 * j
            W[n, o:o + 2], W[n, o + 2:o + 4] = _f16_bytes(d), _f16_bytes(dmin)
            W[n, o + 4:o + 16] = _pack_q4k_scales(sc, mn)
            for g in range(4):   # 64 values per group: low nibbles first 32, high nibbles next 32
                lo, hi = q[64 * g:64 * g + 32], q[64 * g + 32:64 * g + 64]
                W[n, o + 16 + 32 * g:o + 16 + 32 * g + 32] = (lo | (hi << 4)).astype(np.uint8)
            for s in range(8):
                vals = q[32 * s:32 * s + 32].astype(np.float32)
                want[n, 256 * j + 32 * s:256 * j + 32 * s + 32] = \
                    (np.float32(d) * np.float32(sc[s])) * vals - np.float32(dmin) * np.float32(mn[s])
    assert np.array_equal(ml_ref.dequant_rows(W, 1, K), want)


def test_q6_k_round_trip():
    K = 256
    q = rng.integers(-32, 32, K)             # signed 6-bit quants
    sc = rng.integers(-128, 128, 16)         # int8 scales of 16-value sub-blocks
    d = np.float16(0.0021)
    W = np.zeros((1, 210), np.uint8)
    u = (q + 32).astype(np.int64)
    for h in range(2):                       # 128 values per half: ql (64 B), qh (32 B)
        base = 128 * h
        for l in range(32):
            v = [u[base + l], u[base + l + 32], u[base + l + 64], u[base + l + 96]]
            W[0, 64 * h + l] = (v[0] & 0xF) | ((v[2] & 0xF) << 4)
            W[0, 64 * h + l + 32] = (v[1] & 0xF) | ((v[3] & 0xF) << 4)
            W[0, 128 + 32 * h + l] = (v[0] >> 4) | ((v[1] >> 4) << 2) | ((v[2] >> 4) << 4) | ((v[3] >> 4) << 6)
    W[0, 192:208] = sc.astype(np.int8).view(np.uint8)
    W[0, 208:210] = _f16_bytes(d)
    want = np.array([(np.float32(d) * np.float32(sc[k // 16])) * np.float32(q[k]) for k in range(K)], np.float32)
    assert np.array_equal(ml_ref.dequant_rows(W, 2, K)[0], want)


def test_random_blocks_have_finite_small_scales():
    for qt in (0, 1, 2):
        K = 256
        W = ml_ref.random_blocks(rng, qt, 4, K)
        v = ml_ref.dequant_rows(W, qt, K)
        assert np.all(np.isfinite(v)) and np.max(np.abs(v)) < 65504


def test_gelu_forms():
    x = np.linspace(-12, 12, 2001, dtype=np.float32)
    g = ml_ref.gelu(x)
    assert np.array_equal(g[x <= -10], np.zeros(np.sum(x <= -10), np.float32))
    assert np.array_equal(g[x >= 10], x[x >= 10])
    mid = np.abs(x) < 10
    assert np.array_equal(g[mid], g[mid].astype(np.float16).astype(np.float32))   # FP16 table values
    ge = ml_ref.gelu_erf(x)
    assert np.max(np.abs(g - ge)) < 2e-2                                # tanh approximation of the erf form
    assert np.array_equal(ml_ref.relu(x), np.maximum(x, 0))


def test_norms_closed_form():
    X = rng.standard_normal((5, 77)).astype(np.float32)
    Y = ml_ref.rms_norm(X, None, 1e-6)
    assert np.allclose(np.mean(Y.astype(np.float64) ** 2, axis=1), 1.0, rtol=1e-5)
    L = ml_ref.layer_norm(X, None, None, 1e-5)
    assert np.allclose(L.mean(axis=1), 0, atol=1e-6) and np.allclose(L.var(axis=1), 1, rtol=1e-4)


@pytest.mark.parametrize("neox", [0, 1])
def test_rope_is_a_rotation(neox):
    X = rng.standard_normal((4, 3, 64)).astype(np.float32)
    pos = np.array([0, 1, 17, 400], np.int32)
    Y = ml_ref.rope(X, pos, None, neox, 10000.0, 1.0, 0.0, 1.0, (0.0, 0.0))
    assert np.array_equal(Y[0], X[0])                                   # position 0: identity
    i0 = np.arange(32) if neox else 2 * np.arange(32)
    i1 = i0 + 32 if neox else i0 + 1
    nx = X[..., i0] ** 2 + X[..., i1] ** 2
    ny = Y[..., i0] ** 2 + Y[..., i1] ** 2
    assert np.allclose(nx, ny, rtol=1e-5)
    # MROPE with one section and equal positions is NEOX RoPE
    p4 = np.concatenate([pos] * 4)
    M = ml_ref.rope_multi(X, p4, None, (32, 0, 0, 0), 0, 10000.0, 1.0, 0.0, 1.0, (0.0, 0.0))
    N = ml_ref.rope(X, pos, None, 1, 10000.0, 1.0, 0.0, 1.0, (0.0, 0.0))
    assert np.array_equal(M, N)


def test_upscale_nearest_integer_factor_is_repeat():
    S = rng.standard_normal((1, 2, 3, 4)).astype(np.float32)
    D = ml_ref.upscale(S, (1, 2, 6, 12), 0)
    assert np.array_equal(D, np.repeat(np.repeat(S, 2, axis=2), 3, axis=3))
    B = ml_ref.upscale(S, (1, 2, 3, 4), 1)                              # bilinear at scale 1: identity
    assert np.allclose(B, S, atol=1e-6)


def test_attention_single_key_returns_its_value():
    Q = rng.standard_normal((2, 4, 8)).astype(np.float32)
    K = rng.standard_normal((5, 2, 8)).astype(np.float16)
    V = rng.standard_normal((5, 2, 8)).astype(np.float16)
    O = ml_ref.attention(Q, K, V, 0.3, [1, 5])
    assert np.allclose(O[0], V[0].astype(np.float64)[[0, 0, 1, 1]])
