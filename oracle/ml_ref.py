"""CPU restatement of the neural-network operations of the reference (lib/gen9blas_ml.h of kprzybys/gen9-gpu-blas;
kernels in lib/kernels/hgemm.cl, host code in lib/src/ops.c and lib/src/packed.c), in NumPy.

TEST INFRASTRUCTURE: only tests/, __graft_entry__.smoke() and bench.py's CPU legs may use this module, as the checker.
The library never calls it.

Parity unpinned: the reference ships no tests, fixtures or golden vectors for these operations, so this restatement
follows its kernels' arithmetic (which follows ggml-cpu): the same operations in the same order in float32 where
the kernel works in float32 (NumPy float32 arithmetic is correctly rounded and never contracts a multiply-add),
FP16 conversions rounding to nearest even (NumPy's float32 -> float16 cast). The GEMMs accumulate in float64 and round
to FP16 once, as the accurate FP16 GEMM's result is; the GPU accumulates in FP32, so products can differ by one FP16 ulp.
"""
import ctypes
import ctypes.util
import math

import numpy as np

f32, f16 = np.float32, np.float16

_libm = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
_libm.powf.restype, _libm.powf.argtypes = ctypes.c_float, [ctypes.c_float, ctypes.c_float]
for _fn in ("tanhf", "expf", "erff"):
    getattr(_libm, _fn).restype, getattr(_libm, _fn).argtypes = ctypes.c_float, [ctypes.c_float]


def _libm_map(name, x):
    """The C library's float function on every element (ggml-cpu calls tanhf / expf / erff; NumPy's own float32
    tanh differs from glibc's in the last bit for about a fifth of the arguments)."""
    fn = getattr(_libm, name)
    x = np.asarray(x, f32)
    return np.array([fn(float(v)) for v in x.ravel()], f32).reshape(x.shape)


def theta_scale(freq_base, n_dims):
    """powf(freq_base, -2 / n_dims) from the C library, as the host code computes it (lib/src/ops.c:191): NumPy's
    float32 power may differ in the last bit, and RoPE multiplies that bit up to pos * ts^j."""
    return f32(_libm.powf(f32(freq_base), f32(-2.0) / f32(n_dims)))


def to_f16(x):
    """float32 -> FP16, round to nearest even, as float32 values."""
    return np.asarray(x, f32).astype(f16).astype(f32)


# ------------------------------------------------------------------------------------------- activations
def gelu(x):
    """ggml GELU, tanh form, with ggml-cpu's FP16 table: x <= -10 -> 0, x >= 10 -> x, else fp16(gelu(fp16(x))).
    Reference: lib/kernels/hgemm.cl:631-638 (epi_gelu, contraction off)."""
    x = np.asarray(x, f32)
    h = to_f16(x)
    inner = (f32(0.79788456080286535588) * h) * (f32(1) + f32(0.044715) * (h * h))
    g = (f32(0.5) * h) * (f32(1) + _libm_map("tanhf", inner))
    return np.where(x <= -10, f32(0), np.where(x >= 10, x, to_f16(g))).astype(f32)


def gelu_erf(x):
    """ggml GELU_ERF: 0.5 x (1 + erf(x / sqrt 2)) in float32. Reference: lib/kernels/hgemm.cl:1383-1387."""
    x = np.asarray(x, f32)
    e = _libm_map("erff", x * f32(0.70710678118654752440))
    return (f32(0.5) * x) * (f32(1) + e)


def relu(x):
    """ggml RELU (x > 0 ? x : 0). Reference: lib/kernels/hgemm.cl:1377-1381."""
    x = np.asarray(x, f32)
    return np.where(x > 0, x, f32(0)).astype(f32)


def silu_mul(g, u):
    """ggml SWIGLU of FP16 values: g / (1 + e^-g) * u in float32. Reference: lib/kernels/hgemm.cl:680-690."""
    g, u = np.asarray(g, f32), np.asarray(u, f32)
    with np.errstate(over="ignore"):
        return (g / (f32(1) + _libm_map("expf", -g))) * u


# ------------------------------------------------------------------------------------------- norms
def rms_norm(X, w, eps):
    """ggml RMS_NORM [* w]: mean of squares (sum in float64, as ggml-cpu's ggml_float), scale = 1 / sqrt(mean + eps) in
    float32, y = (x * scale) * w. Reference: lib/kernels/hgemm.cl:1003-1024."""
    X = np.asarray(X, f32)
    mean = (np.sum(X.astype(np.float64) ** 2, axis=1) / X.shape[1]).astype(f32)
    scale = f32(1) / np.sqrt(mean + f32(eps)).astype(f32)
    Y = X * scale[:, None]
    return Y * np.asarray(w, f32)[None, :] if w is not None else Y


def layer_norm(X, w, b, eps):
    """ggml NORM [* w] [+ b]: mean, variance of (x - mean) (float64 sums), scale = 1 / sqrt(var + eps) in float32.
    Reference: lib/kernels/hgemm.cl:1272-1300."""
    X = np.asarray(X, f32)
    K = X.shape[1]
    mean = (np.sum(X.astype(np.float64), axis=1) / K).astype(f32)
    d = X - mean[:, None]
    var = (np.sum(d.astype(np.float64) ** 2, axis=1) / K).astype(f32)
    scale = f32(1) / np.sqrt(var + f32(eps)).astype(f32)
    Y = d * scale[:, None]
    if w is not None:
        Y = Y * np.asarray(w, f32)[None, :]
    if b is not None:
        Y = Y + np.asarray(b, f32)[None, :]
    return Y


# ------------------------------------------------------------------------------------------- RoPE
def _yarn(theta_extrap, j, freq_scale, ext_factor, attn_factor, corr):
    theta_interp = f32(freq_scale) * theta_extrap
    th, mscale = theta_interp, f32(attn_factor)
    if ext_factor != 0:
        yv = (f32(j) - f32(corr[0])) / max(f32(0.001), f32(corr[1]) - f32(corr[0]))
        ramp = (f32(1) - min(f32(1), max(f32(0), f32(yv)))) * f32(ext_factor)
        th = theta_interp * (f32(1) - ramp) + theta_extrap * ramp
        mscale = mscale * (f32(1) + f32(0.1) * f32(math.log(float(f32(1) / f32(freq_scale)))))
    return f32(math.cos(float(th))) * mscale, f32(math.sin(float(th))) * mscale


def rope(X, pos, ff, neox, freq_base, freq_scale, ext_factor, attn_factor, corr):
    """ggml ROPE forward on X [n_tok][nh][n_dims]: pair j rotated by theta = pos * theta_scale^j (repeated float32
    multiplication), / ff[j], rope_yarn. NORMAL pairs (2j, 2j+1), NEOX (j, j + n_dims/2).
    Reference: lib/kernels/hgemm.cl:1032-1061, lib/src/ops.c:176-199."""
    X = np.asarray(X, f32)
    n_tok, nh, n_dims = X.shape
    Y = X.copy()
    ts = theta_scale(freq_base, n_dims)
    for t in range(n_tok):
        theta = f32(pos[t])
        for j in range(n_dims // 2):
            te = theta / f32(ff[j]) if ff is not None else theta
            c, s = _yarn(te, j, freq_scale, ext_factor, attn_factor, corr)
            i0, i1 = (j, j + n_dims // 2) if neox else (2 * j, 2 * j + 1)
            x0, x1 = X[t, :, i0], X[t, :, i1]
            Y[t, :, i0] = x0 * c - x1 * s
            Y[t, :, i1] = x0 * s + x1 * c
            theta = theta * ts
    return Y


def rope_multi(X, pos, ff, sections, vision, freq_base, freq_scale, ext_factor, attn_factor, corr):
    """ggml_rope_multi on X [n_tok][nh][ne0]. MROPE (vision 0, ne0 = n_dims): NEOX pairs (j, j + n_dims/2), pair j at
    the position of its sector; VISION (vision 1, ne0 = 2 n_dims): pairs (j, j + n_dims), the power of theta restarted
    at each section start. pos: 4 * n_tok ints (t, h, w, e). Reference: lib/kernels/hgemm.cl:1062-1115."""
    X = np.asarray(X, f32)
    n_tok, nh, ne0 = X.shape
    n_dims = ne0 // 2 if vision else ne0
    npairs = n_dims if vision else n_dims // 2
    s0, s1, s2, s3 = sections
    sd = s0 + s1 + s2 + s3
    ts = theta_scale(freq_base, n_dims)
    Y = X.copy()
    for t in range(n_tok):
        p = [f32(pos[t + c * n_tok]) for c in range(4)]
        th = list(p)

        def restart(sk):
            if sk == 0:
                th[0] = p[0]
            elif sk == s0:
                th[1] = p[1]
            elif sk == s0 + s1:
                th[2] = p[2]
            elif sk == s0 + s1 + s2:
                th[3] = p[3]

        for j in range(npairs):
            sector = j % sd
            sec = 0 if sector < s0 else 1 if sector < s0 + s1 else 2 if sector < s0 + s1 + s2 else 3
            if vision:
                restart(sector)
            theta = th[sec]
            te = theta / f32(ff[j]) if ff is not None else theta
            c, s = _yarn(te, j, freq_scale, ext_factor, attn_factor, corr)
            x0, x1 = X[t, :, j], X[t, :, j + npairs]
            Y[t, :, j] = x0 * c - x1 * s
            Y[t, :, j + npairs] = x0 * s + x1 * c
            th = [v * ts for v in th]
    return Y


# ------------------------------------------------------------------------------------------- layout ops
def im2col(X, KH, KW, OH, OW, s0, s1, p0, p1, d0, d1):
    """ggml IM2COL: X [N, IC, IH, IW] -> [N, OH, OW, IC*KH*KW], zero padding. Reference: lib/kernels/hgemm.cl:1366-1376."""
    X = np.asarray(X, f32)
    N, IC, IH, IW = X.shape
    Y = np.zeros((N, OH, OW, IC * KH * KW), f32)
    for n in range(N):
        for oh in range(OH):
            for ow in range(OW):
                for c in range(IC):
                    for kh in range(KH):
                        for kw in range(KW):
                            iw, ih = ow * s0 + kw * d0 - p0, oh * s1 + kh * d1 - p1
                            if 0 <= ih < IH and 0 <= iw < IW:
                                Y[n, oh, ow, (c * KH + kh) * KW + kw] = X[n, c, ih, iw]
    return Y


def upscale(S, dshape, mode_flags):
    """ggml UPSCALE / interpolate, F32, S [ne3][ne2][ne1][ne0] -> dshape: nearest, bilinear (pixel offset 0.5, or 0
    with align corners), bilinear + antialias (triangle filter). Reference: lib/kernels/hgemm.cl:1130-1172,
    lib/src/ops.c:284-312."""
    S = np.asarray(S, f32)
    sne = S.shape[::-1]
    dne = dshape[::-1]
    mode, ac, aa = mode_flags & 0xFF, (mode_flags >> 8) & 1, (mode_flags >> 9) & 1
    sf = [f32(dne[i]) / f32(sne[i]) for i in range(4)]
    po = f32(0.5)
    if ac:
        po = f32(0)
        for i in (0, 1):
            if dne[i] > 1 and sne[i] > 1:
                sf[i] = f32(dne[i] - 1) / f32(sne[i] - 1)
    D = np.zeros(dshape, f32)
    for i3 in range(dne[3]):
        for i2 in range(dne[2]):
            plane = S[int(f32(i3) / sf[3]), int(f32(i2) / sf[2])]
            for i1 in range(dne[1]):
                for i0 in range(dne[0]):
                    if mode == 0:
                        v = plane[int(f32(i1) / sf[1]), int(f32(i0) / sf[0])]
                    elif aa:
                        sup1, sup0 = max(f32(1), f32(1) / sf[1]), max(f32(1), f32(1) / sf[0])
                        inv1, inv0 = f32(1) / sup1, f32(1) / sup0
                        yy, xx = (f32(i1) + po) / sf[1], (f32(i0) + po) / sf[0]
                        x_min, x_max = max(int(xx - sup0 + po), 0), min(int(xx + sup0 + po), sne[0])
                        y_min, y_max = max(int(yy - sup1 + po), 0), min(int(yy + sup1 + po), sne[1])
                        acc, tw = f32(0), f32(0)
                        for sy in range(y_min, y_max):
                            wy = max(f32(1) - abs((f32(sy) - yy + po) * inv1), f32(0))
                            for sx in range(x_min, x_max):
                                wx = max(f32(1) - abs((f32(sx) - xx + po) * inv0), f32(0))
                                w = wx * wy
                                if w <= 0:
                                    continue
                                acc = acc + plane[sy, sx] * w
                                tw = tw + w
                        v = acc / tw if tw > 0 else acc
                    else:
                        yy, xx = (f32(i1) + po) / sf[1] - po, (f32(i0) + po) / sf[0] - po
                        y0, x0 = int(math.floor(yy)), int(math.floor(xx))
                        y1, x1 = y0 + 1, x0 + 1
                        cl = lambda v, n: max(0, min(v, n - 1))   # noqa: E731
                        y0, y1, x0, x1 = cl(y0, sne[1]), cl(y1, sne[1]), cl(x0, sne[0]), cl(x1, sne[0])
                        dy = max(f32(0), min(yy - f32(y0), f32(1)))
                        dx = max(f32(0), min(xx - f32(x0), f32(1)))
                        a, b, c, d = plane[y0, x0], plane[y0, x1], plane[y1, x0], plane[y1, x1]
                        v = a * (1 - dx) * (1 - dy) + b * dx * (1 - dy) + c * (1 - dx) * dy + d * dx * dy
                    D[i3, i2, i1, i0] = v
    return D


# ------------------------------------------------------------------------------------------- quantized weights
def dequant_rows(W, qtype, K):
    """ggml dequantize_row_q8_0 / _q4_K / _q6_K of N rows (uint8 [N][row_bytes]) -> float32 [N][K], then the caller
    rounds to FP16. Reference: lib/kernels/hgemm.cl:692-745 (gen9blas_dequant_b16, ggml's arithmetic order)."""
    W = np.asarray(W, np.uint8)
    N = W.shape[0]
    out = np.zeros((N, K), f32)
    hf = lambda b, o: f32(np.frombuffer(bytes(b[o:o + 2]), f16)[0])   # noqa: E731
    for n in range(N):
        row = W[n]
        if qtype == 0:
            for j in range(K // 32):
                b = row[j * 34:(j + 1) * 34]
                d = hf(b, 0)
                out[n, j * 32:(j + 1) * 32] = b[2:34].view(np.int8).astype(f32) * d
        elif qtype == 1:
            for j in range(K // 256):
                b = row[j * 144:(j + 1) * 144]
                d, dmin = hf(b, 0), hf(b, 2)
                s, q = b[4:16].astype(np.int64), b[16:144].astype(np.int64)

                def sm(i):
                    if i < 4:
                        return s[i] & 63, s[i + 4] & 63
                    return (s[i + 4] & 0xF) | ((s[i - 4] >> 6) << 4), (s[i + 4] >> 4) | ((s[i] >> 6) << 4)

                for g in range(4):
                    sc0, m0 = sm(2 * g)
                    sc1, m1 = sm(2 * g + 1)
                    d1, mm1, d2, mm2 = d * f32(sc0), dmin * f32(m0), d * f32(sc1), dmin * f32(m1)
                    qq = q[32 * g:32 * g + 32]
                    base = j * 256 + 64 * g
                    out[n, base:base + 32] = d1 * (qq & 0xF).astype(f32) - mm1
                    out[n, base + 32:base + 64] = d2 * (qq >> 4).astype(f32) - mm2
        else:
            for j in range(K // 256):
                b = row[j * 210:(j + 1) * 210]
                d = hf(b, 208)
                for h in range(2):
                    ql = b[64 * h:64 * h + 64].astype(np.int64)
                    qh = b[128 + 32 * h:128 + 32 * h + 32].astype(np.int64)
                    sc = b[192 + 8 * h:192 + 8 * h + 8].view(np.int8).astype(f32)
                    base = j * 256 + 128 * h
                    for l in range(32):
                        is_ = l // 16
                        q1 = ((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32
                        q2 = ((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32
                        q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32
                        q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32
                        out[n, base + l] = d * sc[is_] * f32(q1)
                        out[n, base + l + 32] = d * sc[is_ + 2] * f32(q2)
                        out[n, base + l + 64] = d * sc[is_ + 4] * f32(q3)
                        out[n, base + l + 96] = d * sc[is_ + 6] * f32(q4)
    return out


BLOCK = {0: (32, 34), 1: (256, 144), 2: (256, 210)}


def random_blocks(rng, qtype, N, K, dmax=0.01):
    """N rows of K values in the block layout of qtype with random quants and FP16 block scales in (0, dmax]: any byte
    pattern of the quant and scale fields is a valid block."""
    qb, bb = BLOCK[qtype]
    W = rng.integers(0, 256, size=(N, K // qb * bb), dtype=np.uint8)
    for j in range(K // qb):
        o = j * bb
        scales = (rng.uniform(0.1, 1.0, size=(N, 2)) * dmax).astype(f16).view(np.uint8).reshape(N, 4)
        if qtype == 0:
            W[:, o:o + 2] = scales[:, :2]
        elif qtype == 1:
            W[:, o:o + 4] = scales
        else:
            W[:, o + 208:o + 210] = scales[:, :2]
    return W


# ------------------------------------------------------------------------------------------- FP16-weight GEMMs
def gemm_f16w(A, W16, bias=None, gelu_=False, R=None):
    """gemm_pb_f16w(_ex): C = [gelu](fp16(fp16(A) . W16^T) + bias) [+ R] in float32 (the product accumulated in
    float64 and rounded to FP16 once). Reference: lib/src/packed.c:250-330, epilogue lib/kernels/hgemm.cl:639-662."""
    a = to_f16(A).astype(np.float64)
    with np.errstate(over="ignore"):
        raw = (a @ np.asarray(W16, f16).astype(np.float64).T).astype(f32).astype(f16).astype(f32)
    v = raw.copy()
    if bias is not None:
        v = v + np.asarray(bias, f32)[None, :]
    if gelu_:
        v = gelu(v)
    if R is not None:
        v = v + np.asarray(R, f32)
    return v, raw


def ffn_f16w(X, Wg, Wu, Wd):
    """Gated FFN: y = fp16(fp16(silu(g) * u) . Wd^T) with g, u = fp16(fp16(X) . W^T). Reference: lib/src/packed.c:365-474,
    lib/kernels/hgemm.cl:680-690."""
    _, g = gemm_f16w(X, Wg)
    _, u = gemm_f16w(X, Wu)
    h = to_f16(silu_mul(g, u))
    _, y = gemm_f16w(h, Wd)
    return y


# ------------------------------------------------------------------------------------------- attention
def attention(Q, K, V, scale, vis):
    """Softmax attention of one stream in float64: Q [nq][H][D] (float32), K / V [nk][HKV][D] (FP16), token t sees keys
    [0, vis[t]); query head h uses KV head h // (H / HKV). Returns O [nq][H][D]. Reference: lib/kernels/hgemm.cl:1174-1256
    (split over key chunks and merged; mathematically this softmax)."""
    Q = np.asarray(Q, np.float64)
    K = np.asarray(K, f16).astype(np.float64)
    V = np.asarray(V, f16).astype(np.float64)
    nq, H, D = Q.shape
    HKV = K.shape[1]
    G = H // HKV
    O = np.zeros((nq, H, D))
    for t in range(nq):
        n = vis[t]
        for h in range(H):
            s = (K[:n, h // G, :] @ Q[t, h]) * scale
            p = np.exp(s - s.max())
            O[t, h] = (p @ V[:n, h // G, :]) / p.sum()
    return O
