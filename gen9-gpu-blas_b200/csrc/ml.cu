// ml.cu -- the elementwise ggml operations, the packed GEMM input of a normalisation and attention of the reference's
// neural-network header (lib/gen9blas_ml.h:61-153 of kprzybys/gen9-gpu-blas; host code lib/src/ops.c, lib/src/attn.c;
// kernels gen9blas_rms_norm ... gen9blas_set_rows_f16, gen9blas_attn_dec_part / _comb in lib/kernels/hgemm.cl).
//
// Semantics follow the reference (and through it ggml-cpu): the arithmetic of each op in the same order, without
// multiply-add contraction where the reference turns it off, FP16 conversions rounding to nearest even. What differs
// on B200: operands in device or managed memory are used in place; host memory is staged through device buffers, so a
// call on host memory completes before it returns (the reference's gen9blas_span registration is then not needed:
// gen9blas_span accepts every region). sync = 0 with every operand on the device queues the work, like no-wait mode.
// Row reductions (RMS norm, layer norm) accumulate in FP64 (ggml-cpu's ggml_float); the reference sums in FP32.
// Attention: one split-K kernel over key chunks (online softmax in FP32, exp2 with the scale folded into the query) and a
// merge kernel serve decoding (attn_dec) and the prefill entry points (attn_f16kv, attn_f16kv_streams), which are the
// same computation with one stream and per-token visible key counts.
#include "common.cuh"
#include "gen9blas_ml.h"
#include "internal.h"
#include "sm100.cuh"
#include <cmath>
#include <cstring>
#include <new>

using namespace g9;

namespace {

unsigned grid_n(long long n, int sms) {
    const long long b = (n + 255) / 256;
    return (unsigned)(b < 16LL * sms ? (b > 0 ? b : 1) : 16LL * sms);
}

bool on_device(const void *p) {
    cudaPointerAttributes a;
    if (!p || cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

// Operand handling of these ops: up to three big operands through the staging slots (map_operand), small read-only
// ones (weights, biases, positions, indices) in place when on the device, else copied into the ML work buffer.
struct OpCall {
    Operand ops[3];
    int n = 0;
    bool all_dev = true;
    char *small = nullptr;
    size_t small_used = 0, small_cap = 0;

    int big(const void *p, size_t bytes, bool read, bool written, void **dptr) {
        Operand &o = ops[n];
        G9_TRY(map_operand(o, p, bytes, n, read, written));
        all_dev = all_dev && o.zc;
        *dptr = o.dptr;
        n++;
        return 0;
    }
    int reserve(size_t bytes) {
        small_cap = bytes;
        if (!bytes) return 0;
        void *b = nullptr;
        G9_TRY(ml_buffer(bytes, &b));
        small = (char *)b;
        return 0;
    }
    int in(const void *p, size_t bytes, const void **dptr, cudaStream_t st) {
        if (!p) {
            *dptr = nullptr;
            return 0;
        }
        if (on_device(p)) {
            *dptr = p;
            return 0;
        }
        all_dev = false;
        const size_t at = (small_used + 255) / 256 * 256;
        if (at + bytes > small_cap) return fail(GEN9BLAS_ERR, "internal: small-operand space");
        G9_CU(cudaMemcpyAsync(small + at, p, bytes, cudaMemcpyHostToDevice, st));
        small_used = at + bytes;
        *dptr = small + at;
        return 0;
    }
    // sync = 0 and every operand on the device: queued (like no-wait mode); otherwise waits.
    int finish(int sync) {
        const bool saved = G.nowait;
        G.nowait = !sync && all_dev;
        int r = finish_op(ops, n);
        G.nowait = saved;
        return r;
    }
};

size_t round256(size_t b) { return (b + 255) / 256 * 256; }

// ---------------------------------------------------------------------------------------------- normalisations
// One CTA of 256 threads per row; FP64 partial sums combined in a fixed order (deterministic).
__device__ double block_sum(double v, double *sh) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) sh[w] = v;
    __syncthreads();
    double t = 0.0;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) t += sh[i];
    return t;
}

// ggml RMS_NORM (+ MUL by w): scale = 1 / sqrt(mean(x²) + eps) in FP32 from an FP64 sum; y = (x · scale) · w.
__global__ void __launch_bounds__(256) rms_norm_k(const float *__restrict__ x, long long ldx, const float *__restrict__ w,
                                                  float eps, float *__restrict__ y, long long ldy, int K) {
    __shared__ double sh[8];
    const float *xr = x + blockIdx.x * ldx;
    double s = 0.0;
    for (int i = threadIdx.x; i < K; i += blockDim.x) s += (double)xr[i] * (double)xr[i];
    s = block_sum(s, sh);
    const float mean = (float)(s / K);
    const float scale = __frcp_rn(__fsqrt_rn(__fadd_rn(mean, eps)));
    float *yr = y + blockIdx.x * ldy;
    for (int i = threadIdx.x; i < K; i += blockDim.x) {
        float v = __fmul_rn(xr[i], scale);
        if (w) v = __fmul_rn(v, w[i]);
        yr[i] = v;
    }
}

// The same two norms with 16-byte accesses, for rows (and w, b) 16-byte aligned and K % 4 == 0: the same FP32
// operations per element; the FP64 partial sums are taken four elements at a time.
__global__ void __launch_bounds__(256) rms_norm_v4_k(const float *__restrict__ x, long long ldx, const float *__restrict__ w,
                                                     float eps, float *__restrict__ y, long long ldy, int K) {
    __shared__ double sh[8];
    const float4 *xr = reinterpret_cast<const float4 *>(x + blockIdx.x * ldx);
    const int K4 = K / 4;
    double s = 0.0;
    for (int i = threadIdx.x; i < K4; i += blockDim.x) {
        const float4 v = xr[i];
        s += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
    }
    s = block_sum(s, sh);
    const float mean = (float)(s / K);
    const float scale = __frcp_rn(__fsqrt_rn(__fadd_rn(mean, eps)));
    float4 *yr = reinterpret_cast<float4 *>(y + blockIdx.x * ldy);
    const float4 *w4 = reinterpret_cast<const float4 *>(w);
    for (int i = threadIdx.x; i < K4; i += blockDim.x) {
        const float4 v = xr[i];
        float4 o = make_float4(__fmul_rn(v.x, scale), __fmul_rn(v.y, scale), __fmul_rn(v.z, scale), __fmul_rn(v.w, scale));
        if (w) {
            const float4 q = w4[i];
            o = make_float4(__fmul_rn(o.x, q.x), __fmul_rn(o.y, q.y), __fmul_rn(o.z, q.z), __fmul_rn(o.w, q.w));
        }
        yr[i] = o;
    }
}

__global__ void __launch_bounds__(256) layer_norm_v4_k(const float *__restrict__ x, long long ldx,
                                                       const float *__restrict__ w, const float *__restrict__ b,
                                                       float eps, float *__restrict__ y, long long ldy, int K) {
    __shared__ double sh[8];
    const float4 *xr = reinterpret_cast<const float4 *>(x + blockIdx.x * ldx);
    const int K4 = K / 4;
    double s = 0.0;
    for (int i = threadIdx.x; i < K4; i += blockDim.x) {
        const float4 v = xr[i];
        s += (double)v.x + (double)v.y + (double)v.z + (double)v.w;
    }
    s = block_sum(s, sh);
    const float mean = (float)(s / K);
    double v2 = 0.0;
    for (int i = threadIdx.x; i < K4; i += blockDim.x) {
        const float4 v = xr[i];
        const double d0 = __fsub_rn(v.x, mean), d1 = __fsub_rn(v.y, mean), d2 = __fsub_rn(v.z, mean),
                     d3 = __fsub_rn(v.w, mean);
        v2 += d0 * d0 + d1 * d1 + d2 * d2 + d3 * d3;
    }
    v2 = block_sum(v2, sh);
    const float scale = __frcp_rn(__fsqrt_rn(__fadd_rn((float)(v2 / K), eps)));
    float4 *yr = reinterpret_cast<float4 *>(y + blockIdx.x * ldy);
    for (int i = threadIdx.x; i < K4; i += blockDim.x) {
        const float4 v = xr[i];
        float o[4] = {__fmul_rn(__fsub_rn(v.x, mean), scale), __fmul_rn(__fsub_rn(v.y, mean), scale),
                      __fmul_rn(__fsub_rn(v.z, mean), scale), __fmul_rn(__fsub_rn(v.w, mean), scale)};
        if (w) {
            const float4 q = reinterpret_cast<const float4 *>(w)[i];
            o[0] = __fmul_rn(o[0], q.x); o[1] = __fmul_rn(o[1], q.y); o[2] = __fmul_rn(o[2], q.z); o[3] = __fmul_rn(o[3], q.w);
        }
        if (b) {
            const float4 q = reinterpret_cast<const float4 *>(b)[i];
            o[0] = __fadd_rn(o[0], q.x); o[1] = __fadd_rn(o[1], q.y); o[2] = __fadd_rn(o[2], q.z); o[3] = __fadd_rn(o[3], q.w);
        }
        yr[i] = make_float4(o[0], o[1], o[2], o[3]);
    }
}

bool on16(const void *p) { return ((uintptr_t)p & 15) == 0; }

// ggml NORM (+ MUL by w, ADD b): mean and variance over the row (FP64 sums, FP32 mean / scale),
// y = (x − mean) · scale [· w] [+ b]; pack: also FP16 rows of Kp (zero past K) for a following GEMM.
__global__ void __launch_bounds__(256) layer_norm_k(const float *__restrict__ x, long long ldx, const float *__restrict__ w,
                                                    const float *__restrict__ b, float eps, float *__restrict__ y,
                                                    long long ldy, int K, __half *pack, int Kp) {
    __shared__ double sh[8];
    const float *xr = x + blockIdx.x * ldx;
    double s = 0.0;
    for (int i = threadIdx.x; i < K; i += blockDim.x) s += (double)xr[i];
    s = block_sum(s, sh);
    const float mean = (float)(s / K);
    double v2 = 0.0;
    for (int i = threadIdx.x; i < K; i += blockDim.x) {
        const double d = (double)__fsub_rn(xr[i], mean);
        v2 += d * d;
    }
    v2 = block_sum(v2, sh);
    const float scale = __frcp_rn(__fsqrt_rn(__fadd_rn((float)(v2 / K), eps)));
    float *yr = y + blockIdx.x * ldy;
    for (int i = threadIdx.x; i < (pack ? Kp : K); i += blockDim.x) {
        float v = 0.0f;
        if (i < K) {
            v = __fmul_rn(__fsub_rn(xr[i], mean), scale);
            if (w) v = __fmul_rn(v, w[i]);
            if (b) v = __fadd_rn(v, b[i]);
            yr[i] = v;
        }
        if (pack) pack[(long long)blockIdx.x * Kp + i] = __float2half_rn(v);
    }
}

// ---------------------------------------------------------------------------------------------- elementwise
__global__ void binop_k(int op, int M, int K, const float *__restrict__ a, long long lda, const float *__restrict__ b,
                        long long ldb, int bs0, float *c, long long ldc) {
    const long long n = (long long)M * K;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(e / K), i = (int)(e % K);
        const float u = a[r * lda + i], v = b[r * ldb + (long long)i * bs0];
        c[r * ldc + i] = op ? __fmul_rn(u, v) : __fadd_rn(u, v);
    }
}

__global__ void unary_k(int op, long long n, const float *x, float *y) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const float v = x[i];
        float r;
        if (op == 0) r = gelu_ggml(v);
        else if (op == 1) r = __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, erff(__fmul_rn(v, 0.70710678118654752440f))));
        else r = v > 0.0f ? v : 0.0f;
        y[i] = r;
    }
}

// GELU table: gelu_ggml of every FP16 bit pattern, the function's values on (−10, 10) being fp16(gelu(fp16(x))), a
// function of fp16(x) alone (ggml-cpu reads the same kind of table). Built once per device by gelu_tab_k from the
// same device function as the fused GEMM epilogue, so a lookup gives the bits the computation gives.
__device__ __half g_gelu_tab[65536];

__global__ void gelu_tab_k() {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < 65536) g_gelu_tab[i] = __float2half_rn(gelu_ggml(__half2float(__ushort_as_half((unsigned short)i))));
}

// OP 0: GELU by the table; 1: GELU (erf form); 2: ReLU; 3: GELU computed (gelu_ggml, the table's own values).
template <int OP>
__device__ __forceinline__ float unary_f(float v, const __half *tab) {
    if (OP == 0) {
        if (v <= -10.0f) return 0.0f;
        if (v >= 10.0f) return v;
        return __half2float(tab[__half_as_ushort(__float2half_rn(v))]);
    } else if (OP == 3) {
        return gelu_ggml(v);
    } else if (OP == 1) {
        return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, erff(__fmul_rn(v, 0.70710678118654752440f))));
    }
    return v > 0.0f ? v : 0.0f;
}

// Elementwise op over 16-byte aligned float4 vectors: grid-stride with four vectors in flight per thread, the last
// n % 4 elements by the first threads of CTA 0. OP 0 (GELU) first copies the 128 KB table into shared memory (one
// 1024-thread CTA per SM).
template <int OP>
__global__ void __launch_bounds__(1024) unary_v_k(long long n, const float *x, float *y) {
    extern __shared__ __align__(16) uint8_t ut_sm[];
    const __half *tab = nullptr;
    if (OP == 0) {
        const uint4 *src = reinterpret_cast<const uint4 *>(g_gelu_tab);
        uint4 *dst = reinterpret_cast<uint4 *>(ut_sm);
        for (int i = threadIdx.x; i < 65536 * 2 / 16; i += blockDim.x) dst[i] = src[i];
        __syncthreads();
        tab = reinterpret_cast<const __half *>(ut_sm);
    }
    const long long n4 = n >> 2, stride = (long long)gridDim.x * blockDim.x;
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    float4 *y4 = reinterpret_cast<float4 *>(y);
    long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    for (; i + 3 * stride < n4; i += 4 * stride) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; u++) v[u] = x4[i + u * stride];
#pragma unroll
        for (int u = 0; u < 4; u++)
            y4[i + u * stride] = make_float4(unary_f<OP>(v[u].x, tab), unary_f<OP>(v[u].y, tab), unary_f<OP>(v[u].z, tab),
                                             unary_f<OP>(v[u].w, tab));
    }
    for (; i < n4; i += stride) {
        const float4 v = x4[i];
        y4[i] = make_float4(unary_f<OP>(v.x, tab), unary_f<OP>(v.y, tab), unary_f<OP>(v.z, tab), unary_f<OP>(v.w, tab));
    }
    if (blockIdx.x == 0 && threadIdx.x < (n & 3)) {
        const long long e = n4 * 4 + threadIdx.x;
        y[e] = unary_f<OP>(x[e], tab);
    }
}

__global__ void cvt_heads_k(int rows, int H, int D, const float *__restrict__ x, long long s_row, long long s_head,
                            __half *__restrict__ y) {
    const long long n = (long long)rows * H * D;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
        const int d = (int)(e % D), h = (int)((e / D) % H);
        const long long r = e / ((long long)H * D);
        const float v = fminf(fmaxf(x[r * s_row + (long long)h * s_head + d], -65504.0f), 65504.0f);
        y[e] = __float2half_rn(v);
    }
}

__global__ void im2col_k(int N, int IC, int IH, int IW, const float *__restrict__ x, long long ofs0, long long ofs1, int KH,
                         int KW, int OH, int OW, int s0, int s1, int p0, int p1, int d0, int d1, void *y, int f16) {
    const int Kc = IC * KH * KW;
    const long long n = (long long)N * OH * OW * Kc;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
        const int k = (int)(e % Kc);
        const int ow = (int)((e / Kc) % OW);
        const long long nh = e / ((long long)Kc * OW);
        const int nn = (int)(nh / OH), oh = (int)(nh % OH);
        const int c = k / (KH * KW), kh = (k % (KH * KW)) / KW, kw = k % KW;
        const int iw = ow * s0 + kw * d0 - p0, ih = oh * s1 + kh * d1 - p1;
        const float v = (ih < 0 || ih >= IH || iw < 0 || iw >= IW) ? 0.0f
                                                                     : x[nn * ofs0 + c * ofs1 + (long long)ih * IW + iw];
        if (f16) ((__half *)y)[e] = __float2half_rn(v);
        else ((float *)y)[e] = v;
    }
}

// ggml ROPE forward (NORMAL: pairs (2j, 2j+1); NEOX: (j, j + n_dims/2)), rope_yarn angles: theta = pos·theta_scale^j by
// repeated multiplication, divided by the frequency factor, interpolated / extrapolated as ext_factor says. One thread
// per (pair, token); the angle is applied to all heads.
__global__ void rope_k(int n_dims, int nh, int n_tok, const float *__restrict__ x, long long xs1, long long xs2, float *y,
                       long long ys1, long long ys2, const int *__restrict__ pos, const float *__restrict__ ff, int neox,
                       float theta_scale, float freq_scale, float ext_factor, float attn_factor, float corr0, float corr1) {
    const long long n = (long long)(n_dims / 2) * n_tok;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
        const int j = (int)(e % (n_dims / 2)), t = (int)(e / (n_dims / 2));
        float theta = (float)pos[t];
        for (int k = 0; k < j; k++) theta = __fmul_rn(theta, theta_scale);
        const float theta_extrap = ff ? __fdiv_rn(theta, ff[j]) : theta;
        const float theta_interp = __fmul_rn(freq_scale, theta_extrap);
        float th = theta_interp, mscale = attn_factor;
        if (ext_factor != 0.0f) {
            const float yv = __fdiv_rn(__fsub_rn((float)j, corr0), fmaxf(0.001f, __fsub_rn(corr1, corr0)));
            const float ramp_mix = __fmul_rn(__fsub_rn(1.0f, fminf(1.0f, fmaxf(0.0f, yv))), ext_factor);
            th = __fadd_rn(__fmul_rn(theta_interp, __fsub_rn(1.0f, ramp_mix)), __fmul_rn(theta_extrap, ramp_mix));
            mscale = __fmul_rn(mscale, __fadd_rn(1.0f, __fmul_rn(0.1f, logf(__frcp_rn(freq_scale)))));
        }
        const float c = __fmul_rn(cosf(th), mscale), s = __fmul_rn(sinf(th), mscale);
        const int i0 = neox ? j : 2 * j, i1 = neox ? j + n_dims / 2 : 2 * j + 1;
        for (int h = 0; h < nh; h++) {
            const float *xp = x + t * xs2 + h * xs1;
            float *yp = y + t * ys2 + h * ys1;
            const float x0 = xp[i0], x1 = xp[i1];
            yp[i0] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
            yp[i1] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
        }
    }
}

struct Shape4 {
    long long ne[4], nb[4];
};

// ggml CPY / CONT / DUP between F32 and F16 tensors of up to four dimensions (ne, nb as ggml: nb in bytes); element e in
// row-major order of the source goes to element e of the destination.
__global__ void cpy_any_k(const uint8_t *__restrict__ src, int tin, Shape4 s, uint8_t *dst, int tout, Shape4 d,
                          long long n) {
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
        long long r = e, so = 0, dofs = 0;
        for (int i = 0; i < 4; i++) {
            so += (r % s.ne[i]) * s.nb[i];
            r /= s.ne[i];
        }
        r = e;
        for (int i = 0; i < 4; i++) {
            dofs += (r % d.ne[i]) * d.nb[i];
            r /= d.ne[i];
        }
        const float v = tin == GEN9BLAS_S ? *(const float *)(src + so) : __half2float(*(const __half *)(src + so));
        if (tout == GEN9BLAS_S) *(float *)(dst + dofs) = v;
        else *(__half *)(dst + dofs) = __float2half_rn(v);
    }
}

// ggml_rope_multi. MROPE (indep 0): NEOX pair order (j, j + n_dims/2), pair j takes the position of its sector
// j % (s0+s1+s2+s3) -- t for sector < s0, h below s0+s1, w below s0+s1+s2, e after (pos[t + c·n_tok] for c = 0..3) --
// with theta = p·theta_scale^j by repeated multiplication. VISION (indep 1): pairs (j, j + pairoff), pairoff = n_dims,
// and the running power restarts at each section start the way ggml_mrope_cache_init's else-if chain does (empty
// sections included). Each thread replays the four running thetas up to its pair, as the cache loop would.
__global__ void rope_multi_k(int npairs, int nh, int n_tok, const float *__restrict__ x, long long xs1, long long xs2, float *y,
                             long long ys1, long long ys2, const int *__restrict__ pos, const float *__restrict__ ff, int s0,
                             int s1, int s2, int s3, float theta_scale, float freq_scale, float ext_factor, float attn_factor,
                             float corr0, float corr1, int pairoff, int indep) {
    const long long n = (long long)npairs * n_tok;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
        const int j = (int)(e % npairs), t = (int)(e / npairs);
        const int sd = s0 + s1 + s2 + s3, sector = j % sd;
        const int sec = sector < s0 ? 0 : sector < s0 + s1 ? 1 : sector < s0 + s1 + s2 ? 2 : 3;
        const float p[4] = {(float)pos[t], (float)pos[t + n_tok], (float)pos[t + 2 * n_tok], (float)pos[t + 3 * n_tok]};
        float th4[4] = {p[0], p[1], p[2], p[3]};
        auto restart = [&](int sk) {
            if (sk == 0) th4[0] = p[0];
            else if (sk == s0) th4[1] = p[1];
            else if (sk == s0 + s1) th4[2] = p[2];
            else if (sk == s0 + s1 + s2) th4[3] = p[3];
        };
        for (int k = 0; k < j; k++) {
            if (indep) restart(k % sd);
            for (int c = 0; c < 4; c++) th4[c] = __fmul_rn(th4[c], theta_scale);
        }
        if (indep) restart(sector);
        const float theta = th4[sec];
        const float theta_extrap = ff ? __fdiv_rn(theta, ff[j]) : theta;
        const float theta_interp = __fmul_rn(freq_scale, theta_extrap);
        float th = theta_interp, mscale = attn_factor;
        if (ext_factor != 0.0f) {
            const float yv = __fdiv_rn(__fsub_rn((float)j, corr0), fmaxf(0.001f, __fsub_rn(corr1, corr0)));
            const float ramp_mix = __fmul_rn(__fsub_rn(1.0f, fminf(1.0f, fmaxf(0.0f, yv))), ext_factor);
            th = __fadd_rn(__fmul_rn(theta_interp, __fsub_rn(1.0f, ramp_mix)), __fmul_rn(theta_extrap, ramp_mix));
            mscale = __fmul_rn(mscale, __fadd_rn(1.0f, __fmul_rn(0.1f, logf(__frcp_rn(freq_scale)))));
        }
        const float c = __fmul_rn(cosf(th), mscale), sn = __fmul_rn(sinf(th), mscale);
        for (int h = 0; h < nh; h++) {
            const float *xp = x + t * xs2 + h * xs1;
            float *yp = y + t * ys2 + h * ys1;
            const float x0 = xp[j], x1 = xp[j + pairoff];
            yp[j] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
            yp[j + pairoff] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
        }
    }
}

// ggml UPSCALE / ggml_interpolate, F32, as ggml-cpu: mode 0 nearest (source index = floor(i / sf)), 1 bilinear with
// pixel offset po (0.5, or 0 with align corners) and clamped neighbours, 1 + antialias (triangle filter of support
// max(1, 1/sf), weights normalised). Byte strides; one thread per destination element.
__global__ void upscale_k(const uint8_t *__restrict__ src, Shape4 s, uint8_t *dst, Shape4 d, float sf0, float sf1, float sf2,
                          float sf3, int mode, int aa, float po, long long n) {
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
        long long r = e;
        const int i0 = (int)(r % d.ne[0]);
        r /= d.ne[0];
        const int i1 = (int)(r % d.ne[1]);
        r /= d.ne[1];
        const int i2 = (int)(r % d.ne[2]), i3 = (int)(r / d.ne[2]);
        // source plane and nearest indices, clamped to the source extent (the quotient can only reach it by rounding)
        const long long i02 = min((long long)(i2 / sf2), s.ne[2] - 1), i03 = min((long long)(i3 / sf3), s.ne[3] - 1);
        const uint8_t *s23 = src + i02 * s.nb[2] + i03 * s.nb[3];
        auto at = [&](long long x0, long long y0) { return *(const float *)(s23 + x0 * s.nb[0] + y0 * s.nb[1]); };
        float val;
        if (mode == 0) {
            val = at(min((long long)(i0 / sf0), s.ne[0] - 1), min((long long)(i1 / sf1), s.ne[1] - 1));
        } else if (aa) {
            const float support1 = fmaxf(1.0f, __frcp_rn(sf1)), invscale1 = __frcp_rn(support1);
            const float support0 = fmaxf(1.0f, __frcp_rn(sf0)), invscale0 = __frcp_rn(support0);
            const float yy = __fdiv_rn(__fadd_rn((float)i1, po), sf1), xx = __fdiv_rn(__fadd_rn((float)i0, po), sf0);
            const long long x_min = max((long long)__fadd_rn(__fsub_rn(xx, support0), po), 0LL);
            const long long x_max = min((long long)__fadd_rn(__fadd_rn(xx, support0), po), s.ne[0]);
            const long long y_min = max((long long)__fadd_rn(__fsub_rn(yy, support1), po), 0LL);
            const long long y_max = min((long long)__fadd_rn(__fadd_rn(yy, support1), po), s.ne[1]);
            float acc = 0.0f, tw = 0.0f;
            for (long long sy = y_min; sy < y_max; sy++) {
                const float wy = fmaxf(__fsub_rn(1.0f, fabsf(__fmul_rn(__fadd_rn(__fsub_rn((float)sy, yy), po), invscale1))), 0.0f);
                for (long long sx = x_min; sx < x_max; sx++) {
                    const float wx =
                        fmaxf(__fsub_rn(1.0f, fabsf(__fmul_rn(__fadd_rn(__fsub_rn((float)sx, xx), po), invscale0))), 0.0f);
                    const float w = __fmul_rn(wx, wy);
                    if (w <= 0.0f) continue;
                    acc = __fadd_rn(acc, __fmul_rn(at(sx, sy), w));
                    tw = __fadd_rn(tw, w);
                }
            }
            val = tw > 0.0f ? __fdiv_rn(acc, tw) : acc;
        } else {
            const float yy = __fsub_rn(__fdiv_rn(__fadd_rn((float)i1, po), sf1), po);
            const float xx = __fsub_rn(__fdiv_rn(__fadd_rn((float)i0, po), sf0), po);
            long long y0 = (long long)floorf(yy), x0 = (long long)floorf(xx), y1 = y0 + 1, x1 = x0 + 1;
            y0 = max(0LL, min(y0, s.ne[1] - 1));
            y1 = max(0LL, min(y1, s.ne[1] - 1));
            x0 = max(0LL, min(x0, s.ne[0] - 1));
            x1 = max(0LL, min(x1, s.ne[0] - 1));
            const float dy = fmaxf(0.0f, fminf(__fsub_rn(yy, (float)y0), 1.0f));
            const float dx = fmaxf(0.0f, fminf(__fsub_rn(xx, (float)x0), 1.0f));
            const float a = at(x0, y0), b = at(x1, y0), c = at(x0, y1), dd = at(x1, y1);
            const float ndx = __fsub_rn(1.0f, dx), ndy = __fsub_rn(1.0f, dy);
            val = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(__fmul_rn(a, ndx), ndy), __fmul_rn(__fmul_rn(b, dx), ndy)),
                                      __fmul_rn(__fmul_rn(c, ndx), dy)),
                            __fmul_rn(__fmul_rn(dd, dx), dy));
        }
        *(float *)(dst + i0 * d.nb[0] + i1 * d.nb[1] + i2 * d.nb[2] + i3 * d.nb[3]) = val;
    }
}

// ggml SET_ROWS, F32 rows into F16 rows: dst row idx[i] of plane (i02, i03) = src row i (RTE); indices broadcast over
// the planes as ggml-cpu (i11 = i02 % ne11, i12 = i03 % ne12); an index outside [0, ne1), or an index or destination
// position beyond the byte extents the caller gave, sets *bad and writes nothing.
__global__ void set_rows_k(int nc, int nr, int ne02, int ne03, const float *__restrict__ src, long long s1, long long s2,
                           long long s3, const uint8_t *__restrict__ idx, long long b10, long long b11, long long b12,
                           int idx64, int ne11, int ne12, long long idx_bytes, __half *dst, long long d1, long long d2,
                           long long d3, long long ne1, long long dst_elems, unsigned *bad) {
    const long long n = (long long)nc * nr * ne02 * ne03;
    bool oops = false;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
        const int c = (int)(e % nc);
        const long long rest = e / nc;
        const int i = (int)(rest % nr);
        const long long plane = rest / nr;
        const int i02 = (int)(plane % ne02), i03 = (int)(plane / ne02);
        const long long io = i * b10 + (i02 % ne11) * b11 + (i03 % ne12) * b12;
        if (io < 0 || io + (idx64 ? 8 : 4) > idx_bytes) {   // index strides beyond the index buffer: refused
            oops = true;
            continue;
        }
        const uint8_t *ip = idx + io;
        const long long row = idx64 ? *(const long long *)ip : (long long)*(const int *)ip;
        const long long o = row * d1 + i02 * d2 + i03 * d3 + c;
        if (row < 0 || row >= ne1 || o < 0 || o >= dst_elems) {
            oops = true;
            continue;
        }
        dst[o] = __float2half_rn(src[i * s1 + i02 * s2 + i03 * s3 + c]);
    }
    if (oops) *(volatile unsigned *)bad = 1u;
}

// ---------------------------------------------------------------------------------------------- attention
// Split-K decoding attention. Warp = (chunk, token, KV head, stream) x one query head; lane l holds dims 4l .. 4l + 3
// (D <= 128). Keys of the chunk in blocks of 32: scores (FP32 dot of the scaled query with the FP16 key row, reduced over
// the lanes), online softmax in base 2, values accumulated. Output per (chunk, head): running max m, sum l, D partial
// outputs; a chunk past the visible keys stores l = 0.
constexpr int ATT_CHUNK = 256;
struct AttnArgs {
    int D, H, HKV, ns, nq, nk, nchunk, dvis;
    const float *Q;
    long long qt, qh, qs;
    const __half *K;
    long long kk, kh, ks;
    const __half *V;
    long long vk, vh, vs;
    const int *vis;
    float qscale;
    float *part;
    float *O;
    // tensor-core kernel (stream-K over the 32-key steps of all rows r = (stream-token, KV head)): steps per row,
    // their total over the rows, the grid size, and the device error word a timed-out wait sets
    int nsr;
    long long total;
    int nblk;
    unsigned *err;
    unsigned *cnt;   // per-row arrival counters (zero before and after each launch)
    int early;       // no queued call writes K or V: the first copies may precede griddepcontrol.wait
};

__global__ void __launch_bounds__(256) attn_part_k(AttnArgs a) {
    const int lane = threadIdx.x & 31;
    const long long w = blockIdx.x * 8LL + (threadIdx.x >> 5);   // warp index: ((s · nq + t) · H + h) · nchunk + c
    const long long total = (long long)a.ns * a.nq * a.H * a.nchunk;
    if (w >= total) return;
    const int c = (int)(w % a.nchunk);
    const int h = (int)((w / a.nchunk) % a.H);
    const long long st = w / ((long long)a.nchunk * a.H);
    const int t = (int)(st % a.nq), s = (int)(st / a.nq);
    const int G = a.H / a.HKV, g = h / G;
    int vt = a.vis[s] + a.dvis * t;
    vt = vt < a.nk ? vt : a.nk;
    const int k0 = c * ATT_CHUNK, k1 = min(k0 + ATT_CHUNK, vt);
    float *pp = a.part + w * (2 + a.D);
    if (k0 >= k1) {
        if (lane == 0) {
            pp[0] = -INFINITY;
            pp[1] = 0.0f;
        }
        return;
    }
    const int d0 = 4 * lane;
    const bool live = d0 < a.D;
    float q[4] = {0, 0, 0, 0};
    const float *qp = a.Q + s * a.qs + t * a.qt + h * a.qh;
    for (int i = 0; i < 4; i++)
        if (live && d0 + i < a.D) q[i] = qp[d0 + i] * a.qscale;
    const __half *Kb = a.K + s * a.ks + g * a.kh, *Vb = a.V + s * a.vs + g * a.vh;
    float m = -INFINITY, l = 0.0f, acc[4] = {0, 0, 0, 0};
    for (int kb = k0; kb < k1; kb += 32) {
        const int nv = min(32, k1 - kb);
        float sc = -INFINITY;   // lane j: score of key kb + j
        for (int j = 0; j < nv; j++) {
            const __half *kr = Kb + (long long)(kb + j) * a.kk;
            float p = 0.0f;
            for (int i = 0; i < 4; i++)
                if (live && d0 + i < a.D) p = fmaf(__half2float(kr[d0 + i]), q[i], p);
            for (int o = 16; o > 0; o >>= 1) p += __shfl_xor_sync(0xffffffffu, p, o);
            if (lane == j) sc = p;
        }
        float mx = sc;
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const float mn = fmaxf(m, mx);
        const float alpha = exp2f(m - mn);
        const float p = lane < nv ? exp2f(sc - mn) : 0.0f;
        float ps = p;
        for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
        l = l * alpha + ps;
        for (int i = 0; i < 4; i++) acc[i] *= alpha;
        m = mn;
        for (int j = 0; j < nv; j++) {
            const float pj = __shfl_sync(0xffffffffu, p, j);
            const __half *vr = Vb + (long long)(kb + j) * a.vk;
            for (int i = 0; i < 4; i++)
                if (live && d0 + i < a.D) acc[i] = fmaf(pj, __half2float(vr[d0 + i]), acc[i]);
        }
    }
    if (lane == 0) {
        pp[0] = m;
        pp[1] = l;
    }
    for (int i = 0; i < 4; i++)
        if (live && d0 + i < a.D) pp[2 + d0 + i] = acc[i];
}

// CTA of the stream-K split (grid B over T steps) that holds step x: the last b with ⌊b·T / B⌋ <= x.
__host__ __device__ __forceinline__ long long at_blk_of(long long x, long long T, long long B) { return (x * B + B - 1) / T; }

// O[s][t][h][d] = Σ_c acc_c 2^(m_c − M) / Σ_c l_c 2^(m_c − M) over the chunks c with l > 0 (M their largest m), for
// the per-head kernel's [row][chunk] partials. One 128-thread CTA per output row (s, t, h): the threads reduce M over
// the chunks, then thread d walks them in chunk order (eight chunks' loads in flight) adding its dimension and,
// redundantly in every thread, the denominator. A chunk whose l is not positive is skipped by a select, so whatever
// its other words hold never enters the sums.
__global__ void __launch_bounds__(128) attn_merge_k(AttnArgs a) {
    __shared__ float red[4];
    const long long row = blockIdx.x;   // (s · nq + t) · H + h
    const int D = a.D, stride = 2 + D, d = threadIdx.x, nc = a.nchunk;
    const float *pb = a.part + row * nc * stride;
    const long long pstride = stride;
    float M = -INFINITY;
    for (int c = threadIdx.x; c < nc; c += 128)
        if (pb[c * pstride + 1] > 0.0f) M = fmaxf(M, pb[c * pstride]);
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = M;
    __syncthreads();
    M = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    const int dd = d < D ? d : 0;
    float L = 0.0f, acc = 0.0f;
#pragma unroll 8
    for (int c = 0; c < nc; c++) {
        const float *pc = pb + c * pstride;
        const float lc = pc[1], mc = pc[0], xc = pc[2 + dd];
        const bool use = lc > 0.0f;
        const float w = use ? exp2f(mc - M) : 0.0f;
        L = use ? fmaf(lc, w, L) : L;
        acc = use ? fmaf(xc, w, acc) : acc;
    }
    if (d < D) a.O[row * D + d] = acc / L;
}

// Decoding attention on the tensor cores (D % 16 == 0, D <= 128, G = H / HKV <= 8, 16-byte aligned K / V rows).
// Work: the 32-key steps of all rows r = (stream-token, KV head), ⌈nk / 32⌉ per row and T in all, split stream-K over a
// one-wave grid of B CTAs: CTA b takes steps [⌊bT/B⌋, ⌊(b+1)T/B⌋), a row segment at a time, its 4 warps taking every
// fourth step of the segment (steps past the visible keys are skipped) for all G query heads of the row's KV head (the
// 8 head slots of the MMA's N side), so every K / V row is read from memory once. Per step, with the 32 K rows and V
// rows in this warp's padded shared rows (one 1-D bulk copy per row, issued by the lane of that row and completing on
// the warp's K or V mbarrier; rows past the visible keys are zero-filled):
//   scores  Sᵀ[32 keys × 8 heads] = K · Qᵀ by mma.sync m16n8k16, K from the shared rows (ldmatrix) as A, the query as
//           B in two FP16 parts (hi = fp16(q), lo = fp16(q − hi)) after scaling each head's query by a power of two
//           that puts its largest |q| in [2^13, 2^14), so both parts stay normal and the products keep 22 of the
//           query's 24 bits; FP32 accumulation, the power of two divided out of every score exactly;
//   softmax running max per head over the lanes that hold the head, p = 2^(s − m) in FP32, per-lane partial sums;
//   values  Oᵀ[D × 8 heads] += Vᵀ · Pᵀ, V from the shared rows by ldmatrix.trans as A, P in two FP16 parts as B
//           (movmatrix turns the scores' accumulator layout into the B layout).
// The next step's K rows are requested once this step's are scored and its V rows once these are summed, so each copy
// overlaps the other half of the step. At the end of a segment the warps' (m, l, acc) are merged in shared memory
// into one partial per head slot, written to slot b + r (distinct for every (b, r) pair that shares a step).
constexpr int AT2_WARPS = 4, AT2_KEYS = 32, AT2_GMAX = 8;
constexpr uint64_t AT2_WAIT_NS = 2000000000ull;   // a 256-byte row copy that has not landed after 2 s is an error
__host__ __device__ constexpr int at2_rowb(int D) { return D * 2 + 16; }
__host__ __device__ constexpr size_t at2_stage(int D) { return (size_t)AT2_WARPS * 2 * AT2_KEYS * at2_rowb(D); }
__host__ __device__ constexpr size_t at2_smem(int D) { return at2_stage(D) + AT2_WARPS * 2 * sizeof(uint64_t); }

__device__ __forceinline__ void at_ldsm(unsigned addr, unsigned (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr) : "memory");
}
__device__ __forceinline__ void at_ldsm_t(unsigned addr, unsigned (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr) : "memory");
}
__device__ __forceinline__ unsigned at_movt(unsigned x) {
    unsigned y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(y) : "r"(x));
    return y;
}
__device__ __forceinline__ void at_mma(float (&c)[4], const unsigned (&a)[4], unsigned b0, unsigned b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// (x0, x1) as FP16 hi and lo parts: hi = fp16(x), lo = fp16(x − hi), element 0 in the low half of each word
__device__ __forceinline__ void at_split(float x0, float x1, unsigned &hi, unsigned &lo) {
    const __half2 h = __floats2half2_rn(x0, x1);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(x0 - hf.x, x1 - hf.y);
    hi = *reinterpret_cast<const unsigned *>(&h);
    lo = *reinterpret_cast<const unsigned *>(&l);
}
__device__ __forceinline__ float at_pow2(int e) { return __uint_as_float((unsigned)(e + 127) << 23); }   // |e| <= 126
// one contiguous row of `bytes` bytes (multiple of 16, both addresses 16-byte aligned) into shared memory, completing on
// the mbarrier; no multicast
__device__ __forceinline__ void at_bulk_row(void *dst, const void *src, unsigned bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                     sm100::smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(sm100::smem_u32(bar))
                 : "memory");
}

template <int DT>
__global__ void __launch_bounds__(AT2_WARPS * 32, 3) attn_tc_k(AttnArgs a) {
    using namespace sm100;
    constexpr int D = DT * 16, ROWB = at2_rowb(D);
    extern __shared__ __align__(16) uint8_t at_sm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gq = lane >> 2, tq = lane & 3;
    const int G = a.H / a.HKV;
    uint8_t *kst = at_sm + (size_t)warp * 2 * AT2_KEYS * ROWB;   // this warp's K rows, then its V rows
    uint8_t *vst = kst + AT2_KEYS * ROWB;
    uint64_t *kbar = reinterpret_cast<uint64_t *>(at_sm + at2_stage(D)) + 2 * warp, *vbar = kbar + 1;
    if (lane == 0) {
        mbar_init(kbar, 1);
        mbar_init(vbar, 1);
        fence_barrier_init();
    }
    __syncwarp();
    unsigned kph = 0, vph = 0;          // parity of the next phase of each barrier
    bool kpend = false, vpend = false;  // a phase with copies that have not been waited for
    bool ok = true;
    __shared__ int bad;
    __shared__ bool last;
    if (threadIdx.x == 0) bad = 0;
    const unsigned kbase = smem_u32(kst), vbase = smem_u32(vst);
    const unsigned koff = ((lane & 7) + ((lane >> 3) & 1) * 8) * ROWB + (lane >> 4) * 16;   // A = K rows
    const unsigned voff = ((lane & 7) + (lane >> 4) * 8) * ROWB + ((lane >> 3) & 1) * 16;   // A = Vᵀ (trans)
    const long long T = a.total, B = gridDim.x, b = blockIdx.x;
    const long long lo = b * T / B, hi = (b + 1) * T / B;
    // launched with programmatic stream serialization: the next kernel may start as this one's CTAs leave; this
    // kernel touches Q, the visible counts, the slots, the counters and O only after griddepcontrol.wait (the slots
    // and counters are shared with the previous call of this kernel), K and V before it only when a.early says so
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    bool waited = false;
    if (!a.early) {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        waited = true;
    }
    __syncthreads();
    for (long long r = lo / a.nsr; r * a.nsr < hi; r++) {
        const long long rs0 = r * a.nsr;
        const int g = (int)(r % a.HKV), st = (int)(r / a.HKV);
        const int t = st % a.nq, s = st / a.nq;
        const long long sb = max(lo, rs0) - rs0;   // this segment's steps in the row: [sb, sn), capped below at the
        const long long sn = min(hi, rs0 + a.nsr) - rs0;   // visible keys once their count is known
        const __half *Kb = a.K + s * a.ks + g * a.kh, *Vb = a.V + s * a.vs + g * a.vh;
        int vt = a.nk;   // rows past vt are zero-filled instead of copied; all nk rows exist in the caller's buffers
        // the 32 rows of this warp's i-th step of one tensor: lane j copies key row j, or zero-fills it past vt
        auto stage = [&](const __half *base, long long rs, uint8_t *dst, uint64_t *bar, int i) {
            const int k0 = (int)((sb + warp + (long long)AT2_WARPS * i) * AT2_KEYS);
            const int nrows = min(AT2_KEYS, vt - k0);
            fence_proxy_async();   // earlier zero-fill stores to these rows come before the copies
            if (lane == 0) mbar_arrive_expect_tx(bar, (unsigned)(nrows * D * 2));
            __syncwarp();
            if (lane < nrows) {
                at_bulk_row(dst + lane * ROWB, base + (long long)(k0 + lane) * rs, D * 2, bar);
            } else {
#pragma unroll
                for (int q = 0; q < D / 8; q++) *reinterpret_cast<uint4 *>(dst + lane * ROWB + q * 16) = make_uint4(0u, 0u, 0u, 0u);
            }
        };
        // the first step is requested before the visible count is read, bounded by nk: its K rows past the count are
        // masked in the scores and its V rows past it are zeroed once they land
        if (ok && sb + warp < sn) {
            stage(Kb, a.kk, kst, kbar, 0);
            stage(Vb, a.vk, vst, vbar, 0);
            kpend = vpend = true;
        }
        if (!waited) {
            asm volatile("griddepcontrol.wait;" ::: "memory");
            waited = true;
        }
        vt = max(min(a.vis[s] + a.dvis * t, a.nk), 0);
        const long long se = min(sn, (long long)((vt + AT2_KEYS - 1) / AT2_KEYS));
        const int nmy = se > sb + warp ? (int)((se - sb - warp + AT2_WARPS - 1) / AT2_WARPS) : 0;
        float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.0f, 0.0f};
        float o[DT][4];
#pragma unroll
        for (int dt = 0; dt < DT; dt++) o[dt][0] = o[dt][1] = o[dt][2] = o[dt][3] = 0.0f;
        if (nmy > 0 && ok) {
            // query fragments (B of the scores): lane holds head slot gq, dims 16kt + 2tq + {0, 1} and {8, 9}
            float qv[DT][4];
            float qmax = 0.0f;
            const bool hlive = gq < G;
            const float *qp = a.Q + s * a.qs + t * a.qt + (long long)(g * G + (hlive ? gq : 0)) * a.qh;
#pragma unroll
            for (int kt = 0; kt < DT; kt++)
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float x = hlive ? qp[16 * kt + 2 * tq + (i & 1) + (i >> 1) * 8] * a.qscale : 0.0f;
                    qv[kt][i] = x;
                    qmax = fmaxf(qmax, fabsf(x));
                }
            qmax = fmaxf(qmax, __shfl_xor_sync(0xffffffffu, qmax, 1));
            qmax = fmaxf(qmax, __shfl_xor_sync(0xffffffffu, qmax, 2));   // the four lanes of head slot gq
            int ex = 0;
            if (qmax > 0.0f) {
                const int be = (int)((__float_as_uint(qmax) >> 23) & 0xffu);   // qmax < 2^(be − 126)
                ex = min(max(140 - be, -126), 126);                              // qmax · 2^ex < 2^14
            }
            const float qsc = at_pow2(ex), qinv = at_pow2(-ex);
            unsigned qh[DT][2], ql[DT][2];
#pragma unroll
            for (int kt = 0; kt < DT; kt++)
#pragma unroll
                for (int j = 0; j < 2; j++) at_split(qv[kt][2 * j] * qsc, qv[kt][2 * j + 1] * qsc, qh[kt][j], ql[kt][j]);
            // this lane's score columns are head slots 2tq and 2tq + 1; their scale factors sit in lanes 8tq, 8tq + 4
            const float inv[2] = {__shfl_sync(0xffffffffu, qinv, 8 * tq), __shfl_sync(0xffffffffu, qinv, 8 * tq + 4)};
            for (int i = 0; i < nmy; i++) {
                const int r0 = (int)((sb + warp + (long long)AT2_WARPS * i) * AT2_KEYS);
                const bool more = i + 1 < nmy;
                if (!mbar_wait(kbar, kph, &bad, AT2_WAIT_NS)) {
                    ok = false;
                    break;
                }
                kph ^= 1u;
                kpend = false;
                float sc[2][4];
#pragma unroll
                for (int mt = 0; mt < 2; mt++) {
                    sc[mt][0] = sc[mt][1] = sc[mt][2] = sc[mt][3] = 0.0f;
#pragma unroll
                    for (int kt = 0; kt < DT; kt++) {
                        unsigned af[4];
                        at_ldsm(kbase + koff + mt * 16 * ROWB + kt * 32, af);
                        at_mma(sc[mt], af, qh[kt][0], qh[kt][1]);
                        at_mma(sc[mt], af, ql[kt][0], ql[kt][1]);
                    }
                }
                __syncwarp();   // every lane's K fragments are in registers before the next copy overwrites the rows
                if (more) {
                    stage(Kb, a.kk, kst, kbar, i + 1);
                    kpend = true;
                }
                // sc[mt][2·hh + j]: key r0 + 16mt + gq + 8hh, head slot 2tq + j
                float pr[2][4];
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    float x[4];
                    float mx = -INFINITY;
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const int mt = e >> 1, hh = e & 1;
                        x[e] = r0 + 16 * mt + gq + 8 * hh < vt ? sc[mt][2 * hh + j] * inv[j] : -INFINITY;
                        mx = fmaxf(mx, x[e]);
                    }
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                    const float mn = fmaxf(m[j], mx);
                    const float alpha = exp2f(m[j] - mn);   // 0 on the first step (m = -inf)
                    float ps = 0.0f;
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const float p = exp2f(x[e] - mn);
                        pr[e >> 1][2 * (e & 1) + j] = p;
                        ps += p;
                    }
                    l[j] = fmaf(l[j], alpha, ps);
#pragma unroll
                    for (int dt = 0; dt < DT; dt++) {
                        o[dt][j] *= alpha;
                        o[dt][2 + j] *= alpha;
                    }
                    m[j] = mn;
                }
                if (!mbar_wait(vbar, vph, &bad, AT2_WAIT_NS)) {
                    ok = false;
                    break;
                }
                vph ^= 1u;
                vpend = false;
                if (i == 0 && r0 + lane >= vt) {   // first step: V rows past the visible keys were copied (rows < nk)
#pragma unroll
                    for (int q = 0; q < D / 8; q++) *reinterpret_cast<uint4 *>(vst + lane * ROWB + q * 16) = make_uint4(0u, 0u, 0u, 0u);
                }
                __syncwarp();
#pragma unroll
                for (int ks = 0; ks < 2; ks++) {
                    unsigned h01, l01, h23, l23;
                    at_split(pr[ks][0], pr[ks][1], h01, l01);   // key 16ks + gq, head slots 2tq, 2tq + 1
                    at_split(pr[ks][2], pr[ks][3], h23, l23);   // key 16ks + gq + 8
                    const unsigned bh0 = at_movt(h01), bh1 = at_movt(h23), bl0 = at_movt(l01), bl1 = at_movt(l23);
#pragma unroll
                    for (int dt = 0; dt < DT; dt++) {
                        unsigned af[4];
                        at_ldsm_t(vbase + voff + ks * 16 * ROWB + dt * 32, af);
                        at_mma(o[dt], af, bh0, bh1);
                        at_mma(o[dt], af, bl0, bl1);
                    }
                }
                __syncwarp();   // every lane's V fragments are in registers before the next copy overwrites the rows
                if (more) {
                    stage(Vb, a.vk, vst, vbar, i + 1);
                    vpend = true;
                }
            }
        }
        if (!ok && lane == 0) *(volatile unsigned *)a.err = kDevErrWaitTimeout;
        // copies still in flight: a first step past the visible keys, or a wait that gave up (bounded again)
        if (kpend) {
            if (mbar_wait(kbar, kph, &bad, AT2_WAIT_NS)) kph ^= 1u;
            else if (lane == 0) *(volatile unsigned *)a.err = kDevErrWaitTimeout;
        }
        if (vpend) {
            if (mbar_wait(vbar, vph, &bad, AT2_WAIT_NS)) vph ^= 1u;
            else if (lane == 0) *(volatile unsigned *)a.err = kDevErrWaitTimeout;
        }
        kpend = vpend = false;
#pragma unroll
        for (int j = 0; j < 2; j++) {   // the per-lane sums over the 8 lanes of each head slot
            l[j] += __shfl_xor_sync(0xffffffffu, l[j], 4);
            l[j] += __shfl_xor_sync(0xffffffffu, l[j], 8);
            l[j] += __shfl_xor_sync(0xffffffffu, l[j], 16);
        }
        // merge the four warps: (m, l) per warp and head slot, acc per warp, head slot and dimension
        __syncthreads();   // every warp is done with its staging rows
        float *mw = reinterpret_cast<float *>(at_sm);   // [warp][slot]: m, then l
        float *lw = mw + AT2_WARPS * AT2_GMAX;
        float *aw = lw + AT2_WARPS * AT2_GMAX;         // [warp][slot][D]
#pragma unroll
        for (int j = 0; j < 2; j++) {
            const int hs = 2 * tq + j;
            if (hs >= G) continue;
            if (gq == 0) {
                mw[warp * AT2_GMAX + hs] = m[j];
                lw[warp * AT2_GMAX + hs] = l[j];
            }
            float *ap = aw + (warp * AT2_GMAX + hs) * D + gq;
#pragma unroll
            for (int dt = 0; dt < DT; dt++) {
                ap[16 * dt] = o[dt][j];
                ap[16 * dt + 8] = o[dt][2 + j];
            }
        }
        __syncthreads();
        float *pslot = a.part + (b + r) * G * (2 + D);
        for (int i = threadIdx.x; i < G * D; i += AT2_WARPS * 32) {
            const int h = i / D, d = i - h * D;
            float M = -INFINITY;
            for (int w = 0; w < AT2_WARPS; w++)
                if (lw[w * AT2_GMAX + h] > 0.0f) M = fmaxf(M, mw[w * AT2_GMAX + h]);
            float L = 0.0f, acc = 0.0f;
            if (M > -INFINITY) {
                for (int w = 0; w < AT2_WARPS; w++) {
                    if (!(lw[w * AT2_GMAX + h] > 0.0f)) continue;
                    const float f = exp2f(mw[w * AT2_GMAX + h] - M);
                    L += lw[w * AT2_GMAX + h] * f;
                    acc += aw[(w * AT2_GMAX + h) * D + d] * f;
                }
            }
            float *pp = pslot + h * (2 + D);
            pp[2 + d] = acc;
            if (d == 0) {
                pp[0] = M;
                pp[1] = L;
            }
        }
        // arrival on the row's counter; the CTA that completes the row merges its slots b0 + r .. b1 + r into O
        __syncthreads();   // every slot word is written (and the merge area read) before the arrival
        const long long b0 = at_blk_of(rs0, T, B), b1 = at_blk_of(rs0 + a.nsr - 1, T, B);
        const int nsl = (int)(b1 - b0 + 1);
        if (threadIdx.x == 0) {
            __threadfence();   // release of the CTA's slot words (ordered before by the barrier)
            last = atomicAdd(a.cnt + r, 1u) + 1u == (unsigned)nsl;
            __threadfence();   // acquire of the other CTAs' slot words
        }
        __syncthreads();
        if (last) {
            // thread i's outputs: (head slot, dim) = i + 128k for k < AT2_GMAX·D / 128 while below G·D; the values of
            // the first four slots are requested before the weights are known, so the loads overlap
            constexpr int NO = AT2_GMAX * D / (AT2_WARPS * 32), NJ = 4;
            const float *pb = a.part + (b0 + r) * G * (2 + D);   // [slot][head slot][2 + D], slots in key order
            float *wm = reinterpret_cast<float *>(at_sm);         // [slot][head slot]: 2^(m − M), −1 when l <= 0
            float *hl = wm + nsl * G;                             // [head slot]: the denominator
            float xv[NJ][NO];
#pragma unroll
            for (int jj = 0; jj < NJ; jj++)
#pragma unroll
                for (int k = 0; k < NO; k++) {
                    const int i = threadIdx.x + AT2_WARPS * 32 * k, h = i / D, d = i - h * D;
                    xv[jj][k] = jj < nsl && i < G * D ? __ldcg(pb + ((long long)jj * G + h) * (2 + D) + 2 + d) : 0.0f;
                }
            for (int h = warp; h < G; h += AT2_WARPS) {   // warp: the weights and denominator of head slots h
                float M = -INFINITY, L = 0.0f;
                for (int j0 = 0; j0 < nsl; j0 += 32) {
                    const int j = j0 + lane;
                    float mj = -INFINITY, lj = 0.0f;
                    if (j < nsl) {
                        const float *pp = pb + ((long long)j * G + h) * (2 + D);
                        mj = __ldcg(pp);
                        lj = __ldcg(pp + 1);
                    }
                    float mx = lj > 0.0f ? mj : -INFINITY;
                    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                    const float Mn = fmaxf(M, mx);
                    const float w = lj > 0.0f ? exp2f(mj - Mn) : -1.0f;
                    if (j < nsl) wm[j * G + h] = w;
                    float ls = lj > 0.0f ? lj * w : 0.0f;
                    for (int o = 16; o > 0; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
                    // slots of earlier passes were weighted against M: rescale them to Mn (rows of > 32 slots only)
                    __syncwarp();   // this pass's weights are in shared memory for every lane
                    if (j0 > 0 && Mn > M) {
                        const float f = exp2f(M - Mn);
                        for (int q = lane; q < j0; q += 32)
                            if (wm[q * G + h] >= 0.0f) wm[q * G + h] *= f;
                        L *= f;
                    }
                    L += ls;
                    M = Mn;
                    __syncwarp();
                }
                if (lane == 0) hl[h] = L;
            }
            __syncthreads();
            float acc[NO];
#pragma unroll
            for (int k = 0; k < NO; k++) acc[k] = 0.0f;
            for (int j0 = 0; j0 < nsl; j0 += NJ) {
#pragma unroll
                for (int jj = 0; jj < NJ; jj++)
#pragma unroll
                    for (int k = 0; k < NO; k++) {
                        const int i = threadIdx.x + AT2_WARPS * 32 * k, h = i / D;
                        if (j0 + jj < nsl && i < G * D) {
                            const float w = wm[(j0 + jj) * G + h];
                            acc[k] = w >= 0.0f ? fmaf(xv[jj][k], w, acc[k]) : acc[k];
                        }
                    }
                if (j0 + NJ < nsl) {   // the next four slots' values
#pragma unroll
                    for (int jj = 0; jj < NJ; jj++)
#pragma unroll
                        for (int k = 0; k < NO; k++) {
                            const int i = threadIdx.x + AT2_WARPS * 32 * k, h = i / D, d = i - h * D;
                            const int j = j0 + NJ + jj;
                            xv[jj][k] = j < nsl && i < G * D ? __ldcg(pb + ((long long)j * G + h) * (2 + D) + 2 + d) : 0.0f;
                        }
                }
            }
#pragma unroll
            for (int k = 0; k < NO; k++) {
                const int i = threadIdx.x + AT2_WARPS * 32 * k, h = i / D, d = i - h * D;
                if (i < G * D) a.O[((long long)st * a.H + g * G + h) * D + d] = acc[k] / hl[h];
            }
            if (threadIdx.x == 0) a.cnt[r] = 0u;   // the next call finds the counter at zero
        }
        __syncthreads();   // the merge area is read before the next segment's copies land in the staging rows
    }
}

// Launch of the tensor-core kernel for D = 16·DT; `plan` only reports its resident CTAs per SM (occupancy query once
// per device) and launches nothing.
template <int DT>
int attn_tc_run(const AttnArgs &a, cudaStream_t st, bool plan, int *per_sm) {
    static bool attr[kMaxDevices] = {};
    static int occ[kMaxDevices] = {};
    G9_CU(smem_limit_once(attn_tc_k<DT>, (int)at2_smem(DT * 16), attr));
    DevState *d = dev_state();
    if (plan) {
        if (!occ[d->dev])
            G9_CU(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ[d->dev], attn_tc_k<DT>, AT2_WARPS * 32,
                                                                at2_smem(DT * 16)));
        *per_sm = std::max(occ[d->dev], 1);
        return 0;
    }
    G9_CU(launch_pdl(attn_tc_k<DT>, dim3((unsigned)a.nblk), dim3(AT2_WARPS * 32), at2_smem(DT * 16), st, a));
    return launched("attn_tc");
}

int attn_tc(const AttnArgs &a, cudaStream_t st, bool plan, int *per_sm) {
    switch (a.D / 16) {
    case 1: return attn_tc_run<1>(a, st, plan, per_sm);
    case 2: return attn_tc_run<2>(a, st, plan, per_sm);
    case 3: return attn_tc_run<3>(a, st, plan, per_sm);
    case 4: return attn_tc_run<4>(a, st, plan, per_sm);
    case 5: return attn_tc_run<5>(a, st, plan, per_sm);
    case 6: return attn_tc_run<6>(a, st, plan, per_sm);
    case 7: return attn_tc_run<7>(a, st, plan, per_sm);
    default: return attn_tc_run<8>(a, st, plan, per_sm);
    }
}

bool attn_shape_ok(int D, int H, int HKV) { return D >= 1 && D <= 128 && HKV >= 1 && H >= HKV && H % HKV == 0; }

// Shared host flow of the three attention entry points (device or managed memory for Q, K, V, O and vis).
int attention(AttnArgs a, int sync, const char *who) {
    if (!attn_shape_ok(a.D, a.H, a.HKV)) return GEN9BLAS_DECLINED;
    if (a.ns <= 0 || a.nq <= 0 || a.nk <= 0) return 0;
    DevState *d = dev_state();
    if (!d) return G.status;
    if (!on_device(a.Q) || !on_device(a.K) || !on_device(a.V) || !on_device(a.O))
        return fail(GEN9BLAS_ERR_INVALID_ARG, "%s: Q, K, V and O must be device or managed memory", who);
    // the tensor-core kernel when D is a multiple of 16, rows are 16-byte vectors and a KV head serves at most 8
    // query heads; otherwise the per-head CUDA-core kernel
    const bool tc = a.D % 16 == 0 && a.H / a.HKV <= AT2_GMAX && a.ns * a.nq <= 65535 && a.HKV <= 65535 &&
                    ((uintptr_t)a.K & 15) == 0 && ((uintptr_t)a.V & 15) == 0 && (a.kk * 2) % 16 == 0 &&
                    (a.kh * 2) % 16 == 0 && (a.ks * 2) % 16 == 0 && (a.vk * 2) % 16 == 0 && (a.vh * 2) % 16 == 0 &&
                    (a.vs * 2) % 16 == 0;
    cudaStream_t st = stream();
    size_t part_bytes;
    if (tc) {
        // stream-K over all rows' 32-key steps on one wave of CTAs (never more CTAs than steps, so every CTA's
        // range is non-empty and every slot b + r the merge reads is written)
        int per_sm = 1;
        G9_TRY(attn_tc(a, st, true, &per_sm));
        const long long rows = (long long)a.HKV * a.ns * a.nq;
        a.nsr = (a.nk + AT2_KEYS - 1) / AT2_KEYS;
        a.total = rows * a.nsr;
        // the merging CTA keeps one weight per (slot, head slot) of a row in the staging area
        const long long fit = (long long)(at2_stage(a.D) / sizeof(float)) / (a.H / a.HKV) - 2;
        a.nblk = (int)std::min(std::min<long long>((long long)per_sm * d->sm_count, a.total), fit);
        a.err = d->err_dev;
        G9_TRY(arrival_counters((size_t)rows, &a.cnt));
        // bytes of K and V the kernel may read: every (stream, KV head, key) row of D elements
        const size_t kext = ((size_t)(a.ns - 1) * a.ks + (size_t)(a.HKV - 1) * a.kh + (size_t)(a.nk - 1) * a.kk + a.D) * 2;
        const size_t vext = ((size_t)(a.ns - 1) * a.vs + (size_t)(a.HKV - 1) * a.vh + (size_t)(a.nk - 1) * a.vk + a.D) * 2;
        a.early = !queued_writes_overlap(d, a.K, kext) && !queued_writes_overlap(d, a.V, vext);
        part_bytes = round256((size_t)(a.nblk + rows) * (a.H / a.HKV) * (2 + a.D) * sizeof(float));
    } else {
        a.nchunk = (a.nk + ATT_CHUNK - 1) / ATT_CHUNK;
        part_bytes = round256((size_t)a.ns * a.nq * a.H * a.nchunk * (2 + a.D) * sizeof(float));
    }
    void *buf = nullptr;
    G9_TRY(ml_buffer(part_bytes + (size_t)a.ns * sizeof(int), &buf));
    a.part = (float *)buf;
    if (!on_device(a.vis)) {   // the visible counts (ns ints) behind the partial results
        int *vd = (int *)((char *)buf + part_bytes);
        G9_CU(cudaMemcpyAsync(vd, a.vis, (size_t)a.ns * sizeof(int), cudaMemcpyHostToDevice, st));
        a.vis = vd;
    }
    if (tc) {
        G9_TRY(attn_tc(a, st, false, nullptr));
    } else {
        attn_part_k<<<(unsigned)(((long long)a.ns * a.nq * a.H * a.nchunk + 7) / 8), 256, 0, st>>>(a);
        G9_TRY(launched("attn_part"));
    }
    if (!tc) {
        attn_merge_k<<<(unsigned)((long long)a.ns * a.nq * a.H), 128, 0, st>>>(a);
        G9_TRY(launched("attn_merge"));
    }
    Operand out;
    out.user = out.dptr = a.O;
    out.bytes = (size_t)a.ns * a.nq * a.H * a.D * sizeof(float);
    out.zc = true;
    out.written = true;
    const bool saved = G.nowait;
    G.nowait = !sync;
    int r = finish_op(&out, 1);
    G.nowait = saved;
    return r;
}

}  // namespace

extern "C" {

GEN9BLAS_API int gen9blas_span(const void *p, size_t bytes, int writes) {
    (void)p;
    (void)bytes;
    (void)writes;
    return 0;   // host operands are staged and complete before each call returns: every region counts as registered
}
GEN9BLAS_API void gen9blas_span_clear(void) {}

GEN9BLAS_API int gen9blas_rms_norm(int M, int K, const float *X, int ldx, const float *w, float eps, float *Y, int ldy,
                                   int sync) {
    if (int e = begin_op()) return e;
    if (M <= 0 || K <= 0) return 0;
    if (ldx < K || ldy < K) return fail(GEN9BLAS_ERR_INVALID_ARG, "rms_norm: ldx = %d, ldy = %d < K = %d", ldx, ldy, K);
    DevState *d = dev_state();
    if (!d) return G.status;
    OpCall c;
    void *x, *y;
    const void *wd;
    cudaStream_t st = stream();
    G9_TRY(c.big(X, ((size_t)(M - 1) * ldx + K) * 4, true, false, &x));
    G9_TRY(c.big(Y, ((size_t)(M - 1) * ldy + K) * 4, X == Y || ldy != K, true, &y));
    G9_TRY(c.reserve(w ? round256((size_t)K * 4) : 0));
    G9_TRY(c.in(w, (size_t)K * 4, &wd, st));
    if (K % 4 == 0 && ldx % 4 == 0 && ldy % 4 == 0 && on16(x) && on16(y) && (!wd || on16(wd)))
        rms_norm_v4_k<<<M, 256, 0, st>>>((const float *)x, ldx, (const float *)wd, eps, (float *)y, ldy, K);
    else
        rms_norm_k<<<M, 256, 0, st>>>((const float *)x, ldx, (const float *)wd, eps, (float *)y, ldy, K);
    G9_TRY(launched("rms_norm"));
    return c.finish(sync);
}

GEN9BLAS_API int gen9blas_layer_norm(int M, int K, const float *X, int ldx, const float *w, const float *b, float eps,
                                     float *Y, int ldy, int sync) {
    if (int e = begin_op()) return e;
    if (M <= 0 || K <= 0) return 0;
    if (ldx < K || ldy < K) return fail(GEN9BLAS_ERR_INVALID_ARG, "layer_norm: ldx = %d, ldy = %d < K = %d", ldx, ldy, K);
    DevState *d = dev_state();
    if (!d) return G.status;
    OpCall c;
    void *x, *y;
    const void *wd, *bd;
    cudaStream_t st = stream();
    G9_TRY(c.big(X, ((size_t)(M - 1) * ldx + K) * 4, true, false, &x));
    G9_TRY(c.big(Y, ((size_t)(M - 1) * ldy + K) * 4, X == Y || ldy != K, true, &y));
    G9_TRY(c.reserve(2 * round256((size_t)K * 4)));
    G9_TRY(c.in(w, (size_t)K * 4, &wd, st));
    G9_TRY(c.in(b, (size_t)K * 4, &bd, st));
    if (K % 4 == 0 && ldx % 4 == 0 && ldy % 4 == 0 && on16(x) && on16(y) && (!wd || on16(wd)) &&
        (!bd || on16(bd)))
        layer_norm_v4_k<<<M, 256, 0, st>>>((const float *)x, ldx, (const float *)wd, (const float *)bd, eps, (float *)y,
                                           ldy, K);
    else
        layer_norm_k<<<M, 256, 0, st>>>((const float *)x, ldx, (const float *)wd, (const float *)bd, eps, (float *)y, ldy,
                                        K, nullptr, 0);
    G9_TRY(launched("layer_norm"));
    return c.finish(sync);
}

GEN9BLAS_API int gen9blas_binop_rows(int op, int M, int K, const float *A, int lda, const float *B, int ldb, int bs0,
                                     float *C, int ldc, int sync) {
    if (int e = begin_op()) return e;
    if (M <= 0 || K <= 0) return 0;
    if ((op != 0 && op != 1) || (bs0 != 0 && bs0 != 1) || lda < K || ldc < K || ldb < 0)
        return fail(GEN9BLAS_ERR_INVALID_ARG, "binop_rows: op %d, bs0 %d, lda %d, ldb %d, ldc %d", op, bs0, lda, ldb, ldc);
    DevState *d = dev_state();
    if (!d) return G.status;
    OpCall c;
    void *a, *b, *cc;
    cudaStream_t st = stream();
    const size_t bb = ((size_t)(M - 1) * ldb + (bs0 ? (size_t)K : 1)) * 4;
    G9_TRY(c.big(A, ((size_t)(M - 1) * lda + K) * 4, true, false, &a));
    G9_TRY(c.big(B, bb, true, false, &b));
    G9_TRY(c.big(C, ((size_t)(M - 1) * ldc + K) * 4, C == A || C == B || ldc != K, true, &cc));
    binop_k<<<grid_n((long long)M * K, d->sm_count), 256, 0, st>>>(op, M, K, (const float *)a, lda, (const float *)b, ldb,
                                                                   bs0, (float *)cc, ldc);
    G9_TRY(launched("binop_rows"));
    return c.finish(sync);
}

static int unary(int op, size_t n, const float *X, float *Y, int sync) {
    if (int e = begin_op()) return e;
    if (n == 0) return 0;
    DevState *d = dev_state();
    if (!d) return G.status;
    OpCall c;
    void *x, *y;
    cudaStream_t st = stream();
    G9_TRY(c.big(X, n * 4, true, false, &x));
    if (Y == X) {
        y = x;
        c.ops[0].written = true;
    } else {
        G9_TRY(c.big(Y, n * 4, false, true, &y));
    }
    if (((uintptr_t)x & 15) == 0 && ((uintptr_t)y & 15) == 0) {
        // the table kernel copies 128 KB into every SM first: worth it from a few million elements on (a decode-sized
        // call computes instead; both give the same bits)
        if (op == 0 && n < ((size_t)1 << 22)) {
            unary_v_k<3><<<grid_n((long long)(n + 3) / 4, d->sm_count), 256, 0, st>>>((long long)n, (const float *)x,
                                                                                      (float *)y);
        } else if (op == 0) {
            static bool tab[kMaxDevices] = {}, attr[kMaxDevices] = {};
            if (!tab[d->dev]) {
                gelu_tab_k<<<64, 1024, 0, st>>>();
                G9_TRY(launched("gelu_tab"));
                tab[d->dev] = true;
            }
            G9_CU(smem_limit_once(unary_v_k<0>, 65536 * 2, attr));
            unary_v_k<0><<<d->sm_count, 1024, 65536 * 2, st>>>((long long)n, (const float *)x, (float *)y);
        } else if (op == 1) {
            unary_v_k<1><<<2 * d->sm_count, 512, 0, st>>>((long long)n, (const float *)x, (float *)y);
        } else {
            unary_v_k<2><<<4 * d->sm_count, 512, 0, st>>>((long long)n, (const float *)x, (float *)y);
        }
    } else {
        unary_k<<<grid_n((long long)n, d->sm_count), 256, 0, st>>>(op, (long long)n, (const float *)x, (float *)y);
    }
    G9_TRY(launched("unary"));
    return c.finish(sync);
}
GEN9BLAS_API int gen9blas_gelu(size_t n, const float *X, float *Y, int sync) { return unary(0, n, X, Y, sync); }
GEN9BLAS_API int gen9blas_gelu_erf(size_t n, const float *X, float *Y, int sync) { return unary(1, n, X, Y, sync); }
GEN9BLAS_API int gen9blas_relu(size_t n, const float *X, float *Y, int sync) { return unary(2, n, X, Y, sync); }

GEN9BLAS_API int gen9blas_cvt_f16_heads(int rows, int H, int D, const float *X, int64_t s_row, int64_t s_head, uint16_t *Y,
                                        int sync) {
    if (int e = begin_op()) return e;
    if (rows <= 0 || H <= 0 || D <= 0) return 0;
    if (s_row < 0 || s_head < 0) return fail(GEN9BLAS_ERR_INVALID_ARG, "cvt_f16_heads: negative strides");
    DevState *d = dev_state();
    if (!d) return G.status;
    OpCall c;
    void *x, *y;
    cudaStream_t st = stream();
    const size_t span = ((size_t)(rows - 1) * s_row + (size_t)(H - 1) * s_head + D) * 4;
    G9_TRY(c.big(X, span, true, false, &x));
    G9_TRY(c.big(Y, (size_t)rows * H * D * 2, false, true, &y));
    cvt_heads_k<<<grid_n((long long)rows * H * D, d->sm_count), 256, 0, st>>>(rows, H, D, (const float *)x, s_row, s_head,
                                                                              (__half *)y);
    G9_TRY(launched("cvt_f16_heads"));
    return c.finish(sync);
}

GEN9BLAS_API int gen9blas_im2col(int N, int IC, int IH, int IW, const float *X, int64_t ofs0, int64_t ofs1, int KH, int KW,
                                 int OH, int OW, int s0, int s1, int p0, int p1, int d0, int d1, void *Y, int f16, int sync) {
    if (int e = begin_op()) return e;
    if (N <= 0 || IC <= 0 || OH <= 0 || OW <= 0 || KH <= 0 || KW <= 0) return 0;
    if (IH <= 0 || IW <= 0 || ofs0 < 0 || ofs1 < 0) return fail(GEN9BLAS_ERR_INVALID_ARG, "im2col: bad input geometry");
    DevState *d = dev_state();
    if (!d) return G.status;
    OpCall c;
    void *x, *y;
    cudaStream_t st = stream();
    const size_t xspan = ((size_t)(N - 1) * ofs0 + (size_t)(IC - 1) * ofs1 + (size_t)IH * IW) * 4;
    const long long ny = (long long)N * OH * OW * IC * KH * KW;
    G9_TRY(c.big(X, xspan, true, false, &x));
    G9_TRY(c.big(Y, (size_t)ny * (f16 ? 2 : 4), false, true, &y));
    im2col_k<<<grid_n(ny, d->sm_count), 256, 0, st>>>(N, IC, IH, IW, (const float *)x, ofs0, ofs1, KH, KW, OH, OW, s0, s1, p0,
                                                      p1, d0, d1, y, f16 ? 1 : 0);
    G9_TRY(launched("im2col"));
    return c.finish(sync);
}

GEN9BLAS_API int gen9blas_rope(int n_dims, int nh, int n_tok, const float *X, int64_t xs1, int64_t xs2, float *Y, int64_t ys1,
                               int64_t ys2, const int *pos, const float *ff, int neox, float freq_base, float freq_scale,
                               float ext_factor, float attn_factor, const float corr[2], int sync) {
    if (int e = begin_op()) return e;
    if (n_dims <= 0 || nh <= 0 || n_tok <= 0) return 0;
    if (!pos || !corr) return fail(GEN9BLAS_ERR_INVALID_ARG, "rope: missing pos / corr");
    if (n_dims % 2 || xs1 < n_dims || ys1 < n_dims || xs2 < (int64_t)nh * xs1 - (xs1 - n_dims) ||
        ys2 < (int64_t)nh * ys1 - (ys1 - n_dims))
        return fail(GEN9BLAS_ERR_UNSUPPORTED, "rope: unsupported layout");
    DevState *d = dev_state();
    if (!d) return G.status;
    OpCall c;
    void *x, *y;
    const void *pd, *fd;
    cudaStream_t st = stream();
    const size_t xspan = ((size_t)(n_tok - 1) * xs2 + (size_t)(nh - 1) * xs1 + n_dims) * 4;
    const size_t yspan = ((size_t)(n_tok - 1) * ys2 + (size_t)(nh - 1) * ys1 + n_dims) * 4;
    G9_TRY(c.big(X, xspan, true, false, &x));
    if (Y == X && ys1 == xs1 && ys2 == xs2) {
        y = x;
        c.ops[0].written = true;
    } else {
        G9_TRY(c.big(Y, yspan, true, true, &y));   // copied in: the elements between rotated rows stay
    }
    G9_TRY(c.reserve(round256((size_t)n_tok * 4) + round256((size_t)n_dims / 2 * 4)));
    G9_TRY(c.in(pos, (size_t)n_tok * 4, &pd, st));
    G9_TRY(c.in(ff, (size_t)n_dims / 2 * 4, &fd, st));
    const float theta_scale = powf(freq_base, -2.0f / (float)n_dims);
    rope_k<<<grid_n((long long)n_dims / 2 * n_tok, d->sm_count), 256, 0, st>>>(
        n_dims, nh, n_tok, (const float *)x, xs1, xs2, (float *)y, ys1, ys2, (const int *)pd, (const float *)fd, neox ? 1 : 0,
        theta_scale, freq_scale, ext_factor, attn_factor, corr[0], corr[1]);
    G9_TRY(launched("rope"));
    return c.finish(sync);
}

GEN9BLAS_API int gen9blas_rope_multi(int n_dims, int nh, int n_tok, const float *X, int64_t xs1, int64_t xs2, float *Y,
                                     int64_t ys1, int64_t ys2, const int *pos, const float *ff, const int sections[4],
                                     float freq_base, float freq_scale, float ext_factor, float attn_factor,
                                     const float corr[2], int vision, int sync) {
    if (int e = begin_op()) return e;
    if (n_dims <= 0 || nh <= 0 || n_tok <= 0) return 0;
    if (!pos || !corr || !sections) return fail(GEN9BLAS_ERR_INVALID_ARG, "rope_multi: missing pos / corr / sections");
    const int ne0 = vision ? 2 * n_dims : n_dims;   // rotated elements per head row (vision: all of ne0 = 2·n_dims)
    if (n_dims % 2 || xs1 < ne0 || ys1 < ne0 || xs2 < (int64_t)nh * xs1 - (xs1 - ne0) || ys2 < (int64_t)nh * ys1 - (ys1 - ne0))
        return fail(GEN9BLAS_ERR_UNSUPPORTED, "rope_multi: unsupported layout");
    if (sections[0] + sections[1] + sections[2] + sections[3] <= 0)
        return fail(GEN9BLAS_ERR_INVALID_ARG, "rope_multi: empty sections");
    DevState *d = dev_state();
    if (!d) return G.status;
    const int npairs = vision ? n_dims : n_dims / 2;
    OpCall c;
    void *x, *y;
    const void *pd, *fd;
    cudaStream_t st = stream();
    const size_t xspan = ((size_t)(n_tok - 1) * xs2 + (size_t)(nh - 1) * xs1 + ne0) * 4;
    const size_t yspan = ((size_t)(n_tok - 1) * ys2 + (size_t)(nh - 1) * ys1 + ne0) * 4;
    G9_TRY(c.big(X, xspan, true, false, &x));
    if (Y == X && ys1 == xs1 && ys2 == xs2) {
        y = x;
        c.ops[0].written = true;
    } else {
        G9_TRY(c.big(Y, yspan, true, true, &y));
    }
    G9_TRY(c.reserve(round256((size_t)n_tok * 16) + round256((size_t)npairs * 4)));
    G9_TRY(c.in(pos, (size_t)n_tok * 16, &pd, st));
    G9_TRY(c.in(ff, (size_t)npairs * 4, &fd, st));
    const float theta_scale = powf(freq_base, -2.0f / (float)n_dims);
    rope_multi_k<<<grid_n((long long)npairs * n_tok, d->sm_count), 256, 0, st>>>(
        npairs, nh, n_tok, (const float *)x, xs1, xs2, (float *)y, ys1, ys2, (const int *)pd, (const float *)fd, sections[0],
        sections[1], sections[2], sections[3], theta_scale, freq_scale, ext_factor, attn_factor, corr[0], corr[1], npairs,
        vision ? 1 : 0);
    G9_TRY(launched("rope_multi"));
    return c.finish(sync);
}

// Shape checks of cpy_any / upscale_f32 (reference lib/src/ops.c:240-310): an empty dimension is a no-op, negative
// strides are not supported.
static int shape4(const int64_t ne[4], const int64_t nb[4], size_t es, Shape4 *sh, long long *count, size_t *extent,
                  bool *empty) {
    long long n = 1;
    size_t ext = es;
    *empty = false;
    for (int i = 0; i < 4; i++) {
        if (ne[i] <= 0) *empty = true;
        if (nb[i] < 0) return fail(GEN9BLAS_ERR_UNSUPPORTED, "negative byte stride nb[%d] = %lld", i, (long long)nb[i]);
        sh->ne[i] = ne[i];
        sh->nb[i] = nb[i];
        n *= ne[i] > 0 ? ne[i] : 0;
        if (ne[i] > 0) ext += (size_t)(ne[i] - 1) * (size_t)nb[i];
    }
    *count = n;
    *extent = ext;
    return 0;
}

GEN9BLAS_API int gen9blas_cpy_any(const void *src, int tin, const int64_t sne[4], const int64_t snb[4], void *dst, int tout,
                                  const int64_t dne[4], const int64_t dnb[4], int sync) {
    if (int e = begin_op()) return e;
    if ((tin != GEN9BLAS_S && tin != GEN9BLAS_H) || (tout != GEN9BLAS_S && tout != GEN9BLAS_H))
        return fail(GEN9BLAS_ERR_UNSUPPORTED, "cpy_any: types F32 / F16 only");
    if (!sne || !snb || !dne || !dnb) return fail(GEN9BLAS_ERR_INVALID_ARG, "cpy_any: four ne / nb each");
    Shape4 s, dd;
    long long ns = 0, ndd = 0;
    size_t sspan = 0, dspan = 0;
    bool es, ed;
    G9_TRY(shape4(sne, snb, tin == GEN9BLAS_S ? 4 : 2, &s, &ns, &sspan, &es));
    G9_TRY(shape4(dne, dnb, tout == GEN9BLAS_S ? 4 : 2, &dd, &ndd, &dspan, &ed));
    if (es || ed) return 0;
    if (ns != ndd) return fail(GEN9BLAS_ERR_UNSUPPORTED, "cpy_any: %lld source and %lld destination elements", ns, ndd);
    DevState *d = dev_state();
    if (!d) return G.status;
    OpCall c;
    void *sp, *dp;
    cudaStream_t st = stream();
    G9_TRY(c.big(src, sspan, true, false, &sp));
    G9_TRY(c.big(dst, dspan, true, true, &dp));   // copied in: the bytes between strided elements keep their values
    cpy_any_k<<<grid_n(ns, d->sm_count), 256, 0, st>>>((const uint8_t *)sp, tin, s, (uint8_t *)dp, tout, dd, ns);
    G9_TRY(launched("cpy_any"));
    return c.finish(sync);
}

GEN9BLAS_API int gen9blas_upscale_f32(const float *src, const int64_t sne[4], const int64_t snb[4], float *dst,
                                      const int64_t dne[4], const int64_t dnb[4], int mode_flags, int sync) {
    if (int e = begin_op()) return e;
    if (!sne || !snb || !dne || !dnb) return fail(GEN9BLAS_ERR_INVALID_ARG, "upscale_f32: four ne / nb each");
    Shape4 s, dd;
    long long ns = 0, ndd = 0;
    size_t sspan = 0, dspan = 0;
    bool es, ed;
    G9_TRY(shape4(sne, snb, 4, &s, &ns, &sspan, &es));
    G9_TRY(shape4(dne, dnb, 4, &dd, &ndd, &dspan, &ed));
    if (es || ed) return 0;
    const int mode = mode_flags & 0xFF, ac = (mode_flags >> 8) & 1, aa = (mode_flags >> 9) & 1;
    if ((mode != 0 && mode != 1) || (mode_flags & ~0x3FF))
        return fail(GEN9BLAS_ERR_UNSUPPORTED, "upscale_f32: mode flags 0x%x", mode_flags);
    float sf0 = (float)dne[0] / (float)sne[0], sf1 = (float)dne[1] / (float)sne[1];
    const float sf2 = (float)dne[2] / (float)sne[2], sf3 = (float)dne[3] / (float)sne[3];
    float po = 0.5f;
    if (ac) {   // align corners, as ggml-cpu
        po = 0.0f;
        if (dne[0] > 1 && sne[0] > 1) sf0 = (float)(dne[0] - 1) / (float)(sne[0] - 1);
        if (dne[1] > 1 && sne[1] > 1) sf1 = (float)(dne[1] - 1) / (float)(sne[1] - 1);
    }
    DevState *d = dev_state();
    if (!d) return G.status;
    OpCall c;
    void *sp, *dp;
    cudaStream_t st = stream();
    G9_TRY(c.big(src, sspan, true, false, &sp));
    G9_TRY(c.big(dst, dspan, true, true, &dp));
    upscale_k<<<grid_n(ndd, d->sm_count), 256, 0, st>>>((const uint8_t *)sp, s, (uint8_t *)dp, dd, sf0, sf1, sf2, sf3, mode,
                                                        aa, po, ndd);
    G9_TRY(launched("upscale_f32"));
    return c.finish(sync);
}

GEN9BLAS_API int gen9blas_set_rows_f16(int nc, int nr, int ne02, int ne03, const float *src, int64_t s1, int64_t s2,
                                       int64_t s3, const void *idx, size_t idx_bytes, int64_t b10, int64_t b11, int64_t b12,
                                       int idx64, int ne11, int ne12, uint16_t *dst, size_t dst_bytes, int64_t d1,
                                       int64_t d2, int64_t d3, int64_t ne1, int sync, int *bad) {
    if (bad) *bad = 0;
    if (int e = begin_op()) return e;
    if (nc <= 0 || nr <= 0 || ne02 <= 0 || ne03 <= 0) return 0;
    if (ne11 <= 0 || ne12 <= 0 || !idx || !dst) return fail(GEN9BLAS_ERR_INVALID_ARG, "set_rows_f16: bad index shape");
    DevState *d = dev_state();
    if (!d) return G.status;
    if (!on_device(dst)) return fail(GEN9BLAS_ERR_INVALID_ARG, "set_rows_f16: dst must be device or managed memory");
    OpCall c;
    void *sp;
    const void *ip;
    cudaStream_t st = stream();
    const size_t sspan = ((size_t)(nr - 1) * s1 + (size_t)(ne02 - 1) * s2 + (size_t)(ne03 - 1) * s3 + nc) * 4;
    G9_TRY(c.big(src, sspan, true, false, &sp));
    G9_TRY(c.reserve(round256(idx_bytes)));
    G9_TRY(c.in(idx, idx_bytes, &ip, st));
    *(volatile unsigned *)(d->err_host + 1) = 0u;
    set_rows_k<<<grid_n((long long)nc * nr * ne02 * ne03, d->sm_count), 256, 0, st>>>(
        nc, nr, ne02, ne03, (const float *)sp, s1, s2, s3, (const uint8_t *)ip, b10, b11, b12, idx64 ? 1 : 0, ne11, ne12,
        (long long)idx_bytes, (__half *)dst, d1, d2, d3, ne1, (long long)(dst_bytes / 2), d->err_dev + 1);
    G9_TRY(launched("set_rows_f16"));
    c.ops[c.n].user = c.ops[c.n].dptr = dst;   // the destination is written in place (recorded for no-wait ordering)
    c.ops[c.n].bytes = dst_bytes;
    c.ops[c.n].written = true;
    c.n++;
    const int r = c.finish(sync);
    if (r == 0 && (sync || !c.all_dev) && bad) *bad = *(volatile unsigned *)(d->err_host + 1) != 0u;
    return r;
}

// ---- packed GEMM input written by a layer norm (reference: gen9blas_layer_norm_pack, gemm_pa_f16w_ex)
GEN9BLAS_API gen9blas_packed_a *gen9blas_packed_a_create(void) {
    auto *pa = new (std::nothrow) gen9blas_packed_a;
    if (pa) *pa = gen9blas_packed_a{kPackedAMagic, 0, 0, 0, -1, nullptr, 0};
    return pa;
}

GEN9BLAS_API void gen9blas_packed_a_free(gen9blas_packed_a *pa) {
    if (!pa || pa->magic != kPackedAMagic) return;
    if (pa->rows) cudaFree(pa->rows);   // as the reference: does not wait (flush first)
    pa->magic = 0;
    delete pa;
}

GEN9BLAS_API int gen9blas_layer_norm_pack(int M, int K, const float *X, int ldx, const float *w, const float *b, float eps,
                                          float *Y, int ldy, gen9blas_packed_a *pa, int sync) {
    if (int e = begin_op()) return e;
    if (!pa || pa->magic != kPackedAMagic) return fail(GEN9BLAS_ERR_INVALID_ARG, "layer_norm_pack: no packed A");
    if (M <= 0 || K <= 0) return 0;
    if (ldx < K || ldy < K) return fail(GEN9BLAS_ERR_INVALID_ARG, "layer_norm_pack: ldx = %d, ldy = %d < K = %d", ldx, ldy, K);
    DevState *d = dev_state();
    if (!d) return G.status;
    const int Kp = (K + 7) / 8 * 8;
    const size_t need = (size_t)M * Kp * 2;
    if (!pa->rows || pa->bytes < need || pa->dev != d->dev) {
        if (pa->rows) {
            G9_CU(cudaStreamSynchronize(stream()));
            cudaFree(pa->rows);
            pa->rows = nullptr;
        }
        G9_CU(cudaMalloc((void **)&pa->rows, need));
        pa->bytes = need;
        pa->dev = d->dev;
    }
    pa->M = M;
    pa->K = K;
    pa->Kp = Kp;
    OpCall c;
    void *x, *y;
    const void *wd, *bd;
    cudaStream_t st = stream();
    G9_TRY(c.big(X, ((size_t)(M - 1) * ldx + K) * 4, true, false, &x));
    G9_TRY(c.big(Y, ((size_t)(M - 1) * ldy + K) * 4, X == Y || ldy != K, true, &y));
    G9_TRY(c.reserve(2 * round256((size_t)K * 4)));
    G9_TRY(c.in(w, (size_t)K * 4, &wd, st));
    G9_TRY(c.in(b, (size_t)K * 4, &bd, st));
    layer_norm_k<<<M, 256, 0, st>>>((const float *)x, ldx, (const float *)wd, (const float *)bd, eps, (float *)y, ldy, K,
                                    pa->rows, Kp);
    G9_TRY(launched("layer_norm_pack"));
    return c.finish(sync);
}

// ---- attention
GEN9BLAS_API int gen9blas_attn_dec_supported(int D, int H, int HKV) { return attn_shape_ok(D, H, HKV) ? 1 : 0; }
GEN9BLAS_API int gen9blas_attn_supported(int D, int H, int HKV) { return attn_shape_ok(D, H, HKV) ? 1 : 0; }
GEN9BLAS_API int gen9blas_attn_streams_supported(int D, int H, int HKV) { return attn_shape_ok(D, H, HKV) ? 1 : 0; }

GEN9BLAS_API int gen9blas_attn_dec(int D, int H, int HKV, int ns, int nq, int nk, const float *Q, int64_t qt, int64_t qh,
                                   int64_t qs, const uint16_t *K, int64_t kk, int64_t kh, int64_t ks, size_t k_bytes,
                                   const uint16_t *V, int64_t vk, int64_t vh, int64_t vs, size_t v_bytes, float *O,
                                   float scale, const int *vis, int dvis, int chunk, int sync) {
    (void)k_bytes;
    (void)v_bytes;
    (void)chunk;   // the chunk length is this build's own (chosen per call from the grid it gives)
    if (int e = begin_op()) return e;
    if (!vis) return fail(GEN9BLAS_ERR_INVALID_ARG, "attn_dec: no visible counts");
    AttnArgs a{D, H, HKV, ns, nq, nk, 0, dvis, Q, qt, qh, qs, (const __half *)K, kk, kh, ks, (const __half *)V, vk, vh, vs,
               vis, scale * 1.4426950408889634f, nullptr, O};
    return attention(a, sync, "attn_dec");
}

GEN9BLAS_API int gen9blas_attn_f16kv(int D, int H, int HKV, int nq, int nk, const float *Q, const uint16_t *K, size_t k_bytes,
                                     const uint16_t *V, size_t v_bytes, float *O, float scale, int vis0, int dvis,
                                     int *launches) {
    if (launches) *launches = 0;
    if (int e = begin_op()) return e;
    if (!attn_shape_ok(D, H, HKV) || nq <= 0 || nk <= 0 || vis0 < 1) return GEN9BLAS_DECLINED;
    const size_t row = (size_t)HKV * D * 2;
    if (k_bytes < (size_t)nk * row || v_bytes < (size_t)nk * row) return GEN9BLAS_DECLINED;
    AttnArgs a{D, H, HKV, 1, nq, nk, 0, dvis, Q, (long long)H * D, D, 0, (const __half *)K, (long long)HKV * D, D, 0,
               (const __half *)V, (long long)HKV * D, D, 0, &vis0, scale * 1.4426950408889634f, nullptr, O};
    const int r = attention(a, 1, "attn_f16kv");
    if (r == 0 && launches) *launches = 1;
    return r;
}

GEN9BLAS_API int gen9blas_attn_f16kv_streams(int D, int H, int HKV, int ns, int nq, int nk, const float *Q, int64_t sq,
                                             const uint16_t *K, int64_t sk, size_t k_bytes, const uint16_t *V, int64_t sv,
                                             size_t v_bytes, float *O, float scale, const int *vis0, int dvis, int *launches) {
    if (launches) *launches = 0;
    if (int e = begin_op()) return e;
    if (!attn_shape_ok(D, H, HKV) || ns <= 0 || nq <= 0 || nk <= 0 || !vis0) return GEN9BLAS_DECLINED;
    (void)k_bytes;
    (void)v_bytes;
    if (sq != (long long)nq * H * D) return GEN9BLAS_DECLINED;   // O is [s][t][h][d] contiguous, so Q's streams are too
    AttnArgs a{D, H, HKV, ns, nq, nk, 0, dvis, Q, (long long)H * D, D, sq, (const __half *)K, (long long)HKV * D, D, sk,
               (const __half *)V, (long long)HKV * D, D, sv, vis0, scale * 1.4426950408889634f, nullptr, O};
    const int r = attention(a, 1, "attn_f16kv_streams");
    if (r == 0 && launches) *launches = 1;
    return r;
}

}  // extern "C"
