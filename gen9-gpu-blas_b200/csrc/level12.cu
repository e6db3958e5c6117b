// level12.cu -- bandwidth-bound level-1/2 kernels: axpy, dot/asum/nrm2 (FP64 accumulation), iamax, gemv N/T, ger.
//
// Semantics follow the reference kernels in lib/kernels/level12.cl and their host side lib/src/level12.c:
// - axpy: y = fma(a, x, y) in the compute type R, rounded once to the storage type (level12.cl:135-139);
// - reductions: mode 0 x·y, 1 Σ|x|, 2 Σx² accumulated in FP64, nrm2 = sqrt of mode 2 (level12.cl:189-214,
//   level12.c:171-190);
// - iamax: first index of the largest |x| compared in R, NaN never wins (strict >), ties go to the smaller index,
//   all-NaN gives 0 (level12.cl:215-235, level12.c:192-211);
// - gemv: y = alpha·op(A)·x + beta·y with the products summed in R and the epilogue
//   beta == 0 ? alpha·t : fma(alpha, t, beta·y) (level12.cl:243-283, 418-423);
// - ger: A = fma(alpha·x_i, y_j, A_ij) in R (level12.cl:569-576).
// The kernels are B200 designs: 16-byte vector loads in grid-stride loops sized by the SM count, deterministic
// two-stage reductions finished on the GPU (fixed grid, fixed combine order), and split-rows gemv T with a
// fixed-order second pass. No float atomics, so repeated calls give bit-identical results.
#include "common.cuh"
#include "internal.h"
#include <cmath>
#include <cstring>

namespace g9 {

constexpr int kThreads = 256;

static int grid_for(long long work_items, int per_sm) {
    DevState *d = dev_state();
    long long cap = (long long)(d ? d->sm_count : 148) * per_sm;
    long long g = (work_items + kThreads - 1) / kThreads;
    if (g < 1) g = 1;
    return (int)(g < cap ? g : cap);
}

// ------------------------------------------------------------------------------------------------ axpy
template <typename T, bool VEC>
__global__ void __launch_bounds__(kThreads) axpy_kernel(long long n, typename Compute<T>::R a, const T *__restrict__ x,
                                                        long long ix, T *y, long long iy) {
    using R = typename Compute<T>::R;
    const long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    const long long stride = (long long)gridDim.x * blockDim.x;
    if (VEC) {
        constexpr int W = V16<T>::W;
        const long long nv = n / W;
        for (long long v = tid; v < nv; v += stride) {
            R xv[W], yv[W];
            load16<T>(x + v * W, xv);
            load16_rw<T>(y + v * W, yv);
#pragma unroll
            for (int k = 0; k < W; k++) yv[k] = fma_r(a, xv[k], yv[k]);
            store16<T>(y + v * W, yv);
        }
        for (long long i = nv * W + tid; i < n; i += stride) y[i] = from_r<T>(fma_r(a, to_r(x[i]), to_r(y[i])));
    } else {
        for (long long i = tid; i < n; i += stride) {
            const long long jy = i * iy;
            y[jy] = from_r<T>(fma_r(a, to_r(x[i * ix]), to_r(y[jy])));
        }
    }
}

template <typename T>
static int axpy_t(int n, double a, const void *xv, long long ox, long long ix, void *yv, long long oy, long long iy,
                  cudaStream_t st) {
    using R = typename Compute<T>::R;
    const T *x = (const T *)xv + ox;
    T *y = (T *)yv + oy;
    const bool vec = ix == 1 && iy == 1 && (((uintptr_t)x | (uintptr_t)y) & 15) == 0;
    if (vec) {
        axpy_kernel<T, true><<<grid_for(n / V16<T>::W + 1, 16), kThreads, 0, st>>>(n, (R)a, x, ix, y, iy);
    } else {
        axpy_kernel<T, false><<<grid_for(n, 16), kThreads, 0, st>>>(n, (R)a, x, ix, y, iy);
    }
    return launched("axpy");
}

int launch_axpy(int type, int n, double a, const void *x, long long ox, long long ix, void *y, long long oy, long long iy,
                cudaStream_t st) {
    if (type == GEN9BLAS_S) return axpy_t<float>(n, a, x, ox, ix, y, oy, iy, st);
    if (type == GEN9BLAS_D) return axpy_t<double>(n, a, x, ox, ix, y, oy, iy, st);
    return axpy_t<__half>(n, a, x, ox, ix, y, oy, iy, st);
}

// ------------------------------------------------------------------------------------------------ reductions
// Block-wide sum of doubles in a fixed order (warp shuffles, then the warp results in order).
__device__ __forceinline__ double block_sum(double s, double *sh) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_down_sync(0xffffffffu, s, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) sh[w] = s;
    __syncthreads();
    double t = 0;
    if (threadIdx.x == 0)
        for (int i = 0; i < (int)(blockDim.x >> 5); i++) t += sh[i];
    __syncthreads();
    return t;
}

template <int MODE> __device__ __forceinline__ double red_term(double xv, double yv) {
    if (MODE == 0) return xv * yv;
    if (MODE == 1) return fabs(xv);
    return xv * xv;
}

// Stage 1: one FP64 partial per block.
template <typename T, int MODE, bool VEC>
__global__ void __launch_bounds__(kThreads) reduce_partial(long long n, const T *__restrict__ x, long long ix,
                                                           const T *__restrict__ y, long long iy, double *part) {
    __shared__ double sh[kThreads / 32];
    const long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    const long long stride = (long long)gridDim.x * blockDim.x;
    double s = 0;
    if (VEC) {
        constexpr int W = V16<T>::W;
        // 16-byte loads (per operand) in flight per trip, one accumulation chain each: 4 for single-operand FP32 / FP16
        // sums (4-8 terms per load: longer chains would bound them below HBM speed), 2 otherwise.
        constexpr int U = (sizeof(T) == 8 || MODE == 0) ? 2 : 4;
        using R = typename Compute<T>::R;
        const long long nv = n / W;
        double acc[U];
#pragma unroll
        for (int u = 0; u < U; u++) acc[u] = 0;
        long long v = tid;
        for (; v + (U - 1) * stride < nv; v += U * stride) {
            R xv[U][W], yv[U][W];
#pragma unroll
            for (int u = 0; u < U; u++) load16<T>(x + (v + u * stride) * W, xv[u]);
            if (MODE == 0) {
#pragma unroll
                for (int u = 0; u < U; u++) load16<T>(y + (v + u * stride) * W, yv[u]);
            }
#pragma unroll
            for (int k = 0; k < W; k++)
#pragma unroll
                for (int u = 0; u < U; u++)
                    acc[u] += red_term<MODE>((double)xv[u][k], MODE == 0 ? (double)yv[u][k] : 0.0);
        }
        for (; v < nv; v += stride) {
            R xv[W], yv[W];
            load16<T>(x + v * W, xv);
            if (MODE == 0) load16<T>(y + v * W, yv);
#pragma unroll
            for (int k = 0; k < W; k++) acc[0] += red_term<MODE>((double)xv[k], MODE == 0 ? (double)yv[k] : 0.0);
        }
#pragma unroll
        for (int u = 0; u < U; u++) s += acc[u];
        for (long long i = nv * W + tid; i < n; i += stride)
            s += red_term<MODE>((double)to_r(x[i]), MODE == 0 ? (double)to_r(y[i]) : 0.0);
    } else {
        for (long long i = tid; i < n; i += stride)
            s += red_term<MODE>((double)to_r(x[i * ix]), MODE == 0 ? (double)to_r(y[i * iy]) : 0.0);
    }
    s = block_sum(s, sh);
    if (threadIdx.x == 0) part[blockIdx.x] = s;
}

// Stage 2: fixed-order sum of the partials; mode 2 takes the square root (nrm2).
__global__ void __launch_bounds__(kThreads) reduce_final(int nparts, const double *part, int sqrt_out, double *out) {
    __shared__ double sh[kThreads / 32];
    double s = 0;
    for (int i = threadIdx.x; i < nparts; i += blockDim.x) s += part[i];
    s = block_sum(s, sh);
    if (threadIdx.x == 0) out[0] = sqrt_out ? sqrt(s) : s;
}

template <typename T>
static int reduce_t(int mode, int n, const void *xv, long long ox, long long ix, const void *yv, long long oy, long long iy,
                    double *result_dev, cudaStream_t st) {
    const T *x = (const T *)xv + ox;
    const T *y = yv ? (const T *)yv + oy : x;
    const bool vec = ix == 1 && (mode != 0 || iy == 1) && (((uintptr_t)x | (uintptr_t)(mode == 0 ? y : x)) & 15) == 0;
    const int g = vec ? grid_for(n / V16<T>::W + 1, 8) : grid_for(n, 8);
    double *part = result_dev + 8;   // the scratch holds [result, pad..., partials]
#define G9_RED(M)                                                                                          \
    if (vec) reduce_partial<T, M, true><<<g, kThreads, 0, st>>>(n, x, ix, y, iy, part);                   \
    else reduce_partial<T, M, false><<<g, kThreads, 0, st>>>(n, x, ix, y, iy, part);
    if (mode == 0) { G9_RED(0) } else if (mode == 1) { G9_RED(1) } else { G9_RED(2) }
#undef G9_RED
    G9_TRY(launched("reduce_partial"));
    reduce_final<<<1, kThreads, 0, st>>>(g, part, mode == 2, result_dev);
    return launched("reduce_final");
}

int launch_reduce(int type, int mode, int n, const void *x, long long ox, long long ix, const void *y, long long oy,
                  long long iy, double *result_dev, cudaStream_t st) {
    if (type == GEN9BLAS_S) return reduce_t<float>(mode, n, x, ox, ix, y, oy, iy, result_dev, st);
    if (type == GEN9BLAS_D) return reduce_t<double>(mode, n, x, ox, ix, y, oy, iy, result_dev, st);
    return reduce_t<__half>(mode, n, x, ox, ix, y, oy, iy, result_dev, st);
}

// ------------------------------------------------------------------------------------------------ iamax
constexpr long long kNoIndex = 0x7fffffffffffffffLL;

// (value, index) pairs: the larger value wins, equal values keep the smaller index. NaN is never stored
// (v > best is false for NaN), so the combination is associative and the result does not depend on the grid.
template <typename R> __device__ __forceinline__ void better(R &bv, long long &bi, R v, long long i) {
    if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
}

template <typename R> __device__ __forceinline__ void block_best(R &bv, long long &bi, R *shv, long long *shi) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        R ov = __shfl_down_sync(0xffffffffu, bv, o);
        long long oi = __shfl_down_sync(0xffffffffu, bi, o);
        better(bv, bi, ov, oi);
    }
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) { shv[w] = bv; shi[w] = bi; }
    __syncthreads();
    if (threadIdx.x == 0)
        for (int i = 1; i < (int)(blockDim.x >> 5); i++) better(bv, bi, shv[i], shi[i]);
    __syncthreads();
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(kThreads) iamax_partial(long long n, const T *__restrict__ x, long long ix,
                                                          typename Compute<T>::R *pv, long long *pi) {
    using R = typename Compute<T>::R;
    __shared__ R shv[kThreads / 32];
    __shared__ long long shi[kThreads / 32];
    const long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    const long long stride = (long long)gridDim.x * blockDim.x;
    R bv = (R)-1;
    long long bi = kNoIndex;
    if (VEC) {
        constexpr int W = V16<T>::W;
        constexpr int U = sizeof(T) == 8 ? 2 : 4;   // loads in flight per trip; chain u scans the elements of load u
        const long long nv = n / W;
        R cv[U];
        long long ci[U];
#pragma unroll
        for (int u = 0; u < U; u++) { cv[u] = (R)-1; ci[u] = kNoIndex; }
        long long v = tid;
        for (; v + (U - 1) * stride < nv; v += U * stride) {
            R xv[U][W];
#pragma unroll
            for (int u = 0; u < U; u++) load16<T>(x + (v + u * stride) * W, xv[u]);
#pragma unroll
            for (int u = 0; u < U; u++)
#pragma unroll
                for (int k = 0; k < W; k++) {
                    const R a = fabs(xv[u][k]);
                    if (a > cv[u]) { cv[u] = a; ci[u] = (v + u * stride) * W + k; }
                }
        }
        for (; v < nv; v += stride) {
            R xv[W];
            load16<T>(x + v * W, xv);
#pragma unroll
            for (int k = 0; k < W; k++) {
                const R a = fabs(xv[k]);
                if (a > cv[0]) { cv[0] = a; ci[0] = v * W + k; }
            }
        }
        // Each chain holds the first index of its largest value; the (value, index) combination keeps the smaller
        // index on ties, so the thread's result is the first index of its largest value.
#pragma unroll
        for (int u = 0; u < U; u++) better(bv, bi, cv[u], ci[u]);
        for (long long i = nv * W + tid; i < n; i += stride) {
            const R a = fabs(to_r(x[i]));
            if (a > bv) { bv = a; bi = i; }
        }
    } else {
        for (long long i = tid; i < n; i += stride) {
            const R a = fabs(to_r(x[i * ix]));
            if (a > bv) { bv = a; bi = i; }
        }
    }
    block_best(bv, bi, shv, shi);
    if (threadIdx.x == 0) { pv[blockIdx.x] = bv; pi[blockIdx.x] = bi; }
}

template <typename R>
__global__ void __launch_bounds__(kThreads) iamax_final(int nparts, const R *pv, const long long *pi, long long *out) {
    __shared__ R shv[kThreads / 32];
    __shared__ long long shi[kThreads / 32];
    R bv = (R)-1;
    long long bi = kNoIndex;
    for (int i = threadIdx.x; i < nparts; i += blockDim.x) better(bv, bi, pv[i], pi[i]);
    block_best(bv, bi, shv, shi);
    if (threadIdx.x == 0) out[0] = bi == kNoIndex ? 0 : bi;
}

template <typename T>
static int iamax_t(int n, const void *xv, long long ox, long long ix, long long *result_dev, cudaStream_t st) {
    using R = typename Compute<T>::R;
    const T *x = (const T *)xv + ox;
    const bool vec = ix == 1 && ((uintptr_t)x & 15) == 0;
    const int g = vec ? grid_for(n / V16<T>::W + 1, 8) : grid_for(n, 8);
    long long *pi = result_dev + 8;
    R *pv = reinterpret_cast<R *>(pi + g);
    if (vec) iamax_partial<T, true><<<g, kThreads, 0, st>>>(n, x, ix, pv, pi);
    else iamax_partial<T, false><<<g, kThreads, 0, st>>>(n, x, ix, pv, pi);
    G9_TRY(launched("iamax_partial"));
    iamax_final<R><<<1, kThreads, 0, st>>>(g, pv, pi, result_dev);
    return launched("iamax_final");
}

int launch_iamax(int type, int n, const void *x, long long ox, long long ix, long long *result_dev, cudaStream_t st) {
    if (type == GEN9BLAS_S) return iamax_t<float>(n, x, ox, ix, result_dev, st);
    if (type == GEN9BLAS_D) return iamax_t<double>(n, x, ox, ix, result_dev, st);
    return iamax_t<__half>(n, x, ox, ix, result_dev, st);
}

// ------------------------------------------------------------------------------------------------ gemv N
// One warp computes kRowsN rows; each lane reads 16-byte vectors of the rows and of x (x comes from L1: every warp
// of the block walks the same columns). Sum order: per-lane partials, then a fixed shuffle tree.
constexpr int kRowsN = 2;
constexpr int kTripsN = 4;   // trips of 16-byte loads issued before their FMAs

template <typename T>
__device__ __forceinline__ void gemv_store(T *y, long long k, typename Compute<T>::R alpha, typename Compute<T>::R beta,
                                           typename Compute<T>::R t) {
    y[k] = from_r<T>(beta == 0 ? alpha * t : fma_r(alpha, t, beta * to_r(y[k])));
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(kThreads) gemv_n_kernel(int M, int N, typename Compute<T>::R alpha,
                                                          const T *__restrict__ A, long long lda, const T *__restrict__ x,
                                                          long long ix, typename Compute<T>::R beta, T *y, long long iy) {
    using R = typename Compute<T>::R;
    const int lane = threadIdx.x & 31;
    const long long warp = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    const long long r0 = warp * kRowsN;
    if (r0 >= M) return;
    const int nr = (int)(M - r0 < kRowsN ? M - r0 : kRowsN);
    R s[kRowsN];
#pragma unroll
    for (int r = 0; r < kRowsN; r++) s[r] = 0;
    const T *a0 = A + r0 * lda;
    if (VEC) {
        constexpr int W = V16<T>::W;
        const int nv = N / W;
        int v = lane;
        for (; v + 32 * (kTripsN - 1) < nv; v += 32 * kTripsN) {
            R xv[kTripsN][W], av[kTripsN][kRowsN][W];
#pragma unroll
            for (int u = 0; u < kTripsN; u++) {
                load16<T>(x + (long long)(v + 32 * u) * W, xv[u]);
#pragma unroll
                for (int r = 0; r < kRowsN; r++)
                    load16<T>(a0 + (r < nr ? r : 0) * lda + (long long)(v + 32 * u) * W, av[u][r]);
            }
#pragma unroll
            for (int u = 0; u < kTripsN; u++)
#pragma unroll
                for (int r = 0; r < kRowsN; r++)
#pragma unroll
                    for (int k = 0; k < W; k++) s[r] = fma_r(av[u][r][k], xv[u][k], s[r]);
        }
        for (; v < nv; v += 32) {
            R xv[W];
            load16<T>(x + (long long)v * W, xv);
#pragma unroll
            for (int r = 0; r < kRowsN; r++) {
                if (r < nr) {
                    R av[W];
                    load16<T>(a0 + r * lda + (long long)v * W, av);
#pragma unroll
                    for (int k = 0; k < W; k++) s[r] = fma_r(av[k], xv[k], s[r]);
                }
            }
        }
        for (int j = nv * W + lane; j < N; j += 32) {
            const R xj = to_r(x[j]);
#pragma unroll
            for (int r = 0; r < kRowsN; r++)
                if (r < nr) s[r] = fma_r(to_r(a0[r * lda + j]), xj, s[r]);
        }
    } else {
        for (int j = lane; j < N; j += 32) {
            const R xj = to_r(x[j * ix]);
#pragma unroll
            for (int r = 0; r < kRowsN; r++)
                if (r < nr) s[r] = fma_r(to_r(a0[r * lda + j]), xj, s[r]);
        }
    }
#pragma unroll
    for (int r = 0; r < kRowsN; r++) {
        R t = s[r];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (lane == 0 && r < nr) gemv_store<T>(y, (r0 + r) * iy, alpha, beta, t);
    }
}

// ------------------------------------------------------------------------------------------------ gemv T
// Stage 1: block = 256 threads × W columns (one 16-byte vector each), rows [p·rpp, (p+1)·rpp); partial sums P[p][col].
template <typename T, bool VEC>
__global__ void __launch_bounds__(kThreads) gemv_t_partial(int M, int N, int rpp, const T *__restrict__ A, long long lda,
                                                           const T *__restrict__ x, long long ix,
                                                           typename Compute<T>::R *P) {
    using R = typename Compute<T>::R;
    constexpr int W = VEC ? V16<T>::W : 1;
    const long long c = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * W;
    const int p = blockIdx.y;
    if (c >= N) return;
    const int i0 = p * rpp, i1 = min(M, i0 + rpp);
    R s[W];
#pragma unroll
    for (int k = 0; k < W; k++) s[k] = 0;
    const bool full = c + W <= N;
    if (VEC && full) {
        constexpr int U = 4;   // rows whose 16-byte loads are in flight together (row order of the sums kept)
        int i = i0;
        for (; i + U <= i1; i += U) {
            R av[U][W], xv[U];
#pragma unroll
            for (int u = 0; u < U; u++) {
                load16<T>(A + (long long)(i + u) * lda + c, av[u]);
                xv[u] = to_r(x[(long long)(i + u) * ix]);
            }
#pragma unroll
            for (int u = 0; u < U; u++)
#pragma unroll
                for (int k = 0; k < W; k++) s[k] = fma_r(av[u][k], xv[u], s[k]);
        }
        for (; i < i1; i++) {
            const R xv = to_r(x[i * ix]);
            R av[W];
            load16<T>(A + i * lda + c, av);
#pragma unroll
            for (int k = 0; k < W; k++) s[k] = fma_r(av[k], xv, s[k]);
        }
    } else {
        for (int i = i0; i < i1; i++) {
            const R xv = to_r(x[i * ix]);
#pragma unroll
            for (int k = 0; k < W; k++)
                if (c + k < N) s[k] = fma_r(to_r(A[i * lda + c + k]), xv, s[k]);
        }
    }
    R *out = P + (long long)p * N + c;
#pragma unroll
    for (int k = 0; k < W; k++)
        if (c + k < N) out[k] = s[k];
}

template <typename T>
__global__ void __launch_bounds__(kThreads) gemv_t_final(int N, int parts, const typename Compute<T>::R *P,
                                                         typename Compute<T>::R alpha, typename Compute<T>::R beta, T *y,
                                                         long long iy) {
    using R = typename Compute<T>::R;
    const long long j = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (j >= N) return;
    R t = 0;
    for (int p = 0; p < parts; p++) t += P[(long long)p * N + j];
    gemv_store<T>(y, j * iy, alpha, beta, t);
}

// Row parts of the transposed product: as many as fill exactly one wave of resident blocks together with the column
// blocks (a second, nearly empty wave would double the time).
template <typename T> static int gemv_t_wave_parts(bool vec, int col_blocks, int sm_count) {
    int per_sm = 0;
    if (vec) cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_t_partial<T, true>, kThreads, 0);
    else cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_t_partial<T, false>, kThreads, 0);
    if (per_sm < 1) per_sm = 1;
    const int parts = sm_count * per_sm / col_blocks;
    return parts < 1 ? 1 : parts;
}

template <typename T>
static int gemv_t(int trans, int M, int N, double alpha, const void *Av, int lda, const void *xv, long long ox,
                  long long ix, double beta, void *yv, long long oy, long long iy, cudaStream_t st) {
    using R = typename Compute<T>::R;
    const T *A = (const T *)Av;
    const T *x = (const T *)xv + ox;
    T *y = (T *)yv + oy;
    constexpr int W = V16<T>::W;
    if (!trans) {
        const bool vec = ix == 1 && (((uintptr_t)A | (uintptr_t)x) & 15) == 0 && ((long long)lda * sizeof(T)) % 16 == 0;
        const long long warps = (M + kRowsN - 1) / kRowsN;
        const int blocks = (int)((warps * 32 + kThreads - 1) / kThreads);
        if (vec) gemv_n_kernel<T, true><<<blocks, kThreads, 0, st>>>(M, N, (R)alpha, A, lda, x, ix, (R)beta, y, iy);
        else gemv_n_kernel<T, false><<<blocks, kThreads, 0, st>>>(M, N, (R)alpha, A, lda, x, ix, (R)beta, y, iy);
        return launched("gemv_n");
    }
    const bool vec = (((uintptr_t)A) & 15) == 0 && ((long long)lda * sizeof(T)) % 16 == 0;
    const int w = vec ? W : 1;
    const int col_blocks = (int)(((long long)N + (long long)kThreads * w - 1) / ((long long)kThreads * w));
    DevState *d = dev_state();
    int parts = gemv_t_wave_parts<T>(vec, col_blocks, d ? d->sm_count : 148);
    if (parts > M) parts = M;
    if (parts > 65535) parts = 65535;
    if (parts < 1) parts = 1;
    const int rpp = (M + parts - 1) / parts;
    parts = (M + rpp - 1) / rpp;
    void *P = nullptr;
    G9_TRY(scratch((size_t)parts * N * sizeof(R), &P));
    dim3 grid(col_blocks, parts);
    if (vec) gemv_t_partial<T, true><<<grid, kThreads, 0, st>>>(M, N, rpp, A, lda, x, ix, (R *)P);
    else gemv_t_partial<T, false><<<grid, kThreads, 0, st>>>(M, N, rpp, A, lda, x, ix, (R *)P);
    G9_TRY(launched("gemv_t_partial"));
    gemv_t_final<T><<<(N + kThreads - 1) / kThreads, kThreads, 0, st>>>(N, parts, (const R *)P, (R)alpha, (R)beta, y, iy);
    return launched("gemv_t_final");
}

int launch_gemv(int type, int trans, int M, int N, double alpha, const void *A, int lda, const void *x, long long ox,
                long long ix, double beta, void *y, long long oy, long long iy, cudaStream_t st) {
    if (type == GEN9BLAS_S) return gemv_t<float>(trans, M, N, alpha, A, lda, x, ox, ix, beta, y, oy, iy, st);
    if (type == GEN9BLAS_D) return gemv_t<double>(trans, M, N, alpha, A, lda, x, ox, ix, beta, y, oy, iy, st);
    return gemv_t<__half>(trans, M, N, alpha, A, lda, x, ox, ix, beta, y, oy, iy, st);
}

// ------------------------------------------------------------------------------------------------ ger
// Thread = one 16-byte vector of a row of A (W elements), rows in a grid-stride loop over blockIdx.y.
template <typename T, bool VEC>
__global__ void __launch_bounds__(kThreads) ger_kernel(int M, int N, typename Compute<T>::R alpha, const T *__restrict__ x,
                                                       long long ix, const T *__restrict__ y, long long iy, T *A,
                                                       long long lda) {
    using R = typename Compute<T>::R;
    constexpr int W = VEC ? V16<T>::W : 1;
    const long long c = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * W;
    if (c >= N) return;
    R yv[W];
#pragma unroll
    for (int k = 0; k < W; k++) yv[k] = c + k < N ? to_r(y[(c + k) * iy]) : (R)0;
    const bool full = c + W <= N;
    for (long long i = blockIdx.y; i < M; i += gridDim.y) {
        const R ax = alpha * to_r(x[i * ix]);
        T *row = A + i * lda + c;
        if (VEC && full) {
            R av[W];
            load16_rw<T>(row, av);
#pragma unroll
            for (int k = 0; k < W; k++) av[k] = fma_r(ax, yv[k], av[k]);
            store16<T>(row, av);
        } else {
#pragma unroll
            for (int k = 0; k < W; k++)
                if (c + k < N) row[k] = from_r<T>(fma_r(ax, yv[k], to_r(row[k])));
        }
    }
}

template <typename T>
static int ger_t(int M, int N, double alpha, const void *xv, long long ox, long long ix, const void *yv, long long oy,
                 long long iy, void *Av, int lda, cudaStream_t st) {
    using R = typename Compute<T>::R;
    const T *x = (const T *)xv + ox;
    const T *y = (const T *)yv + oy;
    T *A = (T *)Av;
    const bool vec = (((uintptr_t)A) & 15) == 0 && ((long long)lda * sizeof(T)) % 16 == 0;
    const int w = vec ? V16<T>::W : 1;
    const int col_blocks = (int)(((long long)N + (long long)kThreads * w - 1) / ((long long)kThreads * w));
    DevState *d = dev_state();
    const int want = (d ? d->sm_count : 148) * 16;
    int rows = (want + col_blocks - 1) / col_blocks;
    if (rows > M) rows = M;
    if (rows > 65535) rows = 65535;
    if (rows < 1) rows = 1;
    dim3 grid(col_blocks, rows);
    if (vec) ger_kernel<T, true><<<grid, kThreads, 0, st>>>(M, N, (R)alpha, x, ix, y, iy, A, lda);
    else ger_kernel<T, false><<<grid, kThreads, 0, st>>>(M, N, (R)alpha, x, ix, y, iy, A, lda);
    return launched("ger");
}

int launch_ger(int type, int M, int N, double alpha, const void *x, long long ox, long long ix, const void *y,
               long long oy, long long iy, void *A, int lda, cudaStream_t st) {
    if (type == GEN9BLAS_S) return ger_t<float>(M, N, alpha, x, ox, ix, y, oy, iy, A, lda, st);
    if (type == GEN9BLAS_D) return ger_t<double>(M, N, alpha, x, ox, ix, y, oy, iy, A, lda, st);
    return ger_t<__half>(M, N, alpha, x, ox, ix, y, oy, iy, A, lda, st);
}

}  // namespace g9

// ================================================================================================ C API
using namespace g9;

// Element size of a level-1/2 type; H and HS are the same FP16 type here (ref: lib/src/level12.c:10-15).
static int l12_es(int type) {
    return type == GEN9BLAS_S ? 4 : type == GEN9BLAS_D ? 8 : (type == GEN9BLAS_H || type == GEN9BLAS_HS) ? 2 : 0;
}
static int l12_type(int type) { return type == GEN9BLAS_HS ? GEN9BLAS_H : type; }

// Operation prologue of the reference's BEGIN macro (lib/src/internal.h:58-59): type check, n <= 0 is a no-op,
// a zero increment is an invalid argument.
#define L12_BEGIN(n, bad_inc)                                                                       \
    if (int e_ = begin_op()) return e_;                                                             \
    const int es = l12_es(type);                                                                    \
    if (!es) return fail(GEN9BLAS_ERR_UNSUPPORTED, "type %d unavailable", type);                    \
    if ((n) <= 0) return 0;                                                                         \
    if (bad_inc) return fail(GEN9BLAS_ERR_INVALID_ARG, "vector increment 0");

extern "C" {

GEN9BLAS_API int gen9blas_axpy(int type, int n, double a, const void *x, int incx, void *y, int incy) {
    L12_BEGIN(n, !incx || !incy);
    timer_start();
    Operand op[2];
    G9_TRY(map_operand(op[0], x, vec_span(n, incx) * es, 0, true, false));
    G9_TRY(map_operand(op[1], y, vec_span(n, incy) * es, 1, true, true));
    vec_strided(op[1], n, incy, es);
    timer_kernel();
    G9_TRY(launch_axpy(l12_type(type), n, a, op[0].dptr, vec_off(n, incx), incx, op[1].dptr, vec_off(n, incy), incy, stream()));
    G.last_zc = op[0].zc | op[1].zc << 1;
    int r = finish_op(op, 2);
    timer_stop();
    return r;
}

static int reduction(int type, int mode, int n, const void *x, int incx, const void *y, int incy, double *result) {
    if (result) *result = 0;
    L12_BEGIN(n, !incx || (mode == 0 && !incy));
    if (!result) return fail(GEN9BLAS_ERR_INVALID_ARG, "NULL result");
    timer_start();
    Operand op[2];
    G9_TRY(map_operand(op[0], x, vec_span(n, incx) * es, 0, true, false));
    if (mode == 0) G9_TRY(map_operand(op[1], y, vec_span(n, incy) * es, 1, true, false));
    DevState *d = dev_state();
    const int max_parts = d->sm_count * 4 + 64;
    void *scr = nullptr;
    G9_TRY(scratch((size_t)(8 + max_parts) * sizeof(double), &scr));
    cudaStream_t st = stream();
    timer_kernel();
    G9_TRY(launch_reduce(l12_type(type), mode, n, op[0].dptr, vec_off(n, incx), incx, mode == 0 ? op[1].dptr : nullptr,
                         mode == 0 ? vec_off(n, incy) : 0, incy, (double *)scr, st));
    G9_CU(cudaMemcpyAsync(d->result_host, scr, sizeof(double), cudaMemcpyDeviceToHost, st));
    G9_CU(cudaStreamSynchronize(st));
    *result = d->result_host[0];
    int r = finish_op(op, mode == 0 ? 2 : 1);
    timer_stop();
    return r;
}

GEN9BLAS_API int gen9blas_dot(int type, int n, const void *x, int incx, const void *y, int incy, double *result) {
    return reduction(type, 0, n, x, incx, y, incy, result);
}
GEN9BLAS_API int gen9blas_asum(int type, int n, const void *x, int incx, double *result) {
    return reduction(type, 1, n, x, incx, nullptr, 0, result);
}
GEN9BLAS_API int gen9blas_nrm2(int type, int n, const void *x, int incx, double *result) {
    return reduction(type, 2, n, x, incx, nullptr, 0, result);
}

GEN9BLAS_API int gen9blas_iamax(int type, int n, const void *x, int incx, int64_t *result) {
    if (result) *result = -1;
    L12_BEGIN(n, !incx);
    if (!result) return fail(GEN9BLAS_ERR_INVALID_ARG, "NULL result");
    timer_start();
    Operand op[1];
    G9_TRY(map_operand(op[0], x, vec_span(n, incx) * es, 0, true, false));
    DevState *d = dev_state();
    const int max_parts = d->sm_count * 4 + 64;
    void *scr = nullptr;
    G9_TRY(scratch((size_t)(8 + 2 * max_parts) * sizeof(long long) + 64, &scr));
    cudaStream_t st = stream();
    timer_kernel();
    G9_TRY(launch_iamax(l12_type(type), n, op[0].dptr, vec_off(n, incx), incx, (long long *)scr, st));
    G9_CU(cudaMemcpyAsync(d->result_host, scr, sizeof(long long), cudaMemcpyDeviceToHost, st));
    G9_CU(cudaStreamSynchronize(st));
    long long v;
    memcpy(&v, d->result_host, sizeof v);
    *result = v;
    int r = finish_op(op, 1);
    timer_stop();
    return r;
}

GEN9BLAS_API int gen9blas_gemv(int type, int trans, int M, int N, double alpha, const void *A, int lda, const void *x,
                               int incx, double beta, void *y, int incy) {
    L12_BEGIN(M < N ? M : N, !incx || !incy);
    if (lda < N) return fail(GEN9BLAS_ERR_INVALID_ARG, "lda < N");
    timer_start();
    const int nx = trans ? M : N, ny = trans ? N : M;
    Operand op[3];
    G9_TRY(map_operand(op[0], A, ((size_t)(M - 1) * lda + N) * es, 0, true, false));
    G9_TRY(map_operand(op[1], x, vec_span(nx, incx) * es, 1, true, false));
    // y is read when beta != 0, and copied in when strided so the gaps survive the copy back.
    G9_TRY(map_operand(op[2], y, vec_span(ny, incy) * es, 2, beta != 0.0 || (incy != 1 && incy != -1), true));
    vec_strided(op[2], ny, incy, es);
    timer_kernel();
    G9_TRY(launch_gemv(l12_type(type), trans ? 1 : 0, M, N, alpha, op[0].dptr, lda, op[1].dptr, vec_off(nx, incx), incx,
                       beta, op[2].dptr, vec_off(ny, incy), incy, stream()));
    G.last_zc = op[0].zc | op[1].zc << 1 | op[2].zc << 2;
    int r = finish_op(op, 3);
    timer_stop();
    return r;
}

GEN9BLAS_API int gen9blas_ger(int type, int M, int N, double alpha, const void *x, int incx, const void *y, int incy,
                              void *A, int lda) {
    L12_BEGIN(M < N ? M : N, !incx || !incy);
    if (lda < N) return fail(GEN9BLAS_ERR_INVALID_ARG, "lda < N");
    timer_start();
    Operand op[3];
    G9_TRY(map_operand(op[0], x, vec_span(M, incx) * es, 0, true, false));
    G9_TRY(map_operand(op[1], y, vec_span(N, incy) * es, 1, true, false));
    G9_TRY(map_operand(op[2], A, ((size_t)(M - 1) * lda + N) * es, 2, true, true));
    timer_kernel();
    G9_TRY(launch_ger(l12_type(type), M, N, alpha, op[0].dptr, vec_off(M, incx), incx, op[1].dptr, vec_off(N, incy), incy,
                      op[2].dptr, lda, stream()));
    G.last_zc = op[0].zc | op[1].zc << 1 | op[2].zc << 2;
    int r = finish_op(op, 3);
    timer_stop();
    return r;
}

}  // extern "C"

// ================================================================================================ allocation-free gemv
// gen9blas_gemv_noalloc: the gemv entry point for callers that must not allocate GPU memory. The transposed product
// needs scratch for its split-row partial sums; here that scratch is a fixed array in the library's own device image
// instead of the grow-only buffer of gen9blas_gemv. See include/gen9blas.h for the contract.
namespace g9 {

constexpr size_t kNoAllocScratchBytes = 8u << 20;   // 8 MiB per GPU that loads the library, held until exit

// Partial sums of the transposed product. Device code could name it directly; host code needs its device address,
// which noalloc_scratch() obtains once per device with cudaGetSymbolAddress (the array's name in host code is only a
// host-side stand-in, not a device address).
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

static void *g_noalloc_ptr[kMaxDevices];

static int noalloc_scratch(int dev, void **p) {
    if (!g_noalloc_ptr[dev]) {
        void *ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return fail(GEN9BLAS_ERR, "cudaGetSymbolAddress of the no-allocation scratch failed on device %d: %s", dev,
                        cudaGetErrorString(e));
        }
        g_noalloc_ptr[dev] = ptr;
    }
    *p = g_noalloc_ptr[dev];
    return 0;
}

static bool device_resident(const void *p, int dev) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return (a.type == cudaMemoryTypeDevice && a.device == dev) || a.type == cudaMemoryTypeManaged;
}

template <typename T>
static int gemv_noalloc_t(int trans, int M, int N, double alpha, const T *A, int lda, const T *x, long long ix,
                          double beta, T *y, long long iy, int sm_count, void *P, cudaStream_t st) {
    using R = typename Compute<T>::R;
    if (!trans) {   // the untransposed product uses no scratch: same kernel as gen9blas_gemv
        const bool vec = ix == 1 && (((uintptr_t)A | (uintptr_t)x) & 15) == 0 && ((long long)lda * sizeof(T)) % 16 == 0;
        const long long warps = (M + kRowsN - 1) / kRowsN;
        const int blocks = (int)((warps * 32 + kThreads - 1) / kThreads);
        if (vec) gemv_n_kernel<T, true><<<blocks, kThreads, 0, st>>>(M, N, (R)alpha, A, lda, x, ix, (R)beta, y, iy);
        else gemv_n_kernel<T, false><<<blocks, kThreads, 0, st>>>(M, N, (R)alpha, A, lda, x, ix, (R)beta, y, iy);
        return launched("gemv_n");
    }
    const size_t row_bytes = (size_t)N * sizeof(R);   // one part of the partial sums
    if (row_bytes > kNoAllocScratchBytes)
        return fail(GEN9BLAS_ERR_INVALID_ARG,
                    "gen9blas_gemv_noalloc: trans with N = %d needs %zu bytes of scratch per row part; the fixed "
                    "scratch holds %zu bytes (N <= %zu for this type)", N, row_bytes, kNoAllocScratchBytes,
                    kNoAllocScratchBytes / sizeof(R));
    const bool vec = (((uintptr_t)A) & 15) == 0 && ((long long)lda * sizeof(T)) % 16 == 0;
    const int w = vec ? V16<T>::W : 1;
    const int col_blocks = (int)(((long long)N + (long long)kThreads * w - 1) / ((long long)kThreads * w));
    int parts = gemv_t_wave_parts<T>(vec, col_blocks, sm_count);   // the split of gen9blas_gemv ...
    const long long fit = (long long)(kNoAllocScratchBytes / row_bytes);
    if (parts > fit) parts = (int)fit;                          // ... capped by the fixed scratch
    if (parts > M) parts = M;
    if (parts > 65535) parts = 65535;
    if (parts < 1) parts = 1;
    const int rpp = (M + parts - 1) / parts;
    parts = (M + rpp - 1) / rpp;
    dim3 grid(col_blocks, parts);
    if (vec) gemv_t_partial<T, true><<<grid, kThreads, 0, st>>>(M, N, rpp, A, lda, x, ix, (R *)P);
    else gemv_t_partial<T, false><<<grid, kThreads, 0, st>>>(M, N, rpp, A, lda, x, ix, (R *)P);
    G9_TRY(launched("gemv_t_partial"));
    gemv_t_final<T><<<(N + kThreads - 1) / kThreads, kThreads, 0, st>>>(N, parts, (const R *)P, (R)alpha, (R)beta, y, iy);
    return launched("gemv_t_final");
}

}  // namespace g9

extern "C" GEN9BLAS_API int gen9blas_gemv_noalloc(int type, int trans, int M, int N, double alpha, const void *A, int lda,
                                                  const void *x, int incx, double beta, void *y, int incy) {
    G.status = 0;
    G.err[0] = 0;
    if (int e = gen9blas_init()) return e;
    const int es = l12_es(type);
    if (!es) return fail(GEN9BLAS_ERR_UNSUPPORTED, "type %d unavailable", type);
    if ((M < N ? M : N) <= 0) return 0;
    if (!incx || !incy) return fail(GEN9BLAS_ERR_INVALID_ARG, "vector increment 0");
    if (lda < N) return fail(GEN9BLAS_ERR_INVALID_ARG, "lda < N");
    const int dev = G.cur_dev;
    int cur = -1;
    G9_CU(cudaGetDevice(&cur));
    if (cur != dev) G9_CU(cudaSetDevice(dev));
    if (!device_resident(A, dev) || !device_resident(x, dev) || !device_resident(y, dev))
        return fail(GEN9BLAS_ERR_INVALID_ARG,
                    "gen9blas_gemv_noalloc takes device or managed memory of the current device only (no staging)");
    void *P = nullptr;
    G9_TRY(noalloc_scratch(dev, &P));
    int sm_count = 0;
    G9_CU(cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, dev));
    // The library's stream of this device, so that the call is ordered with the other entry points' work and
    // gen9blas_flush waits for it. Before any other call has set up the device there is no such stream (setting it
    // up would allocate); the call then runs on the per-thread default stream and always waits for it.
    DevState *ds = dev_state_if_ready(dev);
    cudaStream_t st = G.user_stream_set ? G.user_stream : ds ? ds->own_stream : cudaStreamPerThread;
    const int nx = trans ? M : N, ny = trans ? N : M;
    const long long ox = vec_off(nx, incx), oy = vec_off(ny, incy);
    int r;
    switch (l12_type(type)) {
    case GEN9BLAS_S:
        r = gemv_noalloc_t<float>(trans ? 1 : 0, M, N, alpha, (const float *)A, lda, (const float *)x + ox, incx, beta,
                                  (float *)y + oy, incy, sm_count, P, st);
        break;
    case GEN9BLAS_D:
        r = gemv_noalloc_t<double>(trans ? 1 : 0, M, N, alpha, (const double *)A, lda, (const double *)x + ox, incx, beta,
                                   (double *)y + oy, incy, sm_count, P, st);
        break;
    default:
        r = gemv_noalloc_t<__half>(trans ? 1 : 0, M, N, alpha, (const __half *)A, lda, (const __half *)x + ox, incx, beta,
                                   (__half *)y + oy, incy, sm_count, P, st);
    }
    if (r < 0) return r;
    // On a stream that is being captured the launches were recorded into the caller's graph and nothing ran; waiting
    // for that stream would fail and invalidate the capture.
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    G9_CU(cudaStreamIsCapturing(st, &cap));
    if (cap == cudaStreamCaptureStatusActive) return 0;
    if (!G.nowait || st == cudaStreamPerThread) {
        G9_CU(cudaStreamSynchronize(st));
    } else if (ds) {   // queued on the library's stream: later calls that read y early must know
        queued_writes_add(ds, y, vec_span(ny, incy) * (size_t)es, st);
    }
    return 0;
}
