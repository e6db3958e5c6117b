// level12x.cu -- the rest of levels 1-2: scal, copy, swap, rot, rotm, rotg, rotmg; symv, trmv, trsv, syr, syr2; and
// the banded / packed forms gbmv, sbmv, tbmv, tbsv, spmv, tpmv, tpsv, spr, spr2 (types H, S, D; HS = H).
//
// Replaces lib/src/level12.c:54-165, 267-519 and the matching kernels of lib/kernels/level12.cl (kprzybys/
// gen9-gpu-blas). Semantics kept: strided vectors with negative increments addressing the lowest element, increment 0
// an invalid argument, n <= 0 a no-op, beta = 0 never reads y, FP16 computed in FP32 and FP64 in FP64, the row-major
// band layout A(i, j) = A[i·lda + KL + j − i] (symmetric / triangular: upper KL = 0, KU = K; lower KL = K, KU = 0) and
// the packed layouts (upper row i starts at i·n − i(i−1)/2, lower row i at i(i+1)/2). B200 design:
// - level 1: one grid-stride kernel per operation on the strided vectors;
// - matrix-vector products of every layout: one kernel template, one warp per output row, each lane summing a strided
//   share of the row's nonzero range through a layout accessor (symmetric layouts read the mirrored element where the
//   row leaves the stored triangle), a fixed shuffle tree, then alpha·sum + beta·y. In-place products (trmv, tbmv,
//   tpmv) write a work vector that is copied back;
// - rank updates (syr, syr2, spr, spr2): one block per row of the stored triangle;
// - solves: trsv and tpsv run the blocked TRSM of the level-3 code with one right-hand side (tpsv after expanding the
//   packed triangle); tbsv, whose band keeps the dense form out of reach for large n, runs one CTA that walks the rows
//   in dependency order, the threads sharing each row's band dot product.
#include "common.cuh"
#include "internal.h"
#include <cmath>

namespace g9 {

namespace l2x {
enum Layout : int { kDense = 0, kBand = 1, kPacked = 2 };
enum Kind : int { kGeneral = 0, kSymmetric = 1, kTriangular = 2 };
}

// op(A) of one level-2 call: element accessor and nonzero column range of each row.
struct L2Mat {
    const void *A;
    long long lda;
    int layout, kind;
    int rows, cols;   // op(A) dimensions
    int upper, trans, unit;
    int KL, KU;       // band (general: as given; symmetric / triangular: from uplo and K)
    int n;            // order of a packed matrix
};

__device__ __forceinline__ long long packed_index(const L2Mat &m, int i, int j) {   // (i, j) inside the triangle
    return m.upper ? (long long)i * m.n - (long long)i * (i - 1) / 2 + (j - i) : (long long)i * (i + 1) / 2 + j;
}

// Stored element (i, j) of A (storage coordinates, inside the stored structure).
template <typename T> __device__ __forceinline__ typename Compute<T>::R stored(const L2Mat &m, int i, int j) {
    const T *A = (const T *)m.A;
    if (m.layout == l2x::kDense) return to_r(A[(long long)i * m.lda + j]);
    if (m.layout == l2x::kBand) return to_r(A[(long long)i * m.lda + m.KL + j - i]);
    return to_r(A[packed_index(m, i, j)]);
}

// Element (i, j) of op(A), zero outside its structure.
template <typename T> __device__ __forceinline__ typename Compute<T>::R elem(const L2Mat &m, int i, int j) {
    using R = typename Compute<T>::R;
    if (m.kind == l2x::kGeneral) {   // banded general matrix (dense general uses gen9blas_gemv)
        const int a = m.trans ? j : i, b = m.trans ? i : j;
        return (b - a >= -m.KL && b - a <= m.KU) ? stored<T>(m, a, b) : R(0);
    }
    if (m.kind == l2x::kSymmetric) {
        const bool in = m.upper ? j >= i : j <= i;
        const int a = in ? i : j, b = in ? j : i;
        if (m.layout == l2x::kBand && (b - a < -m.KL || b - a > m.KU)) return R(0);
        return stored<T>(m, a, b);
    }
    const int a = m.trans ? j : i, b = m.trans ? i : j;   // triangular: T(a, b)
    if (a == b && m.unit) return R(1);
    if (m.upper ? b < a : b > a) return R(0);
    if (m.layout == l2x::kBand && (b - a < -m.KL || b - a > m.KU)) return R(0);
    return stored<T>(m, a, b);
}

// Nonzero columns [j0, j1) of row i of op(A).
__device__ __forceinline__ void row_range(const L2Mat &m, int i, int &j0, int &j1) {
    j0 = 0;
    j1 = m.cols;
    if (m.kind == l2x::kGeneral) {   // op(A)(i, j) = A(i, j) (or A(j, i)): band offsets from the stored orientation
        const int lo = m.trans ? -m.KU : -m.KL, hi = m.trans ? m.KL : m.KU;
        j0 = max(0, i + lo);
        j1 = min(m.cols, i + hi + 1);
        return;
    }
    if (m.kind == l2x::kSymmetric) {
        if (m.layout == l2x::kBand) {
            const int k = m.KL + m.KU;
            j0 = max(0, i - k);
            j1 = min(m.cols, i + k + 1);
        }
        return;
    }
    const bool right = m.upper != (m.trans != 0);   // op(A) row i is nonzero for j >= i
    const int k = m.layout == l2x::kBand ? m.KL + m.KU : m.cols;
    if (right) { j0 = i; j1 = min(m.cols, i + k + 1); }
    else { j0 = max(0, i - k); j1 = i + 1; }
}

template <typename T> __device__ __forceinline__ T &vat(T *v, long long off, long long inc, int i) {
    return v[off + (long long)i * inc];
}

// y_i = alpha·Σ_j op(A)(i, j)·x_j + beta·y_i, one warp per row.
template <typename T>
__global__ void __launch_bounds__(256) l2x_mv(const L2Mat m, typename Compute<T>::R alpha, const T *__restrict__ x,
                                              long long ox, long long ix, typename Compute<T>::R beta, T *y,
                                              long long oy, long long iy) {
    using R = typename Compute<T>::R;
    const long long w = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (w >= m.rows) return;
    const int i = (int)w;
    int j0, j1;
    row_range(m, i, j0, j1);
    R s = 0;
    for (int j = j0 + lane; j < j1; j += 32) s = fma_r(elem<T>(m, i, j), to_r(x[ox + (long long)j * ix]), s);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) {
        T &yi = vat(y, oy, iy, i);
        yi = from_r<T>(beta == R(0) ? alpha * s : fma_r(beta, to_r(yi), alpha * s));
    }
}

// Stored triangle update: A(i, j) += alpha·(x_i·y_j + y_i·x_j) (two = 1) or alpha·x_i·x_j, one block per row.
template <typename T>
__global__ void l2x_rank(const L2Mat m, typename Compute<T>::R alpha, const T *__restrict__ x, long long ox,
                         long long ix, const T *__restrict__ y, long long oy, long long iy, int two) {
    using R = typename Compute<T>::R;
    const int i = blockIdx.x;
    T *A = (T *)const_cast<void *>(m.A);
    const R xi = to_r(x[ox + (long long)i * ix]);
    const R yi = two ? to_r(y[oy + (long long)i * iy]) : R(0);
    const int j0 = m.upper ? i : 0, j1 = m.upper ? m.n : i + 1;
    for (int j = j0 + threadIdx.x; j < j1; j += blockDim.x) {
        const R xj = to_r(x[ox + (long long)j * ix]);
        R d = xi * xj;
        if (two) d = fma_r(xi, to_r(y[oy + (long long)j * iy]), yi * xj);
        T *a = m.layout == l2x::kDense ? A + (long long)i * m.lda + j : A + packed_index(m, i, j);
        *a = from_r<T>(fma_r(alpha, d, to_r(*a)));
    }
}

// Banded triangular solve op(A)·z = b in place (x holds b), rows in dependency order, one CTA.
template <typename T>
__global__ void __launch_bounds__(256) l2x_tbsv(const L2Mat m, T *x, long long ox, long long ix) {
    using R = typename Compute<T>::R;
    __shared__ R part[8];
    const bool forward = !(m.upper != (m.trans != 0));   // op(A) lower: rows 0, 1, ...
    const int n = m.rows, k = m.KL + m.KU;
    for (int s = 0; s < n; s++) {
        const int i = forward ? s : n - 1 - s;
        const int j0 = forward ? max(0, i - k) : i + 1, j1 = forward ? i : min(n, i + k + 1);
        R acc = 0;
        for (int j = j0 + (int)threadIdx.x; j < j1; j += blockDim.x)
            acc = fma_r(elem<T>(m, i, j), to_r(x[ox + (long long)j * ix]), acc);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
        __syncthreads();
        if (threadIdx.x == 0) {
            R t = 0;
            for (int q = 0; q < (int)(blockDim.x >> 5); q++) t += part[q];
            T &xi = x[ox + (long long)i * ix];
            const R v = to_r(xi) - t;
            xi = from_r<T>(m.unit ? v : v / elem<T>(m, i, i));
        }
        __syncthreads();
    }
}

// Dense n×n matrix (pitch n) of a packed triangle, zeros outside it.
template <typename T>
__global__ void l2x_unpack(const T *__restrict__ Ap, int n, int upper, T *D) {
    const long long total = (long long)n * n;
    L2Mat m{};
    m.n = n;
    m.upper = upper;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x) {
        const int i = (int)(e / n), j = (int)(e % n);
        const bool in = upper ? j >= i : j <= i;
        D[e] = in ? Ap[packed_index(m, i, j)] : from_r<T>(0);
    }
}

// Strided copy / scal / swap / rot / rotm (mode 0..4); h = (h11, h12, h21, h22) for rotm, (c, s) for rot.
template <typename T>
__global__ void l1x(int mode, int n, T *x, long long ox, long long ix, T *y, long long oy, long long iy, double a,
                    double h11, double h12, double h21, double h22) {
    using R = typename Compute<T>::R;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
        T *px = x + ox + e * ix;
        if (mode == 1) {   // scal
            *px = from_r<T>((R)a * to_r(*px));
            continue;
        }
        T *py = y + oy + e * iy;
        if (mode == 0) {   // copy x -> y
            *py = *px;
        } else if (mode == 2) {   // swap
            const T t = *px;
            *px = *py;
            *py = t;
        } else {   // rot (h11 = h22 = c, h12 = s, h21 = -s) and rotm
            const R vx = to_r(*px), vy = to_r(*py);
            *px = from_r<T>(fma_r((R)h11, vx, (R)h12 * vy));
            *py = from_r<T>(fma_r((R)h21, vx, (R)h22 * vy));
        }
    }
}

static int l2x_grid(long long n) {
    DevState *d = dev_state();
    long long g = (n + 255) / 256, cap = (long long)(d ? d->sm_count : 148) * 16;
    return (int)(g < 1 ? 1 : g < cap ? g : cap);
}

// Work buffer of the in-place products and the solves (separate from the GEMM scratch and the level-3 buffer).
static int l2x_buffer(size_t bytes, void **p) {
    DevState *d = dev_state();
    if (!d) return G.status;
    if (d->l2x_n < bytes) {
        if (d->l2x) {
            G9_CU(cudaStreamSynchronize(stream()));
            G9_CU(cudaFree(d->l2x));
            d->l2x = nullptr;
            d->l2x_n = 0;
        }
        const size_t want = bytes < 4096 ? 4096 : (bytes + 0xFFFFF) & ~(size_t)0xFFFFF;
        G9_CU(cudaMalloc(&d->l2x, want));
        d->l2x_n = want;
    }
    *p = d->l2x;
    return 0;
}

template <typename T>
static int mv_t(const L2Mat &m, double alpha, const void *x, long long ox, long long ix, double beta, void *y,
                long long oy, long long iy, cudaStream_t st) {
    using R = typename Compute<T>::R;
    const long long threads = (long long)m.rows * 32;
    l2x_mv<T><<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(m, (R)alpha, (const T *)x, ox, ix, (R)beta, (T *)y, oy, iy);
    return launched("l2x_mv");
}

// x = op(A)·x: the product into a contiguous work vector, then copied over x.
template <typename T>
static int mv_inplace_t(const L2Mat &m, void *x, long long ox, long long ix, cudaStream_t st) {
    void *wv = nullptr;
    G9_TRY(l2x_buffer((size_t)m.rows * sizeof(T), &wv));
    G9_TRY(mv_t<T>(m, 1.0, x, ox, ix, 0.0, wv, 0, 1, st));
    l1x<T><<<l2x_grid(m.rows), 256, 0, st>>>(0, m.rows, (T *)wv, 0, 1, (T *)x, ox, ix, 0, 0, 0, 0, 0);
    return launched("l1x_copy");
}

// Dense triangular solve with one right-hand side through the level-3 TRSM (contiguous copy of x in and out).
template <typename T>
static int trsv_dense_t(int type, int upper, int trans, int unit, int n, const void *A, int lda, void *x, long long ox,
                        long long ix, void *work, cudaStream_t st) {
    T *b = (T *)work;
    l1x<T><<<l2x_grid(n), 256, 0, st>>>(0, n, (T *)x, ox, ix, b, 0, 1, 0, 0, 0, 0, 0);
    G9_TRY(launched("l1x_copy"));
    G9_TRY(launch_trsm_dev(type, 1, upper, trans, unit, n, 1, 1.0, A, lda, b, 1, st));
    l1x<T><<<l2x_grid(n), 256, 0, st>>>(0, n, b, 0, 1, (T *)x, ox, ix, 0, 0, 0, 0, 0);
    return launched("l1x_copy");
}

}  // namespace g9

using namespace g9;

namespace {

int es_of(int type) {
    return type == GEN9BLAS_S ? 4 : type == GEN9BLAS_D ? 8 : (type == GEN9BLAS_H || type == GEN9BLAS_HS) ? 2 : 0;
}
int base_type(int type) { return type == GEN9BLAS_HS ? GEN9BLAS_H : type; }

#define L2X_BEGIN(n, bad_inc)                                                                       \
    if (int e_ = begin_op()) return e_;                                                             \
    const int es = es_of(type);                                                                     \
    if (!es) return fail(GEN9BLAS_ERR_UNSUPPORTED, "type %d unavailable", type);                    \
    type = base_type(type);                                                                         \
    if ((n) <= 0) return 0;                                                                         \
    if (bad_inc) return fail(GEN9BLAS_ERR_INVALID_ARG, "vector increment 0");

#define L2X_DISPATCH(FN, ...)                                                                       \
    (type == GEN9BLAS_S ? FN<float>(__VA_ARGS__) : type == GEN9BLAS_D ? FN<double>(__VA_ARGS__)     \
                                                 : FN<__half>(__VA_ARGS__))

// Bytes of each stored form.
size_t dense_bytes(int rows, int cols, int ld, int es) { return ((size_t)(rows - 1) * ld + cols) * es; }
size_t packed_bytes(int n, int es) { return (size_t)n * (n + 1) / 2 * es; }

L2Mat mat(const void *A, long long lda, int layout, int kind, int rows, int cols, int upper, int trans, int unit, int KL,
          int KU, int n) {
    L2Mat m;
    m.A = A; m.lda = lda; m.layout = layout; m.kind = kind; m.rows = rows; m.cols = cols;
    m.upper = upper; m.trans = trans; m.unit = unit; m.KL = KL; m.KU = KU; m.n = n;
    return m;
}

// Level 1: mode 0 copy (x -> y), 1 scal, 2 swap, 3 rot, 4 rotm.
int l1x_call(int mode, int type, int n, void *x, int incx, void *y, int incy, double a, double h11, double h12,
             double h21, double h22) {
    const bool two = mode != 1;
    L2X_BEGIN(n, !incx || (two && !incy));
    timer_start();
    Operand op[2];
    G9_TRY(map_operand(op[0], x, vec_span(n, incx) * es, 0, true, mode != 0));
    if (two) G9_TRY(map_operand(op[1], y, vec_span(n, incy) * es, 1, mode != 0 || (incy != 1 && incy != -1), true));
    timer_kernel();
    const long long ox = vec_off(n, incx), oy = two ? vec_off(n, incy) : 0;
    cudaStream_t st = stream();
#define G9_L1X(TT)                                                                                                  \
    l1x<TT><<<l2x_grid(n), 256, 0, st>>>(mode, n, (TT *)op[0].dptr, ox, incx, two ? (TT *)op[1].dptr : nullptr, oy, \
                                         incy, a, h11, h12, h21, h22)
    if (type == GEN9BLAS_S) G9_L1X(float);
    else if (type == GEN9BLAS_D) G9_L1X(double);
    else G9_L1X(__half);
#undef G9_L1X
    G9_TRY(launched("l1x"));
    G.last_zc = op[0].zc | (two ? op[1].zc << 1 : 0);
    int r = finish_op(op, two ? 2 : 1);
    timer_stop();
    return r;
}

// y = alpha·op(A)·x + beta·y for a described matrix (A region of `abytes` bytes).
int mv_call(int type, int es, L2Mat m, size_t abytes, double alpha, const void *x, int incx, double beta, void *y,
            int incy) {
    timer_start();
    Operand op[3];
    G9_TRY(map_operand(op[0], m.A, abytes, 0, true, false));
    G9_TRY(map_operand(op[1], x, vec_span(m.cols, incx) * es, 1, true, false));
    G9_TRY(map_operand(op[2], y, vec_span(m.rows, incy) * es, 2, beta != 0.0 || (incy != 1 && incy != -1), true));
    timer_kernel();
    m.A = op[0].dptr;
    G9_TRY(L2X_DISPATCH(mv_t, m, alpha, op[1].dptr, vec_off(m.cols, incx), incx, beta, op[2].dptr, vec_off(m.rows, incy),
                        incy, stream()));
    G.last_zc = op[0].zc | op[1].zc << 1 | op[2].zc << 2;
    int r = finish_op(op, 3);
    timer_stop();
    return r;
}

// x = op(A)·x in place.
int mv_inplace_call(int type, int es, L2Mat m, size_t abytes, void *x, int incx) {
    timer_start();
    Operand op[2];
    G9_TRY(map_operand(op[0], m.A, abytes, 0, true, false));
    G9_TRY(map_operand(op[1], x, vec_span(m.rows, incx) * es, 1, true, true));
    timer_kernel();
    m.A = op[0].dptr;
    G9_TRY(L2X_DISPATCH(mv_inplace_t, m, op[1].dptr, vec_off(m.rows, incx), incx, stream()));
    G.last_zc = op[0].zc | op[1].zc << 1;
    int r = finish_op(op, 2);
    timer_stop();
    return r;
}

// Stored-triangle rank update.
int rank_call(int type, int es, L2Mat m, size_t abytes, double alpha, const void *x, int incx, const void *y, int incy,
              int two) {
    timer_start();
    Operand op[3];
    G9_TRY(map_operand(op[0], x, vec_span(m.n, incx) * es, 0, true, false));
    if (two) G9_TRY(map_operand(op[1], y, vec_span(m.n, incy) * es, 1, true, false));
    G9_TRY(map_operand(op[2], m.A, abytes, 2, true, true));
    timer_kernel();
    m.A = op[2].dptr;
    const long long ox = vec_off(m.n, incx), oy = two ? vec_off(m.n, incy) : 0;
    cudaStream_t st = stream();
#define G9_RANK(TT)                                                                                               \
    l2x_rank<TT><<<m.n, 256, 0, st>>>(m, (Compute<TT>::R)alpha, (const TT *)op[0].dptr, ox, incx,                 \
                                      two ? (const TT *)op[1].dptr : (const TT *)op[0].dptr, oy, two ? incy : incx, two)
    if (type == GEN9BLAS_S) G9_RANK(float);
    else if (type == GEN9BLAS_D) G9_RANK(double);
    else G9_RANK(__half);
#undef G9_RANK
    G9_TRY(launched("l2x_rank"));
    int r = finish_op(op, 3);   // op[1] stays an unmapped, in-place entry without y
    timer_stop();
    return r;
}

}  // namespace

extern "C" {

// ---------------------------------------------------------------- level 1
GEN9BLAS_API int gen9blas_scal(int type, int n, double a, void *x, int incx) {
    return l1x_call(1, type, n, x, incx, nullptr, 1, a, 0, 0, 0, 0);
}
GEN9BLAS_API int gen9blas_copy(int type, int n, const void *x, int incx, void *y, int incy) {
    return l1x_call(0, type, n, const_cast<void *>(x), incx, y, incy, 0, 0, 0, 0, 0);
}
GEN9BLAS_API int gen9blas_swap(int type, int n, void *x, int incx, void *y, int incy) {
    return l1x_call(2, type, n, x, incx, y, incy, 0, 0, 0, 0, 0);
}
GEN9BLAS_API int gen9blas_rot(int type, int n, void *x, int incx, void *y, int incy, double c, double s) {
    return l1x_call(3, type, n, x, incx, y, incy, 0, c, s, -s, c);
}
// param: flag, h11, h21, h12, h22 (BLAS order). flag -2: identity; -1: full H; 0: unit diagonal; 1: h21 = -1, h12 = 1.
GEN9BLAS_API int gen9blas_rotm(int type, int n, void *x, int incx, void *y, int incy, const double *param) {
    if (!param) {
        if (int e = begin_op()) return e;
        return fail(GEN9BLAS_ERR_INVALID_ARG, "NULL param");
    }
    const double flag = param[0];
    if (flag == -2.0) {
        if (int e = begin_op()) return e;
        return 0;
    }
    double h11, h12, h21, h22;
    if (flag < 0) { h11 = param[1]; h21 = param[2]; h12 = param[3]; h22 = param[4]; }
    else if (flag == 0) { h11 = 1; h21 = param[2]; h12 = param[3]; h22 = 1; }
    else { h11 = param[1]; h21 = -1; h12 = 1; h22 = param[4]; }
    return l1x_call(4, type, n, x, incx, y, incy, 0, h11, h12, h21, h22);
}

// Givens rotation parameters on the CPU (a few scalars): [c s; -s c]·[a; b] = [r; 0]; a <- r, b <- z with z encoding
// (c, s) as in BLAS. The overflow-safe form of the published algorithm (LAPACK 3.10 reference BLAS srotg): scale by
// max(|a|, |b|) clamped to the normal range, the sign of r taken from the larger of a and b.
GEN9BLAS_API void gen9blas_rotg(float *a, float *b, float *c, float *s) {
    if (!a || !b || !c || !s) return;
    const float tiny = 1.17549435e-38f;   // smallest normal float
    const float x = *a, y = *b, ax = fabsf(x), ay = fabsf(y);
    if (ay == 0.0f) {
        *c = 1.0f;
        *s = 0.0f;
        *b = 0.0f;
        return;
    }
    if (ax == 0.0f) {
        *c = 0.0f;
        *s = 1.0f;
        *a = y;
        *b = 1.0f;
        return;
    }
    float scale = ax > ay ? ax : ay;
    if (scale < tiny) scale = tiny;
    if (scale > 1.0f / tiny) scale = 1.0f / tiny;
    const float xs = x / scale, ys = y / scale;
    const float sign = ax > ay ? copysignf(1.0f, x) : copysignf(1.0f, y);
    const float r = sign * scale * sqrtf(xs * xs + ys * ys);
    *c = x / r;
    *s = y / r;
    *a = r;
    *b = ax > ay ? *s : (*c != 0.0f ? 1.0f / *c : 1.0f);
}

// Modified Givens rotation parameters on the CPU (the published algorithm of Lawson, Hanson, Kincaid and Krogh as in
// the reference BLAS srotmg): d1, d2 squared scale factors, (x1, y1) the vector; on return param = (flag, h11, h21,
// h12, h22) with the entries the flag implies, d1, d2, x1 updated. Rescaling keeps d1, d2 within [2^-24, 2^24] by
// steps of 4096.
GEN9BLAS_API void gen9blas_rotmg(float *d1, float *d2, float *x1, float y1, float *param) {
    if (!d1 || !d2 || !x1 || !param) return;
    const float g = 4096.0f, g2 = g * g, lo = 1.0f / g2, hi = g2;
    float flag, h11 = 0.0f, h12 = 0.0f, h21 = 0.0f, h22 = 0.0f;
    auto zero_all = [&]() {
        flag = -1.0f;
        h11 = h12 = h21 = h22 = 0.0f;
        *d1 = *d2 = *x1 = 0.0f;
    };
    if (*d1 < 0.0f) {
        zero_all();
    } else {
        const float p2 = *d2 * y1;
        if (p2 == 0.0f) {
            param[0] = -2.0f;
            return;
        }
        const float p1 = *d1 * *x1, q2 = p2 * y1, q1 = p1 * *x1;
        if (fabsf(q1) > fabsf(q2)) {
            h21 = -y1 / *x1;
            h12 = p2 / p1;
            const float u = 1.0f - h12 * h21;
            if (u > 0.0f) {
                flag = 0.0f;
                *d1 /= u;
                *d2 /= u;
                *x1 *= u;
            } else {
                zero_all();
            }
        } else if (q2 < 0.0f) {
            zero_all();
        } else {
            flag = 1.0f;
            h11 = p1 / p2;
            h22 = *x1 / y1;
            const float u = 1.0f + h11 * h22, t = *d2 / u;
            *d2 = *d1 / u;
            *d1 = t;
            *x1 = y1 * u;
        }
        // Rescale d1 (with x1, h11, h12) and d2 (with h21, h22) into [lo, hi]; any rescale makes H a full matrix.
        auto to_full = [&]() {
            if (flag == 0.0f) { h11 = 1.0f; h22 = 1.0f; }
            else if (flag > 0.0f) { h21 = -1.0f; h12 = 1.0f; }
            flag = -1.0f;
        };
        if (*d1 != 0.0f) {
            while (*d1 <= lo || *d1 >= hi) {
                to_full();
                if (*d1 <= lo) { *d1 *= g2; *x1 /= g; h11 /= g; h12 /= g; }
                else { *d1 /= g2; *x1 *= g; h11 *= g; h12 *= g; }
            }
        }
        if (*d2 != 0.0f) {
            while (fabsf(*d2) <= lo || fabsf(*d2) >= hi) {
                to_full();
                if (fabsf(*d2) <= lo) { *d2 *= g2; h21 /= g; h22 /= g; }
                else { *d2 /= g2; h21 *= g; h22 *= g; }
            }
        }
    }
    if (flag < 0.0f) { param[1] = h11; param[2] = h21; param[3] = h12; param[4] = h22; }
    else if (flag == 0.0f) { param[2] = h21; param[3] = h12; }
    else { param[1] = h11; param[4] = h22; }
    param[0] = flag;
}

// ---------------------------------------------------------------- dense level 2
GEN9BLAS_API int gen9blas_symv(int type, int uplo, int n, double alpha, const void *A, int lda, const void *x, int incx,
                               double beta, void *y, int incy) {
    L2X_BEGIN(n, !incx || !incy);
    if (lda < n) return fail(GEN9BLAS_ERR_INVALID_ARG, "lda < n");
    const L2Mat m = mat(A, lda, l2x::kDense, l2x::kSymmetric, n, n, uplo == GEN9BLAS_UPPER, 0, 0, 0, 0, n);
    return mv_call(type, es, m, dense_bytes(n, n, lda, es), alpha, x, incx, beta, y, incy);
}

GEN9BLAS_API int gen9blas_trmv(int type, int uplo, int trans, int diag, int n, const void *A, int lda, void *x, int incx) {
    L2X_BEGIN(n, !incx);
    if (lda < n) return fail(GEN9BLAS_ERR_INVALID_ARG, "lda < n");
    const L2Mat m = mat(A, lda, l2x::kDense, l2x::kTriangular, n, n, uplo == GEN9BLAS_UPPER, trans ? 1 : 0,
                        diag == GEN9BLAS_UNIT, 0, 0, n);
    return mv_inplace_call(type, es, m, dense_bytes(n, n, lda, es), x, incx);
}

GEN9BLAS_API int gen9blas_trsv(int type, int uplo, int trans, int diag, int n, const void *A, int lda, void *x, int incx) {
    L2X_BEGIN(n, !incx);
    if (lda < n) return fail(GEN9BLAS_ERR_INVALID_ARG, "lda < n");
    timer_start();
    Operand op[2];
    G9_TRY(map_operand(op[0], A, dense_bytes(n, n, lda, es), 0, true, false));
    G9_TRY(map_operand(op[1], x, vec_span(n, incx) * es, 1, true, true));
    void *work = nullptr;
    G9_TRY(l2x_buffer((size_t)n * es, &work));
    timer_kernel();
    G9_TRY(L2X_DISPATCH(trsv_dense_t, type, uplo == GEN9BLAS_UPPER, trans ? 1 : 0, diag == GEN9BLAS_UNIT, n, op[0].dptr,
                        lda, op[1].dptr, vec_off(n, incx), incx, work, stream()));
    G.last_zc = op[0].zc | op[1].zc << 1;
    int r = finish_op(op, 2);
    timer_stop();
    return r;
}

GEN9BLAS_API int gen9blas_syr(int type, int uplo, int n, double alpha, const void *x, int incx, void *A, int lda) {
    L2X_BEGIN(n, !incx);
    if (lda < n) return fail(GEN9BLAS_ERR_INVALID_ARG, "lda < n");
    const L2Mat m = mat(A, lda, l2x::kDense, l2x::kSymmetric, n, n, uplo == GEN9BLAS_UPPER, 0, 0, 0, 0, n);
    return rank_call(type, es, m, dense_bytes(n, n, lda, es), alpha, x, incx, nullptr, 1, 0);
}

GEN9BLAS_API int gen9blas_syr2(int type, int uplo, int n, double alpha, const void *x, int incx, const void *y, int incy,
                               void *A, int lda) {
    L2X_BEGIN(n, !incx || !incy);
    if (lda < n) return fail(GEN9BLAS_ERR_INVALID_ARG, "lda < n");
    const L2Mat m = mat(A, lda, l2x::kDense, l2x::kSymmetric, n, n, uplo == GEN9BLAS_UPPER, 0, 0, 0, 0, n);
    return rank_call(type, es, m, dense_bytes(n, n, lda, es), alpha, x, incx, y, incy, 1);
}

// ---------------------------------------------------------------- banded
GEN9BLAS_API int gen9blas_gbmv(int type, int trans, int M, int N, int KL, int KU, double alpha, const void *A, int lda,
                               const void *x, int incx, double beta, void *y, int incy) {
    L2X_BEGIN(M < N ? M : N, !incx || !incy);
    if (KL < 0 || KU < 0 || lda < KL + KU + 1) return fail(GEN9BLAS_ERR_INVALID_ARG, "gbmv: KL, KU or lda");
    const int tr = trans ? 1 : 0;
    const L2Mat m = mat(A, lda, l2x::kBand, l2x::kGeneral, tr ? N : M, tr ? M : N, 0, tr, 0, KL, KU, 0);
    return mv_call(type, es, m, dense_bytes(M, KL + KU + 1, lda, es), alpha, x, incx, beta, y, incy);
}

GEN9BLAS_API int gen9blas_sbmv(int type, int uplo, int N, int K, double alpha, const void *A, int lda, const void *x,
                               int incx, double beta, void *y, int incy) {
    L2X_BEGIN(N, !incx || !incy);
    if (K < 0 || lda < K + 1) return fail(GEN9BLAS_ERR_INVALID_ARG, "sbmv: K or lda");
    const int up = uplo == GEN9BLAS_UPPER;
    const L2Mat m = mat(A, lda, l2x::kBand, l2x::kSymmetric, N, N, up, 0, 0, up ? 0 : K, up ? K : 0, N);
    return mv_call(type, es, m, dense_bytes(N, K + 1, lda, es), alpha, x, incx, beta, y, incy);
}

GEN9BLAS_API int gen9blas_tbmv(int type, int uplo, int trans, int diag, int N, int K, const void *A, int lda, void *x,
                               int incx) {
    L2X_BEGIN(N, !incx);
    if (K < 0 || lda < K + 1) return fail(GEN9BLAS_ERR_INVALID_ARG, "tbmv: K or lda");
    const int up = uplo == GEN9BLAS_UPPER;
    const L2Mat m = mat(A, lda, l2x::kBand, l2x::kTriangular, N, N, up, trans ? 1 : 0, diag == GEN9BLAS_UNIT,
                        up ? 0 : K, up ? K : 0, N);
    return mv_inplace_call(type, es, m, dense_bytes(N, K + 1, lda, es), x, incx);
}

GEN9BLAS_API int gen9blas_tbsv(int type, int uplo, int trans, int diag, int N, int K, const void *A, int lda, void *x,
                               int incx) {
    L2X_BEGIN(N, !incx);
    if (K < 0 || lda < K + 1) return fail(GEN9BLAS_ERR_INVALID_ARG, "tbsv: K or lda");
    const int up = uplo == GEN9BLAS_UPPER;
    L2Mat m = mat(A, lda, l2x::kBand, l2x::kTriangular, N, N, up, trans ? 1 : 0, diag == GEN9BLAS_UNIT, up ? 0 : K,
                  up ? K : 0, N);
    timer_start();
    Operand op[2];
    G9_TRY(map_operand(op[0], A, dense_bytes(N, K + 1, lda, es), 0, true, false));
    G9_TRY(map_operand(op[1], x, vec_span(N, incx) * es, 1, true, true));
    timer_kernel();
    m.A = op[0].dptr;
    const long long ox = vec_off(N, incx);
    cudaStream_t st = stream();
    if (type == GEN9BLAS_S) l2x_tbsv<float><<<1, 256, 0, st>>>(m, (float *)op[1].dptr, ox, incx);
    else if (type == GEN9BLAS_D) l2x_tbsv<double><<<1, 256, 0, st>>>(m, (double *)op[1].dptr, ox, incx);
    else l2x_tbsv<__half><<<1, 256, 0, st>>>(m, (__half *)op[1].dptr, ox, incx);
    G9_TRY(launched("l2x_tbsv"));
    G.last_zc = op[0].zc | op[1].zc << 1;
    int r = finish_op(op, 2);
    timer_stop();
    return r;
}

// ---------------------------------------------------------------- packed
GEN9BLAS_API int gen9blas_spmv(int type, int uplo, int N, double alpha, const void *Ap, const void *x, int incx,
                               double beta, void *y, int incy) {
    L2X_BEGIN(N, !incx || !incy);
    const L2Mat m = mat(Ap, 0, l2x::kPacked, l2x::kSymmetric, N, N, uplo == GEN9BLAS_UPPER, 0, 0, 0, 0, N);
    return mv_call(type, es, m, packed_bytes(N, es), alpha, x, incx, beta, y, incy);
}

GEN9BLAS_API int gen9blas_tpmv(int type, int uplo, int trans, int diag, int N, const void *Ap, void *x, int incx) {
    L2X_BEGIN(N, !incx);
    const L2Mat m = mat(Ap, 0, l2x::kPacked, l2x::kTriangular, N, N, uplo == GEN9BLAS_UPPER, trans ? 1 : 0,
                        diag == GEN9BLAS_UNIT, 0, 0, N);
    return mv_inplace_call(type, es, m, packed_bytes(N, es), x, incx);
}

GEN9BLAS_API int gen9blas_tpsv(int type, int uplo, int trans, int diag, int N, const void *Ap, void *x, int incx) {
    L2X_BEGIN(N, !incx);
    timer_start();
    Operand op[2];
    G9_TRY(map_operand(op[0], Ap, packed_bytes(N, es), 0, true, false));
    G9_TRY(map_operand(op[1], x, vec_span(N, incx) * es, 1, true, true));
    void *work = nullptr;   // [dense triangle N×N | contiguous right-hand side]
    const size_t dbytes = ((size_t)N * N * es + 255) / 256 * 256;
    G9_TRY(l2x_buffer(dbytes + (size_t)N * es, &work));
    timer_kernel();
    cudaStream_t st = stream();
    const int up = uplo == GEN9BLAS_UPPER;
    void *rhs = (char *)work + dbytes;
#define G9_TPSV(TT)                                                                                                   \
    do {                                                                                                              \
        l2x_unpack<TT><<<l2x_grid((long long)N * N), 256, 0, st>>>((const TT *)op[0].dptr, N, up, (TT *)work);        \
        G9_TRY(launched("l2x_unpack"));                                                                                \
        G9_TRY(trsv_dense_t<TT>(type, up, trans ? 1 : 0, diag == GEN9BLAS_UNIT, N, work, N, op[1].dptr,               \
                                vec_off(N, incx), incx, rhs, st));                                                    \
    } while (0)
    if (type == GEN9BLAS_S) G9_TPSV(float);
    else if (type == GEN9BLAS_D) G9_TPSV(double);
    else G9_TPSV(__half);
#undef G9_TPSV
    G.last_zc = op[0].zc | op[1].zc << 1;
    int r = finish_op(op, 2);
    timer_stop();
    return r;
}

GEN9BLAS_API int gen9blas_spr(int type, int uplo, int N, double alpha, const void *x, int incx, void *Ap) {
    L2X_BEGIN(N, !incx);
    const L2Mat m = mat(Ap, 0, l2x::kPacked, l2x::kSymmetric, N, N, uplo == GEN9BLAS_UPPER, 0, 0, 0, 0, N);
    return rank_call(type, es, m, packed_bytes(N, es), alpha, x, incx, nullptr, 1, 0);
}

GEN9BLAS_API int gen9blas_spr2(int type, int uplo, int N, double alpha, const void *x, int incx, const void *y, int incy,
                               void *Ap) {
    L2X_BEGIN(N, !incx || !incy);
    const L2Mat m = mat(Ap, 0, l2x::kPacked, l2x::kSymmetric, N, N, uplo == GEN9BLAS_UPPER, 0, 0, 0, 0, N);
    return rank_call(type, es, m, packed_bytes(N, es), alpha, x, incx, y, incy, 1);
}

}  // extern "C"
