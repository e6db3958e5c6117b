// level3.cu -- level-3 BLAS on the GEMM kernels: SYMM, SYRK, SYR2K, TRMM, TRSM (all four types).
//
// Replaces the reference's lib/src/level3.c:1-215 (kprzybys/gen9-gpu-blas), whose approach is kept: every operation
// becomes GEMMs on full matrices that small kernels build on the device, with triangular shapes cut into row (or
// column) bands so that each band's GEMM only runs over the nonzero range of K (5/8 of the square's work with 4
// bands).
// - SYMM: the symmetric matrix is expanded from its uplo triangle, then one GEMM writes alpha·F·B + beta·C (or B·F).
// - TRMM: the triangular op(A) is expanded (zeros outside, unit diagonal on request), banded GEMMs write alpha·F·B
//   (or B·F) into a work matrix, which is copied over B.
// - SYRK / SYR2K: banded GEMMs of op(A)·op(A)ᵀ (SYR2K: op(A)·op(B)ᵀ, then + op(B)·op(A)ᵀ) into a work matrix; an
//   epilogue writes alpha·P + beta·C on the uplo triangle only (the other triangle of C is not touched).
// - TRSM: reduced to a lower-triangular left solve L·Z = alpha·R (an upper triangle by reversing the index order, the
//   right side by transposition, as the reference does); inverses of the 128×128 diagonal blocks of L are computed in
//   FP64 on the GPU (forward substitution, one CTA per block) and stored in the element type (FP32 / FP64 also compose
//   them into 256- and 512-row inverses with small batched GEMMs); then a recursive halving solve: the top half, one
//   GEMM Y[bottom] -= L[bottom, top]·Y[top] with K = half the range, the bottom half, down to leaves
//   Y_i = inv(L_ii)·Y_i; finally Z is written back into B.
// The work matrices live in a level-3 buffer of their own (the GEMMs use the general scratch buffer).
#include "common.cuh"
#include "internal.h"

namespace g9 {

namespace l3 {
constexpr int kBand = 64;    // band widths are multiples of 64
constexpr int kTrsmNb = 128; // TRSM diagonal block
}

static int elem_bytes(int type) { return type == GEN9BLAS_S ? 4 : type == GEN9BLAS_D ? 8 : 2; }

static int l3_buffer(size_t bytes, void **p) {
    DevState *d = dev_state();
    if (!d) return G.status;
    if (d->l3_n < bytes) {
        if (d->l3) {
            G9_CU(cudaStreamSynchronize(stream()));
            G9_CU(cudaFree(d->l3));
            d->l3 = nullptr;
            d->l3_n = 0;
        }
        const size_t want = (bytes + 0xFFFFF) & ~(size_t)0xFFFFF;
        G9_CU(cudaMalloc(&d->l3, want));
        d->l3_n = want;
    }
    *p = d->l3;
    return 0;
}

// F (n×n, dense, pitch n) from the uplo triangle of A: sym = 1 mirrors the triangle; sym = 0 keeps zeros outside it
// (unit = 1: ones on the diagonal, the diagonal of A is not read); tr = 1 stores the transpose.
template <typename T>
__global__ void l3_expand(const T *__restrict__ A, long long lda, int n, int upper, int sym, int unit, int tr, T *F) {
    const long long total = (long long)n * n;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x) {
        const int i = (int)(e / n), j = (int)(e % n);
        const int r = tr ? j : i, c = tr ? i : j;   // F[i][j] = M[r][c]
        const bool in_tri = upper ? c >= r : c <= r;
        T v;
        if (r == c) v = unit ? from_r<T>(1) : A[(long long)r * lda + c];
        else if (in_tri) v = A[(long long)r * lda + c];
        else v = sym ? A[(long long)c * lda + r] : from_r<T>(0);
        F[e] = v;
    }
}

// C[i][j] = alpha·P[i][j] + beta·C[i][j] on the uplo triangle of the N×N matrix C (beta = 0: C is not read).
template <typename T>
__global__ void l3_tri_epilogue(int N, int upper, typename Compute<T>::R alpha, typename Compute<T>::R beta,
                                const T *__restrict__ P, T *C, long long ldc) {
    using R = typename Compute<T>::R;
    const long long total = (long long)N * N;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x) {
        const int i = (int)(e / N), j = (int)(e % N);
        if (upper ? j < i : j > i) continue;
        T *c = C + (long long)i * ldc + j;
        const R v = alpha * to_r(P[e]);
        *c = from_r<T>(beta == R(0) ? v : fma_r(beta, to_r(*c), v));
    }
}

// ---- TRSM: canonical lower-left form L·Z = alpha·R ----
// Index map r(x) = rev ? n-1-x : x. L[i][j] = op(A)'[r(i)][r(j)] for j <= i (op(A)' = tr ? Aᵀ : A), zero above the
// diagonal, unit = 1: ones on the diagonal.
template <typename T>
__global__ void trsm_build_L(const T *__restrict__ A, long long lda, int n, int tr, int unit, int rev, T *L) {
    const long long total = (long long)n * n;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x) {
        const int i = (int)(e / n), j = (int)(e % n);
        T v = from_r<T>(0);
        if (j == i && unit) {
            v = from_r<T>(1);
        } else if (j <= i) {
            const int a = rev ? n - 1 - i : i, b = rev ? n - 1 - j : j;
            v = tr ? A[(long long)b * lda + a] : A[(long long)a * lda + b];
        }
        L[e] = v;
    }
}

// Y[i][c] = alpha·R[r(i)][c] (n × m, pitch m); R = B (left, n = M) or Bᵀ (right, n = N).
template <typename T>
__global__ void trsm_build_Y(const T *__restrict__ B, long long ldb, int n, int m, int left, int rev,
                             typename Compute<T>::R alpha, T *Y) {
    const long long total = (long long)n * m;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x) {
        const int i = (int)(e / m), c = (int)(e % m);
        const int a = rev ? n - 1 - i : i;
        const T b = left ? B[(long long)a * ldb + c] : B[(long long)c * ldb + a];
        Y[e] = from_r<T>(alpha * to_r(b));
    }
}

// B[r(i)][c] (left) or B[c][r(i)] (right) = Z[i][c].
template <typename T>
__global__ void trsm_write(const T *__restrict__ Z, int n, int m, int left, int rev, T *B, long long ldb) {
    const long long total = (long long)n * m;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x) {
        const int i = (int)(e / m), c = (int)(e % m);
        const int a = rev ? n - 1 - i : i;
        if (left) B[(long long)a * ldb + c] = Z[e];
        else B[(long long)c * ldb + a] = Z[e];
    }
}

// Inverse of each diagonal block L_bb (b = min(nb, n - bb·nb)) by forward substitution in FP64: thread j solves
// L_bb·x = e_j (x kept in shared memory, column j), Inv[bb] = (x rounded to T), zeros above the diagonal.
template <typename T>
__global__ void __launch_bounds__(l3::kTrsmNb) trsm_block_inverse(const T *__restrict__ L, int n, T *Inv) {
    constexpr int NB = l3::kTrsmNb;
    extern __shared__ double xs[];   // [NB][NB]: xs[i * NB + j] = x_j[i]
    const int bb = blockIdx.x, i0 = bb * NB, b = min(NB, n - i0), j = threadIdx.x;
    const T *Lb = L + (long long)i0 * n + i0;
    if (j < b) {
        for (int i = 0; i < b; i++) {
            double s = i == j ? 1.0 : 0.0;
            if (i > j) {
                for (int k = j; k < i; k++) s -= (double)to_r(Lb[(long long)i * n + k]) * xs[k * NB + j];
            }
            xs[i * NB + j] = i < j ? 0.0 : s / (double)to_r(Lb[(long long)i * n + i]);
        }
    }
    T *out = Inv + (long long)bb * NB * NB;
    for (int i = 0; i < NB; i++) {
        const double v = (j < b && i < b) ? xs[i * NB + j] : 0.0;
        out[i * NB + j] = from_r<T>((typename Compute<T>::R)v);
    }
}

// Composed inverse of a 2s × 2s diagonal block from the inverses I0, I1 of its two s × s halves and X = -I1·L10·I0
// (already in place at rows s..2s-1, columns 0..s-1 of the output): copies I0 and I1 in and zeroes the upper right.
// One CTA column per pair p (blockIdx.y).
template <typename T>
__global__ void trsm_compose(const T *__restrict__ Inv, int s, T *Out) {
    const int p = blockIdx.y;
    const T *I0 = Inv + (long long)(2 * p) * s * s, *I1 = I0 + (long long)s * s;
    T *o = Out + (long long)p * 4 * s * s;
    const long long total = (long long)s * s;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x) {
        const int i = (int)(e / s), j = (int)(e % s);
        o[(long long)i * 2 * s + j] = I0[e];
        o[(long long)i * 2 * s + s + j] = from_r<T>(0);
        o[(long long)(s + i) * 2 * s + s + j] = I1[e];
    }
}

static int grid_elems(long long n) {
    DevState *d = dev_state();
    long long g = (n + 255) / 256, cap = (long long)(d ? d->sm_count : 148) * 8;
    return (int)(g < 1 ? 1 : g < cap ? g : cap);
}

// Bands of a triangular product: p bands compute (p + 1) / (2p) of the full square's work. Measured on B200 at
// n = 4096: 8 bands are slower than 4 for SYRK (the narrower band GEMMs lose more than the saved work).
static int bands_of(int n) { return n >= 512 ? 4 : 1; }
static int band_width(int n, int p) { return ((n + p - 1) / p + l3::kBand - 1) / l3::kBand * l3::kBand; }

// ---- host flows on device pointers ----
template <typename T>
static int symm_t(int type, int left, int upper, int M, int N, double alpha, const T *A, int lda, const T *B, int ldb,
                  double beta, T *C, int ldc, cudaStream_t st) {
    const int n = left ? M : N;
    void *buf = nullptr;
    G9_TRY(l3_buffer((size_t)n * n * sizeof(T), &buf));
    T *F = (T *)buf;
    l3_expand<T><<<grid_elems((long long)n * n), 256, 0, st>>>(A, lda, n, upper, 1, 0, 0, F);
    G9_TRY(launched("l3_expand"));
    if (left) return launch_gemm(type, 0, 0, M, N, M, alpha, F, n, 0, B, ldb, 0, beta, C, ldc, 0, 1, st);
    return launch_gemm(type, 0, 0, M, N, N, alpha, B, ldb, 0, F, n, 0, beta, C, ldc, 0, 1, st);
}

template <typename T>
static int trmm_t(int type, int left, int upper, int tA, int unit, int M, int N, double alpha, const T *A, int lda,
                  T *B, int ldb, cudaStream_t st) {
    const int n = left ? M : N;
    const bool lower = !upper != (tA != 0);   // triangle of F = op(A)
    void *buf = nullptr;
    G9_TRY(l3_buffer((size_t)n * n * sizeof(T) + (size_t)M * N * sizeof(T) + 256, &buf));
    T *F = (T *)buf;
    T *P = (T *)((char *)buf + ((size_t)n * n * sizeof(T) + 255) / 256 * 256);
    l3_expand<T><<<grid_elems((long long)n * n), 256, 0, st>>>(A, lda, n, upper, 0, unit, tA, F);
    G9_TRY(launched("l3_expand"));
    const int p = bands_of(n), w = band_width(n, p);
    for (int i0 = 0; i0 < n; i0 += w) {
        const int b = n - i0 < w ? n - i0 : w;
        if (left) {   // rows i0..i0+b of P: k over the nonzero columns of F's rows
            const int k0 = lower ? 0 : i0, k1 = lower ? i0 + b : n;
            G9_TRY(launch_gemm(type, 0, 0, b, N, k1 - k0, alpha, F + (long long)i0 * n + k0, n, 0, B + (long long)k0 * ldb,
                               ldb, 0, 0.0, P + (long long)i0 * N, N, 0, 1, st));
        } else {      // columns i0..i0+b of P: k over the nonzero rows of F's columns
            const int k0 = lower ? i0 : 0, k1 = lower ? n : i0 + b;
            G9_TRY(launch_gemm(type, 0, 0, M, b, k1 - k0, alpha, B + k0, ldb, 0, F + (long long)k0 * n + i0, n, 0, 0.0,
                               P + i0, N, 0, 1, st));
        }
    }
    G9_CU(cudaMemcpy2DAsync(B, (size_t)ldb * sizeof(T), P, (size_t)N * sizeof(T), (size_t)N * sizeof(T), M,
                            cudaMemcpyDeviceToDevice, st));
    return 0;
}

// P (N × N, pitch N) on the bands that cover the uplo triangle: P[rows, cols] = op(X)[rows]·op(Y)[cols]ᵀ
// (accumulate: + instead of =).
template <typename T>
static int tri_product(int type, int upper, int trans, int N, int K, const T *X, int ldx, const T *Y, int ldy, T *P,
                       bool accumulate, cudaStream_t st) {
    const int p = bands_of(N), w = band_width(N, p);
    for (int i0 = 0; i0 < N; i0 += w) {
        const int b = N - i0 < w ? N - i0 : w;
        const int c0 = upper ? i0 : 0, c1 = upper ? N : i0 + b;
        const T *xr = trans ? X + i0 : X + (long long)i0 * ldx;
        const T *yc = trans ? Y + c0 : Y + (long long)c0 * ldy;
        G9_TRY(launch_gemm(type, trans, !trans, b, c1 - c0, K, 1.0, xr, ldx, 0, yc, ldy, 0, accumulate ? 1.0 : 0.0,
                           P + (long long)i0 * N + c0, N, 0, 1, st));
    }
    return 0;
}

template <typename T>
static int syr2k_t(int type, int upper, int trans, int N, int K, double alpha, const T *A, int lda, const T *B, int ldb,
                   double beta, T *C, int ldc, cudaStream_t st) {
    using R = typename Compute<T>::R;
    void *buf = nullptr;
    G9_TRY(l3_buffer((size_t)N * N * sizeof(T), &buf));
    T *P = (T *)buf;
    G9_TRY(tri_product<T>(type, upper, trans, N, K, A, lda, B ? B : A, B ? ldb : lda, P, false, st));
    if (B) G9_TRY(tri_product<T>(type, upper, trans, N, K, B, ldb, A, lda, P, true, st));
    l3_tri_epilogue<T><<<grid_elems((long long)N * N), 256, 0, st>>>(N, upper, (R)alpha, (R)beta, P, C, ldc);
    return launched("l3_tri_epilogue");
}

template <typename T>
static int trsm_t(int type, int left, int upper, int tA, int unit, int M, int N, double alpha, const T *A, int lda,
                  T *B, int ldb, cudaStream_t st) {
    using R = typename Compute<T>::R;
    constexpr int NB = l3::kTrsmNb;
    const int n = left ? M : N, m = left ? N : M;
    const int tr = left ? tA : !tA;
    const bool lower = !upper != (tr != 0);
    const int rev = lower ? 0 : 1;
    const int nbl = (n + NB - 1) / NB;
    // Leaf size: FP32 and FP64 compose the 128-row inverses into 256- and 512-row ones (two small batched GEMMs per
    // level), so that the serial leaves and the smallest updates -- GEMMs too narrow to fill the GPU -- are 4x fewer;
    // FP16 keeps 128-row leaves (its products would round the composed inverses to FP16 twice more).
    int levels = 0;
    if (type == GEN9BLAS_S || type == GEN9BLAS_D) levels = n >= 1024 ? 2 : n >= 512 ? 1 : 0;
    const int LB = NB << levels;
    auto al = [](size_t x) { return (x + 255) / 256 * 256; };
    const size_t bL = al((size_t)n * n * sizeof(T)), bY = al((size_t)n * m * sizeof(T));
    const size_t bI = al((size_t)nbl * NB * NB * sizeof(T)), bT = al((size_t)LB * m * sizeof(T));
    size_t bC[2] = {0, 0}, bW = 0;   // composed inverses (256, 512) and the composition's work blocks
    for (int l = 0; l < levels; l++) {
        const int s2 = NB << (l + 1);
        bC[l] = al((size_t)(n / s2) * s2 * s2 * sizeof(T));
        bW = bW > bC[l] / 4 ? bW : al((size_t)(n / s2) * (s2 / 2) * (s2 / 2) * sizeof(T));
    }
    void *buf = nullptr;
    G9_TRY(l3_buffer(bL + bY + bI + bT + bC[0] + bC[1] + bW, &buf));
    T *L = (T *)buf;
    T *Y = (T *)((char *)buf + bL);
    T *Inv = (T *)((char *)buf + bL + bY);
    T *Tmp = (T *)((char *)buf + bL + bY + bI);
    T *Comp[2] = {(T *)((char *)buf + bL + bY + bI + bT), (T *)((char *)buf + bL + bY + bI + bT + bC[0])};
    T *Work = (T *)((char *)buf + bL + bY + bI + bT + bC[0] + bC[1]);
    trsm_build_L<T><<<grid_elems((long long)n * n), 256, 0, st>>>(A, lda, n, tr, unit, rev, L);
    G9_TRY(launched("trsm_build_L"));
    trsm_build_Y<T><<<grid_elems((long long)n * m), 256, 0, st>>>(B, ldb, n, m, left, rev, (R)alpha, Y);
    G9_TRY(launched("trsm_build_Y"));
    static bool attr[kMaxDevices] = {};
    DevState *d = dev_state();
    const int smem = NB * NB * (int)sizeof(double);
    if (d && !attr[d->dev]) {
        G9_CU(cudaFuncSetAttribute(trsm_block_inverse<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        attr[d->dev] = true;
    }
    trsm_block_inverse<T><<<nbl, NB, smem, st>>>(L, n, Inv);
    G9_TRY(launched("trsm_block_inverse"));
    // inv([L00 0; L10 L11]) = [I0 0; -I1·L10·I0 I1] for every full pair of s-row blocks (s = 128, then 256)
    for (int l = 0; l < levels; l++) {
        const int sz = NB << l, s2 = 2 * sz, np = n / s2;
        if (np == 0) break;
        const T *src = l == 0 ? Inv : Comp[0];
        const long long ss = (long long)sz * sz;
        // Work_p = L10 · I0 (L10 = L[(2p+1)s.., 2p·s..], pitch n)
        G9_TRY(launch_gemm(type, 0, 0, sz, sz, sz, 1.0, L + (long long)sz * n, n, (long long)s2 * n + s2, src, sz,
                           2 * ss, 0.0, Work, sz, ss, np, st));
        // X_p = -I1 · Work_p, straight into rows s..2s-1, columns 0..s-1 of the composed block
        G9_TRY(launch_gemm(type, 0, 0, sz, sz, sz, -1.0, src + ss, sz, 2 * ss, Work, sz, ss, 0.0,
                           Comp[l] + (long long)sz * s2, s2, 4 * ss, np, st));
        trsm_compose<T><<<dim3((unsigned)std::min<long long>((ss + 255) / 256, 64), np), 256, 0, st>>>(src, sz, Comp[l]);
        G9_TRY(launched("trsm_compose"));
    }
    // Recursive halving over power-of-two aligned ranges of rows: solve the top half, subtract its contribution from
    // the bottom half with one GEMM (K = the top half's size), solve the bottom half. The updates are the right-looking
    // ones grouped into few large GEMMs (n = 4096: 2048 × m × 2048 first), which run near the GEMM kernels' large-K
    // rate instead of the K = 128 rate of one update per block (measured on B200, n = 4096: dtrsm 12.7 TF/s block by
    // block). A leaf is Y_i = inv(L_ii) · Y_i with the largest inverse that covers the range exactly (LB rows for a
    // full aligned block, else 128-row blocks; the last block may be shorter).
    auto leaf = [&](int lo, int rows, const T *inv, int ld) -> int {
        T *Yi = Y + (long long)lo * m;
        G9_TRY(launch_gemm(type, 0, 0, rows, m, rows, 1.0, inv, ld, 0, Yi, m, 0, 0.0, Tmp, m, 0, 1, st));
        G9_CU(cudaMemcpyAsync(Yi, Tmp, (size_t)rows * m * sizeof(T), cudaMemcpyDeviceToDevice, st));
        return 0;
    };
    auto solve = [&](auto &&self, int lo, int size) -> int {   // rows [lo, min(lo + size, n)), lo a multiple of size
        const int hi = lo + size < n ? lo + size : n;
        if (size > NB && size <= LB && hi - lo == size) {
            const int l = size == 2 * NB ? 0 : 1;
            return leaf(lo, size, Comp[l] + (long long)(lo / size) * size * size, size);
        }
        if (size <= NB) return leaf(lo, hi - lo, Inv + (long long)(lo / NB) * NB * NB, NB);
        const int mid = lo + size / 2;
        if (mid >= n) return self(self, lo, size / 2);
        G9_TRY(self(self, lo, size / 2));
        // Y[mid:hi] -= L[mid:hi, lo:mid] · Y[lo:mid]
        G9_TRY(launch_gemm(type, 0, 0, hi - mid, m, mid - lo, -1.0, L + (long long)mid * n + lo, n, 0,
                           Y + (long long)lo * m, m, 0, 1.0, Y + (long long)mid * m, m, 0, 1, st));
        return self(self, mid, size / 2);
    };
    int top = NB;
    while (top < n) top *= 2;
    G9_TRY(solve(solve, 0, top));
    trsm_write<T><<<grid_elems((long long)n * m), 256, 0, st>>>(Y, n, m, left, rev, B, ldb);
    return launched("trsm_write");
}

int launch_trsm_dev(int type, int left, int upper, int tA, int unit, int M, int N, double alpha, const void *A, int lda,
                    void *B, int ldb, cudaStream_t st) {
    if (type == GEN9BLAS_S)
        return trsm_t<float>(type, left, upper, tA, unit, M, N, alpha, (const float *)A, lda, (float *)B, ldb, st);
    if (type == GEN9BLAS_D)
        return trsm_t<double>(type, left, upper, tA, unit, M, N, alpha, (const double *)A, lda, (double *)B, ldb, st);
    return trsm_t<__half>(type, left, upper, tA, unit, M, N, alpha, (const __half *)A, lda, (__half *)B, ldb, st);
}

}  // namespace g9

using namespace g9;

// ---- C API (reference lib/gen9blas.h:98-112) ----
namespace {

int l3_check_type(int type) {
    if (type < 0 || type > 3) return fail(GEN9BLAS_ERR_UNSUPPORTED, "type %d unavailable", type);
    return 0;
}
size_t span(int rows, int cols, int ld, int es) { return ((size_t)(rows - 1) * ld + cols) * es; }

}  // namespace

extern "C" {

GEN9BLAS_API int gen9blas_symm(int type, int side, int uplo, int M, int N, double alpha, const void *A, int lda,
                               const void *B, int ldb, double beta, void *C, int ldc) {
    if (int e = begin_op()) return e;
    G9_TRY(l3_check_type(type));
    if (M <= 0 || N <= 0) return 0;
    const int left = side == GEN9BLAS_LEFT, n = left ? M : N, es = elem_bytes(type);
    if (lda < n || ldb < N || ldc < N) return fail(GEN9BLAS_ERR_INVALID_ARG, "symm: leading dimension too small");
    timer_start();
    Operand op[3];
    G9_TRY(map_operand(op[0], A, span(n, n, lda, es), 0, true, false));
    G9_TRY(map_operand(op[1], B, span(M, N, ldb, es), 1, true, false));
    G9_TRY(map_operand(op[2], C, span(M, N, ldc, es), 2, true, true));
    G.last_zc = op[0].zc | op[1].zc << 1 | op[2].zc << 2;
    timer_kernel();
    const int upper = uplo == GEN9BLAS_UPPER;
#define G9_SYMM(TT)                                                                                              \
    symm_t<TT>(type, left, upper, M, N, alpha, (const TT *)op[0].dptr, lda, (const TT *)op[1].dptr, ldb, beta, \
               (TT *)op[2].dptr, ldc, stream())
    G9_TRY(type == GEN9BLAS_S ? G9_SYMM(float) : type == GEN9BLAS_D ? G9_SYMM(double) : G9_SYMM(__half));
#undef G9_SYMM
    int r = finish_op(op, 3);
    timer_stop();
    return r;
}

// SYRK (two = false: B unused) and SYR2K.
static int syrk2(bool two, int type, int uplo, int trans, int N, int K, double alpha, const void *A, int lda,
                 const void *B, int ldb, double beta, void *C, int ldc) {
    if (int e = begin_op()) return e;
    G9_TRY(l3_check_type(type));
    if (N <= 0) return 0;
    const int es = elem_bytes(type);
    trans = trans ? 1 : 0;
    if (K <= 0) K = 0;
    if (ldc < N || (K > 0 && (trans ? lda < N : lda < K)) || (two && K > 0 && (trans ? ldb < N : ldb < K)))
        return fail(GEN9BLAS_ERR_INVALID_ARG, "syrk/syr2k: leading dimension too small");
    timer_start();
    Operand op[3];
    int nop = 0;
    const void *a = nullptr, *b = nullptr;
    if (K > 0) {
        G9_TRY(map_operand(op[0], A, trans ? span(K, N, lda, es) : span(N, K, lda, es), 0, true, false));
        a = op[0].dptr;
        nop = 1;
        if (two) {
            G9_TRY(map_operand(op[1], B, trans ? span(K, N, ldb, es) : span(N, K, ldb, es), 1, true, false));
            b = op[1].dptr;
            nop = 2;
        }
    }
    G9_TRY(map_operand(op[nop], C, span(N, N, ldc, es), 2, true, true));
    void *c = op[nop].dptr;
    nop++;
    timer_kernel();
    const int upper = uplo == GEN9BLAS_UPPER;
    if (K == 0) {   // C = beta·C on the triangle
        void *buf = nullptr;
        G9_TRY(l3_buffer((size_t)N * N * es, &buf));
        G9_CU(cudaMemsetAsync(buf, 0, (size_t)N * N * es, stream()));
#define G9_EPI(TT)                                                                                                   \
    l3_tri_epilogue<TT><<<grid_elems((long long)N * N), 256, 0, stream()>>>(                                    \
        N, upper, (Compute<TT>::R)0, (Compute<TT>::R)beta, (const TT *)buf, (TT *)c, ldc)
        if (type == GEN9BLAS_S) G9_EPI(float);
        else if (type == GEN9BLAS_D) G9_EPI(double);
        else G9_EPI(__half);
#undef G9_EPI
        G9_TRY(launched("l3_tri_epilogue"));
    } else {
#define G9_SYR2K(TT)                                                                                                 \
    syr2k_t<TT>(type, upper, trans, N, K, alpha, (const TT *)a, lda, (const TT *)b, ldb, beta, (TT *)c, ldc, stream())
        G9_TRY(type == GEN9BLAS_S ? G9_SYR2K(float) : type == GEN9BLAS_D ? G9_SYR2K(double) : G9_SYR2K(__half));
#undef G9_SYR2K
    }
    int r = finish_op(op, nop);
    timer_stop();
    return r;
}

GEN9BLAS_API int gen9blas_syrk(int type, int uplo, int trans, int N, int K, double alpha, const void *A, int lda,
                               double beta, void *C, int ldc) {
    return syrk2(false, type, uplo, trans, N, K, alpha, A, lda, nullptr, 0, beta, C, ldc);
}

GEN9BLAS_API int gen9blas_syr2k(int type, int uplo, int trans, int N, int K, double alpha, const void *A, int lda,
                                const void *B, int ldb, double beta, void *C, int ldc) {
    return syrk2(true, type, uplo, trans, N, K, alpha, A, lda, B, ldb, beta, C, ldc);
}

static int trxm(bool solve, int type, int side, int uplo, int transA, int diag, int M, int N, double alpha,
                const void *A, int lda, void *B, int ldb) {
    if (int e = begin_op()) return e;
    G9_TRY(l3_check_type(type));
    if (M <= 0 || N <= 0) return 0;
    const int left = side == GEN9BLAS_LEFT, n = left ? M : N, es = elem_bytes(type);
    if (lda < n || ldb < N) return fail(GEN9BLAS_ERR_INVALID_ARG, "trmm/trsm: leading dimension too small");
    timer_start();
    Operand op[2];
    G9_TRY(map_operand(op[0], A, span(n, n, lda, es), 0, true, false));
    G9_TRY(map_operand(op[1], B, span(M, N, ldb, es), 1, true, true));
    G.last_zc = op[0].zc | op[1].zc << 1;
    timer_kernel();
    const int upper = uplo == GEN9BLAS_UPPER, tA = transA ? 1 : 0, unit = diag == GEN9BLAS_UNIT;
#define G9_TRXM(TT)                                                                                                  \
    (solve ? trsm_t<TT>(type, left, upper, tA, unit, M, N, alpha, (const TT *)op[0].dptr, lda, (TT *)op[1].dptr,   \
                        ldb, stream())                                                                             \
           : trmm_t<TT>(type, left, upper, tA, unit, M, N, alpha, (const TT *)op[0].dptr, lda, (TT *)op[1].dptr,   \
                        ldb, stream()))
    G9_TRY(type == GEN9BLAS_S ? G9_TRXM(float) : type == GEN9BLAS_D ? G9_TRXM(double) : G9_TRXM(__half));
#undef G9_TRXM
    int r = finish_op(op, 2);
    timer_stop();
    return r;
}

GEN9BLAS_API int gen9blas_trmm(int type, int side, int uplo, int transA, int diag, int M, int N, double alpha,
                               const void *A, int lda, void *B, int ldb) {
    return trxm(false, type, side, uplo, transA, diag, M, N, alpha, A, lda, B, ldb);
}

GEN9BLAS_API int gen9blas_trsm(int type, int side, int uplo, int transA, int diag, int M, int N, double alpha,
                               const void *A, int lda, void *B, int ldb) {
    return trxm(true, type, side, uplo, transA, diag, M, N, alpha, A, lda, B, ldb);
}

}  // extern "C"
