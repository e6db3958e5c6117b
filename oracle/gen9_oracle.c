/* gen9_oracle.c -- CPU restatement of the reference gen9blas hot path. TEST INFRASTRUCTURE ONLY.
 *
 * This file is the parity oracle: only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm
 * may load it, and only as the checker. The product (gen9-gpu-blas_b200/) never calls it; there is no CPU fallback.
 *
 * Each oracle_* function has the signature of the gen9blas.h entry point it checks (host pointers only) and restates
 * the arithmetic of the reference kprzybys/gen9-gpu-blas:
 *   oracle_axpy   lib/kernels/level12.cl:135-139   y = fma(a, x, y) in R (FP32 for FP16/FP32, FP64 for FP64)
 *   oracle_dot/asum/nrm2  level12.cl:189-214, lib/src/level12.c:171-190   FP64 sums, nrm2 = sqrt
 *   oracle_iamax  level12.cl:215-235, level12.c:192-211   first max |x| in R, NaN skipped, all-NaN -> 0, n<=0 -> -1
 *   oracle_gemv   level12.cl:243-283, 355-423   sum in R, y = beta == 0 ? alpha·t : fma(alpha, t, beta·y)
 *   oracle_ger    level12.cl:569-576   A = fma(alpha·x_i, y_j, A_ij) in R
 *   oracle_gemm   lib/src/gemm.c:5-74 and 191-263 with the main kernels hgemm_v (FP16 accumulation per FMA,
 *                 hgemm.cl:838-868), hgemm_kc_v (FP16 chunks of 32 into FP32, hgemm.cl:869-898), sgemm_v / dgemm_v
 *                 (FMA chain in K order), the skinny path (FP32 accumulation, gemm.c:185-263 and
 *                 level12.cl:646-862) and the epilogue C = alpha·Cp + beta·C in FP32 (hgemm.cl:557-564).
 * Element-exact functions (axpy, ger, iamax) reproduce the reference's own golden hashes
 * (tools/golden/expected/uhd620-whl/lib.txt: saxpy, daxpy, sger, dger, siamax, diamax); see tests/test_oracle_golden.py.
 * Order-dependent sums (dot, gemv, GEMM) use the sequential order; parity against them is within tolerance.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

enum { T_H = 0, T_S = 1, T_HS = 2, T_D = 3 };
#define OK 0
#define ERR_UNSUPPORTED (-2)
#define ERR_INVALID (-3)

typedef _Float16 f16;   /* used only for conversions (round to nearest even) */

static float h2f(uint16_t h) { f16 v; memcpy(&v, &h, 2); return (float)v; }
static uint16_t f2h(float f) { f16 v = (f16)f; uint16_t h; memcpy(&h, &v, 2); return h; }
static uint16_t d2h(double d) { f16 v = (f16)d; uint16_t h; memcpy(&h, &v, 2); return h; }

static long long voff(int n, int inc) { return inc < 0 ? (long long)(n - 1) * -inc : 0; }
static int l12(int type) { return type == T_HS ? T_H : (type >= 0 && type <= 3 ? type : -1); }

/* element i of a typed vector as double (exact) */
static double ld(int t, const void *p, long long i) {
    if (t == T_S) return ((const float *)p)[i];
    if (t == T_D) return ((const double *)p)[i];
    return h2f(((const uint16_t *)p)[i]);
}

int oracle_axpy(int type, int n, double a, const void *x, int incx, void *y, int incy) {
    int t = l12(type);
    if (t < 0) return ERR_UNSUPPORTED;
    if (n <= 0) return OK;
    if (!incx || !incy) return ERR_INVALID;
    long long ox = voff(n, incx), oy = voff(n, incy);
    for (long long i = 0; i < n; i++) {
        long long jx = ox + i * incx, jy = oy + i * incy;
        if (t == T_D) ((double *)y)[jy] = fma(a, ((const double *)x)[jx], ((double *)y)[jy]);
        else if (t == T_S) ((float *)y)[jy] = fmaf((float)a, ((const float *)x)[jx], ((float *)y)[jy]);
        else ((uint16_t *)y)[jy] = f2h(fmaf((float)a, h2f(((const uint16_t *)x)[jx]), h2f(((uint16_t *)y)[jy])));
    }
    return OK;
}

static int reduction(int type, int mode, int n, const void *x, int incx, const void *y, int incy, double *res) {
    *res = 0;
    int t = l12(type);
    if (t < 0) return ERR_UNSUPPORTED;
    if (n <= 0) return OK;
    if (!incx || (mode == 0 && !incy)) return ERR_INVALID;
    long long ox = voff(n, incx), oy = mode == 0 ? voff(n, incy) : 0;
    double s = 0;
    for (long long i = 0; i < n; i++) {
        double v = ld(t, x, ox + i * incx);
        if (mode == 0) s = fma(v, ld(t, y, oy + i * incy), s);
        else if (mode == 1) s += fabs(v);
        else s = fma(v, v, s);
    }
    *res = mode == 2 ? sqrt(s) : s;
    return OK;
}
int oracle_dot(int type, int n, const void *x, int incx, const void *y, int incy, double *r) {
    return reduction(type, 0, n, x, incx, y, incy, r);
}
int oracle_asum(int type, int n, const void *x, int incx, double *r) { return reduction(type, 1, n, x, incx, 0, 0, r); }
int oracle_nrm2(int type, int n, const void *x, int incx, double *r) { return reduction(type, 2, n, x, incx, 0, 0, r); }

int oracle_iamax(int type, int n, const void *x, int incx, int64_t *result) {
    *result = -1;
    int t = l12(type);
    if (t < 0) return ERR_UNSUPPORTED;
    if (n <= 0) return OK;
    if (!incx) return ERR_INVALID;
    long long ox = voff(n, incx);
    double bv = -1;   /* compared in R: FP16/FP32 values are exact in float, FP64 in double */
    long long bi = -1;
    for (long long i = 0; i < n; i++) {
        double v = fabs(ld(t, x, ox + i * incx));
        if (v > bv) { bv = v; bi = i; }   /* strict >: NaN never wins, ties keep the first index */
    }
    *result = bi < 0 ? 0 : bi;
    return OK;
}

/* store of a result in R with the gemv epilogue: beta == 0 ? alpha·t : fma(alpha, t, beta·y) */
static void st_epi(int t, void *y, long long k, double alpha, double beta, double acc) {
    if (t == T_D) {
        double *p = (double *)y;
        p[k] = beta == 0 ? alpha * acc : fma(alpha, acc, beta * p[k]);
    } else {
        float al = (float)alpha, be = (float)beta, a = (float)acc, old = (float)ld(t, y, k);
        float v = be == 0.0f ? al * a : fmaf(al, a, be * old);
        if (t == T_S) ((float *)y)[k] = v;
        else ((uint16_t *)y)[k] = f2h(v);
    }
}

int oracle_gemv(int type, int trans, int M, int N, double alpha, const void *A, int lda, const void *x, int incx,
                double beta, void *y, int incy) {
    int t = l12(type);
    if (t < 0) return ERR_UNSUPPORTED;
    if ((M < N ? M : N) <= 0) return OK;
    if (!incx || !incy) return ERR_INVALID;
    if (lda < N) return ERR_INVALID;
    int nx = trans ? M : N, ny = trans ? N : M;
    long long ox = voff(nx, incx), oy = voff(ny, incy);
    for (int i = 0; i < ny; i++) {
        double s = 0;   /* accumulate in R */
        float sf = 0;
        for (int j = 0; j < nx; j++) {
            long long ia = trans ? (long long)j * lda + i : (long long)i * lda + j;
            double av = ld(t, A, ia), xv = ld(t, x, ox + (long long)j * incx);
            if (t == T_D) s = fma(av, xv, s);
            else sf = fmaf((float)av, (float)xv, sf);
        }
        st_epi(t, y, oy + (long long)i * incy, alpha, beta, t == T_D ? s : sf);
    }
    return OK;
}

int oracle_ger(int type, int M, int N, double alpha, const void *x, int incx, const void *y, int incy, void *A, int lda) {
    int t = l12(type);
    if (t < 0) return ERR_UNSUPPORTED;
    if ((M < N ? M : N) <= 0) return OK;
    if (!incx || !incy) return ERR_INVALID;
    if (lda < N) return ERR_INVALID;
    long long ox = voff(M, incx), oy = voff(N, incy);
    for (int i = 0; i < M; i++)
        for (int j = 0; j < N; j++) {
            long long k = (long long)i * lda + j;
            double xv = ld(t, x, ox + (long long)i * incx), yv = ld(t, y, oy + (long long)j * incy);
            if (t == T_D) ((double *)A)[k] = fma(alpha * xv, yv, ((double *)A)[k]);
            else {
                float v = fmaf((float)alpha * (float)xv, (float)yv, (float)ld(t, A, k));
                if (t == T_S) ((float *)A)[k] = v;
                else ((uint16_t *)A)[k] = f2h(v);
            }
        }
    return OK;
}

/* Skinny threshold of the reference (gemm.c:191-199): 16 for H/HS/S, never for D. */
static int skinny_threshold(int type) {
    const char *e = getenv("GEN9BLAS_SKINNY");
    if (type == T_D) return 0;
    return e ? atoi(e) : 16;
}

/* One element of the main product p = Σ_k op(A)[m][k]·op(B)[k][n] with the accumulation of each type. */
static double gemm_dot(int type, int skinny, int tA, int tB, int m, int n, int K, const void *A, long long lda,
                       const void *B, long long ldb) {
    int es_t = type == T_HS ? T_H : type;
#define OPA(k) ld(es_t, A, tA ? (long long)(k) * lda + m : (long long)m * lda + (k))
#define OPB(k) ld(es_t, B, tB ? (long long)n * ldb + (k) : (long long)(k) * ldb + n)
    if (type == T_D) {
        double s = 0;
        for (int k = 0; k < K; k++) s = fma(OPA(k), OPB(k), s);
        return s;
    }
    if (type == T_S || skinny) {   /* FP32 FMA chain (skinny FP16 also accumulates in FP32) */
        float s = 0;
        for (int k = 0; k < K; k++) s = fmaf((float)OPA(k), (float)OPB(k), s);
        return type == T_S ? s : h2f(f2h(s));
    }
    if (type == T_H) {             /* FP16 accumulation, one rounding per FMA (exact product + sum in double) */
        uint16_t h = 0;
        for (int k = 0; k < K; k++) h = d2h(OPA(k) * OPB(k) + (double)h2f(h));
        return h2f(h);
    }
    /* T_HS: FP16 chunks of 32 products, each chunk added to an FP32 sum; result rounded to FP16 */
    float f = 0;
    uint16_t h = 0;
    for (int k = 0; k < K; k++) {
        h = d2h(OPA(k) * OPB(k) + (double)h2f(h));
        if ((k + 1) % 32 == 0) { f += h2f(h); h = 0; }
    }
    return h2f(f2h(f + h2f(h)));
#undef OPA
#undef OPB
}

int oracle_gemm_batched(int type, int tA, int tB, int M, int N, int K, double alpha, const void *A, int lda, int64_t sA,
                        const void *B, int ldb, int64_t sB, double beta, void *C, int ldc, int64_t sC, int count) {
    if (type < 0 || type > 3) return ERR_UNSUPPORTED;
    if (M <= 0 || N <= 0 || K <= 0 || count <= 0) return OK;
    int es = type == T_S ? 4 : type == T_D ? 8 : 2;
    int skinny = count == 1 && (M < N ? M : N) <= skinny_threshold(type);
    for (int b = 0; b < count; b++) {
        const char *Ab = (const char *)A + (size_t)b * sA * es;
        const char *Bb = (const char *)B + (size_t)b * sB * es;
        char *Cb = (char *)C + (size_t)b * sC * es;
        for (int m = 0; m < M; m++)
            for (int n = 0; n < N; n++) {
                double p = gemm_dot(type, skinny, tA, tB, m, n, K, Ab, lda, Bb, ldb);
                long long k = (long long)m * ldc + n;
                if (type == T_D) {
                    double *c = (double *)Cb;
                    c[k] = beta == 0 ? alpha * p : fma(beta, c[k], alpha * p);
                } else {
                    float v = (float)alpha * (float)p;
                    if (beta != 0) v = fmaf((float)beta, (float)ld(type == T_S ? T_S : T_H, Cb, k), v);
                    if (type == T_S) ((float *)Cb)[k] = v;
                    else ((uint16_t *)Cb)[k] = f2h(v);
                }
            }
    }
    return OK;
}

int oracle_gemm(int type, int tA, int tB, int M, int N, int K, double alpha, const void *A, int lda, const void *B, int ldb,
                double beta, void *C, int ldc) {
    return oracle_gemm_batched(type, tA, tB, M, N, K, alpha, A, lda, 0, B, ldb, 0, beta, C, ldc, 0, 1);
}
