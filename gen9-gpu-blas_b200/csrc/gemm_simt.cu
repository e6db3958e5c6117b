// gemm_simt.cu -- FP32 (FFMA) and FP64 (DFMA) GEMM on the SIMT pipes, register-blocked and staged through shared memory.
//
// SGEMM replaces the reference's sgemm_v (lib/kernels/sgemm.cl:200-230, 16×16 tile per SIMD16 subgroup on packed
// panels) and the FP64 variant dgemm_v (lib/kernels/dgemm_core.cl:61-94). B200 design: a CTA of 256 threads computes a
// BM×BN tile, each thread an (TM×TN) register block split into two halves (rows r and r + BM/2, columns c and
// c + BN/2) so that every shared-memory vector read of a warp covers contiguous 256-byte spans. Tiles of op(A) and
// op(B) are read from global memory with 16-byte loads along the operand's contiguous dimension (any transpose,
// any leading dimension, predicated at the edges: no packing, no padding buffers), double-buffered through shared
// memory with the next tile prefetched into registers during the current tile's FMAs. Accumulation is plain FP32 (or
// FP64) FMA along K; the epilogue computes alpha·acc + beta·C (beta = 0: C is not read).
#include "common.cuh"
#include "internal.h"

namespace g9 {

template <typename T> struct SimtCfg;
template <> struct SimtCfg<float> { static constexpr int BM = 128, BN = 128, BK = 8, TM = 8, TN = 8; };
template <> struct SimtCfg<double> { static constexpr int BM = 128, BN = 64, BK = 8, TM = 8, TN = 4; };

constexpr int SIMT_THREADS = 256;

// Loads CH consecutive elements of a row of the stored matrix X (pitch ld) starting at (r, c); zero outside.
template <typename T, int CH>
__device__ __forceinline__ void load_chunk(const T *__restrict__ X, long long ld, int rows, int cols, int r, int c, bool vec,
                                           T *out) {
    if (r < rows && vec && c + CH <= cols) {
        const T *p = X + (long long)r * ld + c;
        if (sizeof(T) * CH == 16) {
            if (sizeof(T) == 4) {
                float4 v = __ldg(reinterpret_cast<const float4 *>(p));
                out[0] = v.x; out[1] = v.y; out[2] = v.z; out[3] = v.w;
            } else {
                double2 v = __ldg(reinterpret_cast<const double2 *>(p));
                out[0] = v.x; out[1] = v.y;
            }
            return;
        }
    }
#pragma unroll
    for (int i = 0; i < CH; i++) out[i] = (r < rows && c + i < cols) ? __ldg(X + (long long)r * ld + c + i) : T(0);
}

template <typename T, bool TA, bool TB>
__global__ void __launch_bounds__(SIMT_THREADS) gemm_simt_kernel(int M, int N, int K, T alpha, const T *__restrict__ A,
                                                                 long long lda, long long sA, const T *__restrict__ B,
                                                                 long long ldb, long long sB, T beta, T *C, long long ldc,
                                                                 long long sC, int vecA, int vecB) {
    using Cfg = SimtCfg<T>;
    constexpr int BM = Cfg::BM, BN = Cfg::BN, BK = Cfg::BK, TM = Cfg::TM, TN = Cfg::TN;
    constexpr int CH = 16 / sizeof(T);                     // elements per 16-byte chunk
    constexpr int A_CH = BM * BK / CH / SIMT_THREADS;      // chunks per thread per tile
    constexpr int B_CH = BN * BK / CH / SIMT_THREADS;
    static_assert(A_CH >= 1 && B_CH >= 1, "tile too small for the thread count");
    __shared__ __align__(16) T As[2][BK][BM];
    __shared__ __align__(16) T Bs[2][BK][BN];

    const int batch = blockIdx.z;
    A += batch * sA;
    B += batch * sB;
    C += batch * sC;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int tid = threadIdx.x;
    const int tx = tid % (BN / TN), ty = tid / (BN / TN);

    // Stored shapes: A is M×K (K contiguous) or, transposed, K×M (M contiguous); B is K×N or, transposed, N×K.
    const int a_rows = TA ? K : M, a_cols = TA ? M : K;
    const int b_rows = TB ? N : K, b_cols = TB ? K : N;

    T ra[A_CH][CH], rb[B_CH][CH];
    auto load_tiles = [&](int k0) {
#pragma unroll
        for (int i = 0; i < A_CH; i++) {
            const int c = tid + i * SIMT_THREADS;
            if (!TA) {   // chunk covers k .. k+CH-1 of row m
                const int m = c / (BK / CH), kk = (c % (BK / CH)) * CH;
                load_chunk<T, CH>(A, lda, a_rows, a_cols, m0 + m, k0 + kk, vecA, ra[i]);
            } else {     // chunk covers m .. m+CH-1 of stored row k
                const int k = c / (BM / CH), mm = (c % (BM / CH)) * CH;
                load_chunk<T, CH>(A, lda, a_rows, a_cols, k0 + k, m0 + mm, vecA, ra[i]);
            }
        }
#pragma unroll
        for (int i = 0; i < B_CH; i++) {
            const int c = tid + i * SIMT_THREADS;
            if (!TB) {   // chunk covers n .. n+CH-1 of row k
                const int k = c / (BN / CH), nn = (c % (BN / CH)) * CH;
                load_chunk<T, CH>(B, ldb, b_rows, b_cols, k0 + k, n0 + nn, vecB, rb[i]);
            } else {     // chunk covers k .. k+CH-1 of stored row n
                const int n = c / (BK / CH), kk = (c % (BK / CH)) * CH;
                load_chunk<T, CH>(B, ldb, b_rows, b_cols, n0 + n, k0 + kk, vecB, rb[i]);
            }
        }
    };
    auto store_tiles = [&](int buf) {
#pragma unroll
        for (int i = 0; i < A_CH; i++) {
            const int c = tid + i * SIMT_THREADS;
            if (!TA) {
                const int m = c / (BK / CH), kk = (c % (BK / CH)) * CH;
#pragma unroll
                for (int e = 0; e < CH; e++) As[buf][kk + e][m] = ra[i][e];
            } else {
                const int k = c / (BM / CH), mm = (c % (BM / CH)) * CH;
#pragma unroll
                for (int e = 0; e < CH; e++) As[buf][k][mm + e] = ra[i][e];
            }
        }
#pragma unroll
        for (int i = 0; i < B_CH; i++) {
            const int c = tid + i * SIMT_THREADS;
            if (!TB) {
                const int k = c / (BN / CH), nn = (c % (BN / CH)) * CH;
#pragma unroll
                for (int e = 0; e < CH; e++) Bs[buf][k][nn + e] = rb[i][e];
            } else {
                const int n = c / (BK / CH), kk = (c % (BK / CH)) * CH;
#pragma unroll
                for (int e = 0; e < CH; e++) Bs[buf][kk + e][n] = rb[i][e];
            }
        }
    };

    T acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j++) acc[i][j] = T(0);

    const int nk = (K + BK - 1) / BK;
    load_tiles(0);
    store_tiles(0);
    __syncthreads();
    for (int kb = 0; kb < nk; kb++) {
        const int buf = kb & 1;
        if (kb + 1 < nk) load_tiles((kb + 1) * BK);
#pragma unroll
        for (int k = 0; k < BK; k++) {
            T a[TM], b[TN];
#pragma unroll
            for (int i = 0; i < TM / 2; i++) {
                a[i] = As[buf][k][ty * (TM / 2) + i];
                a[TM / 2 + i] = As[buf][k][BM / 2 + ty * (TM / 2) + i];
            }
#pragma unroll
            for (int j = 0; j < TN / 2; j++) {
                b[j] = Bs[buf][k][tx * (TN / 2) + j];
                b[TN / 2 + j] = Bs[buf][k][BN / 2 + tx * (TN / 2) + j];
            }
#pragma unroll
            for (int i = 0; i < TM; i++)
#pragma unroll
                for (int j = 0; j < TN; j++) acc[i][j] = fma_r(a[i], b[j], acc[i][j]);
        }
        if (kb + 1 < nk) {
            store_tiles(buf ^ 1);
            __syncthreads();
        }
    }

#pragma unroll
    for (int i = 0; i < TM; i++) {
        const int m = m0 + (i < TM / 2 ? ty * (TM / 2) + i : BM / 2 + ty * (TM / 2) + (i - TM / 2));
        if (m >= M) continue;
        T *crow = C + (long long)m * ldc;
#pragma unroll
        for (int j = 0; j < TN; j++) {
            const int n = n0 + (j < TN / 2 ? tx * (TN / 2) + j : BN / 2 + tx * (TN / 2) + (j - TN / 2));
            if (n < N) crow[n] = beta == T(0) ? alpha * acc[i][j] : fma_r(beta, crow[n], alpha * acc[i][j]);
        }
    }
}

template <typename T>
static int gemm_simt_t(int tA, int tB, int M, int N, int K, double alpha, const void *A, int lda, long long sA,
                       const void *B, int ldb, long long sB, double beta, void *C, int ldc, long long sC, int count,
                       cudaStream_t st) {
    using Cfg = SimtCfg<T>;
    const int vecA = ((uintptr_t)A & 15) == 0 && ((long long)lda * sizeof(T)) % 16 == 0 && (count == 1 || (sA * sizeof(T)) % 16 == 0);
    const int vecB = ((uintptr_t)B & 15) == 0 && ((long long)ldb * sizeof(T)) % 16 == 0 && (count == 1 || (sB * sizeof(T)) % 16 == 0);
    dim3 grid((N + Cfg::BN - 1) / Cfg::BN, (M + Cfg::BM - 1) / Cfg::BM, count);
    if (grid.y > 65535 || count > 65535) return fail(GEN9BLAS_ERR_INVALID_ARG, "GEMM grid too large (M %d, count %d)", M, count);
    const T al = (T)alpha, be = (T)beta;
    const T *a = (const T *)A;
    const T *b = (const T *)B;
    T *c = (T *)C;
#define G9_SIMT(TA_, TB_) \
    gemm_simt_kernel<T, TA_, TB_><<<grid, SIMT_THREADS, 0, st>>>(M, N, K, al, a, lda, sA, b, ldb, sB, be, c, ldc, sC, vecA, vecB)
    if (!tA && !tB) G9_SIMT(false, false);
    else if (tA && !tB) G9_SIMT(true, false);
    else if (!tA && tB) G9_SIMT(false, true);
    else G9_SIMT(true, true);
#undef G9_SIMT
    return launched(sizeof(T) == 4 ? "sgemm_ffma" : "dgemm_dfma");
}

int launch_gemm_simt(int type, int tA, int tB, int M, int N, int K, double alpha, const void *A, int lda, long long sA,
                     const void *B, int ldb, long long sB, double beta, void *C, int ldc, long long sC, int count,
                     cudaStream_t st) {
    if (type == GEN9BLAS_S) return gemm_simt_t<float>(tA, tB, M, N, K, alpha, A, lda, sA, B, ldb, sB, beta, C, ldc, sC, count, st);
    return gemm_simt_t<double>(tA, tB, M, N, K, alpha, A, lda, sA, B, ldb, sB, beta, C, ldc, sC, count, st);
}

}  // namespace g9
