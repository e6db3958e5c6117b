// dgemm_dmma.cu -- FP64 GEMM on the FP64 tensor path (DMMA, mma.sync.m16n8k8.f64).
//
// Replaces the reference's dgemm_v (lib/kernels/dgemm_core.cl:61-94: 16×16 FP64 tile per SIMD16 subgroup on packed,
// zero-padded panels, FMA along K). tcgen05.mma has no FP64 kind, so the B200 FP64 tensor path is the warp-level
// mma.sync with .f64 operands: each instruction is a 16×8×8 product on one warp, FP64 products accumulated in FP64.
// Design:
//   - CTA tile 128×64×16, 4 warps as 2 (M) × 2 (N), each warp 64×32 = 4×4 MMA tiles, 64 FP64 accumulators a thread,
//     two CTAs resident per SM;
//   - operands go global → shared memory with cp.async (16-byte copies when the operand's base, pitch and batch stride
//     allow, 8-byte copies otherwise; zero-fill outside the matrix), in a 3-stage ring, each operand stored in its own
//     contiguous direction (no transposition on the way: A as [m][k] or [k][m], B as [k][n] or [n][k]) with a
//     4-element row pad that makes every fragment read of a half-warp hit 16 distinct 8-byte bank pairs;
//   - tiles are visited in groups of 8 tile rows so that concurrently running CTAs share A and B panels in L2;
//   - epilogue alpha·acc + beta·C (beta = 0: C is not read), 16-byte stores where aligned.
// Products are summed along K in ascending order, four at a time inside the instruction; on B200 the results are
// bit-identical to cuBLAS DGEMM for the tested shapes.
#include "common.cuh"
#include "internal.h"

namespace g9 {

namespace dmma {
constexpr int BM = 128, WM = 64, WN = 32;   // CTA rows; warp tile 64×32 (4×4 MMA tiles of 16×8)
constexpr int MT = WM / 16, NT = WN / 8;
constexpr int PAD = 4;
constexpr int GROUP_M = 8;

// BN: CTA columns (warps = 2 × BN/32); BK: K per stage; KS: K per MMA instruction; MINB: resident CTAs per SM.
template <int BN_, int BK_, int STAGES_, int KS_, int MINB_> struct Cfg {
    static constexpr int BN = BN_, BK = BK_, STAGES = STAGES_, KS = KS_, MINB = MINB_;
    static constexpr int THREADS = 2 * (BN / WN) * 32;
    template <bool T_> __host__ __device__ static constexpr int a_stage() { return T_ ? BK * (BM + PAD) : BM * (BK + PAD); }
    template <bool T_> __host__ __device__ static constexpr int b_stage() { return T_ ? BN * (BK + PAD) : BK * (BN + PAD); }
    template <bool TA, bool TB> static constexpr int smem_bytes() { return STAGES * (a_stage<TA>() + b_stage<TB>()) * 8; }
};
}  // namespace dmma

__device__ __forceinline__ void cp_async_f64(double *dst, const double *src, int bytes, int src_bytes) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
    if (bytes == 16)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(src), "r"(src_bytes) : "memory");
    else
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(d), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N_> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N_) : "memory");
}

// D(16×8) += A(16×KS) · B(KS×8), FP64. Thread (g = lane/4, t = lane%4) holds a[2q + h] = A[g + 8h][t + 4q],
// b[q] = B[t + 4q][g], c[2h + e] = C[g + 8h][2t + e].
template <int KS> __device__ __forceinline__ void dmma_op(double (&c)[4], const double (&a)[KS / 2], const double (&b)[KS / 4]);
template <> __device__ __forceinline__ void dmma_op<4>(double (&c)[4], const double (&a)[2], const double (&b)[1]) {
    asm volatile("mma.sync.aligned.m16n8k4.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};\n"
                 : "+d"(c[0]), "+d"(c[1]), "+d"(c[2]), "+d"(c[3])
                 : "d"(a[0]), "d"(a[1]), "d"(b[0]));
}
template <> __device__ __forceinline__ void dmma_op<8>(double (&c)[4], const double (&a)[4], const double (&b)[2]) {
    asm volatile("mma.sync.aligned.m16n8k8.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};\n"
                 : "+d"(c[0]), "+d"(c[1]), "+d"(c[2]), "+d"(c[3])
                 : "d"(a[0]), "d"(a[1]), "d"(a[2]), "d"(a[3]), "d"(b[0]), "d"(b[1]));
}
template <> __device__ __forceinline__ void dmma_op<16>(double (&c)[4], const double (&a)[8], const double (&b)[4]) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5,%6,%7,%8,%9,%10,%11}, "
                 "{%12,%13,%14,%15}, {%0,%1,%2,%3};\n"
                 : "+d"(c[0]), "+d"(c[1]), "+d"(c[2]), "+d"(c[3])
                 : "d"(a[0]), "d"(a[1]), "d"(a[2]), "d"(a[3]), "d"(a[4]), "d"(a[5]), "d"(a[6]), "d"(a[7]),
                   "d"(b[0]), "d"(b[1]), "d"(b[2]), "d"(b[3]));
}

// Copies one (rows × cols) tile window of a stored row-major matrix X (pitch ld, shape xr × xc) starting at (r0, c0)
// into shared memory laid out [row][col] with pitch SP, as VEC-element copies; NCH copies per thread.
template <int ROWS, int COLS, int SP, int VEC, int THREADS>
__device__ __forceinline__ void load_tile(double *s, const double *__restrict__ X, long long ld, int xr, int xc, int r0,
                                          int c0, int tid) {
    constexpr int CPR = COLS / VEC;                          // copies per tile row
    constexpr int NCH = ROWS * CPR / THREADS;
    static_assert(NCH * THREADS == ROWS * CPR, "tile not divisible by the thread count");
#pragma unroll
    for (int i = 0; i < NCH; i++) {
        const int c = tid + i * THREADS;
        const int r = c / CPR, cc = (c % CPR) * VEC;
        const int gr = r0 + r, gc = c0 + cc;
        int nb = 0;
        const double *src = X;
        if (gr < xr && gc < xc) {
            nb = (xc - gc >= VEC ? VEC : xc - gc) * 8;
            src = X + (long long)gr * ld + gc;
        }
        cp_async_f64(s + r * SP + cc, src, VEC * 8, nb);
    }
}

template <class CF, bool TA, bool TB, int VA, int VB>
__global__ void __launch_bounds__(CF::THREADS, CF::MINB)
dgemm_dmma_kernel(int M, int N, int K, double alpha, const double *__restrict__ A, long long lda, long long sA,
                  const double *__restrict__ B, long long ldb, long long sB, double beta, double *C, long long ldc,
                  long long sC, int tiles_m, int tiles_n, int c_vec) {
    using namespace dmma;
    // Programmatic dependent launch (see the SGEMM kernel): let the successor start, wait for the predecessor.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    constexpr int BN = CF::BN, BK = CF::BK, STAGES = CF::STAGES, KS = CF::KS, THREADS = CF::THREADS;
    extern __shared__ __align__(16) double smem[];
    constexpr int AS = CF::template a_stage<TA>(), BS = CF::template b_stage<TB>();
    double *As = smem;
    double *Bs = smem + STAGES * AS;

    A += blockIdx.z * sA;
    B += blockIdx.z * sB;
    C += blockIdx.z * sC;

    // Grouped tile order: GROUP_M tile rows sweep all tile columns before the next group.
    const int bid = blockIdx.x;
    const int per_group = GROUP_M * tiles_n;
    const int grp = bid / per_group;
    const int first_m = grp * GROUP_M;
    const int gsize = min(tiles_m - first_m, GROUP_M);
    const int tm = first_m + (bid % per_group) % gsize;
    const int tn = (bid % per_group) / gsize;
    const int m0 = tm * BM, n0 = tn * BN;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int wm = (warp & 1) * WM, wn = (warp >> 1) * WN;
    const int g = lane >> 2, t = lane & 3;

    // Stored shapes: A is M×K or (transposed) K×M; B is K×N or (transposed) N×K.
    auto issue = [&](int stage, int k0) {
        double *as = As + stage * AS;
        double *bs = Bs + stage * BS;
        if (!TA) load_tile<BM, BK, BK + PAD, VA, THREADS>(as, A, lda, M, K, m0, k0, tid);
        else load_tile<BK, BM, BM + PAD, VA, THREADS>(as, A, lda, K, M, k0, m0, tid);
        if (!TB) load_tile<BK, BN, BN + PAD, VB, THREADS>(bs, B, ldb, K, N, k0, n0, tid);
        else load_tile<BN, BK, BK + PAD, VB, THREADS>(bs, B, ldb, N, K, n0, k0, tid);
    };

    double acc[MT][NT][4];
#pragma unroll
    for (int i = 0; i < MT; i++)
#pragma unroll
        for (int j = 0; j < NT; j++)
#pragma unroll
            for (int e = 0; e < 4; e++) acc[i][j][e] = 0.0;

    const int nk = (K + BK - 1) / BK;
#pragma unroll
    for (int s = 0; s < STAGES - 1; s++) {
        if (s < nk) issue(s, s * BK);
        cp_async_commit();
    }
    for (int kb = 0; kb < nk; kb++) {
        cp_async_wait<STAGES - 2>();
        __syncthreads();
        {
            const int kn = kb + STAGES - 1;
            if (kn < nk) issue(kn % STAGES, kn * BK);
            cp_async_commit();
        }
        const double *as = As + (kb % STAGES) * AS;
        const double *bs = Bs + (kb % STAGES) * BS;
#pragma unroll
        for (int kk = 0; kk < BK; kk += KS) {
            double a[MT][KS / 2], b[NT][KS / 4];
#pragma unroll
            for (int i = 0; i < MT; i++) {
                const int m = wm + i * 16 + g;
#pragma unroll
                for (int q = 0; q < KS / 4; q++) {
                    const int k = kk + t + 4 * q;
#pragma unroll
                    for (int h = 0; h < 2; h++)
                        a[i][2 * q + h] = !TA ? as[(m + 8 * h) * (BK + PAD) + k] : as[k * (BM + PAD) + m + 8 * h];
                }
            }
#pragma unroll
            for (int j = 0; j < NT; j++) {
                const int n = wn + j * 8 + g;
#pragma unroll
                for (int q = 0; q < KS / 4; q++) {
                    const int k = kk + t + 4 * q;
                    b[j][q] = !TB ? bs[k * (BN + PAD) + n] : bs[n * (BK + PAD) + k];
                }
            }
#pragma unroll
            for (int i = 0; i < MT; i++)
#pragma unroll
                for (int j = 0; j < NT; j++) dmma_op<KS>(acc[i][j], a[i], b[j]);
        }
    }
    cp_async_wait<0>();

    // Epilogue: thread holds rows (g, g + 8) × cols (2t, 2t + 1) of every 16×8 tile.
#pragma unroll
    for (int i = 0; i < MT; i++) {
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int m = m0 + wm + i * 16 + g + h * 8;
            if (m >= M) continue;
            double *crow = C + (long long)m * ldc;
#pragma unroll
            for (int j = 0; j < NT; j++) {
                const int n = n0 + wn + j * 8 + 2 * t;
                double v0 = alpha * acc[i][j][2 * h], v1 = alpha * acc[i][j][2 * h + 1];
                if (c_vec && n + 1 < N) {
                    double2 *p = reinterpret_cast<double2 *>(crow + n);
                    if (beta != 0.0) {
                        const double2 o = *p;
                        v0 = fma(beta, o.x, v0);
                        v1 = fma(beta, o.y, v1);
                    }
                    *p = make_double2(v0, v1);
                } else {
                    if (n < N) crow[n] = beta != 0.0 ? fma(beta, crow[n], v0) : v0;
                    if (n + 1 < N) crow[n + 1] = beta != 0.0 ? fma(beta, crow[n + 1], v1) : v1;
                }
            }
        }
    }
}

template <class CF, bool TA, bool TB, int VA, int VB>
static int dmma_go(cudaStream_t st, int M, int N, int K, double alpha, const double *A, long long lda, long long sA,
                   const double *B, long long ldb, long long sB, double beta, double *C, long long ldc, long long sC,
                   int count, int c_vec) {
    constexpr int smem = CF::template smem_bytes<TA, TB>();
    const int tiles_m = (M + dmma::BM - 1) / dmma::BM, tiles_n = (N + CF::BN - 1) / CF::BN;
    const long long tiles = (long long)tiles_m * tiles_n;
    if (tiles > 0x7fffffff || count > 65535)
        return fail(GEN9BLAS_ERR_INVALID_ARG, "DGEMM grid too large (M %d, N %d, count %d)", M, N, count);
    dim3 grid((unsigned)tiles, 1, count);
    auto k = dgemm_dmma_kernel<CF, TA, TB, VA, VB>;
    static bool attr[kMaxDevices] = {};
    G9_CU(smem_limit_once(k, smem, attr));
    launch_pdl(k, grid, dim3(CF::THREADS), (size_t)smem, st, M, N, K, alpha, A, lda, sA, B, ldb, sB, beta, C, ldc, sC,
               tiles_m, tiles_n, c_vec);
    return launched("dgemm_dmma");
}

template <class CF, bool TA, bool TB>
static int dmma_vec(bool va, bool vb, cudaStream_t st, int M, int N, int K, double alpha, const double *a, long long lda,
                    long long sA, const double *b, long long ldb, long long sB, double beta, double *c, long long ldc,
                    long long sC, int count, int c_vec) {
    if (va && vb) return dmma_go<CF, TA, TB, 2, 2>(st, M, N, K, alpha, a, lda, sA, b, ldb, sB, beta, c, ldc, sC, count, c_vec);
    if (va) return dmma_go<CF, TA, TB, 2, 1>(st, M, N, K, alpha, a, lda, sA, b, ldb, sB, beta, c, ldc, sC, count, c_vec);
    if (vb) return dmma_go<CF, TA, TB, 1, 2>(st, M, N, K, alpha, a, lda, sA, b, ldb, sB, beta, c, ldc, sC, count, c_vec);
    return dmma_go<CF, TA, TB, 1, 1>(st, M, N, K, alpha, a, lda, sA, b, ldb, sB, beta, c, ldc, sC, count, c_vec);
}

template <class CF>
static int dmma_trans(int tA, int tB, bool va, bool vb, cudaStream_t st, int M, int N, int K, double alpha,
                      const double *a, long long lda, long long sA, const double *b, long long ldb, long long sB,
                      double beta, double *c, long long ldc, long long sC, int count, int c_vec) {
#define G9_DMMA(TA_, TB_) \
    return dmma_vec<CF, TA_, TB_>(va, vb, st, M, N, K, alpha, a, lda, sA, b, ldb, sB, beta, c, ldc, sC, count, c_vec)
    if (!tA && !tB) G9_DMMA(false, false);
    if (tA && !tB) G9_DMMA(true, false);
    if (!tA && tB) G9_DMMA(false, true);
    G9_DMMA(true, true);
#undef G9_DMMA
}

int launch_dgemm_dmma(int tA, int tB, int M, int N, int K, double alpha, const void *A, int lda, long long sA,
                      const void *B, int ldb, long long sB, double beta, void *C, int ldc, long long sC, int count,
                      cudaStream_t st) {
    const bool va = ((uintptr_t)A & 15) == 0 && (lda % 2) == 0 && (count == 1 || sA % 2 == 0);
    const bool vb = ((uintptr_t)B & 15) == 0 && (ldb % 2) == 0 && (count == 1 || sB % 2 == 0);
    const int c_vec = ((uintptr_t)C & 15) == 0 && (ldc % 2) == 0 && (count == 1 || sC % 2 == 0);
    const double *a = (const double *)A;
    const double *b = (const double *)B;
    double *c = (double *)C;
    // 128×64 CTA tiles, 4 warps, 3 stages of K = 16, m16n8k8 instructions, two CTAs per SM: the second CTA's MMAs
    // cover each CTA's stage barrier (about 7% faster than one 128×128 CTA per SM at n = 4096 on B200).
    using Tile = dmma::Cfg<64, 16, 3, 8, 2>;
    return dmma_trans<Tile>(tA, tB, va, vb, st, M, N, K, alpha, a, lda, sA, b, ldb, sB, beta, c, ldc, sC, count, c_vec);
}

}  // namespace g9
