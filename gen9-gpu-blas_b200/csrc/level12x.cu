// level12x.cu -- the rest of levels 1-2: scal, copy, swap, rot, rotm, rotg, rotmg; symv, trmv, trsv, syr, syr2; and
// the banded / packed forms gbmv, sbmv, tbmv, tbsv, spmv, tpmv, tpsv, spr, spr2 (types H, S, D; HS = H).
//
// Replaces lib/src/level12.c:54-165, 267-519 and the matching kernels of lib/kernels/level12.cl (kprzybys/
// gen9-gpu-blas). Semantics kept: strided vectors with negative increments addressing the lowest element, increment 0
// an invalid argument, n <= 0 a no-op, beta = 0 never reads y, FP16 computed in FP32 and FP64 in FP64, the row-major
// band layout A(i, j) = A[i·lda + KL + j − i] (symmetric / triangular: upper KL = 0, KU = K; lower KL = K, KU = 0) and
// the packed layouts (upper row i starts at i·n − i(i−1)/2, lower row i at i(i+1)/2). B200 design:
// - level 1: one grid-stride kernel per operation (16-byte vectors when both vectors are contiguous and aligned);
// - matrix-vector products of dense and packed symmetric / triangular matrices: strips of 64 rows × 2048 columns of
//   the stored triangle, each read once along its rows, giving row partial sums (the product) and column partial sums
//   (the mirrored half, or the transposed product), added per output in a fixed order by a second kernel;
// - banded products: one kernel template, one warp per output row, each lane summing a strided share of the row's
//   band through a layout accessor, a fixed shuffle tree, then alpha·sum + beta·y. In-place products (trmv, tbmv,
//   tpmv) write a work vector that is copied back;
// - rank updates (syr, syr2, spr, spr2): one block per row of the stored triangle, four elements per thread in
//   flight;
// - solves (trsv, tpsv, tbsv): one cooperative look-back kernel over 64-row blocks in dependency order, FP64 inverses
//   of the diagonal blocks, per-block flags with bounded waits.
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

// Stored-triangle products (dense or packed; symmetric, or triangular with op = A or Aᵀ), the stored triangle read
// once in strips: CTA (p, rb) takes the 64 rows of block rb and the columns of piece p (2048 wide) that lie in the
// stored triangle. Warp w owns rows 8w .. 8w + 7 and walks the strip in 128-column chunks, lane l reading columns
// l + 32e (e < 4) of its 8 rows (32 loads in flight, 8 KB contiguous per row and CTA). Row part (symmetric;
// triangular op = A): each lane keeps its 8 rows' sums, reduced over the warp at the end into Prow[p][i]. Column
// part (symmetric: off-diagonal elements, the mirrored half; triangular op = Aᵀ: every stored element): per chunk the
// 8 warps' column sums are combined in warp order through shared memory into Pcol[rb][j]. A unit diagonal is read
// as 1. l2x_tri_final adds the partials of each output in a fixed order.
constexpr int kTriRows = 64, kTriPiece = 2048;

// Four consecutive elements p[0..3] (VEC: one 16-byte load for FP32, two for FP64, one 8-byte load for FP16; the
// caller guarantees the alignment).
template <typename T, bool VEC>
__device__ __forceinline__ void load4(const T *p, typename Compute<T>::R *v) {
    if constexpr (VEC && sizeof(T) == 4) {
        const float4 q = *reinterpret_cast<const float4 *>(p);
        v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
    } else if constexpr (VEC && sizeof(T) == 8) {
        const double2 q0 = reinterpret_cast<const double2 *>(p)[0], q1 = reinterpret_cast<const double2 *>(p)[1];
        v[0] = q0.x; v[1] = q0.y; v[2] = q1.x; v[3] = q1.y;
    } else if constexpr (VEC && sizeof(T) == 2) {
        const uint2 q = *reinterpret_cast<const uint2 *>(p);
        const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&q.x));
        const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&q.y));
        v[0] = f0.x; v[1] = f0.y; v[2] = f1.x; v[3] = f1.y;
    } else {
#pragma unroll
        for (int k = 0; k < 4; k++) v[k] = to_r(p[k]);
    }
}

// VEC: dense rows whose element (i, 4k) is 16-byte aligned (8-byte for FP16).
template <typename T, bool VEC>
__global__ void __launch_bounds__(256) l2x_tri_strip(const L2Mat m, int use_row, int use_col, const T *__restrict__ x,
                                                     long long ox, long long ix, typename Compute<T>::R *Prow,
                                                     typename Compute<T>::R *Pcol) {
    using R = typename Compute<T>::R;
    __shared__ R csum[8][128];
    const int n = m.n, rb = blockIdx.y, pc = blockIdx.x;
    const int r0 = rb * kTriRows, r1 = min(n, r0 + kTriRows);
    // stored columns of this row block: lower [0, r1), upper [r0, n); this piece's share of them
    const int c_lo = max(m.upper ? r0 : 0, pc * kTriPiece), c_hi = min(m.upper ? n : r1, (pc + 1) * kTriPiece);
    if (c_lo >= c_hi) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool tri = m.kind == l2x::kTriangular;
    const T *A = (const T *)m.A;
    const T *rowp[8];
    R xi[8], racc[8];
#pragma unroll
    for (int u = 0; u < 8; u++) {
        const int i = min(r0 + warp * 8 + u, n - 1);
        long long base;
        if (m.layout == l2x::kDense) base = (long long)i * m.lda;
        else base = m.upper ? (long long)i * n - (long long)i * (i - 1) / 2 - i : (long long)i * (i + 1) / 2;
        rowp[u] = A + base;   // stored element (i, j) at rowp[j]
        xi[u] = to_r(x[ox + (long long)i * ix]);
        racc[u] = 0;
    }
    for (int c0 = c_lo; c0 < c_hi; c0 += 128) {
        // lane l: columns c0 + 4l .. c0 + 4l + 3
        const int j0 = c0 + 4 * lane;
        // interior chunk: every (row of the block, column of the chunk) strictly inside the stored triangle
        const bool interior = c0 + 128 <= c_hi && (m.upper ? c0 >= r1 : c0 + 128 <= r0);
        R xc[4], cacc[4] = {0, 0, 0, 0};
        R a[8][4];
        if (interior) {
            if (ix == 1) load4<T, false>(x + ox + j0, xc);
            else {
#pragma unroll
                for (int k = 0; k < 4; k++) xc[k] = to_r(x[ox + (long long)(j0 + k) * ix]);
            }
#pragma unroll
            for (int u = 0; u < 8; u++) {
                if (r0 + warp * 8 + u < r1) load4<T, VEC>(rowp[u] + j0, a[u]);
                else a[u][0] = a[u][1] = a[u][2] = a[u][3] = R(0);
            }
#pragma unroll
            for (int u = 0; u < 8; u++)
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    racc[u] = fma_r(a[u][k], xc[k], racc[u]);
                    cacc[k] = fma_r(a[u][k], xi[u], cacc[k]);
                }
        } else {
#pragma unroll
            for (int k = 0; k < 4; k++) xc[k] = j0 + k < c_hi ? to_r(x[ox + (long long)(j0 + k) * ix]) : R(0);
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int i = r0 + warp * 8 + u;
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const int j = j0 + k;
                    const bool st = i < r1 && j < c_hi && (m.upper ? j >= i : j <= i);
                    R v = st ? to_r(rowp[u][j]) : R(0);
                    if (tri && m.unit && i == j) v = R(1);
                    a[u][k] = v;
                }
            }
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int i = r0 + warp * 8 + u;
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    racc[u] = fma_r(a[u][k], xc[k], racc[u]);
                    cacc[k] = fma_r((!tri && j0 + k == i) ? R(0) : a[u][k], xi[u], cacc[k]);
                }
            }
        }
        if (use_col) {
#pragma unroll
            for (int k = 0; k < 4; k++) csum[warp][4 * lane + k] = cacc[k];
            __syncthreads();
            if (threadIdx.x < 128) {
                const int j = c0 + threadIdx.x;
                R sum = csum[0][threadIdx.x];
#pragma unroll
                for (int w = 1; w < 8; w++) sum += csum[w][threadIdx.x];
                if (j < c_hi) Pcol[(long long)rb * n + j] = sum;
            }
            __syncthreads();
        }
    }
    if (!use_row) return;
#pragma unroll
    for (int u = 0; u < 8; u++) {
        R sum = racc[u];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        const int i = r0 + warp * 8 + u;
        if (lane == 0 && i < r1) Prow[(long long)pc * n + i] = sum;
    }
}

// y_k = alpha·(row partials of k + column partials of k) + beta·y_k (beta = 0: y not read). Row partials: the pieces
// of k's row block that hold stored columns; column partials: the row blocks whose stored rows reach column k. A
// block takes 32 consecutive outputs (lane = output, coalesced reads); warp w sums every 8th partial of its range and
// the 8 warp sums are added in warp order (fixed order, deterministic).
template <typename T>
__global__ void __launch_bounds__(256) l2x_tri_final(const L2Mat m, int use_row, int use_col,
                                                     const typename Compute<T>::R *__restrict__ Prow,
                                                     const typename Compute<T>::R *__restrict__ Pcol,
                                                     typename Compute<T>::R alpha, typename Compute<T>::R beta, T *y,
                                                     long long oy, long long iy) {
    using R = typename Compute<T>::R;
    __shared__ R part[8][32];
    const int n = m.n, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int k = blockIdx.x * 32 + lane;
    const int kk = k < n ? k : n - 1;
    const int rb = kk / kTriRows, nrb = (n + kTriRows - 1) / kTriRows;
    const int r0 = rb * kTriRows, r1 = min(n, r0 + kTriRows);
    R sum = 0;
    if (use_row) {   // pieces p with [p·2048, (p+1)·2048) meeting this row block's stored columns
        const int p_lo = m.upper ? r0 / kTriPiece : 0, p_hi = m.upper ? (n - 1) / kTriPiece : (r1 - 1) / kTriPiece;
        for (int p = p_lo + warp; p <= p_hi; p += 8) sum += Prow[(long long)p * n + kk];
    }
    if (use_col) {   // row blocks whose stored rows include column kk: lower rows >= kk, upper rows <= kk
        const int b_lo = m.upper ? 0 : rb, b_hi = m.upper ? rb : nrb - 1;
        for (int b = b_lo + warp; b <= b_hi; b += 8) sum += Pcol[(long long)b * n + kk];
    }
    part[warp][lane] = sum;
    __syncthreads();
    if (warp == 0 && k < n) {
        R tot = part[0][lane];
#pragma unroll
        for (int w = 1; w < 8; w++) tot += part[w][lane];
        T &yk = y[oy + (long long)k * iy];
        yk = from_r<T>(beta == R(0) ? alpha * tot : fma_r(beta, to_r(yk), alpha * tot));
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
    // the stored row is contiguous in both layouts; four elements per thread in flight
    T *row = m.layout == l2x::kDense ? A + (long long)i * m.lda : A + packed_index(m, i, j0) - j0;
    const int step = blockDim.x;
    for (int jb = j0 + threadIdx.x; jb < j1; jb += 4 * step) {
        R av[4], d[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int j = jb + u * step;
            av[u] = j < j1 ? to_r(row[j]) : R(0);
            const R xj = j < j1 ? to_r(x[ox + (long long)j * ix]) : R(0);
            d[u] = xi * xj;
            if (two) d[u] = fma_r(xi, j < j1 ? to_r(y[oy + (long long)j * iy]) : R(0), yi * xj);
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int j = jb + u * step;
            if (j < j1) row[j] = from_r<T>(fma_r(alpha, d[u], av[u]));
        }
    }
}

// ---------------------------------------------------------------- triangular solves (trsv, tpsv, tbsv)
// One cooperative kernel over blocks of 64 rows of op(A) in dependency order (op(A) upper: the rows are taken in
// reversed order, which makes it lower). Every CTA owns blocks b = blockIdx.x, + gridDim.x, ...; for a block it
// (1) inverts the diagonal block in FP64 in shared memory (independent of x, so it overlaps the earlier blocks),
// (2) accumulates op(A)[block b][block c]·x_c over the earlier blocks c (band: only the blocks the band reaches):
// groups of G tiles are loaded into registers together with one poll of their x messages, every thread accumulating
// its elements across all groups, and the per-row sums are formed once after the walk; the last tile (block b - 1,
// the chain's last dependency) is multiplied on its own afterwards, so that only its product separates x_{b-1} from
// x_b (measured on B200, n = 16384: strsv 1.14 -> 0.62 ms, dtrsv 1.22 -> 0.85 ms against one tile at a time),
// (3) writes x_b = inv·(b_b − acc) in place and publishes it. Publication is a message per value: a 64-bit word holding
// the value's bits (FP32: the whole value; FP64: one half per word) and the launch's epoch, stored with one relaxed
// 64-bit access, so a reader that sees the epoch sees the value -- one L2 round trip per dependency, no flag and no
// fence. The epochs make the message buffer reusable without resets. All CTAs are co-resident (cooperative launch
// sized by the occupancy), and every wait is bounded: a wait that gives up sets the device error word and the CTA
// returns; the CTAs that wait for it then give up as well.
constexpr int kSvNb = 64;

__device__ __forceinline__ unsigned long long sv_ld_msg(const unsigned long long *a) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
    return v;
}
__device__ __forceinline__ void sv_st_msg(unsigned long long *a, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(a), "l"(v) : "memory");
}
// Words per value in the message buffer.
template <typename R> __host__ __device__ constexpr int sv_words() { return sizeof(R) == 8 ? 2 : 1; }
__device__ __forceinline__ unsigned long long sv_timer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

struct SvArgs {
    L2Mat m;            // triangular, dense / band / packed
    int rev;            // op(A) upper: reversed index order
    void *x;
    long long ox, ix;
    unsigned long long *msg;   // [block][row][sv_words] messages
    unsigned epoch;
    unsigned *err;
    int nb, back;       // blocks; band: earlier blocks a block depends on (0: all)
    unsigned long long limit_ns;
};

template <typename T>
__device__ __forceinline__ typename Compute<T>::R sv_at(const SvArgs &a, int fr, int fc) {   // op(A), forward indices
    const int n = a.m.n;
    return elem<T>(a.m, a.rev ? n - 1 - fr : fr, a.rev ? n - 1 - fc : fc);
}

// Dynamic shared memory: inverse (FP64) | tile | x block | right-hand side | flag word.
template <typename T> constexpr size_t sv_smem_bytes() {
    return sizeof(double) * kSvNb * (kSvNb + 1) + sizeof(typename Compute<T>::R) * (kSvNb * (kSvNb + 1) + kSvNb) +
           sizeof(double) * kSvNb + 16;
}

template <typename T>
__global__ void __launch_bounds__(256, sizeof(T) == 8 ? 1 : 2) l2x_trsv_lb(const SvArgs a) {
    using R = typename Compute<T>::R;
    extern __shared__ __align__(16) unsigned char sv_smem[];
    auto inv = reinterpret_cast<double (*)[kSvNb + 1]>(sv_smem);
    auto tile = reinterpret_cast<R (*)[kSvNb + 1]>(sv_smem + sizeof(double) * kSvNb * (kSvNb + 1));
    R *xs = &tile[kSvNb][0];
    double *rhs = reinterpret_cast<double *>(xs + kSvNb + (sizeof(R) == 4 && kSvNb % 2 ? 1 : 0));
    int &go = *reinterpret_cast<int *>(rhs + kSvNb);
    T *x = (T *)a.x;
    const int n = a.m.n, tid = threadIdx.x, r = tid >> 2, q = tid & 3;
    const bool tr = a.m.trans != 0;   // op(A)(i, j) = A(j, i): A's rows run along the tile's column index
    auto xi = [&](int f) { return a.ox + (long long)(a.rev ? n - 1 - f : f) * a.ix; };
    // element e of a 64 × 64 tile for this thread: consecutive threads follow A's contiguous direction
    auto tij = [&](int e, int &i, int &j) {
        if (tr) { j = e / kSvNb; i = e % kSvNb; } else { i = e / kSvNb; j = e % kSvNb; }
    };
    if (tid == 0) go = 1;
    for (int b = blockIdx.x; b < a.nb; b += gridDim.x) {
        const int f0 = b * kSvNb, rows = min(kSvNb, n - f0);
        __syncthreads();
        // (1) diagonal block (identity past the last row), inverse column c by the 4 lanes of row-group c
        for (int e = tid; e < kSvNb * kSvNb; e += 256) {
            int i, j;
            tij(e, i, j);
            R v = i == j ? R(1) : R(0);
            if (i < rows && j < rows && j <= i) v = sv_at<T>(a, f0 + i, f0 + j);
            tile[i][j] = v;
        }
        if (tid < kSvNb) rhs[tid] = tid < rows ? (double)to_r(x[xi(f0 + tid)]) : 0.0;
        __syncthreads();
        {
            const int c = r;
            for (int i = 0; i < kSvNb; i++) {
                double s = 0.0;
                for (int k = c + q; k < i; k += 4) s += (double)tile[i][k] * inv[k][c];
                s += __shfl_xor_sync(0xffffffffu, s, 1);
                s += __shfl_xor_sync(0xffffffffu, s, 2);
                if (q == 0) inv[i][c] = i < c ? 0.0 : ((i == c ? 1.0 : 0.0) - s) / (double)tile[i][i];
                __syncwarp();
            }
        }
        // (2) earlier blocks, G tiles at a time: every thread loads its 16 elements of each tile of the group into
        // registers (consecutive threads along A's contiguous direction), the 256 threads poll the group's x
        // messages (one word each) into shared memory, and after one barrier each thread accumulates its elements
        // times their x in registers across all tiles; the per-row sums are formed once, after the walk.
        // Non-transposed: a thread holds column j = tid % 64 of rows tid / 64 + 4u (16 partial sums);
        // transposed: row tid % 64 of columns tid / 64 + 4u (one partial sum).
        constexpr int G = sizeof(R) == 8 ? 2 : 4;   // tiles per group: G · 64 values · words per value = 256 words
        constexpr int EPT = kSvNb * kSvNb / 256;    // elements of a tile per thread
        R acc_r[EPT];
#pragma unroll
        for (int u = 0; u < EPT; u++) acc_r[u] = 0;
        unsigned long long *xw = reinterpret_cast<unsigned long long *>(&tile[0][0]);   // [G][64][words]
        __syncthreads();   // the inverse is complete (tile is reused for the group's x words)
        const int c_lo = a.back ? max(0, b - a.back) : 0;
        // the immediate predecessor (tile b - 1, the last dependency) is taken apart after the walk and its reduction,
        // so that only its own product lies on the chain from x_{b-1} to x_b
        const int c_end = b - 1;
        R plast[EPT];
        if (c_lo <= c_end) {
#pragma unroll
            for (int u = 0; u < EPT; u++) {
                int i, j;
                tij(tid + 256 * u, i, j);
                plast[u] = i < rows ? sv_at<T>(a, f0 + i, c_end * kSvNb + j) : R(0);
            }
        }
        for (int cg = c_lo; cg < c_end; cg += G) {
            R pre[G][EPT];
#pragma unroll
            for (int t = 0; t < G; t++) {
                const int c = cg + t;
#pragma unroll
                for (int u = 0; u < EPT; u++) {
                    int i, j;
                    tij(tid + 256 * u, i, j);
                    pre[t][u] = (c < c_end && i < rows) ? sv_at<T>(a, f0 + i, c * kSvNb + j) : R(0);
                }
            }
            {   // word tid of the group's messages: value (tile, row) = tid / words, half tid % words
                const int vi = tid / sv_words<R>(), tt = vi / kSvNb, row = vi % kSvNb;
                unsigned long long v = 0;
                if (cg + tt < c_end) {
                    const unsigned long long *w = a.msg + ((long long)(cg + tt) * kSvNb + row) * sv_words<R>() +
                                                  tid % sv_words<R>();
                    v = sv_ld_msg(w);
                    if ((unsigned)(v >> 32) != a.epoch) {
                        const unsigned long long t0 = sv_timer();
                        for (unsigned it = 0; (unsigned)(v >> 32) != a.epoch; ++it) {
                            v = sv_ld_msg(w);
                            if ((it & 63) == 63 && sv_timer() - t0 > a.limit_ns) {
                                go = 0;
                                break;
                            }
                        }
                    }
                }
                xw[tid] = v;
            }
            __syncthreads();
            if (!go) {
                if (tid == 0) *(volatile unsigned *)a.err = kDevErrWaitTimeout;
                return;
            }
#pragma unroll
            for (int t = 0; t < G; t++) {
#pragma unroll
                for (int u = 0; u < EPT; u++) {
                    int i, j;
                    tij(tid + 256 * u, i, j);
                    R xv;
                    if constexpr (sizeof(R) == 8) {
                        const unsigned long long lo = xw[(t * kSvNb + j) * 2], hi = xw[(t * kSvNb + j) * 2 + 1];
                        xv = __longlong_as_double((long long)((hi << 32) | (lo & 0xffffffffull)));
                    } else {
                        xv = __uint_as_float((unsigned)xw[t * kSvNb + j]);
                    }
                    if (tr) acc_r[0] = fma_r(pre[t][u], xv, acc_r[0]);
                    else acc_r[u] = fma_r(pre[t][u], xv, acc_r[u]);
                }
            }
            __syncthreads();   // the group's x words are consumed
        }
        // per-row sums: red[i][k] holds the partial of row i from thread slot k (64 slots), added in slot order
        R acc = 0;
        {
            auto red = reinterpret_cast<R (*)[kSvNb + 1]>(&tile[0][0]);
            if (!tr) {
#pragma unroll
                for (int u = 0; u < EPT; u++) red[(tid >> 6) + 4 * u][tid & 63] = acc_r[u];
            } else {
                red[tid & 63][tid >> 6] = acc_r[0];
            }
            __syncthreads();
            const int nslot = tr ? 4 : kSvNb;
            for (int k = q; k < nslot; k += 4) acc += red[r][k];
        }
        if (c_lo <= c_end) {   // tile b - 1: stored in shared memory, x_{b-1} polled by 64 threads, row sums
            __syncthreads();   // the partial sums are read
#pragma unroll
            for (int u = 0; u < EPT; u++) {
                int i, j;
                tij(tid + 256 * u, i, j);
                tile[i][j] = plast[u];
            }
            if (tid < kSvNb) {
                const unsigned long long *w = a.msg + ((long long)c_end * kSvNb + tid) * sv_words<R>();
                unsigned long long v0 = sv_ld_msg(w), v1 = sv_words<R>() == 2 ? sv_ld_msg(w + 1) : 0ull;
                auto ready = [&]() {
                    return (unsigned)(v0 >> 32) == a.epoch && (sv_words<R>() == 1 || (unsigned)(v1 >> 32) == a.epoch);
                };
                if (!ready()) {
                    const unsigned long long t0 = sv_timer();
                    for (unsigned it = 0; !ready(); ++it) {
                        v0 = sv_ld_msg(w);
                        if (sv_words<R>() == 2) v1 = sv_ld_msg(w + 1);
                        if ((it & 63) == 63 && sv_timer() - t0 > a.limit_ns) {
                            go = 0;
                            break;
                        }
                    }
                }
                if constexpr (sizeof(R) == 8)
                    xs[tid] = __longlong_as_double((long long)((v1 << 32) | (v0 & 0xffffffffull)));
                else
                    xs[tid] = __uint_as_float((unsigned)v0);
            }
            __syncthreads();
            if (!go) {
                if (tid == 0) *(volatile unsigned *)a.err = kDevErrWaitTimeout;
                return;
            }
            R s2 = 0;
#pragma unroll
            for (int j = q; j < kSvNb; j += 4) s2 = fma_r(tile[r][j], xs[j], s2);
            acc += s2;
        }
        // (3) x_b = inv·(b_b − acc), FP64, 4 lanes per row; then the flag
        acc += __shfl_xor_sync(0xffffffffu, acc, 1);
        acc += __shfl_xor_sync(0xffffffffu, acc, 2);
        __syncthreads();
        if (q == 0) rhs[r] -= (double)acc;
        __syncthreads();
        double v = 0.0;
        for (int k = q; k <= r; k += 4) v += inv[r][k] * rhs[k];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        if (q == 0 && r < rows) {
            const T xv = from_r<T>((R)v);
            x[xi(f0 + r)] = xv;
            const R pv = to_r(xv);   // the rounded value, as the later blocks would read it from x
            unsigned long long *w = a.msg + ((long long)b * kSvNb + r) * sv_words<R>();
            const unsigned long long tag = (unsigned long long)a.epoch << 32;
            if constexpr (sizeof(R) == 8) {
                const unsigned long long bits = (unsigned long long)__double_as_longlong(pv);
                sv_st_msg(w, tag | (bits & 0xffffffffull));
                sv_st_msg(w + 1, tag | (bits >> 32));
            } else {
                sv_st_msg(w, tag | __float_as_uint(pv));
            }
        }
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

// The same on contiguous vectors (increments both 1 or both -1: element pairs share their memory index, so the raw
// regions [x, x + n) and [y, y + n) are processed), 16-byte aligned: 16-byte loads and stores.
template <typename T>
__global__ void __launch_bounds__(256) l1x_vec(int mode, long long n, T *x, T *y, double a,
                                               double h11, double h12, double h21, double h22) {
    using R = typename Compute<T>::R;
    constexpr int W = V16<T>::W;
    const long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x, stride = (long long)gridDim.x * blockDim.x;
    const long long nv = n / W;
    for (long long v = tid; v < nv; v += stride) {
        T *px = x + v * W, *py = y + v * W;
        if (mode == 0) {
            *reinterpret_cast<uint4 *>(py) = *reinterpret_cast<const uint4 *>(px);
        } else if (mode == 2) {
            const uint4 tx = *reinterpret_cast<const uint4 *>(px), ty = *reinterpret_cast<const uint4 *>(py);
            *reinterpret_cast<uint4 *>(px) = ty;
            *reinterpret_cast<uint4 *>(py) = tx;
        } else if (mode == 1) {
            R xv[W];
            load16_rw<T>(px, xv);
#pragma unroll
            for (int k = 0; k < W; k++) xv[k] = (R)a * xv[k];
            store16<T>(px, xv);
        } else {
            R xv[W], yv[W], ox[W];
            load16_rw<T>(px, xv);
            load16_rw<T>(py, yv);
#pragma unroll
            for (int k = 0; k < W; k++) {
                ox[k] = fma_r((R)h11, xv[k], (R)h12 * yv[k]);
                yv[k] = fma_r((R)h21, xv[k], (R)h22 * yv[k]);
            }
            store16<T>(px, ox);
            store16<T>(py, yv);
        }
    }
    for (long long e = nv * W + tid; e < n; e += stride) {   // tail
        T *px = x + e, *py = y + e;
        if (mode == 1) { *px = from_r<T>((R)a * to_r(*px)); continue; }
        if (mode == 0) { *py = *px; continue; }
        if (mode == 2) { const T t = *px; *px = *py; *py = t; continue; }
        const R vx = to_r(*px), vy = to_r(*py);
        *px = from_r<T>(fma_r((R)h11, vx, (R)h12 * vy));
        *py = from_r<T>(fma_r((R)h21, vx, (R)h22 * vy));
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
static int tri_mv_t(const L2Mat &m, double alpha, const void *x, long long ox, long long ix, double beta, void *y,
                    long long oy, long long iy, cudaStream_t st) {
    using R = typename Compute<T>::R;
    const int nrb = (m.n + kTriRows - 1) / kTriRows, np = (m.n + kTriPiece - 1) / kTriPiece;
    const int use_row = m.kind == l2x::kSymmetric || !m.trans, use_col = m.kind == l2x::kSymmetric || m.trans;
    void *p = nullptr;
    G9_TRY(scratch((size_t)(np + nrb) * m.n * sizeof(R), &p));
    R *Prow = (R *)p, *Pcol = Prow + (size_t)np * m.n;
    const size_t va = sizeof(T) == 2 ? 8 : 16;
    const bool vec = m.layout == l2x::kDense && ((uintptr_t)m.A % va) == 0 && ((size_t)m.lda * sizeof(T)) % va == 0;
    if (vec) l2x_tri_strip<T, true><<<dim3(np, nrb), 256, 0, st>>>(m, use_row, use_col, (const T *)x, ox, ix, Prow, Pcol);
    else l2x_tri_strip<T, false><<<dim3(np, nrb), 256, 0, st>>>(m, use_row, use_col, (const T *)x, ox, ix, Prow, Pcol);
    G9_TRY(launched("l2x_tri_strip"));
    l2x_tri_final<T><<<(m.n + 31) / 32, 256, 0, st>>>(m, use_row, use_col, Prow, Pcol, (R)alpha, (R)beta, (T *)y, oy,
                                                      iy);
    return launched("l2x_tri_final");
}

template <typename T>
static int mv_t(const L2Mat &m, double alpha, const void *x, long long ox, long long ix, double beta, void *y,
                long long oy, long long iy, cudaStream_t st) {
    using R = typename Compute<T>::R;
    if (m.layout != l2x::kBand && m.kind != l2x::kGeneral && m.n <= 65535 * kTriRows)
        return tri_mv_t<T>(m, alpha, x, ox, ix, beta, y, oy, iy, st);
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

// op(A)·z = x in place through the look-back kernel (any layout; band: back = the blocks the band reaches).
template <typename T>
static int trsv_lb_t(const L2Mat &m, void *x, long long ox, long long ix, cudaStream_t st) {
    DevState *d = dev_state();
    if (!d) return G.status;
    SvArgs a;
    a.m = m;
    a.rev = (m.upper != 0) != (m.trans != 0);   // op(A) upper
    a.x = x;
    a.ox = ox;
    a.ix = ix;
    a.nb = (m.n + kSvNb - 1) / kSvNb;
    a.back = m.layout == l2x::kBand ? (m.KL + m.KU + kSvNb - 1) / kSvNb : 0;
    a.err = d->err_dev;
    a.limit_ns = 1000000000ull;
    const size_t words = (size_t)a.nb * kSvNb * 2;   // enough for FP64 (two words per value)
    if (d->sv_msg_n < words) {
        if (d->sv_msg) {
            G9_CU(cudaStreamSynchronize(st));
            G9_CU(cudaFree(d->sv_msg));
            d->sv_msg = nullptr;
        }
        const size_t want = (words + 65535) & ~(size_t)65535;
        G9_CU(cudaMalloc((void **)&d->sv_msg, want * sizeof(unsigned long long)));
        G9_CU(cudaMemsetAsync(d->sv_msg, 0, want * sizeof(unsigned long long), st));
        d->sv_msg_n = want;
    }
    if (++d->sv_epoch == 0) d->sv_epoch = 1;
    a.msg = d->sv_msg;
    a.epoch = d->sv_epoch;
    static int per_sm[kMaxDevices] = {};
    static bool attr[kMaxDevices] = {};
    constexpr size_t smem = sv_smem_bytes<T>();
    G9_CU(smem_limit_once(l2x_trsv_lb<T>, (int)smem, attr));
    if (!per_sm[d->dev]) G9_CU(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm[d->dev], l2x_trsv_lb<T>, 256, smem));
    int grid = per_sm[d->dev] * d->sm_count;
    if (grid > a.nb) grid = a.nb;
    if (grid < 1) return fail(GEN9BLAS_ERR, "triangular solve kernel does not fit on an SM");
    void *args[] = {&a};
    G9_CU(cudaLaunchCooperativeKernel((const void *)l2x_trsv_lb<T>, dim3(grid), dim3(256), args, smem, st));
    return launched("l2x_trsv_lb");
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
    vec_strided(op[0], n, incx, es);
    if (two) {
        G9_TRY(map_operand(op[1], y, vec_span(n, incy) * es, 1, mode != 0 || (incy != 1 && incy != -1), true));
        vec_strided(op[1], n, incy, es);
    }
    timer_kernel();
    const long long ox = vec_off(n, incx), oy = two ? vec_off(n, incy) : 0;
    cudaStream_t st = stream();
    const bool contiguous = (incx == 1 || incx == -1) && (!two || incy == incx) &&
                            (((uintptr_t)op[0].dptr | (two ? (uintptr_t)op[1].dptr : 0)) & 15) == 0;
#define G9_L1X(TT)                                                                                                   \
    if (contiguous)                                                                                                  \
        l1x_vec<TT><<<l2x_grid((n + V16<TT>::W - 1) / V16<TT>::W), 256, 0, st>>>(                                    \
            mode, n, (TT *)op[0].dptr, two ? (TT *)op[1].dptr : (TT *)op[0].dptr, a, h11, h12, h21, h22);             \
    else                                                                                                             \
        l1x<TT><<<l2x_grid(n), 256, 0, st>>>(mode, n, (TT *)op[0].dptr, ox, incx, two ? (TT *)op[1].dptr : nullptr,  \
                                             oy, incy, a, h11, h12, h21, h22)
    if (type == GEN9BLAS_S) { G9_L1X(float); }
    else if (type == GEN9BLAS_D) { G9_L1X(double); }
    else { G9_L1X(__half); }
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
    vec_strided(op[2], m.rows, incy, es);
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
    vec_strided(op[1], m.rows, incx, es);
    timer_kernel();
    m.A = op[0].dptr;
    G9_TRY(L2X_DISPATCH(mv_inplace_t, m, op[1].dptr, vec_off(m.rows, incx), incx, stream()));
    G.last_zc = op[0].zc | op[1].zc << 1;
    int r = finish_op(op, 2);
    timer_stop();
    return r;
}

// op(A)·z = x in place (trsv, tpsv, tbsv).
int solve_call(int type, int es, L2Mat m, size_t abytes, void *x, int incx) {
    timer_start();
    Operand op[2];
    G9_TRY(map_operand(op[0], m.A, abytes, 0, true, false));
    G9_TRY(map_operand(op[1], x, vec_span(m.n, incx) * es, 1, true, true));
    vec_strided(op[1], m.n, incx, es);
    timer_kernel();
    m.A = op[0].dptr;
    G9_TRY(L2X_DISPATCH(trsv_lb_t, m, op[1].dptr, vec_off(m.n, incx), incx, stream()));
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
    const L2Mat m = mat(A, lda, l2x::kDense, l2x::kTriangular, n, n, uplo == GEN9BLAS_UPPER, trans ? 1 : 0,
                        diag == GEN9BLAS_UNIT, 0, 0, n);
    return solve_call(type, es, m, dense_bytes(n, n, lda, es), x, incx);
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
    const L2Mat m = mat(A, lda, l2x::kBand, l2x::kTriangular, N, N, up, trans ? 1 : 0, diag == GEN9BLAS_UNIT,
                        up ? 0 : K, up ? K : 0, N);
    return solve_call(type, es, m, dense_bytes(N, K + 1, lda, es), x, incx);
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
    const L2Mat m = mat(Ap, 0, l2x::kPacked, l2x::kTriangular, N, N, uplo == GEN9BLAS_UPPER, trans ? 1 : 0,
                        diag == GEN9BLAS_UNIT, 0, 0, N);
    return solve_call(type, es, m, packed_bytes(N, es), x, incx);
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
