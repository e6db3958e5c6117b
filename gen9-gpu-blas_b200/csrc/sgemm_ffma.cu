// sgemm_ffma.cu -- FP32 GEMM (SGEMM) on the FFMA pipe.
//
// Replaces the reference's sgemm_v (lib/kernels/sgemm.cl:200-230: 16×16 tile per SIMD16 subgroup on packed, zero-padded
// panels, FMA along K, epilogue sgemm.cl:192-198). The result must stay plain FP32 FMA arithmetic (the reference's
// SGEMM tolerance is FP32's), so this is a SIMT kernel, not a tensor-core one. B200 design:
//   - CTA tile 128×128, 256 threads, 8×8 outputs per thread as four 4×4 quadrants (rows r, r + 64; columns c, c + 64);
//     warps are 32×64 blocks of the tile, so each 16-byte shared-memory fragment read of a warp touches 64 or 128
//     contiguous bytes (one wavefront) and every FFMA operand comes from registers;
//   - op(A) and op(B) tiles of K = 16 go global → shared memory with cp.async in a 4-stage ring (three tiles in flight
//     while one is consumed). Both are stored K-major ([k][m], [k][n], 4-float row pad): an operand that is contiguous
//     along M or N is copied 16 bytes at a time, one contiguous along K is transposed on the way with 4-byte copies
//     (8 lanes per stored row so that a warp reads four full 32-byte sectors; the pad spreads the 4-byte writes over
//     all 32 banks). Outside the matrix the copies zero-fill, so any M, N, K, leading dimension and transpose runs
//     without packing;
//   - the FMAs are issued as sm_100's paired fma.rn.f32x2 (two columns of the thread's block per instruction), which
//     halves the FMA instruction count so that fragment loads, copies and loop control no longer take issue slots
//     from the FMA pipe; results are bit-identical to scalar fmaf;
//   - two CTAs per SM (128 registers a thread);
//   - grids smaller than two CTAs per SM split K: each CTA writes its FP32 partial tile to scratch and a second kernel
//     sums the partials in fixed order and applies alpha·sum + beta·C (deterministic);
//   - epilogue alpha·acc + beta·C (beta = 0: C is not read), 16-byte stores where aligned.
#include "common.cuh"
#include "internal.h"

namespace g9 {

namespace sg {
constexpr int BM = 128, BN = 128, THREADS = 256, PAD = 4;
constexpr int LDS_ = BM + PAD;                       // pitch of a stored K row (BM == BN)
constexpr int SMS = 148;
}  // namespace sg

__device__ __forceinline__ void cp_async4(float *dst, const float *src, int src_bytes) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"((unsigned)__cvta_generic_to_shared(dst)), "l"(src),
                 "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async16(float *dst, const float *src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"((unsigned)__cvta_generic_to_shared(dst)),
                 "l"(src), "r"(src_bytes)
                 : "memory");
}
// Paired FP32 arithmetic of sm_100 (fma.rn.f32x2): two independent round-to-nearest FMAs in one instruction, each
// bit-identical to a scalar fmaf.
__device__ __forceinline__ unsigned long long f2_pack(float x, float y) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(x), "f"(y));
    return r;
}
__device__ __forceinline__ float2 f2_unpack(unsigned long long v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}
__device__ __forceinline__ void f2_fma(unsigned long long &c, unsigned long long a, unsigned long long b) {
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(c) : "l"(a), "l"(b));
}

__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N_> __device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N_) : "memory"); }

// Copies successive (BK × 128) K-major windows of one operand into shared memory s[k][x] (pitch LDS_). Pointers and
// row predicates are set up once per CTA; each tile only advances them.
//   KCONT = true : the stored matrix is X[x][k] (K contiguous): 4-byte transposing copies, 4 per thread (thread: one k,
//                  rows xs + 32·i);
//   KCONT = false: the stored matrix is X[k][x] (x contiguous): one 16-byte copy per thread (VEC) or four 4-byte
//                  copies (rows k = tid/128 + 2·i).
template <bool KCONT, bool VEC, int BK> struct TileLoader {
    // KCONT: BK/2 copies, copy c at k = tid%8 + 8·(c % KH), x = tid/8 + 32·(c / KH);
    // VEC:   BK/8 copies, copy c at k = tid/32 + 8·c, x = 4·(tid%32);
    // else:  BK/2 copies, copy c at k = tid/128 + 2·c, x = tid%128.
    static constexpr int KH = BK / 8;
    static constexpr int NC = KCONT ? BK / 2 : VEC ? BK / 8 : BK / 2;
    const float *p0;     // address of copy 0 in tile 0 (any valid address when no copy is inside the matrix)
    long long ld;        // leading dimension
    long long tstep;     // element offset from one tile to the next
    int valid;           // bit g: copies of row group g lie inside the matrix (rows / columns other than k)
    int nb;              // bytes of a 16-byte copy at the matrix edge
    int k0;              // k of copy 0 relative to the tile origin
    int s0;              // shared-memory offset of copy 0

    __device__ __forceinline__ void init(const float *X, long long ld_, int nx, int x0, int kbeg, int tid) {
        using namespace sg;
        ld = ld_;
        valid = 0;
        nb = 4;
        if (KCONT) {
            tstep = BK;
            const int x = tid / 8;
            k0 = tid % 8;
            p0 = X + (long long)(x0 + x) * ld + kbeg + k0;
#pragma unroll
            for (int g = 0; g < NC / KH; g++) valid |= (x0 + x + 32 * g < nx) << g;
            s0 = k0 * LDS_ + x;
        } else if (VEC) {
            tstep = BK * ld;
            const int x = (tid % (BM / 4)) * 4;
            k0 = tid / (BM / 4);
            const int rem = nx - (x0 + x);
            p0 = X + (long long)(kbeg + k0) * ld + x0 + x;
            valid = rem > 0;
            nb = rem >= 4 ? 16 : rem * 4;
            s0 = k0 * LDS_ + x;
        } else {
            tstep = BK * ld;
            const int x = tid % BM;
            k0 = tid / BM;
            p0 = X + (long long)(kbeg + k0) * ld + x0 + x;
            valid = x0 + x < nx;
            s0 = k0 * LDS_ + x;
        }
        if (!valid) p0 = X;
    }
    // Issues tile t; krem = number of k positions of the tile inside the CTA's K range (copies beyond it zero-fill).
    __device__ __forceinline__ void issue(float *s, int t, int krem) {
        using namespace sg;
        const float *pt = p0 + (long long)t * tstep;
#pragma unroll
        for (int c = 0; c < NC; c++) {
            if (KCONT) {
                const int kc = 8 * (c % KH), g = c / KH;
                const bool in = ((valid >> g) & 1) && k0 + kc < krem;
                cp_async4(s + s0 + kc * LDS_ + 32 * g, in ? pt + 32 * g * ld + kc : p0, in ? 4 : 0);
            } else if (VEC) {
                const bool in = valid && k0 + 8 * c < krem;
                cp_async16(s + s0 + 8 * c * LDS_, in ? pt + 8 * c * ld : p0, in ? nb : 0);
            } else {
                const bool in = valid && k0 + 2 * c < krem;
                cp_async4(s + s0 + 2 * c * LDS_, in ? pt + 2 * c * ld : p0, in ? 4 : 0);
            }
        }
    }
};

// Main loop of one 128 × 128 tile over k in [kbeg, kend): acc2[i][q] = outputs (row i, columns 2q and 2q + 1) of the
// thread's 8 × 8 block as FP32 pairs, accumulated in k order. The shared-memory ring must be free on entry (the caller
// synchronises between tiles); on return every cp.async group has completed.
template <bool TA, bool TB, bool VA, bool VB, int BK, int STAGES>
__device__ __forceinline__ void sg_mainloop(const float *A, long long lda, const float *B, long long ldb, int M, int N,
                                            int m0, int n0, int kbeg, int kend, float *smem,
                                            unsigned long long (&acc2)[8][4]) {
    using namespace sg;
    float(*As)[BK][LDS_] = reinterpret_cast<float(*)[BK][LDS_]>(smem);
    float(*Bs)[BK][LDS_] = reinterpret_cast<float(*)[BK][LDS_]>(smem + STAGES * BK * LDS_);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int rm = (warp >> 1) * 16 + (lane >> 3) * 4;   // first row of the thread's upper quadrants
    const int cn = (warp & 1) * 32 + (lane & 7) * 4;     // first column of the thread's left quadrants
    TileLoader<!TA, VA, BK> la;
    TileLoader<TB, VB, BK> lb;
    la.init(A, lda, M, m0, kbeg, tid);
    lb.init(B, ldb, N, n0, kbeg, tid);
    // krem: k positions of tile t that lie inside [kbeg, kend)
    auto issue = [&](int stage, int t) {
        const int krem = kend - kbeg - t * BK;
        la.issue(&As[stage][0][0], t, krem);
        lb.issue(&Bs[stage][0][0], t, krem);
    };
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int q = 0; q < 4; q++) acc2[i][q] = 0ull;
    const int nk = (kend - kbeg + BK - 1) / BK;
#pragma unroll
    for (int s = 0; s < STAGES - 1; s++) {
        if (s < nk) issue(s, s);
        cp_commit();
    }
    for (int kb = 0; kb < nk; kb++) {
        cp_wait<STAGES - 2>();
        __syncthreads();
        {
            const int kn = kb + STAGES - 1;
            if (kn < nk) issue(kn % STAGES, kn);
            cp_commit();
        }
        const int s = kb % STAGES;
#pragma unroll
        for (int k = 0; k < BK; k++) {
            const float4 a0 = *reinterpret_cast<const float4 *>(&As[s][k][rm]);
            const float4 a1 = *reinterpret_cast<const float4 *>(&As[s][k][rm + 64]);
            const float4 b0 = *reinterpret_cast<const float4 *>(&Bs[s][k][cn]);
            const float4 b1 = *reinterpret_cast<const float4 *>(&Bs[s][k][cn + 64]);
            const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const unsigned long long b2[4] = {f2_pack(b0.x, b0.y), f2_pack(b0.z, b0.w), f2_pack(b1.x, b1.y),
                                              f2_pack(b1.z, b1.w)};
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const unsigned long long ai = f2_pack(a[i], a[i]);
#pragma unroll
                for (int q = 0; q < 4; q++) f2_fma(acc2[i][q], ai, b2[q]);
            }
        }
    }
    cp_wait<0>();
}

// Epilogue of a tile: C = alpha·acc + beta·C (beta = 0: C is not read), or (partial != nullptr) the raw sums into the
// dense M × N partial matrix.
__device__ __forceinline__ void sg_store(const unsigned long long (&acc2)[8][4], int M, int N, int m0, int n0,
                                         float alpha, float beta, float *C, long long ldc, int c_vec, float *partial) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int rm = (warp >> 1) * 16 + (lane >> 3) * 4;
    const int cn = (warp & 1) * 32 + (lane & 7) * 4;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int m = m0 + rm + (i & 3) + (i >> 2) * 64;
        if (m >= M) continue;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int n = n0 + cn + h * 64;
            const float2 v01 = f2_unpack(acc2[i][2 * h]), v23 = f2_unpack(acc2[i][2 * h + 1]);
            const float v[4] = {v01.x, v01.y, v23.x, v23.y};
            if (partial) {
                float *p = partial + (long long)m * N + n;
                if (c_vec && n + 3 < N) {
                    *reinterpret_cast<float4 *>(p) = make_float4(v[0], v[1], v[2], v[3]);
                } else {
#pragma unroll
                    for (int e = 0; e < 4; e++)
                        if (n + e < N) p[e] = v[e];
                }
                continue;
            }
            float *p = C + (long long)m * ldc + n;
            if (c_vec && n + 3 < N) {
                float4 o = make_float4(alpha * v[0], alpha * v[1], alpha * v[2], alpha * v[3]);
                if (beta != 0.f) {
                    const float4 c = *reinterpret_cast<const float4 *>(p);
                    o.x = __fmaf_rn(beta, c.x, o.x);
                    o.y = __fmaf_rn(beta, c.y, o.y);
                    o.z = __fmaf_rn(beta, c.z, o.z);
                    o.w = __fmaf_rn(beta, c.w, o.w);
                }
                *reinterpret_cast<float4 *>(p) = o;
            } else {
#pragma unroll
                for (int e = 0; e < 4; e++)
                    if (n + e < N) p[e] = beta != 0.f ? __fmaf_rn(beta, p[e], alpha * v[e]) : alpha * v[e];
            }
        }
    }
}

// partial == nullptr: C = alpha·op(A)·op(B) + beta·C over the whole K (blockIdx.z = batch index).
// partial != nullptr: split K (count == 1): CTA z sums k in [z·kper, (z+1)·kper) and stores its raw tile to
// partial[z] (M × N, dense).
template <bool TA, bool TB, bool VA, bool VB, int BK, int STAGES>
__global__ void __launch_bounds__(sg::THREADS, 2)
sgemm_ffma_kernel(int M, int N, int K, float alpha, const float *__restrict__ A, long long lda, long long sA,
                  const float *__restrict__ B, long long ldb, long long sB, float beta, float *C, long long ldc,
                  long long sC, int c_vec, int kper, float *__restrict__ partial) {
    using namespace sg;
    // Programmatic dependent launch: the next kernel may start while this one runs (it waits before its own loads);
    // this one waits for its predecessor before the first operand access.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    extern __shared__ __align__(16) float sg_smem[];
    const int z = blockIdx.z;
    int kbeg = 0, kend = K;
    if (partial) {
        kbeg = z * kper;
        kend = min(K, kbeg + kper);
        partial += (long long)z * M * N;
    } else {
        A += z * sA;
        B += z * sB;
        C += z * sC;
    }
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    unsigned long long acc2[8][4];
    sg_mainloop<TA, TB, VA, VB, BK, STAGES>(A, lda, B, ldb, M, N, m0, n0, kbeg, kend, sg_smem, acc2);
    sg_store(acc2, M, N, m0, n0, alpha, beta, C, ldc, c_vec, partial);
}

// Stream-K SGEMM for grids of less than one wave (count == 1): the tiles × KI iterations (KI = K chunks of BK) in
// (tile, k) order are split evenly over a one-wave grid (CTA c owns [T·c/G, T·(c+1)/G)), so every SM does the same
// number of FMAs whatever the tile count. A tile lying wholly in a CTA is stored directly. A tile shared by several
// CTAs is finished by the CTA that owns its first chunk, which reaches it in its last segment: each later CTA meets
// the tile in its first segment, leaves its FP32 partial sums in a slot of `part` and raises the slot's flag with
// this launch's epoch (release); the finisher waits for the flags (acquire, bounded: 4 s, then the device error word
// is set and the tile is not stored) and adds the slots in CTA order (deterministic) before the epilogue.
template <bool TA, bool TB, bool VA, bool VB, int BK, int STAGES>
__global__ void __launch_bounds__(sg::THREADS, 2)
sgemm_sk_kernel(int M, int N, int K, float alpha, const float *__restrict__ A, long long lda,
                const float *__restrict__ B, long long ldb, float beta, float *C, long long ldc, int c_vec, int tiles_n,
                int KI, int maxc, float *__restrict__ part, unsigned *flags, unsigned epoch, unsigned *err) {
    using namespace sg;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    extern __shared__ __align__(16) float sg_smem[];
    __shared__ int abort_flag;
    const int G_ = gridDim.x, c = blockIdx.x, tid = threadIdx.x;
    const long long tiles = (long long)tiles_n * ((M + BM - 1) / BM);
    const long long T = tiles * KI;
    long long x = T * c / G_;
    const long long x1 = T * (c + 1) / G_;
    unsigned long long acc2[8][4];
    while (x < x1) {
        const long long tile = x / KI;
        const int k0 = (int)(x % KI), k1 = (int)min((long long)KI, k0 + (x1 - x));
        const int m0 = (int)(tile / tiles_n) * BM, n0 = (int)(tile % tiles_n) * BN;
        __syncthreads();   // the previous segment's stages have been read
        sg_mainloop<TA, TB, VA, VB, BK, STAGES>(A, lda, B, ldb, M, N, m0, n0, k0 * BK, min(K, k1 * BK), sg_smem, acc2);
        const long long y0 = tile * KI;
        const int cf = (int)(((y0 + 1) * G_ - 1) / T), cl = (int)(((y0 + KI) * G_ - 1) / T);   // first / last CTA
        // slot layout: element pair q of thread tid at [q][tid] (coalesced float2 accesses)
        if (k0 > 0) {   // a later part of the tile: hand the partial sums over
            float2 *sl = reinterpret_cast<float2 *>(part + (tile * (maxc - 1) + (c - cf - 1)) * (long long)(BM * BN));
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int q = 0; q < 4; q++) sl[(i * 4 + q) * THREADS + tid] = f2_unpack(acc2[i][q]);
            __threadfence();
            __syncthreads();
            if (tid == 0) asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(flags + tile * (maxc - 1) + (c - cf - 1)),
                                       "r"(epoch)
                                       : "memory");
        } else {
            if (cl > c) {   // the finisher of a shared tile: the later parts, in CTA order
                if (tid == 0) {
                    abort_flag = 0;
                    for (int q = c + 1; q <= cl; q++) {
                        const unsigned *f = flags + tile * (maxc - 1) + (q - cf - 1);
                        unsigned v;
                        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
                        if (v != epoch) {
                            unsigned long long t0, t;
                            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
                            for (;;) {
                                asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
                                if (v == epoch) break;
                                asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
                                if (t - t0 > 4000000000ull) {
                                    abort_flag = 1;
                                    break;
                                }
                            }
                        }
                        if (abort_flag) break;
                    }
                }
                __syncthreads();
                if (abort_flag) {
                    if (tid == 0) *(volatile unsigned *)err = kDevErrWaitTimeout;
                    x += k1 - k0;
                    continue;
                }
                for (int q = c + 1; q <= cl; q++) {
                    const float2 *sl =
                        reinterpret_cast<const float2 *>(part + (tile * (maxc - 1) + (q - cf - 1)) * (long long)(BM * BN));
#pragma unroll
                    for (int i = 0; i < 8; i++)
#pragma unroll
                        for (int r = 0; r < 4; r++) {
                            const float2 v = __ldcg(&sl[(i * 4 + r) * THREADS + tid]);
                            float2 a = f2_unpack(acc2[i][r]);
                            a.x += v.x;
                            a.y += v.y;
                            acc2[i][r] = f2_pack(a.x, a.y);
                        }
                }
            }
            sg_store(acc2, M, N, m0, n0, alpha, beta, C, ldc, c_vec, nullptr);
        }
        x += k1 - k0;
    }
}

// C = alpha·Σ_z partial[z] + beta·C, partials summed in ascending z.
__global__ void sgemm_splitk_sum(int M, int N, int S, float alpha, const float *__restrict__ partial, float beta, float *C,
                                 long long ldc) {
    const long long total = (long long)M * N;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x) {
        float s = partial[e];
        for (int z = 1; z < S; z++) s += partial[(long long)z * total + e];
        const int m = (int)(e / N), n = (int)(e % N);
        float *p = C + (long long)m * ldc + n;
        *p = beta != 0.f ? __fmaf_rn(beta, *p, alpha * s) : alpha * s;
    }
}

template <bool TA, bool TB, int BK, int STAGES>
static int sg_go(bool va, bool vb, dim3 grid, cudaStream_t st, int M, int N, int K, float alpha, const float *a,
                 long long lda, long long sA, const float *b, long long ldb, long long sB, float beta, float *c,
                 long long ldc, long long sC, int c_vec, int kper, float *partial) {
    constexpr int smem = 2 * STAGES * BK * sg::LDS_ * (int)sizeof(float);
    // The vector flag only matters for an operand that is contiguous along M / N (A transposed, B not transposed).
    va = TA && va;
    vb = !TB && vb;
#define G9_SG(VA_, VB_)                                                                                                \
    do {                                                                                                               \
        auto k = sgemm_ffma_kernel<TA, TB, VA_, VB_, BK, STAGES>;                                                      \
        static bool attr[kMaxDevices] = {};                                                                            \
        G9_CU(smem_limit_once(k, smem, attr));                                                                         \
        launch_pdl(k, grid, dim3(sg::THREADS), smem, st, M, N, K, alpha, a, lda, sA, b, ldb, sB, beta, c, ldc, sC,     \
                   c_vec, kper, partial);                                                                              \
    } while (0)
    if (va && vb) G9_SG(TA, !TB);
    else if (va) G9_SG(TA, false);
    else if (vb) G9_SG(false, !TB);
    else G9_SG(false, false);
#undef G9_SG
    return 0;
}

template <bool TA, bool TB, int BK, int STAGES>
static int sk_go(bool va, bool vb, int grid, cudaStream_t st, int M, int N, int K, float alpha, const float *a, long long lda,
                 const float *b, long long ldb, float beta, float *c, long long ldc, int c_vec, int tiles_n, int KI,
                 int maxc, float *part, unsigned *flags, unsigned epoch, unsigned *err) {
    constexpr int smem = 2 * STAGES * BK * sg::LDS_ * (int)sizeof(float);
    va = TA && va;
    vb = !TB && vb;
#define G9_SK(VA_, VB_)                                                                                                \
    do {                                                                                                               \
        auto k = sgemm_sk_kernel<TA, TB, VA_, VB_, BK, STAGES>;                                                        \
        static bool attr[kMaxDevices] = {};                                                                            \
        G9_CU(smem_limit_once(k, smem, attr));                                                                         \
        launch_pdl(k, dim3(grid), dim3(sg::THREADS), smem, st, M, N, K, alpha, a, lda, b, ldb, beta, c, ldc, c_vec,    \
                   tiles_n, KI, maxc, part, flags, epoch, err);                                                        \
    } while (0)
    if (va && vb) G9_SK(TA, !TB);
    else if (va) G9_SK(TA, false);
    else if (vb) G9_SK(false, !TB);
    else G9_SK(false, false);
#undef G9_SK
    return launched("sgemm_sk");
}

template <int BK, int STAGES>
static int sg_cfg(int tA, int tB, int M, int N, int K, float al, const float *a, int lda, long long sA, const float *b,
                  int ldb, long long sB, float be, float *c, int ldc, long long sC, int count, cudaStream_t st,
                  bool va, bool vb, int c_vec) {
    using namespace sg;
    const int tiles_n = (N + BN - 1) / BN, tiles_m = (M + BM - 1) / BM;
    if (tiles_m > 65535 || count > 65535)
        return fail(GEN9BLAS_ERR_INVALID_ARG, "SGEMM grid too large (M %d, count %d)", M, count);
    // Stream-K for a single GEMM of less than one wave of tiles (two CTAs per SM) with K >= 256: the tile × K-chunk
    // iterations are spread evenly over a one-wave grid (sgemm_sk_kernel), so no SM idles or does twice the work of
    // another, and the partial sums of a shared tile stay in L2 until its finisher adds them.
    {
        DevState *d = dev_state();
        if (!d) return G.status;
        const long long tiles = (long long)tiles_m * tiles_n;
        const int KI = (K + BK - 1) / BK, G_ = 2 * d->sm_count;
        const long long T = tiles * KI;
        if (count == 1 && K >= 256 && tiles < G_ && T / G_ >= 4) {
            int maxc = 2;
            for (long long t = 0; t < tiles; t++) {   // CTAs that share tile t: the first and last owners of its chunks
                const long long y0 = t * KI;
                const int cf = (int)(((y0 + 1) * G_ - 1) / T), cl = (int)(((y0 + KI) * G_ - 1) / T);
                if (cl - cf + 1 > maxc) maxc = cl - cf + 1;
            }
            if (tiles * (maxc - 1) <= kGemmFlags) {
                void *p = nullptr;
                G9_TRY(scratch((size_t)tiles * (maxc - 1) * BM * BN * sizeof(float), &p));
                unsigned *flags = nullptr, epoch = 0;
                G9_TRY(gemm_handoff(d, st, &flags, &epoch));
#define G9_SKT(TA_, TB_)                                                                                              \
    return sk_go<TA_, TB_, BK, STAGES>(va, vb, G_, st, M, N, K, al, a, lda, b, ldb, be, c, ldc, c_vec, tiles_n, KI, maxc, \
                                        (float *)p, flags, epoch, d->err_dev)
                if (!tA && !tB) G9_SKT(false, false);
                else if (tA && !tB) G9_SKT(true, false);
                else if (!tA && tB) G9_SKT(false, true);
                else G9_SKT(true, true);
#undef G9_SKT
            }
        }
    }
    // Split K (4 parts, 2 for K < 512) when one matrix fills less than 60 % of one wave (two CTAs per SM), or less than
    // one wave with K >= 2048, where the partial tiles' round trip through HBM is small against the K loop. Measured on
    // B200: n = 1024 (64 tiles) 20 TF/s unsplit, 34 with 4 parts; M = 512, N = 8960, K = 1536 (280 tiles): 4 parts cost
    // 12 %; the K = 4096 band GEMMs of SYRK / TRMM (192-256 tiles) gain 8-11 % from splitting; n = 2048 1.5 %. Three
    // parts load the SMs unevenly and are slower than two.
    int S = 1, kper = K;
    const long long tiles = (long long)tiles_m * tiles_n;
    if (count == 1 && K >= 256 && (tiles * 10 < 2 * SMS * 6 || (tiles < 2 * SMS && K >= 2048))) S = K >= 512 ? 4 : 2;
    if (S > 1) {
        kper = ((K + S - 1) / S + BK - 1) / BK * BK;
        S = (K + kper - 1) / kper;
    }
    float *partial = nullptr;
    if (S > 1) {
        void *p = nullptr;
        G9_TRY(scratch((size_t)S * M * N * sizeof(float), &p));
        partial = (float *)p;
    }
    const int p_vec = partial && N % 4 == 0;
    dim3 grid(tiles_n, tiles_m, S > 1 ? S : count);
#define G9_SGT(TA_, TB_)                                                                                              \
    G9_TRY((sg_go<TA_, TB_, BK, STAGES>(va, vb, grid, st, M, N, K, al, a, lda, sA, b, ldb, sB, be, c, ldc, sC,     \
                                         partial ? p_vec : c_vec, kper, partial)))
    if (!tA && !tB) G9_SGT(false, false);
    else if (tA && !tB) G9_SGT(true, false);
    else if (!tA && tB) G9_SGT(false, true);
    else G9_SGT(true, true);
#undef G9_SGT
    if (S > 1) {
        G9_TRY(launched("sgemm_ffma"));
        const long long total = (long long)M * N;
        const int blocks = (int)((total + 255) / 256 < 8 * SMS ? (total + 255) / 256 : 8 * SMS);
        sgemm_splitk_sum<<<blocks, 256, 0, st>>>(M, N, S, al, partial, be, c, ldc);
        return launched("sgemm_splitk_sum");
    }
    return launched("sgemm_ffma");
}

int launch_sgemm(int tA, int tB, int M, int N, int K, double alpha, const void *A, int lda, long long sA, const void *B,
                 int ldb, long long sB, double beta, void *C, int ldc, long long sC, int count, cudaStream_t st) {
    const bool va = ((uintptr_t)A & 15) == 0 && lda % 4 == 0 && (count == 1 || sA % 4 == 0);
    const bool vb = ((uintptr_t)B & 15) == 0 && ldb % 4 == 0 && (count == 1 || sB % 4 == 0);
    const int c_vec = ((uintptr_t)C & 15) == 0 && ldc % 4 == 0 && (count == 1 || sC % 4 == 0);
    const float al = (float)alpha, be = (float)beta;
    // K = 16 per stage, 4 stages (67.6 KB of shared memory per CTA, two CTAs per SM).
    return sg_cfg<16, 4>(tA, tB, M, N, K, al, (const float *)A, lda, sA, (const float *)B, ldb, sB, be, (float *)C, ldc, sC,
                         count, st, va, vb, c_vec);
}

}  // namespace g9
