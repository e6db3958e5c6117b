// packed.cu -- constant weights kept on the GPU: gen9blas_pack_b / gen9blas_gemm_pb / gen9blas_packed_b_free and the
// small-batch product with F32 activations gen9blas_gemm_pb_skinny.
//
// Reference: lib/gen9blas.h:89-97 and lib/src/packed.c:70-89 (pack_b), 168-171 (packed_b_free), 174-213 (gemm_pb),
// lib/gen9blas_ml.h:25-28 and packed.c:307-329 (gemm_pb_skinny). Same contract: pack_b copies op(B) (K × N; transB:
// B stored N × K) once, the caller may then overwrite or free B; gemm_pb computes C = alpha·op(A)·Bp + beta·C with A of
// the packed type; gemm_pb_skinny takes FP32 activations (M <= 16) against HS-packed FP16 weights and writes FP32;
// pack_b returns NULL on error; packed_b_free waits for queued work first.
//
// What differs on B200: the reference packs into the tile layout of its assembly GEMM, padded to its tile sizes and
// written in launch bands, because each gemm_pb then skips B's packing pass. Here the GEMM kernels read strided
// operands directly, so the packed form is op(B)ᵀ stored K-contiguous -- W[n][k], N rows of Kp elements (Kp = K
// rounded up to 16 bytes, the pad zeroed) in HBM of the GPU that packed it. That is the layout the tensor-core GEMM
// reads as a K-major TMA operand and the skinny decode kernels stream with 16-byte loads, so no call repacks B. The
// handle also owns a region for a zero-padded copy of a small A (M up to the skinny threshold), used when K is not a
// multiple of the 16-byte vector: with both operands padded to Kp every small-batch call takes the vector kernel.
#include "common.cuh"
#include "gen9blas_ml.h"
#include "internal.h"
#include <cstring>
#include <new>

using namespace g9;

struct gen9blas_packed_b {
    unsigned magic;
    int type, K, N, Kp;   // W: N × Kp elements
    int dev;              // CUDA device of the buffers
    int apad_rows;        // rows of the padded-A region (0: none, K is a multiple of the vector)
    void *w;              // packed weights, followed by the padded-A region
    size_t w_bytes;
};

namespace {

constexpr unsigned kPackedMagic = 0x67396262u;

int elem_bytes(int type) { return type == GEN9BLAS_S ? 4 : type == GEN9BLAS_D ? 8 : 2; }

// Band of rows [r0, r0 + rows) of op(B)'s source when B is stored K × N (pitch ls): W[c][r0 + r] = src[r][c].
// 32 × 32 tiles through shared memory (padded against bank conflicts); reads and writes are coalesced.
template <typename T>
__global__ void __launch_bounds__(256) pack_transpose(const T *__restrict__ src, long long ls, int rows, int cols,
                                                      T *__restrict__ dst, long long ldd, long long r0) {
    __shared__ T tile[32][33];
    const int c = blockIdx.x * 32 + threadIdx.x, rb = blockIdx.y * 32;
    for (int j = threadIdx.y; j < 32; j += 8) {
        const int r = rb + j;
        if (r < rows && c < cols) tile[j][threadIdx.x] = src[(long long)r * ls + c];
    }
    __syncthreads();
    const int r = rb + threadIdx.x, cb = blockIdx.x * 32;
    for (int j = threadIdx.y; j < 32; j += 8) {
        const int cc = cb + j;
        if (cc < cols && r < rows) dst[(long long)cc * ldd + r0 + r] = tile[threadIdx.x][j];
    }
}

// op(A) (M × K, element (m, k) at a[m·sm + k·sk]) into dst (M × Kp, zero past K): the padded small operand.
template <typename T>
__global__ void pad_rows(const T *__restrict__ a, long long sm, long long sk, int M, int K, int Kp, T *__restrict__ dst) {
    const long long n = (long long)M * Kp;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int m = (int)(i / Kp), k = (int)(i % Kp);
        dst[i] = k < K ? a[(long long)m * sm + (long long)k * sk] : T(0);
    }
}

template <typename T>
int launch_transpose_band(const void *src, long long ls, int rows, int cols, void *dst, long long ldd, long long r0,
                          cudaStream_t st) {
    dim3 grid((cols + 31) / 32, (rows + 31) / 32), block(32, 8);
    pack_transpose<T><<<grid, block, 0, st>>>((const T *)src, ls, rows, cols, (T *)dst, ldd, r0);
    return launched("pack_transpose");
}

int transpose_band(int es, const void *src, long long ls, int rows, int cols, void *dst, long long ldd, long long r0,
                   cudaStream_t st) {
    if (es == 2) return launch_transpose_band<uint16_t>(src, ls, rows, cols, dst, ldd, r0, st);
    if (es == 4) return launch_transpose_band<uint32_t>(src, ls, rows, cols, dst, ldd, r0, st);
    return launch_transpose_band<uint64_t>(src, ls, rows, cols, dst, ldd, r0, st);
}

int pad_small(int es, const void *a, long long sm, long long sk, int M, int K, int Kp, void *dst, int sms,
              cudaStream_t st) {
    const unsigned blocks = (unsigned)(((long long)M * Kp + 255) / 256 < sms * 4 ? ((long long)M * Kp + 255) / 256 : sms * 4);
    if (es == 2) pad_rows<uint16_t><<<blocks, 256, 0, st>>>((const uint16_t *)a, sm, sk, M, K, Kp, (uint16_t *)dst);
    else if (es == 4) pad_rows<uint32_t><<<blocks, 256, 0, st>>>((const uint32_t *)a, sm, sk, M, K, Kp, (uint32_t *)dst);
    else pad_rows<uint64_t><<<blocks, 256, 0, st>>>((const uint64_t *)a, sm, sk, M, K, Kp, (uint64_t *)dst);
    return launched("pad_rows");
}

bool device_resident(const void *p, int dev) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return (a.type == cudaMemoryTypeDevice && a.device == dev) || a.type == cudaMemoryTypeManaged;
}

// Fills P->w from B. transB: B is N × K (pitch ldb), one 2-D copy with the destination pitch Kp (host or device
// source). Otherwise B is K × N: a device-resident B is transposed in place of the copy; a host B goes through a
// bounded device buffer in bands of rows (64 MiB each), copied then transposed, so packing never holds a second full
// copy of the weights.
int fill_packed(gen9blas_packed_b *P, int tB, const void *B, int ldb, DevState *d, cudaStream_t st) {
    const int es = elem_bytes(P->type);
    const size_t row = (size_t)P->Kp * es;
    if (P->Kp > P->K)
        G9_CU(cudaMemset2DAsync((char *)P->w + (size_t)P->K * es, row, 0, (size_t)(P->Kp - P->K) * es, P->N, st));
    if (tB) {
        G9_CU(cudaMemcpy2DAsync(P->w, row, B, (size_t)ldb * es, (size_t)P->K * es, P->N, cudaMemcpyDefault, st));
        return 0;
    }
    const long long max_rows = 65535LL * 32;   // grid.y limit of the transpose
    if (device_resident(B, d->dev)) {
        for (long long k0 = 0; k0 < P->K; k0 += max_rows) {
            const int rows = (int)(P->K - k0 < max_rows ? P->K - k0 : max_rows);
            G9_TRY(transpose_band(es, (const char *)B + (size_t)k0 * ldb * es, ldb, rows, P->N, P->w, P->Kp, k0, st));
        }
        return 0;
    }
    const size_t band_bytes = (size_t)64 << 20;
    long long band = (long long)(band_bytes / ((size_t)P->N * es));
    if (band < 1) band = 1;
    if (band > max_rows) band = max_rows;
    if (band > P->K) band = P->K;
    void *tmp = nullptr;
    G9_CU(cudaMalloc(&tmp, (size_t)band * P->N * es));
    int r = 0;
    for (long long k0 = 0; k0 < P->K && r == 0; k0 += band) {
        const int rows = (int)(P->K - k0 < band ? P->K - k0 : band);
        cudaError_t e = cudaMemcpy2DAsync(tmp, (size_t)P->N * es, (const char *)B + (size_t)k0 * ldb * es,
                                          (size_t)ldb * es, (size_t)P->N * es, rows, cudaMemcpyDefault, st);
        if (e != cudaSuccess) r = cuda_fail(e, "cudaMemcpy2DAsync (pack band)", __FILE__, __LINE__);
        if (r == 0) r = transpose_band(es, tmp, P->N, rows, P->N, P->w, P->Kp, k0, st);
        // the next band overwrites tmp: finish this one first
        if (r == 0 && (e = cudaStreamSynchronize(st)) != cudaSuccess)
            r = cuda_fail(e, "cudaStreamSynchronize (pack band)", __FILE__, __LINE__);
    }
    cudaFree(tmp);
    return r < 0 ? r : 0;
}

int check_handle(const gen9blas_packed_b *P, DevState *d, const char *who) {
    if (!P || P->magic != kPackedMagic) return fail(GEN9BLAS_ERR_INVALID_ARG, "%s: no packed B", who);
    if (P->dev != d->dev)
        return fail(GEN9BLAS_ERR_INVALID_ARG, "%s: B was packed on device %d, the current device is %d", who, P->dev,
                    d->dev);
    return 0;
}

}  // namespace

extern "C" {

GEN9BLAS_API gen9blas_packed_b *gen9blas_pack_b(int type, int tB, int K, int N, const void *B, int ldb) {
    if (begin_op()) return nullptr;
    if (type < 0 || type > 3) {
        fail(GEN9BLAS_ERR_UNSUPPORTED, "type %d unavailable", type);
        return nullptr;
    }
    if (K <= 0 || N <= 0) {
        fail(GEN9BLAS_ERR_INVALID_ARG, "pack_b: K = %d, N = %d", K, N);
        return nullptr;
    }
    tB = tB ? 1 : 0;
    if (!B || ldb < (tB ? K : N)) {
        fail(GEN9BLAS_ERR_INVALID_ARG, "pack_b: %s (ldb = %d)", B ? "ldb below the row length" : "NULL B", ldb);
        return nullptr;
    }
    DevState *d = dev_state();
    if (!d) return nullptr;
    const int es = elem_bytes(type), vec = 16 / es;
    const int Kp = (K + vec - 1) / vec * vec;
    const int apad_rows = Kp != K ? skinny_threshold(type) : 0;
    const size_t wb = (size_t)N * Kp * es, ab = (size_t)apad_rows * Kp * es;
    auto *P = new (std::nothrow) gen9blas_packed_b;
    if (!P) {
        fail(GEN9BLAS_ERR_OUT_OF_MEMORY, "out of host memory");
        return nullptr;
    }
    *P = gen9blas_packed_b{kPackedMagic, type, K, N, Kp, d->dev, apad_rows, nullptr, wb + ab};
    timer_start();
    timer_kernel();
    cudaError_t e = cudaMalloc(&P->w, P->w_bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        delete P;
        fail(GEN9BLAS_ERR_OUT_OF_MEMORY, "pack_b: %zu bytes of device memory: %s", wb + ab, cudaGetErrorString(e));
        return nullptr;
    }
    cudaStream_t st = stream();
    int r = fill_packed(P, tB, B, ldb, d, st);
    if (r == 0) r = finish_op(nullptr, 0);
    if (r == 0 && G.nowait) {   // the packed copy must be complete before B can change
        e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) r = cuda_fail(e, "cudaStreamSynchronize", __FILE__, __LINE__);
    }
    timer_stop();
    if (r < 0) {
        cudaFree(P->w);
        delete P;
        return nullptr;
    }
    return P;
}

GEN9BLAS_API int gen9blas_gemm_pb(int tA, int M, double alpha, const void *A, int lda, const gen9blas_packed_b *P,
                                  double beta, void *C, int ldc) {
    if (int e = begin_op()) return e;
    DevState *d = dev_state();
    if (!d) return G.status;
    G9_TRY(check_handle(P, d, "gemm_pb"));
    if (M <= 0) return 0;
    tA = tA ? 1 : 0;
    const int K = P->K, N = P->N, es = elem_bytes(P->type);
    if (lda < (tA ? M : K) || ldc < N)
        return fail(GEN9BLAS_ERR_INVALID_ARG, "gemm_pb: lda = %d, ldc = %d for M = %d, N = %d, K = %d", lda, ldc, M, N, K);
    const size_t bA = (tA ? (size_t)(K - 1) * lda + M : (size_t)(M - 1) * lda + K) * es;
    const size_t bC = ((size_t)(M - 1) * ldc + N) * es;
    timer_start();
    Operand op[2];
    G9_TRY(map_operand(op[0], A, bA, 0, true, false));
    G9_TRY(map_operand(op[1], C, bC, 2, beta != 0.0 || ldc != N, true));
    G.last_zc = op[0].zc | 2 | op[1].zc << 2;
    timer_kernel();
    cudaStream_t st = stream();
    if (M <= P->apad_rows) {
        // Small batch with K off the vector: A padded with zeros to Kp like the weights, then the vector skinny kernel.
        void *apad = (char *)P->w + (size_t)N * P->Kp * es;
        G9_TRY(pad_small(es, op[0].dptr, tA ? 1 : lda, tA ? lda : 1, M, K, P->Kp, apad, d->sm_count, st));
        G9_TRY(launch_skinny(P->type, 0, 1, M, N, P->Kp, alpha, apad, P->Kp, P->w, P->Kp, beta, op[1].dptr, ldc, st));
    } else {
        G9_TRY(launch_gemm(P->type, tA, 1, M, N, K, alpha, op[0].dptr, lda, 0, P->w, P->Kp, 0, beta, op[1].dptr, ldc, 0, 1,
                           st));
    }
    int r = finish_op(op, 2);
    timer_stop();
    return r;
}

GEN9BLAS_API int gen9blas_gemm_pb_skinny(int M, const float *A, int lda, const gen9blas_packed_b *P, float *C, int ldc,
                                         int *nonfinite) {
    if (int e = begin_op()) return e;
    DevState *d = dev_state();
    if (!d) return G.status;
    if (nonfinite) *nonfinite = 0;
    if (!P || P->magic != kPackedMagic || P->type != GEN9BLAS_HS)
        return fail(GEN9BLAS_ERR_INVALID_ARG, "gemm_pb_skinny: needs B packed as GEN9BLAS_HS");
    if (M < 1 || M > 16) return GEN9BLAS_DECLINED;
    G9_TRY(check_handle(P, d, "gemm_pb_skinny"));
    const int K = P->K, N = P->N;
    if (lda < K || ldc < N)
        return fail(GEN9BLAS_ERR_INVALID_ARG, "gemm_pb_skinny: lda = %d, ldc = %d for N = %d, K = %d", lda, ldc, N, K);
    timer_start();
    Operand op[2];
    G9_TRY(map_operand(op[0], A, ((size_t)(M - 1) * lda + K) * 4, 0, true, false));
    G9_TRY(map_operand(op[1], C, ((size_t)(M - 1) * ldc + N) * 4, 2, ldc != N, true));
    G.last_zc = op[0].zc | 2 | op[1].zc << 2;
    const bool queued = G.nowait && op[0].zc && op[1].zc;   // no-wait: nothing is read back, *nonfinite stays 0
    *(volatile unsigned *)(d->err_host + 1) = 0u;
    timer_kernel();
    G9_TRY(launch_skinny_f32a(M, N, K, (const float *)op[0].dptr, lda, P->w, P->Kp, (float *)op[1].dptr, ldc,
                              d->err_dev + 1, stream()));
    int r = finish_op(op, 2);
    timer_stop();
    if (r == 0 && !queued && nonfinite) *nonfinite = *(volatile unsigned *)(d->err_host + 1) != 0u;
    return r;
}

GEN9BLAS_API void gen9blas_packed_b_free(gen9blas_packed_b *P) {
    if (!P || P->magic != kPackedMagic) return;
    int cur = -1;
    cudaGetDevice(&cur);
    if (cur != P->dev) cudaSetDevice(P->dev);
    cudaDeviceSynchronize();   // queued calls (no-wait mode, any stream) may still read the weights
    cudaFree(P->w);
    if (cur >= 0 && cur != P->dev) cudaSetDevice(cur);
    P->magic = 0;
    delete P;
}


// ==================================================================================== FP16-weight GEMMs (gen9blas_ml.h)
// The reference's gemm_pb_f16w family (lib/src/packed.c:250-330, 365-474; kernels gen9blas_epilog_hf8x,
// gen9blas_swiglu_pack_a3, gen9blas_dequant_b16 in lib/kernels/hgemm.cl): activations rounded to FP16 once, the accurate
// FP16 GEMM (FP32 accumulation here) writes an FP16 result, an epilogue converts it to F32 and flags inf / NaN.

}  // extern "C"

namespace {

// Activations (F32 or FP16, row pitch lda) -> FP16 rows of Kp elements, zero past K, round to nearest even.
template <typename TA>
__global__ void act_to_f16(const TA *__restrict__ a, long long lda, int M, int K, int Kp, __half *__restrict__ dst) {
    const long long n = (long long)M * Kp;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int m = (int)(i / Kp), k = (int)(i % Kp);
        float v = 0.0f;
        if (k < K) v = to_r(a[(long long)m * lda + k]);
        dst[i] = __float2half_rn(v);
    }
}

// FP16 GEMM result (M × N, pitch ldp) -> F32 C: v = fp32(result); [v += bias[n]]; [v = gelu(v)]; [v += R[m][n]]; a
// non-finite raw value sets *nf. R may be C itself (each element is read before it is written).
__global__ void f16w_epilogue(const __half *__restrict__ c16, long long ldp, int M, int N, float *C, long long ldc,
                              const float *__restrict__ bias, int gelu, const float *R, long long ldr, unsigned *nf) {
    const long long n = (long long)M * N;
    bool bad = false;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int m = (int)(i / N), j = (int)(i % N);
        float v = __half2float(c16[(long long)m * ldp + j]);
        bad |= !isfinite(v);
        if (bias) v = __fadd_rn(v, bias[j]);
        if (gelu) v = gelu_ggml(v);
        if (R) v = __fadd_rn(v, R[(long long)m * ldr + j]);
        C[(long long)m * ldc + j] = v;
    }
    if (bad) *(volatile unsigned *)nf = 1u;
}

// ggml SWIGLU of two FP16 GEMM results: h = silu(g)·u = g / (1 + e^-g) · u in F32, rounded to FP16 into the next GEMM's
// activation rows (Kp, zero past N); a non-finite g, u or h, or |h| beyond FP16, sets *nf.
__global__ void swiglu_f16(const __half *__restrict__ G, const __half *__restrict__ U, int M, int N, __half *__restrict__ H,
                           int Kp, unsigned *nf) {
    const long long n = (long long)M * Kp;
    bool bad = false;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int m = (int)(i / Kp), k = (int)(i % Kp);
        float h = 0.0f;
        if (k < N) {
            const float g = __half2float(G[(long long)m * N + k]), u = __half2float(U[(long long)m * N + k]);
            h = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
            bad |= !isfinite(g) || !isfinite(u) || !(fabsf(h) <= 65504.0f);
        }
        H[i] = __float2half_rn(h);
    }
    if (bad) *(volatile unsigned *)nf = 1u;
}

// ggml block layouts dequantized into packed FP16 weights W[n][k] (pitch Kp): one thread per (row, block), the
// arithmetic of ggml's dequantize_row_* in the same order without contraction, FP16 round to nearest even; a value
// beyond FP16 range (or not finite) sets *oor. Q8_0: 34-byte blocks of 32 (fp16 d, int8 q[32]): d·q. Q4_K: 144-byte
// blocks of 256 (fp16 d, fp16 dmin, 12 bytes of packed 6-bit scales / mins, 128 bytes of 4-bit q): per 64 values two
// (scale, min) pairs, d·sc·q − dmin·m. Q6_K: 210-byte blocks of 256 (128 bytes low 4 bits, 64 bytes high 2 bits,
// int8 scales[16], fp16 d): d·sc·(q − 32).
__device__ __forceinline__ float ld_half_bytes(const uint8_t *p) {
    return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}
__device__ __forceinline__ void q4k_scale_min(int j, const uint8_t *q, int &sc, int &mn) {
    if (j < 4) {
        sc = q[j] & 63;
        mn = q[j + 4] & 63;
    } else {
        sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}
__global__ void dequant_rows(const uint8_t *__restrict__ W, size_t row_bytes, int qtype, int N, int nblk, __half *dst,
                             int Kp, unsigned *oor) {
    const long long total = (long long)N * nblk;
    bool bad = false;
    for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total; t += (long long)gridDim.x * blockDim.x) {
        const int n = (int)(t / nblk), j = (int)(t % nblk);
        __half *d = dst + (long long)n * Kp;
        auto put = [&](int k, float v) {
            bad |= !(fabsf(v) <= 65504.0f);
            d[k] = __float2half_rn(v);
        };
        if (qtype == GEN9BLAS_Q8_0) {
            const uint8_t *b = W + (size_t)n * row_bytes + (size_t)j * 34;
            const float dd = ld_half_bytes(b);
            for (int k = 0; k < 32; k++) put(j * 32 + k, __fmul_rn((float)(int8_t)b[2 + k], dd));
        } else if (qtype == GEN9BLAS_Q4_K) {
            const uint8_t *b = W + (size_t)n * row_bytes + (size_t)j * 144;
            const float dd = ld_half_bytes(b), dmin = ld_half_bytes(b + 2);
            const uint8_t *sc = b + 4, *q = b + 16;
            for (int g = 0; g < 4; g++, q += 32) {
                int s0, m0, s1, m1;
                q4k_scale_min(2 * g, sc, s0, m0);
                q4k_scale_min(2 * g + 1, sc, s1, m1);
                const float d1 = __fmul_rn(dd, (float)s0), mm1 = __fmul_rn(dmin, (float)m0);
                const float d2 = __fmul_rn(dd, (float)s1), mm2 = __fmul_rn(dmin, (float)m1);
                for (int l = 0; l < 32; l++) put(j * 256 + g * 64 + l, __fsub_rn(__fmul_rn(d1, (float)(q[l] & 0xF)), mm1));
                for (int l = 0; l < 32; l++) put(j * 256 + g * 64 + 32 + l, __fsub_rn(__fmul_rn(d2, (float)(q[l] >> 4)), mm2));
            }
        } else {
            const uint8_t *b = W + (size_t)n * row_bytes + (size_t)j * 210;
            const float dd = ld_half_bytes(b + 208);
            const uint8_t *ql = b, *qh = b + 128;
            const int8_t *sc = (const int8_t *)(b + 192);
            for (int h = 0; h < 2; h++, ql += 64, qh += 32, sc += 8) {
                for (int l = 0; l < 32; l++) {
                    const int is = l / 16;
                    const int q1 = (int)((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                    const int q2 = (int)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                    const int q3 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                    const int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                    const int k0 = j * 256 + h * 128;
                    put(k0 + l, __fmul_rn(__fmul_rn(dd, (float)sc[is]), (float)q1));
                    put(k0 + l + 32, __fmul_rn(__fmul_rn(dd, (float)sc[is + 2]), (float)q2));
                    put(k0 + l + 64, __fmul_rn(__fmul_rn(dd, (float)sc[is + 4]), (float)q3));
                    put(k0 + l + 96, __fmul_rn(__fmul_rn(dd, (float)sc[is + 6]), (float)q4));
                }
            }
        }
    }
    if (bad) *(volatile unsigned *)oor = 1u;
}

unsigned grid_for(long long n, int sms) {
    const long long b = (n + 255) / 256;
    return (unsigned)(b < 8LL * sms ? (b > 0 ? b : 1) : 8LL * sms);
}

// One product of the family: FP16 activation rows a16 (M × Kp) times the HS-packed P into c16 (M × N, FP16).
int f16w_gemm(const __half *a16, int M, const gen9blas_packed_b *P, __half *c16, cudaStream_t st) {
    return launch_gemm(GEN9BLAS_HS, 0, 1, M, P->N, P->Kp, 1.0, a16, P->Kp, 0, P->w, P->Kp, 0, 0.0, c16, P->N, 0, 1, st);
}

bool device_or_managed(const void *p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

struct F16wExt {
    const float *bias;
    int gelu;
    const float *R;
    int ldr;
};

// gemm_pb_f16w / _h / _ex: C (F32) = epilogue(fp16(A)·Bp); gemm_pa_f16w_ex: pa holds fp16(A) already (A unused).
int gemm_pb_f16w_any(bool ahalf, int M, const void *A, int lda, const gen9blas_packed_b *P, float *C, int ldc,
                     int *nonfinite, const F16wExt *ext, const char *who, const gen9blas_packed_a *pa = nullptr) {
    if (int e = begin_op()) return e;
    DevState *d = dev_state();
    if (!d) return G.status;
    if (nonfinite) *nonfinite = 0;
    G9_TRY(check_handle(P, d, who));
    if (P->type != GEN9BLAS_HS) return fail(GEN9BLAS_ERR_INVALID_ARG, "%s: needs B packed as GEN9BLAS_HS", who);
    if (pa) {
        if (pa->magic != kPackedAMagic || !pa->rows || pa->K != P->K || pa->Kp != P->Kp || pa->dev != d->dev)
            return fail(GEN9BLAS_ERR_INVALID_ARG, "%s: packed A does not match B (K %d / %d)", who, pa->K, P->K);
        M = pa->M;
        lda = P->K;
    }
    if (M <= 0) return 0;
    const int K = P->K, N = P->N, Kp = P->Kp;
    if (lda < K || ldc < N || (ext && ext->R && ext->ldr < N))
        return fail(GEN9BLAS_ERR_INVALID_ARG, "%s: lda = %d, ldc = %d for N = %d, K = %d", who, lda, ldc, N, K);
    timer_start();
    const size_t ea = ahalf ? 2 : 4;
    Operand op[2];
    if (!pa) G9_TRY(map_operand(op[0], A, ((size_t)(M - 1) * lda + K) * ea, 0, true, false));
    const bool r_is_c = ext && ext->R == C && ext->ldr == ldc;
    // C is read when it is the residual, and copied in when its rows have gaps (the copy back keeps them)
    G9_TRY(map_operand(op[1], C, ((size_t)(M - 1) * ldc + N) * 4, 2, r_is_c || ldc != N, true));
    Operand orr;
    const float *R = nullptr;
    if (ext && ext->R) {
        if (r_is_c) {
            R = (const float *)op[1].dptr;
        } else {
            G9_TRY(map_operand(orr, ext->R, ((size_t)(M - 1) * ext->ldr + N) * 4, 1, true, false));
            R = (const float *)orr.dptr;
        }
    }
    G.last_zc = op[0].zc | 2 | op[1].zc << 2;
    cudaStream_t st = stream();
    void *buf = nullptr;
    const size_t a_bytes = ((size_t)M * Kp * 2 + 255) / 256 * 256, c_bytes = ((size_t)M * N * 2 + 255) / 256 * 256;
    G9_TRY(ml_buffer(a_bytes + c_bytes + (size_t)N * 4, &buf));
    __half *a16 = pa ? pa->rows : (__half *)buf, *c16 = (__half *)((char *)buf + a_bytes);
    const float *bias = nullptr;
    if (ext && ext->bias) {   // device / managed memory in place; host memory copied behind the FP16 result
        if (device_or_managed(ext->bias)) {
            bias = ext->bias;
        } else {
            float *bd = (float *)((char *)buf + a_bytes + c_bytes);
            G9_CU(cudaMemcpyAsync(bd, ext->bias, (size_t)N * 4, cudaMemcpyHostToDevice, st));
            bias = bd;
        }
    }
    const bool queued = G.nowait && op[0].zc && op[1].zc && (!R || r_is_c || orr.zc);
    unsigned *flag = queued ? nowait_slot(d) : nullptr;
    if (!flag) {
        *(volatile unsigned *)(d->err_host + 1) = 0u;
        flag = d->err_dev + 1;
    }
    timer_kernel();
    // M <= 16 on a wide enough, deep enough weight matrix: one kernel (FP16 rounding of the activations as they are
    // loaded, the product, this epilogue), the same arithmetic as the three kernels below. From 9 tokens on, with at
    // least four 16-row weight blocks per SM, F32 activations are rounded to FP16 rows first (act_to_f16, as the
    // chain below does) so that the kernel reads half the activation bytes; it prefetches its weights while the
    // conversion runs (dependent launch). Measured on B200 at M = 16: W 11008 x 4096 28.2 -> 27.2 us; with fewer
    // blocks the conversion's latency shows (W 4096^2 9.96 -> 12.3 us), so those keep the direct F32 loads.
    const void *a1 = pa ? (const void *)pa->rows : op[0].dptr;
    bool h1 = pa || ahalf;
    long long l1 = pa ? Kp : lda;
    int k1 = pa ? Kp : K;
    if (!pa && !ahalf && M > 8 && (N + 15) / 16 >= 4 * d->sm_count && skinny_f16w_fits(M, Kp, N, Kp, P->w)) {
        act_to_f16<float><<<grid_for((long long)M * Kp, d->sm_count), 256, 0, st>>>((const float *)op[0].dptr, lda, M, K,
                                                                                     Kp, a16);
        G9_TRY(launched("act_to_f16"));
        a1 = a16;
        h1 = true;
        l1 = Kp;
        k1 = Kp;
    }
    const int one = launch_skinny_f16w(M, a1, h1, l1, P->w, k1, N, Kp, (float *)op[1].dptr, ldc, bias,
                                       ext ? ext->gelu : 0, R, ext ? ext->ldr : 0, flag, st);
    if (one < 0) return one;
    if (one == 0) {
        int r = finish_op(op, 2);
        timer_stop();
        if (r == 0 && !queued && nonfinite) *nonfinite = *(volatile unsigned *)(d->err_host + 1) != 0u;
        return r;
    }
    if (pa) {
    } else if (ahalf) act_to_f16<__half><<<grid_for((long long)M * Kp, d->sm_count), 256, 0, st>>>((const __half *)op[0].dptr, lda,
                                                                                            M, K, Kp, a16);
    else act_to_f16<float><<<grid_for((long long)M * Kp, d->sm_count), 256, 0, st>>>((const float *)op[0].dptr, lda, M, K,
                                                                                     Kp, a16);
    if (!pa) G9_TRY(launched("act_to_f16"));
    G9_TRY(f16w_gemm(a16, M, P, c16, st));
    f16w_epilogue<<<grid_for((long long)M * N, d->sm_count), 256, 0, st>>>(c16, N, M, N, (float *)op[1].dptr, ldc, bias,
                                                                           ext ? ext->gelu : 0, R, ext ? ext->ldr : 0, flag);
    G9_TRY(launched("f16w_epilogue"));
    int r = finish_op(op, 2);
    timer_stop();
    if (r == 0 && !queued && nonfinite) *nonfinite = *(volatile unsigned *)(d->err_host + 1) != 0u;
    return r;
}

}  // namespace

extern "C" {

GEN9BLAS_API int gen9blas_gemm_pb_f16w(int M, const float *A, int lda, const gen9blas_packed_b *Bp, float *C, int ldc,
                                       int *nonfinite) {
    return gemm_pb_f16w_any(false, M, A, lda, Bp, C, ldc, nonfinite, nullptr, "gemm_pb_f16w");
}

GEN9BLAS_API int gen9blas_gemm_pb_f16w_h(int M, const uint16_t *A, int lda, const gen9blas_packed_b *Bp, float *C, int ldc,
                                         int *nonfinite) {
    return gemm_pb_f16w_any(true, M, A, lda, Bp, C, ldc, nonfinite, nullptr, "gemm_pb_f16w_h");
}

GEN9BLAS_API int gen9blas_gemm_pb_f16w_ex(int M, const float *A, int lda, const gen9blas_packed_b *Bp, float *C, int ldc,
                                          const float *bias, int gelu, const float *R, int ldr, int *nonfinite) {
    const F16wExt e{bias, gelu ? 1 : 0, R, ldr};
    return gemm_pb_f16w_any(false, M, A, lda, Bp, C, ldc, nonfinite, &e, "gemm_pb_f16w_ex");
}

GEN9BLAS_API int gen9blas_gemm_pa_f16w_ex(const gen9blas_packed_a *pa, const gen9blas_packed_b *Bp, float *C, int ldc,
                                          const float *bias, int gelu, const float *R, int ldr, int *nonfinite) {
    if (nonfinite) *nonfinite = 0;
    if (!pa) return fail(GEN9BLAS_ERR_INVALID_ARG, "gemm_pa_f16w_ex: no packed A");
    const F16wExt e{bias, gelu ? 1 : 0, R, ldr};
    return gemm_pb_f16w_any(false, 0, nullptr, 0, Bp, C, ldc, nonfinite, &e, "gemm_pa_f16w_ex", pa);
}

GEN9BLAS_API int gen9blas_gemm_multi_f16w(int M, const float *A, int lda, int n, const gen9blas_packed_b *const *P,
                                          float *const *C, const int *ldc, int *nonfinite) {
    if (int e = begin_op()) return e;
    DevState *d = dev_state();
    if (!d) return G.status;
    if (n < 1 || n > 8 || !P || !C || !ldc || !nonfinite)
        return fail(GEN9BLAS_ERR_INVALID_ARG, "gemm_multi_f16w: 1 to 8 products with their outputs");
    for (int i = 0; i < n; i++) {
        G9_TRY(check_handle(P[i], d, "gemm_multi_f16w"));
        if (P[i]->type != GEN9BLAS_HS || P[i]->K != P[0]->K)
            return fail(GEN9BLAS_ERR_INVALID_ARG, "gemm_multi_f16w: B %d not packed as GEN9BLAS_HS with K = %d", i, P[0]->K);
        if (ldc[i] < P[i]->N) return fail(GEN9BLAS_ERR_INVALID_ARG, "gemm_multi_f16w: ldc[%d] < N", i);
        nonfinite[i] = 0;
    }
    if (M <= 0) return 0;
    for (int i = 0; i < n; i++)   // as the reference: the outputs are written in place (no staging slots for eight)
        if (!device_or_managed(C[i])) return GEN9BLAS_DECLINED;
    const int K = P[0]->K, Kp = P[0]->Kp;
    if (lda < K) return fail(GEN9BLAS_ERR_INVALID_ARG, "gemm_multi_f16w: lda < K");
    timer_start();
    Operand oa;
    G9_TRY(map_operand(oa, A, ((size_t)(M - 1) * lda + K) * 4, 0, true, false));
    int nmax = 0;
    for (int i = 0; i < n; i++) nmax = P[i]->N > nmax ? P[i]->N : nmax;
    void *buf = nullptr;
    const size_t a_bytes = ((size_t)M * Kp * 2 + 255) / 256 * 256;
    G9_TRY(ml_buffer(a_bytes + (size_t)M * nmax * 2, &buf));
    __half *a16 = (__half *)buf, *c16 = (__half *)((char *)buf + a_bytes);
    cudaStream_t st = stream();
    const bool queued = G.nowait && oa.zc;
    unsigned *flags[8];
    for (int i = 0; i < n; i++) {
        flags[i] = queued ? nowait_slot(d) : nullptr;
        if (!flags[i]) {
            (d->err_host + 2)[i] = 0u;   // words 2..9 of the mapped error block: one per output
            flags[i] = d->err_dev + 2 + i;
        }
    }
    timer_kernel();
    act_to_f16<float><<<grid_for((long long)M * Kp, d->sm_count), 256, 0, st>>>((const float *)oa.dptr, lda, M, K, Kp, a16);
    G9_TRY(launched("act_to_f16"));
    for (int i = 0; i < n; i++) {   // the FP16 result buffer is reused: each epilogue runs before the next GEMM
        G9_TRY(f16w_gemm(a16, M, P[i], c16, st));
        f16w_epilogue<<<grid_for((long long)M * P[i]->N, d->sm_count), 256, 0, st>>>(c16, P[i]->N, M, P[i]->N, C[i],
                                                                                     ldc[i], nullptr, 0, nullptr, 0, flags[i]);
        G9_TRY(launched("f16w_epilogue"));
    }
    Operand outs[9];
    outs[0] = oa;
    for (int i = 0; i < n; i++) {   // device-resident outputs: recorded for no-wait ordering, never copied back
        outs[1 + i].user = C[i];
        outs[1 + i].dptr = C[i];
        outs[1 + i].bytes = ((size_t)(M - 1) * ldc[i] + P[i]->N) * 4;
        outs[1 + i].zc = true;
        outs[1 + i].written = true;
    }
    int r = finish_op(outs, 1 + n);
    timer_stop();
    if (r == 0 && !queued)
        for (int i = 0; i < n; i++) nonfinite[i] = (d->err_host + 2)[i] != 0u;
    return r;
}

GEN9BLAS_API int gen9blas_ffn_f16w(int M, const float *X, int ldx, const gen9blas_packed_b *Pg, const gen9blas_packed_b *Pu,
                                   const gen9blas_packed_b *Pd, float *Y, int ldy, int *nonfinite) {
    if (int e = begin_op()) return e;
    DevState *d = dev_state();
    if (!d) return G.status;
    if (nonfinite) *nonfinite = 0;
    G9_TRY(check_handle(Pg, d, "ffn_f16w"));
    G9_TRY(check_handle(Pu, d, "ffn_f16w"));
    G9_TRY(check_handle(Pd, d, "ffn_f16w"));
    if (Pg->type != GEN9BLAS_HS || Pu->type != GEN9BLAS_HS || Pd->type != GEN9BLAS_HS)
        return fail(GEN9BLAS_ERR_INVALID_ARG, "ffn_f16w: needs weights packed as GEN9BLAS_HS");
    if (Pg->K != Pu->K || Pg->N != Pu->N || Pd->K != Pg->N)
        return fail(GEN9BLAS_ERR_INVALID_ARG, "ffn_f16w: shapes do not chain (gate %dx%d, up %dx%d, down %dx%d)", Pg->K,
                    Pg->N, Pu->K, Pu->N, Pd->K, Pd->N);
    if (M <= 0) return 0;
    const int K = Pg->K, Kp = Pg->Kp, N = Pg->N, Nd = Pd->N, Kpd = Pd->Kp;
    if (ldx < K || ldy < Nd) return fail(GEN9BLAS_ERR_INVALID_ARG, "ffn_f16w: ldx = %d, ldy = %d", ldx, ldy);
    timer_start();
    Operand op[2];
    G9_TRY(map_operand(op[0], X, ((size_t)(M - 1) * ldx + K) * 4, 0, true, false));
    G9_TRY(map_operand(op[1], Y, ((size_t)(M - 1) * ldy + Nd) * 4, 2, ldy != Nd, true));
    G.last_zc = op[0].zc | 2 | op[1].zc << 2;
    auto rnd = [](size_t b) { return (b + 255) / 256 * 256; };
    const size_t bx = rnd((size_t)M * Kp * 2), bg = rnd((size_t)M * N * 2), bh = rnd((size_t)M * Kpd * 2);
    void *buf = nullptr;
    G9_TRY(ml_buffer(bx + 2 * bg + bh + (size_t)M * Nd * 2, &buf));
    __half *x16 = (__half *)buf, *g16 = (__half *)((char *)buf + bx), *u16 = (__half *)((char *)buf + bx + bg);
    __half *h16 = (__half *)((char *)buf + bx + 2 * bg), *y16 = (__half *)((char *)buf + bx + 2 * bg + bh);
    cudaStream_t st = stream();
    const bool queued = G.nowait && op[0].zc && op[1].zc;
    unsigned *flag = queued ? nowait_slot(d) : nullptr;
    if (!flag) {
        *(volatile unsigned *)(d->err_host + 1) = 0u;
        flag = d->err_dev + 1;
    }
    timer_kernel();
    // decode sizes: gate and up in one launch whose pairs apply SWIGLU, then the down GEMM with the F32 epilogue in
    // its kernel (two launches; the same operations and roundings as the general chain below)
    int fused = 1;
    if (M <= 16) {
        // from 9 tokens on the F32 rows are rounded to FP16 first: half the activation bytes for the pair kernel, whose
        // 2 x 688 CTAs at 7B shapes hide the conversion (M = 16: 81.5 -> 75.7 us on B200)
        const bool pre = M > 8 && skinny_f16w_fits(M, Kp, N, Kp, Pg->w);
        if (pre) {
            act_to_f16<float><<<grid_for((long long)M * Kp, d->sm_count), 256, 0, st>>>((const float *)op[0].dptr, ldx, M, K,
                                                                                         Kp, x16);
            G9_TRY(launched("act_to_f16"));
        }
        fused = pre ? launch_skinny_swiglu(M, x16, true, Kp, Pg->w, Pu->w, Kp, N, Kp, g16, u16, h16, Kpd, flag, st)
                    : launch_skinny_swiglu(M, op[0].dptr, false, ldx, Pg->w, Pu->w, K, N, Kp, g16, u16, h16, Kpd, flag, st);
        if (fused < 0) return fused;
        if (fused == 0) {
            const int r2 = launch_skinny_f16w(M, h16, true, Kpd, Pd->w, Kpd, Nd, Kpd, (float *)op[1].dptr, ldy, nullptr, 0,
                                              nullptr, 0, flag, st);
            if (r2 < 0) return r2;
            if (r2 == 1) {
                G9_TRY(f16w_gemm(h16, M, Pd, y16, st));
                f16w_epilogue<<<grid_for((long long)M * Nd, d->sm_count), 256, 0, st>>>(
                    y16, Nd, M, Nd, (float *)op[1].dptr, ldy, nullptr, 0, nullptr, 0, flag);
                G9_TRY(launched("f16w_epilogue"));
            }
        }
    }
    if (fused) {
        act_to_f16<float><<<grid_for((long long)M * Kp, d->sm_count), 256, 0, st>>>((const float *)op[0].dptr, ldx, M, K, Kp, x16);
        G9_TRY(launched("act_to_f16"));
        G9_TRY(f16w_gemm(x16, M, Pg, g16, st));
        G9_TRY(f16w_gemm(x16, M, Pu, u16, st));
        swiglu_f16<<<grid_for((long long)M * Kpd, d->sm_count), 256, 0, st>>>(g16, u16, M, N, h16, Kpd, flag);
        G9_TRY(launched("swiglu_f16"));
        G9_TRY(f16w_gemm(h16, M, Pd, y16, st));
        f16w_epilogue<<<grid_for((long long)M * Nd, d->sm_count), 256, 0, st>>>(y16, Nd, M, Nd, (float *)op[1].dptr, ldy,
                                                                                nullptr, 0, nullptr, 0, flag);
        G9_TRY(launched("f16w_epilogue"));
    }
    int r = finish_op(op, 2);
    timer_stop();
    if (r == 0 && !queued && nonfinite) *nonfinite = *(volatile unsigned *)(d->err_host + 1) != 0u;
    return r;
}

GEN9BLAS_API gen9blas_packed_b *gen9blas_pack_b_q(int qtype, int K, int N, const void *W, size_t row_bytes,
                                                  int *out_of_range) {
    if (out_of_range) *out_of_range = 0;
    if (begin_op()) return nullptr;
    const int qb = qtype == GEN9BLAS_Q8_0 ? 32 : 256;
    const size_t bb = qtype == GEN9BLAS_Q8_0 ? 34 : qtype == GEN9BLAS_Q4_K ? 144 : qtype == GEN9BLAS_Q6_K ? 210 : 0;
    if (!bb || K <= 0 || N <= 0 || K % qb || row_bytes < (size_t)K / qb * bb || !W) {
        fail(GEN9BLAS_ERR_INVALID_ARG, "pack_b_q: qtype %d, K = %d, N = %d, row_bytes = %zu", qtype, K, N, row_bytes);
        return nullptr;
    }
    DevState *d = dev_state();
    if (!d) return nullptr;
    auto *P = new (std::nothrow) gen9blas_packed_b;
    if (!P) {
        fail(GEN9BLAS_ERR_OUT_OF_MEMORY, "out of host memory");
        return nullptr;
    }
    // K is a multiple of 32, so the FP16 rows are whole 16-byte vectors: no padded-A region
    *P = gen9blas_packed_b{kPackedMagic, GEN9BLAS_HS, K, N, K, d->dev, 0, nullptr, (size_t)N * K * 2};
    timer_start();
    cudaError_t e = cudaMalloc(&P->w, P->w_bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        delete P;
        fail(GEN9BLAS_ERR_OUT_OF_MEMORY, "pack_b_q: %zu bytes of device memory: %s", (size_t)N * K * 2, cudaGetErrorString(e));
        return nullptr;
    }
    Operand ow;
    cudaStream_t st = stream();
    int r = map_operand(ow, W, (size_t)(N - 1) * row_bytes + (size_t)K / qb * bb, 0, true, false);
    if (r == 0) {
        *(volatile unsigned *)(d->err_host + 1) = 0u;
        timer_kernel();
        dequant_rows<<<grid_for((long long)N * (K / qb), d->sm_count), 256, 0, st>>>(
            (const uint8_t *)ow.dptr, row_bytes, qtype, N, K / qb, (__half *)P->w, K, d->err_dev + 1);
        r = launched("dequant_rows");
    }
    if (r == 0) r = finish_op(nullptr, 0);
    if (r == 0) {   // the packed copy is complete before W may change, also in no-wait mode
        e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) r = cuda_fail(e, "cudaStreamSynchronize", __FILE__, __LINE__);
    }
    timer_stop();
    if (r < 0) {
        cudaFree(P->w);
        delete P;
        return nullptr;
    }
    if (out_of_range) *out_of_range = *(volatile unsigned *)(d->err_host + 1) != 0u;
    return P;
}

GEN9BLAS_API int gen9blas_nowait_pending(void) {
    if (begin_op()) return 0;
    DevState *d = dev_state();
    if (!d || !d->nw_host) return 0;
    int n = 0;
    for (int i = 0; i < d->nw_used; i++) n += d->nw_host[i] != 0u;
    memset(d->nw_host, 0, (size_t)d->nw_used * sizeof(unsigned));
    d->nw_used = 0;
    return n;
}

}  // extern "C"
