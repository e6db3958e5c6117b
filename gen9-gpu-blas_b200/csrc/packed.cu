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

}  // extern "C"
