/* gen9blas.h -- public C ABI of the B200 (sm_100a) build of gen9blas.
 *
 * This header is the drop-in boundary: every function, enum value and argument order below matches the interface
 * of the reference library (lib/gen9blas.h of kprzybys/gen9-gpu-blas, version 0.2), so programs and bindings
 * written against that library (ctypes module, CBLAS shim, Rust FFI) link against libgen9blas.so unchanged.
 * Each declaration cites the reference line it replaces as "ref: lib/gen9blas.h:<line>".
 *
 * Conventions (same as the reference):
 * - Matrices are row-major; element types are uint16_t (IEEE FP16), float or double, passed as void*.
 *   Strides (lda, inc, sA...) are in elements.
 * - Result codes: 0 success, < 0 an error (text in gen9blas_error()), GEN9BLAS_DECLINED = 1 "not handled, nothing
 *   written". Functions returning a pointer return NULL on error; gen9blas_last_status() then holds the code.
 * - Operands may live anywhere the CPU or the GPU can address: device memory (cudaMalloc, torch tensors) and
 *   managed memory (gen9blas_alloc) are used in place; any other host pointer is staged through device work
 *   buffers. Calls are synchronous unless gen9blas_set_nowait(1) is on and every operand is device-resident.
 * - The library keeps process-wide state (work buffers, last error, current device). The caller serialises calls;
 *   gen9blas_error() stays valid until the next call.
 * - Vectors hold n elements spaced inc apart; inc != 0; a negative inc means the pointer is the lowest address
 *   (element 0 is the last one in memory), as in reference BLAS.
 */
#pragma once
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

#define GEN9BLAS_VERSION_MAJOR 0
#define GEN9BLAS_VERSION_MINOR 2
#define GEN9BLAS_VERSION_PATCH 0
#define GEN9BLAS_VERSION (GEN9BLAS_VERSION_MAJOR * 10000 + GEN9BLAS_VERSION_MINOR * 100 + GEN9BLAS_VERSION_PATCH)
#ifndef GEN9BLAS_API
#define GEN9BLAS_API __attribute__((visibility("default")))
#endif

/* Element / accumulation kinds (ref: lib/gen9blas.h:28-32). */
enum { GEN9BLAS_H = 0,    /* FP16 in and out, FP16 accumulation (tcgen05 f16 accumulator in TMEM) */
       GEN9BLAS_S = 1,    /* FP32 */
       GEN9BLAS_HS = 2,   /* FP16 in and out, FP32 accumulation ("accurate") */
       GEN9BLAS_D = 3 };  /* FP64 */
#define GEN9BLAS_KC 32    /* chunk length of the reference's HS accumulation; the B200 HS accumulates all of K in FP32 */
enum { GEN9BLAS_NO_TRANS = 0, GEN9BLAS_TRANS = 1 };   /* ref: lib/gen9blas.h:34 */
enum { GEN9BLAS_LEFT = 0, GEN9BLAS_RIGHT = 1 };       /* ref: lib/gen9blas.h:35 */
enum { GEN9BLAS_LOWER = 0, GEN9BLAS_UPPER = 1 };      /* ref: lib/gen9blas.h:36 */
enum { GEN9BLAS_NON_UNIT = 0, GEN9BLAS_UNIT = 1 };    /* ref: lib/gen9blas.h:37 */

/* Status codes (ref: lib/gen9blas.h:38-46). */
typedef enum {
    GEN9BLAS_OK = 0,
    GEN9BLAS_DECLINED = 1,               /* not handled; nothing was written */
    GEN9BLAS_ERR = -1,                   /* CUDA launch / execution error, device wait timeout */
    GEN9BLAS_ERR_UNSUPPORTED = -2,       /* type or entry point not available in this build */
    GEN9BLAS_ERR_INVALID_ARG = -3,       /* invalid arguments (leading dimension, increment 0, ...) */
    GEN9BLAS_ERR_OUT_OF_MEMORY = -4,     /* device or host allocation failed */
    GEN9BLAS_ERR_NO_DEVICE = -5,         /* initialisation failed: no usable sm_100 GPU (final for the process) */
} gen9blas_status;

/* ---- Library (ref: lib/gen9blas.h:48-78) ---- */
GEN9BLAS_API int gen9blas_version(void);                 /* ref: lib/gen9blas.h:50 */
GEN9BLAS_API int gen9blas_init(void);                    /* ref: lib/gen9blas.h:53; once per process, failure is final */
GEN9BLAS_API int gen9blas_device_gen(void);              /* ref: lib/gen9blas.h:55; B200 build: 100 (sm_100), 0 = none */
enum {
    GEN9BLAS_FEAT_FP16 = 0,
    GEN9BLAS_FEAT_FP32,
    GEN9BLAS_FEAT_FP64,
    GEN9BLAS_FEAT_SKINNY_PB,
    GEN9BLAS_FEAT_EPILOG_EXT,
    GEN9BLAS_FEAT_NORM_PACK,
    GEN9BLAS_FEAT_ROPE_MULTI,
    GEN9BLAS_FEAT_CPY,
    GEN9BLAS_FEAT_SET_ROWS,
};                                                        /* ref: lib/gen9blas.h:56-66 */
GEN9BLAS_API int gen9blas_has(int feature);              /* ref: lib/gen9blas.h:68; 1: FP16/FP32/FP64, SKINNY_PB */
GEN9BLAS_API const char *gen9blas_error(void);           /* ref: lib/gen9blas.h:69 */
GEN9BLAS_API int gen9blas_last_status(void);             /* ref: lib/gen9blas.h:70 */
GEN9BLAS_API double gen9blas_last_time_ms(void);         /* ref: lib/gen9blas.h:71; GEN9BLAS_PROFILE=1: kernel time */
GEN9BLAS_API int gen9blas_last_zero_copy(void);          /* ref: lib/gen9blas.h:72; bits 1 A, 2 B, 4 C used in place */
/* Managed memory (cudaMallocManaged, 4096-byte aligned): CPU-writable and used in place by every kernel
 * (ref: lib/gen9blas.h:76-78, USM host memory there). */
GEN9BLAS_API void *gen9blas_alloc(size_t bytes);
GEN9BLAS_API void gen9blas_free(void *p);
GEN9BLAS_API int gen9blas_is_usm(const void *p, size_t bytes);  /* 1: [p, p+bytes) inside one gen9blas_alloc block */

/* ---- Level 3 (ref: lib/gen9blas.h:80-117) ---- */
/* C = alpha·op(A)·op(B) + beta·C; op(A) M×K (transA: A stored K×M), op(B) K×N (transB: B stored N×K).
 * beta = 0: C is not read. ref: lib/gen9blas.h:82-83 */
GEN9BLAS_API int gen9blas_gemm(int type, int transA, int transB, int M, int N, int K, double alpha, const void *A, int lda,
                               const void *B, int ldb, double beta, void *C, int ldc);
/* Strided batch: matrix b uses A + b·sA, B + b·sB, C + b·sC (elements). ref: lib/gen9blas.h:86-88 */
GEN9BLAS_API int gen9blas_gemm_batched(int type, int transA, int transB, int M, int N, int K, double alpha,
                                       const void *A, int lda, int64_t sA, const void *B, int ldb, int64_t sB,
                                       double beta, void *C, int ldc, int64_t sC, int count);
/* Constant weights kept on the GPU (ref: lib/gen9blas.h:89-97): pack op(B) (K×N; transB: B stored N×K, host or device
 * memory) once into HBM of the current device, multiply many times. gemm_pb: C = alpha·op(A)·Bp + beta·C with op(A)
 * M×K of the type Bp was packed with (GEN9BLAS_H, _S, _HS, _D). pack_b: NULL on error (gen9blas_error()); B may be
 * overwritten or freed once it returns. packed_b_free waits for queued work first. */
typedef struct gen9blas_packed_b gen9blas_packed_b;
GEN9BLAS_API gen9blas_packed_b *gen9blas_pack_b(int type, int transB, int K, int N, const void *B, int ldb);
GEN9BLAS_API int gen9blas_gemm_pb(int transA, int M, double alpha, const void *A, int lda, const gen9blas_packed_b *Bp,
                                  double beta, void *C, int ldc);
GEN9BLAS_API void gen9blas_packed_b_free(gen9blas_packed_b *Bp);
/* Level-3 operations on top of GEMM (ref: lib/gen9blas.h:98-113): SYMM, SYRK, SYR2K, TRMM (all four types) and TRSM
 * (FP32, FP64, FP16 H / HS); only the uplo triangle of A is read, SYRK / SYR2K modify only the uplo triangle of C. */
GEN9BLAS_API int gen9blas_symm(int type, int side, int uplo, int M, int N, double alpha, const void *A, int lda,
                               const void *B, int ldb, double beta, void *C, int ldc);
GEN9BLAS_API int gen9blas_syrk(int type, int uplo, int trans, int N, int K, double alpha, const void *A, int lda,
                               double beta, void *C, int ldc);
GEN9BLAS_API int gen9blas_syr2k(int type, int uplo, int trans, int N, int K, double alpha, const void *A, int lda,
                                const void *B, int ldb, double beta, void *C, int ldc);
GEN9BLAS_API int gen9blas_trmm(int type, int side, int uplo, int transA, int diag, int M, int N, double alpha,
                               const void *A, int lda, void *B, int ldb);
GEN9BLAS_API int gen9blas_trsm(int type, int side, int uplo, int transA, int diag, int M, int N, double alpha,
                               const void *A, int lda, void *B, int ldb);
/* Shortcuts without transposes. ref: lib/gen9blas.h:114-117 */
GEN9BLAS_API int gen9blas_hgemm(int M, int N, int K, double alpha, const uint16_t *A, int lda, const uint16_t *B, int ldb,
                                double beta, uint16_t *C, int ldc);
GEN9BLAS_API int gen9blas_sgemm(int M, int N, int K, double alpha, const float *A, int lda, const float *B, int ldb,
                                double beta, float *C, int ldc);

/* ---- Levels 1-2 (ref: lib/gen9blas.h:119-148). type: GEN9BLAS_S, _D or _H (_HS = _H). FP16 is computed in FP32,
 * reductions accumulate in FP64. ---- */
GEN9BLAS_API int gen9blas_axpy(int type, int n, double a, const void *x, int incx, void *y, int incy);   /* :121 */
GEN9BLAS_API int gen9blas_scal(int type, int n, double a, void *x, int incx);                            /* :122 */
GEN9BLAS_API int gen9blas_copy(int type, int n, const void *x, int incx, void *y, int incy);            /* :123 */
GEN9BLAS_API int gen9blas_swap(int type, int n, void *x, int incx, void *y, int incy);                  /* :124 */
GEN9BLAS_API int gen9blas_rot(int type, int n, void *x, int incx, void *y, int incy, double c, double s); /* :125 */
GEN9BLAS_API int gen9blas_rotm(int type, int n, void *x, int incx, void *y, int incy, const double *param); /* :126 */
GEN9BLAS_API void gen9blas_rotg(float *a, float *b, float *c, float *s);                                 /* :127 */
GEN9BLAS_API void gen9blas_rotmg(float *d1, float *d2, float *x1, float y1, float *param);               /* :128 */
GEN9BLAS_API int gen9blas_dot(int type, int n, const void *x, int incx, const void *y, int incy, double *result); /* :129 */
GEN9BLAS_API int gen9blas_asum(int type, int n, const void *x, int incx, double *result);               /* :130 */
GEN9BLAS_API int gen9blas_nrm2(int type, int n, const void *x, int incx, double *result);               /* :131 */
GEN9BLAS_API int gen9blas_iamax(int type, int n, const void *x, int incx, int64_t *result);             /* :132 */
/* y = alpha·op(A)·x + beta·y, A M×N (trans: x has length M, y length N); beta = 0: y not read. :133-135 */
GEN9BLAS_API int gen9blas_gemv(int type, int trans, int M, int N, double alpha, const void *A, int lda, const void *x, int incx,
                               double beta, void *y, int incy);
GEN9BLAS_API int gen9blas_symv(int type, int uplo, int n, double alpha, const void *A, int lda, const void *x, int incx,
                               double beta, void *y, int incy);                                           /* :137 */
GEN9BLAS_API int gen9blas_trmv(int type, int uplo, int trans, int diag, int n, const void *A, int lda, void *x, int incx);
GEN9BLAS_API int gen9blas_trsv(int type, int uplo, int trans, int diag, int n, const void *A, int lda, void *x, int incx);
GEN9BLAS_API int gen9blas_syr(int type, int uplo, int n, double alpha, const void *x, int incx, void *A, int lda);
GEN9BLAS_API int gen9blas_syr2(int type, int uplo, int n, double alpha, const void *x, int incx, const void *y, int incy,
                               void *A, int lda);
/* A = alpha·x·yᵀ + A, A M×N. ref: lib/gen9blas.h:147-148 */
GEN9BLAS_API int gen9blas_ger(int type, int M, int N, double alpha, const void *x, int incx, const void *y, int incy,
                              void *A, int lda);
/* Banded and packed level 2 (ref: lib/gen9blas.h:150-168), CBLAS RowMajor storage. */
GEN9BLAS_API int gen9blas_gbmv(int type, int trans, int M, int N, int KL, int KU, double alpha, const void *A, int lda,
                               const void *x, int incx, double beta, void *y, int incy);
GEN9BLAS_API int gen9blas_sbmv(int type, int uplo, int N, int K, double alpha, const void *A, int lda, const void *x, int incx,
                               double beta, void *y, int incy);
GEN9BLAS_API int gen9blas_tbmv(int type, int uplo, int trans, int diag, int N, int K, const void *A, int lda, void *x, int incx);
GEN9BLAS_API int gen9blas_tbsv(int type, int uplo, int trans, int diag, int N, int K, const void *A, int lda, void *x, int incx);
GEN9BLAS_API int gen9blas_spmv(int type, int uplo, int N, double alpha, const void *Ap, const void *x, int incx, double beta,
                               void *y, int incy);
GEN9BLAS_API int gen9blas_tpmv(int type, int uplo, int trans, int diag, int N, const void *Ap, void *x, int incx);
GEN9BLAS_API int gen9blas_tpsv(int type, int uplo, int trans, int diag, int N, const void *Ap, void *x, int incx);
GEN9BLAS_API int gen9blas_spr(int type, int uplo, int N, double alpha, const void *x, int incx, void *Ap);
GEN9BLAS_API int gen9blas_spr2(int type, int uplo, int N, double alpha, const void *x, int incx, const void *y, int incy,
                               void *Ap);

/* ---- Additions of the B200 build (no counterpart in lib/gen9blas.h; the reference is single-device) ---- */
/* Selects the CUDA device used by later calls (one process per GPU: call once after start-up). Default: the device
 * current when gen9blas_init ran. Returns 0 or GEN9BLAS_ERR_INVALID_ARG. */
GEN9BLAS_API int gen9blas_set_device(int device);
GEN9BLAS_API int gen9blas_get_device(void);
/* Launches later calls on the given cudaStream_t (NULL: the library's own non-blocking stream of the device). */
GEN9BLAS_API int gen9blas_set_stream(void *cuda_stream);
/* No-wait mode (same names and meaning as lib/gen9blas_ml.h:61,69 of the reference): while on, a call whose operands
 * are all device-resident returns right after its kernels are queued; results are ready after gen9blas_flush()
 * (or any synchronisation of the stream). Calls with host operands still wait. */
GEN9BLAS_API void gen9blas_set_nowait(int on);
GEN9BLAS_API int gen9blas_flush(void);
/* Several GPUs behind one process's calls (the reference's entry point, lib/src/gemm.c:177-180, drives one device).
 * After gen9blas_set_devices(n, ids) with n >= 2 -- or with GEN9BLAS_DEVICES="0,1,..." in the environment, read at
 * the first GEMM -- a gen9blas_gemm / gen9blas_hgemm / gen9blas_sgemm with count 1, min(M, N) above the skinny
 * threshold and 2·M·N·K of at least GEN9BLAS_SHARD_MIN_FLOP (default 2·4096³) is split by column blocks of B and C
 * (multiples of 256 columns) over the listed devices: each computes its block with its own kernels on its own
 * memory, operands reach it by peer copies (NVLink) or host copies, and an operand already in a device's memory is
 * read there in place. Such a call always waits for every device (no-wait mode does not apply to it). ids: CUDA
 * device ordinals (at most 8, distinct, sm_100); n <= 1 turns sharding off. Returns 0 or GEN9BLAS_ERR_INVALID_ARG /
 * GEN9BLAS_ERR_NO_DEVICE. gen9blas_get_devices copies up to max ids and returns how many are set (0: none). */
GEN9BLAS_API int gen9blas_set_devices(int n, const int *ids);
GEN9BLAS_API int gen9blas_get_devices(int *ids, int max);
/* Multi-GPU, one process per GPU (no counterpart in the reference, which drives one device).
 * Device buffers that other ranks write into: any cudaMalloc memory (gen9blas_dev_alloc, torch tensors). For a
 * pointer into such memory gen9blas_ipc_handle fills a 64-byte CUDA IPC handle of its allocation and the pointer's
 * byte offset in it (send both to the other ranks); gen9blas_ipc_open maps a peer's handle into this process and
 * returns the allocation's base, usable by this rank's kernels over NVLink (add the offset). */
GEN9BLAS_API void *gen9blas_dev_alloc(size_t bytes);
GEN9BLAS_API void gen9blas_dev_free(void *p);
GEN9BLAS_API int gen9blas_ipc_handle(const void *dev_ptr, void *handle64, int64_t *offset);
GEN9BLAS_API void *gen9blas_ipc_open(const void *handle64);
GEN9BLAS_API int gen9blas_ipc_close(void *peer_ptr);
/* Fused GEMM + all-gather of a column-sharded FP16 GEMM (type GEN9BLAS_H or _HS): this rank computes its column block
 * C[:, col_offset : col_offset + N] = alpha·op(A)·op(B) (M × N, beta = 0) and the tensor-core kernel's epilogue stores
 * every finished tile into the C of all nranks ranks (rank_C: their device pointers, own C included, row pitch ldc)
 * with plain NVLink stores, overlapping the exchange with the remaining tiles. With M at most 16 (decode: C = X·Wᵀ
 * with the weight rows split over the ranks, transB = 1) the skinny kernel computes the block and stores its outputs
 * the same way. A and B must be device memory. The caller synchronises the ranks (gen9blas_peer_barrier) before
 * reading C. At most 8 ranks. */
GEN9BLAS_API int gen9blas_gemm_allgather(int type, int transA, int transB, int M, int N, int K, double alpha,
                                         const void *A, int lda, const void *B, int ldb, void *const *rank_C,
                                         int nranks, int ldc, int64_t col_offset);
/* Barrier of the ranks over NVLink peer memory, enqueued on the library's stream (no counterpart in the reference).
 * rank_flags[q]: device pointer (own or peer-mapped with gen9blas_ipc_open) to rank q's array of nranks + 1 32-bit
 * words, all zero before the first barrier. The kernel raises this rank's flag in every array (after the stores of
 * the preceding work on this stream) and waits until every rank's flag in this rank's array is raised, so that work
 * enqueued after it sees every rank's stores (e.g. a gen9blas_gemm_allgather result). The epoch of each barrier is
 * counted in the array's last word on the device, so the call can be captured in a CUDA graph and replayed; every
 * rank must run the same sequence of barriers on the same arrays. The wait gives up after timeout_ms (0.1 .. 60000):
 * the call (or, with no-wait, the next synchronising call) returns GEN9BLAS_ERR and the device stays usable. At most
 * 8 ranks. */
GEN9BLAS_API int gen9blas_peer_barrier(void *const *rank_flags, int nranks, int rank, double timeout_ms);
/* Number of kernels this library launched since the process started (launch accounting for benchmarks). */
GEN9BLAS_API long long gen9blas_kernel_launches(void);
/* Diagnostic of the bounded device-side waits: runs a kernel whose mbarrier wait can never complete; the wait gives
 * up after limit_ms (clamped to 0.1 .. 1000 ms), records the timeout in the error word and the kernel returns. The
 * call then returns GEN9BLAS_ERR with the timeout message and the device stays usable. No GPU fault is involved. */
GEN9BLAS_API int gen9blas_selftest_wait(double limit_ms);

/* GEMV that allocates nothing: same arguments, results and error codes as gen9blas_gemv, for callers that must not
 * allocate GPU memory -- a latency-critical loop that cannot afford the device-wide synchronisation of
 * cudaMalloc/cudaFree, or a process whose device memory is all handed to its own pool, where any allocation outside
 * that pool fails. No counterpart in the reference (lib/gen9blas.h has none: its host-memory design always stages).
 * - A, x and y must be device (or managed) memory of the current device; nothing is staged (INVALID_ARG otherwise).
 * - The transposed product keeps its partial sums in an 8 MiB array inside the library's device image, which every
 *   GPU that loads the library holds until the process exits; trans with N above 2,097,152 (FP16/FP32) or 1,048,576
 *   (FP64) elements is rejected with GEN9BLAS_ERR_INVALID_ARG and a message, before any launch.
 * - The first call on a device looks up that array's device address (cudaGetSymbolAddress) with the device current;
 *   make that first call before any stream capture.
 * - All calls share the one array: calls that overlap on the GPU (different streams, or no-wait calls from several
 *   threads) race on it. Every partial sum is written before it is read, so nothing needs clearing between calls.
 * - Runs on the stream set with gen9blas_set_stream, else on the library's own stream of the device, so it is
 *   ordered with the other entry points' work and gen9blas_flush waits for it; waits for that stream unless no-wait
 *   mode is on or the stream is being captured into a CUDA graph (the launches are then only recorded). On a device where no other entry point has run yet, the library has no stream of its own (creating
 *   it would allocate): the call then runs on the per-thread default stream and always waits for it.
 * - Calls no cudaMalloc, cudaFree or other allocating routine. */
GEN9BLAS_API int gen9blas_gemv_noalloc(int type, int trans, int M, int N, double alpha, const void *A, int lda,
                                       const void *x, int incx, double beta, void *y, int incy);

#ifdef __cplusplus
}
#endif
