// gemm.cu -- level-3 entry points: gen9blas_gemm / _gemm_batched / _hgemm / _sgemm and the kernel dispatch.
//
// Host flow of the reference (lib/src/gemm.c:5-74, 177-184): type check, empty dimensions return 0, a small M or N
// (min(M, N) <= skinny threshold, single matrix) goes to the skinny kernels (gemm.c:11-12), everything else to the
// main GEMM. What differs on B200: there is no pack / pad / epilogue pipeline and no launch banding
// (gemm.c:15-55, 119-164); one kernel reads the strided operands through TMA or predicated 16-byte loads and applies
// alpha/beta in its epilogue.
#include "internal.h"

namespace g9 {

int launch_hgemm_tc(int type, int tA, int tB, int M, int N, int K, double alpha, const void *A, int lda, long long sA,
                    const void *B, int ldb, long long sB, double beta, void *C, int ldc, long long sC, int count,
                    cudaStream_t st, void *const *peers = nullptr, int npeers = 0, long long col_off = 0);
int launch_sgemm(int tA, int tB, int M, int N, int K, double alpha, const void *A, int lda, long long sA, const void *B,
                 int ldb, long long sB, double beta, void *C, int ldc, long long sC, int count, cudaStream_t st);
int launch_dgemm_dmma(int tA, int tB, int M, int N, int K, double alpha, const void *A, int lda, long long sA,
                      const void *B, int ldb, long long sB, double beta, void *C, int ldc, long long sC, int count,
                      cudaStream_t st);

static int elem_size(int type) { return type == GEN9BLAS_S ? 4 : type == GEN9BLAS_D ? 8 : 2; }

int launch_gemm(int type, int tA, int tB, int M, int N, int K, double alpha, const void *A, int lda, long long sA,
                const void *B, int ldb, long long sB, double beta, void *C, int ldc, long long sC, int count,
                cudaStream_t st) {
    if (count == 1 && (M < N ? M : N) <= skinny_threshold(type))
        return launch_skinny(type, tA, tB, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, st);
    if (type == GEN9BLAS_H || type == GEN9BLAS_HS)
        return launch_hgemm_tc(type, tA, tB, M, N, K, alpha, A, lda, sA, B, ldb, sB, beta, C, ldc, sC, count, st);
    if (type == GEN9BLAS_D)
        return launch_dgemm_dmma(tA, tB, M, N, K, alpha, A, lda, sA, B, ldb, sB, beta, C, ldc, sC, count, st);
    return launch_sgemm(tA, tB, M, N, K, alpha, A, lda, sA, B, ldb, sB, beta, C, ldc, sC, count, st);
}

// Host memory (pageable or pinned) as seen by the CUDA runtime.
static bool host_memory(const void *p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return true;
    }
    return a.type == cudaMemoryTypeHost || a.type == cudaMemoryTypeUnregistered;
}

// GEMM with A and C in host memory (the reference's common case: NumPy arrays), pipelined over row bands of C:
// B goes to the device first (unless it is device-resident), then band i of A crosses PCIe on the copy-in stream
// while band i - 1 is multiplied on the library's stream and band i - 2 of C returns on the copy-out stream. With
// pinned host memory the H2D and D2H engines and the GEMM run concurrently; with pageable memory the copies are
// synchronous for the host and the pipeline degrades to the plain sequence. Rows of C are copied with 2-D copies
// (pitch ldc), so bytes between rows are never written.
static int gemm_host_pipelined(int type, int tB, int M, int N, int K, double alpha, const void *A, int lda,
                               const void *B, int ldb, double beta, void *C, int ldc) {
    DevState *d = dev_state();
    if (!d) return G.status;
    G9_TRY(pipeline_streams(d));
    const size_t es = elem_size(type);
    const size_t bA = ((size_t)(M - 1) * lda + K) * es, bC = ((size_t)(M - 1) * ldc + N) * es;
    const size_t bB = (tB ? (size_t)(N - 1) * ldb + K : (size_t)(K - 1) * ldb + N) * es;
    const bool b_host = host_memory(B);
    void *dA = nullptr, *dB = const_cast<void *>(B), *dC = nullptr;
    G9_TRY(stage_buffer(0, bA, &dA));
    if (b_host) G9_TRY(stage_buffer(1, bB, &dB));
    G9_TRY(stage_buffer(2, bC, &dC));
    cudaStream_t sm = stream(), si = d->copy_in, so = d->copy_out;
    cudaEvent_t *ev = d->band_ev;
    // the copy streams start after everything already queued on the library's stream
    G9_CU(cudaEventRecord(ev[0], sm));
    G9_CU(cudaStreamWaitEvent(si, ev[0], 0));
    G9_CU(cudaStreamWaitEvent(so, ev[0], 0));
    if (b_host) G9_CU(cudaMemcpyAsync(dB, B, bB, cudaMemcpyHostToDevice, si));
    // four bands of whole 256-row pair tiles. While C bands return, the two directions share the host link (measured
    // on B200, n = 4096: 55 GB/s H2D alone, about 31 GB/s each way together), so the step is bounded by the link;
    // fewer, larger copies come closest (n = 4096 per call: 4 bands 1.58 ms, 8 bands 1.66, 16 bands 1.60-1.66).
    int mb = (M + 3) / 4;
    mb = (mb + 255) / 256 * 256;
    const int nb = (M + mb - 1) / mb;
    G.last_zc = (b_host ? 0 : 2);
    timer_kernel();
    for (int i = 0; i < nb; i++) {
        const int r0 = i * mb, rows = M - r0 < mb ? M - r0 : mb;
        const size_t oa = (size_t)r0 * lda * es, oc = (size_t)r0 * ldc * es;
        G9_CU(cudaMemcpy2DAsync((char *)dA + oa, (size_t)lda * es, (const char *)A + oa, (size_t)lda * es, (size_t)K * es,
                                rows, cudaMemcpyHostToDevice, si));
        if (beta != 0.0)
            G9_CU(cudaMemcpy2DAsync((char *)dC + oc, (size_t)ldc * es, (const char *)C + oc, (size_t)ldc * es,
                                    (size_t)N * es, rows, cudaMemcpyHostToDevice, si));
        G9_CU(cudaEventRecord(ev[1 + 2 * i], si));
        G9_CU(cudaStreamWaitEvent(sm, ev[1 + 2 * i], 0));
        G9_TRY(launch_gemm(type, 0, tB, rows, N, K, alpha, (const char *)dA + oa, lda, 0, dB, ldb, 0, beta,
                           (char *)dC + oc, ldc, 0, 1, sm));
        G9_CU(cudaEventRecord(ev[2 + 2 * i], sm));
        G9_CU(cudaStreamWaitEvent(so, ev[2 + 2 * i], 0));
        G9_CU(cudaMemcpy2DAsync((char *)C + oc, (size_t)ldc * es, (const char *)dC + oc, (size_t)ldc * es, (size_t)N * es,
                                rows, cudaMemcpyDeviceToHost, so));
    }
    // the library's stream continues after the last copy back (later calls may reuse the staging buffers)
    G9_CU(cudaEventRecord(ev[0], so));
    G9_CU(cudaStreamWaitEvent(sm, ev[0], 0));
    G9_CU(cudaStreamSynchronize(sm));
    Operand none[1];
    return finish_op(none, 0);
}

}  // namespace g9

using namespace g9;

extern "C" {

GEN9BLAS_API int gen9blas_gemm_batched(int type, int tA, int tB, int M, int N, int K, double alpha, const void *A, int lda,
                                       int64_t sA, const void *B, int ldb, int64_t sB, double beta, void *C, int ldc,
                                       int64_t sC, int count) {
    if (int e = begin_op()) return e;
    if (type < 0 || type > 3) return fail(GEN9BLAS_ERR_UNSUPPORTED, "type %d unavailable", type);
    if (M <= 0 || N <= 0 || K <= 0 || count <= 0) return 0;
    tA = tA ? 1 : 0;
    tB = tB ? 1 : 0;
    const size_t es = elem_size(type), c1 = count - 1;
    const size_t bA = (c1 * sA + (tA ? (size_t)(K - 1) * lda + M : (size_t)(M - 1) * lda + K)) * es;
    const size_t bB = (c1 * sB + (tB ? (size_t)(N - 1) * ldb + K : (size_t)(K - 1) * ldb + N)) * es;
    const size_t bC = (c1 * sC + (size_t)(M - 1) * ldc + N) * es;
    timer_start();
    // Large single GEMMs over several devices (gen9blas_set_devices / GEN9BLAS_DEVICES): column blocks per device
    if (count == 1) {
        const int r = gemm_sharded(type, tA, tB, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc);
        if (r <= 0) {
            timer_stop();
            return r;
        }
    }
    // Large single GEMMs on host A and C: banded pipeline of copies and kernels
    if (count == 1 && !tA && M >= 1024 && N > skinny_threshold(type) && K > skinny_threshold(type) &&
        bA + bC >= ((size_t)16 << 20) && host_memory(A) && host_memory(C)) {
        int r = gemm_host_pipelined(type, tB, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc);
        timer_stop();
        return r;
    }
    Operand op[3];
    G9_TRY(map_operand(op[0], A, bA, 0, true, false));
    G9_TRY(map_operand(op[1], B, bB, 1, true, false));
    // C is read when beta != 0; it is also copied in when its region has gaps (row pitch or batch stride larger
    // than the data), so that the copy back leaves the caller's bytes between rows untouched.
    const bool c_gaps = ldc != N || (count > 1 && sC != (int64_t)M * ldc);
    G9_TRY(map_operand(op[2], C, bC, 2, beta != 0.0 || c_gaps, true));
    G.last_zc = op[0].zc | op[1].zc << 1 | op[2].zc << 2;
    timer_kernel();
    G9_TRY(launch_gemm(type, tA, tB, M, N, K, alpha, op[0].dptr, lda, sA, op[1].dptr, ldb, sB, beta, op[2].dptr, ldc, sC,
                       count, stream()));
    int r = finish_op(op, 3);
    timer_stop();
    return r;
}

// Fused GEMM + all-gather for column-sharded multi-GPU GEMM: this rank computes its column block
// C[:, col_offset : col_offset + N] = alpha·op(A)·op(B) (beta = 0) and its epilogue stores every finished tile into all
// ranks' C (peer device pointers from gen9blas_ipc_open) over NVLink, overlapping the exchange with the next tiles.
// With M at most the skinny threshold (decode: C = X·W_shardᵀ with the weight rows split over the ranks) the skinny
// kernel computes the block and stores its outputs the same way.
GEN9BLAS_API int gen9blas_gemm_allgather(int type, int tA, int tB, int M, int N, int K, double alpha, const void *A,
                                         int lda, const void *B, int ldb, void *const *rank_C, int nranks, int ldc,
                                         int64_t col_offset) {
    if (int e = begin_op()) return e;
    if (type != GEN9BLAS_H && type != GEN9BLAS_HS)
        return fail(GEN9BLAS_ERR_UNSUPPORTED, "gen9blas_gemm_allgather supports FP16 (GEN9BLAS_H / GEN9BLAS_HS)");
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    if (!rank_C || nranks < 1 || nranks > 8) return fail(GEN9BLAS_ERR_INVALID_ARG, "1..8 destination buffers required");
    if (col_offset < 0 || ldc < col_offset + N) return fail(GEN9BLAS_ERR_INVALID_ARG, "ldc < col_offset + N");
    timer_start();
    Operand op[2];
    const size_t es = 2;
    G9_TRY(map_operand(op[0], A, ((tA ? (size_t)(K - 1) * lda + M : (size_t)(M - 1) * lda + K)) * es, 0, true, false));
    G9_TRY(map_operand(op[1], B, ((tB ? (size_t)(N - 1) * ldb + K : (size_t)(K - 1) * ldb + N)) * es, 1, true, false));
    if (!op[0].zc || !op[1].zc) return fail(GEN9BLAS_ERR_INVALID_ARG, "gen9blas_gemm_allgather takes device operands");
    timer_kernel();
    if (M <= skinny_threshold(type))   // tensor-parallel decode: skinny kernel, outputs stored into every rank's C
        G9_TRY(launch_skinny(type, tA ? 1 : 0, tB ? 1 : 0, M, N, K, alpha, op[0].dptr, lda, op[1].dptr, ldb, 0.0,
                             rank_C[0], ldc, stream(), rank_C, nranks, col_offset));
    else
        G9_TRY(launch_hgemm_tc(type, tA ? 1 : 0, tB ? 1 : 0, M, N, K, alpha, op[0].dptr, lda, 0, op[1].dptr, ldb, 0,
                               0.0, rank_C[0], ldc, 0, 1, stream(), rank_C, nranks, col_offset));
    int r = finish_op(op, 2);
    timer_stop();
    return r;
}

GEN9BLAS_API int gen9blas_gemm(int type, int tA, int tB, int M, int N, int K, double alpha, const void *A, int lda,
                               const void *B, int ldb, double beta, void *C, int ldc) {
    return gen9blas_gemm_batched(type, tA, tB, M, N, K, alpha, A, lda, 0, B, ldb, 0, beta, C, ldc, 0, 1);
}

GEN9BLAS_API int gen9blas_hgemm(int M, int N, int K, double alpha, const uint16_t *A, int lda, const uint16_t *B, int ldb,
                                double beta, uint16_t *C, int ldc) {
    return gen9blas_gemm(GEN9BLAS_H, 0, 0, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc);
}

GEN9BLAS_API int gen9blas_sgemm(int M, int N, int K, double alpha, const float *A, int lda, const float *B, int ldb,
                                double beta, float *C, int ldc) {
    return gen9blas_gemm(GEN9BLAS_S, 0, 0, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc);
}

}  // extern "C"
