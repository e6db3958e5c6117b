/* gen9blas_ml.h -- the small-batch constant-weight product of the reference's neural-network header
 * (lib/gen9blas_ml.h of kprzybys/gen9-gpu-blas, version 0.2), B200 build.
 *
 * Only gen9blas_gemm_pb_skinny is part of this build; the rest of the reference header (FP16-weight GEMMs with fused
 * epilogues, quantized weights, elementwise ggml ops, attention) lies outside the BLAS hot path and is not declared.
 * Conventions (results, threads, handle lifetime) as in gen9blas.h.
 */
#pragma once
#include "gen9blas.h"
#ifdef __cplusplus
extern "C" {
#endif

/* Small batches, 1 <= M <= 16 (several sequences decoded together): C (F32, M×N) = A (F32, M×K) · Bp, Bp packed with
 * GEN9BLAS_HS (FP16 weights W[N][K], e.g. gen9blas_pack_b(GEN9BLAS_HS, 1, K, N, W, K)). The activations are not
 * rounded to FP16: each row is carried as two FP16 parts (~22 significant bits) through FP32-accumulating MMAs.
 * *nonfinite = 1 if any result is inf / NaN (NULL allowed; left 0 for a call queued in no-wait mode).
 * Returns GEN9BLAS_DECLINED (1, nothing written) for M outside 1..16, GEN9BLAS_ERR_INVALID_ARG for a Bp not packed as
 * GEN9BLAS_HS. ref: lib/gen9blas_ml.h:25-28 */
GEN9BLAS_API int gen9blas_gemm_pb_skinny(int M, const float *A, int lda, const gen9blas_packed_b *Bp, float *C, int ldc,
                                         int *nonfinite);

#ifdef __cplusplus
}
#endif
