/* gen9blas_ml.h -- the neural-network operations of the reference (lib/gen9blas_ml.h of kprzybys/gen9-gpu-blas, version
 * 0.2), B200 build: GEMMs with FP16 or quantized weights kept on the GPU and fused epilogues, the elementwise ggml ops
 * of a transformer layer, attention. Conventions (results, threads, handle lifetime, no-wait mode, gen9blas_flush) as
 * in gen9blas.h.
 *
 * Memory: operands in device or managed memory are used in place; host memory is staged through device buffers and the
 * call completes before it returns. The elementwise ops queue their work without a wait (sync = 0) when every operand is
 * device or managed memory; sync = 1 or a staged operand waits. Results follow ggml-cpu's arithmetic (same operation
 * order, no contracted multiply-adds, FP16 conversions rounding to nearest even); the row reductions of the norms sum
 * in FP64 as ggml-cpu does. */
#pragma once
#include "gen9blas.h"
#ifdef __cplusplus
extern "C" {
#endif

/* ---- GEMMs with FP16 weights packed once (gen9blas_pack_b(GEN9BLAS_HS, ...) or gen9blas_pack_b_q) ----
 * C (F32, M×N) = A (F32, M×K) · Bp: A rounded to FP16 once, FP16 products with FP32 accumulation, the result rounded to
 * FP16 once and returned as F32. *nonfinite = 1 if a result is inf / NaN (FP16 overflow): recompute in F32. NULL
 * allowed; left 0 for a call queued in no-wait mode (see gen9blas_nowait_pending). ref: lib/gen9blas_ml.h:11-15 */
GEN9BLAS_API int gen9blas_gemm_pb_f16w(int M, const float *A, int lda, const gen9blas_packed_b *Bp, float *C, int ldc,
                                       int *nonfinite);
/* The same with FP16 activations (lda in elements). ref: lib/gen9blas_ml.h:16-18 */
GEN9BLAS_API int gen9blas_gemm_pb_f16w_h(int M, const uint16_t *A, int lda, const gen9blas_packed_b *Bp, float *C, int ldc,
                                         int *nonfinite);
/* gemm_pb_f16w with its epilogue extended: C = [gelu](A·Bp + bias) [+ R]. bias: N floats or NULL; gelu 0 / 1 (ggml GELU,
 * tanh form with ggml-cpu's FP16 rounding, as gen9blas_gelu); R: M×N (row pitch ldr) or NULL, may be C itself with
 * ldr == ldc. Equal bit for bit to gemm_pb_f16w followed by binop_rows / gelu / binop_rows. *nonfinite: of the raw
 * product. ref: lib/gen9blas_ml.h:19-24 */
GEN9BLAS_API int gen9blas_gemm_pb_f16w_ex(int M, const float *A, int lda, const gen9blas_packed_b *Bp, float *C, int ldc,
                                          const float *bias, int gelu, const float *R, int ldr, int *nonfinite);
/* Small batches, 1 <= M <= 16 (several sequences decoded together): C (F32, M×N) = A (F32, M×K) · Bp, Bp packed with
 * GEN9BLAS_HS (FP16 weights W[N][K], e.g. gen9blas_pack_b(GEN9BLAS_HS, 1, K, N, W, K)). The activations are not
 * rounded to FP16: each row is carried as two FP16 parts (~22 significant bits) through FP32-accumulating MMAs.
 * *nonfinite = 1 if any result is inf / NaN (NULL allowed; left 0 for a call queued in no-wait mode).
 * Returns GEN9BLAS_DECLINED (1, nothing written) for M outside 1..16, GEN9BLAS_ERR_INVALID_ARG for a Bp not packed as
 * GEN9BLAS_HS. ref: lib/gen9blas_ml.h:25-28 */
GEN9BLAS_API int gen9blas_gemm_pb_skinny(int M, const float *A, int lda, const gen9blas_packed_b *Bp, float *C, int ldc,
                                         int *nonfinite);
/* n (1..8) products of one F32 input with HS-packed weights of the same K (Q / K / V), the input rounded to FP16 once;
 * nonfinite[i] per output. Returns GEN9BLAS_DECLINED (nothing written) when an output is not device or managed memory:
 * compute them one by one. ref: lib/gen9blas_ml.h:29-32 */
GEN9BLAS_API int gen9blas_gemm_multi_f16w(int M, const float *A, int lda, int n, const gen9blas_packed_b *const *P,
                                          float *const *C, const int *ldc, int *nonfinite);
/* Gated FFN: Y = (silu(X·Wg) ⊙ (X·Wu))·Wd; X F32 M×K, Y F32 M×Nd; Pg, Pu: K -> N, Pd: N -> Nd, all packed as
 * GEN9BLAS_HS. The intermediates stay FP16 on the GPU. *nonfinite as above (also for an intermediate beyond FP16).
 * ref: lib/gen9blas_ml.h:33-36 */
GEN9BLAS_API int gen9blas_ffn_f16w(int M, const float *X, int ldx, const gen9blas_packed_b *Pg, const gen9blas_packed_b *Pu,
                                   const gen9blas_packed_b *Pd, float *Y, int ldy, int *nonfinite);
/* Quantized weights: N rows of K values in ggml block layout (row n at W + n·row_bytes; GEN9BLAS_Q8_0: K % 32 == 0,
 * GEN9BLAS_Q4_K / GEN9BLAS_Q6_K: K % 256 == 0) dequantized on the GPU into a handle for gemm_pb_f16w -- the same as
 * gen9blas_pack_b(GEN9BLAS_HS, 1, K, N, ...) of ggml's dequantize_row_* values rounded to FP16 (nearest even).
 * *out_of_range = 1 if a value does not fit FP16 (the handle is then unusable: free it, use FP32). NULL on error.
 * ref: lib/gen9blas_ml.h:37-42 */
enum { GEN9BLAS_Q8_0 = 0, GEN9BLAS_Q4_K = 1, GEN9BLAS_Q6_K = 2 };
GEN9BLAS_API gen9blas_packed_b *gen9blas_pack_b_q(int qtype, int K, int N, const void *W, size_t row_bytes,
                                                  int *out_of_range);

/* A GEMM input made once by a LayerNorm and used by several gen9blas_gemm_pa_f16w_ex calls (Q / K / V / fc1 of one
 * block): gen9blas_layer_norm_pack writes the same Y as gen9blas_layer_norm plus the FP16 rows the products read, which
 * then skip their own conversion (the same FP16 values, so the results equal gemm_pb_f16w_ex on Y). The handle holds
 * device memory of the device it was last written on; packed_a_free does not wait (flush first).
 * ref: lib/gen9blas_ml.h:44-53 */
typedef struct gen9blas_packed_a gen9blas_packed_a;
GEN9BLAS_API gen9blas_packed_a *gen9blas_packed_a_create(void);
GEN9BLAS_API void gen9blas_packed_a_free(gen9blas_packed_a *pa);
GEN9BLAS_API int gen9blas_layer_norm_pack(int M, int K, const float *X, int ldx, const float *w, const float *b, float eps,
                                          float *Y, int ldy, gen9blas_packed_a *pa, int sync);
GEN9BLAS_API int gen9blas_gemm_pa_f16w_ex(const gen9blas_packed_a *pa, const gen9blas_packed_b *Bp, float *C, int ldc,
                                          const float *bias, int gelu, const float *R, int ldr, int *nonfinite);

/* ---- Queued work (gen9blas_set_nowait and gen9blas_flush: gen9blas.h) ----
 * While no-wait mode is on, gemm_pb_f16w(_ex), ffn_f16w and gemm_multi_f16w with device-resident operands queue their
 * work with *nonfinite left 0; the GPU sets one flag word per call on FP16 overflow. After gen9blas_flush,
 * gen9blas_nowait_pending returns how many queued calls overflowed and clears the flags: the caller recomputes (or
 * fails) whatever used those results. ref: lib/gen9blas_ml.h:55-62 */
GEN9BLAS_API int gen9blas_nowait_pending(void);
/* Registration of host regions for queued elementwise ops. Here host operands are staged and complete before each call
 * returns, so every region counts as registered: returns 0, and span_clear has nothing to clear.
 * ref: lib/gen9blas_ml.h:63-68 */
GEN9BLAS_API int gen9blas_span(const void *p, size_t bytes, int writes);
GEN9BLAS_API void gen9blas_span_clear(void);

/* ---- Elementwise ops (ggml semantics) ---- ref: lib/gen9blas_ml.h:71-120 */
/* Y = X / sqrt(mean(X²) + eps) [· w], M rows of K (w NULL: no weight). */
GEN9BLAS_API int gen9blas_rms_norm(int M, int K, const float *X, int ldx, const float *w, float eps, float *Y, int ldy,
                                   int sync);
/* ggml NORM (mean / variance over K) [· w] [+ b] (w, b: one row of K or NULL). */
GEN9BLAS_API int gen9blas_layer_norm(int M, int K, const float *X, int ldx, const float *w, const float *b, float eps,
                                     float *Y, int ldy, int sync);
/* C = A + B (op 0) or A · B (op 1), M rows of K. ldb = 0: B is one row broadcast to all rows; bs0 = 0: B has one value
 * per row (broadcast along the row); bs0 = 1: K values per row. */
GEN9BLAS_API int gen9blas_binop_rows(int op, int M, int K, const float *A, int lda, const float *B, int ldb, int bs0,
                                     float *C, int ldc, int sync);
/* ggml GELU (tanh form, ggml-cpu's FP16 table semantics) / GELU_ERF (erf form, F32) / RELU over n contiguous floats;
 * X == Y allowed. */
GEN9BLAS_API int gen9blas_gelu(size_t n, const float *X, float *Y, int sync);
GEN9BLAS_API int gen9blas_gelu_erf(size_t n, const float *X, float *Y, int sync);
GEN9BLAS_API int gen9blas_relu(size_t n, const float *X, float *Y, int sync);
/* ggml IM2COL: X [N, IC, IH, IW] (image / channel offsets ofs0 / ofs1 in floats, rows of IW contiguous) -> Y [N, OH, OW,
 * IC·KH·KW], F32 or FP16 (f16); zero padding. 1-D convolution: IH = KH = OH = 1. */
GEN9BLAS_API int gen9blas_im2col(int N, int IC, int IH, int IW, const float *X, int64_t ofs0, int64_t ofs1, int KH, int KW,
                                 int OH, int OW, int s0, int s1, int p0, int p1, int d0, int d1, void *Y, int f16, int sync);
/* F32 rows × H heads × D (element (r, h, d) at X[r·s_row + h·s_head + d]) -> FP16 [r][h][d] contiguous, saturated to
 * ±65504. */
GEN9BLAS_API int gen9blas_cvt_f16_heads(int rows, int H, int D, const float *X, int64_t s_row, int64_t s_head, uint16_t *Y,
                                        int sync);
/* ggml ROPE forward, modes NORMAL (neox 0) / NEOX (neox 1), rotating all n_dims = head size elements: element (i, h, t)
 * of X / Y at t·s2 + h·s1 + i floats; pos[n_tok]; ff: n_dims/2 frequency factors or NULL; corr:
 * ggml_rope_yarn_corr_dims. GEN9BLAS_ERR_UNSUPPORTED for a layout whose heads overlap. */
GEN9BLAS_API int gen9blas_rope(int n_dims, int nh, int n_tok, const float *X, int64_t xs1, int64_t xs2, float *Y, int64_t ys1,
                               int64_t ys2, const int *pos, const float *ff, int neox, float freq_base, float freq_scale,
                               float ext_factor, float attn_factor, const float corr[2], int sync);
/* ggml_rope_multi: MROPE (vision 0: sections[4], pos = 4·n_tok positions, NEOX pair order, pair j takes the position of
 * its sector j % sum(sections)) or VISION (vision 1: n_dims = ne0 / 2, pairs (i, i + n_dims), the power of theta reset
 * at each section start). */
GEN9BLAS_API int gen9blas_rope_multi(int n_dims, int nh, int n_tok, const float *X, int64_t xs1, int64_t xs2, float *Y,
                                     int64_t ys1, int64_t ys2, const int *pos, const float *ff, const int sections[4],
                                     float freq_base, float freq_scale, float ext_factor, float attn_factor,
                                     const float corr[2], int vision, int sync);
/* ggml CPY / CONT / DUP: src (type tin) -> dst (type tout), GEN9BLAS_S (F32) or GEN9BLAS_H (F16); ne / nb as ggml (nb
 * in bytes, non-negative strides); the destination shape may differ with the same element count (row-major order). */
GEN9BLAS_API int gen9blas_cpy_any(const void *src, int tin, const int64_t sne[4], const int64_t snb[4], void *dst, int tout,
                                  const int64_t dne[4], const int64_t dnb[4], int sync);
/* ggml UPSCALE (ggml_interpolate) F32; mode_flags as ggml: 0 nearest, 1 bilinear, | 1<<8 align corners, | 1<<9
 * antialias. */
GEN9BLAS_API int gen9blas_upscale_f32(const float *src, const int64_t sne[4], const int64_t snb[4], float *dst,
                                      const int64_t dne[4], const int64_t dnb[4], int mode_flags, int sync);
/* ggml SET_ROWS, F32 source rows into an F16 destination (KV-cache writes): dst row idx[i] of plane (i02, i03) = src
 * row i. idx int64 (idx64 = 1) or int32, byte strides b10 / b11 / b12, broadcast over the planes as ggml-cpu. dst must
 * be device or managed memory. A wait (sync = 1 or a staged operand) reports *bad = 1 for an index outside [0, ne1)
 * (that row is not written). */
GEN9BLAS_API int gen9blas_set_rows_f16(int nc, int nr, int ne02, int ne03, const float *src, int64_t s1, int64_t s2,
                                       int64_t s3, const void *idx, size_t idx_bytes, int64_t b10, int64_t b11, int64_t b12,
                                       int idx64, int ne11, int ne12, uint16_t *dst, size_t dst_bytes, int64_t d1,
                                       int64_t d2, int64_t d3, int64_t ne1, int sync, int *bad);

/* ---- Attention ---- ref: lib/gen9blas_ml.h:122-149
 * Shapes: D <= 128, H a multiple of HKV (the *_supported functions say 1 for these). Q, K, V, O device or managed
 * memory. One split-K kernel over chunks of keys (FP32 online softmax, scores in base 2 with the scale folded into the
 * query) and a merge kernel.
 * attn_dec: decoding over KV streams. Q F32 element (d, token t, head h, stream s) at Q[s·qs + t·qt + h·qh + d]; K / V
 * F16 in place, element (d, key k, KV head g, stream s) at [s·ks + k·kk + g·kh + d]; O F32 [s][t][h][d] contiguous.
 * Token t of stream s sees keys [0, min(vis[s] + dvis·t, nk)). chunk: the reference's work-group length, ignored
 * here. Queued (sync = 1 waits). */
GEN9BLAS_API int gen9blas_attn_dec_supported(int D, int H, int HKV);
GEN9BLAS_API int gen9blas_attn_dec(int D, int H, int HKV, int ns, int nq, int nk, const float *Q, int64_t qt, int64_t qh,
                                   int64_t qs, const uint16_t *K, int64_t kk, int64_t kh, int64_t ks, size_t k_bytes,
                                   const uint16_t *V, int64_t vk, int64_t vh, int64_t vs, size_t v_bytes, float *O,
                                   float scale, const int *vis, int dvis, int chunk, int sync);
/* Prefill, llama.cpp layouts: Q and O F32 [token][H][D]; K and V F16 rows of HKV·D values, the first nk rows used.
 * Token t sees keys 0 .. min(nk, vis0 + dvis·t) - 1 (dvis 1: causal). Returns 0, GEN9BLAS_DECLINED (unsupported
 * shape; nothing written) or < 0. *launches = attention launches (1). */
GEN9BLAS_API int gen9blas_attn_supported(int D, int H, int HKV);
GEN9BLAS_API int gen9blas_attn_f16kv(int D, int H, int HKV, int nq, int nk, const float *Q, const uint16_t *K, size_t k_bytes,
                                     const uint16_t *V, size_t v_bytes, float *O, float scale, int vis0, int dvis,
                                     int *launches);
/* Several KV streams in one call: stream s has Q / O at Q + s·sq / O + s·sq (floats, rows [t][h][d], sq = nq·H·D),
 * K / V at K + s·sk / V + s·sv (halves, rows of HKV·D), visible keys min(nk, vis0[s] + dvis·t). */
GEN9BLAS_API int gen9blas_attn_streams_supported(int D, int H, int HKV);
GEN9BLAS_API int gen9blas_attn_f16kv_streams(int D, int H, int HKV, int ns, int nq, int nk, const float *Q, int64_t sq,
                                             const uint16_t *K, int64_t sk, size_t k_bytes, const uint16_t *V, int64_t sv,
                                             size_t v_bytes, float *O, float scale, const int *vis0, int dvis, int *launches);

#ifdef __cplusplus
}
#endif
