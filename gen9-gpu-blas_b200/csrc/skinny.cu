// skinny.cu -- GEMM with a small dimension (min(M, N) <= 16 by default): C = alpha·a·wᵀ + beta·C, where the small
// operand a has Mc rows and the large "weights" operand w has Nc rows of length K.
//
// Replaces the reference's gemm_skinny (lib/src/gemm.c:191-263) and its kernels skinny_k1/k4/k8, skinny_r4/r8
// (weights contiguous along K, lib/kernels/level12.cl:646-801) and skinny_n4 + skinny_n2 (weights contiguous along N,
// level12.cl:803-862). The host logic is the same: the operand roles swap when N is the small side
// (Cᵀ = op(B)ᵀ·op(A)ᵀ, C written with swapped strides, gemm.c:213-221), and accumulation is FP32 (FP64 never takes
// this path, gemm.c:191-199).
//
// B200 kernels:
// - wk_f16_sk: weights FP16, contiguous along K. The (16-row block, K chunk) iterations are split evenly over every
//   warp of a one-wave grid (stream-K), so all SMs stream the same number of weight bytes whatever the shape; each
//   lane streams 16-byte loads of two weight rows (ld.global.nc, deep unroll) into mma.sync m16n8k16 (FP16 in, FP32
//   accumulate). A row block shared by several warps is finished by the warp whose range ends in it (it meets the
//   block last); the others leave epoch-tagged FP32 partial tiles without a fence and stream on, and the finisher adds
//   them in K order (deterministic).
// - wk_f32: weights FP32, contiguous along K, FFMA: a CTA owns 4 rows, 8 warps split K, lanes read float4, warp
//   shuffle reduction, fixed-order combination across warps.
// - wn_partial + wn_final: weights contiguous along N: split-K partial sums P[part][m][n] in FP32, then a fixed-order
//   sum with the alpha/beta epilogue (deterministic, no atomics).
// - generic: any other layout (unaligned rows, K not a multiple of 8): one warp per weight row, scalar loads.
#include "common.cuh"
#include "internal.h"
#include <cstdlib>
#include <cstring>

namespace g9 {

int skinny_threshold(int type) {
    static int forced = -2;
    if (forced == -2) {
        const char *e = getenv("GEN9BLAS_SKINNY");
        forced = e ? atoi(e) : -1;
    }
    if (type == GEN9BLAS_D) return 0;
    if (forced >= 0) return forced;
    return 16;
}

struct SkinnyArgs {
    int Mc, Nc, K;
    float alpha, beta;
    const void *a;   // a[m*sam + k*sak]
    long long sam, sak;
    const void *w;   // w[n*swn + k*swk]
    long long swn, swk;
    void *C;         // C[m*scm + n*scn]
    long long scm, scn;
    // Fused all-gather (tensor-parallel decode): the result is also stored into the C of the other ranks (peer
    // pointers over NVLink, dst[0] == C), at element offset off = m·scm + n·scn + coff. ndst == 1: C only.
    void *dst[8];
    int ndst;
    long long coff;
    // F32 activations (gemm_pb_skinny): a is the FP16 "hi" part of the scaled activations and a + alo the "lo" part
    // (same pitch); a result is multiplied by tscale[m] (2^-s of its row), C is FP32, and a non-finite result sets *nf.
    long long alo;
    const float *tscale;
    unsigned *nf;
    // wk_f16_sk: the weights may be read before griddepcontrol.wait (no queued call writes them).
    int early_w;
    // wk_f16_sk: tag of this launch's partial tiles, and the device error word a finisher's bounded wait reports to.
    unsigned epoch;
    unsigned *err;
    // wk_f16_sk: 1 = every CTA owns whole row blocks (its warps split them; partial tiles meet in shared memory),
    // 0 = warps split the whole iteration space (partial tiles of blocks shared across CTAs go through global memory).
    int aligned;
    // wk_f16_blk with the gemm_pb_f16w epilogue: the FP32 sum rounded to FP16 once (a non-finite one sets *nf), then
    // [+ bias[n]] [gelu] [+ R[m·ldr + n]], stored as F32 at C[m·scm + n].
    const float *bias;
    const float *R;
    long long ldr;
    int gelu;
    // wk_f16_blk gate / up pair (ffn_f16w): CTA 2b takes row block b of w (gate, FP16 result to C) and CTA 2b + 1 the
    // same block of w2 (up, FP16 result to c2), both with pitch scm; the second of the two to finish writes
    // h = fp16(silu(g)·u) for those rows into hsw (pitch ldh, zero from column Nc to ldh), sets *nf for a non-finite
    // g, u or h or |h| beyond FP16, and returns cnt[b] to zero.
    const void *w2;
    void *c2;
    __half *hsw;
    long long ldh;
    unsigned *cnt;
};

template <typename T>
__device__ __forceinline__ void skinny_store(const SkinnyArgs &p, int m, int n, float s) {
    const long long off = (long long)m * p.scm + (long long)n * p.scn + p.coff;
    T *c = (T *)p.C + off;
    float v = p.alpha * s;
    if (p.beta != 0.0f) v = __fmaf_rn(p.beta, to_r(*c), v);
    const T o = from_r<T>(v);
    if (p.ndst == 1) {
        *c = o;
        return;
    }
    for (int q = 0; q < p.ndst; q++) ((T *)p.dst[q])[off] = o;
}

// Store of the F32-activation variant: undo the row's power-of-two scale, FP32 C, flag non-finite results.
__device__ __forceinline__ void skinny_store_f32a(const SkinnyArgs &p, int m, int n, float s) {
    float *c = (float *)p.C + (long long)m * p.scm + (long long)n * p.scn;
    float v = p.alpha * (s * p.tscale[m]);
    if (p.beta != 0.0f) v = __fmaf_rn(p.beta, *c, v);
    if (!isfinite(v)) *(volatile unsigned *)p.nf = 1u;
    *c = v;
}

template <bool F32A>
__device__ __forceinline__ void skinny_out(const SkinnyArgs &p, int m, int n, float s) {
    if constexpr (F32A) skinny_store_f32a(p, m, n, s);
    else skinny_store<__half>(p, m, n, s);
}

// End of every skinny kernel: with peer destinations, the thread's stores are made visible system-wide before the
// kernel ends, so that a rank barrier enqueued after it orders them before its flag (early returns store nothing).
__device__ __forceinline__ void skinny_peer_fence(const SkinnyArgs &p) {
    if (p.ndst > 1) __threadfence_system();
}

// ------------------------------------------------------------------------------------------------ FP16, K-contiguous
constexpr int WK_WARPS = 8;

__device__ __forceinline__ void mma_16816(float *d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ldg_nc16(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Weight stream: read-only, no L1 allocation, and a 256-byte L2 prefetch hint (each lane's 16 bytes sit in a 64-byte
// run of its row, and the warp walks the row in consecutive 64-byte runs).
__device__ __forceinline__ uint4 ldg_w16(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Stream-K hand-over words: a 64-bit relaxed store / load is single-copy atomic, so a value travels with its tag.
__device__ __forceinline__ void st_relaxed_u64(uint64_t *a, uint64_t v) {
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(a), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_u64(const uint64_t *a) {
    uint64_t v;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
constexpr unsigned long long kSkWaitNs = 4000000000ull;   // a finisher's bound on waiting for a partial tile

__device__ __forceinline__ uint32_t word(const uint4 &v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// Requirements (checked on the host): K % 8 == 0, weight rows and token rows contiguous along K with 16-byte aligned
// starts. grid = (CTAs, ceil(Mc / 16)).
// Each warp computes 16 weight rows × 16 tokens with mma.sync.m16n8k16: the weight rows are the MMA's M side and the
// tokens its N side (one or two 8-token tiles). The weights of UNROLL = 8 32-wide K steps are loaded before any is
// used, which keeps 16 independent 16-byte weight loads in flight per lane -- at decode shapes HBM needs ~100 KiB in
// flight per SM. The token fragments (L1 hits) are loaded right before their MMAs (LAZY), which leaves that register
// budget to the weights also with two token tiles (measured on B200: M = 16, W 4096 × 4096, 13.1 µs against 14.3 with
// the tokens prefetched at UNROLL 4). The K order inside a 32-wide step is permuted identically for weights and tokens
// (a dot product does not depend on it), so every lane's 16-byte load is directly an MMA fragment.
//
// Work is spread stream-K style over the whole GPU in one wave. The iteration space is (rb, kc): rb = block of 16
// weight rows, kc = chunk of UNROLL·32 K elements; T = RB·KC iterations are split evenly over all warps of the grid
// (warp w owns [T·w/W, T·(w+1)/W)), so every SM streams the same number of weight bytes whatever the shape. A warp that
// covers a whole row block stores C directly. Otherwise the warp whose range ends in the block (wf, the one owning its
// first chunk) finishes it: the block is the last thing wf does, while the other contributors meet it at the start of
// their ranges (or span it wholly). Each contributor writes its FP32 partial tile to its slot, every value tagged
// with the launch's epoch in one relaxed 64-bit store, and goes on streaming -- no fence, no atomic, nothing that
// leaves a warp without loads in flight. The finisher adds the slots to its own tile in slot order (deterministic),
// waiting (bounded) only for values whose tag is still old; a timeout sets the device error word.
//
// Activation modes (the F32 ones serve gemm_pb_skinny, whose activations arrive split into two FP16 parts, a =
// (hi + lo)·2^-s per row, written by split_f32_rows; both parts go through the MMA into FP32 accumulators, FP16
// products being exact in FP32, so the result carries the activations to ~22 bits):
// - ACT_F16: FP16 activations, Mc tokens.
// - ACT_PAIRED (Mc <= 8 real tokens): hi and lo interleaved as 2·Mc virtual token rows (2m: hi, 2m+1: lo). The loads
//   and MMAs are those of ACT_F16 on the virtual rows, and since lane (g, t) holds virtual tokens 2t and 2t+1 of its
//   D fragment, the hi and lo sums of real token t meet in the same lane: the epilogue adds them. With one tile
//   (Mc <= 4) the token fragments are prefetched with the weights (measured faster there than LAZY).
// - ACT_SPLIT (9..16 real tokens): hi and lo as two matrices (lo at a + alo), both MMA'd into the same accumulator,
//   their fragments loaded right before use.
// In both F32 modes the kernel is launched as the programmatic dependent of split_f32_rows: it issues its first weight
// loads, then waits for the split (griddepcontrol.wait) before the first activation access.
// - ACT_F16S (9..16 tokens): FP16 activations staged per warp in shared memory: at each K chunk, after its weight
//   loads, the warp copies its tokens' UNROLL·32 columns (cp.async, 16 bytes per lane and token row, one burst) into
//   its own region and reads the MMA fragments from there, so the activation round trip to L2 is paid once per chunk
//   rather than once per 32-wide step (two token tiles read 2 x 8 rows a step, and a 16 × K activation block no
//   longer stays in L1). Measured on B200, M = 16, two boxes: W 4096² 12.3 -> 10.8-11.2 µs, 11008 × 4096 23.6 ->
//   21.7-22.1, 4096 × 11008 22.7 -> 21.5-22.6, but 12288 × 4096 23.5 -> 24.2. With up to 8 tokens the fragments
//   stay L1-resident and are read directly (ACT_F16, LAZY; staging them cost M = 1 up to 48 %).
enum { ACT_F16 = 0, ACT_PAIRED = 1, ACT_SPLIT = 2, ACT_F16S = 3, ACT_F32H = 4 };
// ACT_F32H (wk_f16_blk only): F32 activations rounded to FP16 (nearest even) as their fragments are loaded, the
// gemm_pb_f16w semantics.

// ACT_F16S staging: per warp, one row per token of UNROLL·32 FP16 plus a 64-byte pad (the two token rows a
// quarter-warp reads then fall on different banks).
constexpr int SK_ROWB = 8 * 32 * 2 + 64;
__host__ __device__ constexpr int sk_stage_bytes(bool two) { return WK_WARPS * (two ? 16 : 8) * SK_ROWB; }
// Second-iteration weights prefetched into shared memory (the modes other than ACT_F16S): 16 rows per warp.
constexpr int SK_PRE_ROWB = 8 * 32 * 2 + 64;
constexpr int SK_PRE_BYTES = WK_WARPS * 16 * SK_PRE_ROWB;
// Both regions are 16 rows of SK_ROWB bytes per warp, whose last 64 bytes no copy touches: a warp keeps there (row r
// of the tile in the pad of row r) its 16 x 16 FP32 partial tile of the first row block of its CTA when every
// contributor of that block is a warp of the same CTA; the CTA adds those tiles after the main loop. The launch needs
// no more shared memory than the regions (73,728 bytes), so a CTA of the next call still fits beside two of this one.
static_assert(SK_PRE_ROWB == SK_ROWB && SK_ROWB - 8 * 32 * 2 == 64, "pad of 16 floats per staging row");
constexpr int SK_SMEM_BYTES = WK_WARPS * 16 * SK_ROWB;
static_assert(SK_PRE_BYTES == SK_SMEM_BYTES && sk_stage_bytes(true) == SK_SMEM_BYTES, "both regions fill the launch");
__device__ __forceinline__ float *sk_pad_row(uint8_t *smem, int warp_local, int r) {
    return reinterpret_cast<float *>(smem + (warp_local * 16 + r) * SK_ROWB + 8 * 32 * 2);
}
// After the main loop the copied part of a warp's rows is free: row r of its last block's tile sits at its start.
__device__ __forceinline__ float *sk_last_row(uint8_t *smem, int warp_local, int r) {
    return reinterpret_cast<float *>(smem + (warp_local * 16 + r) * SK_ROWB);
}

template <bool TWO_NTILES, int UNROLL, int MODE = ACT_F16, bool LAZY = false>
__global__ void __launch_bounds__(WK_WARPS * 32, 2)
wk_f16_sk(const SkinnyArgs p, int KC, int maxc, uint64_t *__restrict__ part) {
    constexpr bool F32A = MODE == ACT_PAIRED || MODE == ACT_SPLIT;
    constexpr bool late = LAZY || MODE == ACT_SPLIT || MODE == ACT_F16S;   // fragments loaded right before their MMAs
    static_assert(MODE != ACT_F16S || UNROLL == 8, "ACT_F16S staging rows hold 8 K steps");
    extern __shared__ __align__(16) uint8_t sk_stage[];
    // Dependents (the next skinny call, launched with programmatic stream serialization) may start as soon as this
    // grid runs: they take SM slots as this grid's CTAs retire and stream their own weights meanwhile.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int t0 = blockIdx.y * 16;
    const int RB = (p.Nc + 15) / 16;
    const long long T = (long long)RB * KC;
    const int W = gridDim.x * WK_WARPS;
    const int wg = blockIdx.x * WK_WARPS + warp;
    // aligned: CTA c owns row blocks [RB·c/G, RB·(c+1)/G), i.e. iterations [cs0, cs0 + cn), split evenly over its warps
    long long it, it_end;
    if (p.aligned) {
        const long long cs0 = (long long)KC * ((long long)RB * blockIdx.x / gridDim.x);
        const long long cn = (long long)KC * ((long long)RB * (blockIdx.x + 1) / gridDim.x) - cs0;
        it = cs0 + cn * warp / WK_WARPS;
        it_end = cs0 + cn * (warp + 1) / WK_WARPS;
    } else {
        it = T * wg / W;
        it_end = T * (wg + 1) / W;
    }
    const int first_rb = (int)(it / KC);   // the warp's first row block
    const __half *Wt = (const __half *)p.w;
    const __half *A = (const __half *)p.a;
    const int ta0 = min(t0 + g, p.Mc - 1), ta1 = min(t0 + g + 8, p.Mc - 1);
    const __half *a0 = A + (long long)ta0 * p.sam;
    const __half *a1 = A + (long long)ta1 * p.sam;
    const __half *l0 = a0 + p.alo, *l1 = a1 + p.alo;   // ACT_SPLIT: lo parts
    const int Mout = MODE == ACT_PAIRED ? p.Mc / 2 : p.Mc;   // tokens stored
    // The warp's second iteration goes to shared memory (cp.async) before the wait as well, so that with two
    // iterations per warp every weight byte is requested while the preceding kernel finishes (issued right after the
    // first iteration's loads, below). Rows of 512 bytes padded to SK_PRE_ROWB: the two rows a quarter-warp reads then
    // sit on different banks.
    constexpr bool PRE = MODE != ACT_F16S && UNROLL == 8;
    bool waited = false;
    if (!p.early_w) {   // a queued call may still write the weights: nothing is read before the wait
        asm volatile("griddepcontrol.wait;" ::: "memory");
        waited = true;
    }
    long long pre_it = -1;
    // The block this warp finishes (the last one of its range, when other warps contribute to it): its own tile, the
    // block and its number of contributors, merged after the loop, where the streaming state is dead.
    // (aligned mode: the tile of the warp's last row block when another warp shares it.)
    float fin_v[8];
    int fin_r0 = -1, fin_nc = 0;
    long long fin_blk = 0;
    while (it < it_end) {
        const int rb = (int)(it / KC), kc0 = (int)(it % KC);
        const int kc1 = (int)min((long long)KC, kc0 + (it_end - it));
        const int r0 = rb * 16;
        // Rows beyond the edge are clamped (valid addresses); their results are never stored.
        const __half *w0 = Wt + (long long)min(r0 + g, p.Nc - 1) * p.swn;
        const __half *w1 = Wt + (long long)min(r0 + g + 8, p.Nc - 1) * p.swn;
        float d0[4] = {0, 0, 0, 0}, d1[4] = {0, 0, 0, 0};
        for (int kc = kc0; kc < kc1; kc++) {
            uint4 wv0[UNROLL], wv1[UNROLL], av0[UNROLL], av1[UNROLL];
            const uint4 z = make_uint4(0, 0, 0, 0);
            if constexpr (MODE == ACT_F16 && !late) {
                if (!waited) {
                    asm volatile("griddepcontrol.wait;" ::: "memory");
                    waited = true;
                }
#pragma unroll
                for (int u = 0; u < UNROLL; u++) {
                    const int k = (kc * UNROLL + u) * 32 + 8 * t;
                    const bool in = k < p.K;
                    wv0[u] = in ? ldg_w16(w0 + k) : z;
                    wv1[u] = in ? ldg_w16(w1 + k) : z;
                    av0[u] = in ? __ldg(reinterpret_cast<const uint4 *>(a0 + k)) : z;
                    if (TWO_NTILES) av1[u] = in ? __ldg(reinterpret_cast<const uint4 *>(a1 + k)) : z;
                }
            } else {
                if (PRE && (long long)rb * KC + kc == pre_it) {
                    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
                    __syncwarp();
                    const uint8_t *sw = sk_stage + warp * 16 * SK_PRE_ROWB + 16 * t;
#pragma unroll
                    for (int u = 0; u < UNROLL; u++) {
                        wv0[u] = *reinterpret_cast<const uint4 *>(sw + g * SK_PRE_ROWB + 64 * u);
                        wv1[u] = *reinterpret_cast<const uint4 *>(sw + (g + 8) * SK_PRE_ROWB + 64 * u);
                    }
                } else {
#pragma unroll
                    for (int u = 0; u < UNROLL; u++) {
                        const int k = (kc * UNROLL + u) * 32 + 8 * t;
                        const bool in = k < p.K;
                        wv0[u] = in ? ldg_w16(w0 + k) : z;
                        wv1[u] = in ? ldg_w16(w1 + k) : z;
                    }
                    // Right behind the warp's first chunk, its second one goes to shared memory (cp.async), also
                    // before the wait -- after the first chunk, whose data the warp needs first (issued the other way
                    // round, W 12288 x 4096 M = 1 took 19.6 instead of 19.1 µs, 11008 x 4096 18.8 instead of 18.2).
                    if (PRE && pre_it < 0 && (long long)rb * KC + kc + 1 < it_end) {
                        pre_it = (long long)rb * KC + kc + 1;
                        const int prb = (int)(pre_it / KC), pkc = (int)(pre_it % KC);
                        uint8_t *sw = sk_stage + warp * 16 * SK_PRE_ROWB;
                        const int kp = pkc * UNROLL * 32 + 8 * lane;
                        const bool inp = kp < p.K;
#pragma unroll
                        for (int r = 0; r < 16; r++) {
                            const __half *src = Wt + (long long)min(prb * 16 + r, p.Nc - 1) * p.swn + (inp ? kp : 0);
                            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(
                                             (unsigned)__cvta_generic_to_shared(sw + r * SK_PRE_ROWB + 16 * lane)),
                                         "l"(src), "r"(inp ? 16 : 0)
                                         : "memory");
                        }
                        asm volatile("cp.async.commit_group;\n" ::: "memory");
                    }
                }
                if (!waited) {   // everything but the weights may come from the preceding kernel (the split kernel,
                                 // or the previous call of a decode chain): wait for it before the first access
                    asm volatile("griddepcontrol.wait;" ::: "memory");
                    waited = true;
                }
                if constexpr (MODE == ACT_F16S) {
                    // this warp's token rows of the chunk: lane l copies columns 8l .. 8l + 7 of every existing row (rows
                    // past Mc are not copied: their MMA columns are never stored)
                    __syncwarp();   // the previous chunk's fragments have been read by every lane
                    uint8_t *sa = sk_stage + warp * (TWO_NTILES ? 16 : 8) * SK_ROWB;
                    const int k = kc * UNROLL * 32 + 8 * lane;
                    const bool in = k < p.K;
                    const int rows = min(TWO_NTILES ? 16 : 8, p.Mc - t0);
#pragma unroll
                    for (int r = 0; r < (TWO_NTILES ? 16 : 8); r++) {
                        if (r >= rows) break;
                        const __half *src = A + (long long)(t0 + r) * p.sam + (in ? k : 0);
                        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(
                                         (unsigned)__cvta_generic_to_shared(sa + r * SK_ROWB + 16 * lane)),
                                     "l"(src), "r"(in ? 16 : 0)
                                     : "memory");
                    }
                    asm volatile("cp.async.commit_group;\n" ::: "memory");
                    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
                    __syncwarp();
                }
                if constexpr (MODE == ACT_PAIRED && !late) {
#pragma unroll
                    for (int u = 0; u < UNROLL; u++) {
                        const int k = (kc * UNROLL + u) * 32 + 8 * t;
                        const bool in = k < p.K;
                        av0[u] = in ? __ldg(reinterpret_cast<const uint4 *>(a0 + k)) : z;
                        if (TWO_NTILES) av1[u] = in ? __ldg(reinterpret_cast<const uint4 *>(a1 + k)) : z;
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < UNROLL; u++) {
                uint4 lo0 = z, lo1 = z;
                if constexpr (MODE == ACT_F16S) {
                    const uint8_t *sa = sk_stage + warp * (TWO_NTILES ? 16 : 8) * SK_ROWB + (32 * u + 8 * t) * 2;
                    av0[u] = *reinterpret_cast<const uint4 *>(sa + g * SK_ROWB);
                    if (TWO_NTILES) av1[u] = *reinterpret_cast<const uint4 *>(sa + (g + 8) * SK_ROWB);
                } else if constexpr (late) {
                    const int k = (kc * UNROLL + u) * 32 + 8 * t;
                    const bool in = k < p.K;
                    av0[u] = in ? __ldg(reinterpret_cast<const uint4 *>(a0 + k)) : z;
                    if (TWO_NTILES) av1[u] = in ? __ldg(reinterpret_cast<const uint4 *>(a1 + k)) : z;
                    if (MODE == ACT_SPLIT) {
                        lo0 = in ? __ldg(reinterpret_cast<const uint4 *>(l0 + k)) : z;
                        if (TWO_NTILES) lo1 = in ? __ldg(reinterpret_cast<const uint4 *>(l1 + k)) : z;
                    }
                }
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    const uint32_t A0 = word(wv0[u], 2 * j), A1 = word(wv1[u], 2 * j);
                    const uint32_t A2 = word(wv0[u], 2 * j + 1), A3 = word(wv1[u], 2 * j + 1);
                    mma_16816(d0, A0, A1, A2, A3, word(av0[u], 2 * j), word(av0[u], 2 * j + 1));
                    if (TWO_NTILES) mma_16816(d1, A0, A1, A2, A3, word(av1[u], 2 * j), word(av1[u], 2 * j + 1));
                    if constexpr (MODE == ACT_SPLIT) {
                        mma_16816(d0, A0, A1, A2, A3, word(lo0, 2 * j), word(lo0, 2 * j + 1));
                        if (TWO_NTILES) mma_16816(d1, A0, A1, A2, A3, word(lo1, 2 * j), word(lo1, 2 * j + 1));
                    }
                }
            }
        }
        // D fragment: d[0..1] = (row g, tokens 2t, 2t+1), d[2..3] = (row g+8, tokens 2t, 2t+1); d1: tokens + 8.
        // ACT_PAIRED: tokens 2t, 2t+1 are the hi and lo parts of real token t (d1: 4 + t); their sum is its value.
        float v[8];
        int vm[8], vr[8], nv;
        if constexpr (MODE == ACT_PAIRED) {
            v[0] = d0[0] + d0[1]; vr[0] = g;     vm[0] = t;
            v[1] = d0[2] + d0[3]; vr[1] = g + 8; vm[1] = t;
            v[2] = d1[0] + d1[1]; vr[2] = g;     vm[2] = 4 + t;
            v[3] = d1[2] + d1[3]; vr[3] = g + 8; vm[3] = 4 + t;
            nv = TWO_NTILES ? 4 : 2;
        } else {
#pragma unroll
            for (int e = 0; e < 8; e++) {
                v[e] = e < 4 ? d0[e] : d1[e - 4];
                vr[e] = g + ((e & 2) ? 8 : 0);
                vm[e] = 2 * t + (e & 1) + (e >= 4 ? 8 : 0);
            }
            nv = TWO_NTILES ? 8 : 4;
        }
        if (kc0 == 0 && kc1 == KC) {
#pragma unroll
            for (int e = 0; e < 8; e++) {
                if (e >= nv) break;
                const int n = r0 + vr[e], m = t0 + vm[e];
                if (n < p.Nc && m < Mout) skinny_out<F32A>(p, m, n, v[e]);
            }
        } else if (p.aligned) {
            // a block shared with other warps of this CTA: the first block of the range goes to the pads now, the
            // last one (the end of the range) to fin_v; both are added after the loop
            if (rb == first_rb) {
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    if (e >= nv) break;
                    sk_pad_row(sk_stage, warp, vr[e])[vm[e]] = v[e];
                }
                it += kc1 - kc0;
                continue;
            }
#pragma unroll
            for (int e = 0; e < 8; e++) fin_v[e] = v[e];
            fin_r0 = r0;
            break;
        } else {
            const long long x0 = (long long)rb * KC, x1 = x0 + KC - 1;
            const int wf = (int)(((x0 + 1) * W - 1) / T), wl = (int)(((x1 + 1) * W - 1) / T);
            const int nc = wl - wf + 1;
            const long long blk = (long long)blockIdx.y * RB + rb;
            const int cta_w0 = blockIdx.x * WK_WARPS;
            if (wf >= cta_w0 && wl < cta_w0 + WK_WARPS && rb == (T * cta_w0 / W) / KC) {
                // the CTA's first block and every contributor a warp of this CTA: the tile goes to this warp's pads,
                // added after the loop
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    if (e >= nv) break;
                    sk_pad_row(sk_stage, warp, vr[e])[vm[e]] = v[e];
                }
                it += kc1 - kc0;
                continue;
            }
            // Slots of the block: contributor q = wg - wf writes value e of lane l at word e·32 + l of slot q, tagged
            // with this launch's epoch in the upper 32 bits (one relaxed 64-bit store: single-copy atomic, so a tag
            // that matches vouches for its value without any fence).
            uint64_t *slots = part + blk * maxc * 256;
            if (wg != wf) {
                // contributor: the block's later chunks, at the start of this warp's range; it goes on streaming
                uint64_t *sp = slots + (wg - wf) * 256 + lane;
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    if (e >= nv) break;
                    st_relaxed_u64(sp + e * 32, ((uint64_t)p.epoch << 32) | __float_as_uint(v[e]));
                }
            } else {
                // finisher: the block is the last of this warp's range; merged after the loop
#pragma unroll
                for (int e = 0; e < 8; e++) fin_v[e] = v[e];
                fin_r0 = r0;
                fin_nc = nc;
                fin_blk = blk;
                break;
            }
        }
        it += kc1 - kc0;
    }
    if (p.aligned) {
        // Row blocks of this CTA shared by several of its warps: the last-block tiles go to the first 64 bytes of the
        // warp's own staging rows (free now), then thread (row, token) adds the contributors' values in warp order
        // (deterministic) and stores the element.
        if (fin_r0 >= 0) {
            int vm[8], vr[8], nv;
            if constexpr (MODE == ACT_PAIRED) {
                vr[0] = g; vm[0] = t; vr[1] = g + 8; vm[1] = t; vr[2] = g; vm[2] = 4 + t; vr[3] = g + 8; vm[3] = 4 + t;
                nv = TWO_NTILES ? 4 : 2;
            } else {
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    vr[e] = g + ((e & 2) ? 8 : 0);
                    vm[e] = 2 * t + (e & 1) + (e >= 4 ? 8 : 0);
                }
                nv = TWO_NTILES ? 8 : 4;
            }
#pragma unroll
            for (int e = 0; e < 8; e++) {
                if (e >= nv) break;
                sk_last_row(sk_stage, warp, vr[e])[vm[e]] = fin_v[e];
            }
        }
        __syncthreads();
        const int row = threadIdx.x >> 4, tok = threadIdx.x & 15;
        const long long cs0 = (long long)KC * ((long long)RB * blockIdx.x / gridDim.x);
        const long long cn = (long long)KC * ((long long)RB * (blockIdx.x + 1) / gridDim.x) - cs0;
        const long long b0 = cs0 / KC, b1 = (cs0 + cn) / KC;
        for (long long b = b0; b < b1; b++) {
            const long long x0 = b * KC - cs0, x1 = x0 + KC - 1;   // the block's iterations, local to the CTA
            const int wf = (int)(((x0 + 1) * WK_WARPS - 1) / cn), wl = (int)(((x1 + 1) * WK_WARPS - 1) / cn);
            if (wf == wl) continue;   // one warp covered it and stored it
            float acc = 0.0f;
            for (int w = wf; w <= wl; w++) {
                const long long ws = cn * w / WK_WARPS, we = cn * (w + 1) / WK_WARPS;
                if (ws == we) continue;   // a warp without iterations
                acc += (cs0 + ws) / KC == b ? sk_pad_row(sk_stage, w, row)[tok] : sk_last_row(sk_stage, w, row)[tok];
            }
            const int n = (int)b * 16 + row, m = t0 + tok;
            if (n < p.Nc && m < Mout) skinny_out<F32A>(p, m, n, acc);
        }
        skinny_peer_fence(p);
        return;
    }
    if (fin_r0 >= 0) {
        // Finisher of block fin_blk (the warp whose range ends in it, so it meets the block last): it adds the other
        // contributors' values to its own in slot order (deterministic), the loads of SB slots in flight at a time,
        // and waits (bounded) only for values whose tag is not yet this launch's.
        float v[8];
        int vm[8], vr[8], nv;
#pragma unroll
        for (int e = 0; e < 8; e++) v[e] = fin_v[e];
        if constexpr (MODE == ACT_PAIRED) {
            vr[0] = g; vm[0] = t; vr[1] = g + 8; vm[1] = t; vr[2] = g; vm[2] = 4 + t; vr[3] = g + 8; vm[3] = 4 + t;
            nv = TWO_NTILES ? 4 : 2;
        } else {
#pragma unroll
            for (int e = 0; e < 8; e++) {
                vr[e] = g + ((e & 2) ? 8 : 0);
                vm[e] = 2 * t + (e & 1) + (e >= 4 ? 8 : 0);
            }
            nv = TWO_NTILES ? 8 : 4;
        }
        const int nc = fin_nc, r0 = fin_r0;
        const uint64_t *mine = part + fin_blk * maxc * 256 + lane;
        constexpr int SB = TWO_NTILES ? 2 : 4;
        bool ok = true;
        for (int q0 = 1; q0 < nc && ok; q0 += SB) {
            uint64_t x[SB][8];
            bool fresh = true;
#pragma unroll
            for (int j = 0; j < SB; j++) {
#pragma unroll
                for (int e = 0; e < 8; e++)
                    if (q0 + j < nc && e < nv) x[j][e] = ld_relaxed_u64(mine + (q0 + j) * 256 + e * 32);
            }
#pragma unroll
            for (int j = 0; j < SB; j++) {
#pragma unroll
                for (int e = 0; e < 8; e++)
                    if (q0 + j < nc && e < nv) fresh = fresh && (unsigned)(x[j][e] >> 32) == p.epoch;
            }
            if (!fresh) {
                // a contributor has not written yet: poll each value of the batch until its tag is current (tags never
                // go back within a launch), then take the batch again
#pragma unroll 1
                for (int j = 0; j < SB && ok && q0 + j < nc; j++) {
#pragma unroll 1
                    for (int e = 0; e < nv && ok; e++) {
                        const uint64_t *a = mine + (q0 + j) * 256 + e * 32;
                        const unsigned long long t_start = global_ns();
                        while ((unsigned)(ld_relaxed_u64(a) >> 32) != p.epoch)
                            if (global_ns() - t_start > kSkWaitNs) { ok = false; break; }
                    }
                }
                if (!ok) break;
#pragma unroll
                for (int j = 0; j < SB; j++) {
#pragma unroll
                    for (int e = 0; e < 8; e++)
                        if (q0 + j < nc && e < nv) x[j][e] = ld_relaxed_u64(mine + (q0 + j) * 256 + e * 32);
                }
            }
#pragma unroll
            for (int j = 0; j < SB; j++) {
#pragma unroll
                for (int e = 0; e < 8; e++)
                    if (q0 + j < nc && e < nv) v[e] += __uint_as_float((unsigned)x[j][e]);
            }
        }
        if (__all_sync(0xffffffffu, ok)) {
#pragma unroll
            for (int e = 0; e < 8; e++) {
                if (e >= nv) break;
                const int n = r0 + vr[e], m = t0 + vm[e];
                if (n < p.Nc && m < Mout) skinny_out<F32A>(p, m, n, v[e]);
            }
        } else if (lane == 0) {
            atomicExch(p.err, kDevErrWaitTimeout);
        }
    }
    // The CTA's first row block, if all its contributors are this CTA's warps: their tiles are in their pads;
    // thread (row, token) adds them in warp order (deterministic) and stores the element.
    __syncthreads();
    {
        const int cta_w0 = blockIdx.x * WK_WARPS;
        const long long cx0 = T * cta_w0 / W, cx1 = T * (cta_w0 + WK_WARPS) / W;
        const long long b = cx0 / KC, y0 = b * KC, y1 = y0 + KC - 1;
        const int wf = (int)(((y0 + 1) * W - 1) / T), wl = (int)(((y1 + 1) * W - 1) / T);
        if (cx0 < cx1 && wf >= cta_w0 && wl < cta_w0 + WK_WARPS && wl > wf) {
            const int row = threadIdx.x >> 4, tok = threadIdx.x & 15;
            float acc = 0.0f;
            for (int q = wf - cta_w0; q <= wl - cta_w0; q++) acc += sk_pad_row(sk_stage, q, row)[tok];
            const int n = (int)b * 16 + row, m = t0 + tok;
            if (n < p.Nc && m < Mout) skinny_out<F32A>(p, m, n, acc);
        }
    }
    skinny_peer_fence(p);
}

// The 8 K-consecutive token values of a fragment (16 bytes of FP16): FP16 activations as stored, or F32 activations
// rounded to FP16 (ACT_F32H; two 16-byte loads).
template <int MODE>
__device__ __forceinline__ uint4 act_frag(const SkinnyArgs &p, int m, int k) {
    if constexpr (MODE == ACT_F32H) {
        const float4 *f = reinterpret_cast<const float4 *>((const float *)p.a + (long long)m * p.sam + k);
        const float4 x = __ldg(f), y = __ldg(f + 1);
        const __half2 h0 = __floats2half2_rn(x.x, x.y), h1 = __floats2half2_rn(x.z, x.w);
        const __half2 h2 = __floats2half2_rn(y.x, y.y), h3 = __floats2half2_rn(y.z, y.w);
        return make_uint4(*reinterpret_cast<const uint32_t *>(&h0), *reinterpret_cast<const uint32_t *>(&h1),
                          *reinterpret_cast<const uint32_t *>(&h2), *reinterpret_cast<const uint32_t *>(&h3));
    } else {
        return __ldg(reinterpret_cast<const uint4 *>((const __half *)p.a + (long long)m * p.sam + k));
    }
}

// ------------------------------------------------------------------------------------------------ FP16, one block per CTA
// wk_f16_blk: the common decode plan written out -- one 16-row weight block per CTA, up to 8 FP16 tokens, warp w taking
// K chunks [KC·w/8, KC·(w+1)/8) of 256. The warp requests its first chunk into registers and its second into its
// staging rows (cp.async) before the wait, the rest in turn; its 16 × 8 FP32 tile goes to its pads and the CTA adds the
// eight tiles after one barrier. Same MMA fragments, K permutation and stores as wk_f16_sk, without its stream-K
// bookkeeping (W 4096 × 4096 M = 1, calls back to back on B200: 5.8 µs against 7.7 with wk_f16_sk; 4096 × 11008 15.0
// against 17.5). A version looping over several blocks per CTA (next block's requests before the barrier, two pad
// sets) was slower on every shape, including the one-block ones (7.0 and 16.8 µs).
template <bool FULLK, bool TWO, int MODE = ACT_F16, bool F16W = false, bool SWI = false>
__global__ void __launch_bounds__(WK_WARPS * 32, 2) wk_f16_blk(const SkinnyArgs p, int KC) {
    static_assert(MODE == ACT_F16 || MODE == ACT_PAIRED || MODE == ACT_SPLIT || MODE == ACT_F32H, "token modes");
    static_assert(!F16W || MODE == ACT_F16 || MODE == ACT_F32H, "the f16w epilogue takes FP16-rounded tokens");
    static_assert(!SWI || ((MODE == ACT_F16 || MODE == ACT_F32H) && !F16W), "the gate / up pair stores FP16 results");
    constexpr bool F32A = MODE == ACT_PAIRED || MODE == ACT_SPLIT;
    extern __shared__ __align__(16) uint8_t sk_stage[];
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int blk = SWI ? blockIdx.x >> 1 : blockIdx.x, which = SWI ? blockIdx.x & 1 : 0;   // SWI: 0 gate, 1 up
    const int r0 = blk * 16;
    const int c0 = KC * warp / WK_WARPS, c1 = KC * (warp + 1) / WK_WARPS;
    const __half *Wt = (const __half *)(which ? p.w2 : p.w);
    const __half *w0 = Wt + (long long)min(r0 + g, p.Nc - 1) * p.swn;
    const __half *w1 = Wt + (long long)min(r0 + g + 8, p.Nc - 1) * p.swn;
    const __half *a0 = (const __half *)p.a + (long long)min(g, p.Mc - 1) * p.sam;   // token g (clamped: not stored)
    const __half *a1 = (const __half *)p.a + (long long)min(g + 8, p.Mc - 1) * p.sam;   // TWO: token g + 8
    uint8_t *sw = sk_stage + warp * 16 * SK_ROWB;
    const uint4 z = make_uint4(0, 0, 0, 0);
    if (!p.early_w) asm volatile("griddepcontrol.wait;" ::: "memory");
    uint4 wv0[8], wv1[8];
    if (c0 < c1) {
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int k = c0 * 256 + 32 * u + 8 * t;
            const bool in = FULLK || k < p.K;
            wv0[u] = in ? ldg_w16(w0 + k) : z;
            wv1[u] = in ? ldg_w16(w1 + k) : z;
        }
        if (c0 + 1 < c1) {   // the second chunk: lane l copies 16 bytes of each of the 16 rows
            const int kp = (c0 + 1) * 256 + 8 * lane;
            const bool inp = FULLK || kp < p.K;
#pragma unroll
            for (int r = 0; r < 16; r++) {
                const __half *src = Wt + (long long)min(r0 + r, p.Nc - 1) * p.swn + (inp ? kp : 0);
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(
                                 (unsigned)__cvta_generic_to_shared(sw + r * SK_ROWB + 16 * lane)),
                             "l"(src), "r"(inp ? 16 : 0)
                             : "memory");
            }
            asm volatile("cp.async.commit_group;\n" ::: "memory");
        }
    }
    if (p.early_w) asm volatile("griddepcontrol.wait;" ::: "memory");
    float d[4] = {0.0f, 0.0f, 0.0f, 0.0f}, d1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int c = c0; c < c1; c++) {
        if (c == c0 + 1) {
            asm volatile("cp.async.wait_group 0;\n" ::: "memory");
            __syncwarp();
#pragma unroll
            for (int u = 0; u < 8; u++) {
                wv0[u] = *reinterpret_cast<const uint4 *>(sw + g * SK_ROWB + 16 * t + 64 * u);
                wv1[u] = *reinterpret_cast<const uint4 *>(sw + (g + 8) * SK_ROWB + 16 * t + 64 * u);
            }
        } else if (c > c0 + 1) {
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int k = c * 256 + 32 * u + 8 * t;
                const bool in = FULLK || k < p.K;
                wv0[u] = in ? ldg_w16(w0 + k) : z;
                wv1[u] = in ? ldg_w16(w1 + k) : z;
            }
        }
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int k = c * 256 + 32 * u + 8 * t;
            const bool in = FULLK || k < p.K;
            const uint4 av = in ? act_frag<MODE>(p, min(g, p.Mc - 1), k) : z;
#pragma unroll
            for (int j = 0; j < 2; j++)
                mma_16816(d, word(wv0[u], 2 * j), word(wv1[u], 2 * j), word(wv0[u], 2 * j + 1), word(wv1[u], 2 * j + 1),
                          word(av, 2 * j), word(av, 2 * j + 1));
            if (TWO) {
                const uint4 av1 = in ? act_frag<MODE>(p, min(g + 8, p.Mc - 1), k) : z;
#pragma unroll
                for (int j = 0; j < 2; j++)
                    mma_16816(d1, word(wv0[u], 2 * j), word(wv1[u], 2 * j), word(wv0[u], 2 * j + 1),
                              word(wv1[u], 2 * j + 1), word(av1, 2 * j), word(av1, 2 * j + 1));
            }
            if (MODE == ACT_SPLIT) {   // the lo parts of the same tokens into the same accumulators
                const uint4 lv0 = in ? __ldg(reinterpret_cast<const uint4 *>(a0 + p.alo + k)) : z;
#pragma unroll
                for (int j = 0; j < 2; j++)
                    mma_16816(d, word(wv0[u], 2 * j), word(wv1[u], 2 * j), word(wv0[u], 2 * j + 1), word(wv1[u], 2 * j + 1),
                              word(lv0, 2 * j), word(lv0, 2 * j + 1));
                if (TWO) {
                    const uint4 lv1 = in ? __ldg(reinterpret_cast<const uint4 *>(a1 + p.alo + k)) : z;
#pragma unroll
                    for (int j = 0; j < 2; j++)
                        mma_16816(d1, word(wv0[u], 2 * j), word(wv1[u], 2 * j), word(wv0[u], 2 * j + 1),
                                  word(wv1[u], 2 * j + 1), word(lv1, 2 * j), word(lv1, 2 * j + 1));
                }
            }
        }
    }
    // D fragment: d[0..1] = (row g, tokens 2t, 2t+1), d[2..3] = (row g + 8, tokens 2t, 2t+1)
    float *pg = sk_pad_row(sk_stage, warp, g), *pg8 = sk_pad_row(sk_stage, warp, g + 8);
    pg[2 * t] = d[0];
    pg[2 * t + 1] = d[1];
    pg8[2 * t] = d[2];
    pg8[2 * t + 1] = d[3];
    if (TWO) {   // tokens 8 + 2t, 9 + 2t
        pg[8 + 2 * t] = d1[0];
        pg[9 + 2 * t] = d1[1];
        pg8[8 + 2 * t] = d1[2];
        pg8[9 + 2 * t] = d1[3];
    }
    __syncthreads();
    const int row = threadIdx.x >> 4, tok = threadIdx.x & 15;
    if constexpr (MODE == ACT_PAIRED) {
        // virtual token rows 2m (hi) and 2m + 1 (lo) of real token m: their sum is its value
        if (tok < p.Mc / 2 && r0 + row < p.Nc) {
            float acc = 0.0f;
#pragma unroll
            for (int w = 0; w < WK_WARPS; w++) {
                const float *pw = sk_pad_row(sk_stage, w, row);
                acc += pw[2 * tok] + pw[2 * tok + 1];
            }
            skinny_out<true>(p, tok, r0 + row, acc);
        }
    } else if (tok < p.Mc && r0 + row < p.Nc) {
        float acc = 0.0f;
#pragma unroll
        for (int w = 0; w < WK_WARPS; w++) acc += sk_pad_row(sk_stage, w, row)[tok];
        if constexpr (F16W) {
            // as gemm_pb_f16w's separate epilogue, operation for operation: the FP16 result, then bias / GELU / residual
            const int n = r0 + row;
            float v = __half2float(__float2half_rn(acc));
            if (!isfinite(v)) *(volatile unsigned *)p.nf = 1u;
            if (p.bias) v = __fadd_rn(v, p.bias[n]);
            if (p.gelu) v = gelu_ggml(v);
            if (p.R) v = __fadd_rn(v, p.R[(long long)tok * p.ldr + n]);
            reinterpret_cast<float *>(p.C)[(long long)tok * p.scm + n] = v;
        } else if constexpr (SWI) {   // the GEMM's FP16 result, as skinny_store with alpha = 1, beta = 0
            reinterpret_cast<__half *>(which ? p.c2 : p.C)[(long long)tok * p.scm + r0 + row] = __float2half_rn(acc);
        } else {
            skinny_out<F32A>(p, tok, r0 + row, acc);
        }
    }
    if constexpr (SWI) {
        // arrival of this half of the pair; the second arrival applies SWIGLU to the block's rows (the operations of
        // ffn_f16w's separate swiglu_f16, element for element)
        __shared__ int sw_last;
        __syncthreads();   // every FP16 result of this CTA is stored (the release below covers them)
        if (threadIdx.x == 0) {
            __threadfence();
            sw_last = atomicAdd(p.cnt + blk, 1u) == 1u;
            __threadfence();
        }
        __syncthreads();
        if (sw_last) {
            const int n = r0 + row;
            if (tok < p.Mc && n < p.ldh) {
                float h = 0.0f;
                bool bad = false;
                if (n < p.Nc) {
                    const long long o = (long long)tok * p.scm + n;
                    const float gv = __half2float(__ushort_as_half(__ldcg(reinterpret_cast<const unsigned short *>(p.C) + o)));
                    const float uv = __half2float(__ushort_as_half(__ldcg(reinterpret_cast<const unsigned short *>(p.c2) + o)));
                    h = __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv))), uv);
                    bad = !isfinite(gv) || !isfinite(uv) || !(fabsf(h) <= 65504.0f);
                }
                p.hsw[(long long)tok * p.ldh + n] = __float2half_rn(h);
                if (bad) *(volatile unsigned *)p.nf = 1u;
            }
            const int nb = (int)(gridDim.x >> 1);
            if (blk == nb - 1) {   // columns past the last block, up to the pitch: zero
                const long long w0 = (long long)nb * 16, wn = p.ldh - w0;
                for (long long i = threadIdx.x; i < (long long)p.Mc * wn; i += blockDim.x)
                    p.hsw[(i / wn) * p.ldh + w0 + i % wn] = __float2half_rn(0.0f);
            }
            if (threadIdx.x == 0) p.cnt[blk] = 0u;   // the next call finds the counter at zero
        }
    }
    skinny_peer_fence(p);
}

// ------------------------------------------------------------------------------------------------ FP32, K-contiguous
constexpr int WKF_ROWS = 4;

// Requirements: K % 4 == 0, rows 16-byte aligned. grid = (ceil(Nc / 4), ceil(Mc / MT)).
template <int MT>
__global__ void __launch_bounds__(WK_WARPS * 32) wk_f32(const SkinnyArgs p) {
    __shared__ float red[WK_WARPS][WKF_ROWS][MT];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = blockIdx.x * WKF_ROWS, t0 = blockIdx.y * MT;
    const float *W = (const float *)p.w;
    const float *A = (const float *)p.a;
    const int nv = p.K / 4;
    const int per_warp = (nv + WK_WARPS - 1) / WK_WARPS;
    const int v_beg = warp * per_warp, v_end = min(nv, v_beg + per_warp);
    float acc[WKF_ROWS][MT];
#pragma unroll
    for (int r = 0; r < WKF_ROWS; r++)
#pragma unroll
        for (int m = 0; m < MT; m++) acc[r][m] = 0;
    const float *wrow[WKF_ROWS];
#pragma unroll
    for (int r = 0; r < WKF_ROWS; r++) wrow[r] = W + (long long)min(r0 + r, p.Nc - 1) * p.swn;
    const float *arow[MT];
#pragma unroll
    for (int m = 0; m < MT; m++) arow[m] = A + (long long)min(t0 + m, p.Mc - 1) * p.sam;
    for (int v = v_beg + lane; v < v_end; v += 32) {
        float4 wv[WKF_ROWS];
#pragma unroll
        for (int r = 0; r < WKF_ROWS; r++) {
            uint4 u = ldg_nc16(wrow[r] + 4 * v);
            wv[r] = make_float4(__uint_as_float(u.x), __uint_as_float(u.y), __uint_as_float(u.z), __uint_as_float(u.w));
        }
#pragma unroll
        for (int m = 0; m < MT; m++) {
            const float4 av = __ldg(reinterpret_cast<const float4 *>(arow[m] + 4 * v));
#pragma unroll
            for (int r = 0; r < WKF_ROWS; r++) {
                acc[r][m] = __fmaf_rn(wv[r].x, av.x, acc[r][m]);
                acc[r][m] = __fmaf_rn(wv[r].y, av.y, acc[r][m]);
                acc[r][m] = __fmaf_rn(wv[r].z, av.z, acc[r][m]);
                acc[r][m] = __fmaf_rn(wv[r].w, av.w, acc[r][m]);
            }
        }
    }
#pragma unroll
    for (int r = 0; r < WKF_ROWS; r++)
#pragma unroll
        for (int m = 0; m < MT; m++) {
            float s = acc[r][m];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (lane == 0) red[warp][r][m] = s;
        }
    __syncthreads();
    for (int i = threadIdx.x; i < WKF_ROWS * MT; i += blockDim.x) {
        const int r = i / MT, m = i % MT;
        const int n = r0 + r, mm = t0 + m;
        if (n < p.Nc && mm < p.Mc) {
            float s = 0;
#pragma unroll
            for (int w = 0; w < WK_WARPS; w++) s += red[w][r][m];
            skinny_store<float>(p, mm, n, s);
        }
    }
    skinny_peer_fence(p);
}

// ------------------------------------------------------------------------------------------------ N-contiguous
constexpr int WN_THREADS = 256, WN_COLS = 4, WN_MT = 16, WN_KC = 64;

// P[part][m][n] = Σ_{k in part} a[m][k]·w[k][n] for 16 tokens (blockIdx.z) and 4 columns per thread.
template <typename T>
__global__ void __launch_bounds__(WN_THREADS) wn_partial(const SkinnyArgs p, int kpp, float *P) {
    __shared__ float as[WN_MT][WN_KC];
    const int n = (blockIdx.x * WN_THREADS + threadIdx.x) * WN_COLS;
    const int part = blockIdx.y, t0 = blockIdx.z * WN_MT;
    const int kb = part * kpp, ke = min(p.K, kb + kpp);
    const T *W = (const T *)p.w;
    const T *A = (const T *)p.a;
    float acc[WN_MT][WN_COLS];
#pragma unroll
    for (int m = 0; m < WN_MT; m++)
#pragma unroll
        for (int c = 0; c < WN_COLS; c++) acc[m][c] = 0;
    for (int k0 = kb; k0 < ke; k0 += WN_KC) {
        const int kn = min(WN_KC, ke - k0);
        __syncthreads();
        for (int i = threadIdx.x; i < WN_MT * WN_KC; i += WN_THREADS) {
            const int m = i / WN_KC, k = i % WN_KC;
            as[m][k] = (t0 + m < p.Mc && k < kn) ? to_r(A[(long long)(t0 + m) * p.sam + (long long)(k0 + k) * p.sak]) : 0.0f;
        }
        __syncthreads();
        if (n < p.Nc) {
            for (int k = 0; k < kn; k++) {
                const T *wp = W + (long long)(k0 + k) * p.swk + n;
                float wv[WN_COLS];
#pragma unroll
                for (int c = 0; c < WN_COLS; c++) wv[c] = n + c < p.Nc ? to_r(__ldg(wp + c)) : 0.0f;
#pragma unroll
                for (int m = 0; m < WN_MT; m++) {
                    const float av = as[m][k];
#pragma unroll
                    for (int c = 0; c < WN_COLS; c++) acc[m][c] = __fmaf_rn(av, wv[c], acc[m][c]);
                }
            }
        }
    }
    if (n >= p.Nc) return;
#pragma unroll
    for (int m = 0; m < WN_MT; m++) {
        if (t0 + m >= p.Mc) break;
        float *out = P + ((long long)part * p.Mc + t0 + m) * p.Nc + n;
#pragma unroll
        for (int c = 0; c < WN_COLS; c++)
            if (n + c < p.Nc) out[c] = acc[m][c];
    }
}

template <typename T>
__global__ void __launch_bounds__(256) wn_final(const SkinnyArgs p, int parts, const float *P) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= (long long)p.Mc * p.Nc) return;
    const int m = (int)(i / p.Nc), n = (int)(i % p.Nc);
    float s = 0;
    for (int q = 0; q < parts; q++) s += P[((long long)q * p.Mc + m) * p.Nc + n];
    skinny_store<T>(p, m, n, s);
    skinny_peer_fence(p);
}

// ------------------------------------------------------------------------------------------------ generic
// One warp per weight row n, tokens in groups of 8, lanes stride K. Any strides.
template <typename T>
__global__ void __launch_bounds__(256) skinny_generic(const SkinnyArgs p) {
    const int lane = threadIdx.x & 31;
    const long long n = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    if (n >= p.Nc) return;
    const T *W = (const T *)p.w + n * p.swn;
    const T *A = (const T *)p.a;
    for (int m0 = 0; m0 < p.Mc; m0 += 8) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int k = lane; k < p.K; k += 32) {
            const float wv = to_r(W[(long long)k * p.swk]);
#pragma unroll
            for (int j = 0; j < 8; j++)
                if (m0 + j < p.Mc) acc[j] = __fmaf_rn(wv, to_r(A[(long long)(m0 + j) * p.sam + (long long)k * p.sak]), acc[j]);
        }
#pragma unroll
        for (int j = 0; j < 8; j++) {
            float s = acc[j];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (lane == 0 && m0 + j < p.Mc) skinny_store<T>(p, m0 + j, (int)n, s);
        }
    }
    skinny_peer_fence(p);
}

// Dense K-contiguous copy of the small operand (Mc × K, row pitch Kp = K rounded up to 8) for the fast kernels.
template <typename T>
__global__ void repack_small(const T *__restrict__ a, long long sam, long long sak, int Mc, int K, int Kp, T *dst) {
    const long long n = (long long)Mc * Kp;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int m = (int)(i / Kp), k = (int)(i % Kp);
        dst[i] = k < K ? a[(long long)m * sam + (long long)k * sak] : T(0);
    }
}

// Stream-K plan of wk_f16_sk: a one-wave grid of CTAs, K chunks of unroll·32 elements, and the partial-tile slots
// per 16-row block (the most warps that can share one block).
struct SkPlan {
    int KC, RB, mtiles, maxc, aligned;
    long long ctas;
    size_t part_words;   // tagged partial-tile words (global mode): mtiles × RB × maxc slots of 256
};

// Launch plan of wk_f16_sk. Aligned mode (whole row blocks per CTA: the fewest blocks per CTA that keep the grid
// within one wave and give each of the 8 warps a chunk, spread evenly -- 256 blocks: 256 CTAs of one; 768: 256 of
// three) when that still gives at least one CTA per SM and either K spans at least 32 chunks or two token tiles run
// with several blocks per CTA. Measured on B200, same box, µs (global / aligned): W 4096 x 11008 M = 1 19.7 / 17.9,
// M = 16 25.0 / 21.4; 12288 x 4096 M = 16 26.3 / 24.6, M = 1 19.8 / 20.0; 11008 x 4096 equal; 4096 x 4096 M = 1
// 8.0 / 9.1. Otherwise the whole iteration space is split over a one-wave grid with at least ~2 iterations per warp.
static SkPlan sk_plan(int Mc, int Nc, int K, int unroll, int sm_count) {
    SkPlan q;
    q.KC = (K + unroll * 32 - 1) / (unroll * 32);
    q.RB = (Nc + 15) / 16;
    q.mtiles = (Mc + 15) / 16;
    long long per = (q.RB + 2LL * sm_count - 1) / (2LL * sm_count);
    if (per * q.KC < WK_WARPS) per = (WK_WARPS + q.KC - 1) / q.KC;
    const long long g_al = (q.RB + per - 1) / per;
    if (g_al >= sm_count && (q.KC >= 32 || (Mc > 8 && per >= 2))) {
        q.aligned = 1;
        q.ctas = g_al;
        q.maxc = 0;
        q.part_words = 0;
        return q;
    }
    q.aligned = 0;
    const long long iters = (long long)q.RB * q.KC;
    long long ctas = (iters + 2 * WK_WARPS - 1) / (2 * WK_WARPS);   // at least ~2 iterations per warp
    if (ctas > 2 * sm_count) ctas = 2 * sm_count;
    if (ctas < 1) ctas = 1;
    const long long per_w = iters / (ctas * WK_WARPS);
    q.maxc = (int)(per_w == 0 ? q.KC : (q.KC / per_w + 2 < q.KC ? q.KC / per_w + 2 : q.KC));
    q.ctas = ctas;
    q.part_words = (size_t)q.mtiles * q.RB * q.maxc * 256;
    return q;
}

template <typename T>
static int skinny_t(SkinnyArgs p, cudaStream_t st) {
    DevState *d = dev_state();
    if (!d) return G.status;
    const int es = sizeof(T);
    if (p.swk == 1) {
        // Fast path when the weight rows allow 16-byte loads; the small operand is repacked when it does not.
        const int kq = 16 / es;   // elements per 16-byte load
        const bool w_ok = ((uintptr_t)p.w & 15) == 0 && (p.swn * es) % 16 == 0 && p.K % kq == 0;
        if (w_ok) {
            const bool a_ok = p.sak == 1 && ((uintptr_t)p.a & 15) == 0 && (p.sam * es) % 16 == 0;
            // Scratch: the repacked small operand (when needed); the partial tiles have their own buffer.
            const size_t a_bytes = a_ok ? 0 : ((size_t)p.Mc * p.K * es + 255) / 256 * 256;
            const SkPlan q = sk_plan(p.Mc, p.Nc, p.K, 8, d->sm_count);
            void *scr = nullptr;
            if (a_bytes) G9_TRY(scratch(a_bytes, &scr));
            if (!a_ok) {
                repack_small<T><<<d->sm_count * 4, 256, 0, st>>>((const T *)p.a, p.sam, p.sak, p.Mc, p.K, p.K, (T *)scr);
                G9_TRY(launched("repack_small"));
                p.a = scr;
                p.sam = p.K;
                p.sak = 1;
            }
            if (sizeof(T) == 2) {
                p.early_w = !queued_writes_overlap(d, p.w, ((size_t)(p.Nc - 1) * p.swn + p.K) * sizeof(T));
                const int rb = (p.Nc + 15) / 16;
                if (rb >= d->sm_count && q.KC >= WK_WARPS) {
                    // one row block per CTA (several waves when the blocks outnumber two per SM)
                    const bool fullk = p.K % 256 == 0, two_t = p.Mc > 8;
                    const int smem = SK_SMEM_BYTES;
                    static bool attr_b[4][kMaxDevices] = {};
                    auto kern = fullk ? (two_t ? wk_f16_blk<true, true> : wk_f16_blk<true, false>)
                                      : (two_t ? wk_f16_blk<false, true> : wk_f16_blk<false, false>);
                    G9_CU(smem_limit_once(kern, smem, attr_b[(fullk ? 2 : 0) + (two_t ? 1 : 0)]));
                    const dim3 grid((unsigned)rb), blk(WK_WARPS * 32);
                    if (p.ndst == 1) launch_pdl(kern, grid, blk, smem, st, p, q.KC);
                    else kern<<<grid, blk, smem, st>>>(p, q.KC);
                    return launched("skinny_wk_f16_blk");
                }
                uint64_t *part = nullptr;
                if (!q.aligned) G9_TRY(skinny_slots(q.part_words, &part, &p.epoch));
                p.err = d->err_dev;
                p.aligned = q.aligned;
                dim3 grid((unsigned)q.ctas, q.mtiles);
                // Single-device calls overlap the previous call's tail (programmatic dependent launch); the fused
                // all-gather keeps ordinary stream order around its rank barrier.
                const dim3 blk(WK_WARPS * 32);
                const bool two = p.Mc > 8;
                const int smem = SK_SMEM_BYTES;   // staging (two token tiles) or second-iteration weights, CTA tiles
                static bool attr[kMaxDevices] = {};
                if (two) G9_CU(smem_limit_once(wk_f16_sk<true, 8, ACT_F16S, true>, smem, attr));
                static bool attr1[kMaxDevices] = {};
                if (!two) G9_CU(smem_limit_once(wk_f16_sk<false, 8, ACT_F16, true>, SK_SMEM_BYTES, attr1));
                if (p.ndst == 1) {
                    if (two) launch_pdl(wk_f16_sk<true, 8, ACT_F16S, true>, grid, blk, smem, st, p, q.KC, q.maxc, part);
                    else launch_pdl(wk_f16_sk<false, 8, ACT_F16, true>, grid, blk, SK_SMEM_BYTES, st, p, q.KC, q.maxc, part);
                } else if (two) {
                    wk_f16_sk<true, 8, ACT_F16S, true><<<grid, blk, smem, st>>>(p, q.KC, q.maxc, part);
                } else {
                    wk_f16_sk<false, 8, ACT_F16, true><<<grid, blk, SK_SMEM_BYTES, st>>>(p, q.KC, q.maxc, part);
                }
                return launched("skinny_wk_f16_sk");
            }
            const int mt = p.Mc <= 1 ? 1 : p.Mc <= 4 ? 4 : p.Mc <= 8 ? 8 : 16;
            dim3 grid((p.Nc + WKF_ROWS - 1) / WKF_ROWS, (p.Mc + mt - 1) / mt);
            if (mt == 1) wk_f32<1><<<grid, WK_WARPS * 32, 0, st>>>(p);
            else if (mt == 4) wk_f32<4><<<grid, WK_WARPS * 32, 0, st>>>(p);
            else if (mt == 8) wk_f32<8><<<grid, WK_WARPS * 32, 0, st>>>(p);
            else wk_f32<16><<<grid, WK_WARPS * 32, 0, st>>>(p);
            return launched("skinny_wk_f32");
        }
        const long long warps = p.Nc;
        skinny_generic<T><<<(unsigned)((warps * 32 + 255) / 256), 256, 0, st>>>(p);
        return launched("skinny_generic");
    }
    // Weights contiguous along N: split K into parts so that the grid covers the GPU, then a fixed-order sum.
    const int col_blocks = (p.Nc + WN_THREADS * WN_COLS - 1) / (WN_THREADS * WN_COLS);
    const int mtiles = (p.Mc + WN_MT - 1) / WN_MT;
    int parts = (d->sm_count * 4 + col_blocks * mtiles - 1) / (col_blocks * mtiles);
    const int max_parts = (p.K + WN_KC - 1) / WN_KC;
    if (parts > max_parts) parts = max_parts;
    if (parts < 1) parts = 1;
    int kpp = (p.K + parts - 1) / parts;
    kpp = (kpp + WN_KC - 1) / WN_KC * WN_KC;
    parts = (p.K + kpp - 1) / kpp;
    void *P = nullptr;
    G9_TRY(scratch((size_t)parts * p.Mc * p.Nc * sizeof(float), &P));
    dim3 grid(col_blocks, parts, mtiles);
    wn_partial<T><<<grid, WN_THREADS, 0, st>>>(p, kpp, (float *)P);
    G9_TRY(launched("skinny_wn_partial"));
    const long long outs = (long long)p.Mc * p.Nc;
    wn_final<T><<<(unsigned)((outs + 255) / 256), 256, 0, st>>>(p, parts, (const float *)P);
    return launched("skinny_wn_final");
}

// ------------------------------------------------------------------------------------------------ F32 activations
constexpr int SPLIT_THREADS = 512;

// Input of the F32-activation kernel: row m of a, scaled by 2^s (s puts the row's largest magnitude in [2^14, 2^15),
// clamped to |s| <= 126), split into FP16 hi = rn(x) and lo = rn(x - hi) (rows of Kp elements, zero past K);
// tscale[m] = 2^-s. x - hi is exact in FP32, so hi + lo carries x to 2^-22 relative plus 2^-25 absolute (FP16
// subnormals), i.e. 2^-39 of the row's largest value. A row holding inf or NaN is not scaled (s = 0); its results come
// out non-finite and are flagged. One CTA per row, 16-byte loads when the rows allow them (vec4); the second pass
// re-reads the row from L1.
// The kernel lets its dependent grid (the weight-streaming kernel, launched with programmatic stream serialization)
// start right away: that grid issues its first weight loads and then waits (griddepcontrol.wait) for this one.
// Row m of the parts starts at hi + m·rs and lo + m·rs (ACT_PAIRED: rs = 2·Kp, lo = hi + Kp; ACT_SPLIT: rs = Kp, lo
// = hi + M·Kp).
__global__ void __launch_bounds__(SPLIT_THREADS) split_f32_rows(const float *__restrict__ a, long long lda, int K,
                                                               int Kp, bool vec4, __half *__restrict__ hi,
                                                               __half *__restrict__ lo, long long rs,
                                                               float *__restrict__ tscale) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");   // A may be the previous call's output
    __shared__ float red[SPLIT_THREADS / 32];
    __shared__ float sc;
    const int m = blockIdx.x;
    const float *row = a + (long long)m * lda;
    const int K4 = vec4 ? K / 4 : 0;
    float mx = 0.0f;
    for (int i = threadIdx.x; i < K4; i += SPLIT_THREADS) {
        const float4 v = reinterpret_cast<const float4 *>(row)[i];
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
    for (int k = 4 * K4 + threadIdx.x; k < K; k += SPLIT_THREADS) mx = fmaxf(mx, fabsf(row[k]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < SPLIT_THREADS / 32; w++) mx = fmaxf(mx, red[w]);
        const int e = (int)((__float_as_uint(mx) >> 23) & 255u);   // biased exponent; 0 for zero / subnormal
        int s = 0;
        if (mx > 0.0f && e != 255) {
            s = 14 - ((e == 0 ? 1 : e) - 127);
            s = s > 126 ? 126 : s < -126 ? -126 : s;
        }
        sc = __uint_as_float((unsigned)(s + 127) << 23);
        tscale[m] = __uint_as_float((unsigned)(127 - s) << 23);
    }
    __syncthreads();
    const float f = sc;
    __half *h = hi + (long long)m * rs, *l = lo + (long long)m * rs;
    for (int i = threadIdx.x; i < Kp / 4; i += SPLIT_THREADS) {   // Kp is a multiple of 8: 8-byte stores
        const int k = 4 * i;
        float x[4];
        if (i < K4) {
            const float4 v = reinterpret_cast<const float4 *>(row)[i];
            x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
        } else {
#pragma unroll
            for (int j = 0; j < 4; j++) x[j] = k + j < K ? row[k + j] : 0.0f;
        }
        __half2 hv[2], lv[2];
#pragma unroll
        for (int j = 0; j < 2; j++) {
            const float x0 = x[2 * j] * f, x1 = x[2 * j + 1] * f;
            hv[j] = __floats2half2_rn(x0, x1);
            const float2 hf = __half22float2(hv[j]);
            lv[j] = __floats2half2_rn(x0 - hf.x, x1 - hf.y);
        }
        *reinterpret_cast<uint2 *>(h + k) = make_uint2(*reinterpret_cast<uint32_t *>(&hv[0]), *reinterpret_cast<uint32_t *>(&hv[1]));
        *reinterpret_cast<uint2 *>(l + k) = make_uint2(*reinterpret_cast<uint32_t *>(&lv[0]), *reinterpret_cast<uint32_t *>(&lv[1]));
    }
}

template <bool TWO_NTILES, int UNROLL, int MODE, bool LAZY = false>
static int launch_f32a_main(const SkinnyArgs &p, const SkPlan &q, uint64_t *part, cudaStream_t st) {
    static bool attr[kMaxDevices] = {};
    G9_CU(smem_limit_once(wk_f16_sk<TWO_NTILES, UNROLL, MODE, LAZY>, SK_SMEM_BYTES, attr));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)q.ctas, q.mtiles);
    cfg.blockDim = dim3(WK_WARPS * 32);
    cfg.dynamicSmemBytes = SK_SMEM_BYTES;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, wk_f16_sk<TWO_NTILES, UNROLL, MODE, LAZY>, p, q.KC, q.maxc, part);
    return launched("skinny_wk_f16_sk_f32a");
}

int launch_skinny_f32a(int M, int N, int K, const float *A, int lda, const void *W, int ldw, float *C, int ldc,
                       unsigned *nf, cudaStream_t st) {
    DevState *d = dev_state();
    if (!d) return G.status;
    const int Kp = (K + 7) / 8 * 8;
    if (ldw < Kp || ldw % 8 != 0 || ((uintptr_t)W & 15) != 0)
        return fail(GEN9BLAS_ERR_INVALID_ARG, "F32-activation skinny GEMM: weight rows must be padded, 16-byte aligned");
    SkinnyArgs p;
    memset(&p, 0, sizeof(p));
    const bool paired = M <= 8;
    p.Mc = paired ? 2 * M : M;   // ACT_PAIRED: virtual token rows (hi, lo interleaved)
    p.Nc = N; p.K = Kp;
    p.alpha = 1.0f; p.beta = 0.0f;
    p.w = W; p.swn = ldw; p.swk = 1;
    p.C = C; p.scm = ldc; p.scn = 1;
    p.dst[0] = C; p.ndst = 1; p.coff = 0;
    p.sam = Kp; p.sak = 1;
    p.alo = paired ? 0 : (long long)M * Kp;
    p.nf = nf;
    p.early_w = !queued_writes_overlap(d, W, ((size_t)(N - 1) * ldw + Kp) * sizeof(__half));
    const SkPlan q = sk_plan(p.Mc, N, Kp, 8, d->sm_count);
    // Scratch layout: [hi, lo (2·M rows of Kp FP16) | row scales]; the partial tiles have their own buffer.
    const size_t a_bytes = ((size_t)2 * M * Kp * sizeof(__half) + 255) / 256 * 256, s_bytes = 256;
    void *scr = nullptr;
    G9_TRY(scratch(a_bytes + s_bytes, &scr));
    uint64_t *part = nullptr;
    if (!q.aligned) G9_TRY(skinny_slots(q.part_words, &part, &p.epoch));
    p.err = d->err_dev;
    p.aligned = q.aligned;
    __half *hi = (__half *)scr;
    float *ts = (float *)((char *)scr + a_bytes);
    p.a = hi;
    p.tscale = ts;
    const bool vec4 = ((uintptr_t)A & 15) == 0 && lda % 4 == 0;
    if (paired) launch_pdl(split_f32_rows, dim3(M), dim3(SPLIT_THREADS), 0, st, A, (long long)lda, K, Kp, vec4, hi, hi + Kp,
                           2LL * Kp, ts);
    else launch_pdl(split_f32_rows, dim3(M), dim3(SPLIT_THREADS), 0, st, A, (long long)lda, K, Kp, vec4, hi,
                    hi + (size_t)M * Kp, (long long)Kp, ts);
    G9_TRY(launched("skinny_split_f32"));
    if ((N + 15) / 16 >= d->sm_count && q.KC >= WK_WARPS) {   // one row block per CTA, as the FP16-activation path
        const bool fullk = Kp % 256 == 0;
        auto kern = !paired ? (fullk ? wk_f16_blk<true, true, ACT_SPLIT> : wk_f16_blk<false, true, ACT_SPLIT>)
                  : p.Mc > 8 ? (fullk ? wk_f16_blk<true, true, ACT_PAIRED> : wk_f16_blk<false, true, ACT_PAIRED>)
                             : (fullk ? wk_f16_blk<true, false, ACT_PAIRED> : wk_f16_blk<false, false, ACT_PAIRED>);
        static bool attr_b[6][kMaxDevices] = {};
        G9_CU(smem_limit_once(kern, SK_SMEM_BYTES, attr_b[(!paired ? 0 : p.Mc > 8 ? 2 : 4) + (fullk ? 1 : 0)]));
        launch_pdl(kern, dim3((unsigned)((N + 15) / 16)), dim3(WK_WARPS * 32), SK_SMEM_BYTES, st, p, q.KC);
        return launched("skinny_wk_f16_blk_f32a");
    }
    if (!paired) return launch_f32a_main<true, 8, ACT_SPLIT>(p, q, part, st);
    if (p.Mc > 8) return launch_f32a_main<true, 8, ACT_PAIRED, true>(p, q, part, st);
    return launch_f32a_main<false, 8, ACT_PAIRED>(p, q, part, st);
}

bool skinny_f16w_fits(int M, int K, int N, long long ldw, const void *W) {
    DevState *d = dev_state();
    return d && M >= 1 && M <= 16 && (N + 15) / 16 >= d->sm_count && (K + 255) / 256 >= WK_WARPS && K % 8 == 0 &&
           ((uintptr_t)W & 15) == 0 && (ldw * 2) % 16 == 0;
}

int launch_skinny_f16w(int M, const void *A, bool ahalf, long long lda, const void *W, int K, int N, long long ldw,
                       float *C, long long ldc, const float *bias, int gelu, const float *R, long long ldr, unsigned *nf,
                       cudaStream_t st) {
    DevState *d = dev_state();
    if (!d) return G.status;
    const int es = ahalf ? 2 : 4;
    const int KC = (K + 255) / 256;
    if (!skinny_f16w_fits(M, K, N, ldw, W) || ((uintptr_t)A & 15) != 0 || (lda * es) % 16 != 0) return 1;
    SkinnyArgs p;
    memset(&p, 0, sizeof(p));
    p.Mc = M; p.Nc = N; p.K = K;
    p.alpha = 1.0f; p.beta = 0.0f;
    p.a = A; p.sam = lda; p.sak = 1;
    p.w = W; p.swn = ldw; p.swk = 1;
    p.C = C; p.scm = ldc; p.scn = 1;
    p.dst[0] = C; p.ndst = 1;
    p.nf = nf;
    p.bias = bias; p.gelu = gelu; p.R = R; p.ldr = ldr;
    p.early_w = !queued_writes_overlap(d, W, ((size_t)(N - 1) * ldw + K) * sizeof(__half));
    const bool fullk = K % 256 == 0, two = M > 8;
    using Kern = void (*)(const SkinnyArgs, int);
    Kern kern;
    if (ahalf) kern = fullk ? (two ? wk_f16_blk<true, true, ACT_F16, true> : wk_f16_blk<true, false, ACT_F16, true>)
                            : (two ? wk_f16_blk<false, true, ACT_F16, true> : wk_f16_blk<false, false, ACT_F16, true>);
    else kern = fullk ? (two ? wk_f16_blk<true, true, ACT_F32H, true> : wk_f16_blk<true, false, ACT_F32H, true>)
                      : (two ? wk_f16_blk<false, true, ACT_F32H, true> : wk_f16_blk<false, false, ACT_F32H, true>);
    static bool attr[8][kMaxDevices] = {};
    G9_CU(smem_limit_once(kern, SK_SMEM_BYTES, attr[(ahalf ? 4 : 0) + (fullk ? 2 : 0) + (two ? 1 : 0)]));
    launch_pdl(kern, dim3((unsigned)((N + 15) / 16)), dim3(WK_WARPS * 32), SK_SMEM_BYTES, st, p, KC);
    return launched("skinny_wk_f16_blk_f16w");
}

// ffn_f16w's gate and up GEMMs in one launch (M <= 16 tokens: F32 rounded to FP16 as loaded, or FP16 rows (xhalf);
// the one-block kernel's plan): g16 = fp16(X·Wgᵀ), u16 = fp16(X·Wuᵀ) (pitch N) and h16 = fp16(silu(g)·u) (pitch ldh, zero past N). Returns 1,
// launching nothing, where launch_skinny_f16w would decline the shape or layout.
int launch_skinny_swiglu(int M, const void *X, bool xhalf, long long ldx, const void *Wg, const void *Wu, int K, int N,
                         long long ldw, __half *g16, __half *u16, __half *h16, long long ldh, unsigned *nf,
                         cudaStream_t st) {
    DevState *d = dev_state();
    if (!d) return G.status;
    const int KC = (K + 255) / 256, RB = (N + 15) / 16;
    if (M < 1 || M > 16 || RB < d->sm_count || KC < WK_WARPS || K % 8 != 0 || ((uintptr_t)X & 15) != 0 ||
        (ldx * (xhalf ? 2 : 4)) % 16 != 0 || ((uintptr_t)Wg & 15) != 0 || ((uintptr_t)Wu & 15) != 0 ||
        (ldw * 2) % 16 != 0 || ldh < N)
        return 1;
    SkinnyArgs p;
    memset(&p, 0, sizeof(p));
    p.Mc = M; p.Nc = N; p.K = K;
    p.alpha = 1.0f; p.beta = 0.0f;
    p.a = X; p.sam = ldx; p.sak = 1;
    p.w = Wg; p.w2 = Wu; p.swn = ldw; p.swk = 1;
    p.C = g16; p.c2 = u16; p.scm = N; p.scn = 1;
    p.dst[0] = g16; p.ndst = 1;
    p.hsw = h16; p.ldh = ldh;
    p.nf = nf;
    G9_TRY(arrival_counters((size_t)RB, &p.cnt));
    const size_t wext = ((size_t)(N - 1) * ldw + K) * sizeof(__half);
    p.early_w = !queued_writes_overlap(d, Wg, wext) && !queued_writes_overlap(d, Wu, wext);
    const bool fullk = K % 256 == 0, two = M > 8;
    using Kern = void (*)(const SkinnyArgs, int);
    Kern kern;
    if (xhalf) kern = fullk ? (two ? wk_f16_blk<true, true, ACT_F16, false, true> : wk_f16_blk<true, false, ACT_F16, false, true>)
                            : (two ? wk_f16_blk<false, true, ACT_F16, false, true> : wk_f16_blk<false, false, ACT_F16, false, true>);
    else kern = fullk ? (two ? wk_f16_blk<true, true, ACT_F32H, false, true> : wk_f16_blk<true, false, ACT_F32H, false, true>)
                      : (two ? wk_f16_blk<false, true, ACT_F32H, false, true> : wk_f16_blk<false, false, ACT_F32H, false, true>);
    static bool attr[8][kMaxDevices] = {};
    G9_CU(smem_limit_once(kern, SK_SMEM_BYTES, attr[(xhalf ? 4 : 0) + (fullk ? 2 : 0) + (two ? 1 : 0)]));
    launch_pdl(kern, dim3((unsigned)(2 * RB)), dim3(WK_WARPS * 32), SK_SMEM_BYTES, st, p, KC);
    return launched("skinny_wk_f16_blk_swiglu");
}

int launch_skinny(int type, int tA, int tB, int M, int N, int K, double alpha, const void *A, int lda, const void *B,
                  int ldb, double beta, void *C, int ldc, cudaStream_t st, void *const *peers, int npeers,
                  long long col_off) {
    SkinnyArgs p;
    p.K = K;
    p.alpha = (float)alpha;
    p.beta = (float)beta;
    p.C = C;
    p.ndst = 1;
    p.dst[0] = C;
    p.coff = 0;
    p.alo = 0;
    p.tscale = nullptr;
    p.nf = nullptr;
    p.early_w = 0;
    p.epoch = 0;
    p.err = nullptr;
    p.aligned = 0;
    p.bias = nullptr; p.R = nullptr; p.ldr = 0; p.gelu = 0;
    if (peers && npeers > 0) {
        if (npeers > 8) return fail(GEN9BLAS_ERR_INVALID_ARG, "at most 8 ranks for the fused skinny GEMM + all-gather");
        for (int q = 0; q < npeers; q++) p.dst[q] = peers[q];
        p.ndst = npeers;
        p.C = peers[0];
        p.coff = col_off;   // C is row-major with pitch ldc: a column offset is an element offset
    }
    // Role choice of the reference (gemm.c:213-221): the smaller of M and N is the token side.
    if (M <= N) {
        p.Mc = M; p.Nc = N; p.a = A; p.w = B; p.scm = ldc; p.scn = 1;
        p.sam = tA ? 1 : lda; p.sak = tA ? lda : 1;   // op(A)[m][k]
        p.swn = tB ? ldb : 1; p.swk = tB ? 1 : ldb;   // op(B)[k][n]
    } else {
        p.Mc = N; p.Nc = M; p.a = B; p.w = A; p.scm = 1; p.scn = ldc;
        p.sam = tB ? ldb : 1; p.sak = tB ? 1 : ldb;   // op(B)ᵀ[n][k]
        p.swn = tA ? 1 : lda; p.swk = tA ? lda : 1;   // op(A)ᵀ[k][m]
    }
    if (p.swk != 1 && p.swn != 1) return fail(GEN9BLAS_ERR_INVALID_ARG, "skinny GEMM: weights have no contiguous dimension");
    if (type == GEN9BLAS_S) return skinny_t<float>(p, st);
    return skinny_t<__half>(p, st);
}

}  // namespace g9
