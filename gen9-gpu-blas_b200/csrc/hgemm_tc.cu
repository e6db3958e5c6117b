// hgemm_tc.cu -- FP16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
// Computes C = alpha·op(A)·op(B) + beta·C for GEN9BLAS_H (FP16 accumulator in TMEM: the tensor core rounds the
// running sum to FP16 after every K=16 step, the B200 counterpart of the reference's FP16-accumulate hgemm_v,
// lib/kernels/hgemm.cl:838-868) and GEN9BLAS_HS (FP32 accumulator for the whole K, strictly more accurate than the
// reference's FP16 chunks of 32 summed into FP32, hgemm.cl:869-898). The epilogue applies alpha/beta in FP32 and
// rounds once to FP16 (the reference rounds to FP16 first and runs gen9blas_epilog_b, hgemm.cl:557-564).
//
// There is no packing step: TMA reads op(A) and op(B) straight from the row-major operands. A transposed operand
// is an MN-major UMMA operand (transpose bit of the instruction descriptor), so all four transA/transB combinations
// run the same kernel. Operands whose strides break the TMA rules (16-byte aligned base and row pitch) are first
// copied into an aligned scratch layout by a small repack kernel.
//
// Kernel structure (persistent, one CTA per SM, 192 threads):
//   warp 0      TMA producer: 4-stage ring of (A 128×64, B 256×64) FP16 tiles, 128-byte swizzle, mbarrier tx counts;
//   warp 1      MMA issuer: one thread issues tcgen05.mma 128×256×16 into one of two TMEM accumulators
//               (2 × 256 columns), tcgen05.commit frees smem stages and hands finished accumulators to the epilogue;
//   warps 2-5   epilogue: tcgen05.ld 32 lanes × 32 columns, alpha/beta, FP16 stores, then release the accumulator.
// Tiles are visited in groups of 16 M-tiles so that the CTAs working at the same time share A and B in L2.
// Every mbarrier wait is bounded (4 s of global time); a wait that gives up sets the mapped error word and all
// roles leave their loops, drain their in-flight copies / MMAs (bounded) and free TMEM.
#include "common.cuh"
#include "internal.h"
#include "sm100.cuh"
#include <cudaTypedefs.h>
#include <cstdlib>

namespace g9 {
using namespace sm100;

constexpr int TC_BM = 128, TC_BN = 256, TC_BK = 64, TC_STAGES = 4;
constexpr int TC_A_BYTES = TC_BM * TC_BK * 2;   // 16 KiB
constexpr int TC_B_BYTES = TC_BN * TC_BK * 2;   // 32 KiB
constexpr int TC_STAGE_BYTES = TC_A_BYTES + TC_B_BYTES;
constexpr int TC_THREADS = 192;
constexpr int TC_GROUP_M = 16;
constexpr uint32_t TC_TMEM_COLS = 512;           // two 128×256 FP32 accumulators
constexpr int TC_SMEM = TC_STAGES * TC_STAGE_BYTES + 1024 /*alignment*/ + 256 /*barriers*/;
constexpr uint64_t TC_WAIT_NS = 4000000000ull;

struct TcParams {
    int M, N, K, count;
    int tiles_m, tiles_n, total_tiles;
    int a_mn, b_mn;           // 1: operand is MN-major in memory (transposed)
    float alpha, beta;
    int plain;                // alpha == 1 && beta == 0
    __half *C;
    long long ldc, sC;
    int c_vec;                // C base 16-byte aligned and ldc % 8 == 0
    unsigned *err;
    // split-K tail of the pair kernel: tiles [dp_tiles, total_tiles) are split into `split` K ranges; part 0 adds
    // the FP32 partial sums that parts 1..split-1 leave in `partial`, after their flags carry `epoch`.
    int dp_tiles, split, units;
    float *partial;
    unsigned *flags;
    unsigned epoch;
    // destinations of the pair kernel's epilogue: the tile is written to every dst[q] (row-major, pitch ldc) at column
    // col_off + n. One destination (C itself) for an ordinary GEMM; every rank's C for the fused GEMM + all-gather.
    __half *dst[8];
    int ndst;
    long long col_off;
    // pair kernel, alpha = 1, beta = 0, one destination with a TMA-legal C: the epilogue stages each warp's 32 × 32
    // FP16 block in shared memory (64-byte swizzle) and writes it with one TMA store (tmC)
    int tma_c;
    // with tma_c: the kernel computes Cᵀ (the host swapped the operands), so each staged block is written transposed
    // and stored at the swapped coordinates
    int c_t;
    // 1-CTA kernel, split K (FP32 accumulation, one matrix): unit u = (tile u / ks, K part u % ks), part q taking K
    // blocks [nk·q/ks, nk·(q+1)/ks) and storing its FP32 tile into kpart + q·M·N (dense M × N); hgemm_ksum adds the
    // parts in order and applies alpha / beta. ks = 1: whole tiles straight into C.
    int ks;
    float *kpart;
};

__device__ __forceinline__ void tile_coords(const TcParams &p, int tile, int &b, int &mb, int &nb) {
    const int per_batch = p.tiles_m * p.tiles_n;
    b = tile / per_batch;
    const int r = tile - b * per_batch;
    const int group_span = TC_GROUP_M * p.tiles_n;
    const int group = r / group_span;
    const int first_m = group * TC_GROUP_M;
    const int gsz = min(p.tiles_m - first_m, TC_GROUP_M);
    const int in_group = r - group * group_span;
    mb = first_m + in_group % gsz;
    nb = in_group / gsz;
}

__device__ __forceinline__ void report_timeout(const TcParams &p, volatile int *abort) {
    *abort = 1;
    *(volatile unsigned *)p.err = kDevErrWaitTimeout;
    __threadfence_system();
}

// Accumulator chunk (32 columns of one row, as loaded from TMEM) widened to FP32.
template <bool F16ACC> __device__ __forceinline__ void acc_to_f32(const uint32_t *r, float *v) {
    if (F16ACC) {
#pragma unroll
        for (int j = 0; j < 16; j++) {
            float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&r[j]));
            v[2 * j] = f.x;
            v[2 * j + 1] = f.y;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; j++) v[j] = __uint_as_float(r[j]);
    }
}

// Stores 32 columns of one row: alpha·v + beta·C, rounded once to FP16 (beta = 0: C is not read).
__device__ __forceinline__ void store_vals(const TcParams &p, const float *v, __half *crow, int col0) {
    __half *c = crow + col0;
    if (col0 + 32 <= p.N && p.c_vec) {
        uint4 *c4 = reinterpret_cast<uint4 *>(c);
#pragma unroll
        for (int q = 0; q < 4; q++) {
            float o[8];
            if (p.beta != 0.0f) {
                uint4 old = c4[q];
                const __half2 *oh = reinterpret_cast<const __half2 *>(&old);
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    float2 f = __half22float2(oh[e]);
                    o[2 * e] = __fmaf_rn(p.beta, f.x, p.alpha * v[8 * q + 2 * e]);
                    o[2 * e + 1] = __fmaf_rn(p.beta, f.y, p.alpha * v[8 * q + 2 * e + 1]);
                }
            } else {
#pragma unroll
                for (int e = 0; e < 8; e++) o[e] = p.alpha * v[8 * q + e];
            }
            uint4 u;
            __half2 *uh = reinterpret_cast<__half2 *>(&u);
#pragma unroll
            for (int e = 0; e < 4; e++) uh[e] = __floats2half2_rn(o[2 * e], o[2 * e + 1]);
            c4[q] = u;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; j++) {
            if (col0 + j < p.N) {
                float o = p.alpha * v[j];
                if (p.beta != 0.0f) o = __fmaf_rn(p.beta, __half2float(c[j]), o);
                c[j] = __float2half_rn(o);
            }
        }
    }
}

// Epilogue of one 32-column chunk of one row straight from the TMEM registers. FP16 accumulators with alpha = 1,
// beta = 0 are stored as they are (no widening).
template <bool F16ACC>
__device__ __forceinline__ void store_chunk(const TcParams &p, const uint32_t *r, __half *crow, int col0, bool row_ok) {
    if (!row_ok) return;
    if (F16ACC && p.plain && col0 + 32 <= p.N && p.c_vec) {
        uint4 *c4 = reinterpret_cast<uint4 *>(crow + col0);
#pragma unroll
        for (int q = 0; q < 4; q++) c4[q] = make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
        return;
    }
    float v[32];
    acc_to_f32<F16ACC>(r, v);
    store_vals(p, v, crow, col0);
}

template <bool F16ACC>
__global__ void __launch_bounds__(TC_THREADS, 1)
    hgemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + (((raw + 1023) & ~1023u) - raw);
    uint8_t *sA = smem;
    uint8_t *sB = smem + TC_STAGES * TC_A_BYTES;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + TC_STAGES * TC_STAGE_BYTES);
    uint64_t *full = bars;                     // [STAGES] TMA -> MMA
    uint64_t *empty = bars + TC_STAGES;        // [STAGES] MMA -> TMA
    uint64_t *tfull = bars + 2 * TC_STAGES;    // [2] MMA -> epilogue
    uint64_t *tempty = bars + 2 * TC_STAGES + 2;   // [2] epilogue -> MMA
    uint64_t *drain = bars + 2 * TC_STAGES + 4;    // MMA teardown
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * TC_STAGES + 5);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < TC_STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 128);
        }
        mbar_init(drain, 1);
        *abort = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, TC_TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int nk = (p.K + TC_BK - 1) / TC_BK;

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer
        int stage = 0;
        uint32_t phase = 0;
        long long issued = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < p.total_tiles * p.ks && ok; u += gridDim.x) {
            const int tile = u / p.ks, part = u - tile * p.ks;
            int b, mb, nb;
            tile_coords(p, tile, b, mb, nb);
            const int m0 = mb * TC_BM, n0 = nb * TC_BN;
            const int kb0 = nk * part / p.ks, kb1 = nk * (part + 1) / p.ks;
            for (int kb = kb0; kb < kb1; kb++) {
                if (!mbar_wait(&empty[stage], phase ^ 1, abort, TC_WAIT_NS)) { ok = false; break; }
                mbar_arrive_expect_tx(&full[stage], TC_STAGE_BYTES);
                uint8_t *a = sA + stage * TC_A_BYTES;
                uint8_t *bb = sB + stage * TC_B_BYTES;
                const int k0 = kb * TC_BK;
                if (!p.a_mn) {
                    tma_load_3d(a, &tmA, &full[stage], k0, m0, b);
                } else {
                    tma_load_3d(a, &tmA, &full[stage], m0, k0, b);
                    tma_load_3d(a + 8192, &tmA, &full[stage], m0 + 64, k0, b);
                }
                if (!p.b_mn) {
                    tma_load_3d(bb, &tmB, &full[stage], k0, n0, b);
                } else {
#pragma unroll
                    for (int j = 0; j < 4; j++) tma_load_3d(bb + 8192 * j, &tmB, &full[stage], n0 + 64 * j, k0, b);
                }
                issued++;
                if (++stage == TC_STAGES) { stage = 0; phase ^= 1; }
            }
        }
        if (!ok) {
            report_timeout(p, abort);
            // Let the copies already issued land before the CTA exits (bounded).
            const int outstanding = (int)(issued < TC_STAGES ? issued : TC_STAGES);
            for (int i = 1; i <= outstanding; i++) {
                int s = stage - i;
                uint32_t ph = phase;
                if (s < 0) { s += TC_STAGES; ph ^= 1; }
                volatile int no_abort = 0;
                mbar_wait(&full[s], ph, &no_abort, 100000000ull);
            }
        }
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer
        const uint32_t idesc = idesc_f16(F16ACC ? 0 : 1, p.a_mn, p.b_mn, TC_BM, TC_BN);
        int stage = 0;
        uint32_t phase = 0;
        int local = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < p.total_tiles * p.ks && ok; u += gridDim.x, local++) {
            const int part = u % p.ks;
            const int kb0 = nk * part / p.ks, kb1 = nk * (part + 1) / p.ks;
            const int buf = local & 1;
            const uint32_t acc_phase = (local >> 1) & 1;
            if (!mbar_wait(&tempty[buf], acc_phase ^ 1, abort, TC_WAIT_NS)) { ok = false; break; }
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + buf * TC_BN;
            for (int kb = kb0; kb < kb1; kb++) {
                if (!mbar_wait(&full[stage], phase, abort, TC_WAIT_NS)) { ok = false; break; }
                tc_fence_after();
                const uint32_t a_base = smem_u32(sA + stage * TC_A_BYTES);
                const uint32_t b_base = smem_u32(sB + stage * TC_B_BYTES);
#pragma unroll
                for (int k = 0; k < TC_BK / 16; k++) {
                    // K-major: the 16-element K slice is 32 bytes into each 128-byte swizzled row.
                    // MN-major: the slice is 16 K-rows of 128 bytes; MN atoms of 64 elements are 8 KiB apart.
                    const uint64_t ad = p.a_mn ? smem_desc_sw128(a_base + k * 2048, 8192, 1024)
                                               : smem_desc_sw128(a_base + k * 32, 16, 1024);
                    const uint64_t bd = p.b_mn ? smem_desc_sw128(b_base + k * 2048, 8192, 1024)
                                               : smem_desc_sw128(b_base + k * 32, 16, 1024);
                    umma_f16(d_tmem, ad, bd, idesc, kb != kb0 || k != 0);
                }
                umma_commit(&empty[stage]);
                if (++stage == TC_STAGES) { stage = 0; phase ^= 1; }
            }
            if (!ok) break;
            umma_commit(&tfull[buf]);
        }
        if (!ok) report_timeout(p, abort);
        // Wait (bounded) until every MMA issued by this thread has finished before TMEM is freed.
        umma_commit(drain);
        volatile int no_abort = 0;
        mbar_wait(drain, 0, &no_abort, 100000000ull);
    } else if (warp >= 2) {
        // ---------------- epilogue: 128 threads, thread = one accumulator row (TMEM lane)
        const int q = warp & 3;                 // TMEM lane quarter this warp may access
        const int row_in_tile = q * 32 + lane;
        int local = 0;
        for (int u = blockIdx.x; u < p.total_tiles * p.ks; u += gridDim.x, local++) {
            const int tile = u / p.ks, part = u - tile * p.ks;
            int b, mb, nb;
            tile_coords(p, tile, b, mb, nb);
            const int buf = local & 1;
            const uint32_t acc_phase = (local >> 1) & 1;
            if (!mbar_wait(&tfull[buf], acc_phase, abort, TC_WAIT_NS)) {
                report_timeout(p, abort);
                break;
            }
            tc_fence_after();
            const int row = mb * TC_BM + row_in_tile;
            const bool row_ok = row < p.M;
            __half *crow = p.C + (long long)b * p.sC + (long long)(row_ok ? row : 0) * p.ldc;
            float *prow = p.ks > 1 ? p.kpart + ((long long)part * p.M + (row_ok ? row : 0)) * p.N : nullptr;
            const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + buf * TC_BN;
#pragma unroll 1
            for (int c = 0; c < TC_BN / 32; c++) {
                const int col0 = nb * TC_BN + c * 32;
                uint32_t r[32];
                if (F16ACC) tmem_ld_32x32_pack16(t_row + c * 32, r);
                else tmem_ld_32x32(t_row + c * 32, r);
                tmem_ld_wait();
                if (col0 >= p.N) continue;
                if (!F16ACC && prow) {   // split K: the FP32 part (fixed indices keep r in registers)
                    if (row_ok) {
                        if (col0 + 32 <= p.N && (p.N & 3) == 0) {
                            float4 *d4 = reinterpret_cast<float4 *>(prow + col0);
#pragma unroll
                            for (int j = 0; j < 8; j++)
                                d4[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                                    __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
                        } else {
#pragma unroll
                            for (int j = 0; j < 32; j++)
                                if (col0 + j < p.N) prow[col0 + j] = __uint_as_float(r[j]);
                        }
                    }
                } else {
                    store_chunk<F16ACC>(p, r, crow, col0, row_ok);
                }
            }
            tc_fence_before();
            mbar_arrive(&tempty[buf]);
        }
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TC_TMEM_COLS);
    }
}

// C = alpha·Σ_q part[q] + beta·C over the ks K parts of the 1-CTA kernel (in part order), rounded to FP16 as store_vals
// rounds: element i of the dense M × N parts is C[i / N][i % N].
__global__ void hgemm_ksum(const float *__restrict__ part, int ks, int M, int N, float alpha, float beta, __half *C,
                           long long ldc) {
    const long long mn = (long long)M * N;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < mn; i += (long long)gridDim.x * blockDim.x) {
        float s = part[i];
        for (int q = 1; q < ks; q++) s += part[q * mn + i];
        __half *c = C + (i / N) * ldc + i % N;
        const float o = beta != 0.0f ? __fmaf_rn(beta, __half2float(*c), alpha * s) : alpha * s;
        *c = __float2half_rn(o);
    }
}

// ------------------------------------------------------------------------------------------------ CTA-pair kernel
// Same roles and bounded waits as hgemm_tc_kernel, on a cluster of 2 CTAs that computes 256×256 tiles with
// tcgen05.mma.cta_group::2 (M = 256 across the pair's TMEM, N = 256). Each CTA stages only its half of the operands
// per K-block (A: its 128 rows, B: its 128 of the 256 columns), 32 KiB per 64 K instead of 48 KiB for a 128×256
// tile: half the shared-memory fill traffic per FLOP. Protocol of the pair:
// - full[s] of the leader (rank 0) counts the TMA bytes of both CTAs (cta_group::2 loads name the leader's
//   barrier); the leader's producer arms it with the pair's byte count;
// - the leader's MMA thread releases a stage in both CTAs with one multicast commit to empty[s], and hands a
//   finished accumulator to both epilogues with a multicast commit to tfull[b];
// - every epilogue warp of both CTAs arrives (cluster scope) on the leader's tempty[b];
// - a cluster barrier after the barrier setup and before TMEM is freed keeps both CTAs alive while the pair's MMAs
//   read their shared memory. No TMA multicast is used.
constexpr int T2_BM = 256;
// The pair kernel's ring stages hold 128 K (two 64-wide TMA boxes per operand, 64 KiB per stage with BN 256), so each
// barrier handshake (full-barrier wait, fence, commit, stage advance) feeds 8 MMAs instead of 4. Measured on B200 at
// full clock against 6 stages of 64 K in the same 192 KiB: n = 4096 1259 -> 1289-1305 TF/s, n = 8192 1384 -> 1441-1451,
// n = 1024 206 -> 232.
constexpr int T2_BK = 128;
constexpr int T2_A_BYTES = 128 * T2_BK * 2;   // this CTA's 128 rows of A, 32 KiB

// Tile width BN (256 or 128) sets the shared-memory ring and the number of TMEM accumulators (512 / BN columns).
template <int BN> struct PairCfg {
    static constexpr int B_BYTES = (BN / 2) * T2_BK * 2;          // this CTA's BN/2 columns of B
    static constexpr int B_BOX = (BN / 2) * TC_BK * 2;             // one 64-K box of the K-major B
    static constexpr int STAGE_BYTES = T2_A_BYTES + B_BYTES;
    static constexpr int STAGES = (192 * 1024) / STAGE_BYTES;   // 3 (BN 256) or 4 (BN 128)
    static constexpr int NBUF = 512 / BN;                       // TMEM accumulators
    static constexpr int STAGING = 4 * 2 * 2048;                // epilogue: 4 warps × 2 buffers of 32 × 32 FP16
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 1024 + STAGING;
};

__device__ __forceinline__ void tile_coords_pair(const TcParams &p, int tile, int &b, int &mb, int &nb) {
    const int per_batch = p.tiles_m * p.tiles_n;
    b = tile / per_batch;
    const int r = tile - b * per_batch;
    const int group_span = TC_GROUP_M * p.tiles_n;
    const int group = r / group_span;
    const int first_m = group * TC_GROUP_M;
    const int gsz = min(p.tiles_m - first_m, TC_GROUP_M);
    const int in_group = r - group * group_span;
    mb = first_m + in_group % gsz;
    nb = in_group / gsz;
}

// One unit of work of a CTA pair: a whole tile (part -1) or one K range of a split tail tile (part 0 finishes the
// tile, parts 1.. leave FP32 partial sums for it).
struct PairUnit {
    int tile, kb0, kb1, part;
};
__device__ __forceinline__ PairUnit pair_unit(const TcParams &p, int u, int nk) {
    PairUnit w;
    if (u < p.dp_tiles) {
        w.tile = u; w.kb0 = 0; w.kb1 = nk; w.part = -1;
    } else {
        const int v = u - p.dp_tiles;
        w.tile = p.dp_tiles + v / p.split;
        w.part = v % p.split;
        w.kb0 = (int)((long long)nk * w.part / p.split);
        w.kb1 = (int)((long long)nk * (w.part + 1) / p.split);
    }
    return w;
}
__device__ __forceinline__ int partial_slot(const TcParams &p, int tile, int part, uint32_t rank) {
    return ((tile - p.dp_tiles) * (p.split - 1) + (part - 1)) * 2 + (int)rank;
}
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned *a) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_gpu(unsigned *a, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(a), "r"(v) : "memory");
}
__device__ __forceinline__ void epilogue_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

template <bool F16ACC, int BN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(TC_THREADS, 1)
    hgemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const TcParams p) {
    using Cfg = PairCfg<BN>;
    constexpr int STAGES = Cfg::STAGES, NBUF = Cfg::NBUF;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + (((raw + 1023) & ~1023u) - raw);
    uint8_t *sA = smem;
    uint8_t *sB = smem + STAGES * T2_A_BYTES;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGES * Cfg::STAGE_BYTES);
    uint64_t *full = bars;
    uint64_t *empty = bars + STAGES;
    uint64_t *tfull = bars + 2 * STAGES;
    uint64_t *tempty = bars + 2 * STAGES + NBUF;
    uint64_t *drain = bars + 2 * STAGES + 2 * NBUF;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
    uint8_t *staging = smem + STAGES * Cfg::STAGE_BYTES + 1024;   // 1024-byte aligned (64-byte swizzle atoms)

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
    // The next GEMM of the stream (a programmatic dependent launch) may start as soon as this one runs; it takes SM
    // slots as these CTAs retire and sets up its barriers and TMEM meanwhile.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < NBUF; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 8);   // 4 epilogue warps in each CTA of the pair
        }
        mbar_init(drain, 1);
        *abort = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        if (p.tma_c) tma_prefetch_desc(&tmC);
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, TC_TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();   // both CTAs' barriers are initialised before any cross-CTA arrive
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int nk = (p.K + T2_BK - 1) / T2_BK;
    // A, B, C, the split-K scratch and flags may belong to the preceding kernel: wait for it before any access.
    asm volatile("griddepcontrol.wait;" ::: "memory");

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer (both CTAs): this CTA's halves, bytes counted on the leader's full[s]
        int stage = 0;
        uint32_t phase = 0;
        long long issued = 0;
        bool ok = true;
        for (int u = cluster; u < p.units && ok; u += nclusters) {
            const PairUnit w = pair_unit(p, u, nk);
            int b, mb, nb;
            tile_coords_pair(p, w.tile, b, mb, nb);
            const int m0 = mb * T2_BM + 128 * rank, n0 = nb * BN + (BN / 2) * rank;
            for (int kb = w.kb0; kb < w.kb1; kb++) {
                if (!mbar_wait_cluster(&empty[stage], phase ^ 1, abort, TC_WAIT_NS)) { ok = false; break; }
                if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::STAGE_BYTES);
                const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
                uint8_t *a = sA + stage * T2_A_BYTES;
                uint8_t *bb = sB + stage * Cfg::B_BYTES;
                const int k0 = kb * T2_BK;
                // K-major operands: the two 64-K boxes back to back. MN-major operands: per 64-wide M (N) block, its
                // 128 K rows contiguous (two boxes of 64 K), blocks 16 KiB apart.
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    if (!p.a_mn) {
                        tma_load_3d_pair(a + 16384 * h, &tmA, bar, k0 + 64 * h, m0, b);
                    } else {
                        tma_load_3d_pair(a + 8192 * h, &tmA, bar, m0, k0 + 64 * h, b);
                        tma_load_3d_pair(a + 16384 + 8192 * h, &tmA, bar, m0 + 64, k0 + 64 * h, b);
                    }
                    if (!p.b_mn) {
                        tma_load_3d_pair(bb + Cfg::B_BOX * h, &tmB, bar, k0 + 64 * h, n0, b);
                    } else {
#pragma unroll
                        for (int j = 0; j < BN / 128; j++)
                            tma_load_3d_pair(bb + 16384 * j + 8192 * h, &tmB, bar, n0 + 64 * j, k0 + 64 * h, b);
                    }
                }
                issued++;
                if (++stage == STAGES) { stage = 0; phase ^= 1; }
            }
        }
        if (!ok) {
            report_timeout(p, abort);
            // Wait (bounded) until the pair's MMAs released the stages this CTA filled, so no copy is in flight.
            const int outstanding = (int)(issued < STAGES ? issued : STAGES);
            for (int i = 1; i <= outstanding; i++) {
                int s = stage - i;
                uint32_t ph = phase;
                if (s < 0) { s += STAGES; ph ^= 1; }
                volatile int no_abort = 0;
                mbar_wait_cluster(&empty[s], ph, &no_abort, 100000000ull);
            }
        }
    } else if (warp == 1 && lane == 0 && rank == 0) {
        // ---------------- MMA issuer (leader CTA only)
        const uint32_t idesc = idesc_f16(F16ACC ? 0 : 1, p.a_mn, p.b_mn, T2_BM, BN);
        int stage = 0;
        uint32_t phase = 0;
        int local = 0;
        bool ok = true;
        for (int u = cluster; u < p.units && ok; u += nclusters, local++) {
            const PairUnit w = pair_unit(p, u, nk);
            const int buf = local % NBUF;
            const uint32_t acc_phase = (local / NBUF) & 1;
            if (!mbar_wait_cluster(&tempty[buf], acc_phase ^ 1, abort, TC_WAIT_NS)) { ok = false; break; }
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + buf * BN;
            for (int kb = w.kb0; kb < w.kb1; kb++) {
                if (!mbar_wait_cluster(&full[stage], phase, abort, TC_WAIT_NS)) { ok = false; break; }
                tc_fence_after();
                const uint32_t a_base = smem_u32(sA + stage * T2_A_BYTES);
                const uint32_t b_base = smem_u32(sB + stage * Cfg::B_BYTES);
                const int k_left = p.K - kb * T2_BK;   // >= 1; 16-K steps wholly past K hold TMA zero fill: skipped
#pragma unroll
                for (int k = 0; k < T2_BK / 16; k++) {
                    if (k * 16 >= k_left) break;
                    const uint32_t kin = (uint32_t)(k & 3) * 32, kbox = (uint32_t)(k >> 2);
                    const uint64_t ad = p.a_mn ? smem_desc_sw128(a_base + k * 2048, 16384, 1024)
                                               : smem_desc_sw128(a_base + kbox * 16384 + kin, 16, 1024);
                    const uint64_t bd = p.b_mn ? smem_desc_sw128(b_base + k * 2048, 16384, 1024)
                                               : smem_desc_sw128(b_base + kbox * Cfg::B_BOX + kin, 16, 1024);
                    umma_f16_pair(d_tmem, ad, bd, idesc, (kb > w.kb0 || k > 0) ? 1u : 0u);
                }
                umma_commit_pair_mc(&empty[stage], 0x3);
                if (++stage == STAGES) { stage = 0; phase ^= 1; }
            }
            if (!ok) break;
            umma_commit_pair_mc(&tfull[buf], 0x3);
        }
        if (!ok) report_timeout(p, abort);
        umma_commit_pair(drain);
        volatile int no_abort = 0;
        mbar_wait(drain, 0, &no_abort, 100000000ull);
    } else if (warp >= 2) {
        // ---------------- epilogue (both CTAs): this CTA's 128 rows of the 256×BN tile
        const int q = warp & 3;
        const int row_local = q * 32 + lane;
        const int row_in_tile = 128 * rank + row_local;
        int local = 0;
        for (int u = cluster; u < p.units; u += nclusters, local++) {
            const PairUnit w = pair_unit(p, u, nk);
            int b, mb, nb;
            tile_coords_pair(p, w.tile, b, mb, nb);
            const int buf = local % NBUF;
            const uint32_t acc_phase = (local / NBUF) & 1;
            if (!mbar_wait_cluster(&tfull[buf], acc_phase, abort, TC_WAIT_NS)) {
                report_timeout(p, abort);
                break;
            }
            tc_fence_after();
            const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + buf * BN;
            if (w.part > 0) {
                // contributor: FP32 partial sums of this K range to the slot of (tile, part, rank), then its flag
                float *dst = p.partial + (size_t)partial_slot(p, w.tile, w.part, rank) * (128 * BN) + (size_t)row_local * BN;
#pragma unroll 1
                for (int c = 0; c < BN / 32; c++) {
                    uint32_t r[32];
                    if (F16ACC) tmem_ld_32x32_pack16(t_row + c * 32, r);
                    else tmem_ld_32x32(t_row + c * 32, r);
                    tmem_ld_wait();
                    float v[32];
                    acc_to_f32<F16ACC>(r, v);
                    float4 *d4 = reinterpret_cast<float4 *>(dst + c * 32);
#pragma unroll
                    for (int j = 0; j < 8; j++) d4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                }
                __threadfence();   // each thread's partial stores, at GPU scope, before the flag
                epilogue_bar();
                if (threadIdx.x == 64) {
                    __threadfence();
                    st_release_gpu(p.flags + partial_slot(p, w.tile, w.part, rank), p.epoch);
                }
            } else {
                const int row = mb * T2_BM + row_in_tile;
                const bool row_ok = row < p.M;
                const long long roff = (long long)b * p.sC + (long long)(row_ok ? row : 0) * p.ldc + p.col_off;
                bool have = true;
                if (w.part == 0) {
                    // finisher: wait (bounded) until every other part of this tile has left its partial sums
                    for (int j = 1; j < p.split && have; j++) {
                        const unsigned *f = p.flags + partial_slot(p, w.tile, j, rank);
                        if (ld_acquire_gpu(f) != p.epoch) {
                            const uint64_t t0 = globaltimer();
                            while (ld_acquire_gpu(f) != p.epoch) {
                                if (*abort || globaltimer() - t0 > TC_WAIT_NS) { have = false; break; }
                            }
                        }
                    }
                    if (!have) report_timeout(p, abort);
                }
#pragma unroll 1
                for (int c = 0; c < BN / 32; c++) {
                    const int col0 = nb * BN + c * 32;
                    uint32_t r[32];
                    if (F16ACC) tmem_ld_32x32_pack16(t_row + c * 32, r);
                    else tmem_ld_32x32(t_row + c * 32, r);
                    tmem_ld_wait();
                    if (p.tma_c) {
                        // FP16 block of this warp (32 rows × 32 columns) into its staging buffer, then one TMA store;
                        // rows and columns past M and N are clipped by the store. A split tile's finisher first adds
                        // the other parts' FP32 partial sums. The buffer used two chunks ago must have been read by
                        // its store first. Staging rows are 64 bytes with the map's 64-byte swizzle: 16-byte chunk j
                        // of row r sits at chunk j ^ ((r >> 1) & 3), so a warp's row stores spread over all banks.
                        if (!have) continue;
                        uint32_t h[16];
                        if (w.part == 0) {
                            float v[32];
                            acc_to_f32<F16ACC>(r, v);
                            for (int j = 1; j < p.split; j++) {
                                const float4 *s4 = reinterpret_cast<const float4 *>(
                                    p.partial + (size_t)partial_slot(p, w.tile, j, rank) * (128 * BN) +
                                    (size_t)row_local * BN + c * 32);
#pragma unroll
                                for (int e = 0; e < 8; e++) {
                                    const float4 t = s4[e];
                                    v[4 * e] += t.x; v[4 * e + 1] += t.y; v[4 * e + 2] += t.z; v[4 * e + 3] += t.w;
                                }
                            }
#pragma unroll
                            for (int k = 0; k < 16; k++) {
                                const __half2 v2 = __floats2half2_rn(v[2 * k], v[2 * k + 1]);
                                h[k] = *reinterpret_cast<const uint32_t *>(&v2);
                            }
                        } else if (F16ACC) {
#pragma unroll
                            for (int k = 0; k < 16; k++) h[k] = r[k];
                        } else {
#pragma unroll
                            for (int k = 0; k < 16; k++) {
                                const __half2 v2 = __floats2half2_rn(__uint_as_float(r[2 * k]), __uint_as_float(r[2 * k + 1]));
                                h[k] = *reinterpret_cast<const uint32_t *>(&v2);
                            }
                        }
                        uint8_t *stg = staging + ((q * 2) + (c & 1)) * 2048;
                        if (lane == 0) bulk_wait_read<1>();
                        __syncwarp();
                        if (!p.c_t) {
#pragma unroll
                            for (int k = 0; k < 4; k++)
                                *reinterpret_cast<uint4 *>(stg + lane * 64 + ((k ^ ((lane >> 1) & 3)) << 4)) =
                                    make_uint4(h[4 * k], h[4 * k + 1], h[4 * k + 2], h[4 * k + 3]);
                        } else {
                            // this lane's row of the Cᵀ tile is column `lane` of the C block: element j goes to
                            // staging row j, byte 2·lane
#pragma unroll
                            for (int k = 0; k < 16; k++) {
#pragma unroll
                                for (int e = 0; e < 2; e++) {
                                    const int j = 2 * k + e;
                                    *reinterpret_cast<uint16_t *>(stg + j * 64 + ((((lane >> 3) ^ (j >> 1)) & 3) << 4) +
                                                                  (lane & 7) * 2) = (uint16_t)(h[k] >> (16 * e));
                                }
                            }
                        }
                        fence_proxy_async();
                        __syncwarp();
                        const int row_w = mb * T2_BM + 128 * rank + q * 32;
                        if (lane == 0 && row_w < p.M && col0 < p.N) {
                            if (p.c_t) tma_store_3d(&tmC, stg, row_w, col0, b);
                            else tma_store_3d(&tmC, stg, col0, row_w, b);
                            bulk_commit();
                        }
                        continue;
                    }
                    if (!have || col0 >= p.N || !row_ok) continue;
                    // destinations in an order rotated by CTA and chunk, so that at any moment the CTAs of all
                    // ranks write into different ranks' C rather than all into the same one
                    const int rot = (int)(blockIdx.x >> 1) + c;
                    if (w.part < 0) {
                        for (int qq = 0; qq < p.ndst; qq++) {
                            const int q = (qq + rot) % p.ndst;
                            store_chunk<F16ACC>(p, r, p.dst[q] + roff, col0, row_ok);
                        }
                    } else {
                        float v[32];
                        acc_to_f32<F16ACC>(r, v);
                        for (int j = 1; j < p.split; j++) {
                            const float4 *s4 = reinterpret_cast<const float4 *>(
                                p.partial + (size_t)partial_slot(p, w.tile, j, rank) * (128 * BN) + (size_t)row_local * BN +
                                c * 32);
#pragma unroll
                            for (int e = 0; e < 8; e++) {
                                const float4 t = s4[e];
                                v[4 * e] += t.x; v[4 * e + 1] += t.y; v[4 * e + 2] += t.z; v[4 * e + 3] += t.w;
                            }
                        }
                        for (int qq = 0; qq < p.ndst; qq++) store_vals(p, v, p.dst[(qq + rot) % p.ndst] + roff, col0);
                    }
                }
                if (p.ndst > 1) __threadfence_system();   // peer stores ordered before the ranks' next barrier
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[buf]), 0));
        }
        if (p.tma_c && lane == 0) bulk_wait<0>();   // this warp's C stores are complete before the CTA ends
    }
    __syncthreads();
    cluster_sync();   // the pair's MMAs (drained by the leader) no longer read either CTA's shared memory
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, TC_TMEM_COLS);
    }
}

template <bool F16ACC, int BN>
static int launch_pair(const CUtensorMap &mA, const CUtensorMap &mB, const CUtensorMap &mC, const TcParams &p, int grid,
                       cudaStream_t st) {
    static bool attr[kMaxDevices] = {};
    G9_CU(smem_limit_once(hgemm_tc2_kernel<F16ACC, BN>, PairCfg<BN>::SMEM, attr));
    if (p.ndst == 1) {   // programmatic dependent launch (the fused all-gather keeps plain stream order)
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(grid);
        cfg.blockDim = dim3(TC_THREADS);
        cfg.dynamicSmemBytes = PairCfg<BN>::SMEM;
        cfg.stream = st;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        cudaLaunchKernelEx(&cfg, hgemm_tc2_kernel<F16ACC, BN>, mA, mB, mC, p);
    } else {
        hgemm_tc2_kernel<F16ACC, BN><<<grid, TC_THREADS, PairCfg<BN>::SMEM, st>>>(mA, mB, mC, p);
    }
    return launched("hgemm_tc2");
}

// ------------------------------------------------------------------------------------------------ repack
// Copies a rows × cols FP16 matrix (row pitch ld, batch stride s) into a dense layout with a row pitch that is a
// multiple of 8 elements (16 bytes), so that TMA can read it. Used only when the caller's strides are not TMA-legal.
__global__ void repack_f16(const __half *__restrict__ src, long long ld, long long s, int rows, int cols, __half *dst,
                           long long dld, long long ds, int count) {
    const long long n = (long long)rows * cols;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n * count; i += (long long)gridDim.x * blockDim.x) {
        const long long b = i / n, r = (i % n) / cols, c = i % cols;
        dst[b * ds + r * dld + c] = src[b * s + r * ld + c];
    }
}

static int encode_map(CUtensorMap *m, const void *base, long long inner, long long outer, long long ld, long long count,
                      long long bstride, int box_inner, int box_outer) {
    auto enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(tensor_map_encoder());
    if (!enc) return fail(GEN9BLAS_ERR, "cuTensorMapEncodeTiled is not available from the driver");
    cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)outer, (cuuint64_t)count};
    cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)bstride * 2};
    cuuint32_t box[3] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(GEN9BLAS_ERR, "cuTensorMapEncodeTiled failed (%d): inner %lld outer %lld ld %lld count %lld", (int)r,
                    inner, outer, ld, count);
    return 0;
}

// C as a TMA store target: FP16, {N, M, count} with row pitch ldc and batch stride sC (elements), 32 × 32 boxes with
// the 64-byte swizzle that the epilogue's staging writes follow.
static int encode_c_map(CUtensorMap *m, void *base, long long N, long long M, long long ldc, long long count,
                        long long sC) {
    auto enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(tensor_map_encoder());
    if (!enc) return fail(GEN9BLAS_ERR, "cuTensorMapEncodeTiled is not available from the driver");
    cuuint64_t dims[3] = {(cuuint64_t)N, (cuuint64_t)M, (cuuint64_t)count};
    cuuint64_t strides[2] = {(cuuint64_t)ldc * 2, (cuuint64_t)sC * 2};
    cuuint32_t box[3] = {32, 32, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(GEN9BLAS_ERR, "cuTensorMapEncodeTiled (C) failed (%d): N %lld M %lld ldc %lld", (int)r, N, M, ldc);
    return 0;
}

static bool tma_ok(const void *p, long long ld, long long s, int count) {
    return ((uintptr_t)p & 15) == 0 && (ld * 2) % 16 == 0 && (count == 1 || (s * 2) % 16 == 0);
}

// GEN9BLAS_HGEMM_PAIR: 0 keeps the one-CTA kernel, 128 / 256 force the pair tile width (comparisons).
static int pair_setting() {
    static int pair_env = -1;
    if (pair_env < 0) {
        const char *e = getenv("GEN9BLAS_HGEMM_PAIR");
        pair_env = e ? atoi(e) : 1;
    }
    return pair_env;
}

// c_t: the operands arrive swapped (the call computes Cᵀ) and C (M × N here, pitch ldc) receives the transposed tiles;
// only with the pair kernel's TMA-store epilogue.
static int hgemm_tc_impl(int type, int tA, int tB, int M, int N, int K, double alpha, const void *A, int lda, long long sA,
                         const void *B, int ldb, long long sB, double beta, void *C, int ldc, long long sC, int count,
                         cudaStream_t st, void *const *peers, int npeers, long long col_off, int c_t) {
    DevState *d = dev_state();
    if (!d) return G.status;
    if (npeers > 8) return fail(GEN9BLAS_ERR_INVALID_ARG, "at most 8 ranks for the fused GEMM + all-gather");
    const int pair_env = pair_setting();
    const bool pair = (pair_env && M > 128) || npeers > 0;
    const int pairs = d->sm_count / 2;
    // Tile width: 256 feeds the tensor pipe best (L2 -> SMEM bytes per FLOP), but when 256×256 tiles would occupy at
    // most a quarter of the CTA pairs, 256×128 tiles spread the work twice as wide (measured on B200, n = 1024:
    // 150 TF/s with 256, 174 with 128; at n = 2048, 64 tiles: 838 with 256, 575 with 128).
    const long long tiles256 = (long long)((M + T2_BM - 1) / T2_BM) * ((N + 255) / 256) * count;
    const int bn = pair_env == 128 || (pair_env == 1 && tiles256 * 4 <= pairs) ? 128 : 256;
    const int nk = (K + T2_BK - 1) / T2_BK;   // K blocks of the pair kernel's stages
    // Work plan of the pair kernel: whole tiles while full waves of CTA pairs remain; when the last wave would leave
    // at least half of the pairs idle, its tiles are split along K over them (split-K tail, FP32 partials). A single
    // partial wave is not split: there the partial-sum exchange through global memory costs more than the idle pairs
    // (measured on B200: n = 1024, 16 tiles, 14.3 µs whole vs 33.7 µs split 4 ways).
    long long tiles = 0, dp = 0, units = 0;
    int split = 1;
    if (pair) {
        tiles = (long long)((M + T2_BM - 1) / T2_BM) * ((N + bn - 1) / bn) * count;
        const long long waves = tiles / pairs, tail = tiles % pairs;
        if (tail > 0 && waves >= 1 && 2 * tail <= pairs && nk >= 4) {
            split = (int)(pairs / tail);
            if (split > 4) split = 4;
            if (split > nk / 2) split = nk / 2;
        }
        dp = split > 1 ? tiles - tail : tiles;
        units = dp + (tiles - dp) * split;
    }
    const size_t partial_bytes = pair && split > 1 ? (size_t)(tiles - dp) * (split - 1) * 2 * 128 * bn * sizeof(float) : 0;
    // 1-CTA kernel (M <= 128) with at most half the SMs' worth of tiles: K split over them (FP32 accumulation, one
    // matrix, C only), ks parts per tile, each of at least 4 K blocks, summed in order by hgemm_ksum. Measured on
    // B200, gemm_pb_f16w M = 64 (HS): W 4096 x 4096 38.3 -> 28.6 us; W 11008 x 4096 unchanged at 46.6 us.
    int ks = 1;
    if (!pair && type == GEN9BLAS_HS && count == 1 && !(peers && npeers > 0) && !c_t) {
        const long long t1 = (long long)((M + TC_BM - 1) / TC_BM) * ((N + TC_BN - 1) / TC_BN);
        const int nkb = (K + TC_BK - 1) / TC_BK;
        if (2 * t1 <= d->sm_count && nkb >= 8) ks = (int)std::min<long long>(std::min<long long>(d->sm_count / t1, nkb / 4), 16);
    }
    const size_t kpart_bytes = ks > 1 ? ((size_t)ks * M * N * sizeof(float) + 255) / 256 * 256 : 0;

    // Stored shapes: A is rowsA × colsA with pitch lda (tA: K × M, else M × K); B is rowsB × colsB (tB: N × K, else K × N).
    const long long rowsA = tA ? K : M, colsA = tA ? M : K;
    const long long rowsB = tB ? N : K, colsB = tB ? K : N;
    const void *a = A, *b = B;
    long long la = lda, lb = ldb, xa = sA, xb = sB;
    const bool okA = tma_ok(A, lda, sA, count), okB = tma_ok(B, ldb, sB, count);
    const long long pa = (colsA + 7) / 8 * 8, pb = (colsB + 7) / 8 * 8;
    const long long bytesA = okA ? 0 : (rowsA * pa * count * 2 + 255) / 256 * 256;
    const long long bytesB = okB ? 0 : (rowsB * pb * count * 2 + 255) / 256 * 256;
    void *scr = nullptr;
    if (bytesA + bytesB + (long long)(partial_bytes + kpart_bytes) > 0)
        G9_TRY(scratch((size_t)(bytesA + bytesB) + partial_bytes + kpart_bytes, &scr));
    if (bytesA) {
        repack_f16<<<d->sm_count * 8, 256, 0, st>>>((const __half *)A, lda, sA, (int)rowsA, (int)colsA, (__half *)scr, pa,
                                                   rowsA * pa, count);
        G9_TRY(launched("repack_f16"));
        a = scr; la = pa; xa = rowsA * pa;
    }
    if (bytesB) {
        __half *dstB = (__half *)((char *)scr + bytesA);
        repack_f16<<<d->sm_count * 8, 256, 0, st>>>((const __half *)B, ldb, sB, (int)rowsB, (int)colsB, dstB, pb,
                                                   rowsB * pb, count);
        G9_TRY(launched("repack_f16"));
        b = dstB; lb = pb; xb = rowsB * pb;
    }
    if (count == 1) {   // a batch stride is still required by the 3-D map; any legal value works
        xa = (rowsA * la + 7) / 8 * 8;
        xb = (rowsB * lb + 7) / 8 * 8;
    }
    TcParams p;
    p.M = M; p.N = N; p.K = K; p.count = count;
    p.a_mn = tA ? 1 : 0;
    p.b_mn = tB ? 0 : 1;
    p.alpha = (float)alpha;
    p.beta = (float)beta;
    p.plain = alpha == 1.0 && beta == 0.0;
    p.C = (__half *)C;
    p.ldc = ldc;
    p.sC = sC;
    p.c_vec = ((uintptr_t)C & 15) == 0 && (ldc % 8) == 0 && (count == 1 || (sC % 8) == 0);
    p.err = d->err_dev;
    p.dp_tiles = p.split = p.units = 0;
    p.ks = ks;
    p.kpart = ks > 1 ? (float *)((char *)scr + bytesA + bytesB + partial_bytes) : nullptr;
    p.partial = nullptr;
    p.flags = nullptr;
    p.epoch = 0;
    p.dst[0] = (__half *)C;
    p.ndst = 1;
    p.col_off = 0;
    if (peers && npeers > 0) {   // fused GEMM + all-gather: write the tile into every rank's C
        for (int q = 0; q < npeers; q++) p.dst[q] = (__half *)peers[q];
        p.ndst = npeers;
        p.col_off = col_off;
        bool al = (col_off % 8) == 0;
        for (int q = 0; q < npeers; q++) al = al && ((uintptr_t)peers[q] & 15) == 0;
        p.c_vec = p.c_vec && al;
    }
    CUtensorMap mA, mB;
    // K-major operands: box 64 (K) × rows; MN-major operands: box 64 (M or N) × 64 (K).
    if (!tA) G9_TRY(encode_map(&mA, a, K, M, la, count, xa, TC_BK, pair ? 128 : TC_BM));
    else G9_TRY(encode_map(&mA, a, M, K, la, count, xa, 64, TC_BK));
    if (tB) G9_TRY(encode_map(&mB, b, K, N, lb, count, xb, TC_BK, pair ? bn / 2 : TC_BN));
    else G9_TRY(encode_map(&mB, b, N, K, lb, count, xb, 64, TC_BK));

    CUtensorMap mC = mB;   // unused unless p.tma_c
    p.tma_c = 0;
    p.c_t = c_t;
    if (pair && p.plain && !(peers && npeers > 0) && p.c_vec && (count == 1 || (sC * 2) % 16 == 0)) {
        // C's own shape: N × M (columns × rows) when the tiles are not transposed, M × N when they are
        const long long cc = c_t ? M : N, cr = c_t ? N : M;
        G9_TRY(encode_c_map(&mC, C, cc, cr, ldc, count, count == 1 ? (cr * ldc + 7) / 8 * 8 : sC));
        p.tma_c = 1;
    }
    if (c_t && !p.tma_c) return fail(GEN9BLAS_ERR, "internal: transposed HGEMM tiles need the TMA-store epilogue");
    if (pair) {
        p.tiles_m = (M + T2_BM - 1) / T2_BM;
        p.tiles_n = (N + bn - 1) / bn;
        p.total_tiles = (int)tiles;
        p.dp_tiles = (int)dp;
        p.split = split;
        p.units = (int)units;
        if (split > 1) {
            G9_TRY(gemm_handoff(d, st, &p.flags, &p.epoch));
            p.partial = (float *)((char *)scr + bytesA + bytesB);
        }
        const int grid2 = 2 * (int)(units < pairs ? units : pairs);
        if (type == GEN9BLAS_H) return bn == 256 ? launch_pair<true, 256>(mA, mB, mC, p, grid2, st)
                                                 : launch_pair<true, 128>(mA, mB, mC, p, grid2, st);
        return bn == 256 ? launch_pair<false, 256>(mA, mB, mC, p, grid2, st)
                         : launch_pair<false, 128>(mA, mB, mC, p, grid2, st);
    }
    p.tiles_m = (M + TC_BM - 1) / TC_BM;
    p.tiles_n = (N + TC_BN - 1) / TC_BN;
    p.total_tiles = p.tiles_m * p.tiles_n * count;
    const int units1 = p.total_tiles * ks;
    const int grid = units1 < d->sm_count ? units1 : d->sm_count;
    if (type == GEN9BLAS_H) {
        static bool attr[kMaxDevices] = {};
        G9_CU(smem_limit_once(hgemm_tc_kernel<true>, TC_SMEM, attr));
        hgemm_tc_kernel<true><<<grid, TC_THREADS, TC_SMEM, st>>>(mA, mB, p);
    } else {
        static bool attr[kMaxDevices] = {};
        G9_CU(smem_limit_once(hgemm_tc_kernel<false>, TC_SMEM, attr));
        hgemm_tc_kernel<false><<<grid, TC_THREADS, TC_SMEM, st>>>(mA, mB, p);
    }
    G9_TRY(launched("hgemm_tc"));
    if (ks > 1) {
        hgemm_ksum<<<4 * d->sm_count, 256, 0, st>>>(p.kpart, ks, M, N, (float)alpha, (float)beta, (__half *)C, ldc);
        return launched("hgemm_ksum");
    }
    return 0;
}

int launch_hgemm_tc(int type, int tA, int tB, int M, int N, int K, double alpha, const void *A, int lda, long long sA,
                    const void *B, int ldb, long long sB, double beta, void *C, int ldc, long long sC, int count,
                    cudaStream_t st, void *const *peers, int npeers, long long col_off) {
    // Both operands transposed: the tensor pipe runs about 18 % slower when its A operand is MN-major (measured on
    // B200, n = 4096), so C = Aᵀ·Bᵀ is computed as Cᵀ = B·A, with B (stored N × K, K-major) as the MMA's A operand and
    // A (stored K × M) as its MN-major B operand, and the epilogue writes the transposed tiles into C.
    const bool c_legal = ((uintptr_t)C & 15) == 0 && (ldc % 8) == 0 && (count == 1 || (sC % 8) == 0);
    if (tA && tB && !(peers && npeers > 0) && alpha == 1.0 && beta == 0.0 && M > 128 && N > 128 && pair_setting() == 1 &&
        c_legal)
        return hgemm_tc_impl(type, 0, 0, N, M, K, alpha, B, ldb, sB, A, lda, sA, beta, C, ldc, sC, count, st, nullptr, 0,
                             0, 1);
    return hgemm_tc_impl(type, tA, tB, M, N, K, alpha, A, lda, sA, B, ldb, sB, beta, C, ldc, sC, count, st, peers, npeers,
                         col_off, 0);
}

// ------------------------------------------------------------------------------------------------ wait self-test
// One thread waits on an mbarrier that nothing arrives on, through the same bounded wait the GEMM roles use; after
// limit_ns it gives up, sets the mapped error word and returns. Exercises the timeout path without any GPU fault.
__global__ void wait_probe_kernel(unsigned *err, unsigned long long limit_ns) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0 && !mbar_wait(&bar, 0, &abort_flag, limit_ns)) {
        *(volatile unsigned *)err = kDevErrWaitTimeout;
        __threadfence_system();
    }
}

}  // namespace g9

extern "C" GEN9BLAS_API int gen9blas_selftest_wait(double limit_ms) {
    using namespace g9;
    if (int e = begin_op()) return e;
    DevState *d = dev_state();
    if (limit_ms < 0.1) limit_ms = 0.1;
    if (limit_ms > 1000.0) limit_ms = 1000.0;
    wait_probe_kernel<<<1, 32, 0, stream()>>>(d->err_dev, (unsigned long long)(limit_ms * 1e6));
    G9_TRY(launched("wait_probe"));
    return finish_op(nullptr, 0);
}
