// peer.cu -- rank barrier over NVLink peer memory for the fused multi-GPU paths (no counterpart in the reference,
// which drives one device).
//
// After a fused GEMM / skinny all-gather each rank has stored its block into every rank's C. Before a rank reads C it
// must know that all other ranks' stores have landed. Each rank owns a flag array of nranks + 1 words in its own
// device memory, mapped into the other ranks (CUDA IPC); word nranks is the rank's barrier counter. The barrier
// kernel of rank r
//   1. takes epoch = counter + 1 and stores it back (only rank r's own barrier kernels touch its counter, in stream
//      order, so the epoch needs no host argument and a captured CUDA graph can replay the barrier);
//   2. stores the epoch into word r of every rank's array (release, system scope: the stores of the preceding kernel
//      on this stream, which fenced them at system scope, are ordered before the flag);
//   3. waits until every word 0..nranks-1 of its own array has reached the epoch (acquire, system scope), so that the
//      kernels enqueued after it read the complete C.
// All ranks run the same sequence of barriers, so their epochs agree; words are compared with wrap-around arithmetic.
// The wait is bounded by a global-timer limit; a wait that gives up writes the mapped error word and the kernel
// returns, so the call reports GEN9BLAS_ERR and the device stays usable.
#include "internal.h"

namespace g9 {

struct PeerBarrierArgs {
    unsigned *flags[8];   // rank q's flag array (this rank's own array at index `rank`)
    int nranks, rank;
    unsigned long long limit_ns;
    unsigned *err;
};

__device__ __forceinline__ unsigned long long peer_globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__global__ void peer_barrier_kernel(const PeerBarrierArgs a) {
    const int q = threadIdx.x;
    unsigned epoch = 0;
    if (q == 0) {
        unsigned *counter = a.flags[a.rank] + a.nranks;
        epoch = *counter + 1u;
        *counter = epoch;
    }
    epoch = __shfl_sync(0xffffffffu, epoch, 0);
    if (q < a.nranks) {
        __threadfence_system();
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a.flags[q] + a.rank), "r"(epoch) : "memory");
    }
    __syncwarp();
    bool ok = true;
    if (q < a.nranks) {
        const unsigned *mine = a.flags[a.rank] + q;
        const unsigned long long t0 = peer_globaltimer();
        for (unsigned it = 0;; ++it) {
            unsigned v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
            if ((int)(v - epoch) >= 0) break;
            if ((it & 63) == 63 && peer_globaltimer() - t0 > a.limit_ns) {
                ok = false;
                break;
            }
        }
    }
    if (!ok) *(volatile unsigned *)a.err = kDevErrWaitTimeout;
    __syncwarp();
    __threadfence_system();
}

}  // namespace g9

using namespace g9;

extern "C" GEN9BLAS_API int gen9blas_peer_barrier(void *const *rank_flags, int nranks, int rank, double timeout_ms) {
    if (int e = begin_op()) return e;
    if (!rank_flags || nranks < 1 || nranks > 8 || rank < 0 || rank >= nranks)
        return fail(GEN9BLAS_ERR_INVALID_ARG, "gen9blas_peer_barrier: 1..8 ranks and 0 <= rank < nranks required");
    if (!(timeout_ms >= 0.1)) timeout_ms = 0.1;
    if (timeout_ms > 60000.0) timeout_ms = 60000.0;
    DevState *d = dev_state();
    if (!d) return G.status;
    PeerBarrierArgs a;
    for (int q = 0; q < nranks; q++) {
        if (!rank_flags[q] || ((uintptr_t)rank_flags[q] & 3))
            return fail(GEN9BLAS_ERR_INVALID_ARG, "gen9blas_peer_barrier: flag array %d is NULL or misaligned", q);
        a.flags[q] = (unsigned *)rank_flags[q];
    }
    a.nranks = nranks;
    a.rank = rank;
    a.limit_ns = (unsigned long long)(timeout_ms * 1e6);
    a.err = d->err_dev;
    timer_start();
    timer_kernel();
    peer_barrier_kernel<<<1, 32, 0, stream()>>>(a);
    G9_TRY(launched("peer_barrier"));
    int r = finish_op(nullptr, 0);
    timer_stop();
    return r;
}
