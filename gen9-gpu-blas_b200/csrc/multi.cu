// multi.cu -- one process, several GPUs: column-sharded GEMM behind gen9blas_gemm (and so behind the LD_PRELOAD
// CBLAS library and the NumPy module, which call it).
//
// The reference drives one iGPU (lib/src/gemm.c:177-180 has no device choice). Here gen9blas_set_devices (or
// GEN9BLAS_DEVICES="0,1,...", read once) lists the GPUs a large GEMM is split over: device i computes the column
// block C[:, n_i : n_i + nb] = alpha·op(A)·op(B)[:, n_i : n_i + nb] + beta·C[:, ...] with its own kernels on its own
// memory. Per device a pipeline on three streams: its B block first, then row bands of A (and of C when beta != 0)
// on the copy-in stream, one band GEMM per band on the compute stream, and the band of C back on the copy-out stream
// while the next band computes. Copies between GPUs are peer copies over NVLink (peer access is enabled when the
// devices allow it); an operand already in a device's memory is read in place there. No kernel of this library is
// ever given another GPU's memory, and nothing here uses a multicast load.
#include "internal.h"
#include <cstdio>
#include <cstdlib>
#include <cstring>

namespace g9 {

constexpr int kMaxShards = 8;

struct ShardConfig {
    int n = 0;                     // devices (0 or 1: no sharding)
    int ids[kMaxShards] = {};
    double min_flop = 2.0 * 4096.0 * 4096.0 * 4096.0;   // a GEMM shards from 2·M·N·K at least this
    bool env_read = false;
    bool peer_done[kMaxDevices][kMaxDevices] = {};
};
static ShardConfig g_shard;

static int elem_bytes(int type) { return type == GEN9BLAS_S ? 4 : type == GEN9BLAS_D ? 8 : 2; }

static int validate_devices(int n, const int *ids) {
    int count = 0;
    G9_CU(cudaGetDeviceCount(&count));
    if (n < 0 || n > kMaxShards) return fail(GEN9BLAS_ERR_INVALID_ARG, "1 to %d devices, got %d", kMaxShards, n);
    for (int i = 0; i < n; i++) {
        if (ids[i] < 0 || ids[i] >= count || ids[i] >= kMaxDevices)
            return fail(GEN9BLAS_ERR_INVALID_ARG, "device %d out of range (%d devices)", ids[i], count);
        for (int j = 0; j < i; j++)
            if (ids[j] == ids[i]) return fail(GEN9BLAS_ERR_INVALID_ARG, "device %d listed twice", ids[i]);
        int major = 0;
        G9_CU(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, ids[i]));
        if (major != 10) return fail(GEN9BLAS_ERR_NO_DEVICE, "device %d is not sm_100", ids[i]);
    }
    return 0;
}

// GEN9BLAS_DEVICES="0,1,2,3" and GEN9BLAS_SHARD_MIN_FLOP, read at the first sharding decision (an invalid list is an
// error of that call, and is then forgotten).
static int read_env() {
    if (g_shard.env_read) return 0;
    g_shard.env_read = true;
    if (const char *m = getenv("GEN9BLAS_SHARD_MIN_FLOP")) g_shard.min_flop = atof(m);
    const char *e = getenv("GEN9BLAS_DEVICES");
    if (!e || !*e) return 0;
    int ids[kMaxShards], n = 0;
    for (const char *p = e; *p;) {
        char *end = nullptr;
        long v = strtol(p, &end, 10);
        if (end == p || n == kMaxShards) return fail(GEN9BLAS_ERR_INVALID_ARG, "GEN9BLAS_DEVICES=\"%s\": expected up to %d "
                                                     "device numbers separated by commas", e, kMaxShards);
        ids[n++] = (int)v;
        p = *end == ',' ? end + 1 : end;
        if (*end && *end != ',') return fail(GEN9BLAS_ERR_INVALID_ARG, "GEN9BLAS_DEVICES=\"%s\": bad character", e);
    }
    G9_TRY(validate_devices(n, ids));
    g_shard.n = n;
    memcpy(g_shard.ids, ids, sizeof(int) * n);
    return 0;
}

// Makes dev the library's current device (its state and its own stream) for the scope; restores the caller's device
// and stream at the end.
struct DeviceScope {
    int cur;
    bool us_set;
    cudaStream_t us;
    explicit DeviceScope(int dev) : cur(G.cur_dev), us_set(G.user_stream_set), us(G.user_stream) {
        if (dev != cur) {
            G.cur_dev = dev;
            G.user_stream_set = false;
            G.user_stream = nullptr;
        }
    }
    ~DeviceScope() {
        G.cur_dev = cur;
        G.user_stream_set = us_set;
        G.user_stream = us;
        cudaSetDevice(cur);
    }
};

// Device whose memory holds p (-1: host memory, managed memory or unknown).
static int owner_device(const void *p, bool *managed) {
    cudaPointerAttributes a;
    *managed = false;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    *managed = a.type == cudaMemoryTypeManaged;
    return a.type == cudaMemoryTypeDevice ? a.device : -1;
}

static int enable_peer(int a, int b) {
    if (a == b || g_shard.peer_done[a][b]) return 0;
    g_shard.peer_done[a][b] = true;
    int can = 0;
    G9_CU(cudaDeviceCanAccessPeer(&can, a, b));
    if (!can) return 0;   // copies still work, staged by the driver
    G9_CU(cudaSetDevice(a));
    cudaError_t e = cudaDeviceEnablePeerAccess(b, 0);
    if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) return cuda_fail(e, "cudaDeviceEnablePeerAccess", __FILE__, __LINE__);
    cudaGetLastError();
    return 0;
}

static size_t round8(size_t x) { return (x + 7) / 8 * 8; }

// One device's share: columns [n0, n0 + nb) of C. The pointers are the caller's; `home` is the caller's device.
static int run_shard(int dev, int home, cudaEvent_t start, int type, int tA, int tB, int M, int nb, int n0, int K,
                     double alpha, const void *A, int lda, const void *B, int ldb, double beta, void *C, int ldc) {
    DeviceScope scope(dev);
    DevState *d = dev_state();
    if (!d) return G.status;
    G9_TRY(pipeline_streams(d));
    const size_t es = elem_bytes(type);
    bool mA, mB, mC;
    const int oA = owner_device(A, &mA), oB = owner_device(B, &mB), oC = owner_device(C, &mC);
    // in place: memory of this device, or managed memory on the caller's device
    const bool a_in = oA == dev || (mA && dev == home), b_in = oB == dev || (mB && dev == home);
    const bool c_in = oC == dev || (mC && dev == home);
    // local layouts (pitches rounded to 8 elements: 16-byte rows for the tensor-memory-access operands)
    const size_t lda_l = a_in ? lda : round8(tA ? M : K), ldb_l = b_in ? ldb : round8(tB ? K : nb);
    const size_t ldc_l = c_in ? ldc : round8(nb);
    const size_t bytesA = a_in ? 0 : ((size_t)(tA ? K : M) * lda_l * es + 255) / 256 * 256;
    const size_t bytesB = b_in ? 0 : ((size_t)(tB ? nb : K) * ldb_l * es + 255) / 256 * 256;
    const size_t bytesC = c_in ? 0 : (size_t)M * ldc_l * es;
    char *buf = nullptr;
    if (bytesA + bytesB + bytesC) G9_TRY(ensure_buffer(&d->shard, &d->shard_n, bytesA + bytesB + bytesC));
    buf = (char *)d->shard;
    const char *pA = a_in ? (const char *)A : buf;
    const char *pB = b_in ? (const char *)B + (tB ? (size_t)n0 * ldb : (size_t)n0) * es : buf + bytesA;
    char *pC = c_in ? (char *)C + (size_t)n0 * es : buf + bytesA + bytesB;
    cudaStream_t sm = stream(), si = d->copy_in, so = d->copy_out;
    cudaEvent_t *ev = d->band_ev;
    // everything already queued on the caller's stream (which may produce the operands) comes first
    G9_CU(cudaStreamWaitEvent(si, start, 0));
    G9_CU(cudaStreamWaitEvent(sm, start, 0));
    G9_CU(cudaStreamWaitEvent(so, start, 0));
    if (!b_in) {
        const char *src = (const char *)B + (tB ? (size_t)n0 * ldb : (size_t)n0) * es;
        if (tB)
            G9_CU(cudaMemcpy2DAsync((void *)pB, ldb_l * es, src, (size_t)ldb * es, (size_t)K * es, nb, cudaMemcpyDefault, si));
        else
            G9_CU(cudaMemcpy2DAsync((void *)pB, ldb_l * es, src, (size_t)ldb * es, (size_t)nb * es, K, cudaMemcpyDefault, si));
    }
    // row bands of C: four bands of whole 256-row tiles for tall problems, so that copies overlap band GEMMs
    int mb = M >= 1024 ? (((M + 3) / 4 + 255) / 256) * 256 : M;
    const int bands = (M + mb - 1) / mb;
    for (int i = 0; i < bands; i++) {
        const int r0 = i * mb, rows = M - r0 < mb ? M - r0 : mb;
        if (!a_in) {
            if (tA)   // stored K × M: the band is a block of columns
                G9_CU(cudaMemcpy2DAsync((void *)(pA + (size_t)r0 * es), lda_l * es, (const char *)A + (size_t)r0 * es,
                                        (size_t)lda * es, (size_t)rows * es, K, cudaMemcpyDefault, si));
            else
                G9_CU(cudaMemcpy2DAsync((void *)(pA + (size_t)r0 * lda_l * es), lda_l * es,
                                        (const char *)A + (size_t)r0 * lda * es, (size_t)lda * es, (size_t)K * es, rows,
                                        cudaMemcpyDefault, si));
        }
        if (!c_in && beta != 0.0)
            G9_CU(cudaMemcpy2DAsync(pC + (size_t)r0 * ldc_l * es, ldc_l * es, (const char *)C + ((size_t)r0 * ldc + n0) * es,
                                    (size_t)ldc * es, (size_t)nb * es, rows, cudaMemcpyDefault, si));
        G9_CU(cudaEventRecord(ev[1 + 2 * i], si));
        G9_CU(cudaStreamWaitEvent(sm, ev[1 + 2 * i], 0));
        const char *aband = tA ? pA + (size_t)r0 * es : pA + (size_t)r0 * lda_l * es;
        G9_TRY(launch_gemm(type, tA, tB, rows, nb, K, alpha, aband, (int)lda_l, 0, pB, (int)ldb_l, 0, beta,
                           pC + (size_t)r0 * ldc_l * es, (int)ldc_l, 0, 1, sm));
        G9_CU(cudaEventRecord(ev[2 + 2 * i], sm));
        G9_CU(cudaStreamWaitEvent(so, ev[2 + 2 * i], 0));
        if (!c_in)
            G9_CU(cudaMemcpy2DAsync((char *)C + ((size_t)r0 * ldc + n0) * es, (size_t)ldc * es, pC + (size_t)r0 * ldc_l * es,
                                    ldc_l * es, (size_t)nb * es, rows, cudaMemcpyDefault, so));
    }
    return 0;
}

static int sync_shard(int dev) {
    DeviceScope scope(dev);
    DevState *d = dev_state();
    if (!d) return G.status;
    G9_CU(cudaStreamSynchronize(d->copy_in));
    G9_CU(cudaStreamSynchronize(stream()));
    G9_CU(cudaStreamSynchronize(d->copy_out));
    return check_dev_err(d);
}

int gemm_sharded(int type, int tA, int tB, int M, int N, int K, double alpha, const void *A, int lda, const void *B,
                 int ldb, double beta, void *C, int ldc) {
    G9_TRY(read_env());
    if (g_shard.n < 2) return 1;
    const int thr = skinny_threshold(type);
    if ((M < N ? M : N) <= thr || K <= thr || 2.0 * M * N * K < g_shard.min_flop) return 1;
    const int home = G.cur_dev, nd = g_shard.n;
    // column blocks of whole 256-column tiles
    int nbw = (N + nd - 1) / nd;
    nbw = (nbw + 255) / 256 * 256;
    DevState *hd = dev_state();
    if (!hd) return G.status;
    if (!hd->ev0) return fail(GEN9BLAS_ERR, "device state without events");
    for (int i = 0; i < nd; i++) {
        G9_TRY(enable_peer(g_shard.ids[i], home));
        G9_TRY(enable_peer(home, g_shard.ids[i]));
    }
    G9_CU(cudaSetDevice(home));
    // the shards start after the caller's queued work on its stream (it may produce A, B or C); the event is the
    // last of the caller's device's band events, which its own band pipelines (at most 4 bands) never use
    G9_TRY(pipeline_streams(hd));
    cudaEvent_t start = hd->band_ev[2 * 16 + 1];
    G9_CU(cudaEventRecord(start, stream()));
    int first_err = 0;
    int launched_n = 0;
    for (int i = 0; i < nd; i++) {
        const int n0 = i * nbw;
        if (n0 >= N) break;
        const int nb = N - n0 < nbw ? N - n0 : nbw;
        const int r = run_shard(g_shard.ids[i], home, start, type, tA, tB, M, nb, n0, K, alpha, A, lda, B, ldb, beta, C,
                                ldc);
        launched_n = i + 1;
        if (r < 0) {
            first_err = r;
            break;
        }
    }
    char msg[sizeof(G.err)] = {0};
    if (first_err) memcpy(msg, G.err, sizeof msg);
    for (int i = 0; i < launched_n; i++) {   // every device that got work is waited for, also after an error
        const int r = sync_shard(g_shard.ids[i]);
        if (r < 0 && !first_err) {
            first_err = r;
            memcpy(msg, G.err, sizeof msg);
        }
    }
    G9_CU(cudaSetDevice(home));
    bool home_synced = false;
    for (int i = 0; i < launched_n; i++) home_synced = home_synced || g_shard.ids[i] == home;
    if (home_synced) queued_writes_clear(hd);   // the caller's stream was waited for
    G.last_zc = 0;
    if (first_err) {
        memcpy(G.err, msg, sizeof msg);
        G.status = first_err;
        return first_err;
    }
    return 0;
}

}  // namespace g9

using namespace g9;

extern "C" {

GEN9BLAS_API int gen9blas_set_devices(int n, const int *ids) {
    if (int e = begin_op()) return e;
    G9_TRY(read_env());
    if (n > 1 && !ids) return fail(GEN9BLAS_ERR_INVALID_ARG, "NULL device list");
    if (n > 1) G9_TRY(validate_devices(n, ids));
    g_shard.n = n > 1 ? n : 0;
    if (n > 1) memcpy(g_shard.ids, ids, sizeof(int) * n);
    return 0;
}

GEN9BLAS_API int gen9blas_get_devices(int *ids, int max) {
    if (int e = begin_op()) return e;
    G9_TRY(read_env());
    for (int i = 0; i < g_shard.n && i < max; i++)
        if (ids) ids[i] = g_shard.ids[i];
    return g_shard.n;
}

}  // extern "C"
