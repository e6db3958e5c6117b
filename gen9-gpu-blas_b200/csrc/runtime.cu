// runtime.cu -- initialisation, status, memory and the host/device boundary of libgen9blas.so (B200 build).
//
// Replaces the reference runtime lib/src/core.c (init 114-219, has 222-236, wait_gpu 240-258, alloc 288-297,
// get_obj 328-340, to_host 363-367, getters 385-392) and its i915 layer lib/kcl.c. The design differs where the
// hardware differs:
// - "zero-copy" operands are device memory (cudaMalloc, torch tensors) and managed memory (gen9blas_alloc), used in
//   place; any other host pointer is staged through grow-only device buffers (the reference copies into USM buffers);
// - the wait is a stream synchronisation, then a check of a mapped error word that device-side bounded waits set
//   (the reference polls GEM_WAIT with a 60 s limit, kcl.c:361-372);
// - the state is per CUDA device so that one process per GPU (or one process switching devices) works.
#include "internal.h"
#include <cuda.h>
#include <cudaTypedefs.h>
#include <pthread.h>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <ctime>

namespace g9 {

CallState G;
static DevState g_dev[kMaxDevices];
static pthread_once_t g_once = PTHREAD_ONCE_INIT;
static int g_init_status = -1;
static char g_init_err[sizeof(G.err)];

int fail(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(G.err, sizeof G.err, fmt, ap);
    va_end(ap);
    G.status = code;
    return code;
}

int cuda_fail(cudaError_t e, const char *what, const char *file, int line) {
    int code = e == cudaErrorMemoryAllocation ? GEN9BLAS_ERR_OUT_OF_MEMORY : GEN9BLAS_ERR;
    const char *base = strrchr(file, '/');
    return fail(code, "%s:%d: %s = %s (%s)", base ? base + 1 : file, line, what, cudaGetErrorName(e),
                cudaGetErrorString(e));
}

static double now_s() {
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec + ts.tv_nsec * 1e-9;
}

// Once per process: find an sm_100 device. A failure is final, as in the reference (core.c:205-219).
static void init_run() {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0) {
        cudaGetLastError();
        snprintf(g_init_err, sizeof g_init_err, "no CUDA device (%s)", e != cudaSuccess ? cudaGetErrorString(e) : "count 0");
        g_init_status = GEN9BLAS_ERR_NO_DEVICE;
        return;
    }
    int cur = 0;
    cudaGetDevice(&cur);
    int major = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, cur);
    if (major != 10) {
        snprintf(g_init_err, sizeof g_init_err, "device %d has compute capability %d.x; this build runs sm_100a kernels only",
                 cur, major);
        g_init_status = GEN9BLAS_ERR_NO_DEVICE;
        return;
    }
    const char *p = getenv("GEN9BLAS_PROFILE");
    G.profile = p && *p && strcmp(p, "0") != 0;
    G.cur_dev = cur;
    g_init_status = 0;
}

static int device_setup(DevState &d, int dev) {
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != dev) G9_CU(cudaSetDevice(dev));
    d.dev = dev;
    G9_CU(cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev));
    G9_CU(cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev));
    G9_CU(cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev));
    if (d.cc_major != 10) G9_FAIL(GEN9BLAS_ERR_NO_DEVICE, "device %d is not sm_100 (cc %d.%d)", dev, d.cc_major, d.cc_minor);
    G9_CU(cudaStreamCreateWithFlags(&d.own_stream, cudaStreamNonBlocking));
    G9_CU(cudaHostAlloc((void **)&d.result_host, 4096, cudaHostAllocDefault));
    G9_CU(cudaHostAlloc((void **)&d.err_host, 64, cudaHostAllocMapped));
    *d.err_host = kDevErrNone;
    G9_CU(cudaHostGetDevicePointer((void **)&d.err_dev, d.err_host, 0));
    G9_CU(cudaEventCreate(&d.ev0));
    G9_CU(cudaEventCreate(&d.ev1));
    d.ready = true;
    return 0;
}

DevState *dev_state() {
    int dev = G.cur_dev;
    if (dev < 0 || dev >= kMaxDevices) {
        fail(GEN9BLAS_ERR_INVALID_ARG, "device %d out of range", dev);
        return nullptr;
    }
    DevState &d = g_dev[dev];
    int cur = -1;
    cudaGetDevice(&cur);
    if (cur != dev && cudaSetDevice(dev) != cudaSuccess) {
        cudaGetLastError();
        fail(GEN9BLAS_ERR, "cudaSetDevice(%d) failed", dev);
        return nullptr;
    }
    if (!d.ready && device_setup(d, dev) < 0) return nullptr;
    return &d;
}

DevState *dev_state_if_ready(int dev) {
    if (dev < 0 || dev >= kMaxDevices || !g_dev[dev].ready) return nullptr;
    return &g_dev[dev];
}

cudaStream_t stream() {
    if (G.user_stream_set) return G.user_stream;
    DevState *d = dev_state();
    return d ? d->own_stream : nullptr;
}

int begin_op() {
    G.status = 0;
    G.err[0] = 0;
    pthread_once(&g_once, init_run);
    if (g_init_status) return fail(GEN9BLAS_ERR_NO_DEVICE, "%s", g_init_err);
    if (!dev_state()) return G.status ? G.status : GEN9BLAS_ERR;
    return 0;
}

// Host-side fault injection for the error-path tests (no GPU fault is ever provoked): GEN9BLAS_FAULT=alloc makes
// every device buffer allocation report out-of-memory, =launch makes every kernel launch report a launch error,
// =wait makes every call end as if a device-side bounded wait had given up. Read once per process.
enum { kFaultNone = 0, kFaultAlloc, kFaultLaunch, kFaultWait };
static int fault_mode() {
    static int m = -1;
    if (m < 0) {
        const char *e = getenv("GEN9BLAS_FAULT");
        m = !e ? kFaultNone : !strcmp(e, "alloc") ? kFaultAlloc : !strcmp(e, "launch") ? kFaultLaunch
            : !strcmp(e, "wait") ? kFaultWait : kFaultNone;
    }
    return m;
}

int launched(const char *name) {
    G.launches++;
    if (fault_mode() == kFaultLaunch) {
        cudaGetLastError();
        return fail(GEN9BLAS_ERR, "launch of %s failed: injected fault (GEN9BLAS_FAULT=launch)", name);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(GEN9BLAS_ERR, "launch of %s failed: %s", name, cudaGetErrorString(e));
    return 0;
}

static int ensure_dev_buf(void **p, size_t *n, size_t bytes) {
    if (*n >= bytes) return 0;
    if (*p) {
        G9_CU(cudaStreamSynchronize(stream()));
        G9_CU(cudaFree(*p));
        *p = nullptr;
        *n = 0;
    }
    size_t want = bytes < 4096 ? 4096 : (bytes + 0xFFFFF) & ~(size_t)0xFFFFF;   // round to 1 MiB
    if (fault_mode() == kFaultAlloc)
        return fail(GEN9BLAS_ERR_OUT_OF_MEMORY, "cudaMalloc(%zu): injected fault (GEN9BLAS_FAULT=alloc)", want);
    G9_CU(cudaMalloc(p, want));
    *n = want;
    return 0;
}

int ensure_buffer(void **p, size_t *n, size_t bytes) { return ensure_dev_buf(p, n, bytes); }

int ml_buffer(size_t bytes, void **p) {
    DevState *d = dev_state();
    if (!d) return G.status;
    G9_TRY(ensure_dev_buf(&d->ml, &d->ml_n, bytes));
    *p = d->ml;
    return 0;
}

unsigned *nowait_slot(DevState *d) {
    if (!d->nw_host) {
        if (cudaHostAlloc((void **)&d->nw_host, DevState::kNowaitSlots * sizeof(unsigned), cudaHostAllocMapped) !=
                cudaSuccess ||
            cudaHostGetDevicePointer((void **)&d->nw_dev, d->nw_host, 0) != cudaSuccess) {
            cudaGetLastError();
            d->nw_host = nullptr;
            return nullptr;
        }
        memset(d->nw_host, 0, DevState::kNowaitSlots * sizeof(unsigned));
    }
    if (d->nw_used == DevState::kNowaitSlots) return nullptr;
    return d->nw_dev + d->nw_used++;
}

int gemm_handoff(DevState *d, cudaStream_t st, unsigned **flags, unsigned *epoch) {
    if (!d->gemm_flags) {
        G9_CU(cudaMalloc((void **)&d->gemm_flags, kGemmFlags * sizeof(unsigned)));
        G9_CU(cudaMemsetAsync(d->gemm_flags, 0, kGemmFlags * sizeof(unsigned), st));
    }
    if (++d->gemm_epoch == 0) d->gemm_epoch = 1;
    *flags = d->gemm_flags;
    *epoch = d->gemm_epoch;
    return 0;
}

int scratch(size_t bytes, void **p) {
    DevState *d = dev_state();
    if (!d) return G.status;
    G9_TRY(ensure_dev_buf(&d->scratch, &d->scratch_n, bytes));
    *p = d->scratch;
    return 0;
}

int stage_buffer(int slot, size_t bytes, void **p) {
    DevState *d = dev_state();
    if (!d) return G.status;
    G9_TRY(ensure_dev_buf(&d->stage[slot], &d->stage_n[slot], bytes));
    *p = d->stage[slot];
    return 0;
}

int pipeline_streams(DevState *d) {
    if (d->copy_in) return 0;
    G9_CU(cudaStreamCreateWithFlags(&d->copy_in, cudaStreamNonBlocking));
    G9_CU(cudaStreamCreateWithFlags(&d->copy_out, cudaStreamNonBlocking));
    for (auto &e : d->band_ev) G9_CU(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    return 0;
}

int skinny_slots(size_t words, uint64_t **p, unsigned *epoch) {
    DevState *d = dev_state();
    if (!d) return G.status;
    const bool wrap = ++d->sk_epoch == 0;
    if (wrap) d->sk_epoch = 1;
    if (d->sk_part_n < words || wrap) {
        void *buf = d->sk_part;
        size_t bytes = d->sk_part_n * sizeof(uint64_t);
        G9_TRY(ensure_dev_buf(&buf, &bytes, words * sizeof(uint64_t)));
        G9_CU(cudaMemsetAsync(buf, 0, bytes, stream()));
        d->sk_part = (uint64_t *)buf;
        d->sk_part_n = bytes / sizeof(uint64_t);
    }
    *p = d->sk_part;
    *epoch = d->sk_epoch;
    return 0;
}

int arrival_counters(size_t n, unsigned **p) {
    DevState *d = dev_state();
    if (!d) return G.status;
    if (d->at_cnt_n < n) {
        void *buf = d->at_cnt;
        size_t bytes = d->at_cnt_n * sizeof(unsigned);
        G9_TRY(ensure_dev_buf(&buf, &bytes, n * sizeof(unsigned)));
        G9_CU(cudaMemsetAsync(buf, 0, bytes, stream()));
        d->at_cnt = (unsigned *)buf;
        d->at_cnt_n = bytes / sizeof(unsigned);
    }
    *p = d->at_cnt;
    return 0;
}

int map_operand(Operand &op, const void *p, size_t bytes, int slot, bool copy_in, bool written) {
    op.user = p;
    op.bytes = bytes;
    op.written = written;
    DevState *d = dev_state();
    if (!d) return G.status;
    if (!p) return fail(GEN9BLAS_ERR_INVALID_ARG, "NULL operand");
    cudaPointerAttributes a;
    cudaError_t e = cudaPointerGetAttributes(&a, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        a.type = cudaMemoryTypeUnregistered;
    }
    if (a.type == cudaMemoryTypeDevice) {
        if (a.device != d->dev)
            return fail(GEN9BLAS_ERR_INVALID_ARG, "operand is memory of device %d, the current device is %d", a.device, d->dev);
        op.dptr = const_cast<void *>(p);
        op.zc = true;
        return 0;
    }
    if (a.type == cudaMemoryTypeManaged) {
        op.dptr = const_cast<void *>(p);
        op.zc = true;
#if CUDART_VERSION >= 12020
        cudaMemLocation loc;
        loc.type = cudaMemLocationTypeDevice;
        loc.id = d->dev;
        if (cudaMemPrefetchAsync(p, bytes, loc, 0, stream()) != cudaSuccess) cudaGetLastError();
#endif
        return 0;
    }
    // Host memory (pageable or pinned): stage through the slot's device buffer.
    G9_TRY(ensure_dev_buf(&d->stage[slot], &d->stage_n[slot], bytes));
    op.dptr = d->stage[slot];
    op.zc = false;
    if (copy_in) G9_CU(cudaMemcpyAsync(op.dptr, p, bytes, cudaMemcpyHostToDevice, stream()));
    return 0;
}

int check_dev_err(DevState *d) {
    if (fault_mode() == kFaultWait) *(volatile unsigned *)d->err_host = kDevErrWaitTimeout;
    unsigned v = *(volatile unsigned *)d->err_host;
    if (v != kDevErrNone) {
        *(volatile unsigned *)d->err_host = kDevErrNone;
        if (v == kDevErrWaitTimeout)
            return fail(GEN9BLAS_ERR, "a device-side wait gave up (bounded mbarrier wait timed out); results are invalid");
        return fail(GEN9BLAS_ERR, "device-side error code %u", v);
    }
    return 0;
}

// Drops entry i (its write has completed), keeping the others' order irrelevant: the last entry takes its place.
static void queued_drop(DevState *d, int i) {
    const int last = d->queued_n - 1;
    if (i != last) {
        d->queued_lo[i] = d->queued_lo[last];
        d->queued_hi[i] = d->queued_hi[last];
        cudaEvent_t e = d->queued_ev[i];
        d->queued_ev[i] = d->queued_ev[last];
        d->queued_ev[last] = e;
    }
    d->queued_n = last;
}

static bool queued_done(DevState *d, int i) {
    const cudaError_t e = cudaEventQuery(d->queued_ev[i]);
    if (e == cudaErrorNotReady) return false;
    cudaGetLastError();
    return e == cudaSuccess;
}

void queued_writes_add(DevState *d, const void *p, size_t bytes, cudaStream_t st) {
    if (!bytes) return;
    const uintptr_t lo = (uintptr_t)p, hi = lo + bytes;
    int slot = -1;
    for (int i = 0; i < d->queued_n && slot < 0; i++)   // a range that overlaps or touches an entry widens it
        if (lo <= d->queued_hi[i] && d->queued_lo[i] <= hi) slot = i;
    if (slot < 0 && d->queued_n == DevState::kQueuedRanges)
        for (int i = d->queued_n - 1; i >= 0; i--)       // full: forget the writes that have completed
            if (queued_done(d, i)) queued_drop(d, i);
    if (slot < 0) {
        if (d->queued_n == DevState::kQueuedRanges) {    // still full: every later check answers "maybe written"
            d->queued_overflow = true;
            return;
        }
        slot = d->queued_n++;
        d->queued_lo[slot] = lo;
        d->queued_hi[slot] = hi;
    } else {
        if (lo < d->queued_lo[slot]) d->queued_lo[slot] = lo;
        if (hi > d->queued_hi[slot]) d->queued_hi[slot] = hi;
    }
    if (!d->queued_ev[slot] && cudaEventCreateWithFlags(&d->queued_ev[slot], cudaEventDisableTiming) != cudaSuccess) {
        cudaGetLastError();
        d->queued_overflow = true;   // cannot tell when it completes: stay conservative
        return;
    }
    if (cudaEventRecord(d->queued_ev[slot], st) != cudaSuccess) {
        cudaGetLastError();
        d->queued_overflow = true;
    }
}

void queued_writes_clear(DevState *d) {
    d->queued_n = 0;
    d->queued_overflow = false;
}

bool queued_writes_overlap(DevState *d, const void *p, size_t bytes) {
    if (d->queued_overflow) return true;
    const uintptr_t lo = (uintptr_t)p, hi = lo + bytes;
    for (int i = d->queued_n - 1; i >= 0; i--) {
        if (!(lo < d->queued_hi[i] && d->queued_lo[i] < hi)) continue;
        if (!queued_done(d, i)) return true;
        queued_drop(d, i);   // that write has finished
    }
    return false;
}

int finish_op(Operand *ops, int n) {
    DevState *d = dev_state();
    if (!d) return G.status;
    cudaStream_t st = stream();
    bool all_zc = true;
    for (int i = 0; i < n; i++) all_zc = all_zc && ops[i].zc;
    if (G.nowait && all_zc) {
        for (int i = 0; i < n; i++)
            if (ops[i].written) queued_writes_add(d, ops[i].dptr, ops[i].bytes, st);
        return 0;
    }
    for (int i = 0; i < n; i++) {
        if (!ops[i].written || ops[i].zc) continue;
        if (ops[i].pitch)
            G9_CU(cudaMemcpy2DAsync(const_cast<void *>(ops[i].user), ops[i].pitch, ops[i].dptr, ops[i].pitch,
                                    ops[i].width, ops[i].rows, cudaMemcpyDeviceToHost, st));
        else
            G9_CU(cudaMemcpyAsync(const_cast<void *>(ops[i].user), ops[i].dptr, ops[i].bytes, cudaMemcpyDeviceToHost, st));
    }
    G9_CU(cudaStreamSynchronize(st));
    queued_writes_clear(d);
    return check_dev_err(d);
}

static double g_t0;
void timer_start() { g_t0 = now_s(); }
void timer_kernel() {
    if (G.profile && !G.nowait) {   // read back by timer_stop only for synchronous calls
        DevState *d = dev_state();
        if (d) cudaEventRecord(d->ev0, stream());
    }
}
void timer_stop() {
    if (G.profile && !G.nowait) {
        DevState *d = dev_state();
        if (d) {
            cudaEventRecord(d->ev1, stream());
            cudaEventSynchronize(d->ev1);
            float ms = 0;
            if (cudaEventElapsedTime(&ms, d->ev0, d->ev1) == cudaSuccess) {
                G.last_ms = ms;
                return;
            }
            cudaGetLastError();   // the start event was not recorded by this call: wall clock below
        }
    }
    G.last_ms = (now_s() - g_t0) * 1e3;
}

void *tensor_map_encoder() {
    static void *fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            fn = nullptr;
        }
    }
    return fn;
}

}  // namespace g9

using namespace g9;

extern "C" {

GEN9BLAS_API int gen9blas_version(void) { return GEN9BLAS_VERSION; }

GEN9BLAS_API int gen9blas_init(void) {
    pthread_once(&g_once, init_run);
    if (g_init_status) return fail(GEN9BLAS_ERR_NO_DEVICE, "%s", g_init_err);
    return 0;
}

GEN9BLAS_API int gen9blas_device_gen(void) {
    if (gen9blas_init()) return 0;
    DevState *d = dev_state();
    return d ? d->cc_major * 10 + d->cc_minor : 0;
}

GEN9BLAS_API int gen9blas_has(int f) {
    if (gen9blas_init()) return 0;
    switch (f) {
    case GEN9BLAS_FEAT_FP16:
    case GEN9BLAS_FEAT_FP32:
    case GEN9BLAS_FEAT_FP64:
    case GEN9BLAS_FEAT_SKINNY_PB: return 1;   // gen9blas_gemm_pb_skinny
    default: return 0;
    }
}

GEN9BLAS_API const char *gen9blas_error(void) { return G.err; }
GEN9BLAS_API int gen9blas_last_status(void) { return G.status; }
GEN9BLAS_API double gen9blas_last_time_ms(void) { return G.last_ms; }
GEN9BLAS_API int gen9blas_last_zero_copy(void) { return G.last_zc; }
GEN9BLAS_API long long gen9blas_kernel_launches(void) { return G.launches; }

GEN9BLAS_API void *gen9blas_alloc(size_t bytes) {
    if (begin_op()) return nullptr;
    void *p = nullptr;
    cudaError_t e = cudaMallocManaged(&p, bytes ? bytes : 1, cudaMemAttachGlobal);
    if (e != cudaSuccess) {
        cudaGetLastError();
        fail(GEN9BLAS_ERR_OUT_OF_MEMORY, "cudaMallocManaged(%zu) = %s", bytes, cudaGetErrorName(e));
        return nullptr;
    }
    return p;
}

GEN9BLAS_API void gen9blas_free(void *p) {
    if (!p || gen9blas_init()) return;
    cudaDeviceSynchronize();
    if (cudaFree(p) != cudaSuccess) cudaGetLastError();
}

GEN9BLAS_API int gen9blas_is_usm(const void *p, size_t bytes) {
    if (!p || gen9blas_init()) return 0;
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    if (a.type != cudaMemoryTypeManaged) return 0;
    // The CUDA runtime reports the allocation range through the driver only; the end check uses the last byte.
    if (bytes > 1) {
        cudaPointerAttributes b;
        if (cudaPointerGetAttributes(&b, (const char *)p + bytes - 1) != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        return b.type == cudaMemoryTypeManaged;
    }
    return 1;
}

GEN9BLAS_API int gen9blas_set_device(int device) {
    if (gen9blas_init()) return G.status;
    int n = 0;
    cudaGetDeviceCount(&n);
    if (device < 0 || device >= n || device >= kMaxDevices)
        return fail(GEN9BLAS_ERR_INVALID_ARG, "device %d out of range (%d devices)", device, n);
    G.cur_dev = device;
    G.user_stream_set = false;
    G.user_stream = nullptr;
    return dev_state() ? 0 : G.status;
}

GEN9BLAS_API int gen9blas_get_device(void) { return gen9blas_init() ? -1 : G.cur_dev; }

GEN9BLAS_API int gen9blas_set_stream(void *s) {
    if (gen9blas_init()) return G.status;
    G.user_stream = (cudaStream_t)s;
    G.user_stream_set = s != nullptr;
    return 0;
}

GEN9BLAS_API void gen9blas_set_nowait(int on) { G.nowait = on != 0; }

// ---- device buffers shared between the ranks' processes (CUDA IPC over NVLink / NVSwitch) ----
GEN9BLAS_API void *gen9blas_dev_alloc(size_t bytes) {
    if (begin_op()) return nullptr;
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes ? bytes : 1);
    if (e != cudaSuccess) {
        cudaGetLastError();
        fail(GEN9BLAS_ERR_OUT_OF_MEMORY, "cudaMalloc(%zu) = %s", bytes, cudaGetErrorName(e));
        return nullptr;
    }
    return p;
}

GEN9BLAS_API void gen9blas_dev_free(void *p) {
    if (!p || gen9blas_init()) return;
    cudaDeviceSynchronize();
    if (cudaFree(p) != cudaSuccess) cudaGetLastError();
}

GEN9BLAS_API int gen9blas_ipc_handle(const void *dev_ptr, void *handle, int64_t *offset) {
    if (int e = begin_op()) return e;
    if (!dev_ptr || !handle || !offset) return fail(GEN9BLAS_ERR_INVALID_ARG, "NULL argument");
    // The handle names the whole cudaMalloc allocation; the pointer's offset inside it travels alongside.
    static PFN_cuMemGetAddressRange_v3020 range = nullptr;
    if (!range) {
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", (void **)&range, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            return fail(GEN9BLAS_ERR, "cuMemGetAddressRange is not available from the driver");
        }
    }
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, (CUdeviceptr)dev_ptr) != CUDA_SUCCESS)
        return fail(GEN9BLAS_ERR_INVALID_ARG, "not device memory of this process");
    cudaIpcMemHandle_t h;
    G9_CU(cudaIpcGetMemHandle(&h, (void *)base));
    memcpy(handle, &h, sizeof h);
    *offset = (int64_t)((CUdeviceptr)dev_ptr - base);
    return 0;
}

GEN9BLAS_API void *gen9blas_ipc_open(const void *handle) {
    if (begin_op()) return nullptr;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof h);
    void *p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
        cudaGetLastError();
        fail(GEN9BLAS_ERR, "cudaIpcOpenMemHandle = %s", cudaGetErrorName(e));
        return nullptr;
    }
    return p;
}

GEN9BLAS_API int gen9blas_ipc_close(void *peer_ptr) {
    if (int e = begin_op()) return e;
    G9_CU(cudaIpcCloseMemHandle(peer_ptr));
    return 0;
}

GEN9BLAS_API int gen9blas_flush(void) {
    if (begin_op()) return G.status;
    G9_CU(cudaStreamSynchronize(stream()));
    queued_writes_clear(dev_state());
    return check_dev_err(dev_state());
}

}  // extern "C"
