// internal.h -- state and helpers shared by the translation units of libgen9blas.so (B200 build). Not installed.
//
// The reference keeps an OpenCL context, a queue, USM work buffers and per-type kernel tables
// (lib/src/internal.h:22-60, lib/src/core.c:114-203). Here the runtime is the CUDA runtime: one state block per CUDA
// device (stream, staging buffers, scratch, a mapped error word for bounded device-side waits), selected by
// gen9blas_set_device. Everything in this header has hidden visibility.
#pragma once
#include "gen9blas.h"
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

#pragma GCC visibility push(hidden)
namespace g9 {

constexpr int kMaxDevices = 16;
constexpr int kStageSlots = 3;   // staged operands per call (A, B, C or x, y, A)

// Device-side error codes written into DevState::err_host by kernels whose waits gave up.
enum : unsigned { kDevErrNone = 0, kDevErrWaitTimeout = 1, kDevErrTmemAlloc = 2 };

struct DevState {
    bool ready = false;
    int dev = -1;
    int sm_count = 0;
    int cc_major = 0, cc_minor = 0;
    cudaStream_t own_stream = nullptr;
    void *stage[kStageSlots] = {nullptr, nullptr, nullptr};   // device copies of staged host operands
    size_t stage_n[kStageSlots] = {0, 0, 0};
    void *scratch = nullptr;                                   // partial sums, packed operands
    size_t scratch_n = 0;
    double *result_host = nullptr;                             // pinned: scalar results of reductions
    unsigned *err_host = nullptr;                              // mapped pinned words: [0] device-side error code,
    unsigned *err_dev = nullptr;                               // [1] non-finite flag of gemm_pb_skinny; device address
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    unsigned *gemm_flags = nullptr;                            // split-K handoff flags of the HGEMM pair kernel (zeroed)
    unsigned gemm_epoch = 0;                                   // launch counter written into those flags
    void *l3 = nullptr;                                        // level-3 work matrices (grow-only)
    size_t l3_n = 0;
    void *l2x = nullptr;                                       // level-2 work vectors / unpacked triangles (grow-only)
    size_t l2x_n = 0;
    cudaStream_t copy_in = nullptr, copy_out = nullptr;        // host-operand GEMM pipeline: H2D and D2H streams
    cudaEvent_t band_ev[2 * 17] = {};                          // and its events (band inputs ready, band C done)
    unsigned long long *sv_msg = nullptr;                      // value messages of the look-back triangular solve
    size_t sv_msg_n = 0;                                       // (epoch-stamped 64-bit words, zeroed on growth)
    unsigned sv_epoch = 0;
    uint64_t *sk_part = nullptr;                               // epoch-tagged partial tiles of the stream-K skinny
    size_t sk_part_n = 0;                                      // kernel (words; zeroed when created or grown)
    unsigned sk_epoch = 0;                                     // launch counter written into those tags
    unsigned *at_cnt = nullptr;                                // arrival counters of the attention kernel's rows and
    size_t at_cnt_n = 0;                                       // the FFN gate / up pairs (zeroed when created or
                                                               // grown; each call leaves every counter it used at 0)
    // Device ranges written by no-wait calls that may still be queued, each with an event recorded right after the
    // call that wrote it (an entry whose event has completed is dropped); a kernel that reads an input before
    // griddepcontrol.wait checks its input against them.
    static constexpr int kQueuedRanges = 32;
    uintptr_t queued_lo[kQueuedRanges] = {}, queued_hi[kQueuedRanges] = {};
    cudaEvent_t queued_ev[kQueuedRanges] = {};
    int queued_n = 0;
    bool queued_overflow = false;
    void *shard = nullptr;                                     // operand copies of a column-sharded GEMM (grow-only)
    size_t shard_n = 0;
    void *ml = nullptr;                                        // FP16 activations / results of the ML entry points
    size_t ml_n = 0;                                           // (grow-only, apart from the GEMM scratch they feed)
    static constexpr int kNowaitSlots = 4096;                  // overflow flags of queued ML calls (mapped pinned words),
    unsigned *nw_host = nullptr, *nw_dev = nullptr;            // one per call until gen9blas_nowait_pending
    int nw_used = 0;
};

// Process-wide call state (the caller serialises calls, as for the reference).
struct CallState {
    int status = 0;
    char err[1200] = {0};
    double last_ms = 0;
    int last_zc = 0;
    bool profile = false;
    bool nowait = false;
    cudaStream_t user_stream = nullptr;
    bool user_stream_set = false;
    int cur_dev = -1;
    long long launches = 0;
};
extern CallState G;

// Current device state; initialises it on first use. nullptr on failure (status set).
DevState *dev_state();
// The state of device dev if an earlier call has set it up, else nullptr; creates nothing (no stream, no buffer).
DevState *dev_state_if_ready(int dev);
cudaStream_t stream();

int fail(int code, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
int cuda_fail(cudaError_t e, const char *what, const char *file, int line);
#define G9_CU(x)                                                                  \
    do {                                                                          \
        cudaError_t e_ = (x);                                                     \
        if (e_ != cudaSuccess) return ::g9::cuda_fail(e_, #x, __FILE__, __LINE__); \
    } while (0)
#define G9_FAIL(code, ...) return ::g9::fail((code), __VA_ARGS__)
#define G9_TRY(x)            \
    do {                     \
        int r_ = (x);        \
        if (r_ < 0) return r_; \
    } while (0)

// Starts an operation: resets the status, initialises the library and the device. Returns 0 or an error.
int begin_op();
// Records one kernel launch (checks the launch error).
int launched(const char *name);

// One operand of a call: a region [host, host + bytes) the caller passed and the pointer the kernels use.
struct Operand {
    const void *user = nullptr;   // caller's pointer (lowest address of the region)
    void *dptr = nullptr;         // pointer for the kernels (user itself when zero-copy)
    size_t bytes = 0;
    bool zc = true;               // used in place (device or managed memory)
    bool written = false;         // copied back at the end when staged
    // strided vector (|inc| > 1): copied back element by element (rows elements of width bytes, pitch apart), so
    // that the bytes between its elements -- possibly another operand's, e.g. swap(x[0::2], x[1::2]) -- are not
    // rewritten with their staged values
    size_t pitch = 0, width = 0, rows = 0;
};
// Maps an operand: device / managed memory in place, any other memory staged into slot (copy_in: with its contents).
int map_operand(Operand &op, const void *p, size_t bytes, int slot, bool copy_in, bool written);
// Ends a call: waits for the stream (unless no-wait applies), copies staged written operands back, checks the
// device error word. ops may be empty.
int finish_op(Operand *ops, int n);
// Ledger of the outputs of queued no-wait calls (see DevState::queued_lo): add a range, forget them all once the
// library's stream has been waited for, and ask whether [p, p + bytes) may still be written by queued work (true also
// when more ranges were queued than the ledger holds).
void queued_writes_add(DevState *d, const void *p, size_t bytes, cudaStream_t st);
void queued_writes_clear(DevState *d);
bool queued_writes_overlap(DevState *d, const void *p, size_t bytes);
// Hand-over flags of the GEMM kernels that split tiles over CTAs (kGemmFlags zeroed words, created on first use) and
// the epoch of the launch about to be enqueued (never 0).
constexpr int kGemmFlags = 4096;
int gemm_handoff(DevState *d, cudaStream_t st, unsigned **flags, unsigned *epoch);
// Work buffer of the ML entry points on the current device (grow-only, separate from the GEMM scratch).
int ml_buffer(size_t bytes, void **p);
// A flag word for one queued ML call (no-wait mode): its device address, or nullptr when all slots are taken (the
// call then waits and reports through its own flag).
unsigned *nowait_slot(DevState *d);
// Turns the device error word of d (set by bounded device-side waits that gave up) into a status; clears it.
int check_dev_err(DevState *d);
// Grow-only device buffer of the current device (waits for the library's stream before it grows).
int ensure_buffer(void **p, size_t *n, size_t bytes);
// Column-sharded GEMM over the devices set with gen9blas_set_devices / GEN9BLAS_DEVICES: returns 1 when the call does
// not qualify (fewer than two devices, batched, skinny or below the size threshold), else 0 or a negative status.
int gemm_sharded(int type, int tA, int tB, int M, int N, int K, double alpha, const void *A, int lda, const void *B,
                 int ldb, double beta, void *C, int ldc);
// Scratch buffer of at least `bytes` on the current device (grow-only). Waits for queued work before growing.
int scratch(size_t bytes, void **p);
// Device buffer of staging slot `slot` (the one map_operand uses for host operands), at least `bytes` (grow-only).
int stage_buffer(int slot, size_t bytes, void **p);
// The copy streams and band events of the host-operand GEMM pipeline (created on first use).
int pipeline_streams(DevState *d);
// Triangular solve op(A)·X = alpha·B (left) or X·op(A) = alpha·B (right) on device pointers (level-3 TRSM; B is
// overwritten). Uses the level-3 work buffer and the GEMM scratch.
int launch_trsm_dev(int type, int left, int upper, int tA, int unit, int M, int N, double alpha, const void *A, int lda,
                    void *B, int ldb, cudaStream_t st);
// Partial-tile words of the stream-K skinny kernel (at least `words`, zeroed when created or grown) and the epoch of
// the launch about to be enqueued (never 0; the words are zeroed again when the counter wraps).
int skinny_slots(size_t words, uint64_t **p, unsigned *epoch);
// n zero-initialised arrival counters (attention rows, FFN gate / up pairs); each call returns every counter it uses
// to 0, and calls on one stream run in order, so the kernels of successive calls share them.
int arrival_counters(size_t n, unsigned **p);
// Call timing: timer_start at entry (wall clock), timer_kernel right before the main kernels (GEN9BLAS_PROFILE=1:
// CUDA event), timer_stop at the end: last_time_ms is the kernel time with profiling, else the whole call.
void timer_start();
void timer_kernel();
void timer_stop();

// cuTensorMapEncodeTiled from the driver (resolved once through cudaGetDriverEntryPoint).
void *tensor_map_encoder();

// Elements of a strided vector region and offset of element 0 (inc < 0: pointer is the lowest address).
// Marks a staged vector of n elements with increment inc for an element-wise copy back (see Operand).
inline void vec_strided(Operand &op, int n, int inc, size_t es) {
    const size_t a = (size_t)(inc < 0 ? -(long long)inc : inc);
    if (!op.zc && a > 1 && n > 1) {
        op.pitch = a * es;
        op.width = es;
        op.rows = (size_t)n;
    }
}
inline size_t vec_span(int n, int inc) { return (size_t)(n - 1) * (size_t)(inc < 0 ? -(long long)inc : inc) + 1; }
inline long long vec_off(int n, int inc) { return inc < 0 ? (long long)(n - 1) * (long long)(-inc) : 0; }

// ---- kernel entry points implemented in the other translation units (host-side launchers) ----
// All pointers are device-addressable; they enqueue on `st` and return 0 or a negative status.
int launch_axpy(int type, int n, double a, const void *x, long long ox, long long ix, void *y, long long oy, long long iy,
                cudaStream_t st);
int launch_reduce(int type, int mode, int n, const void *x, long long ox, long long ix, const void *y, long long oy,
                  long long iy, double *result_dev, cudaStream_t st);
int launch_iamax(int type, int n, const void *x, long long ox, long long ix, long long *result_dev, cudaStream_t st);
int launch_gemv(int type, int trans, int M, int N, double alpha, const void *A, int lda, const void *x, long long ox,
                long long ix, double beta, void *y, long long oy, long long iy, cudaStream_t st);
int launch_ger(int type, int M, int N, double alpha, const void *x, long long ox, long long ix, const void *y,
               long long oy, long long iy, void *A, int lda, cudaStream_t st);
// Dense GEMM on device pointers (batched, strided). Dispatches to tcgen05 (H/HS), FFMA (S) or FP64 (D) kernels.
int launch_gemm(int type, int tA, int tB, int M, int N, int K, double alpha, const void *A, int lda, long long sA,
                const void *B, int ldb, long long sB, double beta, void *C, int ldc, long long sC, int count,
                cudaStream_t st);
// Skinny GEMM (min(M, N) small) on device pointers.
int launch_skinny(int type, int tA, int tB, int M, int N, int K, double alpha, const void *A, int lda, const void *B,
                  int ldb, double beta, void *C, int ldc, cudaStream_t st, void *const *peers = nullptr, int npeers = 0,
                  long long col_off = 0);
int skinny_threshold(int type);
// Skinny GEMM with FP32 activations and FP16 weights (gemm_pb_skinny): C (M × N, FP32) = A (M × K, FP32) · Wᵀ with W
// N rows of ldw FP16 elements (ldw >= K rounded up to 8, zero past K, rows 16-byte aligned). A non-finite result sets
// *nf (device-visible word).
// gemm_pb_f16w's product in one kernel when its shape takes the one-row-block-per-CTA skinny kernel (M <= 16, N at
// least 16 rows per SM, K >= 2048 and a multiple of 8, 16-byte aligned rows): activations (F32, or FP16 with ahalf)
// rounded to FP16, FP32 sums rounded to FP16, then bias / GELU / residual, F32 C; *nf set on a non-finite FP16 result.
// Returns 1 (nothing enqueued) when the shape does not qualify.
int launch_skinny_swiglu(int M, const void *X, bool xhalf, long long ldx, const void *Wg, const void *Wu, int K, int N,
                         long long ldw, __half *g16, __half *u16, __half *h16, long long ldh, unsigned *nf,
                         cudaStream_t st);
// The shapes launch_skinny_f16w takes (M <= 16, at least one 16-row block per SM, K >= 2048 in 8s, aligned weights).
bool skinny_f16w_fits(int M, int K, int N, long long ldw, const void *W);
int launch_skinny_f16w(int M, const void *A, bool ahalf, long long lda, const void *W, int K, int N, long long ldw,
                       float *C, long long ldc, const float *bias, int gelu, const float *R, long long ldr, unsigned *nf,
                       cudaStream_t st);
int launch_skinny_f32a(int M, int N, int K, const float *A, int lda, const void *W, int ldw, float *C, int ldc,
                       unsigned *nf, cudaStream_t st);

// Raises a kernel's dynamic shared-memory limit to `bytes` once per device. The attribute belongs to the current
// device's context, so a process that calls the library on several devices (gen9blas_set_device) sets it on each;
// `done` is the caller's per-kernel array of kMaxDevices flags.
template <typename... KArgs>
inline cudaError_t smem_limit_once(void (*kernel)(KArgs...), int bytes, bool *done) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    if (done[dev]) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) done[dev] = true;
    return e;
}

// Launch with programmatic stream serialization: the kernel may start while the preceding kernel of the stream
// finishes; it must execute griddepcontrol.wait before it touches anything that kernel may write.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace g9

// A GEMM input written by gen9blas_layer_norm_pack: FP16 rows of Kp elements (zero past K), device memory of dev.
struct gen9blas_packed_a {
    unsigned magic;
    int M, K, Kp, dev;
    __half *rows;
    size_t bytes;
};
constexpr unsigned kPackedAMagic = 0x67397061u;
#pragma GCC visibility pop
