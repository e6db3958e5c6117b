"""bench.py -- headline benchmark of the B200 gen9blas hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload auto|hgemm4096|scaleout]

Workloads:
- hgemm4096 (default at N = 1, configs[1]): HGEMM FP16 n = 4096, row-major, A, B iid N(0,1)/sqrt(n), C = A·B with
  FP16 accumulation (GEN9BLAS_H); one step = one gen9blas_gemm call. The FP32-accumulate mode (GEN9BLAS_HS) is timed
  the same way and reported under "modes".
- rows (N = 1, on request): every BASELINE config row measured on its own (SGEMM n = 1024/4096/8192, HGEMM
  n = 1024..8192 fast and accurate, DGEMM n = 3000/4096 column-major all transposes, skinny GEMM for the four weight
  shapes × M = 1..16, level-1 n = 2^28 and level-2 32768² in FP32 and FP64; level 3 on GEMM at n = 4096; packed
  weights: gemm_pb_skinny on the weight shapes, gemm_pb against gemm), one JSON line per case with its
  roofline fraction, the cuBLAS time for GEMM shapes, and the reference's CPU path on a bounded sample per family.
- case (N = 1, on request): one GEMM shape (--case TYPE:M:N:K[:tA:tB]) called back to back on device-resident
  operands -- the workload of the single-kernel ncu captures in profiles/.
- scaleout (default at N > 1, configs[4]): HGEMM n = 32768 with B and C column-sharded over the N ranks, A
  replicated, C all-gathered over NVLink (NCCL); one step = local GEMM of the rank's column block + all-gather +
  re-layout into the row-major C. Strong scaling (total work fixed).
value: whole-job TFLOP/s from CUDA events on the launching stream (max over ranks), inputs resident in HBM, buffer
sets rotated so that the inputs of consecutive steps exceed L2. e2e: the same metric through the public C ABI with
pinned host buffers (host->device copies of A and B and the device->host copy of C inside the timed region).
--impl reference: the reference's own CPU path (its CBLAS layer lib/src/cblas.c in CPU mode over OpenBLAS, built by
oracle/Makefile into oracle/_ref/) on the same config: cblas_sgemm on the FP16 inputs converted to FP32 (OpenBLAS has
no FP16 GEMM), all host threads.
"""
import argparse
import ctypes
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "gen9-gpu-blas_b200")
METRIC = "HGEMM/SGEMM/DGEMM TFLOPS at n=4096/8192; skinny GEMM µs & HBM GB/s at M=1..16"
H, S, HS, D = 0, 1, 2, 3


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=0)
    ap.add_argument("--warmup", type=int, default=0)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="auto", choices=["auto", "hgemm4096", "scaleout", "rows", "case"],
                    help="rows: one JSON line per BASELINE config row (GEMM, skinny, level 1/2), N = 1 only")
    ap.add_argument("--rows", default="C0,C1,C2,C3a,C3b,C3c,L3,L2X,PB,ML",
                    help="rows workload: which config rows to measure (L3: level 3 on GEMM, L2X: rest of levels 1-2, "
                         "PB: packed weights)")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end (host buffer) measurement")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample (profiling runs)")
    ap.add_argument("--gather", default="fused", choices=["fused", "nccl"],
                    help="scale-out exchange: fused GEMM + NVLink stores (default) or NCCL all-gather")
    ap.add_argument("--case", default=None, metavar="TYPE:M:N:K[:tA:tB]",
                    help="workload 'case': one GEMM shape (TYPE h|hs|s|d) called --steps times on device-resident "
                         "operands after --warmup calls; one JSON line (for profiling a single kernel)")
    return ap.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


# --------------------------------------------------------------------------------------------- clocks during the run
class ClockSampler:
    """Clock samples of one GPU while the timed region runs: NVML queries every millisecond from a thread (read-only:
    SM clock, its maximum, the active clock-event reasons), so that short timed regions are sampled too; nvidia-smi
    (100 ms) where NVML is unavailable."""

    # NVML clock-event reason bits (nvml.h: nvmlClocksEventReason*)
    REASON_BITS = (("sw_power_cap", 0x4), ("hw_slowdown", 0x8), ("sw_thermal_slowdown", 0x20),
                   ("hw_thermal_slowdown", 0x40))

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.nvml = None
        self.samples = []
        self.running = False

    def _nvml_loop(self):
        nv, h = self.nvml
        while self.running:
            try:
                self.samples.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM),
                                     nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                                     if hasattr(nv, "nvmlDeviceGetCurrentClocksEventReasons")
                                     else nv.nvmlDeviceGetCurrentClocksThrottleReasons(h)))
            except Exception:
                pass
            time.sleep(0.001)

    def start(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = None
            try:   # the CUDA device's PCI address: NVML indices need not follow CUDA_VISIBLE_DEVICES
                import torch
                pr = torch.cuda.get_device_properties(self.gpu)
                bus = "%08X:%02X:%02X.0" % (pr.pci_domain_id, pr.pci_bus_id, pr.pci_device_id)
                h = nv.nvmlDeviceGetHandleByPciBusId(bus.encode())
            except Exception:
                h = None
            if h is None:
                vis = os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")
                idx = int(vis[self.gpu]) if self.gpu < len(vis) and vis[self.gpu].strip().isdigit() else self.gpu
                h = nv.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            self.nvml = (nv, h)
            self.running = True
            self.thread = threading.Thread(target=self._nvml_loop, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.FIELDS,
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.nvml:
            self.running = False
            self.thread.join(timeout=2)
            nv = self.nvml[0]
            try:
                nv.nvmlShutdown()
            except Exception:
                pass
            mx = self.max_mhz
            sm = [float(c) for c, _ in self.samples]
            reasons = sorted({nm for _, bits in self.samples for nm, b in self.REASON_BITS if bits & b})
            loaded = [v for v in sm if v > 0.3 * mx] or sm
            return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": mx, "reasons": reasons,
                    "samples": len(sm), "source": "nvml"}
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = float(p[2])
            except ValueError:
                continue
            for nm, v in zip(names, p[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        loaded = [v for v in sm if mx and v > 0.3 * mx] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------------------------------------- reference CPU path
def load_reference_cblas():
    """The reference's CBLAS layer in CPU mode (oracle/_ref) over OpenBLAS; None if it was not built here."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import cpu_blas   # the checkers' locator of OpenBLAS (GEN9BLAS_OPENBLAS or a wheel's bundled copy)
    so = os.path.join(ROOT, "oracle", "_ref", "libgen9blas_blas_ref.so")
    openblas = cpu_blas.openblas()
    if not os.path.exists(so) or openblas is None:
        return None, "port"
    os.environ["GEN9BLAS_BLAS"] = "cpu"
    os.environ["GEN9BLAS_BLAS_CPU"] = openblas
    os.environ.setdefault("OPENBLAS_NUM_THREADS", str(os.cpu_count()))
    cpu_blas.preload_openblas_deps()
    L = ctypes.CDLL(so)
    L.cblas_sgemm.argtypes = [ctypes.c_int] * 6 + [ctypes.c_float, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                                   ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_int]
    return L, "reference"


def cpu_sgemm_sample(n, max_seconds=20.0, min_calls=2, max_calls=5):
    """Times cblas_sgemm(RowMajor, n³) of the reference layer on FP32-converted FP16 inputs (the HGEMM stand-in):
    one untimed call, then calls until max_seconds or max_calls. Returns (TFLOP/s best, kind, calls, threads)."""
    L, kind = load_reference_cblas()
    rng = np.random.default_rng(1)
    A = (rng.standard_normal((n, n)) / np.sqrt(n)).astype(np.float16).astype(np.float32)
    B = (rng.standard_normal((n, n)) / np.sqrt(n)).astype(np.float16).astype(np.float32)
    C = np.empty((n, n), np.float32)
    threads = int(os.environ.get("OPENBLAS_NUM_THREADS", os.cpu_count()))
    if L is None:   # oracle port: the naive restatement is too slow for n³, time a row block and scale
        sys.path.insert(0, os.path.join(ROOT, "tests"))
        import abi
        subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "all"], check=True, capture_output=True)
        O = abi.bind(ctypes.CDLL(os.path.join(ROOT, "oracle", "liboracle.so")), "oracle_")
        rows = 16
        t0 = time.perf_counter()
        O.gemm(S, 0, 0, rows, n, n, 1.0, A.ctypes.data, n, B.ctypes.data, n, 0.0, C.ctypes.data, n)
        dt = time.perf_counter() - t0
        return 2.0 * rows * n * n / dt / 1e12, "port", 1, 1, f"{rows} rows of the n={n} product with the scalar oracle"

    def call():
        L.cblas_sgemm(101, 111, 111, n, n, n, 1.0, A.ctypes.data, n, B.ctypes.data, n, 0.0, C.ctypes.data, n)

    call()
    times, t_start = [], time.perf_counter()
    while len(times) < max_calls and (len(times) < min_calls or time.perf_counter() - t_start < max_seconds):
        t0 = time.perf_counter()
        call()
        times.append(time.perf_counter() - t0)
    return (2.0 * n ** 3 / min(times) / 1e12, kind, len(times), threads,
            f"{len(times)} cblas_sgemm calls n={n} (FP32 stand-in for FP16), best of them")


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    n = 4096
    steps = args.steps or 3
    warm = args.warmup or 1
    L, kind = load_reference_cblas()
    rng = np.random.default_rng(1)
    A = (rng.standard_normal((n, n)) / np.sqrt(n)).astype(np.float16).astype(np.float32)
    B = (rng.standard_normal((n, n)) / np.sqrt(n)).astype(np.float16).astype(np.float32)
    C = np.empty((n, n), np.float32)
    threads = int(os.environ.get("OPENBLAS_NUM_THREADS", os.cpu_count()))
    if L is None:
        v, kind, calls, threads, sample = cpu_sgemm_sample(n)
        ms = 2.0 * n ** 3 / (v * 1e12) * 1e3
    else:
        for _ in range(warm):
            L.cblas_sgemm(101, 111, 111, n, n, n, 1.0, A.ctypes.data, n, B.ctypes.data, n, 0.0, C.ctypes.data, n)
        t0 = time.perf_counter()
        for _ in range(steps):
            L.cblas_sgemm(101, 111, 111, n, n, n, 1.0, A.ctypes.data, n, B.ctypes.data, n, 0.0, C.ctypes.data, n)
        ms = (time.perf_counter() - t0) / steps * 1e3
        v = 2.0 * n ** 3 / (ms * 1e-3) / 1e12
        sample = f"{steps} timed cblas_sgemm calls n={n} after {warm} warm-up (FP32 stand-in for FP16)"
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "TFLOP/s", "n_gpus": args.gpus,
            "steps": steps, "warmup": warm, "ms_per_step": round(ms, 3), "higher_is_better": True,
            "scaling": "strong" if args.gpus > 1 else "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "hgemm4096: reference CBLAS layer (lib/src/cblas.c, CPU mode) -> OpenBLAS "
                                   "cblas_sgemm, n=4096 row-major, FP16 N(0,1)/sqrt(n) inputs converted to FP32",
                       "n": n},
            "cpu_baseline": {"value": round(v, 4), "unit": "TFLOP/s", "cores": threads, "kind": kind,
                             "sample": sample},
            "e2e": {"value": round(v, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(line)
    return 0


# --------------------------------------------------------------------------------------------- our path
def load_lib():
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import abi
    path = os.path.join(PKG, "libgen9blas.so")
    if not os.path.exists(path):
        raise SystemExit("libgen9blas.so is not built (run __graft_entry__.build())")
    L = abi.bind(ctypes.CDLL(path), "gen9blas_")
    if L.init() != 0:
        raise SystemExit("gen9blas_init failed: " + L.error().decode())
    return L


def profile_traffic(name):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary (profiles/<name>.txt)."""
    p = os.path.join(ROOT, "profiles", name + ".txt")
    if not os.path.exists(p):
        return None
    m = re.search(r"traffic_bytes_per_launch\s*[=:]\s*([0-9.eE+]+)", open(p).read())
    return float(m.group(1)) if m else None


def measured_peaks():
    """(dense bf16 TF/s burst, the same sustained under the power cap, HBM GB/s, kind) from MEASURED_PEAKS.json, or
    the pool's earlier figures (kind "fallback") where that file is absent."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        burst = d.get("bf16_tflops") or d.get("bf16_tflops_sustained")
        return burst, d.get("bf16_tflops_sustained") or burst, d.get("hbm_gbs"), "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


def tensor_peak(clk):
    """The tensor-core denominator that fits the clocks sampled over the timed region: the burst figure (cuBLAS timed
    alone at full clock) unless the samples show the power cap (sw_power_cap active, or a median SM clock below 97 %
    of the maximum), then the sustained one (cuBLAS looped for seconds under the cap). Returns (peak, note, both)
    where both = {"burst": ..., "sustained": ...} for the line's record."""
    burst, sust, _, kind = measured_peaks()
    capped, why = False, "no power cap in the clock samples"
    if clk:
        mhz, mx = clk.get("sm_mhz"), clk.get("sm_max_mhz")
        if "sw_power_cap" in (clk.get("reasons") or []):
            capped, why = True, "sw_power_cap active during the timed region"
        elif mhz and mx and mhz < 0.97 * mx:
            capped, why = True, f"median SM clock {mhz:.0f} of {mx:.0f} MHz"
    else:
        why = "no clock samples"
    peak = sust if capped else burst
    note = (f"{kind} cuBLAS bf16 dense, {'sustained' if capped else 'burst'} ({why}), "
            f"{'MEASURED_PEAKS.json' if kind == 'measured' else 'fallback figures'}")
    return peak, note, {"burst": burst, "sustained": sust}


def run_ours(args):
    import torch
    rank, world, local = dist_env()
    workload = args.workload if args.workload != "auto" else ("hgemm4096" if world == 1 else "scaleout")
    if workload == "rows":
        if world != 1:
            raise SystemExit("--workload rows runs on one GPU")
        return run_rows(args, torch)
    if workload == "case":
        if world != 1 or not args.case:
            raise SystemExit("--workload case runs on one GPU and needs --case TYPE:M:N:K[:tA:tB]")
        return run_case(args, torch)
    torch.cuda.set_device(local)
    if world > 1:
        sys.path.insert(0, PKG)
        import g9dist   # process group with a finite timeout; failures raise g9dist.CommError with a status
        g9dist.init_comm("nccl", timeout_s=120.0, device_id=torch.device("cuda", local))
    L = load_lib()
    assert L.set_device(local) == 0, L.error()
    stream = torch.cuda.Stream()
    assert L.set_stream(ctypes.c_void_p(stream.cuda_stream)) == 0
    L.set_nowait(1)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
            torch.cuda.synchronize()

    rng = torch.Generator(device="cuda")
    rng.manual_seed(1 + rank)
    if workload == "hgemm4096":
        n = 4096
        steps = args.steps or 4000
        warm = max(args.warmup or 20, 3)
        sets = 4   # 4 × (A, B, C) × 32 MiB = 384 MiB > 126 MB L2: each step reads inputs that are not L2-resident
        A = [torch.randn(n, n, device="cuda", generator=rng).div_(n ** 0.5).half() for _ in range(sets)]
        B = [torch.randn(n, n, device="cuda", generator=rng).div_(n ** 0.5).half() for _ in range(sets)]
        C = [torch.empty(n, n, device="cuda", dtype=torch.float16) for _ in range(sets)]
        flops = 2.0 * n ** 3

        def step(i, kind=H):
            j = i % sets
            r = L.gemm(kind, 0, 0, n, n, n, 1.0, A[j].data_ptr(), n, B[j].data_ptr(), n, 0.0, C[j].data_ptr(), n)
            if r:
                raise RuntimeError(L.error().decode())

        def timed(kind, k, w):
            with torch.cuda.stream(stream):
                for i in range(w):
                    step(i, kind)
                barrier()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                l0 = L.kernel_launches()
                e0.record(stream)
                for i in range(k):
                    step(i, kind)
                e1.record(stream)
                e1.synchronize()
                launches = L.kernel_launches() - l0
                barrier()
            return e0.elapsed_time(e1), launches

        clocks = ClockSampler(local)
        clocks.start()
        ms_total, launches = timed(H, steps, warm)
        clk = clocks.stop()
        ms_hs, _ = timed(HS, max(steps // 2, 1), warm)
        ms_step = ms_total / steps
        value = flops * steps / (ms_total * 1e-3) / 1e12
        value_hs = flops * max(steps // 2, 1) / (ms_hs * 1e-3) / 1e12
        # e2e through the public API with pinned host buffers (library stages H2D, computes, copies C back)
        e2e = None
        if not args.no_e2e:
            hA = A[0].cpu().pin_memory()
            hB = B[0].cpu().pin_memory()
            hC = torch.empty((n, n), dtype=torch.float16).pin_memory()
            L.set_nowait(0)
            e2e_steps = max(min(steps // 20, 100), 5)
            for _ in range(3):
                L.gemm(H, 0, 0, n, n, n, 1.0, hA.data_ptr(), n, hB.data_ptr(), n, 0.0, hC.data_ptr(), n)
            t0 = time.perf_counter()
            for _ in range(e2e_steps):
                r = L.gemm(H, 0, 0, n, n, n, 1.0, hA.data_ptr(), n, hB.data_ptr(), n, 0.0, hC.data_ptr(), n)
                if r:
                    raise RuntimeError(L.error().decode())
            dt = time.perf_counter() - t0
            L.set_nowait(1)
            e2e = {"value": round(flops * e2e_steps / dt / 1e12, 3), "unit": "TFLOP/s",
                   "h2d_bytes_per_step": 2 * n * n * 2, "d2h_bytes_per_step": n * n * 2,
                   "steps": e2e_steps, "path": "gen9blas_gemm(GEN9BLAS_H) on pinned host pointers"}
        peak_t, peak_note, both = tensor_peak(clk)
        traffic = profile_traffic("hgemm_tc2_n4096")
        roof = {"bound": "tensor", "achieved": round(value, 2), "peak": peak_t, "unit": "TFLOP/s",
                "frac": round(value / peak_t, 4), "traffic": traffic, "kernel": "hgemm_tc2_kernel<true, 256> (CTA pair, 256x256 tiles)",
                "algorithmic": f"2*n^3 = {flops:.4g} FLOP per launch, one launch per step",
                "peak_kind": peak_note,
                "frac_of_burst": round(value / both["burst"], 4), "frac_of_sustained": round(value / both["sustained"], 4),
                "timed_region_ms": round(ms_total, 2)}
        cpu = None
        if rank == 0 and world == 1 and not args.no_cpu:
            v, kind, calls, threads, sample = cpu_sgemm_sample(n)
            cpu = {"value": round(v, 4), "unit": "TFLOP/s", "cores": threads, "kind": kind, "sample": sample}
        line = {"metric": METRIC, "value": round(value, 3), "unit": "TFLOP/s", "n_gpus": world, "steps": steps,
                "warmup": warm, "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f16", "data": "synthetic",
                "config": {"workload": "hgemm4096: BASELINE configs[1], HGEMM FP16 n=4096 row-major NN, "
                                       "A,B iid N(0,1)/sqrt(n), C=A*B, FP16 accumulation (GEN9BLAS_H)",
                           "n": n, "l2": "inputs larger than L2: 4 rotating (A,B,C) sets = 384 MiB"},
                "modes": {"fp16_accumulate_tflops": round(value, 3), "fp32_accumulate_tflops": round(value_hs, 3)},
                "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches, "clocks": clk}
    else:
        line = run_scaleout(args, L, torch, stream, barrier, rank, world, local)
    if rank == 0:
        emit(line)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


def run_scaleout(args, L, torch, stream, barrier, rank, world, local):
    """HGEMM n = 32768, B/C column-sharded, A replicated, C all-gathered (NCCL) and re-laid out; plus the
    tensor-parallel skinny GEMM (M = 8, W 32768 × 8192 FP16 row-sharded)."""
    sys.path.insert(0, PKG)
    import g9dist
    n = 32768
    steps = args.steps or 5
    warm = max(args.warmup or 3, 3)
    nb = n // world
    chunks = 4 if world > 1 else 1
    g = torch.Generator(device="cuda")
    g.manual_seed(7)   # same A on every rank
    A = torch.randn(n, n, device="cuda", generator=g, dtype=torch.float16).div_(n ** 0.5)
    g.manual_seed(100 + rank)
    Bs = torch.randn(n, nb, device="cuda", generator=g, dtype=torch.float16).div_(n ** 0.5)   # this rank's columns
    C = torch.empty(n, n, device="cuda", dtype=torch.float16)
    comm = torch.cuda.Stream()
    flops = 2.0 * n * n * n

    def local_gemm(Ap, Bp, Cp):
        g9dist.gemm_local(L.dll, Ap, Bp, Cp)

    fused = args.gather == "fused" and world > 1
    peers = g9dist.PeerView(L.dll, C, rank, world) if fused else None
    bar = g9dist.PeerBarrier(L.dll, rank, world) if fused else None

    def step():
        with torch.cuda.stream(stream):
            if fused:
                g9dist.fused_column_sharded_gemm(L.dll, A, Bs, C, peers, rank, world, barrier=bar)
            else:
                g9dist.column_sharded_gemm(A, Bs, C, rank, world, local_gemm, chunks=chunks, comm_stream=comm)

    def timed(fn, k):
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        l0 = L.kernel_launches()
        e0.record(stream)
        for _ in range(k):
            fn()
        e1.record(stream)
        e1.synchronize()
        launches = L.kernel_launches() - l0
        ms = torch.tensor([e0.elapsed_time(e1)], device="cuda")
        if world > 1:
            torch.distributed.all_reduce(ms, op=torch.distributed.ReduceOp.MAX)
        barrier()
        return float(ms.item()), launches


    # tensor-parallel skinny GEMM (decode): C (8 × 32768) = A · Wᵀ, W rows split over the ranks. Measured before the
    # long dense GEMM, whose power draw leaves the GPUs at capped clocks for a while.
    Nw, Kw, Mw = 32768, 8192, 8
    nr = Nw // world
    Wsh = torch.randn(nr, Kw, device="cuda", generator=g, dtype=torch.float16).mul_(0.02)
    Aw = torch.randn(Mw, Kw, device="cuda", generator=g, dtype=torch.float16)
    Cw = torch.empty(Mw, Nw, device="cuda", dtype=torch.float16)

    def local_skinny(Ap, Wp, Cp):
        r = L.gemm(H, 0, 1, Ap.shape[0], Wp.shape[0], Ap.shape[1], 1.0, Ap.data_ptr(), Ap.stride(0), Wp.data_ptr(),
                   Wp.stride(0), 0.0, Cp.data_ptr(), Cp.stride(0))
        if r:
            raise RuntimeError(L.error().decode())

    pw = g9dist.PeerView(L.dll, Cw, rank, world) if fused else None

    def tp_step():
        with torch.cuda.stream(stream):
            if fused:
                g9dist.fused_row_sharded_skinny(L.dll, Aw, Wsh, Cw, pw, rank, world, barrier=bar)
            else:
                g9dist.row_sharded_skinny(Aw, Wsh, Cw, rank, world, local_skinny)

    for _ in range(5):
        tp_step()
    tp_run = tp_step
    graph = None
    if fused:
        # Decode steps are launch-bound: the fused step (skinny kernel + NVLink barrier, both stream-ordered and free of
        # host synchronisation) is captured once in a CUDA graph and replayed. The barrier's epoch lives on the device.
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream()
        with torch.cuda.graph(graph, stream=cap, capture_error_mode="relaxed"):
            L.set_stream(ctypes.c_void_p(cap.cuda_stream))
            g9dist.fused_row_sharded_skinny(L.dll, Aw, Wsh, Cw, pw, rank, world, barrier=bar)
        L.set_stream(ctypes.c_void_p(stream.cuda_stream))

        def tp_run():
            with torch.cuda.stream(stream):
                graph.replay()

        for _ in range(5):
            tp_run()
    tp_ms, tp_launches = timed(tp_run, 200)
    tp_us = tp_ms * 1e3 / 200

    for _ in range(warm):
        step()
    clocks = ClockSampler(local)
    clocks.start()
    ms_total, launches = timed(step, steps)
    clk = clocks.stop()
    value = flops * steps / (ms_total * 1e-3) / 1e12

    # The same n = 32768 GEMM on one GPU (rank 0, after the timed region; the other ranks wait at the barrier), so
    # that the line carries its own strong-scaling reference: value / (n_gpus * single_gpu_same_workload).
    single = None
    if world > 1:
        if rank == 0:
            Bfull = torch.randn(n, n, device="cuda", generator=g, dtype=torch.float16).div_(n ** 0.5)
            with torch.cuda.stream(stream):
                local_gemm(A, Bfull, C)
                clk1 = ClockSampler(local)
                clk1.start()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for _ in range(2):
                    local_gemm(A, Bfull, C)
                e1.record(stream)
                e1.synchronize()
                c1 = clk1.stop()
            single = {"tflops": round(2 * flops / (e0.elapsed_time(e1) * 1e-3) / 1e12, 2), "calls": 2,
                      "clocks": {k: c1.get(k) for k in ("sm_mhz", "sm_max_mhz", "reasons")},
                      "what": "rank 0 alone: gen9blas_gemm FP16 n=32768 (A . full B) on its GPU, CUDA events"}
            del Bfull
            torch.cuda.empty_cache()
        barrier()

    # e2e through the public path with this rank's inputs in pinned host memory: every step copies A and the rank's
    # B block to the device, runs the sharded GEMM + gather, and reads the rank's block of C back (together the ranks
    # read all of C). Wall clock between barriers, max over ranks.
    e2e = None
    if not args.no_e2e:
        hA = torch.empty((n, n), dtype=torch.float16, pin_memory=True)
        hB = torch.empty((n, nb), dtype=torch.float16, pin_memory=True)
        hC = torch.empty((n, nb), dtype=torch.float16, pin_memory=True)
        hA.copy_(A)
        hB.copy_(Bs)
        e2e_steps = 3

        def e2e_step():
            with torch.cuda.stream(stream):
                A.copy_(hA, non_blocking=True)
                Bs.copy_(hB, non_blocking=True)
            step()
            with torch.cuda.stream(stream):
                hC.copy_(C[:, rank * nb:(rank + 1) * nb], non_blocking=True)
            stream.synchronize()

        e2e_step()
        barrier()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            e2e_step()
        dt = torch.tensor([time.perf_counter() - t0], device="cuda", dtype=torch.float64)
        if world > 1:
            torch.distributed.all_reduce(dt, op=torch.distributed.ReduceOp.MAX)
        barrier()
        e2e = {"value": round(flops * e2e_steps / float(dt.item()) / 1e12, 3), "unit": "TFLOP/s",
               "h2d_bytes_per_step": world * (n * n * 2 + n * nb * 2), "d2h_bytes_per_step": n * n * 2,
               "steps": e2e_steps,
               "path": "per rank: A and B block pinned host -> device, sharded GEMM + gather, C block -> host; "
                       "bytes summed over the ranks"}
        del hA, hB, hC
    if peers is not None:
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        graph = None
        peers.close()
        pw.close()
        bar.close()
    peak_t, peak_note, both = tensor_peak(clk)
    return {"metric": METRIC, "value": round(value, 3), "unit": "TFLOP/s", "n_gpus": world, "steps": steps,
            "warmup": warm, "ms_per_step": round(ms_total / steps, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": "scaleout: BASELINE configs[4], HGEMM FP16 n=32768, A replicated, B/C column-"
                                   f"sharded over {world} GPU(s); " + (
                                       "fused GEMM + all-gather: the epilogue stores every C tile into all ranks' C "
                                       "over NVLink (CUDA IPC), then an NVLink flag barrier per step" if fused else
                                       f"C all-gathered with NCCL in {chunks} chunk(s) overlapped with the GEMM of the "
                                       "next chunk, then re-laid out row-major"),
                       "n": n, "l2": "inputs larger than L2 (A alone 2 GiB)"},
            "roofline": {"bound": "tensor", "achieved": round(value / world, 2), "peak": peak_t, "unit": "TFLOP/s",
                         "frac": round(value / world / peak_t, 4), "traffic": None,
                         "peak_kind": peak_note + "; per GPU, achieved = whole step per GPU including the gather",
                         "frac_of_burst": round(value / world / both["burst"], 4),
                         "frac_of_sustained": round(value / world / both["sustained"], 4)},
            "skinny_tp": {"shape": "C(8x32768) = A(8x8192) * W^T, W 32768x8192 FP16 row-sharded", "us_per_step":
                          round(tp_us, 2), "weight_GBps_per_gpu": round(nr * Kw * 2 / (tp_us * 1e-6) / 1e9, 1),
                          "includes": ("fused: skinny kernel storing its outputs into every rank's C over NVLink + "
                                       "NVLink flag barrier, replayed as one CUDA graph per step" if fused else
                                       "local skinny GEMM + NCCL all-gather of the outputs + re-layout")},
            "single_gpu_same_workload": single,
            "cpu_baseline": None, "e2e": e2e, "gpu_launches": launches, "clocks": clk}


# --------------------------------------------------------------------------------------------- one GEMM shape
def run_case(args, torch):
    """One GEMM shape called back to back on device-resident operands (uniform[-1,1], N(0,1)/sqrt(K) for FP16), timed
    with CUDA events, plus the max elementwise error of 16 sampled rows against FP64: the workload that the
    single-kernel ncu captures in profiles/ run."""
    parts = args.case.split(":")
    kind = {"h": H, "hs": HS, "s": S, "d": D}[parts[0].lower()]
    M, N, K = (int(v) for v in parts[1:4])
    ta, tb = (int(parts[4]), int(parts[5])) if len(parts) >= 6 else (0, 0)
    dt = {H: torch.float16, HS: torch.float16, S: torch.float32, D: torch.float64}[kind]
    L = load_lib()
    g = torch.Generator(device="cuda").manual_seed(1)
    def mk(r, c):
        if dt == torch.float16:
            return torch.randn(r, c, device="cuda", generator=g, dtype=torch.float32).div_(K ** 0.5).to(dt)
        return torch.rand(r, c, device="cuda", generator=g, dtype=dt).mul_(2).sub_(1)
    A = mk(K, M) if ta else mk(M, K)
    B = mk(N, K) if tb else mk(K, N)
    C = torch.empty(M, N, device="cuda", dtype=dt)
    stream = torch.cuda.Stream()
    assert L.set_stream(ctypes.c_void_p(stream.cuda_stream)) == 0
    L.set_nowait(1)

    def call():
        r = L.gemm(kind, ta, tb, M, N, K, 1.0, A.data_ptr(), A.shape[1], B.data_ptr(), B.shape[1], 0.0, C.data_ptr(), N)
        if r:
            raise RuntimeError(L.error().decode())

    steps, warm = args.steps or 5, max(args.warmup or 3, 1)
    with torch.cuda.stream(stream):
        for _ in range(warm):
            call()
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            call()
        e1.record(stream)
        e1.synchronize()
    ms = e0.elapsed_time(e1) / steps
    rows = torch.randperm(M, generator=torch.Generator().manual_seed(2))[:16].tolist()
    a64 = (A.t() if ta else A).double()[rows]
    b64 = (B.t() if tb else B).double()
    err = float(((C.double()[rows] - a64 @ b64).abs() / (a64.abs() @ b64.abs())).max())
    emit({"workload": "case", "case": args.case, "ms_per_call": round(ms, 5),
          "tflops": round(2.0 * M * N * K / (ms * 1e-3) / 1e12, 2), "max_err_sampled_rows": err, "calls": steps})
    return 0


# --------------------------------------------------------------------------------------------- per-row measurements
CBLAS_ROW, CBLAS_COL, CBLAS_N, CBLAS_T = 101, 102, 111, 112


def cpu_row_samples():
    """The reference's CPU path (oracle/_ref: lib/src/cblas.c in CPU mode over OpenBLAS, all host threads) on bounded
    samples, one per row family: {family: {"value", "unit", "sample"}}. Empty if the reference layer is absent."""
    L, kind = load_reference_cblas()
    if L is None:
        return {}, kind
    f, d, i, vp = ctypes.c_float, ctypes.c_double, ctypes.c_int, ctypes.c_void_p
    L.cblas_dgemm.argtypes = [i] * 6 + [d, vp, i, vp, i, d, vp, i]
    L.cblas_saxpy.argtypes = [i, f, vp, i, vp, i]
    L.cblas_sdot.argtypes = [i, vp, i, vp, i]
    L.cblas_sdot.restype = f
    L.cblas_snrm2.argtypes = [i, vp, i]
    L.cblas_snrm2.restype = f
    L.cblas_isamax.argtypes = [i, vp, i]
    L.cblas_isamax.restype = ctypes.c_size_t
    L.cblas_sgemv.argtypes = [i, i, i, i, f, vp, i, vp, i, f, vp, i]
    L.cblas_sger.argtypes = [i, i, i, f, vp, i, vp, i, vp, i]
    rng = np.random.default_rng(0)

    def best(fn, reps=3):
        fn()
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return min(ts)

    out = {}
    n = 1024
    A, B, C = (rng.uniform(-1, 1, (n, n)).astype(np.float32) for _ in range(3))
    t = best(lambda: L.cblas_sgemm(CBLAS_ROW, CBLAS_N, CBLAS_N, n, n, n, 1.0, A.ctypes.data, n, B.ctypes.data, n, 0.0,
                                   C.ctypes.data, n), 5)
    out["sgemm"] = {"value": round(2 * n ** 3 / t / 1e12, 4), "unit": "TFLOP/s", "sample": "cblas_sgemm n=1024, best of 5"}
    n = 3000
    A, B, C = (rng.uniform(-1, 1, (n, n)) for _ in range(3))
    t = best(lambda: L.cblas_dgemm(CBLAS_COL, CBLAS_N, CBLAS_N, n, n, n, 1.5, A.ctypes.data, n, B.ctypes.data, n, 0.5,
                                   C.ctypes.data, n), 2)
    out["dgemm"] = {"value": round(2 * n ** 3 / t / 1e12, 4), "unit": "TFLOP/s",
                    "sample": "cblas_dgemm ColMajor NN n=3000 alpha=1.5 beta=0.5, best of 2"}
    N, K, M = 4096, 4096, 8
    W = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    X = rng.normal(0, 1, (M, K)).astype(np.float32)
    Y = np.empty((M, N), np.float32)
    t = best(lambda: L.cblas_sgemm(CBLAS_ROW, CBLAS_N, CBLAS_T, M, N, K, 1.0, X.ctypes.data, K, W.ctypes.data, K, 0.0,
                                   Y.ctypes.data, N), 5)
    out["skinny"] = {"value": round(t * 1e6, 1), "unit": "us", "gbps": round(N * K * 4 / t / 1e9, 1),
                     "sample": "cblas_sgemm RowMajor N,T M=8 N=K=4096 (FP32 stand-in for the FP16 weights), best of 5"}
    n = 1 << 26
    x = rng.uniform(-1, 1, n).astype(np.float32)
    y = rng.uniform(-1, 1, n).astype(np.float32)
    for name, fn, nbytes in (("axpy", lambda: L.cblas_saxpy(n, 0.5, x.ctypes.data, 1, y.ctypes.data, 1), 12 * n),
                             ("dot", lambda: L.cblas_sdot(n, x.ctypes.data, 1, y.ctypes.data, 1), 8 * n),
                             ("nrm2", lambda: L.cblas_snrm2(n, x.ctypes.data, 1), 4 * n),
                             ("iamax", lambda: L.cblas_isamax(n, x.ctypes.data, 1), 4 * n)):
        t = best(fn)
        out[name] = {"value": round(nbytes / t / 1e9, 1), "unit": "GB/s", "sample": f"cblas_s{name} n=2^26 FP32, best of 3"}
    m = 16384
    Am = rng.uniform(-1, 1, (m, m)).astype(np.float32)
    xv = rng.uniform(-1, 1, m).astype(np.float32)
    yv = np.zeros(m, np.float32)
    t = best(lambda: L.cblas_sgemv(CBLAS_ROW, CBLAS_N, m, m, 1.0, Am.ctypes.data, m, xv.ctypes.data, 1, 0.0,
                                   yv.ctypes.data, 1))
    out["gemv"] = {"value": round(m * m * 4 / t / 1e9, 1), "unit": "GB/s", "sample": "cblas_sgemv N 16384^2 FP32, best of 3"}
    t = best(lambda: L.cblas_sger(CBLAS_ROW, m, m, 0.5, xv.ctypes.data, 1, yv.ctypes.data, 1, Am.ctypes.data, m))
    out["ger"] = {"value": round(2 * m * m * 4 / t / 1e9, 1), "unit": "GB/s", "sample": "cblas_sger 16384^2 FP32, best of 3"}
    return out, kind


def run_rows(args, torch):
    """One JSON line per BASELINE config row on one GPU (see the module docstring)."""
    os.environ["GEN9BLAS_PROFILE"] = "1"        # gen9blas_last_time_ms = device time of the last call
    L = load_lib()
    stream = torch.cuda.Stream()
    assert L.set_stream(ctypes.c_void_p(stream.cuda_stream)) == 0
    _, _, peak_hbm, peak_kind = measured_peaks()
    mhz_max = 1965.0
    peak_ffma = 148 * 128 * 2 * mhz_max * 1e6 / 1e12
    peak_dmma = 148 * 64 * 2 * mhz_max * 1e6 / 1e12
    g = torch.Generator(device="cuda")
    g.manual_seed(1)
    cpu, cpu_kind = ({}, None) if args.no_cpu else cpu_row_samples()
    rows = []
    want = set(args.rows.split(","))

    def queued_ms(call, reps, warm=3):
        """Device time per call of `reps` calls enqueued back to back behind a sleep kernel (so that host-side call
        overhead does not leave gaps between kernels); CUDA events on the library's stream."""
        L.set_nowait(1)
        with torch.cuda.stream(stream):
            for i in range(warm):
                call(i)
            torch.cuda.synchronize()
            torch.cuda._sleep(int(2e6 + reps * 30e3))
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for i in range(reps):
                call(i)
            e1.record(stream)
            e1.synchronize()
        return e0.elapsed_time(e1) / reps

    def synced_ms(call, reps):
        """Median device time of calls that return a host result (reductions): gen9blas_last_time_ms."""
        L.set_nowait(0)
        call(0)
        ts = []
        for i in range(reps):
            call(i)
            ts.append(L.last_time_ms())
        return statistics.median(ts)

    def chk(r):
        if r:
            raise RuntimeError(L.error().decode())

    def emit_row(row, case, value, unit, ms, bound, achieved, peak, peak_unit, peak_note, extra=None, cpu_key=None):
        line = {"row": row, "case": case, "value": round(value, 3), "unit": unit, "us": round(ms * 1e3, 2),
                "roofline": {"bound": bound, "achieved": round(achieved, 2), "peak": round(peak, 1), "unit": peak_unit,
                             "frac": round(achieved / peak, 4), "peak_kind": peak_note}}
        if extra:
            line.update(extra)
        if cpu_key and cpu_key in cpu:
            line["cpu_baseline"] = dict(cpu[cpu_key], kind=cpu_kind, cores=os.cpu_count())
        rows.append(line)
        emit(line)

    def gemm_rows(row, kind, dt, n, ta=0, tb=0, colmajor=False, alpha=1.0, beta=0.0, sets=None, label="", cpu_key=None):
        es = torch.tensor([], dtype=dt).element_size()
        sets = sets or (4 if 12 * n * n * es < 2e9 else 2)
        mk = (lambda: torch.randn(n, n, device="cuda", generator=g, dtype=torch.float32).div_(n ** 0.5).to(dt)) \
            if dt == torch.float16 else (lambda: torch.rand(n, n, device="cuda", generator=g, dtype=dt).mul_(2).sub_(1))
        A = [mk() for _ in range(sets)]
        B = [mk() for _ in range(sets)]
        C = [mk() for _ in range(sets)]

        def call(i):
            j = i % sets
            if colmajor:   # column-major C = op(A)·op(B) is row-major Cᵀ = op(B)ᵀ·op(A)ᵀ (the CBLAS swap identity)
                chk(L.gemm(kind, tb, ta, n, n, n, alpha, B[j].data_ptr(), n, A[j].data_ptr(), n, beta, C[j].data_ptr(), n))
            else:
                chk(L.gemm(kind, ta, tb, n, n, n, alpha, A[j].data_ptr(), n, B[j].data_ptr(), n, beta, C[j].data_ptr(), n))

        reps = max(4, min(200, int(0.25 / (2 * n ** 3 / 50e12))))
        clocks = ClockSampler(torch.cuda.current_device())
        clocks.start()
        ms = queued_ms(call, reps)
        clk = clocks.stop()
        # cuBLAS on the same operands (torch.matmul / addmm), TF32 off
        torch.backends.cuda.matmul.allow_tf32 = False
        with torch.cuda.stream(stream):
            opA = (lambda j: A[j].t()) if ta else (lambda j: A[j])
            opB = (lambda j: B[j].t()) if tb else (lambda j: B[j])
            for j in range(2):
                torch.matmul(opA(j % sets), opB(j % sets), out=C[j % sets])
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for i in range(reps):
                torch.matmul(opA(i % sets), opB(i % sets), out=C[i % sets])
            e1.record(stream)
            e1.synchronize()
        ms_cublas = e0.elapsed_time(e1) / reps
        tf = 2 * n ** 3 / (ms * 1e-3) / 1e12
        peak, note = {torch.float16: tensor_peak(clk)[:2],
                      torch.float32: (peak_ffma, "FP32 FFMA nominal: 148 SMs x 128 lanes x 2 x 1965 MHz"),
                      torch.float64: (peak_dmma, "FP64 DMMA nominal: 148 SMs x 64 FMA/clk x 2 x 1965 MHz")}[dt]
        emit_row(row, label, tf, "TFLOP/s", ms, "tensor" if dt != torch.float32 else "ffma", tf, peak, "TFLOP/s", note,
                 {"cublas_tflops": round(2 * n ** 3 / (ms_cublas * 1e-3) / 1e12, 2),
                  "clocks": {k: clk.get(k) for k in ("sm_mhz", "sm_max_mhz", "reasons")}}, cpu_key)
        del A, B, C
        torch.cuda.empty_cache()

    for n in (1024, 4096, 8192) if "C0" in want else ():
        gemm_rows("C0", S, torch.float32, n, label=f"sgemm n={n} RM NN", cpu_key="sgemm" if n == 1024 else None)
    for n in (1024, 2048, 3000, 4096, 8192) if "C1" in want else ():
        for kind, nm in ((H, "fast (FP16 accumulate)"), (HS, "accurate (FP32 accumulate)")):
            gemm_rows("C1", kind, torch.float16, n, label=f"hgemm n={n} RM NN {nm}")
    for n in (3000, 4096) if "C3a" in want else ():
        for ta, tb in ((0, 0), (1, 0), (0, 1), (1, 1)):
            gemm_rows("C3a", D, torch.float64, n, ta, tb, colmajor=True, alpha=1.5, beta=0.5,
                      label=f"dgemm n={n} col-major {'NT'[ta]}{'NT'[tb]} alpha=1.5 beta=0.5",
                      cpu_key="dgemm" if (n, ta, tb) == (3000, 0, 0) else None)

    # skinny: C (M × N) = A (M × K) · Wᵀ, W resident in HBM, rotated over copies that exceed L2
    for N, K in ((4096, 4096), (12288, 4096), (11008, 4096), (4096, 11008)) if "C2" in want else ():
        copies = max(2, int(512e6 // (N * K * 2)) + 1)
        Ws = [torch.randn(N, K, device="cuda", generator=g, dtype=torch.float32).mul_(0.02).half() for _ in range(copies)]
        for M in (1, 2, 4, 8, 16):
            X = torch.randn(M, K, device="cuda", generator=g, dtype=torch.float32).half()
            Y = torch.empty(M, N, device="cuda", dtype=torch.float16)

            def call(i, M=M, X=X, Y=Y):
                chk(L.gemm(H, 0, 1, M, N, K, 1.0, X.data_ptr(), K, Ws[i % copies].data_ptr(), K, 0.0, Y.data_ptr(), N))

            ms = queued_ms(call, 200)
            with torch.cuda.stream(stream):
                for i in range(3):
                    torch.matmul(X, Ws[i % copies].t(), out=Y)
                torch.cuda._sleep(int(2e6 + 200 * 30e3))
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for i in range(200):
                    torch.matmul(X, Ws[i % copies].t(), out=Y)
                e1.record(stream)
                e1.synchronize()
            ms_cublas = e0.elapsed_time(e1) / 200
            nbytes = N * K * 2 + M * K * 2 + M * N * 2
            gbps = nbytes / (ms * 1e-3) / 1e9
            emit_row("C2", f"skinny M={M} W={N}x{K}", ms * 1e3, "us", ms, "hbm", gbps, peak_hbm, "GB/s",
                     f"{peak_kind} HBM copy, MEASURED_PEAKS.json",
                     {"gbps": round(gbps, 1), "cublas_us": round(ms_cublas * 1e3, 2),
                      },
                     "skinny" if (N, K, M) == (4096, 4096, 8) else None)
        del Ws
        torch.cuda.empty_cache()

    # level 1 (n = 2^28) and level 2 (32768²), FP32 and FP64
    n1 = 1 << 28
    for kind, dt, tag in ((S, torch.float32, "s"), (D, torch.float64, "d")) if want & {"C3b", "C3c"} else ():
        es = 4 if kind == S else 8
        x = torch.rand(n1, device="cuda", generator=g, dtype=dt).mul_(2).sub_(1)
        y = torch.rand(n1, device="cuda", generator=g, dtype=dt).mul_(2).sub_(1)
        res = ctypes.c_double()
        ires = ctypes.c_int64()
        ms = queued_ms(lambda i: chk(L.axpy(kind, n1, 0.5, x.data_ptr(), 1, y.data_ptr(), 1)), 10)
        emit_row("C3b", f"{tag}axpy n=2^28", 3 * n1 * es / (ms * 1e-3) / 1e9, "GB/s", ms, "hbm",
                 3 * n1 * es / (ms * 1e-3) / 1e9, peak_hbm, "GB/s", f"{peak_kind} HBM copy", None,
                 "axpy" if kind == S else None)
        for nm, fn, nb in (("dot", lambda i: chk(L.dot(kind, n1, x.data_ptr(), 1, y.data_ptr(), 1, ctypes.byref(res))), 2),
                           ("nrm2", lambda i: chk(L.nrm2(kind, n1, x.data_ptr(), 1, ctypes.byref(res))), 1),
                           ("asum", lambda i: chk(L.asum(kind, n1, x.data_ptr(), 1, ctypes.byref(res))), 1),
                           ("iamax", lambda i: chk(L.iamax(kind, n1, x.data_ptr(), 1, ctypes.byref(ires))), 1)):
            ms = synced_ms(fn, 10)
            gbps = nb * n1 * es / (ms * 1e-3) / 1e9
            emit_row("C3b", f"{tag}{nm} n=2^28", gbps, "GB/s", ms, "hbm", gbps, peak_hbm, "GB/s",
                     f"{peak_kind} HBM copy; time = gen9blas_last_time_ms (includes the 8-byte result copy)", None,
                     nm if kind == S and nm in ("dot", "nrm2", "iamax") else None)
        del x, y
        torch.cuda.empty_cache()
        m = 32768
        A = torch.rand(m, m, device="cuda", generator=g, dtype=dt).mul_(2).sub_(1)
        xv = torch.rand(m, device="cuda", generator=g, dtype=dt)
        yv = torch.rand(m, device="cuda", generator=g, dtype=dt)
        for trans in (0, 1):
            ms = queued_ms(lambda i: chk(L.gemv(kind, trans, m, m, 1.0, A.data_ptr(), m, xv.data_ptr(), 1, 0.0,
                                                yv.data_ptr(), 1)), 10)
            gbps = (m * m + 2 * m) * es / (ms * 1e-3) / 1e9
            emit_row("C3c", f"{tag}gemv {'NT'[trans]} 32768^2", gbps, "GB/s", ms, "hbm", gbps, peak_hbm, "GB/s",
                     f"{peak_kind} HBM copy", None, "gemv" if kind == S and trans == 0 else None)
        ms = queued_ms(lambda i: chk(L.ger(kind, m, m, 1e-3, xv.data_ptr(), 1, yv.data_ptr(), 1, A.data_ptr(), m)), 10)
        gbps = 2 * m * m * es / (ms * 1e-3) / 1e9
        emit_row("C3c", f"{tag}ger 32768^2", gbps, "GB/s", ms, "hbm", gbps, peak_hbm, "GB/s", f"{peak_kind} HBM copy",
                 None, "ger" if kind == S else None)
        del A, xv, yv
        torch.cuda.empty_cache()

    # constant weights (packed once): gemm_pb_skinny (F32 activations x FP16 weights) on the decoder shapes, and
    # gemm_pb against gemm on the same operands for large M
    if "PB" in want:
        pb_sigs = {"pack_b": ([ctypes.c_int] * 4 + [ctypes.c_void_p, ctypes.c_int], ctypes.c_void_p),
                   "packed_b_free": ([ctypes.c_void_p], None),
                   "gemm_pb": ([ctypes.c_int, ctypes.c_int, ctypes.c_double, ctypes.c_void_p, ctypes.c_int,
                                ctypes.c_void_p, ctypes.c_double, ctypes.c_void_p, ctypes.c_int], ctypes.c_int),
                   "gemm_pb_skinny": ([ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.c_int, ctypes.c_void_p], ctypes.c_int)}
        for nm, (a_t, r_t) in pb_sigs.items():
            getattr(L.dll, "gen9blas_" + nm).argtypes, getattr(L.dll, "gen9blas_" + nm).restype = a_t, r_t
        for N, K in ((4096, 4096), (12288, 4096), (11008, 4096), (4096, 11008)):
            copies = max(2, int(512e6 // (N * K * 2)) + 1)
            Ps = []
            for _ in range(copies):
                W = torch.randn(N, K, device="cuda", generator=g, dtype=torch.float32).mul_(0.02).half()
                Ps.append(L.dll.gen9blas_pack_b(HS, 1, K, N, W.data_ptr(), K))
                assert Ps[-1], L.error().decode()
                del W
            for M in (1, 4, 8, 16):
                X = torch.randn(M, K, device="cuda", generator=g, dtype=torch.float32)
                Y = torch.empty(M, N, device="cuda", dtype=torch.float32)

                def call(i, M=M, X=X, Y=Y):
                    chk(L.dll.gen9blas_gemm_pb_skinny(M, X.data_ptr(), K, Ps[i % copies], Y.data_ptr(), N, None))

                ms = queued_ms(call, 200)
                nbytes = N * K * 2 + M * K * 4 + M * N * 4
                gbps = nbytes / (ms * 1e-3) / 1e9
                emit_row("PB", f"gemm_pb_skinny M={M} W={N}x{K} (F32 x FP16)", ms * 1e3, "us", ms, "hbm", gbps,
                         peak_hbm, "GB/s", f"{peak_kind} HBM copy, MEASURED_PEAKS.json", {"gbps": round(gbps, 1)})
            for P in Ps:
                L.dll.gen9blas_packed_b_free(P)
        for kind, dt, M, N, K in ((HS, torch.float16, 4096, 4096, 4096), (H, torch.float16, 4096, 4096, 4096),
                                  (S, torch.float32, 512, 8960, 1536)):
            A = torch.rand(M, K, device="cuda", generator=g, dtype=torch.float32).sub_(0.5).to(dt)
            Wt = torch.rand(N, K, device="cuda", generator=g, dtype=torch.float32).sub_(0.5).to(dt)
            Cm = torch.empty(M, N, device="cuda", dtype=dt)
            P = L.dll.gen9blas_pack_b(kind, 1, K, N, Wt.data_ptr(), K)
            assert P, L.error().decode()
            reps = max(4, min(200, int(0.25 / (2 * M * N * K / 50e12))))
            clocks = ClockSampler(torch.cuda.current_device())
            clocks.start()
            ms = queued_ms(lambda i: chk(L.dll.gen9blas_gemm_pb(0, M, 1.0, A.data_ptr(), K, P, 0.0, Cm.data_ptr(), N)),
                           reps)
            clk = clocks.stop()
            ms_g = queued_ms(lambda i: chk(L.gemm(kind, 0, 1, M, N, K, 1.0, A.data_ptr(), K, Wt.data_ptr(), K, 0.0,
                                                  Cm.data_ptr(), N)), reps)
            tf = 2 * M * N * K / (ms * 1e-3) / 1e12
            peak, note = (tensor_peak(clk)[:2] if dt == torch.float16
                          else (peak_ffma, "FP32 FFMA nominal: 148 SMs x 128 lanes x 2 x 1965 MHz"))
            tag = {H: "h", HS: "hs", S: "s"}[kind]
            emit_row("PB", f"gemm_pb {tag} {M}x{N}x{K}", tf, "TFLOP/s", ms, "tensor" if dt == torch.float16 else "ffma",
                     tf, peak, "TFLOP/s", note, {"gemm_same_operands_tflops": round(2 * M * N * K / (ms_g * 1e-3) / 1e12, 2)})
            L.dll.gen9blas_packed_b_free(P)
            del A, Wt, Cm
        torch.cuda.empty_cache()

    # ML operations of gen9blas_ml.h on decode / prefill shapes, device-resident operands, queued (sync = 0 or no-wait
    # mode). Every case here is bound by HBM at these sizes: the roofline is algorithmic bytes against the copy rate.
    if "ML" in want:
        def hbm_row(case, ms, nbytes, extra=None):
            gbps = nbytes / (ms * 1e-3) / 1e9
            emit_row("ML", case, ms * 1e3, "us", ms, "hbm", gbps, peak_hbm, "GB/s",
                     f"{peak_kind} HBM copy, MEASURED_PEAKS.json", dict({"gbps": round(gbps, 1)}, **(extra or {})))

        def packed(n, k):
            W = torch.randn(n, k, device="cuda", generator=g).mul_(0.02).half()
            torch.cuda.synchronize()   # the weights exist before the library's stream copies them
            P = L.pack_b(HS, 1, k, n, W.data_ptr(), k)
            assert P, L.error().decode()
            return P

        nfp = ctypes.c_int(0)
        for N, K in ((4096, 4096), (11008, 4096)):
            copies = max(2, int(512e6 // (N * K * 2)) + 1)
            Ps = [packed(N, K) for _ in range(copies)]
            for M in (1, 16, 64):
                X = torch.randn(M, K, device="cuda", generator=g, dtype=torch.float32)
                Y = torch.empty(M, N, device="cuda", dtype=torch.float32)
                ms = queued_ms(lambda i, X=X, Y=Y, M=M: chk(L.gemm_pb_f16w(M, X.data_ptr(), K, Ps[i % copies],
                                                                          Y.data_ptr(), N, ctypes.addressof(nfp))), 200)
                L.flush()
                L.nowait_pending()
                hbm_row(f"gemm_pb_f16w M={M} W={N}x{K} (F32 act -> FP16, FP16 weights)", ms,
                        N * K * 2 + M * K * 4 + M * N * 4)
            for P in Ps:
                L.packed_b_free(P)
        # gated FFN of a 7B layer: gate and up 4096 -> 11008, down 11008 -> 4096
        Pg = [packed(11008, 4096) for _ in range(2)]
        Pu = [packed(11008, 4096) for _ in range(2)]
        Pd = [packed(4096, 11008) for _ in range(2)]
        for M in (1, 16):
            X = torch.randn(M, 4096, device="cuda", generator=g, dtype=torch.float32)
            Y = torch.empty(M, 4096, device="cuda", dtype=torch.float32)
            ms = queued_ms(lambda i, X=X, Y=Y, M=M: chk(L.ffn_f16w(M, X.data_ptr(), 4096, Pg[i % 2], Pu[i % 2],
                                                                  Pd[i % 2], Y.data_ptr(), 4096,
                                                                  ctypes.addressof(nfp))), 100)
            L.flush()
            L.nowait_pending()
            hbm_row(f"ffn_f16w M={M} 4096->11008->4096 (two weight sets)", ms, 3 * 11008 * 4096 * 2 + M * 4096 * 8)
        for P in Pg + Pu + Pd:
            L.packed_b_free(P)
        # row / element operations at prefill size
        R, Kr = 8192, 4096
        Xs = [torch.randn(R, Kr, device="cuda", generator=g) for _ in range(2)]
        Ys = [torch.empty(R, Kr, device="cuda") for _ in range(2)]
        w = torch.randn(Kr, device="cuda", generator=g)
        ms = queued_ms(lambda i: chk(L.rms_norm(R, Kr, Xs[i % 2].data_ptr(), Kr, w.data_ptr(), 1e-6,
                                                Ys[i % 2].data_ptr(), Kr, 0)), 50)
        hbm_row(f"rms_norm {R}x{Kr} F32 (with weight)", ms, 2 * R * Kr * 4 + Kr * 4)
        ms = queued_ms(lambda i: chk(L.gelu(R * Kr, Xs[i % 2].data_ptr(), Ys[i % 2].data_ptr(), 0)), 50)
        hbm_row(f"gelu {R * Kr} F32", ms, 2 * R * Kr * 4)
        nt, nh, nd = 8192, 32, 128
        pos = torch.arange(nt, device="cuda", dtype=torch.int32)
        corr = (ctypes.c_float * 2)(0.0, 0.0)
        Xr = Xs[0].view(-1)[:nt * nh * nd]
        ms = queued_ms(lambda i: chk(L.rope(nd, nh, nt, Xr.data_ptr(), nd, nh * nd, Xr.data_ptr(), nd, nh * nd,
                                            pos.data_ptr(), None, 1, 10000.0, 1.0, 0.0, 1.0,
                                            ctypes.addressof(corr), 0)), 50)
        hbm_row(f"rope NEOX {nt} tokens x {nh} heads x {nd} (in place)", ms, 2 * nt * nh * nd * 4 + nt * 4)
        del Xs, Ys
        # decoding attention over a KV cache: 8 streams, one new token each, H 32 / HKV 8, D 128, 4096 keys
        ns, nk, nhq, nhkv, hd = 8, 4096, 32, 8, 128
        Kc = [torch.randn(ns, nk, nhkv, hd, device="cuda", generator=g).half() for _ in range(2)]
        Vc = [torch.randn(ns, nk, nhkv, hd, device="cuda", generator=g).half() for _ in range(2)]
        Q = torch.randn(ns, 1, nhq, hd, device="cuda", generator=g)
        O = torch.empty(ns, 1, nhq, hd, device="cuda")
        vis = torch.full((ns,), nk, device="cuda", dtype=torch.int32)
        kk, kh, ks = nhkv * hd, hd, nk * nhkv * hd
        ms = queued_ms(lambda i: chk(L.attn_dec(hd, nhq, nhkv, ns, 1, nk, Q.data_ptr(), nhq * hd, hd, nhq * hd,
                                                Kc[i % 2].data_ptr(), kk, kh, ks, Kc[0].numel() * 2,
                                                Vc[i % 2].data_ptr(), kk, kh, ks, Vc[0].numel() * 2, O.data_ptr(),
                                                hd ** -0.5, vis.data_ptr(), 0, 256, 0)), 50)
        hbm_row(f"attn_dec {ns} streams x {nk} keys, H {nhq} / HKV {nhkv}, D {hd}", ms, 2 * ns * nk * nhkv * hd * 2)
        del Kc, Vc
        torch.cuda.empty_cache()

    # rest of levels 1-2 (the scope table's next row): level 1 at n = 2^28, level 2 at n = 16384 (dense, band K = 64,
    # packed), FP32 and FP64; each against its algorithmic HBM bytes (the stored elements read and written once)
    if "L2X" in want:
        ci, cd, cp = ctypes.c_int, ctypes.c_double, ctypes.c_void_p
        sigs = {"scal": [ci, ci, cd, cp, ci], "copy": [ci, ci, cp, ci, cp, ci], "swap": [ci, ci, cp, ci, cp, ci],
                "rot": [ci, ci, cp, ci, cp, ci, cd, cd], "symv": [ci, ci, ci, cd, cp, ci, cp, ci, cd, cp, ci],
                "trmv": [ci] * 5 + [cp, ci, cp, ci], "trsv": [ci] * 5 + [cp, ci, cp, ci],
                "syr": [ci, ci, ci, cd, cp, ci, cp, ci], "syr2": [ci, ci, ci, cd, cp, ci, cp, ci, cp, ci],
                "gbmv": [ci] * 6 + [cd, cp, ci, cp, ci, cd, cp, ci], "sbmv": [ci] * 4 + [cd, cp, ci, cp, ci, cd, cp, ci],
                "tbmv": [ci] * 6 + [cp, ci, cp, ci], "tbsv": [ci] * 6 + [cp, ci, cp, ci],
                "spmv": [ci] * 3 + [cd, cp, cp, ci, cd, cp, ci], "tpmv": [ci] * 5 + [cp, cp, ci],
                "tpsv": [ci] * 5 + [cp, cp, ci], "spr": [ci] * 3 + [cd, cp, ci, cp],
                "spr2": [ci] * 3 + [cd, cp, ci, cp, ci, cp]}
        fn = {}
        for nm, a_t in sigs.items():
            f = getattr(L.dll, "gen9blas_" + nm)
            f.argtypes, f.restype = a_t, ctypes.c_int
            fn[nm] = f
        n1 = 1 << 28
        m, kb = 16384, 64
        for kind, dt, tag in ((S, torch.float32, "s"), (D, torch.float64, "d")):
            es = 4 if kind == S else 8
            x = torch.rand(n1, device="cuda", generator=g, dtype=dt)
            y = torch.rand(n1, device="cuda", generator=g, dtype=dt)
            px, py = x.data_ptr(), y.data_ptr()
            for nm, call, nbytes in (
                    ("scal", lambda i: chk(fn["scal"](kind, n1, 0.999, px, 1)), 2 * n1 * es),
                    ("copy", lambda i: chk(fn["copy"](kind, n1, px, 1, py, 1)), 2 * n1 * es),
                    ("swap", lambda i: chk(fn["swap"](kind, n1, px, 1, py, 1)), 4 * n1 * es),
                    ("rot", lambda i: chk(fn["rot"](kind, n1, px, 1, py, 1, 0.6, 0.8)), 4 * n1 * es)):
                ms = queued_ms(call, 10)
                gbps = nbytes / (ms * 1e-3) / 1e9
                emit_row("L2X", f"{tag}{nm} n=2^28", gbps, "GB/s", ms, "hbm", gbps, peak_hbm, "GB/s", f"{peak_kind} HBM copy")
            del x, y
            A = torch.rand(m, m, device="cuda", generator=g, dtype=dt).div_(m)
            A.diagonal().fill_(1.0)
            xv = torch.rand(m, device="cuda", generator=g, dtype=dt)
            yv = torch.rand(m, device="cuda", generator=g, dtype=dt)
            Bd = torch.rand(m, 2 * kb + 1, device="cuda", generator=g, dtype=dt).div_(kb)
            Bd[:, kb] = 1.0    # diagonal of the band (general: column KL; lower symmetric / triangular: column K)
            Bs = Bd[:, kb:].contiguous()   # K + 1 columns, diagonal in column 0 (upper storage)
            npk = m * (m + 1) // 2
            Ap = torch.rand(npk, device="cuda", generator=g, dtype=dt).div_(m)
            pA, pX, pY, pB, pS, pP = A.data_ptr(), xv.data_ptr(), yv.data_ptr(), Bd.data_ptr(), Bs.data_ptr(), Ap.data_ptr()
            tri = m * (m + 1) // 2 * es
            band = m * (2 * kb + 1) * es
            sband = m * (kb + 1) * es
            vec = m * es
            cases = (
                ("symv", lambda i: chk(fn["symv"](kind, 0, m, 1.0, pA, m, pX, 1, 0.0, pY, 1)), tri + 2 * vec),
                ("trmv", lambda i: chk(fn["trmv"](kind, 0, 0, 0, m, pA, m, pX, 1)), tri + 2 * vec),
                ("trsv", lambda i: chk(fn["trsv"](kind, 0, 0, 0, m, pA, m, pX, 1)), tri + 2 * vec),
                ("syr", lambda i: chk(fn["syr"](kind, 0, m, 1e-9, pX, 1, pA, m)), 2 * tri + vec),
                ("syr2", lambda i: chk(fn["syr2"](kind, 0, m, 1e-9, pX, 1, pY, 1, pA, m)), 2 * tri + 2 * vec),
                ("gbmv", lambda i: chk(fn["gbmv"](kind, 0, m, m, kb, kb, 1.0, pB, 2 * kb + 1, pX, 1, 0.0, pY, 1)),
                 band + 2 * vec),
                ("sbmv", lambda i: chk(fn["sbmv"](kind, 1, m, kb, 1.0, pS, kb + 1, pX, 1, 0.0, pY, 1)), sband + 2 * vec),
                ("tbmv", lambda i: chk(fn["tbmv"](kind, 1, 0, 0, m, kb, pS, kb + 1, pX, 1)), sband + 2 * vec),
                ("tbsv", lambda i: chk(fn["tbsv"](kind, 1, 0, 0, m, kb, pS, kb + 1, pX, 1)), sband + 2 * vec),
                ("spmv", lambda i: chk(fn["spmv"](kind, 0, m, 1.0, pP, pX, 1, 0.0, pY, 1)), tri + 2 * vec),
                ("tpmv", lambda i: chk(fn["tpmv"](kind, 0, 0, 0, m, pP, pX, 1)), tri + 2 * vec),
                ("tpsv", lambda i: chk(fn["tpsv"](kind, 0, 0, 0, m, pP, pX, 1)), tri + 2 * vec),
                ("spr", lambda i: chk(fn["spr"](kind, 0, m, 1e-9, pX, 1, pP)), 2 * tri + vec),
                ("spr2", lambda i: chk(fn["spr2"](kind, 0, m, 1e-9, pX, 1, pY, 1, pP)), 2 * tri + 2 * vec))
            for nm, call, nbytes in cases:
                ms = queued_ms(call, 5, warm=1)
                gbps = nbytes / (ms * 1e-3) / 1e9
                shape = f"n={m}" + (f" K={kb}" if nm[1] == "b" else "")
                emit_row("L2X", f"{tag}{nm} {shape}", gbps, "GB/s", ms, "hbm", gbps, peak_hbm, "GB/s",
                         f"{peak_kind} HBM copy; bytes = stored elements read (+ written) once")
            del A, xv, yv, Bd, Bs, Ap
            torch.cuda.empty_cache()

    # level 3 on GEMM (the scope table's next row): n = 4096, FP32 and FP64, left / lower / no transpose
    f = ctypes.c_int, ctypes.c_double, ctypes.c_void_p
    for fn, args_t in (("symm", [f[0]] * 5 + [f[1], f[2], f[0], f[2], f[0], f[1], f[2], f[0]]),
                       ("syrk", [f[0]] * 5 + [f[1], f[2], f[0], f[1], f[2], f[0]]),
                       ("syr2k", [f[0]] * 5 + [f[1], f[2], f[0], f[2], f[0], f[1], f[2], f[0]]),
                       ("trmm", [f[0]] * 7 + [f[1], f[2], f[0], f[2], f[0]]),
                       ("trsm", [f[0]] * 7 + [f[1], f[2], f[0], f[2], f[0]])):
        getattr(L.dll, "gen9blas_" + fn).argtypes = args_t
    n3 = 4096
    for kind, dt, tag in ((S, torch.float32, "s"), (D, torch.float64, "d")) if "L3" in want else ():
        A = torch.rand(n3, n3, device="cuda", generator=g, dtype=dt).mul_(2).sub_(1)
        A.diagonal().add_(float(n3))    # well-conditioned triangle for TRSM
        Bm = torch.rand(n3, n3, device="cuda", generator=g, dtype=dt).mul_(2).sub_(1)
        Cm = torch.zeros(n3, n3, device="cuda", dtype=dt)
        peak, note = ((peak_ffma, "FP32 FFMA nominal: 148 SMs x 128 lanes x 2 x 1965 MHz") if kind == S else
                      (peak_dmma, "FP64 DMMA nominal: 148 SMs x 64 FMA/clk x 2 x 1965 MHz"))
        cases = (("symm", 2.0 * n3 ** 3, lambda i: chk(L.dll.gen9blas_symm(kind, 0, 0, n3, n3, 1.0, A.data_ptr(), n3,
                                                                          Bm.data_ptr(), n3, 0.0, Cm.data_ptr(), n3))),
                 ("syrk", 1.0 * n3 ** 3, lambda i: chk(L.dll.gen9blas_syrk(kind, 0, 0, n3, n3, 1.0, A.data_ptr(), n3, 0.0,
                                                                          Cm.data_ptr(), n3))),
                 ("syr2k", 2.0 * n3 ** 3, lambda i: chk(L.dll.gen9blas_syr2k(kind, 0, 0, n3, n3, 1.0, A.data_ptr(), n3,
                                                                            Bm.data_ptr(), n3, 0.0, Cm.data_ptr(), n3))),
                 ("trmm", 1.0 * n3 ** 3, lambda i: chk(L.dll.gen9blas_trmm(kind, 0, 0, 0, 0, n3, n3, 1.0, A.data_ptr(),
                                                                          n3, Cm.data_ptr(), n3))),
                 ("trsm", 1.0 * n3 ** 3, lambda i: chk(L.dll.gen9blas_trsm(kind, 0, 0, 0, 0, n3, n3, 1.0, A.data_ptr(),
                                                                          n3, Cm.data_ptr(), n3))))
        for nm, fl, call in cases:
            Cm.copy_(Bm)
            ms = queued_ms(call, 5, warm=1)
            tf = fl / (ms * 1e-3) / 1e12
            extra = None
            if nm == "trsm":   # cuBLAS trsm through torch on the same triangle
                Lt = torch.tril(A)
                with torch.cuda.stream(stream):
                    torch.linalg.solve_triangular(Lt, Bm, upper=False)
                    torch.cuda.synchronize()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                    for _ in range(5):
                        torch.linalg.solve_triangular(Lt, Bm, upper=False)
                    e1.record(stream)
                    e1.synchronize()
                extra = {"cublas_tflops": round(fl / (e0.elapsed_time(e1) / 5 * 1e-3) / 1e12, 2)}
                del Lt
            emit_row("L3", f"{tag}{nm} n=4096 left lower", tf, "TFLOP/s", ms, "tensor" if kind == D else "ffma", tf,
                     peak, "TFLOP/s", note + "; FLOP = the operation's own count (SYRK and TRMM/TRSM n^3)", extra)
        del A, Bm, Cm
        torch.cuda.empty_cache()
    return 0


_OUT_FD = None


def emit(line):
    """Prints the result line on the original stdout (libraries such as NCCL print banners on fd 1 during the run,
    which is redirected to stderr so that rank 0's stdout carries exactly one JSON line)."""
    os.write(_OUT_FD if _OUT_FD is not None else 1, (json.dumps(line) + "\n").encode())


def main():
    global _OUT_FD
    args = parse()
    sys.stdout.flush()
    _OUT_FD = os.dup(1)
    os.dup2(2, 1)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
