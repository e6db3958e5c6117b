"""CPU checks of bench.py's contract pieces that need no GPU: the reference arm's JSON line (it times the reference's
own CPU path, oracle/_ref, or the oracle port where that is not built), its silence on ranks other than 0, the clock
sampler's decoding of throttle reasons, and the roofline inputs read from committed files."""
import json
import os
import subprocess
import sys
import threading

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402

BASE_KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
             "vs_baseline", "dtype", "data", "config"}


def run_bench(args, env_extra=None, timeout=600):
    env = dict(os.environ)
    env.pop("RANK", None)
    env.pop("WORLD_SIZE", None)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py")] + args, capture_output=True, text=True,
                          env=env, timeout=timeout, cwd=ROOT)


def test_reference_arm_prints_one_contract_line():
    r = run_bench(["--impl", "reference", "--steps", "1", "--warmup", "1"])
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert BASE_KEYS <= set(d), set(d) ^ BASE_KEYS
    assert d["impl"] == "reference" and d["metric"] == bench.METRIC
    assert d["unit"] == "TFLOP/s" and d["higher_is_better"] is True and d["value"] > 0
    assert d["steps"] == 1 and d["warmup"] == 1 and d["n_gpus"] == 1
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["value"] == d["value"] and cb["cores"] >= 1 and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["n"] == 4096 and "workload" in d["config"]


def test_reference_arm_other_ranks_are_silent():
    r = run_bench(["--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "1"],
                  {"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


class _FakeNvml:
    def nvmlShutdown(self):
        pass


def _stopped(sampler):
    sampler.thread = threading.Thread(target=lambda: None)
    sampler.thread.start()
    return sampler.stop()


def test_clock_sampler_nvml_reasons_and_loaded_median():
    s = bench.ClockSampler(0)
    s.nvml = (_FakeNvml(), None)
    s.max_mhz = 1965.0
    # (SM MHz, reason bits): sw_power_cap = 0x4, hw_slowdown = 0x8; an idle sample below 30 % of max is not "loaded"
    s.samples = [(1965, 0x4), (1500, 0x4 | 0x8), (1600, 0x0), (300, 0x0)]
    out = _stopped(s)
    assert out["reasons"] == ["hw_slowdown", "sw_power_cap"]
    assert out["sm_mhz"] == 1600.0 and out["sm_max_mhz"] == 1965.0 and out["samples"] == 4
    assert out["source"] == "nvml"


def test_clock_sampler_nvidia_smi_lines():
    class _Proc:
        def terminate(self):
            pass

        def wait(self, timeout=None):
            return 0

    s = bench.ClockSampler(0)
    s.proc = _Proc()
    s.lines = ["0, 1500, 1965, 980.1, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
               "0, 1400, 1965, 990.5, 0x0000000000000044, Not Active, Active, Not Active, Active",
               "garbage line"]
    out = _stopped(s)
    assert out["reasons"] == ["hw_thermal_slowdown", "sw_power_cap"]
    assert out["sm_mhz"] == 1450.0 and out["sm_max_mhz"] == 1965.0 and out["samples"] == 2


def test_roofline_inputs_from_committed_files():
    traffic = bench.profile_traffic("hgemm_tc2_n4096")
    assert traffic is not None and 80e6 < traffic < 120e6   # DRAM bytes of one n = 4096 launch (A + B + C ≈ 100.7 MB)
    assert bench.profile_traffic("no_such_profile") is None
    burst, sust, peak_hbm, kind = bench.measured_peaks()
    if os.path.exists(os.path.join(ROOT, "MEASURED_PEAKS.json")):
        d = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        assert kind == "measured" and burst == d["bf16_tflops"] and sust == d["bf16_tflops_sustained"]
        assert peak_hbm == d["hbm_gbs"]
    else:
        assert kind == "fallback" and (burst, sust) == (1590.0, 1400.0)


def test_tensor_peak_follows_the_sampled_clocks():
    """Burst denominator for a region at full clock with no cap; sustained when the power cap shows or the median SM
    clock sits below the maximum; burst (noted) when nothing was sampled."""
    burst, sust, _, _ = bench.measured_peaks()
    full = {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": []}
    p, note, both = bench.tensor_peak(full)
    assert p == burst and "burst" in note and both == {"burst": burst, "sustained": sust}
    p, note, _ = bench.tensor_peak(dict(full, reasons=["sw_power_cap"]))
    assert p == sust and "sw_power_cap" in note
    p, note, _ = bench.tensor_peak(dict(full, sm_mhz=1357.0))
    assert p == sust and "1357" in note
    p, note, _ = bench.tensor_peak(None)
    assert p == burst and "no clock samples" in note


def test_no_function_shadows_the_type_constants():
    """bench.py's functions read the module's GEMM type constants (H, S, HS, D); a function that also assigns one of
    those names makes it local for the whole function, and the earlier reads then fail (UnboundLocalError) only when
    the workload that reads them runs. Checked on the source: no function assigns them."""
    import ast
    src = open(os.path.join(ROOT, "bench.py")).read()
    tree = ast.parse(src)
    consts = {"H", "S", "HS", "D"}
    bad = []
    for fn in [n for n in ast.walk(tree) if isinstance(n, (ast.FunctionDef, ast.AsyncFunctionDef))]:
        for node in ast.walk(fn):
            if isinstance(node, ast.Name) and isinstance(node.ctx, ast.Store) and node.id in consts:
                bad.append((fn.name, node.id, node.lineno))
    assert not bad, bad
