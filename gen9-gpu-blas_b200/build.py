"""Build recipe of libgen9blas.so (sm_100a) and of the LD_PRELOAD CBLAS/BLAS library libgen9blas_blas.so.

    python gen9-gpu-blas_b200/build.py [--force] [--ptxas-verbose]

Compiles every csrc/*.cu with nvcc for sm_100a only (-gencode arch=compute_100a,code=sm_100a), links them with the
static CUDA runtime into gen9-gpu-blas_b200/libgen9blas.so, then builds shim/ into libgen9blas_blas.so. Objects go to
gen9-gpu-blas_b200/_build/ (git-ignored). Incremental: a target is rebuilt when any of its sources or headers is newer.
The outputs stay in-tree so that they travel with the repository snapshot.
"""
import argparse
import concurrent.futures
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
SHIM = os.path.join(HERE, "shim")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libgen9blas.so")
SHIM_LIB = os.path.join(HERE, "libgen9blas_blas.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden,-O3",
                  "-I", os.path.join(ROOT, "include"), "-I", CSRC]


def _newer(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd, log=None):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if log is not None:
        log.append(r.stdout + r.stderr)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {os.path.basename(cmd[-1])}")
    return r


def build_core(force=False, ptxas_verbose=False):
    os.makedirs(OBJ, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))
    jobs, objs, logs = [], [], []
    for src in sources:
        obj = os.path.join(OBJ, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or _newer(obj, [src] + headers):
            cmd = [NVCC] + NVFLAGS + (["-Xptxas", "-v"] if ptxas_verbose else []) + ["-c", src, "-o", obj]
            jobs.append(cmd)
    if jobs:
        with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            for f in [ex.submit(_run, j, logs) for j in jobs]:
                f.result()
    if force or jobs or _newer(LIB, objs):
        _run([NVCC] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs + ["-lpthread", "-ldl", "-lrt"])
    if ptxas_verbose:
        with open(os.path.join(OBJ, "ptxas.log"), "w") as f:
            f.write("\n".join(logs))
    return LIB


def build_shim(force=False):
    """libgen9blas_blas.so: own CBLAS/BLAS symbols over libgen9blas.so, every other BLAS symbol forwarded."""
    src = os.path.join(SHIM, "cblas_shim.c")
    gen = os.path.join(SHIM, "gen_forward.py")
    syms = os.path.join(SHIM, "blas_symbols.txt")
    if not os.path.exists(src):
        return None
    os.makedirs(OBJ, exist_ok=True)
    inc = ["-I", os.path.join(ROOT, "include")]
    obj = os.path.join(OBJ, "cblas_shim.o")
    own = os.path.join(OBJ, "shim_own_symbols.txt")
    fwd = os.path.join(OBJ, "cblas_forward.c")
    hdr = os.path.join(ROOT, "include", "gen9blas.h")
    if force or _newer(obj, [src, hdr]):
        _run(["gcc", "-O2", "-fPIC", "-fvisibility=hidden", "-c"] + inc + [src, "-o", obj])
    if force or _newer(fwd, [obj, gen, syms]):
        nm = _run(["nm", "--defined-only", "-g", obj]).stdout
        names = sorted({ln.split()[-1] for ln in nm.splitlines() if ln.split() and ln.split()[-2] in ("T", "D", "R", "B")})
        with open(own, "w") as f:
            f.write("\n".join(n for n in names if not n.startswith("g9_")) + "\n")
        out = _run([sys.executable, gen, syms, own]).stdout
        with open(fwd, "w") as f:
            f.write(out)
    if force or _newer(SHIM_LIB, [obj, fwd, LIB]):
        _run(["gcc", "-O2", "-fPIC", "-shared", "-o", SHIM_LIB, obj, fwd, "-L", HERE, "-lgen9blas",
              "-Wl,-rpath,$ORIGIN", "-ldl", "-lpthread"])
    return SHIM_LIB


def build(force=False, ptxas_verbose=False):
    lib = build_core(force, ptxas_verbose)
    shim = build_shim(force)
    return lib, shim


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.ptxas_verbose))
