"""TEST INFRASTRUCTURE ONLY: where the checkers find the CPU BLAS (OpenBLAS) and the reference checkout.

The reference's CBLAS layer (lib/src/cblas.c of kprzybys/gen9-gpu-blas) forwards its arithmetic to a CPU BLAS
chosen by GEN9BLAS_BLAS_CPU; the parity checkers and the CPU baseline use the same OpenBLAS. Nothing of the product
(gen9-gpu-blas_b200/) imports this module.

- openblas(): GEN9BLAS_OPENBLAS (path of a libopenblas shared object with plain cblas_* names) if set, else the
  first libopenblas*.so found in a wheel's bundled-library folder (site-packages/*.libs/, e.g. the OpenCV wheel's
  OpenBLAS 0.3.15). Returns None when neither exists; callers skip or report "unavailable".
- load_openblas(): the above, with the libraries it depends on from the same folder loaded first (RTLD_GLOBAL).
- reference_dir(): GEN9BLAS_REFERENCE if set, else a checkout named "reference" beside this repository; None when
  neither holds lib/src/cblas.c.
"""
import ctypes
import glob
import os
import site

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def openblas():
    env = os.environ.get("GEN9BLAS_OPENBLAS")
    if env:
        return env if os.path.exists(env) else None
    dirs = list(site.getsitepackages())
    try:
        dirs.append(site.getusersitepackages())
    except AttributeError:
        pass
    for d in dirs:
        hits = sorted(glob.glob(os.path.join(d, "*.libs", "libopenblas*.so*")))
        if hits:
            return hits[0]
    return None


def preload_openblas_deps():
    """Loads the libraries OpenBLAS depends on (libgfortran, libquadmath of its wheel folder) with RTLD_GLOBAL, so that
    a library that dlopens OpenBLAS by path (the CBLAS layers, through GEN9BLAS_BLAS_CPU) finds them. Returns the
    OpenBLAS path or None."""
    path = openblas()
    if path is None:
        return None
    folder = os.path.dirname(path)
    for pattern in ("libquadmath*.so*", "libgfortran*.so*"):   # in dependency order
        for dep in sorted(glob.glob(os.path.join(folder, pattern))):
            ctypes.CDLL(dep, mode=ctypes.RTLD_GLOBAL)
    return path


def load_openblas():
    """ctypes handle of OpenBLAS (its wheel folder's dependencies loaded globally first), or None."""
    path = preload_openblas_deps()
    return ctypes.CDLL(path) if path else None


def reference_dir():
    for d in (os.environ.get("GEN9BLAS_REFERENCE"), os.path.join(os.path.dirname(ROOT), "reference")):
        if d and os.path.exists(os.path.join(d, "lib", "src", "cblas.c")):
            return d
    return None


if __name__ == "__main__":
    import sys
    what = sys.argv[1] if len(sys.argv) > 1 else "openblas"
    r = reference_dir() if what == "reference" else openblas()
    if r is None:
        sys.exit(1)
    print(r)
