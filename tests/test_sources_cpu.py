"""Source rules the library keeps, checked on the committed text (no GPU, no build):

- no bulk or TMA load with cluster multicast anywhere: the multi-GPU paths read peer memory, and a multicast load
  whose source is another GPU's memory hangs the GPU; the only multicast qualifier allowed is on tcgen05.commit
  (an mbarrier arrive in the CTA pair, no memory load);
- none of the batched asynchronous copy calls of the CUDA runtime and driver (they raised GPU faults on B200 with
  this driver); copies are one cudaMemcpyAsync each;
- the product (the package, bench.py's timed path) never imports or loads anything under oracle/.

The patterns are assembled from pieces so that this file does not itself contain the names it looks for."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SOURCE_DIRS = ("gen9-gpu-blas_b200", "include", "oracle", "profiles", "tests")   # plus the files at the top level
SKIP_DIRS = {"_build", "_ref", "__pycache__"}
SOURCE_EXT = {".cu", ".cuh", ".h", ".hpp", ".c", ".cc", ".cpp", ".py", ".sh", ".txt", ".json", ".mk"}

BATCH_COPY = re.compile("cu(?:da)?Memcpy(?:3D)?Batch" + "Async")
MULTICAST = re.compile("multi" + "cast::cluster")
BULK_COPY, MC_WORD = "cp.async" + ".bulk", "multi" + "cast"


def is_source(f):
    return os.path.splitext(f)[1] in SOURCE_EXT or f == "Makefile"


def source_files():
    for f in os.listdir(ROOT):
        if os.path.isfile(os.path.join(ROOT, f)) and is_source(f):
            yield os.path.join(ROOT, f)
    for top in SOURCE_DIRS:
        for dirpath, dirnames, filenames in os.walk(os.path.join(ROOT, top)):
            dirnames[:] = [d for d in dirnames if d not in SKIP_DIRS]
            for f in filenames:
                if is_source(f):
                    yield os.path.join(dirpath, f)


def read(path):
    with open(path, encoding="utf-8", errors="replace") as fh:
        return fh.read()


def test_no_batched_async_copy_calls():
    hits = []
    for p in source_files():
        for i, line in enumerate(read(p).splitlines(), 1):
            if BATCH_COPY.search(line):
                hits.append(f"{os.path.relpath(p, ROOT)}:{i}")
    assert not hits, hits


def test_multicast_only_on_tcgen05_commit():
    hits = []
    for p in source_files():
        for i, line in enumerate(read(p).splitlines(), 1):
            if MULTICAST.search(line) and "tcgen05.commit" not in line:
                hits.append(f"{os.path.relpath(p, ROOT)}:{i}")
            if BULK_COPY in line and MC_WORD in line:
                hits.append(f"{os.path.relpath(p, ROOT)}:{i} (bulk copy)")
    assert not hits, hits


def test_product_does_not_reach_the_oracle():
    pkg = os.path.join(ROOT, "gen9-gpu-blas_b200")
    pat = re.compile(r"\boracle\b")
    hits = []
    for dirpath, dirnames, filenames in os.walk(pkg):
        dirnames[:] = [d for d in dirnames if d not in SKIP_DIRS]
        for f in filenames:
            if not is_source(f):
                continue
            p = os.path.join(dirpath, f)
            for i, line in enumerate(read(p).splitlines(), 1):
                code = line.split("//")[0].split("#")[0] if not f.endswith(".txt") else ""
                if pat.search(code) and ("import" in code or "dlopen" in code or "CDLL" in code or ".so" in code):
                    hits.append(f"{os.path.relpath(p, ROOT)}:{i}")
    assert not hits, hits
