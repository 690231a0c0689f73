"""Build the B200 library in-tree: harp-q_b200/lib/libharpq_b200.so (sm_100a).

Sources are compiled with nvcc for ``-gencode arch=compute_100a,code=sm_100a`` and
linked with the static CUDA runtime (its symbols hidden) plus cuBLAS for the
materialize-then-SGEMM oracle entry point.  The native test program
(tests/native/api_test.cu) is linked against the library as
harp-q_b200/lib/hqb_api_test.  Rebuilds only what is out of date.
"""

from __future__ import annotations

import os
import subprocess
import sys
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
OBJ_DIR = LIB_DIR / "obj"
LIB = LIB_DIR / "libharpq_b200.so"
API_TEST = LIB_DIR / "hqb_api_test"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
SOURCES = ["hqb_plane.cu", "hqb_bulk.cu", "hqb_raw.cu", "hqb_raw_i8.cu", "hqb_step.cu", "hqb_prefill.cu", "harpq_native.cu", "hqb_static_scratch.cu"]
CFLAGS = [*ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
          "-Xcompiler", "-ffp-contract=off",
          "-I", str(REPO / "include"), "-I", str(CSRC)]


def _headers() -> list[Path]:
    return [*CSRC.glob("*.h"), *CSRC.glob("*.cuh"), *(REPO / "include").rglob("*.h"),
            *(REPO / "include").rglob("*.hpp")]


def _stale(out: Path, deps: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps if d.exists())


def _run(cmd: list[str]) -> None:
    if os.environ.get("HQB_BUILD_VERBOSE"):
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)


def _compile(cmd: list[str], obj: Path) -> None:
    # The object is dated to the start of its compile, so a source edited while the
    # compiler runs is newer than the object and is compiled again next time.
    t0 = time.time()
    _run(cmd)
    os.utime(obj, (t0, t0))


def build(force: bool = False, ptxas_verbose: bool = False) -> Path:
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    headers = _headers()
    objs, jobs = [], []
    for src in SOURCES:
        obj = OBJ_DIR / (src + ".o")
        if force or ptxas_verbose or _stale(obj, [CSRC / src, *headers]):
            extra = ["-Xptxas", "-v"] if ptxas_verbose else []
            jobs.append(([NVCC, *CFLAGS, *extra, "-c", str(CSRC / src), "-o", str(obj)], obj))
        objs.append(obj)
    # the translation units compile independently; the largest (hqb_plane.cu) sets the time
    with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as pool:
        for f in [pool.submit(_compile, cmd, obj) for cmd, obj in jobs]:
            f.result()
    if force or _stale(LIB, objs):
        # link beside the library and rename over it, so a reader never sees a partial file
        tmp = LIB.with_name(LIB.name + ".tmp")
        _run([NVCC, *ARCH, "-shared", "-cudart", "static", "-Xlinker", "--exclude-libs,ALL",
              *map(str, objs), "-o", str(tmp), "-lcublas"])
        os.replace(tmp, LIB)
    test_src = REPO / "tests" / "native" / "api_test.cu"
    if test_src.exists() and (force or _stale(API_TEST, [test_src, LIB, *headers])):
        _run([NVCC, *CFLAGS, str(test_src), "-o", str(API_TEST), "-L", str(LIB_DIR), "-lharpq_b200",
              "-Xlinker", "-rpath=$ORIGIN"])
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, ptxas_verbose="--ptxas-verbose" in sys.argv)
