"""Build recipe for the CPU oracle and, when the reference checkout is present,
for oracle/_ref (binaries compiled from the reference's own sources, in place).

TEST INFRASTRUCTURE ONLY.  Outputs:

* oracle/liboracle.so                — harpq_oracle.c (plain C restatement), always.
* oracle/_ref/libharpq_ref.so        — reference native/src/stage_codec.cpp + ref_shim.cpp
                                       (CPU reference: decode, ProgressiveLinearReference).
* oracle/_ref/libharpq_ref_gpu.so    — reference native/src/progressive_gemv.cu +
                                       stage_codec.cpp + ref_gpu_shim.cu for sm_100a
                                       (the reference's own fused GEMV kernel, as a
                                       timed GPU comparison).
* oracle/_ref/ref_*_test             — the reference's own C++/CUDA tests
                                       (stage_codec_test.cpp, progressive_gemv_test.cu,
                                       cuda_oracle_test.cu) compiled against THIS
                                       repository's headers and product library: the
                                       drop-in check for the native API.

oracle/_ref is git-ignored but travels with the working tree, so these binaries
are usable on a machine without the reference checkout.  Reference sources are
only read where they lie; nothing is copied into the repository.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

ORACLE = Path(__file__).resolve().parent
REPO = ORACLE.parent
REF_OUT = ORACLE / "_ref"
# The reference checkout: $HQB_REFERENCE, else a directory named "reference" beside this
# repository's directory.  Absent on machines that only run the prebuilt files.
DEFAULT_REFERENCE = Path(os.environ.get("HQB_REFERENCE", str(REPO.parent / "reference")))
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _stale(out: Path, inputs: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(p.exists() and p.stat().st_mtime > t for p in inputs)


def _run(cmd: list[str]) -> None:
    subprocess.run(cmd, check=True)


def build_oracle(force: bool = False) -> Path:
    out = ORACLE / "liboracle.so"
    srcs = [ORACLE / "harpq_oracle.c", ORACLE / "harpq_oracle.h"]
    if force or _stale(out, srcs):
        _run(["gcc", "-O2", "-ffp-contract=off", "-fPIC", "-shared", "-std=c11",
              str(ORACLE / "harpq_oracle.c"), "-o", str(out), "-lm"])
    return out


def build_reference_cpu(ref: Path, force: bool = False) -> Path | None:
    src = ref / "native" / "src" / "stage_codec.cpp"
    if not src.exists():
        return None
    REF_OUT.mkdir(exist_ok=True)
    out = REF_OUT / "libharpq_ref.so"
    if force or _stale(out, [src, ORACLE / "ref_shim.cpp"]):
        _run(["g++", "-O3", "-std=c++17", "-fPIC", "-shared", "-fvisibility=hidden",
              "-fvisibility-inlines-hidden", "-Wl,-Bsymbolic",
              "-I", str(ref / "native" / "include"),
              str(ORACLE / "ref_shim.cpp"), str(src), "-o", str(out)])
    return out


def build_reference_gpu(ref: Path, force: bool = False) -> Path | None:
    src = ref / "native" / "src" / "progressive_gemv.cu"
    if not src.exists():
        return None
    REF_OUT.mkdir(exist_ok=True)
    out = REF_OUT / "libharpq_ref_gpu.so"
    inputs = [src, ref / "native" / "src" / "stage_codec.cpp", ORACLE / "ref_gpu_shim.cu"]
    if force or _stale(out, inputs):
        _run([NVCC, *ARCH, "-O3", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-fvisibility=hidden", "-Xcompiler", "-fvisibility-inlines-hidden",
              "-Xlinker", "-Bsymbolic", "-cudart", "static",
              "-I", str(ref / "native" / "include"),
              str(ORACLE / "ref_gpu_shim.cu"), str(src), str(ref / "native" / "src" / "stage_codec.cpp"),
              "-o", str(out)])
    return out


def build_reference_tests(ref: Path, product_lib: Path, force: bool = False) -> list[Path]:
    """The reference's own tests, compiled against this repository's API."""
    tests_dir = ref / "native" / "tests"
    if not tests_dir.exists() or not product_lib.exists():
        return []
    REF_OUT.mkdir(exist_ok=True)
    inc = ["-I", str(REPO / "include"), "-I", str(tests_dir)]
    link = ["-L", str(product_lib.parent), "-lharpq_b200",
            "-Xlinker", f"-rpath={product_lib.parent}",
            "-Xlinker", "-rpath=$ORIGIN/../../harp-q_b200/lib"]
    built = []
    for name, src in (("ref_stage_codec_test", tests_dir / "stage_codec_test.cpp"),
                      ("ref_progressive_gemv_test", tests_dir / "progressive_gemv_test.cu"),
                      ("ref_cuda_oracle_test", tests_dir / "cuda_oracle_test.cu")):
        out = REF_OUT / name
        headers = list((REPO / "include" / "harpq").rglob("*.hpp"))
        if force or _stale(out, [src, product_lib, *headers]):
            _run([NVCC, *ARCH, "-O2", "-std=c++17", *inc, "-x", "cu" if src.suffix == ".cu" else "c++",
                  str(src), "-o", str(out), *link])
        built.append(out)
    return built


def main() -> int:
    force = "--force" in sys.argv
    build_oracle(force)
    ref = DEFAULT_REFERENCE
    if ref.exists():
        build_reference_cpu(ref, force)
        build_reference_gpu(ref, force)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
