"""Build the B200 Ozaki backend in-tree.

Produces
  oztt_b200/liboztt.so            the CUDA kernels for sm_100a, the planner, the C ABI
                                  (include/oztt_cuda.h) and the C++ API (include/ozTTgemm/ozTTgemm.hpp)
  oztt_b200/_build/gemm_example   examples/gemm.cpp linked against it
  oztt_b200/_build/correctness    tests/cpp/correctness.cpp linked against it
Object files go to oztt_b200/_build/. Nothing is installed outside the repository; the built files
travel with the repository snapshot to the GPU machine.

Run as ``python -m oztt_b200.build`` or through ``__graft_entry__.build()``.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "oztt_b200"
CSRC = PKG / "csrc"
OUT = PKG / "_build"
LIB = PKG / "liboztt.so"

NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
# The system compiler: the environment's CXX may name a toolchain without OpenMP support files.
CXX = "/usr/bin/g++" if Path("/usr/bin/g++").exists() else (shutil.which("g++") or "g++")
CUDA_HOME = Path(NVCC).resolve().parent.parent

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-ffp-contract=off",
              "-ccbin", CXX, f"-I{ROOT / 'include'}"]
CXX_FLAGS = ["-std=gnu++20", "-O2", "-fPIC", "-fno-fast-math", "-ffp-contract=off", "-pthread",
             f"-I{ROOT / 'include'}", f"-I{CUDA_HOME / 'include'}"]

# The host planners run the reference's selection arithmetic over every input element: built for the
# x86-64-v3 level (AVX2, FMA, SSE4.1 rounding) so that fma and nearbyint are single instructions.
# Contraction stays off, so every operation rounds as written and the decisions do not change.
CXX_FLAGS_BY_SOURCE = {"planner.cpp": ["-O3", "-march=x86-64-v3"], "planner1.cpp": ["-O3", "-march=x86-64-v3"],
                       "planner_digit.cpp": ["-O3", "-march=x86-64-v3"]}

CU_SOURCES = ["split.cu", "gemm_i8.cu", "recon.cu", "ii_int8.cu", "ii_digit.cu", "noalloc.cu", "scheme1.cu",
              "stats.cu", "profile.cu", "streamed.cu", "plan1_dev.cu", "resident.cu"]
CPP_SOURCES = ["planner.cpp", "planner1.cpp", "planner_digit.cpp", "context.cpp", "evaluation.cpp"]


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build step failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build_library(force: bool = False) -> Path:
    OUT.mkdir(parents=True, exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.hpp")) + [ROOT / "include" / "oztt_cuda.h",
                                                                      ROOT / "include" / "ozTTgemm" / "ozTTgemm.hpp",
                                                                      ROOT / "include" / "evaluation_hooks.hpp"]
    objs = []
    for src in CU_SOURCES:
        s, o = CSRC / src, OUT / (src + ".o")
        if force or _stale(o, [s] + headers):
            _run([NVCC, *ARCH, *NVCC_FLAGS, "-c", str(s), "-o", str(o)])
        objs.append(o)
    for src in CPP_SOURCES:
        s, o = CSRC / src, OUT / (src + ".o")
        if force or _stale(o, [s] + headers):
            _run([CXX, *CXX_FLAGS, *CXX_FLAGS_BY_SOURCE.get(src, []), "-c", str(s), "-o", str(o)])
        objs.append(o)
    if force or _stale(LIB, objs):
        # every symbol resolved at link time: a missing definition fails the build, not the first load
        _run([NVCC, *ARCH, "-shared", "-ccbin", CXX, "-Xlinker", "--no-undefined", "-o", str(LIB), *map(str, objs),
              "-lpthread"])
    return LIB


def build_programs(force: bool = False) -> None:
    progs = {
        "gemm_example": ROOT / "examples" / "gemm.cpp",
        "correctness": ROOT / "tests" / "cpp" / "correctness.cpp",
    }
    for name, src in progs.items():
        if not src.exists():
            continue
        exe = OUT / name
        if force or _stale(exe, [src, LIB]):
            _run([CXX, "-std=gnu++20", "-O2", f"-I{ROOT / 'include'}", str(src), "-o", str(exe),
                  f"-L{PKG}", "-loztt", f"-Wl,-rpath,{PKG}", "-pthread"])


def reference_root() -> Path:
    """Where the reference tree is looked for (test tooling only): the directory named by the environment
    variable OZTT_REFERENCE_DIR, else a directory named `reference` beside the repository."""
    return Path(os.environ.get("OZTT_REFERENCE_DIR", str(ROOT.parent / "reference"))).resolve()


def build_oracle() -> None:
    """The CPU checker libraries (test infrastructure): oracle/liboz2oracle.so always, and
    oracle/_ref/*.so and the reference's caller programs when the reference tree is present on this
    machine (reference_root())."""
    make = shutil.which("make") or "make"
    _run([make, "-s", "-C", str(ROOT / "oracle"), "all"])
    ref = reference_root()
    if (ref / "src" / "backend").is_dir():
        _run([make, "-s", "-C", str(ROOT / "oracle"), "ref", f"REF={ref}"])
        # the reference's own callers of the public API, compiled unchanged against liboztt.so
        _run([make, "-s", "-C", str(ROOT / "oracle"), "callers", f"REF={ref}"])


def build(force: bool = False) -> None:
    build_library(force)
    build_programs(force)
    build_oracle()


if __name__ == "__main__":
    build(force="--force" in sys.argv)
    print(f"built {LIB}")
