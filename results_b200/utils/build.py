"""In-tree build of the native libraries.

Two shared objects are produced under ``results_b200/lib``:

* ``liblz_cuda.so`` -- every ``csrc/*.cu`` and ``csrc/*.cpp`` file, compiled by
  nvcc for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``) with the
  CUDA runtime linked statically and the driver API resolved at run time, so
  the library loads on machines without a GPU driver.
* ``liblz_cpu.so`` -- the CPU oracle (``csrc/cpu/*.cpp``: rANS codec, split,
  fp8 packing), built with g++ and no CUDA dependency.

The build is incremental (object files are rebuilt when a source or any
header is newer) and runs translation units in parallel.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
CSRC = ROOT / "csrc"
LIB_DIR = ROOT / "results_b200" / "lib"
OBJ_DIR = ROOT / "_build" / "obj"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-Wall",
    "-diag-suppress=177",
]
CXX = os.environ.get("CXX", "g++")
CPU_FLAGS = ["-O3", "-std=c++17", "-fPIC", "-shared", "-Wall", "-march=x86-64-v2", "-pthread"]

CUDA_LIB = LIB_DIR / "liblz_cuda.so"
CPU_LIB = LIB_DIR / "liblz_cpu.so"


def _newest(paths) -> float:
    return max((p.stat().st_mtime for p in paths), default=0.0)


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh"))


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if proc.returncode != 0:
        raise RuntimeError("build failed:\n" + " ".join(cmd) + "\n" + proc.stdout)
    if os.environ.get("LZ_BUILD_VERBOSE"):
        sys.stderr.write(proc.stdout)


def cuda_sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))


def cpu_sources() -> list[Path]:
    return sorted((CSRC / "cpu").glob("*.cpp"))


def build_cpu(force: bool = False) -> Path:
    srcs = cpu_sources()
    hdrs = sorted((CSRC / "cpu").glob("*.h")) + [CSRC / "lz_codec_format.h"]
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    if not force and CPU_LIB.exists() and CPU_LIB.stat().st_mtime >= _newest(srcs + hdrs):
        return CPU_LIB
    tmp = CPU_LIB.with_suffix(f".so.tmp{os.getpid()}")
    _run([CXX, *CPU_FLAGS, *map(str, srcs), "-o", str(tmp)])
    os.replace(tmp, CPU_LIB)
    return CPU_LIB


def bounds_requested() -> bool:
    """LZ_BOUNDS=1 selects the range-checked debug build of the CUDA library."""
    return os.environ.get("LZ_BOUNDS", "0") not in ("", "0")


def cuda_lib_name(bounds: bool | None = None) -> str:
    return "liblz_cuda_bounds.so" if (bounds_requested() if bounds is None else bounds) else "liblz_cuda.so"


def build_cuda(force: bool = False, jobs: int | None = None, ptxas_verbose: bool = False,
               bounds: bool | None = None) -> Path:
    """Compile every csrc/*.cu for sm_100a and link the runtime library.

    ``bounds`` (default: environment LZ_BOUNDS) builds the debug variant with
    -DLZ_BOUNDS=1 into ``liblz_cuda_bounds.so``: every peer / multicast store
    range is checked against the mapped heaps and a violation is recorded in
    the status word (code 3, bounds) instead of being executed.
    """
    if not Path(NVCC).exists():
        raise RuntimeError(f"nvcc not found at {NVCC}")
    bounds = bounds_requested() if bounds is None else bounds
    srcs = cuda_sources()
    hdr_time = _newest(_headers())
    obj_dir = OBJ_DIR.with_name(OBJ_DIR.name + "_bounds") if bounds else OBJ_DIR
    lib = LIB_DIR / cuda_lib_name(bounds)
    obj_dir.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    objs = []
    todo = []
    for s in srcs:
        o = obj_dir / (s.name + ".o")
        objs.append(o)
        if force or not o.exists() or o.stat().st_mtime < max(s.stat().st_mtime, hdr_time):
            todo.append((s, o))
    flags = list(NVCC_FLAGS)
    if ptxas_verbose:
        flags += ["-Xptxas", "-v"]
    if bounds:
        flags += ["-DLZ_BOUNDS=1"]

    def compile_one(so):
        s, o = so
        tmp = o.with_suffix(f".o.tmp{os.getpid()}")
        _run([NVCC, *flags, "-I", str(CSRC), "-c", str(s), "-o", str(tmp)])
        os.replace(tmp, o)

    jobs = jobs or min(len(todo) or 1, os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        list(ex.map(compile_one, todo))
    if todo or force or not lib.exists() or lib.stat().st_mtime < _newest(objs):
        tmp = lib.with_suffix(f".so.tmp{os.getpid()}")
        _run([NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", *map(str, objs), "-o", str(tmp),
              "-lpthread", "-ldl", "-lrt"])
        os.replace(tmp, lib)
    return lib


def build_all(force: bool = False) -> tuple[Path, Path]:
    return build_cpu(force), build_cuda(force)


def clean() -> None:
    for p in (CUDA_LIB, CPU_LIB):
        if p.exists():
            p.unlink()
    if OBJ_DIR.exists():
        shutil.rmtree(OBJ_DIR)


if __name__ == "__main__":
    import argparse

    ap = argparse.ArgumentParser(description="build the native libraries in-tree")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    ap.add_argument("--cpu-only", action="store_true")
    a = ap.parse_args()
    print(build_cpu(a.force))
    if not a.cpu_only:
        print(build_cuda(a.force, ptxas_verbose=a.ptxas_verbose))
