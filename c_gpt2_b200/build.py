"""Build the sm_100a shared libraries in-tree.

    libgpt2_w8a8.so              kernels (nvcc, sm_100a) + C host engine (gcc),
                                 CUDA runtime linked statically and hidden
    libcuda_kernels_{small,medium,large}.so
                                 the reference-shaped drop-in ABI
                                 (include/cuda_kernels.h), one per model size

Run `python -m c_gpt2_b200.build` (or `__graft_entry__.build()`). Rebuilds
only when a source or header is newer than its output.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
HOST = PKG / "host"
INCLUDE = ROOT / "include"
LIBDIR = PKG / "lib"
BUILD = PKG / "_build"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                     "-Xcompiler", "-Wall", f"-I{INCLUDE}"]
CC_FLAGS = ["-O2", "-fPIC", "-std=gnu11", "-Wall", "-Wextra", "-Wno-unused-parameter",
            f"-I{INCLUDE}", f"-I{CUDA_HOME / 'include'}"]

SIZES = {"small": "GPT2_SMALL_MODEL", "medium": "GPT2_MEDIUM_MODEL", "large": "GPT2_LARGE_MODEL"}
CORE_LIB = LIBDIR / "libgpt2_w8a8.so"


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")))


def _stale(out: Path, deps: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} {cmd[-1]}")


def build(verbose: bool = False) -> list[Path]:
    """Compile everything that is out of date; returns the library paths."""
    if not Path(NVCC).exists() and shutil.which("nvcc") is None:
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    BUILD.mkdir(exist_ok=True)
    LIBDIR.mkdir(exist_ok=True)
    headers = _headers()
    jobs = []
    objs = []
    for cu in sorted(CSRC.glob("*.cu")):
        o = BUILD / (cu.stem + ".o")
        objs.append(o)
        if _stale(o, [cu] + headers):
            jobs.append([NVCC] + NVCC_FLAGS + ["-c", str(cu), "-o", str(o)])
    for c in ["engine.c"]:
        src = HOST / c
        o = BUILD / (Path(c).stem + ".o")
        objs.append(o)
        if _stale(o, [src] + headers):
            jobs.append(["gcc"] + CC_FLAGS + ["-c", str(src), "-o", str(o)])
    if jobs:
        with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
            list(ex.map(_run, jobs))
    if _stale(CORE_LIB, objs):
        _run([NVCC] + ARCH + ["-shared", "-o", str(CORE_LIB)] + [str(o) for o in objs] +
             ["-cudart", "static", "-Xlinker", "--exclude-libs,ALL",
              "-Xlinker", "-Bsymbolic", "-lpthread", "-ldl", "-lrt"])
    libs = [CORE_LIB]
    compat_src = HOST / "compat_cuda_kernels.c"
    for size, macro in SIZES.items():
        out = LIBDIR / f"libcuda_kernels_{size}.so"
        libs.append(out)
        if _stale(out, [compat_src, CORE_LIB] + headers):
            _run(["gcc"] + CC_FLAGS + [f"-D{macro}", "-shared", str(compat_src), "-o", str(out),
                                      f"-L{LIBDIR}", "-lgpt2_w8a8", "-Wl,-rpath,$ORIGIN"])
    if verbose:
        for lib in libs:
            print(lib)
    return libs


if __name__ == "__main__":
    build(verbose=True)
