"""Build libssd_b200.so (CUDA kernels + C ABI) in-tree for sm_100a with nvcc.

Usage: python build.py [--force] [--debug]
Each .cu file compiles to an object in _build/ (in parallel), then one shared library
is linked into mamba2_b200/libssd_b200.so.  Rebuilds only when a source or header is
newer than the library.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import pathlib
import subprocess
import sys

HERE = pathlib.Path(__file__).resolve().parent
REPO = HERE.parent
CSRC = HERE / "csrc"
INCLUDE = REPO / "include"
BUILD = HERE / "_build"
LIB = HERE / "mamba2_b200" / "libssd_b200.so"
# SSD_DEBUG variant: every global index of the fused kernel checked, out-of-range accesses
# skipped and reported through the device status word
LIB_DEBUG = HERE / "mamba2_b200" / "libssd_b200_debug.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3", "--use_fast_math",
         "-Xptxas", "-v" if os.environ.get("SSD_PTXAS_VERBOSE") else "-O3",
         f"-I{INCLUDE}", f"-I{CSRC}"]


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _stale(lib=LIB) -> bool:
    if not lib.exists():
        return True
    t = lib.stat().st_mtime
    deps = list(CSRC.glob("*")) + list(INCLUDE.glob("*.h")) + [pathlib.Path(__file__)]
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: pathlib.Path, debug: bool = False) -> pathlib.Path:
    obj = (BUILD / "debug" if debug else BUILD) / (src.stem + ".o")
    cmd = [NVCC, *ARCH, *FLAGS, *(["-DSSD_DEBUG"] if debug else []), "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    if os.environ.get("SSD_PTXAS_VERBOSE"):
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, debug: bool = False) -> pathlib.Path:
    lib = LIB_DEBUG if debug else LIB
    if not force and not _stale(lib):
        return lib
    (BUILD / "debug" if debug else BUILD).mkdir(parents=True, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda src: _compile(src, debug), _sources()))
    cmd = [NVCC, *ARCH, "-shared", "-o", str(lib), *map(str, objs), "-lcuda"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, debug="--debug" in sys.argv))
