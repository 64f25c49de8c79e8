"""Build libssd_b200.so (CUDA kernels + C ABI) in-tree for sm_100a with nvcc.

Usage: python build.py [--force]
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
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3", "--use_fast_math",
         "-Xptxas", "-v" if os.environ.get("SSD_PTXAS_VERBOSE") else "-O3",
         f"-I{INCLUDE}", f"-I{CSRC}"]


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = list(CSRC.glob("*")) + list(INCLUDE.glob("*.h")) + [pathlib.Path(__file__)]
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: pathlib.Path) -> pathlib.Path:
    obj = BUILD / (src.stem + ".o")
    cmd = [NVCC, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    if os.environ.get("SSD_PTXAS_VERBOSE"):
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False) -> pathlib.Path:
    if not force and not _stale():
        return LIB
    BUILD.mkdir(exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(_compile, _sources()))
    cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcuda"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
