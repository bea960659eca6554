"""Build libnvfp4_b200.so in-tree: every .cu under csrc/ compiled by nvcc for sm_100a, then linked into one shared
library next to this file.  No torch extension machinery: the library has a plain C ABI (include/nvfp4_b200.h)
plus the reference's C++ operator symbols (include/fp4_gemm.h, include/nvfp4_quant.h)."""
from __future__ import annotations

import concurrent.futures as cf
import os
import pathlib
import shutil
import subprocess

PKG = pathlib.Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libnvfp4_b200.so"
NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-I", str(ROOT / "include"), "-I", str(CSRC)]


def _stale(obj: pathlib.Path, src: pathlib.Path) -> bool:
    if not obj.exists():
        return True
    deps = [src] + list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h"))
    return any(d.stat().st_mtime > obj.stat().st_mtime for d in deps)


def _compile(src: pathlib.Path, verbose_ptxas: bool) -> pathlib.Path:
    obj = BUILD / (src.stem + ".o")
    if _stale(obj, src):
        extra = ["-Xptxas", "-v"] if verbose_ptxas else []
        subprocess.check_call([NVCC, *ARCH, *FLAGS, *extra, "-c", str(src), "-o", str(obj)])
    return obj


def build(verbose_ptxas: bool = False) -> pathlib.Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose_ptxas), srcs))
    if not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        subprocess.check_call([NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart"])
    return LIB


if __name__ == "__main__":
    import sys
    print(build(verbose_ptxas="-v" in sys.argv))
