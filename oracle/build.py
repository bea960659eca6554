"""Build recipe for the oracle's native parts.  TEST INFRASTRUCTURE ONLY.

* ``oracle/liborc_nvfp4.so``: the C restatement (nvfp4_oracle_c.c), gcc with OpenMP, no FMA contraction.
* ``oracle/_ref/libref_nvfp4.so``: the reference's own sources ``kernels/nvfp4_quant.cu`` and
  ``kernels/fp4_gemm.cu``, compiled unmodified where they lie in the reference checkout (nvcc, sm_100a, links
  cuBLASLt) together with ``ref_shim.cpp``, which only forwards C calls to the reference's C++ functions.  Tests use
  it to compare against the reference's cuBLASLt GEMM and its host swizzle.
* ``oracle/_ref/test_fp4_gemm_linked``: the reference's own GEMM test program ``tests/test_fp4_gemm.cu``, compiled
  unmodified against this repository's ``include/`` headers and linked to ``libnvfp4_b200.so`` instead of the
  reference's kernels: the link-level proof that the library is a drop-in for the reference's C++ API.
The reference parts are built only when a reference checkout is given (``ref_root`` argument, or the
``NVFP4_REFERENCE_ROOT`` environment variable); outputs go to ``oracle/_ref/`` only.
"""
from __future__ import annotations

import os
import pathlib
import shutil
import subprocess

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parent
NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"


def _newer(out: pathlib.Path, *srcs: pathlib.Path) -> bool:
    return out.exists() and all(out.stat().st_mtime >= s.stat().st_mtime for s in srcs if s.exists())


def build_c_oracle(force: bool = False) -> pathlib.Path:
    src = HERE / "nvfp4_oracle_c.c"
    out = HERE / "liborc_nvfp4.so"
    if force or not _newer(out, src):
        subprocess.check_call(["gcc", "-O2", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off", "-o", str(out),
                               str(src), "-lm"])
    return out


def reference_root(ref_root: str | os.PathLike | None = None) -> pathlib.Path | None:
    """The reference checkout: the argument, else $NVFP4_REFERENCE_ROOT; None if neither names one that exists."""
    r = ref_root if ref_root is not None else os.environ.get("NVFP4_REFERENCE_ROOT")
    if not r:
        return None
    r = pathlib.Path(r)
    return r if (r / "kernels" / "fp4_gemm.cu").exists() else None


def build_reference(ref_root=None, force: bool = False) -> pathlib.Path | None:
    ref = reference_root(ref_root)
    if ref is None:
        return None
    outdir = HERE / "_ref"
    outdir.mkdir(exist_ok=True)
    out = outdir / "libref_nvfp4.so"
    srcs = [ref / "kernels" / "nvfp4_quant.cu", ref / "kernels" / "fp4_gemm.cu", HERE / "ref_shim.cpp"]
    if force or not _newer(out, *srcs):
        subprocess.check_call([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
                               "-Xcompiler", "-fPIC", "-shared", "-I", str(ref / "include"),
                               "-o", str(out)] + [str(s) for s in srcs] + ["-lcublasLt"])
    return out


def build_reference_linked_test(ref_root=None, force: bool = False) -> pathlib.Path | None:
    """The reference's tests/test_fp4_gemm.cu, unmodified, against include/ and libnvfp4_b200.so (found at run time
    through an rpath relative to the binary, so the pair travels together)."""
    ref = reference_root(ref_root)
    lib = ROOT / "gemma-cuda-server_b200" / "libnvfp4_b200.so"
    if ref is None or not lib.exists():
        return None
    outdir = HERE / "_ref"
    outdir.mkdir(exist_ok=True)
    out = outdir / "test_fp4_gemm_linked"
    src = ref / "tests" / "test_fp4_gemm.cu"
    if force or not _newer(out, src, lib, ROOT / "include" / "fp4_gemm.h"):
        subprocess.check_call([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-O2", "-std=c++17",
                               "-I", str(ROOT / "include"), "-o", str(out), str(src),
                               "-L", str(lib.parent), "-lnvfp4_b200", "-lcublasLt",
                               "-Xlinker", "-rpath=$ORIGIN/../../gemma-cuda-server_b200"])
    return out


if __name__ == "__main__":
    import sys
    root = sys.argv[1] if len(sys.argv) > 1 else None
    print(build_c_oracle(force=True))
    print(build_reference(root, force=True))
    print(build_reference_linked_test(root, force=True))
