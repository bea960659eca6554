"""Build recipe for the oracle's native parts.  TEST INFRASTRUCTURE ONLY.

* ``oracle/liborc_nvfp4.so``: the C restatement (nvfp4_oracle_c.c), gcc with OpenMP, no FMA contraction.
* ``oracle/_ref/libref_nvfp4.so``: the reference's own sources ``kernels/nvfp4_quant.cu`` and
  ``kernels/fp4_gemm.cu``, compiled unmodified where they lie in the reference checkout (nvcc, sm_100a, links
  cuBLASLt) together with ``ref_shim.cpp``, which only forwards C calls to the reference's C++ functions.  Built
  only when the reference checkout is present; tests use it to compare against the reference's cuBLASLt GEMM and
  its host swizzle.  Outputs go to ``oracle/_ref/`` only.
"""
from __future__ import annotations

import os
import pathlib
import shutil
import subprocess

HERE = pathlib.Path(__file__).resolve().parent
REF = pathlib.Path(os.environ.get("NVFP4_REFERENCE_ROOT", "/root/reference"))
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


def build_reference(force: bool = False) -> pathlib.Path | None:
    if not (REF / "kernels" / "fp4_gemm.cu").exists():
        return None
    outdir = HERE / "_ref"
    outdir.mkdir(exist_ok=True)
    out = outdir / "libref_nvfp4.so"
    srcs = [REF / "kernels" / "nvfp4_quant.cu", REF / "kernels" / "fp4_gemm.cu", HERE / "ref_shim.cpp"]
    if force or not _newer(out, *srcs):
        subprocess.check_call([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
                               "-Xcompiler", "-fPIC", "-shared", "-I", str(REF / "include"),
                               "-o", str(out)] + [str(s) for s in srcs] + ["-lcublasLt"])
    return out


if __name__ == "__main__":
    print(build_c_oracle(force=True))
    print(build_reference(force=True))
