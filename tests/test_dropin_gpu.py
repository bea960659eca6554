"""The drop-in boundary at link level, on the GPU.

1. The reference's own GEMM test program (tests/test_fp4_gemm.cu of the reference), compiled unmodified against the
   headers in include/ and linked to libnvfp4_b200.so instead of the reference's kernels (oracle/build.py), runs on
   the fixtures of the reference's generator (scripts/gen_fp4_gemm_testcase.py, committed as
   tests/golden/gemm_cases.npz) and must print its own verdict "GATE PASS" (tests/test_fp4_gemm.cu:76-78).
2. The reference's void entry points (nvfp4_quantize_activations, w4a16_gemm, fp4_gemv) report failure only
   through the CUDA error state its callers check with cudaGetLastError (src/forward.cu:23); an argument error must
   therefore leave an error there instead of returning silently."""
import ctypes
import pathlib
import subprocess

import numpy as np
import pytest
import torch

from gpu_util import require_gpu

pytestmark = pytest.mark.gpu
ROOT = pathlib.Path(__file__).resolve().parent.parent
LINKED = ROOT / "oracle" / "_ref" / "test_fp4_gemm_linked"


def _write_case(g, tag, d: pathlib.Path):
    """The generator's output files (gen_fp4_gemm_testcase.py:73-79): packed codes, logical scales, fp32 Y_ref and
    dims.txt = "M N K\\nAg Bg\\n"."""
    M, N, K = [int(v) for v in g[f"{tag}__dims"]]
    g[f"{tag}__a_packed"].astype(np.uint8).tofile(d / "A_packed.bin")
    g[f"{tag}__b_packed"].astype(np.uint8).tofile(d / "B_packed.bin")
    g[f"{tag}__a_sf"].astype(np.uint8).tofile(d / "A_scales.bin")
    g[f"{tag}__b_sf"].astype(np.uint8).tofile(d / "B_scales.bin")
    g[f"{tag}__y_ref"].astype(np.float32).tofile(d / "Y_ref.bin")
    (d / "dims.txt").write_text(f"{M} {N} {K}\n{float(g[f'{tag}__ag']):.8e} {float(g[f'{tag}__bg']):.8e}\n")


@pytest.mark.parametrize("tag", ["default", "ragged"])
def test_reference_gemm_test_program_linked_to_this_library(golden, tag, tmp_path):
    require_gpu()
    if not LINKED.exists():
        pytest.skip("oracle/_ref/test_fp4_gemm_linked not built (needs the reference checkout at build time)")
    _write_case(golden("gemm_cases.npz"), tag, tmp_path)
    r = subprocess.run([str(LINKED), str(tmp_path)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and "GATE PASS" in r.stdout, r.stdout + r.stderr


def _cudart():
    # the CUDA runtime instance libnvfp4_b200.so uses (same soname, so the loader hands back the loaded copy)
    rt = ctypes.CDLL("libcudart.so.12")
    rt.cudaGetLastError.restype = ctypes.c_int
    return rt


def test_void_entry_points_leave_cuda_error_on_bad_arguments():
    p = require_gpu()
    L = p.lib()
    rt = _cudart()
    torch.cuda.synchronize()
    assert rt.cudaGetLastError() == 0
    buf = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    ptr = ctypes.c_void_p(buf.data_ptr())
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    q = getattr(L, "_Z26nvfp4_quantize_activationsPKfPhS1_iifP11CUstream_st")
    q.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_void_p]
    q(ptr, ptr, ptr, 4, 17, 1.0, stream)                       # K = 17: not a multiple of 16
    assert rt.cudaGetLastError() != 0
    assert rt.cudaGetLastError() == 0                          # read once, then clear (the runtime's semantics)
    w = getattr(L, "_Z10w4a16_gemmPfPKhS1_fPKviiiP11CUstream_st")
    w.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_float, ctypes.c_void_p] + [ctypes.c_int] * 3 + [ctypes.c_void_p]
    w(ptr, ptr, ptr, 1.0, ptr, 1, 64, 24, stream)               # K = 24
    assert rt.cudaGetLastError() != 0
    v = getattr(L, "_Z8fp4_gemvPfPKhS1_fPKviiP11CUstream_st")
    v.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_float, ctypes.c_void_p] + [ctypes.c_int] * 2 + [ctypes.c_void_p]
    v(None, ptr, ptr, 1.0, ptr, 64, 64, stream)                 # null output
    assert rt.cudaGetLastError() != 0
    x, codes, scales = (ctypes.c_void_p(buf.data_ptr() + off) for off in (0, 4096, 8192))
    q(x, codes, scales, 4, 64, 1.0, stream)                    # a valid call leaves the state clean
    torch.cuda.synchronize()
    assert rt.cudaGetLastError() == 0
