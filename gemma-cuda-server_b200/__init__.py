"""B200 (sm_100a) NVFP4 quantised-matmul path -- Python host mirror of the C ABI in include/nvfp4_b200.h.

The compute lives in libnvfp4_b200.so (hand-written CUDA for sm_100a, built in-tree by build.py).  This module only
binds it with ctypes; torch supplies device memory and streams.  There is no CPU or library fallback: if the
library is missing, or a call fails, an exception is raised.

Two layers:
* the reference's operator API under its own names and argument order (include/nvfp4_quant.h:10-11,
  include/fp4_gemm.h:13-35 of the reference): ``nvfp4_quantize_activations``, ``nvfp4_scale_buffer_bytes``,
  ``nvfp4_swizzle_scales``, ``nvfp4_gemm``, ``w4a16_gemm``, ``fp4_gemv`` -- device pointers as torch tensors;
* tensor-level helpers used by the tests and the benchmark: ``quantize``, ``amax``, ``gemm``.
"""
from __future__ import annotations

import ctypes
import pathlib

import torch

PKG = pathlib.Path(__file__).resolve().parent
LIB_PATH = PKG / "libnvfp4_b200.so"

_P = ctypes.c_void_p
_lib = None

STATUS = {0: "OK", -1: "ERR_SHAPE", -2: "ERR_ALIGN", -3: "ERR_NULL", -4: "ERR_CUDA", -5: "ERR_ARCH",
          -6: "ERR_TIMEOUT", -7: "ERR_ARG"}
OUT_BF16_ROWMAJOR, OUT_F32_COLMAJOR, OUT_F32_ROWMAJOR = 0, 1, 2


class NvFp4Error(RuntimeError):
    def __init__(self, fn: str, code: int):
        self.code = code
        extra = ""
        if code == -4 and _lib is not None:
            extra = f" (cudaError {_lib.nvfp4b_last_cuda_error()})"
        super().__init__(f"{fn}: {STATUS.get(code, code)}{extra}")


def lib() -> ctypes.CDLL:
    """The loaded library; raises if it has not been built (no fallback exists)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH.name} is not built; run build.py (or __graft_entry__.build())")
        L = ctypes.CDLL(str(LIB_PATH))
        sig = {
            "nvfp4b_version": ([], ctypes.c_char_p),
            "nvfp4b_last_cuda_error": ([], ctypes.c_int),
            "nvfp4b_scale_buffer_bytes": ([ctypes.c_int, ctypes.c_int], ctypes.c_size_t),
            "nvfp4b_amax_bf16": ([_P, ctypes.c_longlong, _P, _P], ctypes.c_int),
            "nvfp4b_quantize_bf16": ([_P, ctypes.c_int, ctypes.c_int, ctypes.c_float, _P, _P, _P, _P], ctypes.c_int),
            "nvfp4b_quantize_f32": ([_P, ctypes.c_int, ctypes.c_int, ctypes.c_float, _P, _P, _P, _P], ctypes.c_int),
            "nvfp4b_swizzle_scales": ([_P, _P, ctypes.c_int, ctypes.c_int, _P], ctypes.c_int),
            "nvfp4b_gemm": ([_P, _P, ctypes.c_float, _P, _P, _P, ctypes.c_float, ctypes.c_int, ctypes.c_int,
                             ctypes.c_int, _P, ctypes.c_int, ctypes.c_longlong, _P], ctypes.c_int),
            "nvfp4b_read_device_error": ([ctypes.c_int], ctypes.c_int),
            "nvfp4b_w4a16_gemm": ([_P, _P, _P, ctypes.c_float, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P],
                                  ctypes.c_int),
        }
        for name, (args, res) in sig.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _lib = L
    return _lib


def _ptr(t):
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()


def _stream(stream=None):
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def _check(fn: str, code: int) -> None:
    if code != 0:
        raise NvFp4Error(fn, code)


# ----------------------------------------------------------------------------------------------------------------
# Reference operator API (same names / argument meaning as the reference's C++ headers)
# ----------------------------------------------------------------------------------------------------------------

def nvfp4_scale_buffer_bytes(outer: int, K: int) -> int:
    """include/fp4_gemm.h:13 of the reference."""
    return int(lib().nvfp4b_scale_buffer_bytes(outer, K))


def nvfp4_quantize_activations(dX, dPacked, dScalesSwz, M: int, K: int, gscale: float, stream=None) -> None:
    """include/nvfp4_quant.h:10-11 of the reference: fp32 [M, K] -> codes + tile-layout scales (static gscale)."""
    _check("nvfp4_quantize_activations",
           lib().nvfp4b_quantize_f32(_ptr(dX), M, K, float(gscale), None, _ptr(dPacked), _ptr(dScalesSwz),
                                     _stream(stream)))


def nvfp4_swizzle_scales(logical, outer: int, K: int):
    """include/fp4_gemm.h:17 of the reference, on the device: logical [outer, K/16] uint8 -> tile layout."""
    out = torch.empty(nvfp4_scale_buffer_bytes(outer, K), dtype=torch.uint8, device=logical.device)
    _check("nvfp4_swizzle_scales", lib().nvfp4b_swizzle_scales(_ptr(logical), _ptr(out), outer, K, _stream()))
    return out


def nvfp4_gemm(dD, dA_packed, dA_scales_swz, a_gscale: float, dB_packed, dB_scales_swz, b_gscale: float,
               M: int, N: int, K: int, stream=None) -> int:
    """include/fp4_gemm.h:31-35 of the reference: fp32 column-major D (ld = M).  Returns 0 on success."""
    return int(lib().nvfp4b_gemm(_ptr(dA_packed), _ptr(dA_scales_swz), float(a_gscale), None, _ptr(dB_packed),
                                 _ptr(dB_scales_swz), float(b_gscale), M, N, K, _ptr(dD), OUT_F32_COLMAJOR, M,
                                 _stream(stream)))


def w4a16_gemm(out, wp, ws, w_gscale: float, x16, M: int, N: int, K: int, stream=None) -> None:
    """include/fp4_gemm.h:21-22 of the reference (any M here)."""
    _check("w4a16_gemm", lib().nvfp4b_w4a16_gemm(_ptr(out), _ptr(wp), _ptr(ws), float(w_gscale), _ptr(x16), M, N, K,
                                                 _stream(stream)))


def fp4_gemv(y, wp, ws, w_gscale: float, x16, N: int, K: int, stream=None) -> None:
    """include/fp4_gemm.h:26-27 of the reference."""
    w4a16_gemm(y, wp, ws, w_gscale, x16, 1, N, K, stream)


# ----------------------------------------------------------------------------------------------------------------
# Tensor-level helpers
# ----------------------------------------------------------------------------------------------------------------

def amax(x: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """max |x| of a bf16 tensor as a 1-element fp32 device tensor."""
    assert x.dtype == torch.bfloat16 and x.is_cuda and x.is_contiguous()
    if out is None:
        out = torch.empty(1, dtype=torch.float32, device=x.device)
    _check("nvfp4b_amax_bf16", lib().nvfp4b_amax_bf16(_ptr(x), x.numel(), _ptr(out), _stream(stream)))
    return out


def quantize(x: torch.Tensor, gscale: float | None = None, amax_dev: torch.Tensor | None = None,
             packed: torch.Tensor | None = None, scales: torch.Tensor | None = None, stream=None):
    """NVFP4-quantise a row-major bf16 or fp32 [M, K] device tensor.

    Exactly one of ``gscale`` (static) or ``amax_dev`` (device amax -> gscale = 2688/amax on the device) is given.
    Returns (codes [M, K/2] uint8, tile-layout scales uint8).
    """
    assert x.is_cuda and x.dim() == 2 and x.is_contiguous()
    assert (gscale is None) != (amax_dev is None), "give gscale or amax_dev"
    M, K = x.shape
    if packed is None:
        packed = torch.empty((M, K // 2), dtype=torch.uint8, device=x.device)
    if scales is None:
        scales = torch.empty(nvfp4_scale_buffer_bytes(M, K), dtype=torch.uint8, device=x.device)
    fn = lib().nvfp4b_quantize_bf16 if x.dtype == torch.bfloat16 else lib().nvfp4b_quantize_f32
    assert x.dtype in (torch.bfloat16, torch.float32)
    _check("quantize", fn(_ptr(x), M, K, float(gscale or 0.0), _ptr(amax_dev), _ptr(packed), _ptr(scales),
                          _stream(stream)))
    return packed, scales


def gemm(a, a_scales, a_dequant: float, b, b_scales, b_dequant: float, out: torch.Tensor | None = None,
         out_kind: int = OUT_BF16_ROWMAJOR, a_amax: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """D = a_dequant * b_dequant * A @ B^T on the NVFP4 tensor cores.  A: codes [M, K/2]; B: codes [N, K/2]."""
    M, K = a.shape[0], a.shape[1] * 2
    N = b.shape[0]
    if out is None:
        if out_kind == OUT_BF16_ROWMAJOR:
            out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
        elif out_kind == OUT_F32_ROWMAJOR:
            out = torch.empty((M, N), dtype=torch.float32, device=a.device)
        else:
            out = torch.empty((N, M), dtype=torch.float32, device=a.device)   # column-major [M, N]
    ldd = M if out_kind == OUT_F32_COLMAJOR else N
    _check("gemm", lib().nvfp4b_gemm(_ptr(a), _ptr(a_scales), float(a_dequant), _ptr(a_amax), _ptr(b),
                                     _ptr(b_scales), float(b_dequant), M, N, K, _ptr(out), out_kind, ldd,
                                     _stream(stream)))
    return out


def read_device_error(reset: bool = True) -> int:
    return int(lib().nvfp4b_read_device_error(1 if reset else 0))
