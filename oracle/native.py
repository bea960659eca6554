"""ctypes access to the oracle's native parts (TEST INFRASTRUCTURE ONLY): the C restatement and, when built,
the reference's own compiled sources in oracle/_ref/."""
from __future__ import annotations

import ctypes
import pathlib

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
_c = None
_ref = None
_P = ctypes.c_void_p


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(_P)


def lib():
    global _c
    if _c is None:
        path = HERE / "liborc_nvfp4.so"
        if not path.exists():
            from build import build_c_oracle  # type: ignore
            build_c_oracle()
        _c = ctypes.CDLL(str(path))
        _c.orc_quantize_rows_bf16.argtypes = [_P, ctypes.c_int, ctypes.c_int, ctypes.c_float, _P, _P]
        _c.orc_quantize_rows_f32.argtypes = [_P, ctypes.c_int, ctypes.c_int, ctypes.c_float, _P, _P]
        _c.orc_amax_bf16.argtypes = [_P, ctypes.c_longlong]
        _c.orc_amax_bf16.restype = ctypes.c_float
        _c.orc_swizzle_scales.argtypes = [_P, _P, ctypes.c_int, ctypes.c_int]
        _c.orc_num_threads.restype = ctypes.c_int
        _c.orc_dequantize_rows.argtypes = [_P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_float, _P]
    return _c


def quantize_bf16(bits: np.ndarray, gscale) -> tuple[np.ndarray, np.ndarray]:
    """bf16 bit patterns [M, K] -> (packed [M, K/2], logical scale bytes [M, K/16])."""
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    m, k = bits.shape
    packed = np.empty((m, k // 2), np.uint8)
    sf = np.empty((m, k // 16), np.uint8)
    lib().orc_quantize_rows_bf16(_ptr(bits), m, k, float(np.float32(gscale)), _ptr(packed), _ptr(sf))
    return packed, sf


def quantize_f32(x: np.ndarray, gscale) -> tuple[np.ndarray, np.ndarray]:
    x = np.ascontiguousarray(x, dtype=np.float32)
    m, k = x.shape
    packed = np.empty((m, k // 2), np.uint8)
    sf = np.empty((m, k // 16), np.uint8)
    lib().orc_quantize_rows_f32(_ptr(x), m, k, float(np.float32(gscale)), _ptr(packed), _ptr(sf))
    return packed, sf


def dequantize(packed: np.ndarray, sf_logical: np.ndarray, gscale) -> np.ndarray:
    """float64 [rows, K] = e2m1(code) * (e4m3(scale) / gscale); same values as nvfp4_oracle.dequantize, threaded."""
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    sf_logical = np.ascontiguousarray(sf_logical, dtype=np.uint8)
    rows, k = packed.shape[0], packed.shape[1] * 2
    assert sf_logical.shape == (rows, k // 16)
    out = np.empty((rows, k), np.float64)
    lib().orc_dequantize_rows(_ptr(packed), _ptr(sf_logical), rows, k, float(np.float32(gscale)), _ptr(out))
    return out


def amax_bf16(bits: np.ndarray) -> np.float32:
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    return np.float32(lib().orc_amax_bf16(_ptr(bits), bits.size))


def swizzle(logical: np.ndarray, outer: int, k: int) -> np.ndarray:
    logical = np.ascontiguousarray(logical, dtype=np.uint8)
    out = np.empty(((outer + 127) // 128) * ((k // 16 + 3) // 4) * 512, np.uint8)
    lib().orc_swizzle_scales(_ptr(logical), _ptr(out), outer, k)
    return out


def num_threads() -> int:
    return int(lib().orc_num_threads())


def ref_lib():
    """The reference's own compiled kernels/nvfp4_quant.cu + kernels/fp4_gemm.cu, or None if not built."""
    global _ref
    if _ref is None:
        path = HERE / "_ref" / "libref_nvfp4.so"
        if not path.exists():
            return None
        _ref = ctypes.CDLL(str(path))
        _ref.ref_scale_buffer_bytes.argtypes = [ctypes.c_int, ctypes.c_int]
        _ref.ref_scale_buffer_bytes.restype = ctypes.c_size_t
        _ref.ref_swizzle_scales.argtypes = [_P, _P, ctypes.c_int, ctypes.c_int]
        _ref.ref_quantize_activations.argtypes = [_P, _P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_float, _P]
        _ref.ref_nvfp4_gemm.argtypes = [_P, _P, _P, ctypes.c_float, _P, _P, ctypes.c_float,
                                        ctypes.c_int, ctypes.c_int, ctypes.c_int, _P]
        _ref.ref_nvfp4_gemm.restype = ctypes.c_int
        _ref.ref_w4a16_gemm.argtypes = [_P, _P, _P, ctypes.c_float, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P]
        _ref.ref_fp4_gemv.argtypes = [_P, _P, _P, ctypes.c_float, _P, ctypes.c_int, ctypes.c_int, _P]
    return _ref
