"""B200 (sm_100a) NVFP4 quantised-matmul path -- Python host mirror of the C ABI in include/nvfp4_b200.h.

The compute lives in libnvfp4_b200.so (hand-written CUDA for sm_100a, built in-tree by build.py).  This module only
binds it with ctypes; torch supplies device memory and streams.  There is no CPU or library fallback: if the
library is missing, or a call fails, an exception is raised.

Two layers:
* the reference's operator API under its own names and argument order (include/nvfp4_quant.h:10-11,
  include/fp4_gemm.h:13-35 of the reference): ``nvfp4_quantize_activations``, ``nvfp4_scale_buffer_bytes``,
  ``nvfp4_swizzle_scales``, ``nvfp4_gemm``, ``w4a16_gemm``, ``fp4_gemv`` -- device pointers as torch tensors;
* tensor-level helpers used by the tests and the benchmark: ``quantize``, ``amax``, ``gemm``, ``linear``, the MoE
  layer (``moe_route``, ``moe_forward`` with its chained and fused-norm forms, ``moe_layer`` with the router fused
  in, ``MoeExperts``), and the
  expert-parallel entry points (``ep_*`` over NCCL slots, ``ep_p2p_*`` over peer memory with the ``ipc_*`` set-up
  helpers; ``expert_parallel.py`` orchestrates them).
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
          -6: "ERR_TIMEOUT", -7: "ERR_ARG", -8: "ERR_SCRATCH"}
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
            "nvfp4b_hbm_read_stream": ([_P, ctypes.c_longlong, ctypes.c_int, _P], ctypes.c_int),
            "nvfp4b_gemm_set_tile_config": ([ctypes.c_int], ctypes.c_int),
            "nvfp4b_w4a16_gemm": ([_P, _P, _P, ctypes.c_float, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P],
                                  ctypes.c_int),
            "nvfp4b_amax_f32": ([_P, ctypes.c_longlong, _P, _P], ctypes.c_int),
            "nvfp4b_linear_workspace_bytes": ([ctypes.c_int, ctypes.c_int], ctypes.c_size_t),
            "nvfp4b_linear": ([_P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P, _P, _P, ctypes.c_float,
                               ctypes.c_float, ctypes.c_int, _P, ctypes.c_size_t, _P], ctypes.c_int),
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
    """max |x| of a bf16 or fp32 tensor as a 1-element fp32 device tensor."""
    assert x.dtype in (torch.bfloat16, torch.float32) and x.is_cuda and x.is_contiguous()
    if out is None:
        out = torch.empty(1, dtype=torch.float32, device=x.device)
    fn = lib().nvfp4b_amax_bf16 if x.dtype == torch.bfloat16 else lib().nvfp4b_amax_f32
    _check("amax", fn(_ptr(x), x.numel(), _ptr(out), _stream(stream)))
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


LINEAR_AUTO, LINEAR_W4A16, LINEAR_W4A4 = 0, 1, 2
LINEAR_W4A4_MIN_M = 128


def linear_workspace(M: int, K: int, device="cuda") -> torch.Tensor:
    return torch.empty(int(lib().nvfp4b_linear_workspace_bytes(M, K)), dtype=torch.uint8, device=device)


def linear(out, x, w, w_scales, w_scales_tiled, w_gscale: float, a_gscale: float | None = None,
           mode: int = LINEAR_AUTO, workspace=None, stream=None) -> torch.Tensor:
    """The reference's linear() (src/forward.cu:424-445): out[M, N] = x[M, K] @ W[N, K]^T, fp32 row-major in and
    out, W = NVFP4 codes [N, K/2] with raw scales [N, K/16] (W4A16 path) and/or their tile-layout copy (W4A4 path).
    a_gscale: static activation global scale; None = dynamic from the device amax of x."""
    M, K = x.shape
    N = w.shape[0]
    if workspace is None:
        workspace = linear_workspace(M, K, x.device)
    _check("linear", lib().nvfp4b_linear(_ptr(out), _ptr(x), M, N, K, _ptr(w), _ptr(w_scales), _ptr(w_scales_tiled),
                                         float(w_gscale), float(a_gscale or 0.0), mode, _ptr(workspace),
                                         workspace.numel(), _stream(stream)))
    return out


def set_gemm_tile_config(config: int) -> None:
    """0 = automatic, 1 = 128x256 tiles (4 stages, one accumulator), 2 = 128x128 tiles (6 stages, two),
    3 = 256x256 tiles on a CTA pair (tcgen05 cta_group::2, 5 stages)."""
    _check("set_gemm_tile_config", lib().nvfp4b_gemm_set_tile_config(config))


def read_device_error(reset: bool = True) -> int:
    return int(lib().nvfp4b_read_device_error(1 if reset else 0))


def hbm_read_stream(buf: torch.Tensor, rows: int, row_bytes: int) -> None:
    """Reads rows x row_bytes bytes of `buf` through the GEMMs' TMA path and discards them (roofline measurement)."""
    if buf.numel() * buf.element_size() < rows * row_bytes:
        raise ValueError("hbm_read_stream: buffer smaller than rows * row_bytes")
    _check("hbm_read_stream", lib().nvfp4b_hbm_read_stream(buf.data_ptr(), rows, row_bytes, _stream()))


# ----------------------------------------------------------------------------------------------------------------
# MoE (include/nvfp4_b200.h: nvfp4b_moe_*)
# ----------------------------------------------------------------------------------------------------------------

class _Experts(ctypes.Structure):
    _fields_ = [("num_experts", ctypes.c_int), ("hidden", ctypes.c_int), ("inter", ctypes.c_int),
                ("w13", _P), ("w13_scales", _P), ("w2", _P), ("w2_scales", _P),
                ("w1_gscale", _P), ("w3_gscale", _P), ("w2_gscale", _P), ("a2_gscale", _P)]


class _View(ctypes.Structure):
    _fields_ = [(n, _P) for n in ["m_tiles", "tile_expert", "seg_start", "seg_count", "row_token", "row_weight",
                                  "row_assign", "y", "dest", "a_codes", "a_scales", "h_codes", "h_scales"]]


def _moe_sigs():
    L = lib()
    if getattr(L, "_moe_ready", False):
        return L
    sig = {
        "nvfp4b_moe_workspace_bytes": ([ctypes.c_int] * 5, ctypes.c_size_t),
        "nvfp4b_moe_max_rows": ([ctypes.c_int] * 3, ctypes.c_int),
        "nvfp4b_moe_route": ([_P, ctypes.c_int, ctypes.c_int, _P, ctypes.c_int, ctypes.c_int, _P, ctypes.c_int, _P,
                              _P, _P, _P], ctypes.c_int),
        "nvfp4b_moe_route_noalloc": ([_P, ctypes.c_int, ctypes.c_int, _P, ctypes.c_int, ctypes.c_int, _P,
                                      ctypes.c_int, _P, _P, _P], ctypes.c_int),
        "nvfp4b_moe_forward": ([_P, ctypes.c_int, _P, _P, ctypes.c_int, ctypes.POINTER(_Experts), ctypes.c_float, _P,
                                _P, ctypes.c_int, _P, _P], ctypes.c_int),
        "nvfp4b_moe_forward_norm": ([_P, ctypes.c_int, _P, _P, ctypes.c_int, ctypes.POINTER(_Experts), _P,
                                     ctypes.c_float, ctypes.c_float, _P, ctypes.c_int, _P, _P], ctypes.c_int),
        "nvfp4b_moe_forward_chain": ([_P, ctypes.c_int, _P, _P, ctypes.c_int, ctypes.POINTER(_Experts),
                                      ctypes.c_float, _P, _P, ctypes.c_int, _P, _P, _P, _P], ctypes.c_int),
        "nvfp4b_moe_layer": ([_P, ctypes.c_int, _P, ctypes.c_int, _P, ctypes.c_int, ctypes.POINTER(_Experts),
                              ctypes.c_float, _P, _P, ctypes.c_int, _P, _P, _P, _P, _P, _P], ctypes.c_int),
        "nvfp4b_moe_calibrate": ([_P, ctypes.c_int, _P, _P, ctypes.c_int, ctypes.POINTER(_Experts), ctypes.c_float,
                                  _P, _P, _P, _P], ctypes.c_int),
        "nvfp4b_moe_workspace_view": ([_P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       ctypes.POINTER(_View)], ctypes.c_int),
        "nvfp4b_moe_pack_expert": ([_P] * 6 + [ctypes.c_int, ctypes.c_int] + [_P] * 5, ctypes.c_int),
        "nvfp4b_moe_dispatch": ([_P, ctypes.c_int, _P, _P, ctypes.c_int, ctypes.POINTER(_Experts), ctypes.c_float,
                                 _P, _P, _P], ctypes.c_int),
        "nvfp4b_moe_gate_up": ([ctypes.c_int, ctypes.c_int, ctypes.POINTER(_Experts), ctypes.c_float, _P, _P, _P],
                               ctypes.c_int),
        "nvfp4b_moe_down": ([ctypes.c_int, ctypes.c_int, _P, ctypes.POINTER(_Experts), _P, ctypes.c_int, _P, _P],
                            ctypes.c_int),
    }
    for name, (args, res) in sig.items():
        f = getattr(L, name)
        f.argtypes = args
        f.restype = res
    L._moe_ready = True
    return L


class MoeExperts:
    """Device arena of E experts in the layout nvfp4b_moe_forward reads (see nvfp4b_moe_experts)."""

    def __init__(self, E: int, H: int, I: int, device="cuda"):
        self.E, self.H, self.I = E, H, I
        dev = torch.device(device)
        self.w13 = torch.empty((E, 2 * I, H // 2), dtype=torch.uint8, device=dev)
        self.w13_sf_bytes = nvfp4_scale_buffer_bytes(2 * I, H)
        self.w13_scales = torch.zeros((E, self.w13_sf_bytes), dtype=torch.uint8, device=dev)
        self.w2 = torch.empty((E, H, I // 2), dtype=torch.uint8, device=dev)
        self.w2_sf_bytes = nvfp4_scale_buffer_bytes(H, I)
        self.w2_scales = torch.zeros((E, self.w2_sf_bytes), dtype=torch.uint8, device=dev)
        self.w1_gscale = torch.ones(E, dtype=torch.float32, device=dev)
        self.w3_gscale = torch.ones(E, dtype=torch.float32, device=dev)
        self.w2_gscale = torch.ones(E, dtype=torch.float32, device=dev)
        self.a2_gscale = torch.ones(E, dtype=torch.float32, device=dev)

    def pack(self, e: int, gate, gate_sf_logical, up, up_sf_logical, down, down_sf_logical, stream=None):
        """Checkpoint layout (codes [N, K/2], logical e4m3 scales [N, K/16], all device uint8) -> arena slot e."""
        _check("moe_pack_expert", _moe_sigs().nvfp4b_moe_pack_expert(
            _ptr(gate), _ptr(gate_sf_logical), _ptr(up), _ptr(up_sf_logical), _ptr(down), _ptr(down_sf_logical),
            self.H, self.I, _ptr(self.w13[e]), _ptr(self.w13_scales[e]), _ptr(self.w2[e]), _ptr(self.w2_scales[e]),
            _stream(stream)))

    def slice(self, e0: int, e1: int) -> "MoeExperts":
        """Experts [e0, e1) as an arena of their own (views, no copy): the local shard of an expert-parallel rank."""
        v = object.__new__(MoeExperts)
        v.E, v.H, v.I = e1 - e0, self.H, self.I
        v.w13_sf_bytes, v.w2_sf_bytes = self.w13_sf_bytes, self.w2_sf_bytes
        for name in ("w13", "w13_scales", "w2", "w2_scales", "w1_gscale", "w3_gscale", "w2_gscale", "a2_gscale"):
            setattr(v, name, getattr(self, name)[e0:e1])
        return v

    def struct(self) -> _Experts:
        return _Experts(self.E, self.H, self.I, _ptr(self.w13), _ptr(self.w13_scales), _ptr(self.w2),
                        _ptr(self.w2_scales), _ptr(self.w1_gscale), _ptr(self.w3_gscale), _ptr(self.w2_gscale),
                        _ptr(self.a2_gscale))


def moe_workspace(T: int, H: int, I: int, E: int, topk: int, device="cuda") -> torch.Tensor:
    n = _moe_sigs().nvfp4b_moe_workspace_bytes(T, H, I, E, topk)
    return torch.empty(n, dtype=torch.uint8, device=device)


def moe_max_rows(T: int, E: int, topk: int) -> int:
    return int(_moe_sigs().nvfp4b_moe_max_rows(T, E, topk))


def moe_route(x, proj, topk: int, workspace, per_expert_scale=None, norm: bool = False, ids=None, weights=None,
              stream=None):
    """Router: x [T, H] bf16, proj [E, H] bf16 -> (ids [T, topk] int32, weights [T, topk] fp32)."""
    T, H = x.shape
    E = proj.shape[0]
    if ids is None:
        ids = torch.empty((T, topk), dtype=torch.int32, device=x.device)
    if weights is None:
        weights = torch.empty((T, topk), dtype=torch.float32, device=x.device)
    _check("moe_route", _moe_sigs().nvfp4b_moe_route(_ptr(x), T, H, _ptr(proj), E, topk, _ptr(per_expert_scale),
                                                      1 if norm else 0, _ptr(ids), _ptr(weights), _ptr(workspace),
                                                      _stream(stream)))
    return ids, weights


def moe_route_noalloc(x, proj, topk: int, ids, weights, per_expert_scale=None, norm: bool = False, stream=None):
    """moe_route without a workspace: the library's fixed per-device scratch holds the partial logits (T * E must be
    <= 262144).  ids/weights are caller-provided, so the call allocates nothing; calls that overlap in time on one
    device must not be issued (they share the scratch)."""
    T, H = x.shape
    E = proj.shape[0]
    _check("moe_route_noalloc", _moe_sigs().nvfp4b_moe_route_noalloc(
        _ptr(x), T, H, _ptr(proj), E, topk, _ptr(per_expert_scale), 1 if norm else 0, _ptr(ids), _ptr(weights),
        _stream(stream)))
    return ids, weights


MOE_ACCUMULATE, MOE_ATOMIC = 1, 2


def moe_forward(x, ids, weights, experts: MoeExperts, workspace, in_gscale: float | None = None, in_amax=None,
                out=None, accumulate: bool = False, atomic: bool = False, x_next=None, amax_next=None, stream=None):
    """MoE layer (dispatch -> gate/up -> down + combine) -> out [T, H] fp32.  With x_next (bf16 [T, H]) and amax_next
    (fp32 [1]) the combine also writes bf16(out) and its max |.| there (nvfp4b_moe_forward_chain)."""
    T = x.shape[0]
    topk = ids.shape[1]
    if out is None:
        out = torch.empty((T, experts.H), dtype=torch.float32, device=x.device)
    st = experts.struct()
    flags = (MOE_ACCUMULATE if accumulate else 0) | (MOE_ATOMIC if atomic else 0)
    if x_next is not None:
        _check("moe_forward_chain", _moe_sigs().nvfp4b_moe_forward_chain(
            _ptr(x), T, _ptr(ids), _ptr(weights), topk, ctypes.byref(st), float(in_gscale or 0.0), _ptr(in_amax),
            _ptr(out), flags, _ptr(workspace), _ptr(x_next), _ptr(amax_next), _stream(stream)))
        return out
    _check("moe_forward", _moe_sigs().nvfp4b_moe_forward(
        _ptr(x), T, _ptr(ids), _ptr(weights), topk, ctypes.byref(st), float(in_gscale or 0.0), _ptr(in_amax),
        _ptr(out), flags, _ptr(workspace), _stream(stream)))
    return out


def moe_layer(x, proj, topk: int, experts: MoeExperts, workspace, ids=None, weights=None, per_expert_scale=None,
              norm: bool = False, in_gscale: float | None = None, in_amax=None, out=None, accumulate: bool = False,
              atomic: bool = False, x_next=None, amax_next=None, stream=None):
    """Router + MoE layer in one call (nvfp4b_moe_layer): the same as moe_route followed by moe_forward (with
    x_next / amax_next: the chained form).  Returns out; ids [T, topk] / weights [T, topk] receive the routing."""
    T = x.shape[0]
    if out is None:
        out = torch.empty((T, experts.H), dtype=torch.float32, device=x.device)
    if ids is None:
        ids = torch.empty((T, topk), dtype=torch.int32, device=x.device)
    if weights is None:
        weights = torch.empty((T, topk), dtype=torch.float32, device=x.device)
    st = experts.struct()
    flags = (MOE_ACCUMULATE if accumulate else 0) | (MOE_ATOMIC if atomic else 0)
    _check("moe_layer", _moe_sigs().nvfp4b_moe_layer(
        _ptr(x), T, _ptr(proj), topk, _ptr(per_expert_scale), 1 if norm else 0, ctypes.byref(st),
        float(in_gscale or 0.0), _ptr(in_amax), _ptr(out), flags, _ptr(ids), _ptr(weights), _ptr(workspace),
        _ptr(x_next), _ptr(amax_next), _stream(stream)))
    return out


def moe_forward_norm(x, ids, weights, experts: MoeExperts, workspace, norm_weight, in_gscale: float,
                     eps: float = 1e-6, out=None, accumulate: bool = False, stream=None):
    """MoE layer whose input rows are RMS-normalised (x * rsqrt(mean(x^2) + eps) * norm_weight, fp32) inside the
    quantise-dispatch; static activation global scale in_gscale."""
    T = x.shape[0]
    topk = ids.shape[1]
    if out is None:
        out = torch.empty((T, experts.H), dtype=torch.float32, device=x.device)
    st = experts.struct()
    _check("moe_forward_norm", _moe_sigs().nvfp4b_moe_forward_norm(
        _ptr(x), T, _ptr(ids), _ptr(weights), topk, ctypes.byref(st), _ptr(norm_weight), float(eps),
        float(in_gscale), _ptr(out), MOE_ACCUMULATE if accumulate else 0, _ptr(workspace), _stream(stream)))
    return out


def moe_dispatch(x, ids, weights, experts: MoeExperts, workspace, in_gscale=None, in_amax=None, stream=None):
    st = experts.struct()
    _check("moe_dispatch", _moe_sigs().nvfp4b_moe_dispatch(
        _ptr(x), x.shape[0], _ptr(ids), _ptr(weights), ids.shape[1], ctypes.byref(st), float(in_gscale or 0.0),
        _ptr(in_amax), _ptr(workspace), _stream(stream)))


def moe_gate_up(T: int, topk: int, experts: MoeExperts, workspace, in_gscale=None, in_amax=None, stream=None):
    st = experts.struct()
    _check("moe_gate_up", _moe_sigs().nvfp4b_moe_gate_up(T, topk, ctypes.byref(st), float(in_gscale or 0.0),
                                                          _ptr(in_amax), _ptr(workspace), _stream(stream)))


def moe_down(T: int, topk: int, weights, experts: MoeExperts, out, workspace, accumulate: bool = False,
             atomic: bool = False, stream=None):
    st = experts.struct()
    flags = (MOE_ACCUMULATE if accumulate else 0) | (MOE_ATOMIC if atomic else 0)
    _check("moe_down", _moe_sigs().nvfp4b_moe_down(T, topk, _ptr(weights), ctypes.byref(st), _ptr(out), flags,
                                                    _ptr(workspace), _stream(stream)))


def moe_calibrate(x, ids, weights, experts: MoeExperts, workspace, in_gscale: float | None = None, in_amax=None,
                  stream=None):
    """Per-expert max |h| of the gate/up output over the routed rows -> [E] fp32 device tensor."""
    T = x.shape[0]
    h_amax = torch.empty(experts.E, dtype=torch.float32, device=x.device)
    st = experts.struct()
    _check("moe_calibrate", _moe_sigs().nvfp4b_moe_calibrate(
        _ptr(x), T, _ptr(ids), _ptr(weights), ids.shape[1], ctypes.byref(st), float(in_gscale or 0.0),
        _ptr(in_amax), _ptr(h_amax), _ptr(workspace), _stream(stream)))
    return h_amax


def moe_view(workspace, T: int, H: int, I: int, E: int, topk: int) -> dict:
    """Tensors aliasing the dispatch plan and NVFP4 buffers inside a MoE workspace (for tests and debugging)."""
    v = _View()
    _check("moe_view", _moe_sigs().nvfp4b_moe_workspace_view(_ptr(workspace), T, H, I, E, topk, ctypes.byref(v)))
    rows = moe_max_rows(T, E, topk)
    base = workspace.data_ptr()

    def sl(ptr, nbytes, dtype):
        off = ptr - base
        return workspace[off:off + nbytes].view(dtype)

    return {
        "m_tiles": sl(v.m_tiles, 4, torch.int32),
        "tile_expert": sl(v.tile_expert, (rows // 128) * 4, torch.int32),
        "seg_start": sl(v.seg_start, E * 4, torch.int32),
        "seg_count": sl(v.seg_count, E * 4, torch.int32),
        "row_token": sl(v.row_token, rows * 4, torch.int32),
        "row_weight": sl(v.row_weight, rows * 4, torch.float32),
        "row_assign": sl(v.row_assign, rows * 4, torch.int32),
        "dest": sl(v.dest, T * topk * 4, torch.int32),
        "a_codes": sl(v.a_codes, rows * H // 2, torch.uint8).view(rows, H // 2),
        "a_scales": sl(v.a_scales, nvfp4_scale_buffer_bytes(rows, H), torch.uint8),
        "h_codes": sl(v.h_codes, rows * I // 2, torch.uint8).view(rows, I // 2),
        "h_scales": sl(v.h_scales, nvfp4_scale_buffer_bytes(rows, I), torch.uint8),
        "y": sl(v.y, T * topk * H * 2, torch.float16).view(T * topk, H),
        "rows": rows,
    }


# ---- expert parallelism (the collectives are torch.distributed's; see expert_parallel.py) ----------------------

def _ep_sigs():
    L = _moe_sigs()
    if getattr(L, "_ep_ready", False):
        return L
    sig = {
        "nvfp4b_ep_record_bytes": ([ctypes.c_int], ctypes.c_size_t),
        "nvfp4b_ep_dispatch": ([_P, ctypes.c_int, ctypes.c_int, _P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                ctypes.c_int, ctypes.c_float, _P, _P, _P, _P, _P, _P], ctypes.c_int),
        "nvfp4b_ep_expert_forward": ([_P, ctypes.c_int, ctypes.c_int, _P, ctypes.POINTER(_Experts), _P, _P],
                                     ctypes.c_int),
        "nvfp4b_ep_combine": ([_P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P, _P, ctypes.c_int, _P],
                              ctypes.c_int),
    }
    for name, (args, res) in sig.items():
        f = getattr(L, name)
        f.argtypes = args
        f.restype = res
    L._ep_ready = True
    return L


def ep_record_bytes(H: int) -> int:
    return int(_ep_sigs().nvfp4b_ep_record_bytes(H))


def ep_dispatch(x, ids, weights, E: int, G: int, capacity: int, workspace, records, send_counts, overflow,
                in_gscale: float | None = None, in_amax=None, stream=None) -> None:
    """Source side: records [G * capacity, ep_record_bytes(H)] uint8, destination-major slots; send_counts int32
    [G]; overflow int32 [1] (or-ed with 1 when a destination gets more than capacity records)."""
    T, H = x.shape
    topk = ids.shape[1]
    _check("ep_dispatch", _ep_sigs().nvfp4b_ep_dispatch(
        _ptr(x), T, H, _ptr(ids), _ptr(weights), topk, E, G, capacity, float(in_gscale or 0.0), _ptr(in_amax),
        _ptr(workspace), _ptr(records), _ptr(send_counts), _ptr(overflow), _stream(stream)))


def ep_expert_forward(records, G: int, capacity: int, recv_counts, experts: MoeExperts, workspace, stream=None):
    """Expert side: the weighted fp16 output rows of the G * capacity received slots, a view [G * capacity, H] of
    the workspace (rows of empty slots are undefined)."""
    ex = experts.struct()
    _check("ep_expert_forward", _ep_sigs().nvfp4b_ep_expert_forward(
        _ptr(records), G, capacity, _ptr(recv_counts), ctypes.byref(ex), _ptr(workspace), _stream(stream)))
    return moe_view(workspace, G * capacity, experts.H, experts.I, experts.E, 1)["y"]


def ep_combine(y_back, T: int, topk: int, E: int, workspace, out, accumulate: bool = False, stream=None):
    """Source side: out[t] (+)= slot-ordered sum of the rows returned for token t."""
    H = out.shape[1]
    _check("ep_combine", _ep_sigs().nvfp4b_ep_combine(
        _ptr(y_back), T, H, topk, E, _ptr(workspace), _ptr(out), MOE_ACCUMULATE if accumulate else 0,
        _stream(stream)))
    return out


# ----------------------------------------------------------------------------------------------------------------
# Expert parallelism over NVLink peer memory (include/nvfp4_b200.h: nvfp4b_ep_p2p_*, nvfp4b_ipc_*)
# ----------------------------------------------------------------------------------------------------------------

class EpPeers(ctypes.Structure):
    """nvfp4b_ep_peers: this rank's view of every rank's exchange buffers (device pointers)."""
    _fields_ = [("rank", ctypes.c_int), ("G", ctypes.c_int), ("capacity", ctypes.c_int),
                ("recv", _P), ("back", _P), ("counts", _P), ("flags", _P),
                ("my_recv", _P), ("my_back", _P), ("my_counts", _P), ("my_flags", _P), ("state", _P)]


def _p2p_sigs():
    L = _ep_sigs()
    if getattr(L, "_p2p_ready", False):
        return L
    PP = ctypes.POINTER(EpPeers)
    sig = {
        "nvfp4b_ep_p2p_buffer_bytes": ([ctypes.c_int, ctypes.c_int, ctypes.c_int, _P], ctypes.c_size_t),
        "nvfp4b_ep_p2p_dispatch": ([_P, ctypes.c_int, ctypes.c_int, _P, _P, ctypes.c_int, ctypes.c_int,
                                    ctypes.c_float, _P, _P, PP, _P, _P], ctypes.c_int),
        "nvfp4b_ep_p2p_expert_forward": ([ctypes.POINTER(_Experts), _P, PP, _P], ctypes.c_int),
        "nvfp4b_ep_p2p_combine": ([ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P, PP, _P,
                                   ctypes.c_int, _P], ctypes.c_int),
        "nvfp4b_ep_p2p_combine_chain": ([ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P, PP, _P,
                                         ctypes.c_int, _P, _P, _P], ctypes.c_int),
        "nvfp4b_ep_set_peer_wait_ns": ([ctypes.c_ulonglong], ctypes.c_int),
        "nvfp4b_ep_p2p_layer": ([_P, ctypes.c_int, _P, ctypes.c_int, _P, ctypes.c_int, ctypes.c_int,
                                 ctypes.POINTER(_Experts), ctypes.c_float, _P, _P, ctypes.c_int, _P, _P, _P, _P, PP,
                                 _P, _P, _P, _P], ctypes.c_int),
        "nvfp4b_ep_p2p_state": ([PP, _P], ctypes.c_int),
        "nvfp4b_ep_p2p_recv_counts": ([PP, _P], ctypes.c_int),
        "nvfp4b_ipc_alloc": ([ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
        "nvfp4b_ipc_free": ([_P], ctypes.c_int),
        "nvfp4b_ipc_handle": ([_P, _P], ctypes.c_int),
        "nvfp4b_ipc_open": ([_P, ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
        "nvfp4b_ipc_close": ([_P], ctypes.c_int),
    }
    for name, (args, res) in sig.items():
        f = getattr(L, name)
        f.argtypes = args
        f.restype = res
    L._p2p_ready = True
    return L


def ep_p2p_buffer_layout(G: int, capacity: int, H: int):
    """(bytes, [offset of receive slots, return rows, counts, flags, state]) of one rank's exchange buffers."""
    off = (ctypes.c_size_t * 5)()
    n = int(_p2p_sigs().nvfp4b_ep_p2p_buffer_bytes(G, capacity, H, off))
    if n == 0:
        raise NvFp4Error("ep_p2p_buffer_bytes", -1)
    return n, [int(v) for v in off]


def ep_set_peer_wait_ns(ns: int) -> None:
    """Bound (nanoseconds, per flag) of the waits on other ranks' flags in kernels launched from now on; 0 restores
    the default of 10 s.  A wait that runs out records device error 4 (read_device_error) instead of hanging."""
    _check("ep_set_peer_wait_ns", _p2p_sigs().nvfp4b_ep_set_peer_wait_ns(int(ns)))


PEER_TIMEOUT = 4      # device error code of an expired wait on another rank's flag


def ep_p2p_state(peers: EpPeers) -> list[int]:
    """Debug read of a rank's 4 private words (synchronous)."""
    out = (ctypes.c_uint * 4)()
    _check("ep_p2p_state", _p2p_sigs().nvfp4b_ep_p2p_state(ctypes.byref(peers), out))
    return list(out)


def ep_p2p_recv_counts(peers: EpPeers) -> list[int]:
    """Debug read of the records a rank received from each source in its last layer (synchronous)."""
    out = (ctypes.c_int * peers.G)()
    _check("ep_p2p_recv_counts", _p2p_sigs().nvfp4b_ep_p2p_recv_counts(ctypes.byref(peers), out))
    return list(out)


def ipc_alloc(nbytes: int) -> int:
    p = ctypes.c_void_p()
    _check("ipc_alloc", _p2p_sigs().nvfp4b_ipc_alloc(nbytes, ctypes.byref(p)))
    return int(p.value)


def ipc_free(ptr: int) -> None:
    _check("ipc_free", _p2p_sigs().nvfp4b_ipc_free(ptr))


def ipc_handle(ptr: int) -> bytes:
    buf = ctypes.create_string_buffer(64)
    _check("ipc_handle", _p2p_sigs().nvfp4b_ipc_handle(ptr, buf))
    return buf.raw


def ipc_open(handle: bytes) -> int:
    p = ctypes.c_void_p()
    buf = ctypes.create_string_buffer(bytes(handle), 64)
    _check("ipc_open", _p2p_sigs().nvfp4b_ipc_open(buf, ctypes.byref(p)))
    return int(p.value)


def ipc_close(ptr: int) -> None:
    _check("ipc_close", _p2p_sigs().nvfp4b_ipc_close(ptr))


def ep_p2p_dispatch(x, ids, weights, E: int, workspace, peers: EpPeers, overflow, in_gscale: float | None = None,
                    in_amax=None, stream=None) -> None:
    """Source side over peer memory: records into the destination ranks' receive slots, flags raised."""
    T, H = x.shape
    topk = ids.shape[1]
    _check("ep_p2p_dispatch", _p2p_sigs().nvfp4b_ep_p2p_dispatch(
        _ptr(x), T, H, _ptr(ids), _ptr(weights), topk, E, float(in_gscale or 0.0), _ptr(in_amax), _ptr(workspace),
        ctypes.byref(peers), _ptr(overflow), _stream(stream)))


def ep_p2p_expert_forward(experts: MoeExperts, workspace, peers: EpPeers, stream=None) -> None:
    """Expert side over peer memory: waits for the records, rows stored into the source ranks' return rows."""
    ex = experts.struct()
    _check("ep_p2p_expert_forward", _p2p_sigs().nvfp4b_ep_p2p_expert_forward(
        ctypes.byref(ex), _ptr(workspace), ctypes.byref(peers), _stream(stream)))


def ep_p2p_layer(x, proj, topk: int, E: int, experts: MoeExperts, src_ws, exp_ws, peers: EpPeers, overflow, ids,
                 weights, out, accumulate: bool = False, in_gscale: float | None = None, in_amax=None,
                 per_expert_scale=None, norm: bool = False, x_next=None, amax_next=None, stream=None):
    """Router + one expert-parallel layer on this rank (nvfp4b_ep_p2p_layer): route, dispatch over peer memory, the
    local experts, combine (+ the chained next input and amax)."""
    T = x.shape[0]
    ex = experts.struct()
    _check("ep_p2p_layer", _p2p_sigs().nvfp4b_ep_p2p_layer(
        _ptr(x), T, _ptr(proj), topk, _ptr(per_expert_scale), 1 if norm else 0, E, ctypes.byref(ex),
        float(in_gscale or 0.0), _ptr(in_amax), _ptr(out), MOE_ACCUMULATE if accumulate else 0, _ptr(ids),
        _ptr(weights), _ptr(src_ws), _ptr(exp_ws), ctypes.byref(peers), _ptr(overflow), _ptr(x_next),
        _ptr(amax_next), _stream(stream)))
    return out


def ep_p2p_combine(T: int, topk: int, E: int, workspace, peers: EpPeers, out, accumulate: bool = False,
                   x_next=None, amax_next=None, stream=None):
    """Source side over peer memory: waits for the rows, slot-ordered sum into out (+ the chained bf16 copy and
    amax when x_next / amax_next are given)."""
    H = out.shape[1]
    flags = MOE_ACCUMULATE if accumulate else 0
    if x_next is not None:
        _check("ep_p2p_combine_chain", _p2p_sigs().nvfp4b_ep_p2p_combine_chain(
            T, H, topk, E, _ptr(workspace), ctypes.byref(peers), _ptr(out), flags, _ptr(x_next), _ptr(amax_next),
            _stream(stream)))
        return out
    _check("ep_p2p_combine", _p2p_sigs().nvfp4b_ep_p2p_combine(
        T, H, topk, E, _ptr(workspace), ctypes.byref(peers), _ptr(out), flags, _stream(stream)))
    return out
