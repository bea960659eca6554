"""CPU oracle for the NVFP4 quantized-matmul path.  TEST INFRASTRUCTURE ONLY.

This module restates, in vectorised numpy, the reference's own NVFP4 arithmetic so that the CUDA path can be
checked against it.  It is never on the product path: only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` import it, and only as the checker.

Parity is pinned: ``tests/test_oracle_golden.py`` compares every function here with golden vectors produced by
running the reference's own functions (``tests/golden/make_golden.py`` extracts them from
``scripts/nvfp4_ref.py``, ``scripts/gen_fp4_gemm_testcase.py`` and ``scripts/ref_forward.py``).

Reference semantics restated here (paths relative to the reference project):

* e2m1 value table                       ``scripts/nvfp4_ref.py:33``
* e4m3 byte -> value                     ``scripts/nvfp4_ref.py:34-40``
* nearest non-negative e4m3, ties toward the smaller value, zero encoded as byte 0x80
                                         ``scripts/nvfp4_ref.py:41-52``
* nearest e2m1, ties toward the smaller magnitude, sign from ``x < 0``
                                         ``scripts/nvfp4_ref.py:53-61``
* nibble packing, even element in the low nibble
                                         ``scripts/nvfp4_ref.py:63-69``
* per-row NVFP4 quantisation (float64)   ``scripts/nvfp4_ref.py:71-82``
* global scale = 2688 / amax             ``scripts/nvfp4_ref.py:9-11,100``
* 128x4 scale-factor tile swizzle        ``kernels/fp4_gemm.cu:14-33``
* float64 dequant GEMM                   ``scripts/nvfp4_ref.py:102``, ``scripts/gen_fp4_gemm_testcase.py:60``
* router softmax -> top-8 -> renorm      ``scripts/ref_forward.py:160-173``
* expert FFN gelu_tanh(gate)*up -> down  ``scripts/ref_forward.py:175-192``
* gelu_tanh / softmax / rmsnorm          ``scripts/ref_forward.py:67-83``
"""
from __future__ import annotations

import numpy as np

# ----------------------------------------------------------------------------------------------------------------
# Format tables
# ----------------------------------------------------------------------------------------------------------------

#: e2m1 code -> value (code bit 3 is the sign).  scripts/nvfp4_ref.py:33
E2M1_VALUE = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6, 0, -0.5, -1, -1.5, -2, -3, -4, -6], dtype=np.float64)
#: non-negative e2m1 magnitudes, ascending.  scripts/nvfp4_ref.py:53
E2M1_MAG = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6], dtype=np.float64)

FP4_MAX = 6.0
E4M3_MAX = 448.0
#: compressed-tensors global-scale numerator, 448 * 6.  scripts/nvfp4_ref.py:9-11
GSCALE_NUM = E4M3_MAX * FP4_MAX


def _e4m3_decode_table() -> np.ndarray:
    """byte -> float64 value of an OCP e4m3 (fn) byte; 0x7F/0xFF are NaN.  scripts/nvfp4_ref.py:34-40"""
    b = np.arange(256)
    sign = np.where(b >> 7, -1.0, 1.0)
    exp = (b >> 3) & 0xF
    man = b & 0x7
    val = np.where(exp == 0, (man / 8.0) * 2.0 ** -6, (1 + man / 8.0) * 2.0 ** (exp - 7.0))
    val = np.where((exp == 0xF) & (man == 0x7), np.nan, val)
    return sign * val


E4M3_VALUE = _e4m3_decode_table()

# The encoder grid: the distinct finite non-negative e4m3 values, ascending (0, 2^-9, ..., 448).
_E4M3_GRID = np.unique(E4M3_VALUE[np.isfinite(E4M3_VALUE) & (E4M3_VALUE >= 0)])


def _grid_bytes() -> np.ndarray:
    # The reference builds {value: byte} by iterating bytes 0..255 in order, so for the value 0.0 the later byte
    # 0x80 (-0.0, which compares >= 0) overwrites 0x00.  scripts/nvfp4_ref.py:50
    out = np.zeros(len(_E4M3_GRID), dtype=np.uint8)
    for i, v in enumerate(_E4M3_GRID):
        hits = [b for b in range(256) if np.isfinite(E4M3_VALUE[b]) and E4M3_VALUE[b] >= 0 and E4M3_VALUE[b] == v]
        out[i] = hits[-1]
    return out


_E4M3_GRID_BYTE = _grid_bytes()


# ----------------------------------------------------------------------------------------------------------------
# Rounding
# ----------------------------------------------------------------------------------------------------------------

def e4m3_round_pos(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Nearest non-negative finite e4m3 value, ties toward the smaller value.

    Returns (bytes uint8, values float64).  An input that rounds to zero encodes as byte 0x80.  Inputs above 448
    saturate to 448 (byte 0x7E).  scripts/nvfp4_ref.py:43-52
    """
    x = np.asarray(x, dtype=np.float64)
    hi = np.clip(np.searchsorted(_E4M3_GRID, x), 0, len(_E4M3_GRID) - 1)
    lo = np.clip(hi - 1, 0, len(_E4M3_GRID) - 1)
    take_lo = np.abs(x - _E4M3_GRID[lo]) <= np.abs(x - _E4M3_GRID[hi])
    idx = np.where(take_lo, lo, hi)
    return _E4M3_GRID_BYTE[idx], _E4M3_GRID[idx]


def e2m1_round(x: np.ndarray) -> np.ndarray:
    """Nearest e2m1 code, magnitude ties toward the smaller magnitude; sign bit set iff x < 0.

    Magnitudes above 6 saturate to 6.  scripts/nvfp4_ref.py:54-61
    """
    x = np.asarray(x, dtype=np.float64)
    a = np.abs(x)
    hi = np.clip(np.searchsorted(E2M1_MAG, a), 0, 7)
    lo = np.clip(hi - 1, 0, 7)
    take_lo = np.abs(a - E2M1_MAG[lo]) <= np.abs(a - E2M1_MAG[hi])
    mag = np.where(take_lo, lo, hi).astype(np.uint8)
    return mag | ((x < 0).astype(np.uint8) << 3)


def pack_nibbles(codes: np.ndarray) -> np.ndarray:
    """[R, K] 4-bit codes -> [R, K/2] bytes, even element in the low nibble.  scripts/nvfp4_ref.py:68-69"""
    codes = np.asarray(codes, dtype=np.uint8)
    return (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)


def unpack_nibbles(packed: np.ndarray) -> np.ndarray:
    """[R, K/2] bytes -> [R, K] 4-bit codes.  scripts/nvfp4_ref.py:63-67"""
    packed = np.asarray(packed, dtype=np.uint8)
    out = np.empty((packed.shape[0], packed.shape[1] * 2), dtype=np.uint8)
    out[:, 0::2] = packed & 0xF
    out[:, 1::2] = packed >> 4
    return out


# ----------------------------------------------------------------------------------------------------------------
# Quantisation
# ----------------------------------------------------------------------------------------------------------------

def global_scale_from_amax(amax) -> np.float32:
    """fp32 global scale 2688 / max(amax, 1e-9), computed as one correctly-rounded fp32 division.

    The reference computes the same ratio in float64 (scripts/nvfp4_ref.py:100); the device entry points take an
    fp32 scale, so both sides use this fp32 value (the reference's own CUDA path also passes fp32,
    include/nvfp4_quant.h:10-11).
    """
    a = np.maximum(np.float32(amax), np.float32(1e-9))
    return np.float32(np.float32(GSCALE_NUM) / a)


def quantize_rows(x: np.ndarray, gscale) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """NVFP4-quantise rows of ``x`` [R, K] with global scale ``gscale``; all arithmetic in float64.

    Returns (packed [R, K/2] uint8, logical scale bytes [R, K/16] uint8, dequantised [R, K] float64).
    Per 16-element block: stored scale = e4m3(gscale * (block_amax / 6)); local = e4m3_value / gscale (1 for a
    zero scale); codes = e2m1(x / local).  scripts/nvfp4_ref.py:71-82
    """
    x = np.asarray(x, dtype=np.float64)
    rows, k = x.shape
    assert k % 16 == 0, "K must be a multiple of 16"
    g = float(gscale)
    blk = x.reshape(rows, k // 16, 16)
    bamax = np.abs(blk).max(axis=2)
    sf_byte, sf_val = e4m3_round_pos(g * (bamax / 6.0))
    local = np.where(sf_val > 0, sf_val / g, 1.0)
    codes = e2m1_round(blk / local[:, :, None]).reshape(rows, k)
    deq = (E2M1_VALUE[codes].reshape(rows, k // 16, 16) * local[:, :, None]).reshape(rows, k)
    return pack_nibbles(codes), sf_byte.astype(np.uint8), deq


def dequantize(packed: np.ndarray, sf_logical: np.ndarray, gscale) -> np.ndarray:
    """code * e4m3 / gscale per element, float64.  scripts/ref_forward.py:51-64 (dequant_linear)."""
    codes = unpack_nibbles(packed)
    rows, k = codes.shape
    sv = E4M3_VALUE[np.asarray(sf_logical, dtype=np.uint8)]
    return (E2M1_VALUE[codes].reshape(rows, k // 16, 16) * (sv / float(gscale))[:, :, None]).reshape(rows, k)


# ----------------------------------------------------------------------------------------------------------------
# Scale-factor layout
# ----------------------------------------------------------------------------------------------------------------

def scale_buffer_bytes(outer: int, k: int) -> int:
    """ceil(outer/128) * ceil((K/16)/4) tiles of 512 bytes.  kernels/fp4_gemm.cu:14-19"""
    kb = k // 16
    return ((outer + 127) // 128) * ((kb + 3) // 4) * 512


def swizzle_offsets(outer: int, k: int) -> np.ndarray:
    """Physical byte offset of every logical scale (m, b), shape [outer, K/16].  kernels/fp4_gemm.cu:21-33"""
    kb = k // 16
    tile_cols = (kb + 3) // 4
    m = np.arange(outer)[:, None]
    b = np.arange(kb)[None, :]
    tile = (m // 128) * tile_cols + (b // 4)
    within = (m % 32) * 16 + ((m % 128) // 32) * 4 + (b % 4)
    return (tile * 512 + within).astype(np.int64)


def swizzle_scales(logical: np.ndarray, outer: int, k: int) -> np.ndarray:
    """Logical [outer, K/16] -> padded 128x4-tile layout, padding zero.  kernels/fp4_gemm.cu:21-33"""
    out = np.zeros(scale_buffer_bytes(outer, k), dtype=np.uint8)
    out[swizzle_offsets(outer, k)] = np.asarray(logical, dtype=np.uint8).reshape(outer, k // 16)
    return out


def unswizzle_scales(swz: np.ndarray, outer: int, k: int) -> np.ndarray:
    """Inverse of :func:`swizzle_scales` (padding dropped)."""
    return np.asarray(swz, dtype=np.uint8)[swizzle_offsets(outer, k)]


# ----------------------------------------------------------------------------------------------------------------
# GEMM and MoE references
# ----------------------------------------------------------------------------------------------------------------

def gemm_dequant_ref(a_packed, a_sf, a_gscale, b_packed, b_sf, b_gscale) -> np.ndarray:
    """Y[M, N] = deq(A) @ deq(B)^T in float64, with deq = code * e4m3 / gscale.

    The product is the same as the reference's D = (1/gA)(1/gB) A B^T (scripts/nvfp4_ref.py:102,
    tests/test_linear_real.cu:59-60).
    """
    return dequantize(a_packed, a_sf, a_gscale) @ dequantize(b_packed, b_sf, b_gscale).T


def gelu_tanh(x):
    """0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))) in float32.  scripts/ref_forward.py:75-77"""
    x = np.asarray(x, dtype=np.float32)
    return (0.5 * x * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (x + 0.044715 * x ** 3)))).astype(np.float32)


def softmax(x, axis=-1):
    """float32 softmax.  scripts/ref_forward.py:79-83"""
    x = np.asarray(x, dtype=np.float32)
    x = x - x.max(axis=axis, keepdims=True)
    e = np.exp(x)
    return (e / e.sum(axis=axis, keepdims=True)).astype(np.float32)


def rmsnorm(x, weight=None, eps=1e-6):
    """float32 RMS norm.  scripts/ref_forward.py:67-73"""
    x = np.asarray(x, dtype=np.float32)
    xn = x * np.power(np.mean(x * x, axis=-1, keepdims=True) + eps, -0.5)
    if weight is not None:
        xn = xn * np.asarray(weight, dtype=np.float32)
    return xn.astype(np.float32)


def route(logits, top_k=8, per_expert_scale=None):
    """softmax over experts -> top-k (ties to the lower expert id) -> renormalise -> x per_expert_scale.

    Returns (weights [T, k] float32, ids [T, k] int64).  scripts/ref_forward.py:168-173; the tie order follows
    the reference kernel's lowest-index rule (src/forward.cu:213-231) where numpy's argsort leaves it open.
    """
    probs = softmax(logits, axis=-1)
    ids = np.argsort(-probs, axis=-1, kind="stable")[:, :top_k]
    w = np.take_along_axis(probs, ids, axis=-1)
    w = w / w.sum(axis=-1, keepdims=True)
    if per_expert_scale is not None:
        w = w * np.asarray(per_expert_scale, dtype=np.float32)[ids]
    return w.astype(np.float32), ids


def router_logits(residual, proj, scale=None, hidden=None):
    """Router logits.  With ``scale`` given: rmsnorm(no weight) * scale * H^-0.5 first (scripts/ref_forward.py:
    164-167); without it the hidden state is projected directly (the single-layer benchmark configuration)."""
    x = np.asarray(residual, dtype=np.float32)
    if scale is not None:
        h = x.shape[-1] if hidden is None else hidden
        x = rmsnorm(x, None) * np.asarray(scale, dtype=np.float32) * np.float32(h ** -0.5)
    return (x @ np.asarray(proj, dtype=np.float32).T).astype(np.float32)


def experts_ref(x, weights, ids, w_gate, w_up, w_down):
    """Per-token expert FFN: out[t] = sum_j w_tj * Wd_e (gelu_tanh(Wg_e x) * (Wu_e x)).

    ``w_gate/w_up/w_down`` map expert id -> dense float32 matrices.  scripts/ref_forward.py:175-192
    """
    x = np.asarray(x, dtype=np.float32)
    out = np.zeros((x.shape[0], w_down[int(ids[0, 0])].shape[0]), dtype=np.float32)
    for t in range(x.shape[0]):
        for j in range(ids.shape[1]):
            e = int(ids[t, j])
            y = gelu_tanh(w_gate[e] @ x[t]) * (w_up[e] @ x[t])
            out[t] += np.float32(weights[t, j]) * (w_down[e] @ y)
    return out


# ----------------------------------------------------------------------------------------------------------------
# Synthetic inputs (seeded; identical on every machine)
# ----------------------------------------------------------------------------------------------------------------

def f32_to_bf16_bits(x32: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16 bit patterns (uint16).  Inputs are finite."""
    u = np.ascontiguousarray(x32, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def synth_bf16(shape, sigma=1.0, seed=0, outlier_frac=0.0, outlier_mult=50.0):
    """Seeded N(0, sigma^2) drawn in float64, optional outliers scaled before the cast, float32 -> bf16 (RNE).

    Returns bf16 bit patterns (uint16).  Outliers: exactly round(frac * n) distinct entries chosen with
    ``rng.choice(n, k, replace=False)`` and multiplied by ``outlier_mult``.
    """
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(shape) * sigma
    if outlier_frac > 0:
        n = x.size
        k = int(round(outlier_frac * n))
        sel = rng.choice(n, k, replace=False)
        x.reshape(-1)[sel] *= outlier_mult
    return f32_to_bf16_bits(x.astype(np.float32))


# ----------------------------------------------------------------------------------------------------------------
# MoE, W4A4 (the device path's numerics): activations and the intermediate h are NVFP4-quantised
# ----------------------------------------------------------------------------------------------------------------

def moe_dispatch_ref(ids: np.ndarray, num_experts: int, pad: int = 128):
    """Stable counting sort of the (token, slot) assignments by expert, each segment padded to `pad` rows.

    Returns dict: seg_start [E], seg_count [E], dest [T*k] (row of each assignment), row_token [rows] (-1 = pad),
    m_tiles.  Within a segment rows keep assignment order (token-major, slot-minor).
    """
    flat = np.asarray(ids, dtype=np.int64).reshape(-1)
    k = ids.shape[1]
    counts = np.bincount(flat, minlength=num_experts)
    padded = (counts + pad - 1) // pad * pad
    start = np.concatenate([[0], np.cumsum(padded)[:-1]])
    order = np.argsort(flat, kind="stable")
    dest = np.empty(flat.size, np.int64)
    rank = np.arange(flat.size) - np.concatenate([[0], np.cumsum(counts)[:-1]])[flat[order]]
    dest[order] = start[flat[order]] + rank
    rows = int(padded.sum())
    row_token = np.full(rows, -1, np.int64)
    row_token[dest] = np.arange(flat.size) // k
    return {"seg_start": start, "seg_count": counts, "dest": dest, "row_token": row_token, "m_tiles": rows // pad}


def gelu_tanh64(x):
    """float64 form of gelu_tanh (scripts/ref_forward.py:75-77)."""
    return 0.5 * x * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (x + 0.044715 * x ** 3)))


def moe_w4a4_ref(x, ids, weights, experts, g_in, g_h, h_override=None, tokens=None):
    """W4A4 expert FFN: out[t] = sum_j w_tj * deq(Wd_e) @ deq(q(gelu_tanh(deq(Wg_e) x~) * (deq(Wu_e) x~), g_h[e]))
    with x~ = deq(q(x, g_in)).  The structure is scripts/ref_forward.py:175-192 (experts) applied to NVFP4
    activations; weights are NVFP4 (code * e4m3 / g).

    experts: e -> dict(gate=(packed, sf_logical, g), up=(...), down=(...)).
    h_override: e -> (h_codes_rows, h_sf_logical_rows) to use instead of quantising the float64 h (lets a test
    check the down projection against the device's own intermediate).  tokens: restrict the output to these.
    Returns float64 [T, H] (rows outside `tokens` are zero) and, per expert, the float64 h.
    """
    x = np.asarray(x, dtype=np.float64)
    T, H = x.shape
    k = ids.shape[1]
    px, sx, xd = quantize_rows(x, g_in)
    out = np.zeros((T, H), dtype=np.float64)
    keep = np.ones(T, bool) if tokens is None else np.isin(np.arange(T), tokens)
    hs = {}
    for e in np.unique(ids):
        e = int(e)
        sel = np.nonzero((np.asarray(ids) == e) & keep[:, None])
        if sel[0].size == 0:
            continue
        t_list, j_list = sel[0], sel[1]
        order = np.lexsort((j_list, t_list))          # token-major, slot-minor (the dispatch order)
        t_list, j_list = t_list[order], j_list[order]
        ex = experts[e]
        wg = dequantize(*ex["gate"])
        wu = dequantize(*ex["up"])
        wd = dequantize(*ex["down"])
        xe = xd[t_list]
        h = gelu_tanh64(xe @ wg.T) * (xe @ wu.T)
        hs[e] = h
        if h_override is not None and e in h_override:
            hc, hsf = h_override[e]
            hd = dequantize(hc, hsf, g_h[e])
        else:
            _, _, hd = quantize_rows(h, g_h[e])
        y = hd @ wd.T
        np.add.at(out, t_list, np.asarray(weights, np.float64)[t_list, j_list][:, None] * y)
    return out, hs
