"""The C restatement of the quantiser against the pinned numpy oracle and the golden vectors, and the swizzle
against the reference's own compiled host swizzle (kernels/fp4_gemm.cu:21-33)."""
import ctypes

import numpy as np
import pytest

import native
import nvfp4_oracle as orc


@pytest.mark.parametrize("case", ["bf16_outliers", "bf16_weight_ragged", "edges", "fp32_linear"])
def test_c_oracle_matches_golden(golden, case):
    g = golden("quant_cases.npz")
    x = g[f"{case}__x"]
    packed, sf = native.quantize_f32(x, g[f"{case}__gscale"])
    assert np.array_equal(packed, g[f"{case}__packed"]) and np.array_equal(sf, g[f"{case}__sf"])
    if case.startswith("bf16"):
        bits = orc.f32_to_bf16_bits(x)
        assert np.array_equal(orc.bf16_bits_to_f32(bits), x)
        p2, s2 = native.quantize_bf16(bits, g[f"{case}__gscale"])
        assert np.array_equal(p2, packed) and np.array_equal(s2, sf)


def test_c_oracle_matches_numpy_oracle_cfg1_slice():
    bits = orc.synth_bf16((64, 2816), 1.0, seed=0, outlier_frac=0.001)
    amax = native.amax_bf16(bits)
    x = orc.bf16_bits_to_f32(bits)
    assert amax == np.abs(x).max()
    gs = orc.global_scale_from_amax(amax)
    p_np, s_np, _ = orc.quantize_rows(x.astype(np.float64), gs)
    p_c, s_c = native.quantize_bf16(bits, gs)
    assert np.array_equal(p_np, p_c) and np.array_equal(s_np, s_c)


def test_swizzle_matches_reference_binary():
    ref = native.ref_lib()
    if ref is None:
        pytest.skip("reference sources not built (oracle/build.py needs the reference checkout)")
    rng = np.random.default_rng(1)
    for outer, k in [(1, 16), (130, 192), (256, 2816), (7, 48), (1408, 2816)]:
        logical = rng.integers(0, 256, size=(outer, k // 16), dtype=np.uint8)
        nbytes = ref.ref_scale_buffer_bytes(outer, k)
        assert nbytes == orc.scale_buffer_bytes(outer, k)
        out = np.full(nbytes, 0xAB, np.uint8)
        ref.ref_swizzle_scales(logical.ctypes.data_as(ctypes.c_void_p), out.ctypes.data_as(ctypes.c_void_p),
                               outer, k)
        assert np.array_equal(out, orc.swizzle_scales(logical, outer, k))
        assert np.array_equal(out, native.swizzle(logical, outer, k))


def test_c_dequantize_matches_numpy_oracle():
    """The threaded C dequantiser (used by the large GPU parity tests) gives the numpy oracle's float64 values."""
    import native
    import nvfp4_oracle as orc
    rng = np.random.default_rng(3)
    for rows, k in [(1, 16), (37, 96), (300, 2816)]:
        pk = rng.integers(0, 256, (rows, k // 2), dtype=np.uint8)
        sf = rng.integers(0, 0x7F, (rows, k // 16), dtype=np.uint8)
        sf[0, 0] = 0x80                                     # the oracle's zero-block byte
        g = np.float32(2688.0 / 3.7)
        assert np.array_equal(native.dequantize(pk, sf, g), orc.dequantize(pk, sf, g))
