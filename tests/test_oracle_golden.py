"""The CPU oracle against golden vectors produced by the reference's own functions (tests/golden/make_golden.py).

These pin the oracle: every later GPU parity test trusts it only because these pass.
"""
import numpy as np
import pytest

import nvfp4_oracle as orc

QUANT_CASES = ["bf16_outliers", "fp32_linear", "bf16_weight_ragged", "edges"]


def test_e4m3_encoder_matches_reference(golden):
    g = golden("quant_cases.npz")
    b, v = orc.e4m3_round_pos(g["e4m3_probe__x"])
    assert np.array_equal(b, g["e4m3_probe__byte"])
    assert np.array_equal(v, g["e4m3_probe__val"])
    # the quirks the device kernel must follow: zero -> 0x80, ties toward the smaller value, saturation
    assert orc.e4m3_round_pos(np.array([0.0]))[0][0] == 0x80
    assert orc.e4m3_round_pos(np.array([1.1875]))[0][0] == 0x39
    assert orc.e4m3_round_pos(np.array([1e6]))[0][0] == 0x7E


def test_e2m1_encoder_matches_reference(golden):
    g = golden("quant_cases.npz")
    assert np.array_equal(orc.e2m1_round(g["e2m1_probe__x"]), g["e2m1_probe__code"])
    ties = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0])
    assert list(orc.e2m1_round(ties)) == [0, 1, 2, 3, 4, 5, 6]      # always the smaller magnitude


@pytest.mark.parametrize("case", QUANT_CASES)
def test_quantize_rows_matches_reference(golden, case):
    g = golden("quant_cases.npz")
    x = g[f"{case}__x"].astype(np.float64)
    packed, sf, deq = orc.quantize_rows(x, g[f"{case}__gscale"])
    assert np.array_equal(packed, g[f"{case}__packed"])
    assert np.array_equal(sf, g[f"{case}__sf"])
    if f"{case}__deq" in g:
        assert np.array_equal(deq, g[f"{case}__deq"])
    # dequantize() inverts the encoding exactly
    assert np.array_equal(orc.dequantize(packed, sf, g[f"{case}__gscale"]), deq)


def test_swizzle_layout_roundtrip_and_padding():
    rng = np.random.default_rng(0)
    for outer, k in [(1, 16), (130, 192), (256, 2816), (7, 48)]:
        logical = rng.integers(1, 256, size=(outer, k // 16), dtype=np.uint8)
        swz = orc.swizzle_scales(logical, outer, k)
        assert swz.size == orc.scale_buffer_bytes(outer, k)
        assert np.array_equal(orc.unswizzle_scales(swz, outer, k), logical)
        mask = np.zeros(swz.size, bool)
        mask[orc.swizzle_offsets(outer, k)] = True
        assert not swz[~mask].any()                                     # padding is zero
    # one tile: (m%32)*16 + ((m%128)/32)*4 + b%4 (kernels/fp4_gemm.cu:21-33)
    off = orc.swizzle_offsets(128, 64)
    assert off[33, 2] == 1 * 16 + 1 * 4 + 2 and off[127, 3] == 31 * 16 + 3 * 4 + 3


@pytest.mark.parametrize("tag", ["default", "ragged"])
def test_gemm_reference_matches_generator(golden, tag):
    g = golden("gemm_cases.npz")
    # the generator's global scales multiply (dequant = code * sf * g); the oracle divides, so pass 1/g
    y = orc.gemm_dequant_ref(g[f"{tag}__a_packed"], g[f"{tag}__a_sf"], 1.0 / np.float64(g[f"{tag}__ag"]),
                             g[f"{tag}__b_packed"], g[f"{tag}__b_sf"], 1.0 / np.float64(g[f"{tag}__bg"]))
    ref = g[f"{tag}__y_ref"].astype(np.float64)
    assert np.allclose(y, ref, rtol=1e-6, atol=1e-6 * np.abs(ref).max())


def test_router_and_experts_match_reference(golden):
    g = golden("moe_case.npz")
    H, E = int(g["H"]), int(g["E"])
    logits = orc.router_logits(g["resid"], g["proj"], scale=g["scale"], hidden=H)
    w, ids = orc.route(logits, 8, g["pes"])
    assert np.array_equal(ids, g["topi"])
    assert np.allclose(w, g["topw"], rtol=1e-6, atol=1e-7)
    deq = {}
    for kind in ["gate_proj", "up_proj", "down_proj"]:
        deq[kind] = {e: orc.dequantize(g[f"{kind}__{e}__packed"], g[f"{kind}__{e}__sf"],
                                       g[f"{kind}__{e}__g"]).astype(np.float32) for e in range(E)}
    out = orc.experts_ref(g["xm"], g["topw"], g["topi"], deq["gate_proj"], deq["up_proj"], deq["down_proj"])
    assert np.allclose(out, g["out"], rtol=1e-5, atol=1e-5 * np.abs(g["out"]).max())


def test_synthetic_inputs_are_deterministic():
    a = orc.synth_bf16((16, 2816), 1.0, seed=0, outlier_frac=0.001)
    b = orc.synth_bf16((16, 2816), 1.0, seed=0, outlier_frac=0.001)
    assert np.array_equal(a, b)
    x = orc.bf16_bits_to_f32(a)
    assert (np.abs(x) > 10).sum() >= 20                     # the 45 outliers (x50) are present
