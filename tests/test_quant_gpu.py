"""NVFP4 activation quantiser on the GPU vs the pinned CPU oracle: codes and scale bytes bit-exact, padding
written, global amax exact.  Calls go through the C ABI (libnvfp4_b200.so)."""
import numpy as np
import pytest
import torch

import native
import nvfp4_oracle as orc
from gpu_util import bf16_to_dev, poisoned, require_gpu

pytestmark = pytest.mark.gpu


def _run_quant(p, x_dev, M, K, gscale=None, amax_dev=None):
    packed = poisoned(M * K // 2).view(M, K // 2)
    scales = poisoned(p.nvfp4_scale_buffer_bytes(M, K))
    p.quantize(x_dev, gscale=gscale, amax_dev=amax_dev, packed=packed, scales=scales)
    torch.cuda.synchronize()
    return packed.cpu().numpy(), scales.cpu().numpy()


def _check_scales(sc, M, K, sf_ref):
    assert np.array_equal(orc.unswizzle_scales(sc, M, K), sf_ref)
    mask = np.zeros(sc.size, bool)
    mask[orc.swizzle_offsets(M, K)] = True
    assert not sc[~mask].any(), "padding bytes must be overwritten with zero"


@pytest.mark.parametrize("case", ["bf16_outliers", "bf16_weight_ragged", "edges", "fp32_linear"])
def test_golden_cases_bit_exact(golden, case):
    p = require_gpu()
    g = golden("quant_cases.npz")
    x = g[f"{case}__x"]
    M, K = x.shape
    gs = float(g[f"{case}__gscale"])
    # fp32 input path (the reference entry point's type)
    pk, sc = _run_quant(p, torch.from_numpy(x).cuda(), M, K, gscale=gs)
    assert np.array_equal(pk, g[f"{case}__packed"])
    _check_scales(sc, M, K, g[f"{case}__sf"])
    bits = orc.f32_to_bf16_bits(x)
    if np.array_equal(orc.bf16_bits_to_f32(bits), x):          # bf16-representable cases: same result via bf16
        pk2, sc2 = _run_quant(p, bf16_to_dev(bits), M, K, gscale=gs)
        assert np.array_equal(pk2, pk) and np.array_equal(sc2, sc)


@pytest.mark.parametrize("T", [1, 16, 128, 1024, 8192])
def test_cfg1_sweep_dynamic_scale_bit_exact(T):
    """cfg1: bf16 [T, 2816] ~ N(0,1) with 0.1% x50 outliers; device amax -> gscale -> quantise."""
    p = require_gpu()
    K = 2816
    bits = orc.synth_bf16((T, K), 1.0, seed=100 + T, outlier_frac=0.001)
    x = bf16_to_dev(bits)
    amax_dev = p.amax(x)
    pk, sc = _run_quant(p, x, T, K, amax_dev=amax_dev)
    amax_ref = native.amax_bf16(bits)
    assert np.float32(amax_dev.item()) == amax_ref
    gs = orc.global_scale_from_amax(amax_ref)
    pk_ref, sf_ref = native.quantize_bf16(bits, gs)
    assert np.array_equal(pk, pk_ref)
    _check_scales(sc, T, K, sf_ref)


@pytest.mark.parametrize("M,K", [(1, 16), (3, 48), (129, 80), (200, 2048), (37, 4096), (9, 11264), (3, 24000)])
def test_ragged_shapes(M, K):
    p = require_gpu()
    bits = orc.synth_bf16((M, K), 0.7, seed=M * 7 + K)
    x32 = orc.bf16_bits_to_f32(bits)
    gs = orc.global_scale_from_amax(np.abs(x32).max())
    pk, sc = _run_quant(p, bf16_to_dev(bits), M, K, gscale=float(gs))
    pk_ref, sf_ref, _ = orc.quantize_rows(x32.astype(np.float64), gs)
    assert np.array_equal(pk, pk_ref)
    _check_scales(sc, M, K, sf_ref)


def test_rounding_boundaries_exhaustive():
    """Inputs placed exactly on, and one ulp either side of, every e2m1 decision boundary of blocks with many
    different scales: exercises the exact float64 path of the kernel."""
    p = require_gpu()
    rng = np.random.default_rng(9)
    rows = []
    gs = np.float32(rng.uniform(20, 4000))
    mids = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0])
    for _ in range(512):
        bamax = np.float32(rng.uniform(0.01, 50))
        b_, v_ = orc.e4m3_round_pos(np.array([float(gs) * (float(bamax) / 6.0)]))
        L = v_[0] / float(gs) if v_[0] > 0 else 1.0
        row = [bamax]
        for m in mids[rng.permutation(7)][:5]:
            t = np.float32(m * L)
            row += [t, np.nextafter(t, np.float32(0)), np.nextafter(t, np.float32(1e9))]
        row = np.array(row[:16], np.float32)
        row = np.minimum(np.abs(row), bamax) * np.where(rng.random(16) < 0.5, -1, 1).astype(np.float32)
        row[0] = bamax
        rows.append(np.concatenate([row, row[::-1]]))
    x = np.array(rows, np.float32)
    M, K = x.shape
    pk, sc = _run_quant(p, torch.from_numpy(x).cuda(), M, K, gscale=float(gs))
    pk_ref, sf_ref, _ = orc.quantize_rows(x.astype(np.float64), gs)
    assert np.array_equal(pk, pk_ref)
    _check_scales(sc, M, K, sf_ref)


def test_reference_entry_point_name():
    """The reference-named entry point (fp32 in, static gscale) behaves like the C ABI call."""
    p = require_gpu()
    bits = orc.synth_bf16((128, 512), 0.5, seed=7)
    x = torch.from_numpy(orc.bf16_bits_to_f32(bits)).cuda()
    gs = float(orc.global_scale_from_amax(np.abs(orc.bf16_bits_to_f32(bits)).max()))
    packed = torch.empty((128, 256), dtype=torch.uint8, device="cuda")
    scales = poisoned(p.nvfp4_scale_buffer_bytes(128, 512))
    p.nvfp4_quantize_activations(x, packed, scales, 128, 512, gs)
    torch.cuda.synchronize()
    pk_ref, sf_ref = native.quantize_bf16(bits, gs)
    assert np.array_equal(packed.cpu().numpy(), pk_ref)
    assert np.array_equal(orc.unswizzle_scales(scales.cpu().numpy(), 128, 512), sf_ref)


def test_device_swizzle_matches_host():
    p = require_gpu()
    rng = np.random.default_rng(2)
    for outer, k in [(130, 192), (2816, 704), (1, 16)]:
        logical = rng.integers(0, 256, (outer, k // 16), dtype=np.uint8)
        out = p.nvfp4_swizzle_scales(torch.from_numpy(logical).cuda(), outer, k)
        assert np.array_equal(out.cpu().numpy(), orc.swizzle_scales(logical, outer, k))
