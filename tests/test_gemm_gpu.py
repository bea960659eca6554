"""W4A4 NVFP4 GEMM (tcgen05 kind::mxf4nvf4) on the GPU vs the float64 dequant-matmul oracle.

Gates: the reference's own GEMM gate (tests/test_fp4_gemm.cu:61-77) on its generator's fixtures, and the
elementwise W4A4 bar |Y - Yref| <= 1e-2 |Yref| + 1e-3 max|Yref| (max-norm rel <= 1e-2) on seeded bf16 inputs."""
import numpy as np
import pytest
import torch

import native
import nvfp4_oracle as orc
from gpu_util import bf16_to_dev, gate_fp4_gemm, gate_w4a4, require_gpu

pytestmark = pytest.mark.gpu


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.fixture(params=[1, 2, 3], ids=["tile256", "tile128", "pair"])
def tile_config(request):
    """Every dense tile configuration: 128x256 and 128x128 single-CTA tiles, 256x256 CTA-pair tiles."""
    p = require_gpu()
    p.set_gemm_tile_config(request.param)
    yield request.param
    p.set_gemm_tile_config(0)


@pytest.mark.parametrize("tag", ["default", "ragged"])
def test_reference_generator_cases_colmajor(golden, tag, tile_config):
    """tests/test_fp4_gemm.cu flow: host-swizzled scales, nvfp4_gemm -> fp32 column-major D (ld = M)."""
    p = require_gpu()
    g = golden("gemm_cases.npz")
    M, N, K = [int(v) for v in g[f"{tag}__dims"]]
    ag, bg = float(g[f"{tag}__ag"]), float(g[f"{tag}__bg"])
    A, B = _dev(g[f"{tag}__a_packed"]), _dev(g[f"{tag}__b_packed"])
    As = _dev(orc.swizzle_scales(g[f"{tag}__a_sf"], M, K))
    Bs = _dev(orc.swizzle_scales(g[f"{tag}__b_sf"], N, K))
    D = torch.full((N, M), float("nan"), dtype=torch.float32, device="cuda")
    rc = p.nvfp4_gemm(D, A, As, ag, B, Bs, bg, M, N, K)
    torch.cuda.synchronize()
    assert rc == 0
    assert p.read_device_error() == 0
    got = D.cpu().numpy().T          # column-major [M, N]
    ok, msg = gate_fp4_gemm(got, g[f"{tag}__y_ref"])
    assert ok, msg


def _quantized_operands(M, N, K, seed):
    xb = orc.synth_bf16((M, K), 1.0, seed=seed)
    wb = orc.synth_bf16((N, K), 0.02, seed=seed + 1)
    gx = orc.global_scale_from_amax(native.amax_bf16(xb))
    gw = orc.global_scale_from_amax(native.amax_bf16(wb))
    px, sx = native.quantize_bf16(xb, gx)
    pw, sw = native.quantize_bf16(wb, gw)
    return xb, wb, (px, sx, gx), (pw, sw, gw)


@pytest.mark.parametrize("M,N,K", [(16, 2048, 2048),                 # cfg0
                                   (128, 2816, 2816), (256, 8448, 2816), (128, 14336, 4096),   # cfg2 (reduced M)
                                   (1, 256, 64), (130, 200, 192), (77, 136, 96), (300, 384, 2048)])
def test_gemm_bf16_vs_dequant_oracle(M, N, K, tile_config):
    p = require_gpu()
    _, _, (px, sx, gx), (pw, sw, gw) = _quantized_operands(M, N, K, seed=M + N + K)
    A, As = _dev(px), _dev(orc.swizzle_scales(sx, M, K))
    B, Bs = _dev(pw), _dev(orc.swizzle_scales(sw, N, K))
    Y = p.gemm(A, As, 1.0 / float(gx), B, Bs, 1.0 / float(gw))
    torch.cuda.synchronize()
    assert p.read_device_error() == 0
    ref = orc.gemm_dequant_ref(px, sx, gx, pw, sw, gw)
    ok, msg = gate_w4a4(Y.float().cpu().numpy(), ref)
    assert ok, msg


def test_gemm_fp32_rowmajor_and_dynamic_alpha(tile_config):
    """fp32 row-major output; activation dequant taken from a device amax (the dynamic-scale pipeline)."""
    p = require_gpu()
    M, N, K = 256, 384, 1024
    xb, wb, (px, sx, gx), (pw, sw, gw) = _quantized_operands(M, N, K, seed=5)
    x = bf16_to_dev(xb)
    amax = p.amax(x)
    xq, xs = p.quantize(x, amax_dev=amax)
    B, Bs = _dev(pw), _dev(orc.swizzle_scales(sw, N, K))
    Y = p.gemm(xq, xs, 0.0, B, Bs, 1.0 / float(gw), out_kind=p.OUT_F32_ROWMAJOR, a_amax=amax)
    torch.cuda.synchronize()
    ref = orc.gemm_dequant_ref(px, sx, gx, pw, sw, gw)
    ok, msg = gate_w4a4(Y.cpu().numpy(), ref)
    assert ok, msg


def test_gemm_full_size_cfg2_sampled_rows(tile_config):
    """cfg2 at M=4096, (K, N) = (4096, 14336): full-size launch, oracle on 96 sampled rows."""
    p = require_gpu()
    M, N, K = 4096, 14336, 4096
    rng = np.random.default_rng(0)
    xb = orc.synth_bf16((M, K), 1.0, seed=41)
    wb = orc.synth_bf16((N, K), 0.02, seed=42)
    x, w = bf16_to_dev(xb), bf16_to_dev(wb)
    gx = orc.global_scale_from_amax(native.amax_bf16(xb))
    gw = orc.global_scale_from_amax(native.amax_bf16(wb))
    xq, xs = p.quantize(x, gscale=float(gx))
    wq, ws = p.quantize(w, gscale=float(gw))
    Y = p.gemm(xq, xs, 1.0 / float(gx), wq, ws, 1.0 / float(gw))
    torch.cuda.synchronize()
    assert p.read_device_error() == 0
    rows = np.sort(rng.choice(M, 96, replace=False))
    px, sx = native.quantize_bf16(xb[rows], gx)
    pw, sw = native.quantize_bf16(wb, gw)
    ref = orc.gemm_dequant_ref(px, sx, gx, pw, sw, gw)
    ok, msg = gate_w4a4(Y[torch.from_numpy(rows).cuda()].float().cpu().numpy(), ref)
    assert ok, msg


def test_gemm_matches_reference_cublaslt_when_built():
    """Same operands through the reference's own nvfp4_gemm (cuBLASLt), built from its sources in oracle/_ref."""
    p = require_gpu()
    ref_lib = native.ref_lib()
    if ref_lib is None:
        pytest.skip("oracle/_ref not built")
    M, N, K = 256, 512, 1024
    _, _, (px, sx, gx), (pw, sw, gw) = _quantized_operands(M, N, K, seed=17)
    A, As = _dev(px), _dev(orc.swizzle_scales(sx, M, K))
    B, Bs = _dev(pw), _dev(orc.swizzle_scales(sw, N, K))
    D_ours = torch.empty((N, M), dtype=torch.float32, device="cuda")
    D_ref = torch.empty((N, M), dtype=torch.float32, device="cuda")
    assert p.nvfp4_gemm(D_ours, A, As, 1.0 / float(gx), B, Bs, 1.0 / float(gw), M, N, K) == 0
    rc = ref_lib.ref_nvfp4_gemm(D_ref.data_ptr(), A.data_ptr(), As.data_ptr(), 1.0 / float(gx), B.data_ptr(),
                                Bs.data_ptr(), 1.0 / float(gw), M, N, K, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    if rc != 0:
        pytest.skip(f"reference cuBLASLt nvfp4_gemm returned {rc} on this box")
    ok, msg = gate_fp4_gemm(D_ours.cpu().numpy(), D_ref.cpu().numpy())
    assert ok, msg


# ---- cfg2 at full size: every (M, K, N) point of the dense prefill sweep ------------------------------------------

_CFG2_SHAPES = [(M, K, N) for M in (128, 1024, 4096, 8192) for (K, N) in ((2816, 2816), (2816, 8448), (4096, 14336))]
# every shape with the automatic tile choice, and with the other kernel family (the CTA-pair 256x256 kernel is the
# automatic choice above 128 rows, the single-CTA 128x256 kernel at 128 rows)
_CFG2_CASES = [(M, K, N, cfg) for (M, K, N) in _CFG2_SHAPES for cfg in (0, 3 if M <= 128 else 1)]
_cfg2_cache = {}


def _cfg2_operands(p, M, K, N):
    """Full-size NVFP4 operands of one cfg2 point (quantised on the device, bit-exact to the oracle) and the float64
    dequant-matmul of 66 rows (the first, the last and 64 sampled ones); one shape cached at a time."""
    key = (M, K, N)
    if key not in _cfg2_cache:
        _cfg2_cache.clear()
        xb = orc.synth_bf16((M, K), 1.0, seed=M + K)
        wb = orc.synth_bf16((N, K), 0.02, seed=N + K + 1)
        gx = orc.global_scale_from_amax(native.amax_bf16(xb))
        gw = orc.global_scale_from_amax(native.amax_bf16(wb))
        xq, xs = p.quantize(bf16_to_dev(xb), gscale=float(gx))
        wq, ws = p.quantize(bf16_to_dev(wb), gscale=float(gw))
        rng = np.random.default_rng(M * 7 + N)
        rows = np.concatenate([[0], np.sort(rng.choice(np.arange(1, M - 1), 64, replace=False)), [M - 1]])
        px, sx = native.quantize_bf16(xb[rows], gx)
        pw, sw = native.quantize_bf16(wb, gw)
        ref = native.dequantize(px, sx, gx) @ native.dequantize(pw, sw, gw).T
        torch.cuda.synchronize()
        _cfg2_cache[key] = (xq, xs, gx, wq, ws, gw, rows, ref)
    return _cfg2_cache[key]


@pytest.mark.parametrize("M,K,N,cfg", _CFG2_CASES, ids=[f"M{m}-K{k}-N{n}-cfg{c}" for m, k, n, c in _CFG2_CASES])
def test_gemm_cfg2_grid_full_size_sampled_rows(M, K, N, cfg):
    """BASELINE cfg2: M in {128, 1024, 4096, 8192} x (K, N) in {(2816, 2816), (2816, 8448), (4096, 14336)}, full-size
    launch, bf16 out with the fused global-scale multiply, oracle on 66 rows (W4A4 bar)."""
    p = require_gpu()
    xq, xs, gx, wq, ws, gw, rows, ref = _cfg2_operands(p, M, K, N)
    p.set_gemm_tile_config(cfg)
    try:
        Y = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        p.gemm(xq, xs, 1.0 / float(gx), wq, ws, 1.0 / float(gw), out=Y)
        torch.cuda.synchronize()
    finally:
        p.set_gemm_tile_config(0)
    assert p.read_device_error() == 0
    assert not torch.isnan(Y).any()                      # every output written (full-size launch)
    ok, msg = gate_w4a4(Y[torch.from_numpy(rows).cuda()].float().cpu().numpy(), ref)
    assert ok, msg


def test_hbm_read_stream_measurement_kernel():
    """nvfp4b_hbm_read_stream (the bench's read ceiling): full and partial 256-row boxes, several boxes per SM; it
    completes without a device error and leaves its input untouched."""
    p = require_gpu()
    buf = torch.randint(0, 256, (3000 * 1408 + 64,), dtype=torch.uint8, device="cuda")
    before = buf.clone()
    for rows in (3000, 256, 1, 70000 // 1408 * 10):
        p.hbm_read_stream(buf, rows, 1408)
    big = torch.empty(148 * 3 * 256 * 1408, dtype=torch.uint8, device="cuda")
    p.hbm_read_stream(big, 148 * 3 * 256, 1408)
    torch.cuda.synchronize()
    assert p.read_device_error() == 0
    assert torch.equal(buf, before)
