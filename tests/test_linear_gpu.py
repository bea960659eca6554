"""The dense Linear entry (nvfp4b_linear, the call site src/forward.cu:424-445 of the reference): fp32 row-major in
and out, W4A16 below NVFP4B_LINEAR_W4A4_MIN_M rows and W4A4 (NVFP4 activations, tcgen05 GEMM) from there on.
W4A4 results are checked against the oracle's quantiser + float64 dequant-matmul, W4A16 results against the float64
product of the fp16 activations and the dequantised weights."""
import numpy as np
import pytest
import torch

import oracle.native as native
import oracle.nvfp4_oracle as orc
from tests.gpu_util import gate_w4a4, require_gpu

pytestmark = pytest.mark.gpu


def _weights(N, K, seed):
    wb = orc.synth_bf16((N, K), sigma=0.02, seed=seed)
    gw = np.float32(orc.global_scale_from_amax(native.amax_bf16(wb)))
    wp, ws = native.quantize_bf16(wb, gw)
    return wp, ws, gw


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _call(p, x, wp, ws, gw, N, a_gscale, mode):
    M, K = x.shape
    W, S = _dev(wp), _dev(ws)
    St = _dev(orc.swizzle_scales(ws, N, K))
    out = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    p.linear(out, _dev(x), W, S, St, float(gw), a_gscale=a_gscale, mode=mode)
    torch.cuda.synchronize()
    assert p.read_device_error() == 0
    return out.cpu().numpy()


@pytest.mark.parametrize("M,N,K,static", [(128, 256, 2816, True), (256, 384, 2112, True), (300, 200, 1024, False),
                                          (1024, 512, 2816, False)])
def test_linear_w4a4_vs_oracle(M, N, K, static):
    p = require_gpu()
    rng = np.random.default_rng(M + K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    wp, ws, gw = _weights(N, K, seed=N)
    gx = np.float32(orc.global_scale_from_amax(np.float32(np.abs(x).max())))
    if static:
        gx = np.float32(gx * np.float32(0.75))          # a calibrated static scale need not equal 2688/amax
    got = _call(p, x, wp, ws, gw, N, float(gx) if static else None, p.LINEAR_AUTO)
    xp, xs = native.quantize_f32(x, gx)
    ref = orc.gemm_dequant_ref(xp, xs, gx, wp, ws, gw)
    ok, msg = gate_w4a4(got, ref)
    assert ok, msg


def test_linear_w4a4_equals_quantize_then_gemm():
    """The fused entry is the quantiser + GEMM composition, bit for bit (same kernels, same scales)."""
    p = require_gpu()
    M, N, K = 384, 640, 2816
    rng = np.random.default_rng(11)
    x = rng.standard_normal((M, K)).astype(np.float32)
    wp, ws, gw = _weights(N, K, seed=3)
    got = _call(p, x, wp, ws, gw, N, None, p.LINEAR_W4A4)
    X = _dev(x)
    amax = p.amax(X)
    xq, xs = p.quantize(X, amax_dev=amax)
    ref = p.gemm(xq, xs, 1.0, _dev(wp), _dev(orc.swizzle_scales(ws, N, K)), 1.0 / float(gw),
                 out_kind=p.OUT_F32_ROWMAJOR, a_amax=amax)
    torch.cuda.synchronize()
    assert np.array_equal(got, ref.cpu().numpy())
    assert float(amax.item()) == float(np.abs(x).max())


@pytest.mark.parametrize("M,N,K,mode", [(1, 512, 2816, 0), (16, 300, 2112, 0), (127, 128, 1024, 0),
                                        (200, 96, 2816, 1), (5, 64, 1040, 1)])
def test_linear_w4a16_vs_oracle(M, N, K, mode):
    p = require_gpu()
    rng = np.random.default_rng(M * 3 + N)
    x = rng.standard_normal((M, K)).astype(np.float32)
    wp, ws, gw = _weights(N, K, seed=M)
    got = _call(p, x, wp, ws, gw, N, None, mode)
    x16 = x.astype(np.float16).astype(np.float64)
    wd = orc.dequantize(wp, ws, gw)
    ref, bound = x16 @ wd.T, np.abs(x16) @ np.abs(wd).T
    d = np.abs(got.astype(np.float64) - ref)
    assert np.all(d <= 1e-5 * bound), f"max err {d.max():.3e}"
