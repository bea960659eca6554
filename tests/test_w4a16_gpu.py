"""W4A16 decode kernels (``w4a16_gemm`` / ``fp4_gemv``, kernels/fp4_gemm.cu:45-111 of the reference): NVFP4 weights
(raw row-major codes [N, K/2] and e4m3 scales [N, K/16], dequant code * e4m3 / w_gscale) times fp16 activations,
fp32 row-major out [M, N].  Checked against the float64 dequant-matmul of the oracle, and against the reference's own
kernels (built from its sources into oracle/_ref) where those accept the shape (M <= 16)."""
import numpy as np
import pytest
import torch

import oracle.native as native
import oracle.nvfp4_oracle as orc
from tests.gpu_util import require_gpu

pytestmark = pytest.mark.gpu


def _operands(M, N, K, seed):
    rng = np.random.default_rng(seed)
    wb = orc.synth_bf16((N, K), sigma=0.02, seed=seed + 1)
    gw = orc.global_scale_from_amax(native.amax_bf16(wb))
    wp, ws = native.quantize_bf16(wb, gw)
    x16 = rng.standard_normal((M, K)).astype(np.float16)
    return wp, ws, np.float32(gw), x16


def _reference(wp, ws, gw, x16):
    """float64 dequant(W) @ x^T and the bound sum |w| |x| used for the fp32-accumulation tolerance."""
    wd = orc.dequantize(wp, ws, gw)
    x = x16.astype(np.float64)
    return x @ wd.T, np.abs(x) @ np.abs(wd).T


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _check_fp32_accumulation(got, ref, bound):
    # fp32 accumulation: every partial sum is rounded at most ~K/32 + 40 times, each by 2^-24 of at most sum|w||x|.
    d = np.abs(got.astype(np.float64) - ref)
    lim = 1e-5 * bound + 1e-30
    assert np.all(d <= lim), f"max err {d.max():.3e}, worst ratio {(d / lim).max():.3f}"


# M <= 2 with K % 256 == 0: the TMA-fed kernel ((1, 60000, 256): more 256-row tasks than SMs); M <= 8: the
# register-fed kernel ((3, 60000, 256): more row groups than resident warps; (6, 129, 2080): K % 64 != 0); larger M
# with K % 64 == 0: passes of 16 rows through the cp.async ring kernel (M = 37, 130: several passes, the last of
# <= 8 rows); (12, 50, 2080): the FFMA kernel.
@pytest.mark.parametrize("M,N,K", [(1, 512, 2816), (5, 300, 2048), (16, 256, 4096), (37, 200, 2816),
                                   (130, 96, 1024), (1, 1000, 2112), (1, 60000, 256), (2, 4100, 2816),
                                   (3, 60000, 256), (8, 4100, 2816), (13, 4100, 2816), (6, 129, 2080),
                                   (12, 50, 2080), (2, 40, 96)])
def test_w4a16_vs_dequant_oracle(M, N, K):
    p = require_gpu()
    wp, ws, gw, x16 = _operands(M, N, K, seed=M * 7 + N)
    out = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    p.w4a16_gemm(out, _dev(wp), _dev(ws), float(gw), _dev(x16).view(torch.float16), M, N, K)
    torch.cuda.synchronize()
    ref, bound = _reference(wp, ws, gw, x16)
    _check_fp32_accumulation(out.cpu().numpy(), ref, bound)


@pytest.mark.parametrize("M,N,K,offset", [(3, 70, 2064, 0), (9, 33, 1040, 0), (4, 64, 2048, 8)])
def test_w4a16_byte_path(M, N, K, offset):
    """K % 32 != 0, or activations not 16-byte aligned: the byte-granular kernel, same result bar."""
    p = require_gpu()
    wp, ws, gw, x16 = _operands(M, N, K, seed=K + offset)
    buf = torch.zeros(M * K + offset // 2 + 8, dtype=torch.float16, device="cuda")
    x_dev = buf[offset // 2: offset // 2 + M * K].view(M, K)
    x_dev.copy_(torch.from_numpy(x16).cuda())
    out = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    p.w4a16_gemm(out, _dev(wp), _dev(ws), float(gw), x_dev, M, N, K)
    torch.cuda.synchronize()
    ref, bound = _reference(wp, ws, gw, x16)
    _check_fp32_accumulation(out.cpu().numpy(), ref, bound)


def test_fp4_gemv_is_w4a16_at_m1():
    p = require_gpu()
    N, K = 777, 2816
    wp, ws, gw, x16 = _operands(1, N, K, seed=5)
    y = torch.full((N,), float("nan"), dtype=torch.float32, device="cuda")
    p.fp4_gemv(y, _dev(wp), _dev(ws), float(gw), _dev(x16).view(torch.float16), N, K)
    torch.cuda.synchronize()
    ref, bound = _reference(wp, ws, gw, x16)
    _check_fp32_accumulation(y.cpu().numpy()[None, :], ref, bound)


def test_w4a16_rejects_bad_shapes():
    p = require_gpu()
    out = torch.empty(16, dtype=torch.float32, device="cuda")
    w = torch.empty(64, dtype=torch.uint8, device="cuda")
    x = torch.empty(64, dtype=torch.float16, device="cuda")
    with pytest.raises(p.NvFp4Error):
        p.w4a16_gemm(out, w, w, 1.0, x, 1, 2, 24)       # K % 16 != 0
    with pytest.raises(p.NvFp4Error):
        p.w4a16_gemm(out, w, w, 1.0, x, 0, 2, 32)       # M == 0


@pytest.mark.parametrize("M,N,K", [(1, 512, 2816), (8, 384, 2048), (16, 256, 2816)])
def test_w4a16_matches_reference_kernels_when_built(M, N, K):
    """Same operands through the reference's own w4a16_gemm / fp4_gemv.  The reference sums groups of 8 products in
    half2 before the fp32 accumulate, so the bar is the W4A4 one (1e-2 relative elementwise + 1e-3 of the max)."""
    p = require_gpu()
    ref_lib = native.ref_lib()
    if ref_lib is None:
        pytest.skip("oracle/_ref not built")
    from tests.gpu_util import gate_w4a4
    wp, ws, gw, x16 = _operands(M, N, K, seed=99 + M)
    W, S, X = _dev(wp), _dev(ws), _dev(x16).view(torch.float16)
    ours = torch.empty((M, N), dtype=torch.float32, device="cuda")
    theirs = torch.empty((M, N), dtype=torch.float32, device="cuda")
    p.w4a16_gemm(ours, W, S, float(gw), X, M, N, K)
    stream = torch.cuda.current_stream().cuda_stream
    if M == 1:
        ref_lib.ref_fp4_gemv(theirs.data_ptr(), W.data_ptr(), S.data_ptr(), float(gw), X.data_ptr(), N, K, stream)
    else:
        ref_lib.ref_w4a16_gemm(theirs.data_ptr(), W.data_ptr(), S.data_ptr(), float(gw), X.data_ptr(), M, N, K,
                               stream)
    torch.cuda.synchronize()
    ok, msg = gate_w4a4(ours.cpu().numpy(), theirs.cpu().numpy())
    assert ok, msg
