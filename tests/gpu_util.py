"""Helpers shared by the GPU tests (device upload of seeded inputs, gates from the reference's tests)."""
import numpy as np
import pytest
import torch

from __graft_entry__ import load_package


def pkg():
    return load_package()


def require_gpu():
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    p = load_package()
    p.lib()          # raises if the sm_100a library is missing: no fallback exists
    return p


def bf16_to_dev(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits, dtype=np.uint16).view(np.int16)).view(torch.bfloat16).cuda()


def poisoned(n: int, byte: int = 0xFF) -> torch.Tensor:
    return torch.full((n,), byte, dtype=torch.uint8, device="cuda")


def gate_fp4_gemm(got: np.ndarray, ref: np.ndarray):
    """tests/test_fp4_gemm.cu:61-77 of the reference: max_abs < 1e-3 (amax + 1) and no element with
    |d| > 1e-2 (|ref| + 1e-3 amax)."""
    d = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    amax = np.abs(ref).max()
    nbad = int((d > 1e-2 * (np.abs(ref) + 1e-3 * amax)).sum())
    return d.max() < 1e-3 * (amax + 1.0) and nbad == 0, f"max_abs={d.max():.3e} amax={amax:.3f} nbad={nbad}"


def gate_w4a4(got: np.ndarray, ref: np.ndarray):
    """Parity bar for W4A4 GEMM/MoE outputs vs the float64 dequant-matmul: elementwise
    |Y - Yref| <= 1e-2 |Yref| + 1e-3 max|Yref|, and max-norm relative error <= 1e-2."""
    d = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    amax = np.abs(ref).max()
    ok = bool(np.all(d <= 1e-2 * np.abs(ref) + 1e-3 * amax)) and d.max() <= 1e-2 * amax
    return ok, f"max_abs={d.max():.3e} rel={d.max() / max(amax, 1e-30):.3e} amax={amax:.3f}"
