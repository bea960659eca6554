"""nvfp4b_moe_route_noalloc: the router entry point that takes no workspace and allocates nothing (its split-K
partials live in a fixed device array inside the library).  Collected last so that it runs both after every other
test and, alone, in a fresh process; it must agree with nvfp4b_moe_route on the same inputs, on consecutive calls."""
import numpy as np
import pytest
import torch

import nvfp4_oracle as orc
from gpu_util import bf16_to_dev, pkg, require_gpu

ERR_SCRATCH = -8


def test_oversize_rejected_before_launch():
    # 4 splits * T * E * 4 bytes > 4 MiB: rejected by the argument checks, no device touched.
    p = pkg()
    L = p._moe_sigs()
    buf = 16  # any non-null, 16-byte-aligned address: nothing is dereferenced on this path
    st = L.nvfp4b_moe_route_noalloc(buf, 2049, 512, buf, 128, 8, None, 0, buf, buf, None)
    assert st == ERR_SCRATCH


def _inputs(T, H, E, seed):
    xb = orc.synth_bf16((T, H), 1.0, seed=seed)
    rb = orc.synth_bf16((E, H), 0.02, seed=seed + 1)
    pes = (1.0 + 0.05 * np.random.default_rng(seed + 2).standard_normal(E)).astype(np.float32)
    return bf16_to_dev(xb), bf16_to_dev(rb), torch.from_numpy(pes).cuda()


@pytest.mark.gpu
@pytest.mark.parametrize("T,H,E,topk,norm", [(300, 512, 64, 8, True), (2048, 2816, 128, 8, False),
                                             (5, 320, 32, 4, True)])
def test_noalloc_route_matches_workspace_route(T, H, E, topk, norm):
    p = require_gpu()
    x, proj, pes = _inputs(T, H, E, seed=T + H)
    ws = p.moe_workspace(T, H, 64, E, topk)
    ids_ref, w_ref = p.moe_route(x, proj, topk, ws, per_expert_scale=pes, norm=norm)
    torch.cuda.synchronize()
    for call in range(2):                       # two calls in a row reuse the same device scratch
        ids = torch.full((T, topk), -1, dtype=torch.int32, device="cuda")
        w = torch.full((T, topk), float("nan"), dtype=torch.float32, device="cuda")
        p.moe_route_noalloc(x, proj, topk, ids, w, per_expert_scale=pes, norm=norm)
        torch.cuda.synchronize()
        assert p.read_device_error() == 0
        # same kernels on the same inputs: identical ids, weights equal to fp32 rounding
        assert torch.equal(ids, ids_ref), f"call {call}: ids differ"
        assert torch.allclose(w, w_ref, rtol=1e-6, atol=0), f"call {call}: weights differ"
