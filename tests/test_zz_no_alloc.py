"""nvfp4b_moe_route_noalloc: the router entry point that takes no workspace and allocates nothing.

It exists for callers that cannot allocate device memory on the call path: a decode loop that reserves all of its
memory once at start-up (a cudaMalloc per step would synchronise the device and break stream capture), or a host
runtime whose memory planner owns every byte of the device.  Its split-K partial logits live in a fixed 4 MiB array
inside the library instead.

The file is collected last, so that a run which stops at the first failure has already run every other test.  The
checks: the entry point agrees with nvfp4b_moe_route on the same inputs on two calls in a row (the second call
reuses the array the first one left behind), it allocates nothing (torch's allocator and the device's free memory
are unchanged across a call), and the same holds in a fresh process whose first router call is this one (that call
looks the array up and loads the library's kernels on the device)."""
import os
import pathlib
import subprocess
import sys

import numpy as np
import pytest
import torch

import nvfp4_oracle as orc
from gpu_util import bf16_to_dev, pkg, require_gpu

ERR_SCRATCH = -8
ROOT = pathlib.Path(__file__).resolve().parent.parent


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
        torch.cuda.synchronize()
        used, free = torch.cuda.memory_allocated(), torch.cuda.mem_get_info()[0]
        p.moe_route_noalloc(x, proj, topk, ids, w, per_expert_scale=pes, norm=norm)
        torch.cuda.synchronize()
        assert torch.cuda.memory_allocated() == used
        if call == 1:                           # the first call may still load kernels; later ones take nothing
            assert torch.cuda.mem_get_info()[0] == free
        assert p.read_device_error() == 0
        # same kernels on the same inputs: identical ids, weights equal to fp32 rounding
        assert torch.equal(ids, ids_ref), f"call {call}: ids differ"
        assert torch.allclose(w, w_ref, rtol=1e-6, atol=0), f"call {call}: weights differ"


_FRESH = r"""
import sys
import torch
sys.path.insert(0, sys.argv[1])
from __graft_entry__ import load_package
p = load_package()
T, H, E, k = 512, 2816, 128, 8
g = torch.Generator(device="cuda").manual_seed(11)
x = torch.randn((T, H), generator=g, device="cuda").to(torch.bfloat16)
proj = (torch.randn((E, H), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
outs = []
for call in range(2):                           # the very first router call of this process is the no-alloc one
    ids = torch.full((T, k), -1, dtype=torch.int32, device="cuda")
    w = torch.full((T, k), float("nan"), device="cuda")
    torch.cuda.synchronize()
    used, free = torch.cuda.memory_allocated(), torch.cuda.mem_get_info()[0]
    p.moe_route_noalloc(x, proj, k, ids, w)
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated() == used, "torch allocation during the call"
    if call == 1:
        assert torch.cuda.mem_get_info()[0] == free, "device memory taken by the second call"
    assert p.read_device_error() == 0
    outs.append((ids, w))
ws = p.moe_workspace(T, H, 64, E, k)
ids_ref, w_ref = p.moe_route(x, proj, k, ws)
torch.cuda.synchronize()
for ids, w in outs:
    assert torch.equal(ids, ids_ref) and torch.allclose(w, w_ref, rtol=1e-6, atol=0)
print("FRESH_OK")
"""


@pytest.mark.gpu
def test_noalloc_route_first_call_in_fresh_process():
    require_gpu()
    env = dict(os.environ)
    r = subprocess.run([sys.executable, "-c", _FRESH, str(ROOT)], capture_output=True, text=True, timeout=300,
                       env=env)
    assert r.returncode == 0 and "FRESH_OK" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]
