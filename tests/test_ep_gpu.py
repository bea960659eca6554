"""Expert-parallel MoE device path (nvfp4b_ep_dispatch / _expert_forward / _combine) on one GPU.

At G = 1 the path must reproduce nvfp4b_moe_forward bit for bit (same quantisation, same per-row scales, the same
fp16 rows summed in slot order).  G = 2 and 4 are emulated on the one GPU: every rank's records are exchanged by
copies in rank order (what the all-to-all does), each rank owning E/G experts; each rank's output must equal
nvfp4b_moe_forward over the full expert arena for that rank's tokens, bit for bit."""
import numpy as np
import pytest
import torch

from gpu_util import require_gpu
from test_moe_gpu import make_problem, route_and_calibrate

pytestmark = pytest.mark.gpu


def _ref(p, P, x, ids, w, amax):
    return p.moe_forward(x, ids, w, P["arena"], P["ws"], in_amax=amax).clone()


def test_ep_single_rank_bit_identical_to_moe_forward():
    p, P = make_problem(200, 512, 128, 32, 8, seed=41)
    ids, w, _, _ = route_and_calibrate(p, P)
    amax = p.amax(P["x"])
    ref = _ref(p, P, P["x"], ids, w, amax)
    import gemma_cuda_server_b200.expert_parallel as epm
    ops = epm.KernelOps(p, P["arena"], P["E"], P["topk"], T_cap=256, G=1)
    layer = epm.ExpertParallelMoE(ops)
    out = torch.full_like(ref, float("nan"))
    layer.forward(P["x"], ids, w, out, in_amax=amax)
    torch.cuda.synchronize()
    assert p.read_device_error() == 0
    assert torch.equal(out, ref)
    base = torch.randn_like(ref)
    out2 = base.clone()
    layer.forward(P["x"], ids, w, out2, in_amax=amax, accumulate=True)
    ref2 = p.moe_forward(P["x"], ids, w, P["arena"], P["ws"], in_amax=amax, out=base.clone(), accumulate=True)
    torch.cuda.synchronize()
    assert torch.equal(out2, ref2)                      # same order: out, then the slots in order


@pytest.mark.parametrize("G", [2, 4])
def test_ep_emulated_ranks_bit_identical(G):
    T = 96
    p, P = make_problem(T * G, 512, 128, 32, 8, seed=43)
    ids_all, w_all, _, _ = route_and_calibrate(p, P)
    import gemma_cuda_server_b200.expert_parallel as epm
    E, k = P["E"], P["topk"]
    ops = [epm.KernelOps(p, P["arena"].slice(r * E // G, (r + 1) * E // G), E, k, T_cap=T, G=G) for r in range(G)]
    xs = [P["x"][r * T:(r + 1) * T].contiguous() for r in range(G)]
    ids = [ids_all[r * T:(r + 1) * T].contiguous() for r in range(G)]
    ws = [w_all[r * T:(r + 1) * T].contiguous() for r in range(G)]
    amaxes = [p.amax(x) for x in xs]
    counts = []
    for r in range(G):
        sc, _ = ops[r].dispatch(xs[r], ids[r], ws[r], in_amax=amaxes[r])
        counts.append(sc.tolist())
    # records: source rank order inside every destination (all-to-all semantics)
    recv_n = [sum(counts[s][d] for s in range(G)) for d in range(G)]
    for d in range(G):
        off = 0
        for s in range(G):
            start = sum(counts[s][:d])
            n = counts[s][d]
            ops[d].recv[off:off + n].copy_(ops[s].send[start:start + n])
            off += n
    rows = [ops[d].expert(ops[d].recv[:recv_n[d]], recv_n[d]).clone() for d in range(G)]
    for s in range(G):
        off_back = 0
        for d in range(G):
            n = counts[s][d]
            src_off = sum(counts[q][d] for q in range(s))
            ops[s].back[off_back:off_back + n].copy_(rows[d][src_off:src_off + n])
            off_back += n
    torch.cuda.synchronize()
    assert p.read_device_error() == 0
    for r in range(G):
        out = torch.full((T, P["H"]), float("nan"), device="cuda")
        ops[r].combine(ops[r].back[:sum(counts[r])], out, False)
        ref = _ref(p, P, xs[r], ids[r], ws[r], amaxes[r])
        torch.cuda.synchronize()
        assert torch.equal(out, ref), f"rank {r}: max diff {(out - ref).abs().max().item()}"
