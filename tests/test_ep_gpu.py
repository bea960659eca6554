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


def _emulate(p, P, G, T, capacity=None):
    """G ranks on one GPU: each rank's slots are exchanged by copies (what the all-to-all does)."""
    import gemma_cuda_server_b200.expert_parallel as epm
    E, k = P["E"], P["topk"]
    ops = [epm.KernelOps(p, P["arena"].slice(r * E // G, (r + 1) * E // G), E, k, T_cap=T, G=G, capacity=capacity)
           for r in range(G)]
    C = ops[0].capacity
    xs = [P["x"][r * T:(r + 1) * T].contiguous() for r in range(G)]
    ids = [P["ids"][r * T:(r + 1) * T].contiguous() for r in range(G)]
    ws = [P["w"][r * T:(r + 1) * T].contiguous() for r in range(G)]
    amaxes = [p.amax(x) for x in xs]
    for r in range(G):
        ops[r].dispatch(xs[r], ids[r], ws[r], in_amax=amaxes[r])
    for d in range(G):
        for s in range(G):
            ops[d].counts[G + s] = ops[s].counts[d]
            ops[d].recv[s * C:(s + 1) * C].copy_(ops[s].send[d * C:(d + 1) * C])
    rows = [ops[d].expert(ops[d].recv, ops[d].counts[G:]).clone() for d in range(G)]
    for s in range(G):
        for d in range(G):
            ops[s].back[d * C:(d + 1) * C].copy_(rows[d][s * C:(s + 1) * C])
    outs = []
    for r in range(G):
        out = torch.full((T, P["H"]), float("nan"), device="cuda")
        ops[r].combine(ops[r].back, out, False)
        outs.append(out)
    torch.cuda.synchronize()
    return ops, xs, ids, ws, amaxes, outs


@pytest.mark.parametrize("G", [2, 4])
def test_ep_emulated_ranks_bit_identical(G):
    T = 96
    p, P = make_problem(T * G, 512, 128, 32, 8, seed=43)
    P["ids"], P["w"], _, _ = route_and_calibrate(p, P)
    ops, xs, ids, ws, amaxes, outs = _emulate(p, P, G, T)
    assert p.read_device_error() == 0
    assert not any(int(o.overflow.item()) for o in ops)
    for r in range(G):
        ref = _ref(p, P, xs[r], ids[r], ws[r], amaxes[r])
        torch.cuda.synchronize()
        assert torch.equal(outs[r], ref), f"rank {r}: max diff {(outs[r] - ref).abs().max().item()}"


def test_ep_overflow_is_flagged():
    """A capacity below a rank pair's record count sets the overflow flag (the excess records are dropped)."""
    G, T = 2, 64
    p, P = make_problem(T * G, 512, 128, 32, 8, seed=47)
    P["ids"], P["w"], _, _ = route_and_calibrate(p, P)
    ops, *_ = _emulate(p, P, G, T, capacity=16)          # ~T*8/2 = 256 records per pair on average
    assert all(int(o.overflow.item()) == 1 for o in ops)
    assert all(int(c) <= 16 for o in ops for c in o.counts.tolist())


# ---- exchange over peer memory (nvfp4b_ep_p2p_*): records and rows stored into the other ranks' buffers ----------

def _emulate_p2p(p, P, G, T, capacity=None, layers=1):
    """G ranks on one GPU sharing exchange buffers: every rank's dispatch, then every rank's experts, then every
    rank's combine, on one stream (each wait finds its flags already raised).  `layers` repeats the layer to check
    that the per-layer epochs advance."""
    import gemma_cuda_server_b200.expert_parallel as epm
    E, k, H = P["E"], P["topk"], P["H"]
    C = capacity or epm.P2PKernelOps.default_capacity(T, k, G)
    ex = epm.PeerExchange.local_group(p, G, C, H)
    ops = [epm.P2PKernelOps(p, P["arena"].slice(r * E // G, (r + 1) * E // G), E, k, T, ex[r]) for r in range(G)]
    xs = [P["x"][r * T:(r + 1) * T].contiguous() for r in range(G)]
    ids = [P["ids"][r * T:(r + 1) * T].contiguous() for r in range(G)]
    ws = [P["w"][r * T:(r + 1) * T].contiguous() for r in range(G)]
    amaxes = [p.amax(x) for x in xs]
    outs = [torch.full((T, H), float("nan"), device="cuda") for _ in range(G)]
    for _ in range(layers):
        for r in range(G):
            ops[r].dispatch(xs[r], ids[r], ws[r], in_amax=amaxes[r])
        for r in range(G):
            ops[r].expert()
        for r in range(G):
            ops[r].combine(outs[r], False)
    torch.cuda.synchronize()
    return ex, ops, xs, ids, ws, amaxes, outs


@pytest.mark.parametrize("G,layers", [(1, 1), (2, 3), (4, 2)])
def test_ep_p2p_emulated_ranks_bit_identical(G, layers):
    T = 96
    p, P = make_problem(T * G, 512, 128, 32, 8, seed=53)
    P["ids"], P["w"], _, _ = route_and_calibrate(p, P)
    ex, ops, xs, ids, ws, amaxes, outs = _emulate_p2p(p, P, G, T, layers=layers)
    try:
        assert p.read_device_error() == 0
        assert not any(int(o.overflow.item()) for o in ops)
        for r in range(G):
            ref = _ref(p, P, xs[r], ids[r], ws[r], amaxes[r])
            torch.cuda.synchronize()
            assert torch.equal(outs[r], ref), f"rank {r}: max diff {(outs[r] - ref).abs().max().item()}"
        for e in ex:                                   # epoch = layers run; completion counters back at zero
            assert e.state_words()[:3] == [layers, 0, 0]
        total = sum(sum(e.recv_counts()) for e in ex)
        assert total == G * T * P["topk"]              # every assignment crossed exactly once
    finally:
        for e in ex:
            e.close()


def test_ep_p2p_overflow_is_flagged():
    G, T = 2, 64
    p, P = make_problem(T * G, 512, 128, 32, 8, seed=59)
    P["ids"], P["w"], _, _ = route_and_calibrate(p, P)
    ex, ops, *_ = _emulate_p2p(p, P, G, T, capacity=16)
    try:
        assert p.read_device_error() == 0
        assert all(int(o.overflow.item()) == 1 for o in ops)
        assert all(c <= 16 for e in ex for c in e.recv_counts())
    finally:
        for e in ex:
            e.close()


# ---- chained outputs of the combine (residual stream: the next layer's bf16 input and its amax) -----------------

def test_moe_forward_chain_outputs():
    """nvfp4b_moe_forward_chain: out as nvfp4b_moe_forward, plus x_next = bf16(out) and amax_next = max |x_next|,
    also when x_next / amax_next are the layer's own x / amax (in place)."""
    p, P = make_problem(200, 512, 128, 32, 8, seed=67)
    ids, w, _, _ = route_and_calibrate(p, P)
    amax = p.amax(P["x"])
    base = torch.randn((200, 512), device="cuda")
    ref = p.moe_forward(P["x"], ids, w, P["arena"], P["ws"], in_amax=amax, out=base.clone(), accumulate=True)
    ref_x = ref.to(torch.bfloat16)
    ref_a = ref_x.float().abs().max()
    out, xn, an = base.clone(), torch.empty_like(P["x"]), torch.full((1,), 123.0, device="cuda")
    p.moe_forward(P["x"], ids, w, P["arena"], P["ws"], in_amax=amax, out=out, accumulate=True, x_next=xn,
                  amax_next=an)
    x2, a2, out2 = P["x"].clone(), amax.clone(), base.clone()
    p.moe_forward(x2, ids, w, P["arena"], P["ws"], in_amax=a2, out=out2, accumulate=True, x_next=x2, amax_next=a2)
    torch.cuda.synchronize()
    assert p.read_device_error() == 0
    assert torch.equal(out, ref) and torch.equal(xn, ref_x) and an.item() == ref_a.item()
    assert torch.equal(out2, ref) and torch.equal(x2, ref_x) and a2.item() == ref_a.item()


def test_ep_p2p_combine_chain_outputs():
    """The peer-memory combine with the chained outputs, G = 2 emulated: same out, x_next = bf16(out), amax."""
    import gemma_cuda_server_b200.expert_parallel as epm
    G, T = 2, 96
    p, P = make_problem(T * G, 512, 128, 32, 8, seed=71)
    P["ids"], P["w"], _, _ = route_and_calibrate(p, P)
    E, k, H = P["E"], P["topk"], P["H"]
    ex = epm.PeerExchange.local_group(p, G, epm.P2PKernelOps.default_capacity(T, k, G), H)
    try:
        ops = [epm.P2PKernelOps(p, P["arena"].slice(r * E // G, (r + 1) * E // G), E, k, T, ex[r]) for r in range(G)]
        xs = [P["x"][r * T:(r + 1) * T].clone() for r in range(G)]
        amaxes = [p.amax(x) for x in xs]
        refs = [p.moe_forward(xs[r], P["ids"][r * T:(r + 1) * T].contiguous(), P["w"][r * T:(r + 1) * T].contiguous(),
                              P["arena"], P["ws"], in_amax=amaxes[r]).clone() for r in range(G)]
        outs = [torch.zeros((T, H), device="cuda") for _ in range(G)]
        for r in range(G):
            ops[r].dispatch(xs[r], P["ids"][r * T:(r + 1) * T].contiguous(), P["w"][r * T:(r + 1) * T].contiguous(),
                            in_amax=amaxes[r])
        for r in range(G):
            ops[r].expert()
        for r in range(G):                       # in place: the rank's own x and amax become the next layer's
            ops[r].combine(outs[r], True, x_next=xs[r], amax_next=amaxes[r])
        torch.cuda.synchronize()
        assert p.read_device_error() == 0
        for r in range(G):
            assert torch.equal(outs[r], refs[r])
            assert torch.equal(xs[r], refs[r].to(torch.bfloat16))
            assert amaxes[r].item() == refs[r].to(torch.bfloat16).float().abs().max().item()
    finally:
        for e in ex:
            e.close()


def test_ep_p2p_missing_rank_ends_in_timeout_not_hang():
    """A rank that never dispatches (G = 2 emulated, rank 1 absent): rank 0's expert side waits for rank 1's records
    and its combine for rank 1's rows.  With the peer-wait bound set to 50 ms the first wait runs out, the device
    error word reads the peer-timeout code, the later wait does not spin at all, and the stream completes.  The
    epochs of that exchange are then out of step, so a new exchange is made; it runs clean and bit-identical."""
    import time
    import gemma_cuda_server_b200.expert_parallel as epm
    G, T = 2, 64
    p, P = make_problem(T * G, 512, 128, 32, 8, seed=61)
    P["ids"], P["w"], _, _ = route_and_calibrate(p, P)
    E, k, H = P["E"], P["topk"], P["H"]
    assert p.read_device_error() == 0
    p.ep_set_peer_wait_ns(50_000_000)
    ex = epm.PeerExchange.local_group(p, G, epm.P2PKernelOps.default_capacity(T, k, G), H)
    try:
        ops = [epm.P2PKernelOps(p, P["arena"].slice(r * E // G, (r + 1) * E // G), E, k, T, ex[r]) for r in range(G)]
        x0 = P["x"][:T].contiguous()
        amax0 = p.amax(x0)
        torch.cuda.synchronize()
        t0 = time.monotonic()
        ops[0].dispatch(x0, P["ids"][:T].contiguous(), P["w"][:T].contiguous(), in_amax=amax0)
        ops[0].expert()                                   # rank 1's records never land
        out = torch.zeros((T, H), device="cuda")
        ops[0].combine(out, False)                        # nor do rank 1's rows
        torch.cuda.synchronize()
        elapsed = time.monotonic() - t0
        assert p.read_device_error(reset=True) == p.PEER_TIMEOUT
        assert elapsed < 5.0, elapsed                     # one 50 ms wait, not 10 s per flag per block
        assert torch.isfinite(out).all()                  # the kernels went on with what had landed
    finally:
        p.ep_set_peer_wait_ns(0)
        for e in ex:
            e.close()
    assert p.read_device_error() == 0
    ex, ops, xs, ids, ws, amaxes, outs = _emulate_p2p(p, P, G, T)
    try:
        assert p.read_device_error() == 0
        for r in range(G):
            assert torch.equal(outs[r], _ref(p, P, xs[r], ids[r], ws[r], amaxes[r]))
    finally:
        for e in ex:
            e.close()
