"""Expert-parallel MoE over NVLink peer memory on real GPUs: one process per GPU (NCCL process group only for the
set-up exchange of CUDA IPC handles), each rank owning E/G experts and T tokens.  Every rank's output must equal
nvfp4b_moe_forward over the full expert arena for its tokens, bit for bit, eagerly and when the layer is replayed
from a CUDA graph; the router-fused form (nvfp4b_ep_p2p_layer) must equal nvfp4b_moe_layer likewise.  Needs at least 2 GPUs (skipped otherwise)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

T, H, I, E, TOPK = 96, 512, 128, 32, 8


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    ex = None
    try:
        from __graft_entry__ import load_package
        load_package()
        from test_moe_gpu import make_problem, route_and_calibrate
        import gemma_cuda_server_b200.expert_parallel as epm
        p, P = make_problem(T * world, H, I, E, TOPK, seed=61)
        ids_all, w_all, _, _ = route_and_calibrate(p, P)
        x = P["x"][rank * T:(rank + 1) * T].contiguous()
        ids = ids_all[rank * T:(rank + 1) * T].contiguous()
        w = w_all[rank * T:(rank + 1) * T].contiguous()
        amax = p.amax(x)
        ref = p.moe_forward(x, ids, w, P["arena"], P["ws"], in_amax=amax).clone()
        C = epm.P2PKernelOps.default_capacity(T, TOPK, world)
        ex = epm.PeerExchange.create(p, world, C, H)
        ops = epm.P2PKernelOps(p, P["arena"].slice(rank * E // world, (rank + 1) * E // world), E, TOPK, T, ex)
        layer = epm.ExpertParallelMoE(ops)
        results = []
        out = torch.full((T, H), float("nan"), device="cuda")
        for _ in range(3):
            out.fill_(float("nan"))
            layer.forward(x, ids, w, out, in_amax=amax)
            torch.cuda.synchronize()
            results.append(torch.equal(out, ref))
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                layer.forward(x, ids, w, out, in_amax=amax)
        torch.cuda.current_stream().wait_stream(s)
        for _ in range(2):
            out.fill_(float("nan"))
            torch.cuda.synchronize()
            dist.barrier()
            g.replay()
            torch.cuda.synchronize()
            results.append(torch.equal(out, ref))
        # the fused form (nvfp4b_ep_p2p_layer: router + layer on this rank in one call) against the single-GPU
        # router-fused layer over the full arena, eagerly, twice
        ids_f = torch.empty((T, TOPK), dtype=torch.int32, device="cuda")
        w_f = torch.empty((T, TOPK), dtype=torch.float32, device="cuda")
        ref_ids = torch.empty_like(ids_f)
        ref_w = torch.empty_like(w_f)
        ref_f = p.moe_layer(x, P["proj"], TOPK, P["arena"], P["ws"], ids=ref_ids, weights=ref_w, in_amax=amax).clone()
        for _ in range(2):
            out.fill_(float("nan"))
            layer.forward_routed(x, P["proj"], ids_f, w_f, out, in_amax=amax)
            torch.cuda.synchronize()
            dist.barrier()
            results.append(torch.equal(out, ref_f) and torch.equal(ids_f, ref_ids) and torch.equal(w_f, ref_w))
        err = p.read_device_error()
        state = ex.state_words()
        del g
        q.put((rank, results, err, state, int(ops.overflow.item())))
    finally:
        torch.cuda.synchronize()
        dist.barrier()
        if ex is not None:
            ex.close()
        dist.barrier()
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ep_p2p_processes_bit_identical(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = dict((r, rest) for r, *rest in (q.get(timeout=5) for _ in range(world)))
    for r, (results, err, state, overflow) in res.items():
        assert err == 0, (r, err)
        assert overflow == 0
        assert all(results), (r, results)
        assert state[:3] == [7, 0, 0], (r, state)      # 3 eager layers + 2 replays + 2 fused; counters reset
