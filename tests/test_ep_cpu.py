"""Expert-parallel orchestration on CPU: two gloo ranks run ExpertParallelMoE (expert_parallel.py) with float64 stand-in
ops (same record order, same per-expert function on both sides), and the result must equal the single-process
layer over all experts.  This covers the collective steps (count exchange, fixed-slot record all-to-all, return trip,
slot-ordered combine) without a GPU; the device ops are checked against the oracle in test_ep_gpu.py."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from __graft_entry__ import load_package

E, H, TOPK, T = 16, 32, 4, 24


def expert_fn(e: int, x: np.ndarray) -> np.ndarray:
    """Per-expert stand-in for the FFN, identical on every rank (seeded by the global expert id)."""
    rng = np.random.default_rng(1000 + e)
    a = rng.standard_normal((H, 8)) * 0.3
    b = rng.standard_normal((8, H)) * 0.3
    return np.tanh(x @ a) @ b


def routing(rank: int):
    rng = np.random.default_rng(rank)
    x = rng.standard_normal((T, H))
    ids = np.stack([rng.choice(E, TOPK, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.random((T, TOPK))
    w /= w.sum(1, keepdims=True)
    return x, ids, w


class OracleOps:
    """float64 CPU stand-in with KernelOps' interface: records in destination-major fixed slots (capacity =
    T * topk per destination), each destination's records in expert order, token order inside an expert."""

    def __init__(self, rank: int, G: int):
        self.rank, self.G, self.topk, self.E = rank, G, TOPK, E
        self.C = T * TOPK
        self.counts = torch.zeros(2 * G, dtype=torch.int32)
        self.send = torch.zeros((G * self.C, H + 2), dtype=torch.float64)
        self.recv = torch.zeros_like(self.send)
        self.back = torch.zeros((G * self.C, H), dtype=torch.float64)

    def dispatch(self, x, ids, weights, in_gscale=None, in_amax=None):
        x, ids, weights = x.numpy(), ids.numpy(), weights.numpy()
        el = E // self.G
        a = np.argsort(ids.reshape(-1), kind="stable")              # expert order, token order inside an expert
        e = ids.reshape(-1)[a]
        d = e // el
        per_rank = np.bincount(d, minlength=self.G)
        starts = np.concatenate([[0], np.cumsum(per_rank)[:-1]])
        slot = d * self.C + (np.arange(a.size) - starts[d])
        self.slot = np.empty_like(a)
        self.slot[a] = slot
        rec = np.concatenate([x[a // TOPK], (e % el)[:, None], weights.reshape(-1)[a][:, None]], 1)
        self.send.zero_()
        self.send[torch.from_numpy(slot)] = torch.from_numpy(rec)
        self.T = x.shape[0]
        self.counts[:self.G] = torch.from_numpy(per_rank.astype(np.int32))
        return self.counts[:self.G], self.counts[self.G:]

    def expert(self, records, recv_counts):
        r = records.numpy()
        out = np.zeros((r.shape[0], H))
        for s in range(self.G):
            for j in range(int(recv_counts[s])):
                i = s * self.C + j
                e = self.rank * (E // self.G) + int(r[i, H])
                out[i] = r[i, H + 1] * expert_fn(e, r[i:i + 1, :H])[0]
        return torch.from_numpy(out)

    def combine(self, back, out, accumulate):
        b = back.numpy()
        res = np.zeros((self.T, H))
        for t in range(self.T):
            for j in range(TOPK):
                res[t] += b[self.slot[t * TOPK + j]]
        out.copy_(torch.from_numpy(res) + (out if accumulate else 0))
        return out


def reference(rank: int) -> np.ndarray:
    x, ids, w = routing(rank)
    out = np.zeros((T, H))
    for t in range(T):
        for j in range(TOPK):
            out[t] += w[t, j] * expert_fn(int(ids[t, j]), x[t:t + 1])[0]
    return out


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        load_package()
        import gemma_cuda_server_b200.expert_parallel as epm
        x, ids, w = routing(rank)
        layer = epm.ExpertParallelMoE(OracleOps(rank, world))
        out = torch.zeros((T, H), dtype=torch.float64)
        layer.forward(torch.from_numpy(x), torch.from_numpy(ids), torch.from_numpy(w), out)
        q.put((rank, float(np.abs(out.numpy() - reference(rank)).max())))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [1, 2])
def test_expert_parallel_orchestration_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    errs = dict(q.get(timeout=5) for _ in range(world))
    assert max(errs.values()) < 1e-12, errs
