"""Host side of the peer-memory exchange on CPU: PeerExchange.create over two gloo ranks with a stand-in for the
library's IPC calls.  Every rank must end up with device tables whose column g addresses rank g's buffers (its own
allocation for itself, the mapping of rank g's handle otherwise) at the offsets of nvfp4b_ep_p2p_buffer_bytes, and
close() must unmap exactly the peers' mappings and free exactly its own allocation."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from __graft_entry__ import load_package

G, C, H = 2, 96, 512


class FakeIpc:
    """The IPC part of the library on CPU: rank r's allocation is at 1 GiB * (r + 1); a handle names its owner; the
    mapping of rank s's handle in rank r lands at 1 TiB * (r + 1) + s * 1 GiB."""

    def __init__(self, pkg, rank):
        self.pkg, self.rank = pkg, rank
        self.freed, self.closed = [], []
        self.EpPeers = pkg.EpPeers

    def ep_p2p_buffer_layout(self, G, C, H):
        return self.pkg.ep_p2p_buffer_layout(G, C, H)      # the real layout (host-only call)

    def ipc_alloc(self, nbytes):
        return (1 << 30) * (self.rank + 1)

    def ipc_handle(self, ptr):
        return bytes([ptr >> 30]) + bytes(63)

    def ipc_open(self, handle):
        owner = handle[0] - 1
        return (1 << 40) * (self.rank + 1) + owner * (1 << 30)

    def ipc_close(self, ptr):
        self.closed.append(ptr)

    def ipc_free(self, ptr):
        self.freed.append(ptr)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pkg = load_package()
        import gemma_cuda_server_b200.expert_parallel as epm
        fake = FakeIpc(pkg, rank)
        ex = epm.PeerExchange.create(fake, world, C, H, device="cpu")
        _, off = pkg.ep_p2p_buffer_layout(world, C, H)
        tables = ex.tables.tolist()
        p = ex.peers
        own = (1 << 30) * (rank + 1)
        mine = (p.rank, p.G, p.capacity, p.my_recv, p.my_back, p.my_counts, p.my_flags, p.state)
        ex.close()
        q.put((rank, tables, off, own, mine, fake.freed, fake.closed))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_peer_exchange_tables_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, G, port, q)) for r in range(G)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = {r: rest for r, *rest in (q.get(timeout=5) for _ in range(G))}
    for r, (tables, off, own, mine, freed, closed) in res.items():
        for g in range(G):
            base = own if g == r else (1 << 40) * (r + 1) + g * (1 << 30)
            for i in range(4):
                assert tables[i][g] == base + off[i], (r, g, i)
        assert mine == (r, G, C, own + off[0], own + off[1], own + off[2], own + off[3], own + off[4])
        assert freed == [own]
        assert closed == [(1 << 40) * (r + 1) + g * (1 << 30) for g in range(G) if g != r]


# ---- failures of the set-up, made on the host: a layout mismatch, a rank that never joins --------------------------

def _fault_worker(rank, world, port, mode, q):
    import datetime
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    try:
        pkg = load_package()
        import gemma_cuda_server_b200.expert_parallel as epm
        fake = FakeIpc(pkg, rank)
        if mode == "absent" and rank == 1:
            time.sleep(12)                     # joined the process group, never posts its exchange handle
            q.put((rank, "absent", 0.0, fake.freed))
            return
        cap = C + 16 if (mode == "mismatch" and rank == 1) else C
        t0 = time.monotonic()
        try:
            epm.PeerExchange.create(fake, world, cap, H, device="cpu")
            outcome = "created"
        except ValueError as e:
            outcome = "ValueError: " + str(e)
        except RuntimeError as e:              # gloo collective timeout / peer gone
            outcome = "RuntimeError"
        q.put((rank, outcome, time.monotonic() - t0, fake.freed))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run_fault(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fault_worker, args=(r, G, port, mode, q)) for r in range(G)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return {r: rest for r, *rest in (q.get(timeout=5) for _ in range(G))}


def test_peer_exchange_layout_mismatch_stops_every_rank():
    """One rank built for another capacity: every rank raises before mapping anything, and frees its allocation."""
    res = _run_fault("mismatch")
    for r, (outcome, _, freed) in res.items():
        assert outcome.startswith("ValueError") and "disagree" in outcome, (r, outcome)
        assert freed == [(1 << 30) * (r + 1)]


def test_peer_exchange_absent_rank_times_out():
    """A rank that never posts its handle: the other rank's set-up ends with an error within the process group's
    timeout (3 s here) instead of waiting for ever, and frees its allocation."""
    res = _run_fault("absent")
    outcome, elapsed, freed = res[0]
    assert outcome == "RuntimeError", outcome
    assert elapsed < 10.0, elapsed
    assert freed == [1 << 30]
