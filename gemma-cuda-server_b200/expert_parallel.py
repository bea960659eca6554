"""Expert-parallel MoE layer: E experts sharded over the ranks of a torch.distributed group (E/G consecutive experts
per rank), routed assignments exchanged with all-to-all collectives (NCCL over NVLink on B200s, one process per GPU).

The reference runs the MoE of a layer on one GPU (src/forward.cu:516-553: router, per-expert W4A16 GEMVs, weighted
sum).  This is the expert-parallel form of the same computation.  One layer, per rank:

  1. route (caller): ids [T, k], weights [T, k]
  2. ops.dispatch: one record per assignment (NVFP4 codes + scales of the token, local expert, router weight,
     activation global scale) into fixed destination-major slots (capacity per destination); counts per rank
  3. all-to-all of the counts (G ints) and of the record slots
  4. ops.expert: the local experts on the received slots -> weighted fp16 rows, one per slot
  5. all-to-all of the row slots back to their sources
  6. ops.combine: slot-ordered fp32 sum into out (bit-identical to the single-GPU layer at G = 1)

P2PKernelOps runs the same layer with steps 3 and 5 fused into the kernels around them (nvfp4b_ep_p2p_*): the pack
kernel stores records straight into the destination ranks' receive slots and the down-projection epilogue stores
rows straight into the source ranks' return rows, over NVLink peer memory shared through CUDA IPC (PeerExchange);
per-(rank pair, layer) flags replace the collectives, so forward() issues no collective at all.

Every buffer has a fixed size, so nothing is read back to the host and a whole stack of layers can be captured in
one CUDA graph.  A destination receiving more than `capacity` records from one source sets the overflow flag
(check with overflowed() after the step); capacity = T_cap * topk never overflows.  `ops` does the device work;
KernelOps is the sm_100a implementation (the C ABI of libnvfp4_b200.so).  The collectives are issued on the
caller's current stream, in the same order on every rank.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def default_capacity(T_cap: int, topk: int, G: int) -> int:
    """Record slots per (source, destination) pair: the even share n = T_cap * topk / G plus 8 sqrt(n) + 32 (eight
    standard deviations of a uniform router's count), rounded up to 16, at most T_cap * topk (which cannot
    overflow)."""
    share = T_cap * topk / G
    return min(T_cap * topk, int(share + 8 * share ** 0.5 + 32 + 15) // 16 * 16)


def no_drop_capacity(T_cap: int, topk: int, G: int) -> int:
    """Record slots per (source, destination) pair that can never overflow: every assignment of T_cap tokens.  On the
    peer-memory path only the records that exist cross the link, so this costs memory only: G * T_cap * topk *
    (record + fp16 row) bytes per rank (237 MB at G = 8, 512 tokens, top-8, H = 2816)."""
    return T_cap * topk


class KernelOps:
    """Device side of one expert-parallel layer on this rank: buffers sized for up to T_cap tokens per rank and
    `capacity` records per (source, destination) pair.  The all-to-alls move every slot, so the default is the even
    share n = T_cap * topk / G plus 8 sqrt(n) + 32 (eight standard deviations of a uniform router's count), at most
    T_cap * topk (which cannot overflow)."""

    def __init__(self, pkg, experts, E: int, topk: int, T_cap: int, G: int, capacity: int | None = None,
                 device="cuda"):
        if E % G:
            raise ValueError(f"{E} experts do not split over {G} ranks")
        if experts.E != E // G:
            raise ValueError(f"local arena holds {experts.E} experts, expected {E // G}")
        self.pkg, self.experts, self.E, self.topk, self.T_cap, self.G = pkg, experts, E, topk, T_cap, G
        H, I = experts.H, experts.I
        self.H = H
        if capacity is None:
            capacity = default_capacity(T_cap, topk, G)
        self.capacity = capacity
        self.record_bytes = pkg.ep_record_bytes(H)
        n = G * capacity
        self.src_ws = pkg.moe_workspace(T_cap, H, 32, E, topk, device=device)
        self.exp_ws = pkg.moe_workspace(n, H, I, E // G, 1, device=device)
        self.send = torch.empty((n, self.record_bytes), dtype=torch.uint8, device=device)
        self.recv = torch.empty((n, self.record_bytes), dtype=torch.uint8, device=device)
        self.back = torch.empty((n, H), dtype=torch.float16, device=device)
        self.counts = torch.zeros(2 * G, dtype=torch.int32, device=device)
        self.overflow = torch.zeros(1, dtype=torch.int32, device=device)

    def dispatch(self, x, ids, weights, in_gscale=None, in_amax=None):
        T = x.shape[0]
        if T > self.T_cap:
            raise ValueError(f"{T} tokens exceed the capacity {self.T_cap}")
        self.T = T
        self.pkg.ep_dispatch(x, ids, weights, self.E, self.G, self.capacity, self.src_ws, self.send,
                             self.counts[:self.G], self.overflow, in_gscale=in_gscale, in_amax=in_amax)
        return self.counts[:self.G], self.counts[self.G:]

    def expert(self, records, recv_counts):
        return self.pkg.ep_expert_forward(records, self.G, self.capacity, recv_counts, self.experts, self.exp_ws)

    def combine(self, back, out, accumulate: bool):
        return self.pkg.ep_combine(back, self.T, self.topk, self.E, self.src_ws, out, accumulate=accumulate)


class PeerExchange:
    """One rank's exchange buffers (one zeroed device allocation: receive slots, return rows, counts, flags,
    private state) and the device tables of every rank's buffers, as the nvfp4b_ep_peers the kernels take."""

    def __init__(self, pkg, rank: int, G: int, capacity: int, H: int, base: int, bases: list[int],
                 owned: list[int], opened: list[int], device="cuda"):
        self.pkg, self.rank, self.G, self.capacity, self.H = pkg, rank, G, capacity, H
        self.base, self._owned, self._opened = base, owned, opened
        _, off = pkg.ep_p2p_buffer_layout(G, capacity, H)
        self.off = off
        self.tables = torch.tensor([[b + off[i] for b in bases] for i in range(4)], dtype=torch.int64, device=device)
        tp = self.tables.data_ptr()
        self.peers = pkg.EpPeers(rank, G, capacity, tp, tp + 8 * G, tp + 16 * G, tp + 24 * G,
                                 base + off[0], base + off[1], base + off[2], base + off[3], base + off[4])

    @classmethod
    def local_group(cls, pkg, G: int, capacity: int, H: int, device="cuda") -> list["PeerExchange"]:
        """G exchanges on the current device that address one another: emulated ranks for single-GPU tests.  Their
        layers must run rank after rank on one stream (dispatch of every rank, then experts, then combines)."""
        nbytes, _ = pkg.ep_p2p_buffer_layout(G, capacity, H)
        bases = [pkg.ipc_alloc(nbytes) for _ in range(G)]
        return [cls(pkg, r, G, capacity, H, bases[r], bases, [bases[r]], [], device) for r in range(G)]

    @classmethod
    def create(cls, pkg, G: int, capacity: int, H: int, group=None, device="cuda") -> "PeerExchange":
        """This process's exchange in a group of G processes, one per GPU of the node: allocates, shares the CUDA
        IPC handle with every rank (all_gather_object over `group`) and maps the others' buffers."""
        rank = dist.get_rank(group)
        if dist.get_world_size(group) != G:
            raise ValueError(f"exchange for {G} ranks created in a group of {dist.get_world_size(group)}")
        nbytes, _ = pkg.ep_p2p_buffer_layout(G, capacity, H)
        base = pkg.ipc_alloc(nbytes)
        # Every rank publishes its handle with the layout it was built for: a rank that disagrees on G, capacity or
        # H would store records and rows at offsets the others do not read, so a mismatch stops every rank here.
        mine = (pkg.ipc_handle(base), G, capacity, H)
        got = [None] * G
        try:
            dist.all_gather_object(got, mine, group=group)
            layouts = {(g, c, h) for _, g, c, h in got}
            if len(layouts) != 1:
                raise ValueError(f"ranks disagree on the exchange layout (G, capacity, H): {sorted(layouts)}")
        except BaseException:
            pkg.ipc_free(base)
            raise
        bases, opened = [], []
        for r, (h, *_) in enumerate(got):
            if r == rank:
                bases.append(base)
            else:
                p = pkg.ipc_open(h)
                opened.append(p)
                bases.append(p)
        return cls(pkg, rank, G, capacity, H, base, bases, [base], opened, device)

    def recv_counts(self) -> list[int]:
        """Records this rank received from each source in the last layer (synchronous read)."""
        return self.pkg.ep_p2p_recv_counts(self.peers)

    def state_words(self) -> list[int]:
        """This rank's private words [layer epoch, pack completions, down completions, spare] (synchronous)."""
        return self.pkg.ep_p2p_state(self.peers)

    def close(self):
        """Unmaps the peers' buffers and frees this rank's (call once every rank is done with them)."""
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        for p in self._opened:
            self.pkg.ipc_close(p)
        for p in self._owned:
            self.pkg.ipc_free(p)
        self._opened, self._owned = [], []


class P2PKernelOps:
    """Device side of one expert-parallel layer whose exchanges run over peer memory (no collective)."""

    p2p = True

    def __init__(self, pkg, experts, E: int, topk: int, T_cap: int, exchange: PeerExchange, device="cuda"):
        G = exchange.G
        if E % G:
            raise ValueError(f"{E} experts do not split over {G} ranks")
        if experts.E != E // G:
            raise ValueError(f"local arena holds {experts.E} experts, expected {E // G}")
        self.pkg, self.experts, self.E, self.topk, self.T_cap, self.G = pkg, experts, E, topk, T_cap, G
        self.ex = exchange
        self.capacity = exchange.capacity
        self.H = experts.H
        self.src_ws = pkg.moe_workspace(T_cap, experts.H, 32, E, topk, device=device)
        self.exp_ws = pkg.moe_workspace(G * self.capacity, experts.H, experts.I, E // G, 1, device=device)
        self.overflow = torch.zeros(1, dtype=torch.int32, device=device)

    # Skewed routing (real routers are far from uniform) must not drop tokens, and padding never crosses the link
    # here, so the peer-memory path defaults to the capacity that cannot overflow.
    default_capacity = staticmethod(no_drop_capacity)

    def dispatch(self, x, ids, weights, in_gscale=None, in_amax=None):
        T = x.shape[0]
        if T > self.T_cap:
            raise ValueError(f"{T} tokens exceed the capacity {self.T_cap}")
        self.T = T
        self.pkg.ep_p2p_dispatch(x, ids, weights, self.E, self.src_ws, self.ex.peers, self.overflow,
                                 in_gscale=in_gscale, in_amax=in_amax)

    def expert(self):
        self.pkg.ep_p2p_expert_forward(self.experts, self.exp_ws, self.ex.peers)

    def combine(self, out, accumulate: bool, x_next=None, amax_next=None):
        return self.pkg.ep_p2p_combine(self.T, self.topk, self.E, self.src_ws, self.ex.peers, out,
                                       accumulate=accumulate, x_next=x_next, amax_next=amax_next)

    def routed_layer(self, x, proj, ids, weights, out, in_gscale=None, in_amax=None, accumulate: bool = False,
                     x_next=None, amax_next=None):
        """Router and the whole layer on this rank in one call (nvfp4b_ep_p2p_layer)."""
        if x.shape[0] > self.T_cap:
            raise ValueError(f"{x.shape[0]} tokens exceed the capacity {self.T_cap}")
        self.T = x.shape[0]
        return self.pkg.ep_p2p_layer(x, proj, self.topk, self.E, self.experts, self.src_ws, self.exp_ws,
                                     self.ex.peers, self.overflow, ids, weights, out, accumulate=accumulate,
                                     in_gscale=in_gscale, in_amax=in_amax, x_next=x_next, amax_next=amax_next)


class LocalOps:
    """One GPU holding every expert: the layer is the single-GPU MoE (nvfp4b_moe_forward: dispatch with the
    quantiser fused in, grouped GEMMs, slot-ordered combine) -- no records and no exchange.  Same result, bit for
    bit, as the expert-parallel paths at G = 1."""

    local = True

    def __init__(self, pkg, experts, E: int, topk: int, T_cap: int, device="cuda"):
        if experts.E != E:
            raise ValueError(f"local arena holds {experts.E} experts, expected {E}")
        self.pkg, self.experts, self.E, self.topk, self.T_cap, self.G = pkg, experts, E, topk, T_cap, 1
        self.H = experts.H
        self.src_ws = pkg.moe_workspace(T_cap, experts.H, experts.I, E, topk, device=device)
        self.overflow = torch.zeros(1, dtype=torch.int32, device=device)

    def layer(self, x, ids, weights, out, in_gscale=None, in_amax=None, accumulate: bool = False, x_next=None,
              amax_next=None):
        if x.shape[0] > self.T_cap:
            raise ValueError(f"{x.shape[0]} tokens exceed the capacity {self.T_cap}")
        return self.pkg.moe_forward(x, ids, weights, self.experts, self.src_ws, in_gscale=in_gscale, in_amax=in_amax,
                                    out=out, accumulate=accumulate, x_next=x_next, amax_next=amax_next)

    def routed_layer(self, x, proj, ids, weights, out, in_gscale=None, in_amax=None, accumulate: bool = False,
                     x_next=None, amax_next=None):
        """Router and layer in one call (nvfp4b_moe_layer: the top-k fused with the dispatch ranking)."""
        if x.shape[0] > self.T_cap:
            raise ValueError(f"{x.shape[0]} tokens exceed the capacity {self.T_cap}")
        return self.pkg.moe_layer(x, proj, self.topk, self.experts, self.src_ws, ids=ids, weights=weights,
                                  in_gscale=in_gscale, in_amax=in_amax, out=out, accumulate=accumulate,
                                  x_next=x_next, amax_next=amax_next)


class ExpertParallelMoE:
    """Runs layers through `ops` over `group` (None = the default group; world size 1 runs with no collective)."""

    def __init__(self, ops, group=None):
        self.ops, self.group = ops, group
        self.G = ops.G
        if self.G > 1 and dist.get_world_size(group) != self.G:
            raise ValueError("ops were built for a different group size")

    def forward(self, x, ids, weights, out, in_gscale=None, in_amax=None, accumulate: bool = False, mark=None,
                x_next=None, amax_next=None):
        """out[t] (+)= the layer's output for token t.  With x_next (bf16, may be x itself) and amax_next (fp32 [1],
        may be in_amax) also x_next = bf16(out) and amax_next = max |x_next|: the next layer's input on a residual
        stream, fused into the combine where the path has it.  `mark(name)`, if given, is called around the
        expert-side kernels ("kernel" / "kernel_end") so a caller can time them with events on the current stream."""
        ops, G, grp = self.ops, self.G, self.group
        if getattr(ops, "local", False):
            if mark is not None:
                mark("kernel")
            ops.layer(x, ids, weights, out, in_gscale=in_gscale, in_amax=in_amax, accumulate=accumulate,
                      x_next=x_next, amax_next=amax_next)
            if mark is not None:
                mark("kernel_end")
            return out
        if getattr(ops, "p2p", False):
            ops.dispatch(x, ids, weights, in_gscale=in_gscale, in_amax=in_amax)
            if mark is not None:
                mark("kernel")
            ops.expert()
            if mark is not None:
                mark("kernel_end")
            return ops.combine(out, accumulate, x_next=x_next, amax_next=amax_next)
        send_counts, recv_counts = ops.dispatch(x, ids, weights, in_gscale=in_gscale, in_amax=in_amax)
        if G > 1:
            dist.all_to_all_single(recv_counts, send_counts, group=grp)
            dist.all_to_all_single(ops.recv, ops.send, group=grp)
            recv = ops.recv
        else:
            recv_counts.copy_(send_counts)
            recv = ops.send
        if mark is not None:
            mark("kernel")
        rows = ops.expert(recv, recv_counts)
        if mark is not None:
            mark("kernel_end")
        if G > 1:
            dist.all_to_all_single(ops.back, rows, group=grp)
            back = ops.back
        else:
            back = rows
        ops.combine(back, out, accumulate)
        if x_next is not None:
            x_next.copy_(out)
            ops.pkg.amax(x_next, out=amax_next)
        return out

    def forward_routed(self, x, proj, ids, weights, out, in_gscale=None, in_amax=None, accumulate: bool = False,
                       mark=None, x_next=None, amax_next=None):
        """Router (x @ proj^T, softmax top-k into ids / weights) and the layer.  One GPU holding every expert runs the
        fused nvfp4b_moe_layer, the peer-memory path the fused nvfp4b_ep_p2p_layer; the NCCL path routes and then
        exchanges.  `mark` brackets the timed part (the whole layer with its router for the fused forms)."""
        ops = self.ops
        if getattr(ops, "local", False) or getattr(ops, "p2p", False):
            if mark is not None:
                mark("kernel")
            ops.routed_layer(x, proj, ids, weights, out, in_gscale=in_gscale, in_amax=in_amax,
                             accumulate=accumulate, x_next=x_next, amax_next=amax_next)
            if mark is not None:
                mark("kernel_end")
            return out
        ops.pkg.moe_route(x, proj, ops.topk, ops.src_ws, ids=ids, weights=weights)
        return self.forward(x, ids, weights, out, in_gscale=in_gscale, in_amax=in_amax, accumulate=accumulate,
                            mark=mark, x_next=x_next, amax_next=amax_next)

    def overflowed(self, reset: bool = True) -> bool:
        """True if a layer since the last reset had more than `capacity` records for one rank pair (host read)."""
        v = bool(self.ops.overflow.item())
        if reset:
            self.ops.overflow.zero_()
        return v
