"""Expert-parallel MoE layer: E experts sharded over the ranks of a torch.distributed group (E/G consecutive experts
per rank), routed assignments exchanged with all-to-all collectives (NCCL over NVLink on B200s, one process per GPU).

The reference runs the MoE of a layer on one GPU (src/forward.cu:516-553: router, per-expert W4A16 GEMVs, weighted
sum).  This is the expert-parallel form of the same computation.  One layer, per rank:

  1. route (caller): ids [T, k], weights [T, k]
  2. ops.dispatch: one record per assignment (NVFP4 codes + scales of the token, local expert, router weight,
     activation global scale), sorted by destination rank; per-rank counts
  3. all-to-all of the counts, then ONE device->host read of the count vectors (they are the split sizes)
  4. all-to-all of the records (uneven splits)
  5. ops.expert: the local experts on the received records -> weighted fp16 rows [n_recv, H]
  6. all-to-all of the rows back to their sources (the reverse splits)
  7. ops.combine: slot-ordered fp32 sum into out (bit-identical to the single-GPU layer at G = 1)

`ops` does the device work; KernelOps is the sm_100a implementation (the C ABI of libnvfp4_b200.so).  Steps 3, 4
and 6 are the only collectives, issued on the caller's current stream, in the same order on every rank.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class KernelOps:
    """Device side of one expert-parallel layer on this rank: buffers sized for up to T_cap tokens per rank."""

    def __init__(self, pkg, experts, E: int, topk: int, T_cap: int, G: int, device="cuda"):
        if E % G:
            raise ValueError(f"{E} experts do not split over {G} ranks")
        if experts.E != E // G:
            raise ValueError(f"local arena holds {experts.E} experts, expected {E // G}")
        self.pkg, self.experts, self.E, self.topk, self.T_cap, self.G = pkg, experts, E, topk, T_cap, G
        H, I = experts.H, experts.I
        self.H = H
        self.record_bytes = pkg.ep_record_bytes(H)
        self.n_cap = G * T_cap * topk                       # worst case: every rank routes everything here
        self.src_ws = pkg.moe_workspace(T_cap, H, 32, E, topk, device=device)
        self.exp_ws = pkg.moe_workspace(self.n_cap, H, I, E // G, 1, device=device)
        self.send = torch.empty((T_cap * topk, self.record_bytes), dtype=torch.uint8, device=device)
        self.recv = torch.empty((self.n_cap, self.record_bytes), dtype=torch.uint8, device=device)
        self.back = torch.empty((T_cap * topk, H), dtype=torch.float16, device=device)
        self.counts = torch.empty(2 * G, dtype=torch.int32, device=device)

    def dispatch(self, x, ids, weights, in_gscale=None, in_amax=None):
        T = x.shape[0]
        if T > self.T_cap:
            raise ValueError(f"{T} tokens exceed the capacity {self.T_cap}")
        self.T = T
        self.pkg.ep_dispatch(x, ids, weights, self.E, self.G, self.src_ws, self.send, self.counts[:self.G],
                             in_gscale=in_gscale, in_amax=in_amax)
        return self.counts[:self.G], self.counts[self.G:]

    def expert(self, records, n: int):
        return self.pkg.ep_expert_forward(records, n, self.n_cap, self.experts, self.exp_ws)

    def combine(self, back, out, accumulate: bool):
        return self.pkg.ep_combine(back, self.T, self.topk, self.E, self.src_ws, out, accumulate=accumulate)


class ExpertParallelMoE:
    """Runs layers through `ops` over `group` (None = the default group; world size 1 runs with no collective)."""

    def __init__(self, ops, group=None):
        self.ops, self.group = ops, group
        self.G = ops.G
        if self.G > 1 and dist.get_world_size(group) != self.G:
            raise ValueError("ops were built for a different group size")

    def forward(self, x, ids, weights, out, in_gscale=None, in_amax=None, accumulate: bool = False):
        ops, G, grp = self.ops, self.G, self.group
        send_counts, recv_counts = ops.dispatch(x, ids, weights, in_gscale=in_gscale, in_amax=in_amax)
        if G > 1:
            dist.all_to_all_single(recv_counts, send_counts, group=grp)
        else:
            recv_counts.copy_(send_counts)
        counts = ops.counts.tolist()                         # the split sizes: one device->host read per layer
        sc, rc = counts[:G], counts[G:]
        n_send, n_recv = sum(sc), sum(rc)
        if G > 1:
            recv = ops.recv[:n_recv]
            dist.all_to_all_single(recv, ops.send[:n_send], output_split_sizes=rc, input_split_sizes=sc, group=grp)
        else:
            recv = ops.send[:n_send]
        rows = ops.expert(recv, n_recv)
        if G > 1:
            back = ops.back[:n_send]
            dist.all_to_all_single(back, rows, output_split_sizes=sc, input_split_sizes=rc, group=grp)
        else:
            back = rows
        return ops.combine(back, out, accumulate)
