"""Sequence partition of batched decode across GPUs (one process per GPU).

Independent sequences share nothing, so the batch is split by sequence with
the greedy longest-processing-time rule of tle_partition_lpt (balances the
attended rows, i.e. the KV bytes each GPU streams).  Each rank keeps the full
KV cache of its own sequences in its HBM and decodes them locally; the only
exchange is the all-gather of the per-sequence outputs (8 KB each), after
which every rank holds out[n_seqs][2048] in the original sequence order.

The reference is single-process (no collective exists there); this module is
the plumbing for the multi-GPU rows of the hot path.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Sequence


@dataclass
class ShardPlan:
    world: int
    owner: List[int]          # rank of every sequence
    local: List[List[int]]    # sequences of every rank, in sequence order
    max_local: int            # rows per rank in the gather buffer
    gather_row: List[int]     # row of sequence s in the gathered buffer

    def mine(self, rank: int) -> List[int]:
        return self.local[rank]


def plan(lengths: Sequence[int], world: int) -> ShardPlan:
    import tle
    owner = tle.partition_lpt(lengths, world)
    local = [[s for s in range(len(lengths)) if owner[s] == r] for r in range(world)]
    max_local = max(1, max(len(x) for x in local))
    gather_row = [0] * len(lengths)
    for r in range(world):
        for i, s in enumerate(local[r]):
            gather_row[s] = r * max_local + i
    return ShardPlan(world, owner, local, max_local, gather_row)


class OutputGather:
    """All-gathers every rank's [max_local][width] output block and reorders
    the rows into sequence order (one collective + one device gather)."""

    def __init__(self, p: ShardPlan, width: int, device, group=None):
        import torch
        self.p = p
        self.group = group
        self.buf = torch.zeros((p.world * p.max_local, width), device=device)
        self.index = torch.tensor(p.gather_row, dtype=torch.long, device=device)

    def __call__(self, local_out):
        import torch.distributed as dist
        if self.p.world == 1:
            return local_out  # one rank holds every sequence, already in order
        dist.all_gather_into_tensor(self.buf, local_out, group=self.group)
        return self.buf.index_select(0, self.index)
