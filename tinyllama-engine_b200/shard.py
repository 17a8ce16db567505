"""Sequence partition of batched decode across GPUs (one process per GPU).

Independent sequences share nothing, so the batch is split by sequence with
the greedy longest-processing-time rule of tle_partition_lpt (balances the
attended rows, i.e. the KV bytes each GPU streams).  Each rank keeps the full
KV cache of its own sequences in its HBM and decodes them locally; the only
exchange is the all-gather of the per-sequence outputs (8 KB each), after
which every rank holds out[n_seqs][2048] in the original sequence order.

The reference is single-process (no collective exists there); this module is
the plumbing for the multi-GPU rows of the hot path.

Context split (one long sequence over the GPUs): rank r holds rows
[r L / W, (r+1) L / W) of the sequence's KV cache; every rank decodes its
shard with tle_attention_lse (output normalised over its rows plus each
head's score log-sum-exp), the (out, lse) pairs are all-gathered (8.3 KB per
rank) and tle_merge_lse combines them into the attention over all rows.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Sequence, Tuple


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
    """LPT partition of the sequences; a batch of equal lengths that divides
    evenly is cut into contiguous equal blocks instead (the same balance, and
    the gathered buffer is then already in sequence order)."""
    import tle
    lengths = [int(x) for x in lengths]
    n = len(lengths)
    if n and n % world == 0 and len(set(lengths)) == 1:
        owner = [s // (n // world) for s in range(n)]
    else:
        owner = tle.partition_lpt(lengths, world)
    local = [[s for s in range(len(lengths)) if owner[s] == r] for r in range(world)]
    max_local = max(1, max(len(x) for x in local))
    gather_row = [0] * len(lengths)
    for r in range(world):
        for i, s in enumerate(local[r]):
            gather_row[s] = r * max_local + i
    return ShardPlan(world, owner, local, max_local, gather_row)


class OutputGather:
    """All-gathers every rank's [max_local][width] output block (one NCCL
    collective) and returns the rows in sequence order: a view of the gather
    buffer when the plan's blocks are contiguous and full (no copy), else a
    device gather of the rows.  A rank that decodes straight into
    ``local_slot(rank)`` makes the collective in place (nothing to copy in)."""

    def __init__(self, p: ShardPlan, width: int, device, group=None):
        import torch
        self.p = p
        self.group = group
        self.n = len(p.gather_row)
        self.buf = torch.zeros((p.world * p.max_local, width), device=device)
        self.in_order = p.gather_row == list(range(self.n))
        self.index = torch.tensor(p.gather_row, dtype=torch.long, device=device)

    def local_slot(self, rank: int):
        """This rank's block of the gather buffer: decode into it to gather in place."""
        return self.buf[rank * self.p.max_local:(rank + 1) * self.p.max_local]

    def __call__(self, local_out):
        import torch.distributed as dist
        if self.p.world == 1:
            return local_out  # one rank holds every sequence, already in order
        dist.all_gather_into_tensor(self.buf, local_out, group=self.group)
        if self.in_order:
            return self.buf[:self.n]
        return self.buf.index_select(0, self.index)


@dataclass
class ContextPlan:
    world: int
    bounds: List[Tuple[int, int]]   # global rows [r0, r1) held by each rank

    def local_rows(self, rank: int) -> int:
        r0, r1 = self.bounds[rank]
        return r1 - r0


def context_plan(n_rows: int, world: int) -> ContextPlan:
    """Contiguous, balanced row ranges; the last rank holds the newest row."""
    if n_rows < world:
        raise ValueError(f"{n_rows} rows cannot be split over {world} ranks")
    cuts = [r * n_rows // world for r in range(world + 1)]
    return ContextPlan(world, [(cuts[r], cuts[r + 1]) for r in range(world)])


class ContextSplitDecode:
    """Decode of one sequence whose KV rows are split over the ranks.

    ``key_cache``/``value_cache`` are this rank's shard, [n_layers][n_ctx][256]
    with local row i = global row bounds[rank][0] + i.  ``step`` takes q and k
    already rotated for the global position (tle.rope) and returns the full
    attention output on every rank.
    """

    def __init__(self, plan: ContextPlan, rank: int, key_cache, value_cache, n_ctx: int, shape,
                 device, group=None):
        import torch
        import tle
        self.p, self.rank, self.group = plan, rank, group
        self.kc, self.vc, self.n_ctx, self.shape = key_cache, value_cache, n_ctx, shape
        self.ws = tle.attention_workspace(shape, n_ctx)
        self.local = torch.empty(2048 + 32, device=device)          # out | lse
        self.gathered = torch.empty((plan.world, 2048 + 32), device=device)
        self.out = torch.empty(2048, device=device)

    def step(self, q_rot, k_rot, v, layer: int, pos: int, stream=None):
        import torch.distributed as dist
        import tle
        r0, r1 = self.p.bounds[self.rank]
        out_l, lse_l = self.local[:2048], self.local[2048:]
        if self.rank == self.p.world - 1:            # holds row pos: append there
            tle.attention_lse(out_l, lse_l, q_rot, k_rot, v, self.kc, self.vc, layer, pos - r0,
                              self.n_ctx, self.shape, self.ws, stream)
        else:                                        # all rows cached: last row stands in
            row = r1 - r0 - 1
            tle.attention_lse(out_l, lse_l, q_rot, self.kc[layer, row], self.vc[layer, row],
                              self.kc, self.vc, layer, row, self.n_ctx, self.shape, self.ws, stream)
        if self.p.world > 1:
            dist.all_gather_into_tensor(self.gathered, self.local, group=self.group)
        else:
            self.gathered[0].copy_(self.local)
        parts = self.gathered[:, :2048].contiguous()
        lses = self.gathered[:, 2048:].contiguous()
        tle.merge_lse(self.out, parts, lses, stream)
        return self.out
