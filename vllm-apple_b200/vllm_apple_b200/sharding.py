"""Sequence sharding of a decode batch across GPUs (one process per GPU).

Decode attention shards with no exchange at all: each rank owns whole
sequences together with their KV pages, so the attention step runs with no
collective.  The only optional exchange is gathering the per-rank outputs
back into batch order after the step (``gather_outputs``: one all-gather over
NCCL / NVLink, timed separately from the attention step).

Partition: greedy longest-processing-time bin packing on context length,
which balances KV bytes (the HBM traffic) rather than sequence counts.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


def lpt_partition(lengths, world: int) -> list[list[int]]:
    """Indices of the sequences owned by each of ``world`` ranks (deterministic)."""
    if world <= 0:
        raise ValueError("world must be positive")
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    loads = [0] * world
    bins: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda j: (loads[j], j))
        bins[r].append(i)
        loads[r] += int(lengths[i])
    return [sorted(b) for b in bins]


@dataclass
class ShardPlan:
    lengths: list[int]
    world: int

    def __post_init__(self):
        self.shards = lpt_partition(self.lengths, self.world)
        self.loads = [sum(int(self.lengths[i]) for i in s) for s in self.shards]

    @property
    def imbalance(self) -> float:
        """max load / mean load (1.0 = perfectly balanced)."""
        mean = sum(self.loads) / max(self.world, 1)
        return max(self.loads) / mean if mean else 1.0

    def owner(self) -> list[int]:
        own = [0] * len(self.lengths)
        for r, s in enumerate(self.shards):
            for i in s:
                own[i] = r
        return own


def gather_outputs(local_out: torch.Tensor, plan: ShardPlan, rank: int, group=None) -> torch.Tensor:
    """All-gather each rank's [len(shard), ...] outputs and return the full
    batch [B, ...] in the original sequence order (on every rank)."""
    import torch.distributed as dist
    width = max(len(s) for s in plan.shards)
    pad = torch.zeros((width,) + tuple(local_out.shape[1:]), dtype=local_out.dtype,
                      device=local_out.device)
    pad[:local_out.shape[0]] = local_out
    bufs = [torch.empty_like(pad) for _ in range(plan.world)]
    dist.all_gather(bufs, pad, group=group)
    full = torch.empty((len(plan.lengths),) + tuple(local_out.shape[1:]), dtype=local_out.dtype,
                       device=local_out.device)
    for r, s in enumerate(plan.shards):
        if s:
            full[torch.as_tensor(s, device=full.device)] = bufs[r][:len(s)]
    return full
