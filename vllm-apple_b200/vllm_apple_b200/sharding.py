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


class OutputGather:
    """All-gather of the per-rank decode outputs back into batch order.

    Each rank contributes its ``[len(shard), ...]`` rows padded to the widest
    shard; one ``all_gather_into_tensor`` (NCCL over NVLink) fills a
    ``[world * width, ...]`` buffer, and one device gather with a permutation
    built once puts the rows in the original sequence order.  Buffers are
    allocated once, so repeated calls launch exactly one collective and two
    small copy kernels."""

    def __init__(self, plan: ShardPlan, row_shape, dtype, device, group=None):
        self.plan, self.group = plan, group
        self.width = max(len(s) for s in plan.shards)
        self.pad = torch.zeros((self.width,) + tuple(row_shape), dtype=dtype, device=device)
        self.buf = torch.empty((plan.world * self.width,) + tuple(row_shape), dtype=dtype,
                               device=device)
        src = torch.empty(len(plan.lengths), dtype=torch.int64)
        for r, s in enumerate(plan.shards):
            for j, i in enumerate(s):
                src[i] = r * self.width + j
        self.src = src.to(device)
        self.full = torch.empty((len(plan.lengths),) + tuple(row_shape), dtype=dtype,
                                device=device)

    @property
    def bytes_per_rank(self) -> int:
        return self.pad.numel() * self.pad.element_size()

    def __call__(self, local_out: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist
        self.pad[:local_out.shape[0]].copy_(local_out)
        dist.all_gather_into_tensor(self.buf, self.pad, group=self.group)
        torch.index_select(self.buf, 0, self.src, out=self.full)
        return self.full


def gather_outputs(local_out: torch.Tensor, plan: ShardPlan, rank: int, group=None) -> torch.Tensor:
    """All-gather each rank's [len(shard), ...] outputs and return the full
    batch [B, ...] in the original sequence order (on every rank)."""
    g = OutputGather(plan, local_out.shape[1:], local_out.dtype, local_out.device, group)
    return g(local_out).clone()
