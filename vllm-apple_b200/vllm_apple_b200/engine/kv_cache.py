"""Engine-owned paged KV cache and its host-side validation rules.

Mirrors EngineKVCache (vllm_apple/engine/kv_cache.py:82-701): one K and one V
buffer per layer in the engine layout [num_blocks, num_kv_heads, block_size,
head_size] fp16, plus the step-boundary validation of block tables and slot
mappings (-1 = unused/padding is allowed, anything below raises, anything at
or beyond the capacity raises).  Validation runs on host copies of the
metadata before the step is encoded, exactly where the reference runs it.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch


@dataclass
class KVCacheDescriptor:
    num_blocks: int
    block_size: int
    num_kv_heads: int
    head_size: int
    num_layers: int = 1

    def __post_init__(self):
        for name in ("num_blocks", "block_size", "num_kv_heads", "head_size", "num_layers"):
            if getattr(self, name) <= 0:
                raise ValueError(f"{name} must be positive")


def _host(a):
    if isinstance(a, torch.Tensor):
        if a.is_cuda:
            raise RuntimeError("validation takes host (CPU) metadata; copy it before the "
                               "engine boundary")
        return a.numpy()
    return np.asarray(a)


class EngineKVCache:
    def __init__(self, engine_context, descriptor: KVCacheDescriptor, zero: bool = True):
        self._context = engine_context
        self._desc = descriptor
        d = descriptor
        shape = (d.num_blocks, d.num_kv_heads, d.block_size, d.head_size)
        alloc = torch.zeros if zero else torch.empty
        dev = engine_context.device
        self._k = [alloc(shape, dtype=torch.float16, device=dev) for _ in range(d.num_layers)]
        self._v = [alloc(shape, dtype=torch.float16, device=dev) for _ in range(d.num_layers)]

    num_layers = property(lambda self: self._desc.num_layers)
    num_blocks = property(lambda self: self._desc.num_blocks)
    block_size = property(lambda self: self._desc.block_size)
    num_kv_heads = property(lambda self: self._desc.num_kv_heads)
    head_size = property(lambda self: self._desc.head_size)

    @property
    def strides(self) -> dict:
        d = self._desc
        return {"block": d.num_kv_heads * d.block_size * d.head_size,
                "head": d.block_size * d.head_size, "token": d.head_size}

    def get_buffers(self, layer_idx: int):
        return self._k[layer_idx], self._v[layer_idx]

    def get_key_buffer(self, layer_idx: int):
        return self._k[layer_idx]

    def get_value_buffer(self, layer_idx: int):
        return self._v[layer_idx]

    def validate_block_table(self, block_table, context: str = "") -> None:
        bt = _host(block_table)
        sfx = f" ({context})" if context else ""
        if bt.size == 0:
            return
        mx = bt.max()
        if mx >= self._desc.num_blocks:
            raise ValueError(f"Block table contains index {mx} >= num_blocks "
                             f"{self._desc.num_blocks}{sfx}")
        bad = bt < -1
        if bad.any():
            raise ValueError(f"Block table contains invalid index {bt[bad].min()}{sfx}")

    def validate_slot_mapping(self, slot_mapping, context: str = "") -> None:
        sm = _host(slot_mapping)
        sfx = f" ({context})" if context else ""
        max_valid = self._desc.num_blocks * self._desc.block_size - 1
        ok = sm >= 0
        if ok.any() and sm[ok].max() > max_valid:
            raise ValueError(f"Slot mapping contains index {sm[ok].max()} > max valid slot "
                             f"{max_valid} (num_blocks={self._desc.num_blocks}, "
                             f"block_size={self._desc.block_size}){sfx}")
        bad = sm < -1
        if bad.any():
            raise ValueError(f"Slot mapping contains invalid index {sm[bad].min()}{sfx}")

    def sync_from_torch_cache(self, torch_caches, block_table, seq_lens) -> None:
        """Copy the active blocks of vLLM-layout caches ``[2, nb, bs, H, D]`` (one per
        layer) into the engine caches, on the device (reference kv_cache.py:518-684;
        there the copy is a host loop over blocks)."""
        from .. import ops
        if len(torch_caches) != self._desc.num_layers:
            raise ValueError(f"torch_caches has {len(torch_caches)} layers, "
                             f"expected {self._desc.num_layers}")
        dev = self._k[0].device
        bt = block_table.to(device=dev, dtype=torch.int32).contiguous()
        sl = seq_lens.to(device=dev, dtype=torch.int32).contiguous()
        for layer, kv in enumerate(torch_caches):
            ops.kv_sync_blocks(kv[0], kv[1], self._k[layer], self._v[layer], bt, sl,
                               src_layout="nhd", dst_layout="hnd")

    def get_slot_offset(self, slot_idx: int):
        return divmod(int(slot_idx), self._desc.block_size)

    def reset(self) -> None:
        for t in self._k + self._v:
            t.zero_()

    def get_total_memory_bytes(self) -> int:
        return sum(t.numel() * 2 for t in self._k + self._v)
