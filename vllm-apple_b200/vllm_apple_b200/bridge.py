"""Host-tensor bridge of the v1 plugin path, on the B200 kernels.

Mirrors the reference's bridge classes so that code written against them keeps
working: ``MetalPagedAttentionFused`` (vllm_apple/metal/bridge/
metal_paged_attention_fused.py:82-537), ``MetalPagedAttentionV2``
(metal_paged_attention_v2.py:25-551) and ``metal_write_kv_batch``
(metal_paged_attention_v2.py:610-680).  Same constructors, method names,
argument order and return values.  Where the reference takes an MTLBuffer for the
KV cache, this takes the device-resident cache tensor ``[num_blocks, num_kv_heads,
block_size, head_size]`` fp16 (the engine layout the reference's buffers hold);
query / new K,V / block table / sequence lengths / output may live on the host
(as in the reference, which stages them into fresh buffers every call) or on the
GPU.  Host inputs are copied to the device, the kernels run on the current stream,
the result is copied back into ``output`` and the call returns after the copy, as
the reference's ``waitUntilCompleted`` does.
"""
from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from . import _lib
from . import ops


def _dev(t: torch.Tensor, device: torch.device, dtype=None) -> torch.Tensor:
    t = t if dtype is None else t.to(dtype)
    return t.to(device, non_blocking=False).contiguous()


def _cache_device(key_buffer: torch.Tensor) -> torch.device:
    if not isinstance(key_buffer, torch.Tensor) or not key_buffer.is_cuda:
        raise TypeError("key/value caches must be CUDA tensors [num_blocks, num_kv_heads, "
                        "block_size, head_size] (they stand in for the reference's MTLBuffers)")
    return key_buffer.device


class MetalPagedAttentionFused:
    """Fused KV write + decode attention for a batch of one-token sequences
    (reference: metal_paged_attention_fused.py:82-537)."""

    def __init__(self, num_kv_heads: int, num_query_heads: int, head_size: int,
                 block_size: int, scale: Optional[float] = None, max_num_blocks: int = 4096,
                 max_batch_size: int = 64):
        if num_query_heads % num_kv_heads:
            raise ValueError("num_query_heads must be a multiple of num_kv_heads")
        self.num_kv_heads = num_kv_heads
        self.num_query_heads = num_query_heads
        self.head_size = head_size
        self.block_size = block_size
        self.scale = scale if scale is not None else 1.0 / (head_size ** 0.5)
        self.max_num_blocks = max_num_blocks
        self.max_batch_size = max_batch_size
        self.queries_per_kv = num_query_heads // num_kv_heads
        # one fused kernel for every supported head size (the reference picks between an
        # h128 and a generic shader)
        self.kernel_name = "paged_decode_kernel"
        self.using_fused = True
        _lib.load()

    @property
    def is_fused_available(self) -> bool:
        return True

    def _run(self, query, new_keys, new_values, key_buffer, value_buffer, block_table,
             seq_lens, output):
        dev = _cache_device(key_buffer)
        q = _dev(query, dev, torch.float16)
        bt = _dev(block_table, dev, torch.int32)
        sl = _dev(seq_lens, dev, torch.int32)
        nk = None if new_keys is None else _dev(new_keys, dev, torch.float16)
        nv = None if new_values is None else _dev(new_values, dev, torch.float16)
        out = output if (output.is_cuda and output.is_contiguous()) else torch.empty_like(q)
        max_len = int(seq_lens.max().item()) if seq_lens.numel() else 0
        with torch.cuda.device(dev):
            ops.paged_decode(out, q, key_buffer, value_buffer, bt, sl, scale=self.scale,
                             max_seq_len=max_len, new_k=nk, new_v=nv, layout="hnd")
            ops.check_device_errors(dev.index)
        if out is not output:
            output.copy_(out.to(output.device))
        return output

    def forward_fused(self, query: torch.Tensor, new_keys: torch.Tensor,
                      new_values: torch.Tensor, key_buffer, value_buffer,
                      block_table: torch.Tensor, seq_lens: torch.Tensor,
                      output: torch.Tensor) -> torch.Tensor:
        """Write new_keys / new_values at position seq_lens-1 of every sequence and
        attend over the paged cache, in one kernel."""
        return self._run(query, new_keys, new_values, key_buffer, value_buffer, block_table,
                         seq_lens, output)

    def forward_with_metal_buffers(self, query: torch.Tensor, key_buffer, value_buffer,
                                   block_table: torch.Tensor, seq_lens: torch.Tensor,
                                   output: torch.Tensor) -> torch.Tensor:
        """Attention over an already-populated cache (no write)."""
        return self._run(query, None, None, key_buffer, value_buffer, block_table, seq_lens,
                         output)


class MetalPagedAttentionV2:
    """Non-fused decode attention with a cache the object can own
    (reference: metal_paged_attention_v2.py:25-551)."""

    SUPPORTED_HEAD_SIZES = {32, 64, 96, 128}

    def __init__(self, num_kv_heads: int, num_query_heads: int, head_size: int,
                 block_size: int, scale: float, max_num_blocks: int = 256,
                 max_batch_size: int = 64):
        if head_size not in self.SUPPORTED_HEAD_SIZES:
            raise ValueError(f"head_size={head_size} not supported. "
                             f"Supported: {sorted(self.SUPPORTED_HEAD_SIZES)}")
        self.num_kv_heads = num_kv_heads
        self.num_query_heads = num_query_heads
        self.head_size = head_size
        self.block_size = block_size
        self.scale = scale
        self.queries_per_kv = num_query_heads // num_kv_heads
        self.max_num_blocks = max_num_blocks
        self.max_batch_size = max_batch_size
        self.key_buf: Optional[torch.Tensor] = None
        self.value_buf: Optional[torch.Tensor] = None
        self._kv_cache_set = False
        self._kv_cache_version = 0
        self._fused = MetalPagedAttentionFused(num_kv_heads, num_query_heads, head_size,
                                               block_size, scale)

    def _ensure_buffers(self, shape, device):
        if self.key_buf is None or tuple(self.key_buf.shape) != tuple(shape) \
                or self.key_buf.device != device:
            self.key_buf = torch.empty(shape, dtype=torch.float16, device=device)
            self.value_buf = torch.empty_like(self.key_buf)

    @staticmethod
    def _device() -> torch.device:
        if not torch.cuda.is_available():
            raise RuntimeError("MetalPagedAttentionV2 needs a CUDA device")
        return torch.device("cuda", torch.cuda.current_device())

    def set_kv_cache(self, key_cache: torch.Tensor, value_cache: torch.Tensor):
        """Copy the whole cache ([num_blocks, num_kv_heads, block_size, head_size]) into
        the object's device buffers."""
        dev = key_cache.device if key_cache.is_cuda else self._device()
        self._ensure_buffers(key_cache.shape, dev)
        self.key_buf.copy_(key_cache.to(torch.float16))
        self.value_buf.copy_(value_cache.to(torch.float16))
        self._kv_cache_set = True
        self._kv_cache_version += 1

    def update_kv_cache_block(self, block_idx: int, key_block: torch.Tensor,
                              value_block: torch.Tensor):
        """Overwrite one block ([num_kv_heads, block_size, head_size])."""
        if self.key_buf is None:
            raise RuntimeError("set_kv_cache() must be called before update_kv_cache_block()")
        self.key_buf[block_idx].copy_(key_block.to(torch.float16))
        self.value_buf[block_idx].copy_(value_block.to(torch.float16))

    def forward(self, query: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                block_table: torch.Tensor, seq_lens: torch.Tensor,
                output: Optional[torch.Tensor] = None, skip_kv_copy: bool = False
                ) -> torch.Tensor:
        """Decode attention; the cache is taken from key_cache / value_cache unless
        skip_kv_copy (then the buffers set by set_kv_cache are used)."""
        if output is None:
            output = torch.empty_like(query)
        if skip_kv_copy:
            if not self._kv_cache_set:
                raise RuntimeError("skip_kv_copy=True but set_kv_cache() was never called")
            kc, vc = self.key_buf, self.value_buf
        elif key_cache.is_cuda and key_cache.dtype == torch.float16 \
                and key_cache.is_contiguous() and value_cache.is_contiguous():
            kc, vc = key_cache, value_cache
        else:
            self.set_kv_cache(key_cache, value_cache)
            kc, vc = self.key_buf, self.value_buf
        return self._fused.forward_with_metal_buffers(query, kc, vc, block_table, seq_lens,
                                                      output)

    def forward_with_metal_buffers(self, query: torch.Tensor, key_buffer, value_buffer,
                                   block_table: torch.Tensor, seq_lens: torch.Tensor,
                                   output: torch.Tensor) -> torch.Tensor:
        return self._fused.forward_with_metal_buffers(query, key_buffer, value_buffer,
                                                      block_table, seq_lens, output)


def metal_write_kv_batch(key_mv, value_mv, key_np, value_np, block_ids, token_offsets,
                         num_tokens: int, num_kv_heads: int, head_size: int,
                         stride_block: int, stride_head: int, stride_token: int) -> None:
    """Scatter num_tokens new K/V rows into the cache at (block_ids[i], token_offsets[i])
    (reference: metal_paged_attention_v2.py:610-680, kv_write.c:33-107).

    key_mv / value_mv are the CUDA cache tensors (the reference's MTLBuffer contents);
    key_np / value_np ([num_tokens, num_kv_heads, head_size] fp16) and the int64 index
    arrays may be numpy arrays or tensors, on the host or the device."""
    dev = _cache_device(key_mv)

    def t(x, dtype):
        if isinstance(x, np.ndarray):
            x = torch.from_numpy(np.ascontiguousarray(x))
        return _dev(x, dev, dtype)

    k, v = t(key_np, torch.float16), t(value_np, torch.float16)
    bid, off = t(block_ids, torch.int64), t(token_offsets, torch.int64)
    with torch.cuda.device(dev):
        ops.write_kv_batch(key_mv, value_mv, k, v, bid, off, int(num_tokens), int(num_kv_heads),
                           int(head_size), int(stride_block), int(stride_head),
                           int(stride_token))
        torch.cuda.current_stream(dev).synchronize()
