"""Encode-only engine ops with the reference's signatures, backed by the C ABI.

Each class keeps the constructor and ``encode*`` signatures of its reference
counterpart; buffers are CUDA tensors or :class:`EngineTensor` views instead
of MTLBuffers, byte offsets keep their meaning, and encoding enqueues the
sm_100a kernels on the step's stream (no waits).

  PagedAttentionOp      vllm_apple/engine/ops/attention.py:160-599
  KVWriteOp             vllm_apple/engine/ops/kv_write.py:185-412
  EngineRMSNorm         vllm_apple/engine/ops/rmsnorm.py:176-340
  EngineRoPE            vllm_apple/engine/ops/elementwise.py:610-766
  EngineElementwiseOps  vllm_apple/engine/ops/elementwise.py (encode_silu_mul :496-532)
"""
from __future__ import annotations

import math
from typing import Any, Dict, Optional

import numpy as np
import torch

from .. import _lib
from .. import ops as _ops
from .context import EngineTensor, buffer_dtype, resolve

_H = 2  # bytes per fp16 element


def _dev(step_ctx) -> int:
    return step_ctx.context.device.index


def _err(step_ctx) -> int:
    return _ops.err_flag(_dev(step_ctx)).data_ptr()


class PagedAttentionOp:
    """Paged attention: decode with the fused KV write, and token-parallel prefill.

    KV cache buffers use the engine layout [num_blocks, num_kv_heads,
    block_size, head_size] fp16 (separate K and V buffers); Q/O are
    [tokens, num_query_heads, head_size]; new K/V [tokens, num_kv_heads, head_size].
    """

    def __init__(self, context: Any, num_kv_heads: int, num_query_heads: int, head_size: int,
                 block_size: int, scale: Optional[float] = None):
        if num_query_heads % num_kv_heads:
            raise ValueError("num_query_heads must be a multiple of num_kv_heads")
        self._context = context
        self.num_kv_heads = num_kv_heads
        self.num_query_heads = num_query_heads
        self.head_size = head_size
        self.block_size = block_size
        self.scale = scale if scale is not None else 1.0 / (head_size ** 0.5)
        self.queries_per_kv = num_query_heads // num_kv_heads
        self.kv_stride_block = num_kv_heads * block_size * head_size
        self.kv_stride_head = block_size * head_size
        self.kv_stride_token = head_size
        self.q_stride_token = num_query_heads * head_size
        self.q_stride_head = head_size
        self.o_stride_token = num_query_heads * head_size
        self.o_stride_head = head_size
        self.new_kv_stride_token = num_kv_heads * head_size
        self.new_kv_stride_head = head_size
        self._kernel_name = "va_paged_decode"
        _lib.load()

    def _num_blocks(self, key_buffer) -> int:
        _, size = resolve(key_buffer)
        return size // (self.kv_stride_block * _H)

    def encode_decode_fused(self, step_ctx, query_buffer, new_keys_buffer, new_values_buffer,
                            key_buffer, value_buffer, block_table_buffer, seq_lens_buffer,
                            output_buffer, num_seqs: int, max_seq_len: int,
                            max_blocks_per_seq: int = 0, query_offset: int = 0,
                            new_keys_offset: int = 0, new_values_offset: int = 0,
                            output_offset: int = 0) -> None:
        """Write each sequence's new K/V row at position seq_len-1 and attend over
        positions 0..seq_len-1 (one dispatch, split-KV for long contexts)."""
        step_ctx.require_encoding("encode()")
        if max_blocks_per_seq == 0:
            max_blocks_per_seq = (max_seq_len + self.block_size - 1) // self.block_size
        self._decode(step_ctx, query_buffer, query_offset, new_keys_buffer, new_keys_offset,
                     new_values_buffer, new_values_offset, key_buffer, value_buffer,
                     block_table_buffer, seq_lens_buffer, output_buffer, output_offset,
                     num_seqs, max_seq_len, max_blocks_per_seq)

    def encode_decode(self, step_ctx, query_buffer, key_buffer, value_buffer,
                      block_table_buffer, seq_lens_buffer, output_buffer, num_seqs: int,
                      max_seq_len: int, max_blocks_per_seq: int = 0, query_offset: int = 0,
                      output_offset: int = 0) -> None:
        """Decode attention over a cache that already holds the new rows."""
        step_ctx.require_encoding("encode()")
        if max_blocks_per_seq == 0:
            max_blocks_per_seq = (max_seq_len + self.block_size - 1) // self.block_size
        self._decode(step_ctx, query_buffer, query_offset, None, 0, None, 0, key_buffer,
                     value_buffer, block_table_buffer, seq_lens_buffer, output_buffer,
                     output_offset, num_seqs, max_seq_len, max_blocks_per_seq)

    def _decode(self, step_ctx, qb, qo, nkb, nko, nvb, nvo, kb, vb, btb, slb, ob, oo, num_seqs,
                max_seq_len, max_blocks):
        lib = _lib.load()
        dev = _dev(step_ctx)
        q, _ = resolve(qb, qo)
        out, _ = resolve(ob, oo)
        nk = resolve(nkb, nko)[0] if nkb is not None else None
        nv = resolve(nvb, nvo)[0] if nvb is not None else None
        kc, _ = resolve(kb)
        vc, _ = resolve(vb)
        bt, _ = resolve(btb)
        sl, _ = resolve(slb)
        nbytes = lib.va_paged_decode_workspace_size(num_seqs, self.num_query_heads,
                                                    self.num_kv_heads, self.head_size,
                                                    self.block_size, max_seq_len)
        ws = _ops.workspace(dev, "decode", nbytes, step_ctx.stream) if nbytes else None
        _lib.check(lib.va_paged_decode(
            out, q, kc, vc, bt, sl, nk, nv, num_seqs, self.num_query_heads, self.num_kv_heads,
            self.head_size, self.block_size, max_blocks, max_seq_len, self._num_blocks(kb),
            float(self.scale), self.kv_stride_block, self.kv_stride_head, self.kv_stride_token,
            self.q_stride_token, self.q_stride_head, self.o_stride_token, self.o_stride_head,
            self.new_kv_stride_token, self.new_kv_stride_head,
            None if ws is None else ws.data_ptr(), 0 if ws is None else ws.numel(),
            _err(step_ctx), step_ctx.stream_handle), "va_paged_decode")
        step_ctx.note_dispatch(2 if nbytes else 1)

    def encode_prefill(self, step_ctx, query_buffer, key_buffer, value_buffer,
                       block_table_buffer, token_to_seq_buffer, positions_buffer, output_buffer,
                       num_tokens: int, num_seqs: int, max_seq_len: int,
                       max_blocks_per_seq: int, query_offset: int = 0,
                       output_offset: int = 0) -> None:
        """Token-parallel causal attention over the cache (K/V already written)."""
        step_ctx.require_encoding("encode_prefill()")
        lib = _lib.load()
        dev = _dev(step_ctx)
        q, _ = resolve(query_buffer, query_offset)
        out, _ = resolve(output_buffer, output_offset)
        kc, _ = resolve(key_buffer)
        vc, _ = resolve(value_buffer)
        nbytes = lib.va_paged_prefill_workspace_size(num_tokens, num_seqs, self.num_query_heads,
                                                     self.num_kv_heads, self.head_size,
                                                     self.block_size, max_blocks_per_seq)
        ws = _ops.workspace(dev, "prefill", nbytes, step_ctx.stream)
        _lib.check(lib.va_paged_prefill(
            out, q, kc, vc, resolve(block_table_buffer)[0], resolve(token_to_seq_buffer)[0],
            resolve(positions_buffer)[0], num_tokens, num_seqs, self.num_query_heads,
            self.num_kv_heads, self.head_size, self.block_size, max_blocks_per_seq,
            self._num_blocks(key_buffer), float(self.scale), self.kv_stride_block,
            self.kv_stride_head, self.kv_stride_token, self.q_stride_token, self.q_stride_head,
            self.o_stride_token, self.o_stride_head, ws.data_ptr(), ws.numel(),
            _err(step_ctx), step_ctx.stream_handle), "va_paged_prefill")
        step_ctx.note_dispatch(2)

    def encode_with_kv_write(self, step_ctx, query_buffer, new_keys_buffer, new_values_buffer,
                             key_buffer, value_buffer, block_table_buffer, seq_lens_buffer,
                             output_buffer, num_seqs: int, max_seq_len: int,
                             max_blocks_per_seq: int = 0) -> None:
        self.encode_decode_fused(step_ctx=step_ctx, query_buffer=query_buffer,
                                 new_keys_buffer=new_keys_buffer,
                                 new_values_buffer=new_values_buffer, key_buffer=key_buffer,
                                 value_buffer=value_buffer,
                                 block_table_buffer=block_table_buffer,
                                 seq_lens_buffer=seq_lens_buffer, output_buffer=output_buffer,
                                 num_seqs=num_seqs, max_seq_len=max_seq_len,
                                 max_blocks_per_seq=max_blocks_per_seq)

    def get_params_dict(self) -> Dict[str, Any]:
        return {"num_kv_heads": self.num_kv_heads, "num_query_heads": self.num_query_heads,
                "head_size": self.head_size, "block_size": self.block_size,
                "scale": self.scale, "kernel": "va_paged_decode",
                "prefill_kernel": "va_paged_prefill"}


class KVWriteOp:
    """KV-cache writes: decode (block table + seq_lens) and prefill (slot mapping)."""

    def __init__(self, context: Any, num_kv_heads: int, head_size: int, block_size: int):
        self._context = context
        self.num_kv_heads = num_kv_heads
        self.head_size = head_size
        self.block_size = block_size
        self.kv_stride_block = num_kv_heads * block_size * head_size
        self.kv_stride_head = block_size * head_size
        self.kv_stride_token = head_size
        self.new_kv_stride_token = num_kv_heads * head_size
        self.new_kv_stride_head = head_size
        _lib.load()

    def _num_blocks(self, key_buffer) -> int:
        return resolve(key_buffer)[1] // (self.kv_stride_block * _H)

    def encode_decode(self, step_ctx, new_keys_buffer, new_values_buffer, key_buffer,
                      value_buffer, block_table_buffer, seq_lens_buffer, num_seqs: int,
                      new_keys_offset: int = 0, new_values_offset: int = 0,
                      max_blocks_per_seq: int = 128) -> None:
        step_ctx.require_encoding("encode_decode()")
        _lib.check(_lib.load().va_kv_write_decode(
            resolve(key_buffer)[0], resolve(value_buffer)[0],
            resolve(new_keys_buffer, new_keys_offset)[0],
            resolve(new_values_buffer, new_values_offset)[0], resolve(block_table_buffer)[0],
            resolve(seq_lens_buffer)[0], num_seqs, max_blocks_per_seq, self.num_kv_heads,
            self.head_size, self.block_size, self._num_blocks(key_buffer), self.kv_stride_block,
            self.kv_stride_head, self.kv_stride_token, self.new_kv_stride_token,
            self.new_kv_stride_head, _err(step_ctx), step_ctx.stream_handle),
            "va_kv_write_decode")
        step_ctx.note_dispatch()

    def encode_prefill(self, step_ctx, new_keys_buffer, new_values_buffer, key_buffer,
                       value_buffer, slot_mapping_buffer, num_tokens: int,
                       new_keys_offset: int = 0, new_values_offset: int = 0) -> None:
        """Scatter by slot; the slot buffer is int32 (engine convention) unless it is
        an int64 tensor/view (vLLM convention).  Slot -1 rows are skipped."""
        step_ctx.require_encoding("encode_prefill()")
        is64 = int(buffer_dtype(slot_mapping_buffer) == torch.int64)
        _lib.check(_lib.load().va_kv_write_slots(
            resolve(key_buffer)[0], resolve(value_buffer)[0],
            resolve(new_keys_buffer, new_keys_offset)[0],
            resolve(new_values_buffer, new_values_offset)[0], resolve(slot_mapping_buffer)[0],
            is64, num_tokens, self.num_kv_heads, self.head_size, self.block_size,
            self._num_blocks(key_buffer), self.kv_stride_block, self.kv_stride_head,
            self.kv_stride_token, self.new_kv_stride_token, self.new_kv_stride_head,
            _err(step_ctx), step_ctx.stream_handle), "va_kv_write_slots")
        step_ctx.note_dispatch()

    def encode_prefill_with_rope(self, step_ctx, rope: "EngineRoPE", query_buffer,
                                 new_keys_buffer, new_values_buffer, key_buffer, value_buffer,
                                 slot_mapping_buffer, positions_buffer, num_tokens: int,
                                 query_offset: int = 0, new_keys_offset: int = 0,
                                 new_values_offset: int = 0) -> None:
        """RoPE of Q and K (in place) fused with the K/V scatter by slot: the
        reference encodes EngineRoPE.encode then encode_prefill (runner.py:942-1055)."""
        step_ctx.require_encoding("encode_prefill_with_rope()")
        if not rope.is_neox_style or rope.rotary_dim != self.head_size:
            raise ValueError("the fused path covers Neox RoPE over the whole head")
        is64 = int(buffer_dtype(slot_mapping_buffer) == torch.int64)
        D = self.head_size
        _lib.check(_lib.load().va_rope_kv_write_slots(
            resolve(query_buffer, query_offset)[0], resolve(new_keys_buffer, new_keys_offset)[0],
            resolve(new_values_buffer, new_values_offset)[0], resolve(key_buffer)[0],
            resolve(value_buffer)[0], rope._cos_cache.data_ptr(), rope._sin_cache.data_ptr(),
            resolve(positions_buffer)[0], resolve(slot_mapping_buffer)[0], is64, num_tokens,
            rope.num_heads, self.num_kv_heads, D, self.block_size, self._num_blocks(key_buffer),
            rope.max_position, rope.num_heads * D, self.num_kv_heads * D, self.num_kv_heads * D,
            self.kv_stride_block, self.kv_stride_head, self.kv_stride_token, _err(step_ctx),
            step_ctx.stream_handle), "va_rope_kv_write_slots")
        step_ctx.note_dispatch()

    def get_params_dict(self) -> Dict[str, Any]:
        return {"num_kv_heads": self.num_kv_heads, "head_size": self.head_size,
                "block_size": self.block_size, "decode_kernel": "va_kv_write_decode",
                "prefill_kernel": "va_kv_write_slots"}


class EngineRMSNorm:
    """``out = x * rsqrt(mean(x^2) + eps) * w (+ residual)`` per token row."""

    def __init__(self, context: Any, hidden_size: int, eps: float = 1e-6,
                 weight_buffer: Optional[Any] = None):
        self._context = context
        self.hidden_size = hidden_size
        self.eps = eps
        self._weight_buffer = weight_buffer
        _lib.load()

    def set_weights(self, weight_buffer: Any) -> None:
        self._weight_buffer = weight_buffer

    def encode(self, step_ctx, input_buffer, output_buffer, num_tokens: int,
               residual_buffer: Optional[Any] = None) -> None:
        if self._weight_buffer is None:
            raise RuntimeError("Weights not set - call set_weights() first")
        step_ctx.require_encoding("encode()")
        H = self.hidden_size
        res = resolve(residual_buffer)[0] if residual_buffer is not None else None
        _lib.check(_lib.load().va_rmsnorm(
            resolve(output_buffer)[0], resolve(input_buffer)[0], resolve(self._weight_buffer)[0],
            res, num_tokens, H, float(self.eps), H, H, H, step_ctx.stream_handle), "va_rmsnorm")
        step_ctx.note_dispatch()

    def get_output_size(self, num_tokens: int) -> int:
        return num_tokens * self.hidden_size * _H

    def get_params_dict(self) -> Dict[str, Any]:
        return {"hidden_size": self.hidden_size, "eps": self.eps}


def rope_cos_sin_cache(rotary_dim: int, max_position: int, base: float):
    """fp32 cos/sin tables [max_position, rotary_dim/2] built with the same
    fp32 steps as the reference's EngineRoPE._precompute_cache
    (elementwise.py:680-697), so kernel and reference see identical angles."""
    half = rotary_dim // 2
    inv_freq = 1.0 / (base ** (np.arange(0, half, dtype=np.float32) / half))
    freqs = np.outer(np.arange(max_position, dtype=np.float32), inv_freq)
    return np.cos(freqs).astype(np.float32), np.sin(freqs).astype(np.float32)


class EngineRoPE:
    """In-place rotary embedding of Q and K (Neox split-half by default)."""

    def __init__(self, context: Any, head_size: int, num_heads: int, num_kv_heads: int,
                 rotary_dim: Optional[int] = None, max_position: int = 8192,
                 base: float = 10000.0, is_neox_style: bool = True):
        self._context = context
        self.head_size = head_size
        self.num_heads = num_heads
        self.num_kv_heads = num_kv_heads
        self.rotary_dim = rotary_dim or head_size
        self.max_position = max_position
        self.base = base
        self.is_neox_style = is_neox_style
        cos, sin = rope_cos_sin_cache(self.rotary_dim, max_position, base)
        dev = context.device
        self._cos_cache = torch.from_numpy(cos).to(dev)
        self._sin_cache = torch.from_numpy(sin).to(dev)
        _lib.load()

    def encode(self, step_ctx, query, key, positions, num_tokens: int,
               max_position_in_batch: Optional[int] = None) -> None:
        step_ctx.require_encoding("encode()")
        if max_position_in_batch is not None and max_position_in_batch >= self.max_position:
            raise ValueError(
                f"Position ID {max_position_in_batch} exceeds max_position {self.max_position}. "
                f"Increase max_position in EngineRoPE constructor.")
        D = self.head_size
        _lib.check(_lib.load().va_rope(
            resolve(query)[0], resolve(key)[0], self._cos_cache.data_ptr(),
            self._sin_cache.data_ptr(), resolve(positions)[0], num_tokens, self.num_heads,
            self.num_kv_heads, D, self.rotary_dim, self.max_position, self.num_heads * D,
            self.num_kv_heads * D, int(self.is_neox_style), _err(step_ctx),
            step_ctx.stream_handle), "va_rope")
        step_ctx.note_dispatch()


class EngineElementwiseOps:
    """Elementwise ops of the step (SiLU-mul of the gated MLP)."""

    def __init__(self, context: Any):
        self._context = context
        _lib.load()

    def encode_silu_mul(self, step_ctx, gate, up, output, num_elements: int) -> None:
        step_ctx.require_encoding("encode()")
        _lib.check(_lib.load().va_silu_mul(resolve(output)[0], resolve(gate)[0], resolve(up)[0],
                                           num_elements, step_ctx.stream_handle), "va_silu_mul")
        step_ctx.note_dispatch()


TOPK_K_ENV = "VLLM_METAL_TOPK_K"


class EngineTopK:
    """Top-k logits per token on the device, so sampling reads back k (index, value)
    pairs instead of the whole vocabulary row.

    Mirrors ``EngineTopK`` (vllm_apple/engine/ops/topk.py:40-412): same constructor
    (``k`` defaults to 50, ``VLLM_METAL_TOPK_K`` overrides it), same ``encode``
    signature and outputs (int32 indices and fp16 values, ``[num_tokens, k]``,
    largest first).  The selection runs in ``va_topk`` for any 1 <= k <= 1024.
    """

    def __init__(self, context: Any, k: int = 50):
        import os
        self._context = context
        self._k = k
        env_k = os.environ.get(TOPK_K_ENV)
        if env_k:
            try:
                self._k = int(env_k)
            except ValueError:
                pass
        _lib.load()

    def encode(self, step_ctx, logits, indices_out, values_out, num_tokens: int,
               vocab_size: int, k: Optional[int] = None) -> None:
        step_ctx.require_encoding("encode()")
        k = k or self._k
        lib = _lib.load()
        nbytes = lib.va_topk_workspace_size(num_tokens, vocab_size, k)
        ws = _ops.workspace(_dev(step_ctx), "topk", nbytes, step_ctx.stream) if nbytes else None
        _lib.check(lib.va_topk_ws(resolve(indices_out)[0], resolve(values_out)[0],
                                  resolve(logits)[0], num_tokens, vocab_size, vocab_size, k,
                                  0 if ws is None else ws.data_ptr(), nbytes,
                                  step_ctx.stream_handle), "va_topk_ws")
        step_ctx.note_dispatch()

    @property
    def k(self) -> int:
        return self._k

    def get_stats(self) -> Dict[str, Any]:
        return {"k": self._k}
