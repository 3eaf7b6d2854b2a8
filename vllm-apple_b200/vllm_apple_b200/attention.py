"""vLLM v1 attention backend on the sm_100a kernels (drop-in for METAL_ATTN).

Same classes and signatures as the reference's
vllm_apple/v1/attention/backends/metal_attn.py:
  MetalAttentionBackend (:124-199), MetalAttentionMetadata (:202-250),
  MetalAttentionMetadataBuilder (:253-321), MetalAttentionImpl (:324-764).

Behaviour kept from the reference: decodes are ordered first
(``num_decode_tokens``), ``output`` is caller-allocated and written in place,
``attn_metadata is None`` returns ``output`` (warm-up), bf16 activations are
computed in fp16 and copied back, FP8 KV caches and quantised outputs raise
``NotImplementedError``, ALiBi / soft-cap only warn, a layer that shares
another layer's KV (``kv_sharing_target_layer_name``) does not write the cache.

What changes, on purpose:
  * the KV cache is vLLM's own ``(2, num_blocks, block_size, H, D)`` tensor,
    resident on the GPU (``get_kv_cache_device() == "cuda"``); there is no
    private per-layer cache and no host staging (reference :654-660, :847-943).
  * decode rows take one fused launch (KV write + split-KV attention) at any
    batch size (the reference switches to a non-fused path above
    VLLM_METAL_FUSED_MAX_SEQS).
  * prefill rows attend to the cached prior context of their sequence (chunked
    prefill), through the paged cache, on tensor cores; the reference's plugin
    prefill attends only to the new tokens (:1078-1149).
  * encoder (non-causal) attention runs on the same kernels: the new K/V go to
    a scratch paged cache and every token of a sequence sees all of it.
"""
from __future__ import annotations

import logging
from dataclasses import dataclass
from typing import ClassVar, Optional

import torch

from . import ops

logger = logging.getLogger(__name__)

try:  # vLLM is the host framework; the backend subclasses its interfaces when present
    from vllm.v1.attention.backend import (AttentionBackend, AttentionImpl, AttentionType,
                                           AttentionMetadataBuilder)
    from vllm.v1.attention.backends.utils import split_decodes_and_prefills
    from vllm.utils.torch_utils import is_quantized_kv_cache
    HAS_VLLM = True
except Exception:  # pragma: no cover - exercised only where vLLM is absent
    HAS_VLLM = False

    class AttentionBackend:  # minimal stand-ins with the same surface
        pass

    class AttentionImpl:
        pass

    class AttentionMetadataBuilder:
        def __class_getitem__(cls, item):
            return cls

        def __init__(self, kv_cache_spec, layer_names, vllm_config, device):
            self.kv_cache_spec, self.layer_names = kv_cache_spec, layer_names
            self.vllm_config, self.device = vllm_config, device

    class AttentionType:
        DECODER = "decoder"
        ENCODER = "encoder"
        ENCODER_ONLY = "encoder_only"
        ENCODER_DECODER = "encoder_decoder"

    def is_quantized_kv_cache(kv_cache_dtype: str) -> bool:
        return kv_cache_dtype.startswith("fp8")

    split_decodes_and_prefills = None


class MetalAttentionBackend(AttentionBackend):
    """Paged attention with the fused KV write on B200 (backend name kept)."""

    accept_output_buffer: bool = True
    supported_dtypes: ClassVar[list[torch.dtype]] = [torch.float16, torch.bfloat16]

    @classmethod
    def get_supported_dtypes(cls) -> list[torch.dtype]:
        return [torch.float16, torch.bfloat16]

    @classmethod
    def get_supported_head_sizes(cls) -> list[int]:
        return [32, 64, 96, 128]

    @staticmethod
    def get_name() -> str:
        return "METAL_ATTN"

    @classmethod
    def supports_attn_type(cls, attn_type: str) -> bool:
        return attn_type in (AttentionType.DECODER, AttentionType.ENCODER,
                             AttentionType.ENCODER_ONLY)

    @staticmethod
    def get_impl_cls() -> type["MetalAttentionImpl"]:
        return MetalAttentionImpl

    @staticmethod
    def get_builder_cls() -> type["MetalAttentionMetadataBuilder"]:
        return MetalAttentionMetadataBuilder

    @staticmethod
    def get_kv_cache_shape(num_blocks: int, block_size: int, num_kv_heads: int, head_size: int,
                           cache_dtype_str: str = "auto") -> tuple[int, ...]:
        """``[2, num_blocks, block_size, num_kv_heads, head_size]`` (0 = K, 1 = V)."""
        return 2, num_blocks, block_size, num_kv_heads, head_size

    @staticmethod
    def use_cascade_attention(*args, **kwargs) -> bool:
        return False

    @staticmethod
    def get_kv_cache_device() -> str:
        return "cuda"


B200AttentionBackend = MetalAttentionBackend


@dataclass
class MetalAttentionMetadata:
    num_actual_tokens: int
    max_query_len: int
    query_start_loc: torch.Tensor
    max_seq_len: int
    seq_lens: torch.Tensor
    block_table: torch.Tensor
    slot_mapping: torch.Tensor
    scheduler_metadata: Optional[torch.Tensor]
    causal: bool = True
    num_decode_tokens: int = 0
    _query_start_loc_cpu: Optional[list] = None
    _seq_lens_cpu: Optional[list] = None
    # device-side prefill row metadata, built once per step and shared by every layer
    _prefill_token_to_seq: Optional[torch.Tensor] = None
    _prefill_positions: Optional[torch.Tensor] = None

    @property
    def query_start_loc_cpu(self) -> list:
        if self._query_start_loc_cpu is None:
            self._query_start_loc_cpu = self.query_start_loc.tolist()
        return self._query_start_loc_cpu

    @property
    def seq_lens_cpu(self) -> list:
        if self._seq_lens_cpu is None:
            self._seq_lens_cpu = self.seq_lens.tolist()
        return self._seq_lens_cpu

    def prefill_rows(self, device):
        """(token_to_seq, positions) int32 on ``device`` for tokens
        num_decode_tokens..num_actual_tokens-1 (sequence index is absolute); the
        i-th new token of a sequence sits at position seq_len - query_len + i.
        Built once per step on the device and shared by every layer."""
        if self._prefill_token_to_seq is None:
            qsl = self.query_start_loc.to(device=device, dtype=torch.int32)
            sl = self.seq_lens.to(device=device, dtype=torch.int32)
            bt = self.block_table.to(device=device, dtype=torch.int32).contiguous()
            nd = self.num_decode_tokens
            tok, pos, _ = ops.build_prefill_metadata(qsl.contiguous(), sl.contiguous(), bt,
                                                     self.num_actual_tokens - nd,
                                                     first_token=nd, with_slots=False)
            self._prefill_token_to_seq, self._prefill_positions = tok, pos
        return self._prefill_token_to_seq, self._prefill_positions


class MetalAttentionMetadataBuilder(AttentionMetadataBuilder[MetalAttentionMetadata]):
    """Builds the per-step metadata; decodes are reordered to the front."""

    def __init__(self, kv_cache_spec, layer_names: list[str], vllm_config, device: torch.device):
        super().__init__(kv_cache_spec, layer_names, vllm_config, device)
        if hasattr(self, "_init_reorder_batch_threshold"):
            self._init_reorder_batch_threshold(1, False)
        else:
            self.reorder_batch_threshold = 1
        self.kv_cache_spec = kv_cache_spec
        self.vllm_config = vllm_config
        pc = vllm_config.parallel_config
        self.num_kv_heads = vllm_config.model_config.get_num_kv_heads(pc)
        self.num_heads = vllm_config.model_config.get_num_attention_heads(pc)
        self.head_dim = kv_cache_spec.head_size
        self.dtype = vllm_config.model_config.dtype
        self.block_size = vllm_config.cache_config.block_size

    def build(self, common_prefix_len: int, common_attn_metadata, fast_build: bool = False
              ) -> MetalAttentionMetadata:
        c = common_attn_metadata
        num_decode_tokens = 0
        if c.causal and split_decodes_and_prefills is not None:
            _, _, num_decode_tokens, _ = split_decodes_and_prefills(
                c, decode_threshold=self.reorder_batch_threshold, require_uniform=True)
        md = MetalAttentionMetadata(
            num_actual_tokens=c.num_actual_tokens, max_query_len=c.max_query_len,
            query_start_loc=c.query_start_loc, max_seq_len=c.max_seq_len, seq_lens=c.seq_lens,
            block_table=c.block_table_tensor, slot_mapping=c.slot_mapping,
            scheduler_metadata=None, causal=c.causal, num_decode_tokens=num_decode_tokens)
        qcpu = getattr(c, "query_start_loc_cpu", None)
        # the cached host copy, when the runner made one (reading vLLM's
        # ``seq_lens_cpu`` property would force a device sync)
        scpu = getattr(c, "_seq_lens_cpu", None)
        if qcpu is not None:
            md._query_start_loc_cpu = qcpu.tolist()
        if scpu is not None:
            md._seq_lens_cpu = scpu.tolist()
        return md


def _i32(t: torch.Tensor) -> torch.Tensor:
    return t if (t.dtype == torch.int32 and t.is_contiguous()) else t.to(torch.int32).contiguous()


class MetalAttentionImpl(AttentionImpl):
    """Decode rows: one fused launch (KV write + split-KV attention).
    Prefill rows: KV scatter by slot, then causal paged attention on tensor cores."""

    def __init__(self, num_heads: int, head_size: int, scale: float, num_kv_heads: int,
                 alibi_slopes: Optional[list[float]], sliding_window: Optional[int],
                 kv_cache_dtype: str, logits_soft_cap: Optional[float] = None,
                 attn_type: str = AttentionType.DECODER,
                 kv_sharing_target_layer_name: Optional[str] = None,
                 sinks: Optional[torch.Tensor] = None) -> None:
        self.kv_sharing_target_layer_name = kv_sharing_target_layer_name
        self._is_kv_shared = kv_sharing_target_layer_name is not None
        self.num_heads = num_heads
        self.head_size = head_size
        self.scale = float(scale)
        if logits_soft_cap is not None:
            logger.warning("METAL_ATTN does not support logits softcap, outputs may be "
                           "slightly off")
        self.logits_soft_cap = logits_soft_cap or 0
        self.num_kv_heads = num_kv_heads
        if alibi_slopes is not None:
            logger.warning("METAL_ATTN does not support ALiBi slopes, ignoring")
        self.alibi_slopes = None
        if sliding_window is None:
            self.sliding_window = (-1, -1)
        elif attn_type == AttentionType.ENCODER_ONLY:
            self.sliding_window = (sliding_window - 1, sliding_window - 1)
        else:
            self.sliding_window = (sliding_window - 1, 0)
        self.kv_cache_dtype = kv_cache_dtype
        self.num_queries_per_kv = num_heads // num_kv_heads
        if is_quantized_kv_cache(kv_cache_dtype):
            raise NotImplementedError("FP8 KV cache is unsupported in METAL_ATTN")
        self.attn_type = attn_type
        self.sinks = sinks

    def forward(self, layer, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                kv_cache: torch.Tensor, attn_metadata: Optional[MetalAttentionMetadata],
                output: Optional[torch.Tensor] = None, output_scale: Optional[torch.Tensor] = None,
                output_block_scale: Optional[torch.Tensor] = None) -> torch.Tensor:
        assert output is not None, "Output tensor must be provided."
        if output_scale is not None or output_block_scale is not None:
            raise NotImplementedError(
                "Fused output quantization is not yet supported for MetalAttentionImpl")
        if attn_metadata is None:
            return output
        orig_out = output
        convert = query.dtype == torch.bfloat16
        if convert:
            query = query.to(torch.float16)
            key = key.to(torch.float16) if key is not None else None
            value = value.to(torch.float16) if value is not None else None
            output = torch.empty_like(output, dtype=torch.float16)

        T = attn_metadata.num_actual_tokens
        q3 = query[:T].view(T, self.num_heads, self.head_size)
        o3 = output[:T].view(T, self.num_heads, self.head_size)
        if self.attn_type in (AttentionType.ENCODER_ONLY, AttentionType.ENCODER):
            self._encoder(q3, key, value, o3, attn_metadata)
        else:
            self._decoder(q3, key, value, kv_cache, o3, attn_metadata)
        if convert:
            orig_out[:T].copy_(output[:T].to(orig_out.dtype))
            return orig_out
        return output

    def _kv3(self, t: Optional[torch.Tensor], T: int) -> Optional[torch.Tensor]:
        return None if t is None else t[:T].view(T, self.num_kv_heads, self.head_size)

    def _decoder(self, q3, key, value, kv_cache, o3, md: MetalAttentionMetadata) -> None:
        T = md.num_actual_tokens
        nd = md.num_decode_tokens
        kc, vc = kv_cache[0], kv_cache[1]
        k3, v3 = self._kv3(key, T), self._kv3(value, T)
        write = (not self._is_kv_shared) and key is not None and value is not None
        bt = _i32(md.block_table)
        sl = _i32(md.seq_lens)
        if T > nd:
            if write:
                ops.kv_write_slots(kc, vc, k3[nd:], v3[nd:], md.slot_mapping[nd:T].contiguous(),
                                   layout="nhd")
            tok, pos = md.prefill_rows(q3.device)
            ops.paged_prefill(o3[nd:], q3[nd:], kc, vc, bt, tok, pos, scale=self.scale,
                              layout="nhd", num_seqs=bt.shape[0])
        if nd:
            ops.paged_decode(o3[:nd], q3[:nd], kc, vc, bt, sl, scale=self.scale,
                             max_seq_len=max(int(md.max_seq_len), 1),
                             new_k=k3[:nd] if write else None, new_v=v3[:nd] if write else None,
                             layout="nhd", num_seqs=nd)

    def _encoder(self, q3, key, value, o3, md: MetalAttentionMetadata) -> None:
        """Non-causal attention over each sequence's new tokens: scatter K/V into
        a scratch paged cache (one run of blocks per sequence) and let every
        token see its whole sequence."""
        T = md.num_actual_tokens
        bs = 16
        bt, slots, tok, pos, total = encoder_layout(md.query_start_loc_cpu, bs)
        dev = q3.device
        kc = torch.zeros(total, bs, self.num_kv_heads, self.head_size, dtype=torch.float16,
                         device=dev)
        vc = torch.zeros_like(kc)
        k3 = self._kv3(key, T)
        v3 = self._kv3(value, T)
        ops.kv_write_slots(kc, vc, k3, v3, slots.to(dev), layout="nhd")
        ops.paged_prefill(o3, q3, kc, vc, bt.to(dev), tok.to(dev), pos.to(dev), scale=self.scale,
                          layout="nhd")


def encoder_layout(query_start_loc, bs: int):
    """Scratch cache layout of a non-causal (encoder) batch, built with tensor ops:
    sequence s gets ceil(len_s / bs) consecutive blocks; returns the block table
    [S, width] int32 (-1 padded), the slot of every token (int64), its sequence
    (int32), the position every token attends up to (the sequence's last, int32)
    and the number of blocks (>= 1)."""
    qsl = torch.as_tensor(query_start_loc, dtype=torch.int64)
    S = qsl.numel() - 1
    lens = qsl[1:] - qsl[:-1]
    nblk = (lens + bs - 1) // bs
    width = max(int(nblk.max()) if S > 0 else 1, 1)
    first = torch.cumsum(nblk, 0) - nblk  # first block of each sequence
    col = torch.arange(width, dtype=torch.int64)
    bt = torch.where(col[None, :] < nblk[:, None], first[:, None] + col[None, :],
                     torch.full((), -1, dtype=torch.int64)).to(torch.int32)
    tok = torch.repeat_interleave(torch.arange(S, dtype=torch.int64), lens)
    off = torch.arange(tok.numel(), dtype=torch.int64) - qsl[:-1][tok]
    slots = first[tok] * bs + off
    pos = (lens - 1)[tok].to(torch.int32)
    total = max(int(nblk.sum()), 1)
    return bt, slots, tok.to(torch.int32), pos, total


B200AttentionImpl = MetalAttentionImpl
