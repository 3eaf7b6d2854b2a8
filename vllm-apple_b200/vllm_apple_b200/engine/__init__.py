"""Encode-only engine API of the hot path (the reference's vllm_apple.engine ops),
running on CUDA streams over the sm_100a C ABI."""
from .context import EngineContext, EnginePhase, EngineStepContext, EngineTensor  # noqa: F401
from .kv_cache import EngineKVCache, KVCacheDescriptor  # noqa: F401
from .ops import (EngineElementwiseOps, EngineRMSNorm, EngineRoPE, EngineTopK,  # noqa: F401
                  KVWriteOp, PagedAttentionOp, rope_cos_sin_cache)

# The reference names its context MetalEngineContext; keep that name importable.
MetalEngineContext = EngineContext
