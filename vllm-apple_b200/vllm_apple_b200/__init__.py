"""vllm_apple_b200 -- the vllm_apple paged-attention hot path on B200 (sm_100a).

Layers:
  ``_lib``       ctypes binding of the C ABI library (include/vllm_apple_b200.h)
  ``ops``        torch-facing functional wrappers (one op = one C-ABI call)
  ``engine``     mirror of the reference's encode-only engine ops
                 (PagedAttentionOp, KVWriteOp, EngineRMSNorm, EngineRoPE,
                 EngineElementwiseOps) over CUDA streams
  ``attention``  mirror of the reference's vLLM attention backend
                 (MetalAttentionBackend / MetalAttentionImpl / metadata)
  ``workloads``  seeded synthetic inputs of the benchmark configurations
  ``sharding``   sequence sharding across GPUs (no collective on the path)
"""
from . import _lib, ops  # noqa: F401

__version__ = "0.1.0"


def library_path():
    return _lib.LIB_PATH
