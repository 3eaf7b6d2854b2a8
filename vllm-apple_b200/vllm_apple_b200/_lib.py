"""ctypes binding of ``libvllm_apple_b200.so`` (the sm_100a C ABI).

The library is the only compute path: if it is missing or fails to load, every
op raises -- there is no CPU or PyTorch fallback.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import c_float, c_int, c_int32, c_int64, c_size_t, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libvllm_apple_b200.so"

VA_OK = 0
VA_ERR_INVALID_ARG = 1
VA_ERR_UNSUPPORTED = 2
VA_ERR_LAUNCH = 3
VA_ERR_WORKSPACE = 4
VA_ERR_SCRATCH_LIMIT = 5

VA_FLAG_BAD_SLOT = 0x1
VA_FLAG_BAD_BLOCK = 0x2
VA_FLAG_CTX_OVERFLOW = 0x4
VA_FLAG_WAIT_TIMEOUT = 0x8
VA_FLAG_BAD_POSITION = 0x10

_STATUS = {
    VA_ERR_INVALID_ARG: "invalid argument (size, stride or 16-byte alignment)",
    VA_ERR_UNSUPPORTED: "shape outside the compiled sm_100a variants",
    VA_ERR_LAUNCH: "CUDA launch failed",
    VA_ERR_WORKSPACE: "workspace missing or too small",
    VA_ERR_SCRATCH_LIMIT: "shape needs more than the library's built-in decode scratch",
}

FLAG_NAMES = {
    VA_FLAG_BAD_SLOT: "slot outside the cache",
    VA_FLAG_BAD_BLOCK: "block id outside the cache inside a context",
    VA_FLAG_CTX_OVERFLOW: "context longer than the block table / max_seq_len",
    VA_FLAG_WAIT_TIMEOUT: "bounded barrier wait gave up",
    VA_FLAG_BAD_POSITION: "rotary position outside [0, max_position)",
}

P = c_void_p
I64 = c_int64

# name -> (restype, argtypes); every entry is declared in include/vllm_apple_b200.h
SIGNATURES = {
    "va_version": (ctypes.c_char_p, []),
    "va_kv_write_slots": (c_int, [P, P, P, P, P, c_int, I64, c_int, c_int, c_int, I64, I64, I64,
                                  I64, I64, I64, P, P]),
    "va_kv_write_decode": (c_int, [P, P, P, P, P, P, I64, I64, c_int, c_int, c_int, I64, I64, I64,
                                   I64, I64, I64, P, P]),
    "va_write_kv_batch": (c_int, [P, P, P, P, P, P, c_int, c_int, c_int, c_int, c_int, c_int, P]),
    "va_paged_decode_workspace_size": (c_size_t, [I64, c_int, c_int, c_int, c_int, I64]),
    "va_paged_decode": (c_int, [P, P, P, P, P, P, P, P, I64, c_int, c_int, c_int, c_int, I64, I64,
                                I64, c_float, I64, I64, I64, I64, I64, I64, I64, I64, I64, P,
                                c_size_t, P, P]),
    "va_paged_decode_noalloc": (c_int, [P, P, P, P, P, P, P, P, I64, c_int, c_int, c_int, c_int,
                                        I64, I64, I64, c_float, I64, I64, I64, I64, I64, I64,
                                        I64, I64, I64, P, P]),
    "va_paged_prefill_workspace_size": (c_size_t, [I64, I64, c_int, c_int, c_int, c_int, I64]),
    "va_paged_prefill": (c_int, [P, P, P, P, P, P, P, I64, I64, c_int, c_int, c_int, c_int, I64,
                                 I64, c_float, I64, I64, I64, I64, I64, I64, I64, P, c_size_t, P,
                                 P]),
    "va_rope_kv_write_slots": (c_int, [P, P, P, P, P, P, P, P, P, c_int, I64, c_int, c_int, c_int,
                                       c_int, I64, I64, I64, I64, I64, I64, I64, I64, P, P]),
    "va_build_prefill_metadata": (c_int, [P, P, P, I64, I64, I64, I64, c_int, P, P, P, P]),
    "va_kv_sync_blocks": (c_int, [P, P, P, P, P, P, I64, I64, c_int, c_int, c_int, I64, I64, I64,
                                  I64, I64, I64, I64, P]),
    "va_rmsnorm": (c_int, [P, P, P, P, I64, I64, c_float, I64, I64, I64, P]),
    "va_rope": (c_int, [P, P, P, P, P, I64, c_int, c_int, c_int, c_int, I64, I64, I64, c_int, P,
                        P]),
    "va_silu_mul": (c_int, [P, P, P, I64, P]),
    "va_topk": (c_int, [P, P, P, I64, I64, I64, c_int, P]),
    "va_topk_workspace_size": (c_size_t, [I64, I64, c_int]),
    "va_topk_ws": (c_int, [P, P, P, I64, I64, I64, c_int, P, c_size_t, P]),
}

_lib = None


class VAError(RuntimeError):
    """A C-ABI call returned a non-zero status."""


def load(path: Path | str | None = None) -> ctypes.CDLL:
    """Load (once) and declare the library; raises if it is not built.

    ``VLLM_APPLE_B200_LIB`` may name an alternative build of the same ABI
    (used for tuning sweeps); by default the in-tree build is loaded."""
    global _lib
    if path is None:
        if _lib is not None:
            return _lib
        env = os.environ.get("VLLM_APPLE_B200_LIB")
        p = Path(env) if env else LIB_PATH
    else:
        p = Path(path)
    if not p.exists():
        raise RuntimeError(
            f"{p} is missing: build the sm_100a library first "
            "(python -m vllm_apple_b200.build); there is no fallback path")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def check(status: int, what: str) -> None:
    if status != VA_OK:
        raise VAError(f"{what}: status {status} ({_STATUS.get(status, 'unknown')})")


def describe_flags(bits: int) -> list[str]:
    return [txt for b, txt in FLAG_NAMES.items() if bits & b]
