"""The C-ABI library: loads without a GPU, exports every declared symbol, and
its host-side planning entry points behave (no compute is launched here)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "vllm_apple_b200.h")


def declared_symbols():
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"VA_API\s+[\w\s\*]+?\b(va_\w+)\s*\(", txt)))


@pytest.fixture(scope="module")
def lib():
    from vllm_apple_b200 import _lib
    return _lib.load()


def test_header_declares_the_abi():
    syms = declared_symbols()
    for s in ("va_kv_write_slots", "va_kv_write_decode", "va_write_kv_batch", "va_paged_decode",
              "va_paged_prefill", "va_rmsnorm", "va_rope", "va_silu_mul"):
        assert s in syms


def test_library_exports_every_declared_symbol(lib):
    for s in declared_symbols():
        assert hasattr(lib, s), f"{s} not exported"


def test_ctypes_signatures_cover_the_header():
    from vllm_apple_b200 import _lib
    assert set(_lib.SIGNATURES) == set(declared_symbols())


def test_version(lib):
    assert b"sm_100a" in lib.va_version()


def test_decode_workspace_size(lib):
    f = lib.va_paged_decode_workspace_size
    # a single short sequence never splits -> no workspace
    assert f(1, 32, 8, 128, 16, 64) == 0
    big = f(128, 32, 8, 128, 16, 8192)
    assert big > 0 and big % 256 == 0
    assert f(0, 32, 8, 128, 16, 8192) == 0
    assert f(4, 32, 5, 128, 16, 8192) == 0  # invalid head counts


def test_prefill_workspace_size(lib):
    assert lib.va_paged_prefill_workspace_size(0, 0, 32, 8, 128, 16, 512) == 0
    # tile plan + one-token-row list + split partials of routed decode rows
    assert lib.va_paged_prefill_workspace_size(2108, 64, 32, 8, 128, 16, 513) > 2108 * 8


def test_invalid_arguments_rejected_before_launch(lib):
    # head counts that do not divide, null pointers, bad sizes: status 1, nothing launched
    P = ctypes.c_void_p
    assert lib.va_paged_decode(P(16), P(16), P(16), P(16), P(16), P(16), None, None, 4, 32, 5,
                               128, 16, 8, 128, 64, 0.1, 0, 0, 0, 0, 0, 0, 0, 0, 0, None, 0,
                               None, None) == 1
    assert lib.va_kv_write_slots(None, None, None, None, None, 0, 5, 8, 128, 16, 4, 0, 0, 0, 0, 0,
                                 None, None) == 1
    assert lib.va_silu_mul(None, None, None, -1, None) == 1
    assert lib.va_rope(None, None, None, None, None, 3, 2, 1, 64, 63, 10, 64, 64, 1, None,
                       None) == 1
    # zero-size work is a no-op success
    assert lib.va_silu_mul(None, None, None, 0, None) == 0
    assert lib.va_kv_write_slots(None, None, None, None, None, 0, 0, 8, 128, 16, 4, 0, 0, 0, 0, 0,
                                 None, None) == 0


def test_unsupported_shapes_reported(lib):
    P = ctypes.c_void_p
    # head_size 80 is not a compiled variant
    assert lib.va_paged_decode(P(16), P(16), P(16), P(16), P(16), P(16), None, None, 4, 8, 8, 80,
                               16, 8, 128, 64, 0.1, 0, 0, 0, 0, 0, 0, 0, 0, 0, None, 0, None,
                               None) == 2


def test_ops_refuse_cpu_tensors():
    import torch
    from vllm_apple_b200 import ops
    x = torch.zeros(4, 8, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.silu_mul(x, x, x)


def test_decode_plan_regimes(lib):
    """The planner's two regimes, seen through the workspace they need (host-side,
    no GPU): a grid of >= 1024 (sequence, kv head) CTAs runs longest first and, at
    head_size > 64, unsplit below 8192 tokens -- its workspace is only the order
    (one int per sequence, 256-byte aligned); smaller grids split and need fp32
    partials (acc + (m, l) per sequence, q head and split)."""
    f = lib.va_paged_decode_workspace_size
    # 22B shape, 128 sequences x 8 kv heads = 1024 CTAs: ordered, unsplit
    assert f(128, 32, 8, 128, 16, 8192) == 512
    assert f(1024, 32, 8, 128, 16, 8192) == 4096
    # ... but contexts past 512 pages still split (partials + order)
    assert f(128, 32, 8, 128, 16, 16384) > 128 * 32 * 2 * 128 * 4
    # 64 sequences (512 CTAs): split rule, 128 pages per split at 8192 tokens
    assert f(64, 32, 8, 128, 16, 8192) == 64 * 32 * 4 * 128 * 4 + 64 * 32 * 4 * 2 * 4
    # Qwen shape at 1024 units stays split (and ordered): partials + order
    w = f(512, 14, 2, 64, 16, 4096)
    assert w > 512 * 4 and (w - ((512 * 4 + 255) // 256) * 256) % 256 == 0


def test_topk_entry_points_host_side(lib):
    """Top-k argument checks and the workspace contract, host side only: every row
    runs whole on one CTA, so no workspace is ever needed; invalid arguments are
    rejected before any launch and empty batches succeed without one."""
    P = ctypes.c_void_p
    for T, V, k in ((1, 131072, 50), (64, 32000, 8), (1024, 151936, 1024), (3, 7, 3)):
        assert lib.va_topk_workspace_size(T, V, k) == 0
    # k out of range, row stride below the vocabulary, negative sizes, null buffers
    assert lib.va_topk(P(16), P(16), P(16), 4, 100, 100, 0, None) == 1
    assert lib.va_topk(P(16), P(16), P(16), 4, 100, 99, 5, None) == 1
    assert lib.va_topk(P(16), P(16), P(16), -1, 100, 100, 5, None) == 1
    assert lib.va_topk(None, None, None, 4, 100, 100, 5, None) == 1
    assert lib.va_topk(P(16), P(16), P(16), 4, 100, 100, 1025, None) == 2
    assert lib.va_topk_ws(None, None, None, 4, 100, 100, 5, None, 0, None) == 1
    assert lib.va_topk(None, None, None, 0, 100, 100, 5, None) == 0
    assert lib.va_topk_ws(None, None, None, 0, 100, 100, 5, None, 0, None) == 0
