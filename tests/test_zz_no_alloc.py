"""Decode through the entry point that allocates nothing.

Some hosts cannot hand this library a workspace: they reach it only through
the C ABI with no CUDA allocator of their own, or run a serving loop that must
not call cudaMalloc once it is up.  va_paged_decode_noalloc keeps its split-KV
scratch in memory built into the library.  Here it must give the same output
as va_paged_decode with a caller workspace, on two calls in a row (the shared
scratch keeps the previous call's contents), and refuse shapes that need more
scratch than it has.  This file is collected last on purpose.
"""
import numpy as np
import pytest
import torch

from _util import ATOL, max_abs, np16

pytestmark = pytest.mark.gpu


def _args(c, out, q, kc, vc, bt, sl, max_len):
    nb, H, bs, D = kc.shape
    return (out.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(),
            sl.data_ptr(), None, None, c.batch, c.Hq, c.Hkv, D, bs, bt.shape[1], max_len, nb,
            c.scale, H * bs * D, bs * D, D, c.Hq * D, D, c.Hq * D, D, 0, 0)


@pytest.mark.parametrize("config,batch", [("devstral_b128", 24), ("qwen_b64", None), ("devstral_b128", 256)])
def test_noalloc_decode_matches_workspace_decode(config, batch):
    from vllm_apple_b200 import _lib, ops
    from vllm_apple_b200.workloads import make_decode_case
    lib = _lib.load()
    c = make_decode_case(config, seed=4, batch=batch)
    kc, vc = c.k_cache.cuda(), c.v_cache.cuda()
    q, bt, sl = c.q.cuda(), c.block_table.cuda(), c.seq_lens.cuda()
    max_len = c.max_seq_len
    need = lib.va_paged_decode_workspace_size(c.batch, c.Hq, c.Hkv, c.D, c.bs, max_len)
    assert need > 0, "the case must exercise the split-KV scratch"
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream

    ref_out = torch.empty_like(q)
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    a = _args(c, ref_out, q, kc, vc, bt, sl, max_len)
    assert lib.va_paged_decode(*a, ws.data_ptr(), need, err.data_ptr(), stream) == 0

    for _ in range(2):  # two calls in a row share the same built-in scratch
        out = torch.full_like(q, 7.0)
        a = _args(c, out, q, kc, vc, bt, sl, max_len)
        assert lib.va_paged_decode_noalloc(*a, err.data_ptr(), stream) == 0
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert max_abs(np16(out), np16(ref_out)) <= ATOL
        assert torch.equal(out, ref_out)


def _header_scratch_bytes():
    """VA_DECODE_STATIC_SCRATCH_BYTES as the public header defines it."""
    import os
    import re
    hdr = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                       "vllm_apple_b200.h")
    m = re.search(r"#define VA_DECODE_STATIC_SCRATCH_BYTES \((\d+)u << (\d+)\)", open(hdr).read())
    assert m, "VA_DECODE_STATIC_SCRATCH_BYTES not found in the header"
    return int(m.group(1)) << int(m.group(2))


def test_noalloc_rejects_shapes_beyond_its_scratch():
    from vllm_apple_b200 import _lib
    lib = _lib.load()
    limit = _header_scratch_bytes()
    # 4096 sequences of up to 65536 tokens need far more split scratch than is built in
    need = lib.va_paged_decode_workspace_size(4096, 32, 8, 128, 16, 65536)
    assert need > limit
    # Every pointer is NULL: whatever order the checks run in, nothing can launch
    # (va_paged_decode itself rejects NULL buffers before any launch).
    rc = lib.va_paged_decode_noalloc(None, None, None, None, None, None, None, None,
                                     4096, 32, 8, 128, 16, 4096, 65536, 1 << 20, 0.1,
                                     8 * 16 * 128, 16 * 128, 128, 4096, 128, 4096, 128, 0, 0,
                                     None, None)
    assert rc == _lib.VA_ERR_SCRATCH_LIMIT
    # a shape va_paged_decode does not support reports that, not the scratch limit
    rc = lib.va_paged_decode_noalloc(None, None, None, None, None, None, None, None,
                                     4096, 32, 8, 128, 32, 4096, 65536, 1 << 20, 0.1,
                                     8 * 32 * 128, 32 * 128, 128, 4096, 128, 4096, 128, 0, 0,
                                     None, None)
    assert rc == _lib.VA_ERR_UNSUPPORTED
