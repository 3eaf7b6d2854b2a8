"""Decode paged attention (with the fused KV write) vs the oracle.

Attention outputs: max-abs <= 2e-3 vs the float64 oracle (fp16 I/O).
KV writes: bit-exact, and every other cache byte unchanged.
"""
import math

import numpy as np
import pytest
import torch

from _util import ATOL, bits, max_abs, np16
from oracle import paged_attention as ref

pytestmark = pytest.mark.gpu


def _ops():
    from vllm_apple_b200 import ops
    return ops


def _run_case(c, fused=True, seq_lens=None):
    ops = _ops()
    sl = c.seq_lens if seq_lens is None else seq_lens
    dk, dv = c.k_cache.cuda(), c.v_cache.cuda()
    q = c.q.cuda()
    out = torch.full_like(q, 7.0)
    max_len = max(int(sl.max()), 1)
    if fused:
        ops.paged_decode(out, q, dk, dv, c.block_table.cuda(), sl.cuda(), scale=c.scale,
                         max_seq_len=max_len, new_k=c.new_k.cuda(), new_v=c.new_v.cuda(),
                         layout=c.layout)
    else:
        ops.kv_write_decode(dk, dv, c.new_k.cuda(), c.new_v.cuda(), c.block_table.cuda(),
                            sl.cuda(), c.layout)
        ops.paged_decode(out, q, dk, dv, c.block_table.cuda(), sl.cuda(), scale=c.scale,
                         max_seq_len=max_len, layout=c.layout)
    torch.cuda.synchronize()
    bad = ops.check_device_errors(raise_on_error=False)
    return out, dk, dv, bad


def _oracle(c, seq_lens=None):
    sl = c.seq_lens if seq_lens is None else seq_lens
    rk, rv = c.k_cache.cpu().numpy().copy(), c.v_cache.cpu().numpy().copy()
    ref.kv_write_decode(rk, rv, c.new_k.numpy(), c.new_v.numpy(), c.block_table.numpy(),
                        sl.numpy(), layout=c.layout)
    o = ref.paged_decode(c.q.numpy(), rk, rv, c.block_table.numpy(), sl.numpy(), c.scale,
                         layout=c.layout)
    return o, rk, rv


@pytest.mark.parametrize("config", ["qwen_b4", "qwen_b64", "devstral_b128"])
@pytest.mark.parametrize("layout", ["hnd", "nhd"])
def test_decode_configs(config, layout):
    from vllm_apple_b200.workloads import make_decode_case
    c = make_decode_case(config, layout=layout, seed=0)
    out, dk, dv, bad = _run_case(c)
    assert bad == 0
    o, rk, rv = _oracle(c)
    err = max_abs(np16(out), o)
    assert err <= ATOL, f"{config}/{layout}: max abs err {err}"
    np.testing.assert_array_equal(bits(dk), rk.view(np.int16))
    np.testing.assert_array_equal(bits(dv), rv.view(np.int16))


def test_decode_unfused_equals_fused():
    from vllm_apple_b200.workloads import make_decode_case
    c = make_decode_case("qwen_b64", seed=5)
    o1, k1, v1, _ = _run_case(c, fused=True)
    o2, k2, v2, _ = _run_case(c, fused=False)
    np.testing.assert_array_equal(bits(o1), bits(o2))
    np.testing.assert_array_equal(bits(k1), bits(k2))


@pytest.mark.parametrize("Hq,Hkv,D", [(32, 4, 64), (8, 8, 128), (16, 2, 96), (8, 2, 32),
                                      (64, 4, 128), (12, 4, 128), (40, 8, 128)])
def test_decode_head_shapes(Hq, Hkv, D):
    """GQA groups 1..16 (>8 splits the group across CTAs), every head size."""
    from vllm_apple_b200 import workloads as w
    g = torch.Generator().manual_seed(Hq * 131 + D)
    L = torch.randint(1, 1500, (9,), generator=g)
    bt, nb = w.assign_blocks(L.tolist(), 16, 0, g)
    c = w.DecodeCase("custom", Hq, Hkv, D, 16, "hnd", nb, L.to(torch.int32), bt,
                     torch.zeros(9, dtype=torch.int64),
                     torch.randn(9, Hq, D, generator=g).half(),
                     torch.randn(9, Hkv, D, generator=g).half(),
                     torch.randn(9, Hkv, D, generator=g).half(),
                     torch.randn(nb, Hkv, 16, D, generator=g).half(),
                     torch.randn(nb, Hkv, 16, D, generator=g).half())
    out, dk, dv, bad = _run_case(c)
    assert bad == 0
    o, rk, _ = _oracle(c)
    assert max_abs(np16(out), o) <= ATOL
    np.testing.assert_array_equal(bits(dk), rk.view(np.int16))


def test_decode_single_token_known_answer():
    """seq_len = 1: the output is the new value row repeated over the GQA group,
    exactly (reference test_metal_kernels.py:380-438)."""
    ops = _ops()
    g = torch.Generator().manual_seed(9)
    B, Hq, Hkv, D = 1, 32, 4, 64
    q = torch.randn(B, Hq, D, generator=g).half().cuda()
    nk = torch.randn(B, Hkv, D, generator=g).half().cuda()
    nv = torch.randn(B, Hkv, D, generator=g).half().cuda()
    kc = torch.zeros(8, Hkv, 16, D, dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    out = torch.empty_like(q)
    bt = torch.zeros(B, 1, dtype=torch.int32, device="cuda")
    sl = torch.ones(B, dtype=torch.int32, device="cuda")
    ops.paged_decode(out, q, kc, vc, bt, sl, scale=1 / math.sqrt(D), max_seq_len=1,
                     new_k=nk, new_v=nv)
    exp = nv.repeat_interleave(Hq // Hkv, dim=1)
    assert torch.equal(out, exp)
    assert torch.equal(kc[0, :, 0], nk[0])


def test_decode_skips_empty_rows_and_flags_bad_blocks():
    from vllm_apple_b200.workloads import make_decode_case
    c = make_decode_case("qwen_b4", seed=1)
    sl = c.seq_lens.clone()
    sl[1] = 0
    out, _, _, bad = _run_case(c, seq_lens=sl)
    assert bad == 0
    assert torch.all(out[1].cpu() == 7.0), "row with seq_len 0 must stay untouched"
    o, _, _ = _oracle(c, seq_lens=sl)
    keep = [0, 2, 3]
    assert max_abs(np16(out)[keep], o[keep]) <= ATOL
    # an invalid block id inside a context is reported, never faults
    c.block_table[2, 0] = c.num_blocks + 5
    _, _, _, bad = _run_case(c)
    assert bad & 0x2


def test_decode_repeated_calls_reuse_workspace():
    """Split-KV tickets reset themselves: two calls in a row agree bit-for-bit."""
    from vllm_apple_b200.workloads import make_decode_case
    c = make_decode_case("devstral_b128", seed=2, batch=16)
    o1, _, _, _ = _run_case(c, fused=False)
    o2, _, _, _ = _run_case(c, fused=False)
    np.testing.assert_array_equal(bits(o1), bits(o2))
