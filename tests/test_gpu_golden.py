"""The CUDA path against the reference's own outputs (golden fixtures)."""
import os

import numpy as np
import pytest
import torch

from _util import ATOL, bits, max_abs, np16

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_decode_fused_vs_reference_golden():
    from vllm_apple_b200 import ops
    g = dict(np.load(os.path.join(GOLD, "decode_qwen_b4.npz")))
    cache = torch.from_numpy(g["cache_in"]).cuda()
    kc, vc = cache[0], cache[1]                       # vLLM layout (nb, bs, H, D)
    q = torch.from_numpy(g["q"]).cuda()
    out = torch.empty_like(q)
    ops.paged_decode(out, q, kc, vc, torch.from_numpy(g["block_table"]).cuda(),
                     torch.from_numpy(g["seq_lens"]).cuda(), scale=1 / np.sqrt(64),
                     max_seq_len=int(g["seq_lens"].max()), new_k=torch.from_numpy(g["k"]).cuda(),
                     new_v=torch.from_numpy(g["v"]).cuda(), layout="nhd")
    assert ops.check_device_errors() == 0
    assert max_abs(np16(out), g["out"]) <= ATOL
    np.testing.assert_array_equal(bits(cache), g["cache_out"].view(np.int16))


def test_prefill_vs_reference_golden():
    from vllm_apple_b200 import ops
    g = dict(np.load(os.path.join(GOLD, "prefill_noprior.npz")))
    cache = torch.from_numpy(g["cache_in"]).cuda()
    kc, vc = cache[0], cache[1]
    ops.kv_write_slots(kc, vc, torch.from_numpy(g["k"]).cuda(), torch.from_numpy(g["v"]).cuda(),
                       torch.from_numpy(g["slot_mapping"]).cuda(), layout="nhd")
    np.testing.assert_array_equal(bits(cache), g["cache_out"].view(np.int16))
    q = torch.from_numpy(g["q"]).cuda()
    out = torch.empty_like(q)
    ops.paged_prefill(out, q, kc, vc, torch.from_numpy(g["block_table"]).cuda(),
                      torch.from_numpy(g["token_to_seq"]).cuda(),
                      torch.from_numpy(g["positions"]).cuda(), scale=1 / np.sqrt(64),
                      layout="nhd")
    assert ops.check_device_errors() == 0
    assert max_abs(np16(out), g["out"]) <= ATOL


def test_rope_equivalence_with_reference_test_formula():
    """Port of tests/unit/test_rope_equiv.py: 14 heads, D=64, positions 0..15,
    theta 1e4, against the rotate-half torch formula, tolerance 1e-3 (tables in
    fp32 here, as the engine builds them)."""
    from vllm_apple_b200.engine.ops import rope_cos_sin_cache
    from vllm_apple_b200 import ops
    T, H, D, base = 16, 14, 64, 1e4
    torch.manual_seed(0)
    q = torch.randn(T, H, D).half()
    k = torch.randn(T, 2, D).half()
    pos = torch.arange(T, dtype=torch.int32)
    inv = 1.0 / (base ** (torch.arange(0, D, 2).float() / D))
    fr = torch.outer(torch.arange(64).float(), inv)
    emb = torch.cat((fr, fr), -1)
    cos, sin = emb.cos()[pos.long()].unsqueeze(1), emb.sin()[pos.long()].unsqueeze(1)

    def rot(x):
        x1, x2 = x[..., :D // 2], x[..., D // 2:]
        return x * cos + torch.cat((-x2, x1), -1) * sin

    qe, ke = rot(q.float()), rot(k.float())
    c, s = rope_cos_sin_cache(D, 64, base)
    dq, dk = q.cuda(), k.cuda()
    ops.rope(dq, dk, torch.from_numpy(c).cuda(), torch.from_numpy(s).cuda(), pos.cuda())
    # the reference test's 1e-3, plus the fp16 rounding of the output (half an ulp)
    assert bool(((dq.cpu().float() - qe).abs() <= 1e-3 + 2 ** -11 * qe.abs()).all())
    assert bool(((dk.cpu().float() - ke).abs() <= 1e-3 + 2 ** -11 * ke.abs()).all())


@pytest.mark.parametrize("name,D", [("decode_config1.npz", 64), ("decode_22b_600.npz", 128)])
def test_decode_config_goldens_on_gpu(name, D):
    """The fused decode on the reference-produced config-1 step and 22B-shaped sequence:
    KV bytes equal the reference's, outputs within 2e-3 of its fp32 result."""
    from vllm_apple_b200 import ops
    g = dict(np.load(os.path.join(GOLD, name)))
    cache = torch.from_numpy(g["cache_in"]).cuda()
    kc, vc = cache[0], cache[1]
    q = torch.from_numpy(g["q"]).cuda()
    out = torch.empty_like(q)
    ops.paged_decode(out, q, kc, vc, torch.from_numpy(g["block_table"]).cuda(),
                     torch.from_numpy(g["seq_lens"]).cuda(), scale=1 / np.sqrt(D),
                     max_seq_len=int(g["seq_lens"].max()), new_k=torch.from_numpy(g["k"]).cuda(),
                     new_v=torch.from_numpy(g["v"]).cuda(), layout="nhd")
    assert ops.check_device_errors() == 0
    assert max_abs(np16(out), g["out"]) <= ATOL
    exp = g["cache_in"].copy()
    bs = exp.shape[2]
    sl = g["slot_mapping"]
    exp[:, sl // bs, sl % bs] = g["written_rows"]
    np.testing.assert_array_equal(bits(cache), exp.view(np.int16))
