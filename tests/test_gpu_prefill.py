"""Token-parallel causal paged attention (prefill / mixed batch) vs the oracle."""
import numpy as np
import pytest
import torch

from _util import ATOL, bits, max_abs, np16
from oracle import paged_attention as ref

pytestmark = pytest.mark.gpu


def _ops():
    from vllm_apple_b200 import ops
    return ops


def _run(c, token_to_seq=None, positions=None):
    """Scatter all new K/V rows by slot, then prefill attention (engine order)."""
    ops = _ops()
    dk, dv = c.k_cache.cuda(), c.v_cache.cuda()
    ops.kv_write_slots(dk, dv, c.k.cuda(), c.v.cuda(), c.slot_mapping.cuda(), c.layout)
    q = c.q.cuda()
    out = torch.full_like(q, 7.0)
    ts = c.token_to_seq if token_to_seq is None else token_to_seq
    ps = c.positions if positions is None else positions
    ops.paged_prefill(out, q, dk, dv, c.block_table.cuda(), ts.cuda(), ps.cuda(),
                      scale=c.scale, layout=c.layout)
    torch.cuda.synchronize()
    return out, dk, dv, ops.check_device_errors(raise_on_error=False)


def _oracle(c, token_to_seq=None, positions=None):
    rk, rv = c.k_cache.cpu().numpy().copy(), c.v_cache.cpu().numpy().copy()
    ref.kv_write_slots_vectorized(rk, rv, c.k.numpy(), c.v.numpy(), c.slot_mapping.numpy(),
                                  c.layout)
    ts = c.token_to_seq if token_to_seq is None else token_to_seq
    ps = c.positions if positions is None else positions
    o = ref.paged_prefill(c.q.numpy(), rk, rv, c.block_table.numpy(), ts.numpy(), ps.numpy(),
                          c.scale, layout=c.layout)
    return o, rk, rv


@pytest.mark.parametrize("layout", ["hnd", "nhd"])
def test_mixed_batch_config4(layout):
    """Config 4: 4 chunks of 512 tokens over prior context + 60 decode rows."""
    from vllm_apple_b200.workloads import make_mixed_case
    c = make_mixed_case(layout=layout, seed=0)
    out, dk, dv, bad = _run(c)
    assert bad == 0
    o, rk, rv = _oracle(c)
    err = max_abs(np16(out), o)
    assert err <= ATOL, f"max abs err {err}"
    np.testing.assert_array_equal(bits(dk), rk.view(np.int16))
    np.testing.assert_array_equal(bits(dv), rv.view(np.int16))


@pytest.mark.parametrize("Hq,Hkv,D", [(14, 2, 64), (8, 8, 128), (16, 2, 96), (8, 2, 32),
                                      (64, 4, 128)])
def test_prefill_shapes(Hq, Hkv, D):
    from vllm_apple_b200.workloads import make_mixed_case
    c = make_mixed_case(Hq=Hq, Hkv=Hkv, D=D, num_chunks=3, chunk=70, prior=(0, 300),
                        num_decode=5, decode_len=(1, 400), seed=Hq + D)
    out, _, _, bad = _run(c)
    assert bad == 0
    o, _, _ = _oracle(c)
    assert max_abs(np16(out), o) <= ATOL


def test_prefill_from_empty_cache_is_plain_causal_attention():
    """No prior context: the engine semantics equal causal SDPA over the chunk."""
    from vllm_apple_b200.workloads import make_mixed_case
    c = make_mixed_case(num_chunks=2, chunk=100, prior=(0, 0), num_decode=0, seed=3)
    out, _, _, _ = _run(c)
    q = c.q.float().view(2, 100, 32, 128).transpose(1, 2)
    k = c.k.float().view(2, 100, 8, 128).transpose(1, 2).repeat_interleave(4, dim=1)
    v = c.v.float().view(2, 100, 8, 128).transpose(1, 2).repeat_interleave(4, dim=1)
    exp = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True,
                                                           scale=c.scale)
    exp = exp.transpose(1, 2).reshape(200, 32, 128)
    assert max_abs(np16(out), exp.numpy()) <= ATOL


def test_prefill_skips_invalid_tokens():
    from vllm_apple_b200.workloads import make_mixed_case
    c = make_mixed_case(num_chunks=1, chunk=40, prior=(10, 10), num_decode=3,
                        decode_len=(20, 60), seed=4)
    ts = c.token_to_seq.clone()
    ps = c.positions.clone()
    ts[1] = -1          # invalid sequence
    ps[5] = -1          # negative position
    out, _, _, _ = _run(c, ts, ps)
    o, _, _ = _oracle(c, ts, ps)
    assert torch.all(out[1].cpu() == 7.0) and torch.all(out[5].cpu() == 7.0)
    keep = [i for i in range(c.num_tokens) if i not in (1, 5)]
    assert max_abs(np16(out)[keep], o[keep]) <= ATOL


@pytest.mark.parametrize("bs", [8, 32, 64])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("layout", ["hnd", "nhd"])
def test_prefill_block_sizes(bs, D, layout):
    """Pages of 8..64 tokens: chunk-to-page arithmetic, TMA boxes per lane, the
    row-by-row copy of the page holding the end of the context."""
    from vllm_apple_b200.workloads import make_mixed_case
    c = make_mixed_case(D=D, bs=bs, layout=layout, num_chunks=3, chunk=150, prior=(0, 700),
                        num_decode=4, decode_len=(1, 500), seed=bs + D)
    out, _, _, bad = _run(c)
    assert bad == 0
    o, _, _ = _oracle(c)
    assert max_abs(np16(out), o) <= ATOL


def test_prefill_bad_block_is_flagged_and_skipped():
    """An out-of-range block id inside a chunk's context: tokens that would read it
    are left unwritten and the bad-block flag is raised; earlier tokens are exact."""
    from vllm_apple_b200 import ops
    from vllm_apple_b200.workloads import make_mixed_case
    c = make_mixed_case(num_chunks=1, chunk=200, prior=(300, 300), num_decode=0, seed=9)
    bs = c.bs
    page = (300 + 100) // bs           # a page covering chunk positions ~400
    bt = c.block_table.clone()
    bt[0, page] = c.num_blocks + 7
    ops = _ops()
    dk, dv = c.k_cache.cuda(), c.v_cache.cuda()
    ops.kv_write_slots(dk, dv, c.k.cuda(), c.v.cuda(), c.slot_mapping.cuda(), c.layout)
    q = c.q.cuda()
    out = torch.full_like(q, 7.0)
    ops.paged_prefill(out, q, dk, dv, bt.cuda(), c.token_to_seq.cuda(), c.positions.cuda(),
                      scale=c.scale, layout=c.layout)
    torch.cuda.synchronize()
    flags = ops.check_device_errors(raise_on_error=False)
    assert flags & 2  # VA_FLAG_BAD_BLOCK
    o, _, _ = _oracle(c)
    pos = c.positions.numpy()
    first_bad = page * bs
    good = pos < first_bad
    assert good.any() and (~good).any()
    assert max_abs(np16(out)[good], o[good]) <= ATOL
    assert torch.all(out.cpu()[torch.from_numpy(~good)] == 7.0)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("layout", ["hnd", "nhd"])
def test_prefill_long_context_key_range_parts(D, layout):
    """Few tiles over long prior contexts: each tile's keys are cut into ranges
    processed by different CTAs (partial O, m, l merged by the part that finishes
    last, in part order).  Results as the oracle, and repeated calls agree bit for
    bit (the merge order does not depend on which part finishes last)."""
    from vllm_apple_b200.workloads import make_mixed_case
    Hq, Hkv = (32, 8) if D == 128 else (14, 2)
    c = make_mixed_case(D=D, Hq=Hq, Hkv=Hkv, layout=layout, num_chunks=2, chunk=64,
                        prior=(3000, 6000), num_decode=2, decode_len=(100, 3000), seed=D + 1)
    out, _, _, bad = _run(c)
    assert bad == 0
    o, _, _ = _oracle(c)
    assert max_abs(np16(out), o) <= ATOL
    out2, _, _, _ = _run(c)
    assert torch.equal(out, out2)


@pytest.mark.parametrize("where", ["early", "late"])
def test_prefill_bad_block_in_a_cut_tile(where):
    """A bad block id inside one key range of a tile that is cut into parts: rows
    whose context reaches it stay unwritten (all of them when it lies in an early
    range), the others are exact, and the flag is raised."""
    from vllm_apple_b200 import ops
    from vllm_apple_b200.workloads import make_mixed_case
    c = make_mixed_case(num_chunks=1, chunk=64, prior=(4000, 4000), num_decode=0, seed=11)
    bs = c.bs
    page = 1000 // bs if where == "early" else (4000 + 30) // bs
    bt = c.block_table.clone()
    bt[0, page] = c.num_blocks + 3
    dk, dv = c.k_cache.cuda(), c.v_cache.cuda()
    ops.kv_write_slots(dk, dv, c.k.cuda(), c.v.cuda(), c.slot_mapping.cuda(), c.layout)
    q = c.q.cuda()
    out = torch.full_like(q, 7.0)
    ops.paged_prefill(out, q, dk, dv, bt.cuda(), c.token_to_seq.cuda(), c.positions.cuda(),
                      scale=c.scale, layout=c.layout)
    torch.cuda.synchronize()
    assert ops.check_device_errors(raise_on_error=False) & 2
    o, _, _ = _oracle(c)
    good = c.positions.numpy() < page * bs
    if where == "early":
        assert not good.any()
    else:
        assert good.any() and (~good).any()
        assert max_abs(np16(out)[good], o[good]) <= ATOL
    assert torch.all(out.cpu()[torch.from_numpy(~good)] == 7.0)
