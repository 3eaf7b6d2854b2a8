"""KV-cache writes on the GPU must be bit-exact to the oracle (and leave all
other cache bytes untouched)."""
import numpy as np
import pytest
import torch

from _util import bits
from oracle import paged_attention as ref

pytestmark = pytest.mark.gpu


def _ops():
    from vllm_apple_b200 import ops
    return ops


@pytest.mark.parametrize("layout", ["hnd", "nhd"])
@pytest.mark.parametrize("slot_dtype", [torch.int32, torch.int64])
@pytest.mark.parametrize("H,D,bs", [(2, 64, 16), (8, 128, 16), (4, 96, 16), (3, 32, 32)])
def test_kv_write_slots_bit_exact(layout, slot_dtype, H, D, bs):
    ops = _ops()
    g = torch.Generator().manual_seed(1)
    nb, T = 64, 300
    shape = (nb, H, bs, D) if layout == "hnd" else (nb, bs, H, D)
    kc = torch.randn(shape, generator=g).half()
    vc = torch.randn(shape, generator=g).half()
    nk = torch.randn(T, H, D, generator=g).half()
    nv = torch.randn(T, H, D, generator=g).half()
    slots = torch.randperm(nb * bs, generator=g)[:T].to(torch.int64)
    slots[::7] = -1  # padding rows are skipped
    rk, rv = kc.numpy().copy(), vc.numpy().copy()
    ref.kv_write_slots(rk, rv, nk.numpy(), nv.numpy(), slots.numpy(), layout)
    dk, dv = kc.cuda(), vc.cuda()
    ops.kv_write_slots(dk, dv, nk.cuda(), nv.cuda(), slots.to(slot_dtype).cuda(), layout)
    assert ops.check_device_errors() == 0
    np.testing.assert_array_equal(bits(dk), rk.view(np.int16))
    np.testing.assert_array_equal(bits(dv), rv.view(np.int16))


def test_kv_write_slots_strided_rows_planar_qkv():
    """New K/V rows as views into a planar [Q | K | V] buffer (engine layout)."""
    ops = _ops()
    g = torch.Generator().manual_seed(2)
    T, Hq, H, D, bs, nb = 37, 32, 8, 128, 16, 32
    qkv = torch.randn(T * (Hq + 2 * H) * D, generator=g).half()
    k = qkv[T * Hq * D: T * (Hq + H) * D].view(T, H, D)
    v = qkv[T * (Hq + H) * D:].view(T, H, D)
    kc = torch.zeros(nb, H, bs, D, dtype=torch.float16)
    vc = torch.zeros_like(kc)
    slots = torch.randperm(nb * bs, generator=g)[:T]
    rk, rv = kc.numpy().copy(), vc.numpy().copy()
    ref.kv_write_slots(rk, rv, k.numpy(), v.numpy(), slots.numpy(), "hnd")
    dq = qkv.cuda()
    dk = dq[T * Hq * D: T * (Hq + H) * D].view(T, H, D)
    dv = dq[T * (Hq + H) * D:].view(T, H, D)
    ck, cv = kc.cuda(), vc.cuda()
    ops.kv_write_slots(ck, cv, dk, dv, slots.cuda(), "hnd")
    np.testing.assert_array_equal(bits(ck), rk.view(np.int16))
    np.testing.assert_array_equal(bits(cv), rv.view(np.int16))


def test_kv_write_slots_out_of_range_flagged_not_written():
    ops = _ops()
    H, D, bs, nb = 2, 64, 16, 4
    kc = torch.zeros(nb, H, bs, D, dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    nk = torch.ones(3, H, D, dtype=torch.float16, device="cuda")
    slots = torch.tensor([5, nb * bs, -3], dtype=torch.int64, device="cuda")
    ops.kv_write_slots(kc, vc, nk, nk.clone(), slots, "hnd")
    with pytest.raises(Exception):
        ops.check_device_errors()
    assert int((kc != 0).sum()) == H * D  # only slot 5 written


@pytest.mark.parametrize("layout", ["hnd", "nhd"])
def test_kv_write_decode_bit_exact(layout):
    ops = _ops()
    from vllm_apple_b200.workloads import make_decode_case
    c = make_decode_case("qwen_b64", layout=layout, seed=3)
    sl = c.seq_lens.clone()
    sl[5] = 0  # skipped row
    rk, rv = c.k_cache.numpy().copy(), c.v_cache.numpy().copy()
    ref.kv_write_decode(rk, rv, c.new_k.numpy(), c.new_v.numpy(), c.block_table.numpy(),
                        sl.numpy(), layout=layout)
    dk, dv = c.k_cache.cuda(), c.v_cache.cuda()
    ops.kv_write_decode(dk, dv, c.new_k.cuda(), c.new_v.cuda(), c.block_table.cuda(), sl.cuda(),
                        layout)
    assert ops.check_device_errors() == 0
    np.testing.assert_array_equal(bits(dk), rk.view(np.int16))
    np.testing.assert_array_equal(bits(dv), rv.view(np.int16))


def test_write_kv_batch_matches_reference_signature():
    """Device twin of metal_write_kv_batch vs the C oracle semantics."""
    ops = _ops()
    g = torch.Generator().manual_seed(4)
    nb, H, bs, D, T = 16, 4, 16, 64, 50
    kc = torch.randn(nb * H * bs * D, generator=g).half()
    vc = torch.randn(nb * H * bs * D, generator=g).half()
    nk = torch.randn(T, H, D, generator=g).half()
    nv = torch.randn(T, H, D, generator=g).half()
    slots = torch.randperm(nb * bs, generator=g)[:T]
    blk, off = (slots // bs).to(torch.int64), (slots % bs).to(torch.int64)
    rk, rv = kc.numpy().copy(), vc.numpy().copy()
    ref.write_kv_batch(rk, rv, nk.numpy(), nv.numpy(), blk.numpy(), off.numpy(), T, H, D,
                       H * bs * D, bs * D, D)
    dk, dv = kc.cuda(), vc.cuda()
    ops.write_kv_batch(dk, dv, nk.cuda(), nv.cuda(), blk.cuda(), off.cuda(), T, H, D,
                       H * bs * D, bs * D, D)
    np.testing.assert_array_equal(bits(dk), rk.view(np.int16))
    np.testing.assert_array_equal(bits(dv), rv.view(np.int16))
