"""The host-tensor bridge classes of the v1 plugin path vs the oracle."""
import numpy as np
import pytest
import torch

from _util import ATOL, max_abs, np16
from oracle import paged_attention as ref

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("workload", ["qwen_b4", "devstral_b128"])
def test_fused_bridge_host_tensors(workload):
    from vllm_apple_b200.bridge import MetalPagedAttentionFused
    from vllm_apple_b200.workloads import make_decode_case
    c = make_decode_case(workload, seed=3)
    kc, vc = c.k_cache.cuda(), c.v_cache.cuda()
    op = MetalPagedAttentionFused(c.Hkv, c.Hq, c.D, c.bs)
    assert op.is_fused_available
    out = torch.zeros_like(c.q)  # host output, as in the reference
    ret = op.forward_fused(c.q, c.new_k, c.new_v, kc, vc, c.block_table, c.seq_lens, out)
    assert ret is out and out.device.type == "cpu"
    rk, rv = c.k_cache.numpy().copy(), c.v_cache.numpy().copy()
    ref.kv_write_decode(rk, rv, c.new_k.numpy(), c.new_v.numpy(), c.block_table.numpy(),
                        c.seq_lens.numpy())
    o = ref.paged_decode(c.q.numpy(), rk, rv, c.block_table.numpy(), c.seq_lens.numpy(),
                         c.scale)
    assert max_abs(out.numpy(), o) <= ATOL
    np.testing.assert_array_equal(kc.cpu().numpy().view(np.int16), rk.view(np.int16))
    # non-fused over the now-populated cache gives the same output
    out2 = torch.zeros_like(c.q)
    op.forward_with_metal_buffers(c.q, kc, vc, c.block_table, c.seq_lens, out2)
    assert torch.equal(out, out2)


def test_v2_owned_cache_and_block_update():
    from vllm_apple_b200.bridge import MetalPagedAttentionV2
    from vllm_apple_b200.workloads import make_decode_case
    c = make_decode_case("qwen_b4", seed=5)
    rk, rv = c.k_cache.numpy().copy(), c.v_cache.numpy().copy()
    ref.kv_write_decode(rk, rv, c.new_k.numpy(), c.new_v.numpy(), c.block_table.numpy(),
                        c.seq_lens.numpy())
    op = MetalPagedAttentionV2(c.Hkv, c.Hq, c.D, c.bs, c.scale)
    op.set_kv_cache(torch.from_numpy(rk), torch.from_numpy(rv))
    out = op.forward(c.q, None, None, c.block_table, c.seq_lens, skip_kv_copy=True)
    o = ref.paged_decode(c.q.numpy(), rk, rv, c.block_table.numpy(), c.seq_lens.numpy(),
                         c.scale)
    assert max_abs(np16(out), o) <= ATOL
    # a changed block is seen after update_kv_cache_block
    blk = int(c.block_table[0, 0])
    rk[blk] = 0.5
    op.update_kv_cache_block(blk, torch.from_numpy(rk[blk]), torch.from_numpy(rv[blk]))
    out = op.forward(c.q, torch.from_numpy(rk), torch.from_numpy(rv), c.block_table,
                     c.seq_lens)
    o = ref.paged_decode(c.q.numpy(), rk, rv, c.block_table.numpy(), c.seq_lens.numpy(),
                         c.scale)
    assert max_abs(np16(out), o) <= ATOL


def test_metal_write_kv_batch_twin_bit_exact():
    from vllm_apple_b200.bridge import metal_write_kv_batch
    g = np.random.default_rng(0)
    nb, H, bs, D, T = 64, 2, 16, 64, 100
    kc = np.zeros((nb, H, bs, D), np.float16)
    vc = np.zeros_like(kc)
    k = g.standard_normal((T, H, D)).astype(np.float16)
    v = g.standard_normal((T, H, D)).astype(np.float16)
    slots = g.permutation(nb * bs)[:T]
    bid, off = (slots // bs).astype(np.int64), (slots % bs).astype(np.int64)
    dk, dv = torch.from_numpy(kc).cuda(), torch.from_numpy(vc).cuda()
    metal_write_kv_batch(dk, dv, k, v, bid, off, T, H, D, H * bs * D, bs * D, D)
    ref.write_kv_batch(kc.reshape(-1), vc.reshape(-1), k, v, bid, off, T, H, D, H * bs * D,
                       bs * D, D)  # the oracle writes flat buffers (views)
    np.testing.assert_array_equal(dk.cpu().numpy().view(np.int16), kc.view(np.int16))
    np.testing.assert_array_equal(dv.cpu().numpy().view(np.int16), vc.view(np.int16))

