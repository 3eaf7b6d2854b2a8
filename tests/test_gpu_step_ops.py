"""Step-level ops on the GPU vs the oracle: fused RoPE + KV scatter,
device-side prefill metadata, layout sync of active blocks."""
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
@pytest.mark.parametrize("Hq,Hkv,D", [(32, 8, 128), (14, 2, 64)])
def test_rope_kv_write_equals_rope_then_scatter(layout, Hq, Hkv, D):
    ops = _ops()
    from vllm_apple_b200.engine.ops import rope_cos_sin_cache
    from vllm_apple_b200.workloads import make_mixed_case
    m = make_mixed_case(layout=layout, Hq=Hq, Hkv=Hkv, D=D, num_chunks=2, chunk=50,
                        prior=(0, 300), num_decode=5, decode_len=(10, 400), seed=Hq)
    cos, sin = rope_cos_sin_cache(D, 4096, 1e6)
    m.slot_mapping[3] = -1  # padding row
    # oracle: RoPE (fp32 ops) then scatter
    eq, ek = ref.rope(m.q.numpy(), m.k.numpy(), cos, sin, m.positions.numpy())
    eq16, ek16 = eq.astype(np.float32).astype(np.float16), ek.astype(np.float32).astype(np.float16)
    rk, rv = m.k_cache.numpy().copy(), m.v_cache.numpy().copy()
    ref.kv_write_slots_vectorized(rk, rv, ek16, m.v.numpy(), m.slot_mapping.numpy(), layout)
    # fused kernel
    q, k, v = m.q.cuda(), m.k.cuda(), m.v.cuda()
    kc, vc = m.k_cache.cuda(), m.v_cache.cuda()
    ops.rope_kv_write_slots(q, k, v, kc, vc, torch.from_numpy(cos).cuda(),
                            torch.from_numpy(sin).cuda(), m.positions.cuda(),
                            m.slot_mapping.cuda(), layout=layout)
    assert ops.check_device_errors() == 0
    np.testing.assert_array_equal(q.cpu().numpy(), eq16)
    np.testing.assert_array_equal(k.cpu().numpy(), ek16)
    np.testing.assert_array_equal(bits(kc), rk.view(np.int16))
    np.testing.assert_array_equal(bits(vc), rv.view(np.int16))


def test_prefill_metadata_on_device():
    ops = _ops()
    from vllm_apple_b200.workloads import make_mixed_case
    m = make_mixed_case(num_chunks=3, chunk=40, prior=(0, 300), num_decode=7,
                        decode_len=(10, 400), seed=5)
    ts, ps, sm = ops.build_prefill_metadata(m.query_start_loc.cuda(), m.seq_lens.cuda(),
                                            m.block_table.cuda(), m.num_tokens)
    tok, pos, slots = ref.prefill_metadata(m.query_start_loc.numpy(), m.seq_lens.numpy(),
                                           m.block_table.numpy(), 16)
    assert np.array_equal(ts.cpu().numpy(), tok) and np.array_equal(ps.cpu().numpy(), pos)
    assert np.array_equal(sm.cpu().numpy(), slots)
    assert np.array_equal(slots, m.slot_mapping.numpy())
    # a sub-range (e.g. the prefill part after the decode rows)
    ts2, ps2, _ = ops.build_prefill_metadata(m.query_start_loc.cuda(), m.seq_lens.cuda(),
                                             m.block_table.cuda(), m.num_tokens - 7,
                                             first_token=7, with_slots=False)
    assert np.array_equal(ts2.cpu().numpy(), tok[7:]) and np.array_equal(ps2.cpu().numpy(),
                                                                         pos[7:])


def test_kv_sync_blocks_bit_exact():
    ops = _ops()
    from vllm_apple_b200.workloads import make_decode_case
    c = make_decode_case("qwen_b64", layout="nhd", seed=2)
    L = c.seq_lens.clone()
    L[3] = 0
    bt = c.block_table.clone()
    bt[5, 0] = c.num_blocks + 3  # out of range: skipped
    dk = torch.zeros(c.num_blocks, c.Hkv, 16, c.D, dtype=torch.float16)
    dv = torch.zeros_like(dk)
    ek, ev = dk.numpy().copy(), dv.numpy().copy()
    ref.kv_sync_blocks(c.k_cache.numpy(), c.v_cache.numpy(), ek, ev, bt.numpy(), L.numpy())
    gk, gv = dk.cuda(), dv.cuda()
    ops.kv_sync_blocks(c.k_cache.cuda(), c.v_cache.cuda(), gk, gv, bt.cuda(), L.cuda())
    np.testing.assert_array_equal(bits(gk), ek.view(np.int16))
    np.testing.assert_array_equal(bits(gv), ev.view(np.int16))
