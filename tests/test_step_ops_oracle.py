"""CPU checks of the oracle for the step-level ops (layout sync, metadata),
including the reference's own sync test cases."""
import numpy as np

from oracle import paged_attention as ref


def test_prefill_metadata_matches_runner_rule():
    qsl = np.array([0, 1, 1, 4, 9], np.int32)        # an empty sequence included
    L = np.array([10, 3, 7, 20], np.int32)
    bt = np.arange(4 * 2).reshape(4, 2).astype(np.int32)
    tok, pos, slots = ref.prefill_metadata(qsl, L, bt, 16)
    assert tok.tolist() == [0, 2, 2, 2, 3, 3, 3, 3, 3]
    assert pos.tolist() == [9, 4, 5, 6, 15, 16, 17, 18, 19]
    assert slots[0] == 0 * 16 + 9 and slots[4] == 6 * 16 + 15 and slots[5] == 7 * 16 + 0


def test_kv_sync_transposes_active_blocks_only():
    """Ported from the reference's tests/metal/test_kv_sync.py: patterned values,
    NHD -> HND per block; unused and out-of-range block ids are skipped."""
    nb, bs, H, D = 6, 16, 2, 8
    src_k = np.arange(nb * bs * H * D, dtype=np.float32).reshape(nb, bs, H, D).astype(np.float16)
    src_v = (-src_k).astype(np.float16)
    dst_k = np.zeros((nb, H, bs, D), np.float16)
    dst_v = np.zeros_like(dst_k)
    bt = np.array([[2, 4, -1], [1, 7, 3]], np.int32)   # 7 is beyond the cache
    L = np.array([20, 40], np.int32)                   # seq 0: 2 blocks; seq 1: 3 blocks
    ref.kv_sync_blocks(src_k, src_v, dst_k, dst_v, bt, L)
    for b in (1, 2, 3, 4):
        assert np.array_equal(dst_k[b], src_k[b].transpose(1, 0, 2))
        assert np.array_equal(dst_v[b], src_v[b].transpose(1, 0, 2))
    assert not dst_k[0].any() and not dst_k[5].any()
