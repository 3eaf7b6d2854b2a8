"""MetalAttentionMetadataBuilder.build with vLLM's own CommonAttentionMetadata.

The builder must split a reordered batch exactly as the reference's does
(vllm_apple/v1/attention/backends/metal_attn.py:253-321): the reorder
threshold is 1 and the decode count comes from vLLM's
``split_decodes_and_prefills(..., decode_threshold=1, require_uniform=True)``.
The CPU tests check the split against that function on batches that mix
decodes and prefills; the GPU test runs ``forward`` on the metadata the builder
made and compares with the oracle.
"""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from _util import ATOL, bits, max_abs

vllm_backend = pytest.importorskip("vllm.v1.attention.backend")


def _fake_config(Hq, Hkv, D, bs=16):
    model = SimpleNamespace(get_num_kv_heads=lambda pc: Hkv,
                            get_num_attention_heads=lambda pc: Hq, dtype=torch.float16)
    return SimpleNamespace(parallel_config=SimpleNamespace(decode_context_parallel_size=1),
                           model_config=model, cache_config=SimpleNamespace(block_size=bs),
                           speculative_config=None), SimpleNamespace(head_size=D,
                                                                     sliding_window=None)


def _builder(Hq=16, Hkv=4, D=128, device="cpu"):
    from vllm_apple_b200.attention import MetalAttentionMetadataBuilder
    cfg, spec = _fake_config(Hq, Hkv, D)
    return MetalAttentionMetadataBuilder(spec, ["layers.0.attn"], cfg, torch.device(device))


def _common(query_lens, seq_lens, bt, device="cpu", causal=True, slots=None):
    from vllm.v1.attention.backend import CommonAttentionMetadata
    ql = torch.tensor(query_lens, dtype=torch.int32)
    qsl = torch.zeros(len(ql) + 1, dtype=torch.int32)
    qsl[1:] = torch.cumsum(ql, 0)
    sl = torch.tensor(seq_lens, dtype=torch.int32)
    T = int(qsl[-1])
    return CommonAttentionMetadata(
        query_start_loc=qsl.to(device), query_start_loc_cpu=qsl, seq_lens=sl.to(device),
        num_reqs=len(ql), num_actual_tokens=T, max_query_len=int(ql.max()),
        max_seq_len=int(sl.max()), block_table_tensor=bt.to(device),
        slot_mapping=(torch.zeros(T, dtype=torch.int64) if slots is None else slots).to(device),
        causal=causal, _seq_lens_cpu=sl)


@pytest.mark.parametrize("query_lens", [
    [1, 1, 1, 40, 7],          # decodes first, then prefills
    [1, 1, 1, 1],              # all decodes
    [1, 1, 0, 0],              # padded uniform decode batch (CUDA-graph padding)
    [5, 1, 1],                 # a prefill first: no decodes
    [3, 3, 3],                 # uniform 3-token queries: all "decodes" only if <= threshold
    [1, 2, 1, 9],              # short extend after a decode
])
def test_build_split_matches_vllm(query_lens):
    from vllm.v1.attention.backends.utils import split_decodes_and_prefills
    b = _builder()
    assert b.reorder_batch_threshold == 1
    seq_lens = [q + 100 * (i + 1) for i, q in enumerate(query_lens)]
    bt = torch.zeros(len(query_lens), 64, dtype=torch.int32)
    c = _common(query_lens, seq_lens, bt)
    md = b.build(0, c)
    _, _, nd, _ = split_decodes_and_prefills(c, decode_threshold=1, require_uniform=True)
    assert md.num_decode_tokens == nd
    assert md.num_actual_tokens == c.num_actual_tokens
    assert md.max_query_len == c.max_query_len and md.max_seq_len == c.max_seq_len
    assert md.block_table is c.block_table_tensor and md.slot_mapping is c.slot_mapping
    assert md.query_start_loc_cpu == c.query_start_loc_cpu.tolist()
    assert md.seq_lens_cpu == seq_lens


def test_build_expected_counts():
    b = _builder()
    bt = torch.zeros(5, 8, dtype=torch.int32)
    md = b.build(0, _common([1, 1, 1, 40, 7], [50, 60, 70, 80, 90], bt))
    assert md.num_decode_tokens == 3
    md = b.build(0, _common([1, 2, 1, 9], [50, 60, 70, 80], bt[:4]))
    assert md.num_decode_tokens == 1  # the 2-token extend ends the decode run
    md = b.build(0, _common([3, 3, 3], [50, 60, 70], bt[:3]))
    assert md.num_decode_tokens == 0  # require_uniform with threshold 1: no decodes


def test_build_non_causal_has_no_decodes():
    b = _builder()
    bt = torch.zeros(3, 8, dtype=torch.int32)
    md = b.build(0, _common([1, 1, 5], [10, 20, 30], bt, causal=False))
    assert md.num_decode_tokens == 0 and md.causal is False


@pytest.mark.gpu
def test_forward_on_builder_metadata():
    """forward over a mixed batch whose metadata comes from build()."""
    from oracle import paged_attention as ref
    from vllm_apple_b200.attention import MetalAttentionImpl
    from vllm_apple_b200.workloads import make_mixed_case
    m = make_mixed_case(layout="nhd", Hq=16, Hkv=4, D=128, num_chunks=2, chunk=80,
                        prior=(10, 600), num_decode=6, decode_len=(30, 1500), seed=21)
    ql = torch.diff(m.query_start_loc).tolist()
    c = _common(ql, m.seq_lens.tolist(), m.block_table, device="cuda", slots=m.slot_mapping)
    md = _builder(device="cuda").build(0, c)
    assert md.num_decode_tokens == 6
    kv = torch.stack([m.k_cache, m.v_cache]).cuda()
    T = m.num_tokens
    out = torch.zeros(T, 16 * 128, dtype=torch.float16, device="cuda")
    impl = MetalAttentionImpl(num_heads=16, head_size=128, scale=m.scale, num_kv_heads=4,
                              alibi_slopes=None, sliding_window=None, kv_cache_dtype="auto")
    impl.forward(None, m.q.cuda().reshape(T, -1), m.k.cuda().reshape(T, -1),
                 m.v.cuda().reshape(T, -1), kv, md, out)
    torch.cuda.synchronize()
    rk, rv = m.k_cache.numpy().copy(), m.v_cache.numpy().copy()
    ref.kv_write_slots_vectorized(rk, rv, m.k.numpy(), m.v.numpy(), m.slot_mapping.numpy(), "nhd")
    o = ref.paged_prefill(m.q.numpy(), rk, rv, m.block_table.numpy(), m.token_to_seq.numpy(),
                          m.positions.numpy(), m.scale, layout="nhd")
    assert max_abs(out.cpu().numpy().reshape(T, 16, 128), o) <= ATOL
    np.testing.assert_array_equal(bits(kv[0]), rk.view(np.int16))
    np.testing.assert_array_equal(bits(kv[1]), rv.view(np.int16))
