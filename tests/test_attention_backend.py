"""The vLLM attention-backend mirror: static surface and error behaviour (CPU),
forward parity through the impl (GPU)."""
import numpy as np
import pytest
import torch

from _util import ATOL, bits, max_abs


def _mod():
    from vllm_apple_b200 import attention
    return attention


def test_backend_surface_matches_reference():
    a = _mod()
    B = a.MetalAttentionBackend
    assert B.get_name() == "METAL_ATTN"
    assert B.get_supported_head_sizes() == [32, 64, 96, 128]
    assert B.get_kv_cache_shape(100, 16, 8, 128) == (2, 100, 16, 8, 128)
    assert B.get_impl_cls() is a.MetalAttentionImpl
    assert B.get_builder_cls() is a.MetalAttentionMetadataBuilder
    assert B.accept_output_buffer and not B.use_cascade_attention()
    assert torch.bfloat16 in B.get_supported_dtypes()


def _impl(**kw):
    a = _mod()
    args = dict(num_heads=8, head_size=64, scale=0.125, num_kv_heads=2, alibi_slopes=None,
                sliding_window=None, kv_cache_dtype="auto")
    args.update(kw)
    return a.MetalAttentionImpl(**args)


def test_impl_error_behaviour():
    with pytest.raises(NotImplementedError):
        _impl(kv_cache_dtype="fp8")
    impl = _impl()
    out = torch.zeros(3, 8 * 64)
    assert impl.forward(None, out, out, out, None, None, out) is out  # warm-up
    with pytest.raises(NotImplementedError):
        impl.forward(None, out, out, out, None, None, out, output_scale=torch.ones(1))


@pytest.mark.gpu
def test_prefill_rows_chunked_positions():
    a = _mod()
    md = a.MetalAttentionMetadata(
        num_actual_tokens=5, max_query_len=3, query_start_loc=torch.tensor([0, 1, 2, 5]),
        max_seq_len=40, seq_lens=torch.tensor([10, 20, 40]),
        block_table=torch.zeros(3, 3, dtype=torch.int32), slot_mapping=None,
        scheduler_metadata=None, num_decode_tokens=2)
    tok, pos = md.prefill_rows("cuda")
    assert tok.tolist() == [2, 2, 2] and pos.tolist() == [37, 38, 39]


def _metadata(m, nd):
    a = _mod()
    return a.MetalAttentionMetadata(
        num_actual_tokens=m.num_tokens, max_query_len=int(torch.diff(m.query_start_loc).max()),
        query_start_loc=m.query_start_loc, max_seq_len=int(m.seq_lens.max()),
        seq_lens=m.seq_lens.cuda(), block_table=m.block_table.cuda(),
        slot_mapping=m.slot_mapping.cuda(), scheduler_metadata=None, causal=True,
        num_decode_tokens=nd)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_forward_mixed_batch(dtype):
    from oracle import paged_attention as ref
    from vllm_apple_b200.workloads import make_mixed_case
    m = make_mixed_case(layout="nhd", Hq=16, Hkv=4, D=128, num_chunks=2, chunk=96,
                        prior=(10, 700), num_decode=7, decode_len=(30, 2000), seed=11)
    kv = torch.stack([m.k_cache, m.v_cache]).cuda()
    T = m.num_tokens
    q = m.q.to(dtype).cuda().reshape(T, -1)
    k = m.k.to(dtype).cuda().reshape(T, -1)
    v = m.v.to(dtype).cuda().reshape(T, -1)
    out = torch.zeros(T, 16 * 128, dtype=dtype, device="cuda")
    impl = _impl(num_heads=16, head_size=128, scale=m.scale, num_kv_heads=4)
    impl.forward(None, q, k, v, kv, _metadata(m, 7), out)
    torch.cuda.synchronize()
    rk, rv = m.k_cache.numpy().copy(), m.v_cache.numpy().copy()
    kk, vv = m.k.to(dtype).half().numpy(), m.v.to(dtype).half().numpy()
    ref.kv_write_slots_vectorized(rk, rv, kk, vv, m.slot_mapping.numpy(), "nhd")
    o = ref.paged_prefill(m.q.to(dtype).half().numpy(), rk, rv, m.block_table.numpy(),
                          m.token_to_seq.numpy(), m.positions.numpy(), m.scale, layout="nhd")
    tol = ATOL if dtype == torch.float16 else 1e-2  # bf16 output rounding: 2^-9 relative
    assert max_abs(out.float().cpu().numpy().reshape(T, 16, 128), o) <= tol
    np.testing.assert_array_equal(bits(kv[0]), rk.view(np.int16))
    np.testing.assert_array_equal(bits(kv[1]), rv.view(np.int16))


@pytest.mark.gpu
def test_forward_kv_shared_layer_does_not_write():
    from vllm_apple_b200.workloads import make_mixed_case
    m = make_mixed_case(layout="nhd", Hq=8, Hkv=2, D=64, num_chunks=1, chunk=20, prior=(5, 50),
                        num_decode=3, decode_len=(10, 100), seed=2)
    kv = torch.stack([m.k_cache, m.v_cache]).cuda()
    before = kv.clone()
    T = m.num_tokens
    out = torch.zeros(T, 8 * 64, dtype=torch.float16, device="cuda")
    impl = _impl(kv_sharing_target_layer_name="layers.0.attn")
    impl.forward(None, m.q.cuda().reshape(T, -1), m.k.cuda().reshape(T, -1),
                 m.v.cuda().reshape(T, -1), kv, _metadata(m, 3), out)
    torch.cuda.synchronize()
    assert torch.equal(kv, before)


@pytest.mark.gpu
def test_forward_encoder_only_is_full_attention():
    a = _mod()
    torch.manual_seed(0)
    lens = [5, 33]
    T = sum(lens)
    q = torch.randn(T, 8 * 64, dtype=torch.float16, device="cuda")
    k = torch.randn(T, 2 * 64, dtype=torch.float16, device="cuda")
    v = torch.randn(T, 2 * 64, dtype=torch.float16, device="cuda")
    md = a.MetalAttentionMetadata(
        num_actual_tokens=T, max_query_len=33, query_start_loc=torch.tensor([0, 5, 38]),
        max_seq_len=33, seq_lens=torch.tensor(lens, device="cuda"), block_table=None,
        slot_mapping=None, scheduler_metadata=None, causal=False)
    impl = _impl(attn_type="encoder_only")
    out = torch.zeros_like(q)
    impl.forward(None, q, k, v, None, md, out)
    torch.cuda.synchronize()
    at = 0
    for n in lens:
        qq = q[at:at + n].float().view(n, 8, 64).transpose(0, 1)
        kk = k[at:at + n].float().view(n, 2, 64).transpose(0, 1).repeat_interleave(4, 0)
        vv = v[at:at + n].float().view(n, 2, 64).transpose(0, 1).repeat_interleave(4, 0)
        e = torch.nn.functional.scaled_dot_product_attention(qq, kk, vv, scale=0.125)
        got = out[at:at + n].float().view(n, 8, 64).transpose(0, 1)
        assert (got - e).abs().max().item() <= ATOL
        at += n
