"""The engine-op drop-in surface, driven through EngineStepContext, vs the oracle.

Every call goes through the reference's own op signatures
(vllm_apple/engine/ops/attention.py:290-537, kv_write.py:261-402,
rmsnorm.py:226-321, elementwise.py:496-532 and :699-766) with buffers laid out
as the reference's runner lays them out: Q, K and V of a step are planes of
ONE buffer, K at byte offset ``T*Hq*D*2`` and V after it
(vllm_apple/engine/runner.py:919-934).  Here the planar buffer itself also
starts at a non-zero byte offset inside a larger allocation, and outputs are
written at a non-zero byte offset, so every offset argument is exercised.

Bars: KV writes bit-exact (whole caches compared); attention and RMSNorm
max-abs <= 2e-3 vs the float64 oracle; RoPE bit-exact to the fp32 formula;
SiLU-mul within 1 fp16 ulp.
"""
import numpy as np
import pytest
import torch

from _util import ATOL, bits, max_abs, ulp_distance_fp16
from oracle import paged_attention as ref

pytestmark = pytest.mark.gpu

PAD = 4096  # bytes before the planar QKV block inside the buffer


def _ctx():
    from vllm_apple_b200.engine import EngineContext
    return EngineContext(0)


def _planar(q, k, v, pad=PAD):
    """One uint8 device buffer [pad | Q plane | K plane | V plane | tail]; returns
    (buffer, q offset, k offset, v offset) in bytes."""
    parts = [t.contiguous().view(torch.uint8).reshape(-1) for t in (q, k, v)]
    total = pad + sum(p.numel() for p in parts) + 256
    buf = torch.zeros(total, dtype=torch.uint8)
    offs, at = [], pad
    for p in parts:
        buf[at:at + p.numel()] = p
        offs.append(at)
        at += p.numel()
    return buf.cuda(), offs[0], offs[1], offs[2]


def _plane(buf, off, shape):
    n = int(np.prod(shape)) * 2
    return buf[off:off + n].view(torch.float16).view(shape)


def _decode_case(config, batch=None, seed=0):
    from vllm_apple_b200.workloads import make_decode_case
    return make_decode_case(config, seed=seed, batch=batch)


@pytest.mark.parametrize("config,batch", [("qwen_b4", None), ("devstral_b128", 24)])
def test_encode_decode_fused_planar_offsets(config, batch):
    from vllm_apple_b200.engine import PagedAttentionOp
    c = _decode_case(config, batch, seed=3)
    ctx = _ctx()
    op = PagedAttentionOp(ctx, c.Hkv, c.Hq, c.D, c.bs, c.scale)
    buf, qo, ko, vo = _planar(c.q, c.new_k, c.new_v)
    kc, vc = c.k_cache.cuda(), c.v_cache.cuda()
    B = c.batch
    out_off = 512
    out_buf = torch.full((out_off // 2 + B * c.Hq * c.D + 64,), 7.0, dtype=torch.float16,
                         device="cuda")
    with ctx.new_step(step_kind="decode", num_seqs=B) as sc:
        op.encode_decode_fused(sc, buf, buf, buf, kc, vc, c.block_table.cuda(),
                               c.seq_lens.cuda(), out_buf, B, c.max_seq_len,
                               max_blocks_per_seq=c.block_table.shape[1], query_offset=qo,
                               new_keys_offset=ko, new_values_offset=vo,
                               output_offset=out_off)
        sc.submit()
        sc.wait_until_completed()
    got = out_buf[out_off // 2:out_off // 2 + B * c.Hq * c.D].view(B, c.Hq, c.D).cpu().numpy()
    assert torch.all(out_buf[:out_off // 2].cpu() == 7.0), "bytes before output_offset written"
    rk, rv = c.k_cache.numpy().copy(), c.v_cache.numpy().copy()
    ref.kv_write_decode(rk, rv, c.new_k.numpy(), c.new_v.numpy(), c.block_table.numpy(),
                        c.seq_lens.numpy())
    o = ref.paged_decode(c.q.numpy(), rk, rv, c.block_table.numpy(), c.seq_lens.numpy(), c.scale)
    assert max_abs(got, o) <= ATOL
    np.testing.assert_array_equal(bits(kc), rk.view(np.int16))
    np.testing.assert_array_equal(bits(vc), rv.view(np.int16))


def test_kv_write_encode_decode_then_encode_decode():
    """KVWriteOp.encode_decode (planar K/V offsets) followed by the non-fused
    PagedAttentionOp.encode_decode in the same step."""
    from vllm_apple_b200.engine import KVWriteOp, PagedAttentionOp
    c = _decode_case("qwen_b64", seed=4)
    ctx = _ctx()
    kvw = KVWriteOp(ctx, c.Hkv, c.D, c.bs)
    op = PagedAttentionOp(ctx, c.Hkv, c.Hq, c.D, c.bs, c.scale)
    buf, qo, ko, vo = _planar(c.q, c.new_k, c.new_v)
    kc, vc = c.k_cache.cuda(), c.v_cache.cuda()
    bt, sl = c.block_table.cuda(), c.seq_lens.cuda()
    B = c.batch
    out = torch.empty(B, c.Hq, c.D, dtype=torch.float16, device="cuda")
    with ctx.new_step(step_kind="decode", num_seqs=B) as sc:
        kvw.encode_decode(sc, buf, buf, kc, vc, bt, sl, B, new_keys_offset=ko,
                          new_values_offset=vo, max_blocks_per_seq=bt.shape[1])
        sc.memory_barrier()
        op.encode_decode(sc, buf, kc, vc, bt, sl, out, B, c.max_seq_len,
                         max_blocks_per_seq=bt.shape[1], query_offset=qo)
        sc.submit()
        sc.wait_until_completed()
    rk, rv = c.k_cache.numpy().copy(), c.v_cache.numpy().copy()
    ref.kv_write_decode(rk, rv, c.new_k.numpy(), c.new_v.numpy(), c.block_table.numpy(),
                        c.seq_lens.numpy())
    np.testing.assert_array_equal(bits(kc), rk.view(np.int16))
    np.testing.assert_array_equal(bits(vc), rv.view(np.int16))
    o = ref.paged_decode(c.q.numpy(), rk, rv, c.block_table.numpy(), c.seq_lens.numpy(), c.scale)
    assert max_abs(out.cpu().numpy(), o) <= ATOL


@pytest.mark.parametrize("slot_dtype", [torch.int32, torch.int64])
@pytest.mark.parametrize("D", [128, 64])
def test_kv_write_encode_prefill_then_encode_prefill(slot_dtype, D):
    """A chunked-prefill mixed batch: KVWriteOp.encode_prefill by slot (int32 engine
    or int64 vLLM slots, one padding slot) then PagedAttentionOp.encode_prefill over
    the planar QKV buffer, output at a byte offset."""
    from vllm_apple_b200.engine import KVWriteOp, PagedAttentionOp
    from vllm_apple_b200.workloads import make_mixed_case
    Hq, Hkv = (32, 8) if D == 128 else (14, 2)
    m = make_mixed_case(seed=7, Hq=Hq, Hkv=Hkv, D=D, num_chunks=2, chunk=96, prior=(0, 700),
                        num_decode=5, decode_len=(20, 900))
    m.slot_mapping[2] = -1  # a padding row: its K/V are not written
    ctx = _ctx()
    kvw = KVWriteOp(ctx, Hkv, D, m.bs)
    op = PagedAttentionOp(ctx, Hkv, Hq, D, m.bs, m.scale)
    buf, qo, ko, vo = _planar(m.q, m.k, m.v)
    kc, vc = m.k_cache.cuda(), m.v_cache.cuda()
    T, S = m.num_tokens, len(m.seq_lens)
    out_off = 1024
    out_buf = torch.zeros(out_off // 2 + T * Hq * D, dtype=torch.float16, device="cuda")
    slots = m.slot_mapping.to(slot_dtype).cuda()
    with ctx.new_step(step_kind="prefill", num_tokens=T, num_seqs=S) as sc:
        kvw.encode_prefill(sc, buf, buf, kc, vc, slots, T, new_keys_offset=ko,
                           new_values_offset=vo)
        sc.memory_barrier()
        op.encode_prefill(sc, buf, kc, vc, m.block_table.cuda(), m.token_to_seq.cuda(),
                          m.positions.cuda(), out_buf, T, S, int(m.seq_lens.max()),
                          m.block_table.shape[1], query_offset=qo, output_offset=out_off)
        sc.submit()
        sc.wait_until_completed()
    rk, rv = m.k_cache.numpy().copy(), m.v_cache.numpy().copy()
    ref.kv_write_slots_vectorized(rk, rv, m.k.numpy(), m.v.numpy(), m.slot_mapping.numpy(), "hnd")
    np.testing.assert_array_equal(bits(kc), rk.view(np.int16))
    np.testing.assert_array_equal(bits(vc), rv.view(np.int16))
    o = ref.paged_prefill(m.q.numpy(), rk, rv, m.block_table.numpy(), m.token_to_seq.numpy(),
                          m.positions.numpy(), m.scale, layout="hnd")
    got = out_buf[out_off // 2:].view(T, Hq, D).cpu().numpy()
    assert max_abs(got, o) <= ATOL


def test_kv_write_encode_prefill_with_rope():
    """RoPE of Q and K fused with the slot scatter equals EngineRoPE.encode followed
    by KVWriteOp.encode_prefill (the reference's two dispatches)."""
    from vllm_apple_b200.engine import EngineRoPE, KVWriteOp
    from vllm_apple_b200.workloads import make_mixed_case
    m = make_mixed_case(seed=8, num_chunks=2, chunk=64, prior=(0, 500), num_decode=4,
                        decode_len=(20, 600))
    ctx = _ctx()
    rope = EngineRoPE(ctx, m.D, m.Hq, m.Hkv, max_position=4096, base=1e6)
    kvw = KVWriteOp(ctx, m.Hkv, m.D, m.bs)
    T = m.num_tokens
    # fused
    buf, qo, ko, vo = _planar(m.q, m.k, m.v)
    kc, vc = m.k_cache.cuda(), m.v_cache.cuda()
    with ctx.new_step(step_kind="prefill", num_tokens=T) as sc:
        kvw.encode_prefill_with_rope(sc, rope, buf, buf, buf, kc, vc, m.slot_mapping.cuda(),
                                     m.positions.cuda(), T, query_offset=qo, new_keys_offset=ko,
                                     new_values_offset=vo)
        sc.submit()
        sc.wait_until_completed()
    # two dispatches
    buf2, qo2, ko2, vo2 = _planar(m.q, m.k, m.v)
    kc2, vc2 = m.k_cache.cuda(), m.v_cache.cuda()
    from vllm_apple_b200.engine.context import EngineTensor
    q2 = EngineTensor(buf2, (T, m.Hq, m.D), offset=qo2)
    k2 = EngineTensor(buf2, (T, m.Hkv, m.D), offset=ko2)
    with ctx.new_step(step_kind="prefill", num_tokens=T) as sc:
        rope.encode(sc, q2, k2, m.positions.cuda(), T,
                    max_position_in_batch=int(m.positions.max()))
        sc.memory_barrier()
        kvw.encode_prefill(sc, buf2, buf2, kc2, vc2, m.slot_mapping.cuda(), T,
                           new_keys_offset=ko2, new_values_offset=vo2)
        sc.submit()
        sc.wait_until_completed()
    assert torch.equal(buf, buf2)
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)
    # and both equal the oracle: fp32 RoPE formula then scatter
    cos, sin = ref.rope_cos_sin_cache(m.D, 4096, 1e6)
    eq, ek = ref.rope(m.q.numpy(), m.k.numpy(), cos, sin, m.positions.numpy())
    ek16 = ek.astype(np.float32).astype(np.float16)
    np.testing.assert_array_equal(_plane(buf, qo, (T, m.Hq, m.D)).cpu().numpy(),
                                  eq.astype(np.float32).astype(np.float16))
    rk, rv = m.k_cache.numpy().copy(), m.v_cache.numpy().copy()
    ref.kv_write_slots_vectorized(rk, rv, ek16, m.v.numpy(), m.slot_mapping.numpy(), "hnd")
    np.testing.assert_array_equal(bits(kc), rk.view(np.int16))
    np.testing.assert_array_equal(bits(vc), rv.view(np.int16))


@pytest.mark.parametrize("residual", [False, True])
def test_engine_rmsnorm_encode(residual):
    from vllm_apple_b200.engine import EngineRMSNorm
    from vllm_apple_b200.engine.context import EngineTensor
    ctx = _ctx()
    g = torch.Generator().manual_seed(11)
    T, H = 37, 5120
    x = torch.randn(T, H, generator=g).half()
    w = (1 + 0.02 * torch.randn(H, generator=g)).half()
    r = torch.randn(T, H, generator=g).half()
    norm = EngineRMSNorm(ctx, H, eps=1e-5)
    with pytest.raises(RuntimeError, match="set_weights"):
        with ctx.new_step() as sc:
            norm.encode(sc, x.cuda(), torch.empty_like(x).cuda(), T)
    # weights and input as views at byte offsets into engine buffers
    wbuf = torch.zeros(256 + H * 2, dtype=torch.uint8, device="cuda")
    wbuf[256:].view(torch.float16).copy_(w.cuda())
    norm.set_weights(EngineTensor(wbuf, (H,), offset=256))
    xbuf = torch.zeros(1024 + T * H * 2, dtype=torch.uint8, device="cuda")
    xbuf[1024:].view(torch.float16).copy_(x.reshape(-1).cuda())
    out = torch.empty(T, H, dtype=torch.float16, device="cuda")
    with ctx.new_step() as sc:
        norm.encode(sc, EngineTensor(xbuf, (T, H), offset=1024), out, T,
                    residual_buffer=r.cuda() if residual else None)
        sc.submit()
        sc.wait_until_completed()
    exp = ref.rmsnorm(x.numpy(), w.numpy(), 1e-5, r.numpy() if residual else None)
    assert max_abs(out.cpu().numpy(), exp) <= ATOL
    assert norm.get_output_size(T) == T * H * 2


def test_engine_rope_encode_and_bound_check():
    from vllm_apple_b200.engine import EngineRoPE
    ctx = _ctx()
    g = torch.Generator().manual_seed(12)
    T, Hq, Hkv, D = 300, 32, 8, 128
    q = torch.randn(T, Hq, D, generator=g).half()
    k = torch.randn(T, Hkv, D, generator=g).half()
    pos = torch.randint(0, 32768, (T,), generator=g).to(torch.int32)
    rope = EngineRoPE(ctx, D, Hq, Hkv, max_position=32768, base=1e6)
    dq, dk = q.cuda(), k.cuda()
    with ctx.new_step() as sc:
        rope.encode(sc, dq, dk, pos.cuda(), T, max_position_in_batch=int(pos.max()))
        sc.submit()
        sc.wait_until_completed()
    cos, sin = ref.rope_cos_sin_cache(D, 32768, 1e6)
    eq, ek = ref.rope(q.numpy(), k.numpy(), cos, sin, pos.numpy())
    np.testing.assert_array_equal(dq.cpu().numpy(), eq.astype(np.float32).astype(np.float16))
    np.testing.assert_array_equal(dk.cpu().numpy(), ek.astype(np.float32).astype(np.float16))
    # the reference's host-side range check (elementwise.py:729-733): position ids
    # must stay below max_position; nothing is encoded when it fails
    before = dq.clone()
    with ctx.new_step() as sc:
        with pytest.raises(ValueError, match="exceeds max_position"):
            rope.encode(sc, dq, dk, pos.cuda(), T, max_position_in_batch=32768)
    torch.cuda.synchronize()
    assert torch.equal(dq, before)
    with pytest.raises(RuntimeError, match="outside ENCODE"):
        rope.encode(ctx.new_step(), dq, dk, pos.cuda(), T)


def test_engine_silu_mul_encode():
    from vllm_apple_b200.engine import EngineElementwiseOps
    from vllm_apple_b200.engine.context import EngineTensor
    ctx = _ctx()
    g = torch.Generator().manual_seed(13)
    T, I = 64, 32768
    gate = torch.randn(T, I, generator=g).half()
    up = torch.randn(T, I, generator=g).half()
    # gate and up as the two halves of one gate_up buffer (the merged projection)
    gu = torch.cat([gate.reshape(-1), up.reshape(-1)]).cuda()
    n = T * I
    out = torch.empty(n, dtype=torch.float16, device="cuda")
    ew = EngineElementwiseOps(ctx)
    with ctx.new_step() as sc:
        ew.encode_silu_mul(sc, EngineTensor(gu, (n,), offset=0),
                           EngineTensor(gu, (n,), offset=n * 2), out, n)
        sc.submit()
        sc.wait_until_completed()
    exp = ref.silu_mul(gate.numpy().reshape(-1), up.numpy().reshape(-1))
    got = out.cpu().numpy()
    assert int(ulp_distance_fp16(got, exp).max()) <= 1
    small = np.abs(exp) < 4
    assert max_abs(got[small], exp[small]) <= ATOL
