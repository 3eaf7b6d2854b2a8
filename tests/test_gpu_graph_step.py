"""A decode step captured into a CUDA graph replays the eager result, and picks
up new inputs copied into its fixed buffers."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_captured_decode_step_replays_eager_result():
    from vllm_apple_b200.engine import EngineContext, PagedAttentionOp
    from vllm_apple_b200.engine.context import CapturedStep, EngineStepContext
    from vllm_apple_b200.workloads import make_decode_case
    ctx = EngineContext(0)
    c = make_decode_case("devstral_b128", seed=3, batch=16)
    op = PagedAttentionOp(ctx, c.Hkv, c.Hq, c.D, c.bs, 1 / math.sqrt(c.D))
    kc, vc = c.k_cache.cuda(), c.v_cache.cuda()
    q, nk, nv = c.q.cuda(), c.new_k.cuda(), c.new_v.cuda()
    bt, sl = c.block_table.cuda(), c.seq_lens.cuda()
    out = torch.zeros_like(q)
    max_len = c.max_seq_len

    def encode(sc):
        op.encode_decode_fused(sc, q, nk, nv, kc, vc, bt, sl, out, c.batch, max_len,
                               max_blocks_per_seq=bt.shape[1])

    with EngineStepContext(ctx) as sc:
        encode(sc)
    torch.cuda.synchronize()
    eager = out.clone()
    step = CapturedStep(ctx, encode)
    out.zero_()
    step.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    # next step: new queries in the same buffer
    q.copy_(torch.randn_like(q))
    with EngineStepContext(ctx) as sc:
        encode(sc)
    torch.cuda.synchronize()
    eager2 = out.clone()
    out.zero_()
    step.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager2) and not torch.equal(eager2, eager)
