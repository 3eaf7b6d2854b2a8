"""Parity of the exact configurations the benchmark times.

``bench.py`` times the fused decode (KV write + attention, engine layout) of
the 22B-shaped batch of 1024 sequences on one GPU, and the LPT shards of that
batch on 2, 4 and 8 GPUs (each rank builds its shard with
``make_decode_case(..., seq_subset=shard, lengths=L_all)``).  Each case runs
here exactly as the bench builds it (all of them large enough to run unsplit,
longest sequence first, through the on-device ordering):

* KV write: the whole K and V caches after the call equal the caches before
  it with the new rows written at ``seq_len - 1`` (bit-exact; every untouched
  byte is compared too);
* attention: a seeded sample of 64 sequences, all 32 heads, against the float64
  oracle (``oracle.paged_attention.paged_decode``, restating
  ``mps_attn.py:284-357``) at max-abs 2e-3.
"""
import numpy as np
import pytest
import torch

from _util import ATOL
from oracle import paged_attention as ref

pytestmark = pytest.mark.gpu

WORKLOAD = "devstral_b1024"
SAMPLE = 64


def _global_lengths():
    from vllm_apple_b200.workloads import DECODE_CONFIGS, draw_lengths
    c = DECODE_CONFIGS[WORKLOAD]
    return draw_lengths(c["dist"], c["batch"], torch.Generator().manual_seed(0))


def _expected_cache(cache_before, new_rows, bt, seq_lens, bs):
    """The cache after the decode write, built on the device by indexing."""
    exp = cache_before.clone()
    B = seq_lens.numel()
    pos = seq_lens.long() - 1
    blk = bt[torch.arange(B, device=bt.device), pos // bs].long()
    exp[blk, :, pos % bs, :] = new_rows  # engine layout [nb, Hkv, bs, D]
    return exp


def _oracle_sample(c, k_before, v_before, out, idx):
    """Oracle decode of the sequences ``idx``: their pages are gathered into a
    compact CPU cache (pre-write contents), the oracle KV write applied, then
    the oracle attention compared with the GPU output rows."""
    bs = c.bs
    bt = c.block_table[idx]
    sl = c.seq_lens[idx]
    npg = ((sl.long() + bs - 1) // bs)
    blocks = torch.cat([bt[i, :int(npg[i])] for i in range(len(idx))]).long()
    kc = k_before[blocks.to(k_before.device)].cpu().numpy()
    vc = v_before[blocks.to(v_before.device)].cpu().numpy()
    cbt = np.full(bt.shape, -1, np.int32)
    at = 0
    for i in range(len(idx)):
        n = int(npg[i])
        cbt[i, :n] = np.arange(at, at + n, dtype=np.int32)
        at += n
    nk, nv = c.new_k[idx].numpy(), c.new_v[idx].numpy()
    ref.kv_write_decode(kc, vc, nk, nv, cbt, sl.numpy(), layout="hnd")
    o = ref.paged_decode(c.q[idx].numpy(), kc, vc, cbt, sl.numpy(), c.scale, layout="hnd")
    got = out[torch.as_tensor(idx, device=out.device)].cpu().numpy().astype(np.float64)
    return float(np.abs(got - o).max())


def _run_shard(world, rank):
    from vllm_apple_b200 import ops
    from vllm_apple_b200.workloads import lpt_shard, make_decode_case
    dev = torch.device("cuda", 0)
    L_all = _global_lengths()
    shards = lpt_shard(L_all.tolist(), world)
    c = make_decode_case(WORKLOAD, device=dev, seed=0, seq_subset=shards[rank], lengths=L_all)
    q, nk, nv = c.q.to(dev), c.new_k.to(dev), c.new_v.to(dev)
    bt, sl = c.block_table.to(dev), c.seq_lens.to(dev)
    out = torch.full_like(q, 7.0)
    k_before, v_before = c.k_cache.clone(), c.v_cache.clone()
    ops.paged_decode(out, q, c.k_cache, c.v_cache, bt, sl, scale=c.scale,
                     max_seq_len=c.max_seq_len, new_k=nk, new_v=nv, layout="hnd")
    torch.cuda.synchronize()
    assert ops.check_device_errors(0, raise_on_error=False) == 0
    # whole-cache bit-exact check of the KV write
    exp_k = _expected_cache(k_before, nk, bt, sl, c.bs)
    assert torch.equal(c.k_cache.view(torch.int16), exp_k.view(torch.int16)), "K cache differs"
    del exp_k
    exp_v = _expected_cache(v_before, nv, bt, sl, c.bs)
    assert torch.equal(c.v_cache.view(torch.int16), exp_v.view(torch.int16)), "V cache differs"
    del exp_v
    # every output row was written (no row left at the fill value)
    assert not bool((out == 7.0).all(dim=2).all(dim=1).any())
    g = torch.Generator().manual_seed(1000 * world + rank)
    n = c.batch
    idx = sorted(torch.randperm(n, generator=g)[:min(SAMPLE, n)].tolist())
    # always include the longest sequence (most splits) of the shard
    longest = int(torch.argmax(c.seq_lens))
    if longest not in idx:
        idx[0] = longest
        idx.sort()
    err = _oracle_sample(c, k_before, v_before, out, idx)
    assert err <= ATOL, f"world {world} rank {rank}: max abs err {err}"
    return c.batch


def test_bench_config_full_batch():
    """The single-GPU bench step: 1024 sequences, one split each."""
    assert _run_shard(1, 0) == 1024


@pytest.mark.parametrize("world", [2, 4, 8])
def test_bench_config_lpt_shards(world):
    """Every rank's shard of the scaling bench, in turn on one GPU."""
    total = 0
    for rank in range(world):
        total += _run_shard(world, rank)
        torch.cuda.empty_cache()
    assert total == 1024
