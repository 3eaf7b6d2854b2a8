"""Host-side logic: workload generators, sharding, engine validation rules,
engine tensor views and step phases (no GPU)."""
import numpy as np
import pytest
import torch

from vllm_apple_b200 import workloads as w
from vllm_apple_b200.sharding import ShardPlan, lpt_partition


@pytest.mark.parametrize("config", list(w.DECODE_CONFIGS))
def test_decode_case_metadata_consistent(config):
    c = w.DECODE_CONFIGS[config]
    gen = torch.Generator().manual_seed(0)
    L = w.draw_lengths(c["dist"], c["batch"], gen)
    kind = c["dist"][0]
    lo, hi = (c["dist"][1], c["dist"][2]) if kind == "uniform" else (c["dist"][3], c["dist"][4])
    assert int(L.min()) >= lo and int(L.max()) <= hi
    bt, nb = w.assign_blocks(L.tolist(), 16, c["pool"], gen)
    need = ((L + 15) // 16).tolist()
    used = np.concatenate([bt[i, :n].numpy() for i, n in enumerate(need)])
    assert len(np.unique(used)) == len(used), "blocks must be disjoint"
    assert used.max() < nb and nb >= max(c["pool"], 1)
    for i, n in enumerate(need):
        assert np.all(bt[i, n:].numpy() == -1)


def test_lognormal_median_and_slots():
    c = w.make_decode_case("qwen_b4", seed=0)
    Lm1 = c.seq_lens.long() - 1
    blk = c.block_table[torch.arange(c.batch), Lm1 // 16].long()
    assert torch.equal(c.slot_mapping, blk * 16 + Lm1 % 16)
    gen = torch.Generator().manual_seed(0)
    L = w.draw_lengths(("lognormal", 2048, 0.6, 512, 8192), 20000, gen)
    assert 1900 < float(L.median()) < 2200


def test_algorithmic_bytes_formula():
    c = w.make_decode_case("devstral_b128", seed=0, batch=4)
    B, Hq, Hkv, D = 4, 32, 8, 128
    pages = int(((c.seq_lens.long() + 15) // 16).sum())
    expect = (c.context_tokens * Hkv * D * 4 + B * Hq * D * 4 + B * Hkv * D * 8 + pages * 4
              + B * 4)
    assert c.algorithmic_bytes() == expect
    assert c.context_tokens * Hkv * D * 4 / c.context_tokens == 4096  # 4 KiB / token at 22B


def test_mixed_case_layout():
    m = w.make_mixed_case(seed=0)
    assert m.num_tokens == 4 * 512 + 60
    assert m.num_decode_tokens == 60
    # decode rows first, each at position seq_len-1
    assert torch.equal(m.positions[:60].long(), m.seq_lens[:60].long() - 1)
    # slots consistent with block table and positions
    blk = m.block_table[m.token_to_seq.long(), m.positions.long() // 16].long()
    assert torch.equal(m.slot_mapping, blk * 16 + m.positions.long() % 16)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_lpt_partition_balanced_and_complete(world):
    gen = torch.Generator().manual_seed(0)
    L = w.draw_lengths(("lognormal", 2048, 0.6, 512, 8192), 1024, gen).tolist()
    plan = ShardPlan(L, world)
    flat = sorted(i for s in plan.shards for i in s)
    assert flat == list(range(1024))
    assert plan.imbalance < 1.01
    assert lpt_partition(L, world) == plan.shards  # deterministic


def test_kv_cache_validation_rules():
    """Mirror of the reference's slot/block rules (tests/unit/test_engine.py:343-420):
    -1 is padding, anything below raises, anything at/over capacity raises."""
    from vllm_apple_b200.engine.kv_cache import EngineKVCache, KVCacheDescriptor

    class Ctx:
        device = torch.device("cpu")

    kv = EngineKVCache(Ctx(), KVCacheDescriptor(num_blocks=4, block_size=16, num_kv_heads=2,
                                                head_size=8))
    kv.validate_slot_mapping(torch.tensor([-1, 0, 63]))
    with pytest.raises(ValueError, match="> max valid slot"):
        kv.validate_slot_mapping(torch.tensor([64]))
    with pytest.raises(ValueError, match="invalid index -2"):
        kv.validate_slot_mapping(torch.tensor([3, -2]))
    kv.validate_block_table(torch.tensor([[0, 3, -1]]))
    with pytest.raises(ValueError, match=">= num_blocks"):
        kv.validate_block_table(torch.tensor([[4]]))
    with pytest.raises(ValueError, match="invalid index"):
        kv.validate_block_table(torch.tensor([[1, -5]]))
    assert kv.strides == {"block": 2 * 16 * 8, "head": 16 * 8, "token": 8}


def test_engine_tensor_view_bounds():
    from vllm_apple_b200.engine.context import EngineTensor, resolve
    buf = torch.zeros(1024, dtype=torch.uint8)
    t = EngineTensor(buf, (4, 8), torch.float16, offset=256)
    assert t.nbytes == 64 and t.as_torch().shape == (4, 8)
    with pytest.raises(ValueError):
        EngineTensor(buf, (1024,), torch.float16, offset=0)
    with pytest.raises(RuntimeError):
        resolve(buf)  # host buffers are refused: no CPU fallback


def test_step_phases():
    from vllm_apple_b200.engine.context import EngineStepContext

    class Ctx:
        device = torch.device("cpu")

    sc = EngineStepContext(Ctx(), 0)
    with pytest.raises(RuntimeError, match="outside ENCODE"):
        sc.require_encoding("encode()")
    with pytest.raises(RuntimeError):
        sc.wait_until_completed()
    with sc:
        assert sc.is_encoding
        sc.memory_barrier()
    assert not sc.is_encoding


def test_bridge_constructors_mirror_the_reference():
    """Bridge classes keep the reference's constructor checks and attributes
    (metal_paged_attention_v2.py:37-60, metal_paged_attention_fused.py:98-157)."""
    import pytest as _pytest
    from vllm_apple_b200.bridge import MetalPagedAttentionFused, MetalPagedAttentionV2
    with _pytest.raises(ValueError):
        MetalPagedAttentionV2(2, 14, 80, 16, 0.1)
    v2 = MetalPagedAttentionV2(2, 14, 64, 16, 0.125)
    assert v2.queries_per_kv == 7 and v2.max_num_blocks == 256
    f = MetalPagedAttentionFused(8, 32, 128, 16)
    assert abs(f.scale - 128 ** -0.5) < 1e-12 and f.is_fused_available and f.queries_per_kv == 4


def test_bench_row_cpu_legs_run_on_the_host():
    """The CPU baselines beside each bench row (oracle restatements on a sample) run
    without a GPU and report positive throughput in the row's unit."""
    import sys as _sys
    import os as _os
    import torch as _torch
    _sys.path.insert(0, _os.path.dirname(_os.path.dirname(__file__)))
    import bench
    for row, unit in (("topk", "GB/s"),):  # (the elementwise cases are 1.6 GB to build)
        _step, nbytes, flops, launches, cfg, cpu = bench.row_case(row, _torch.device("cpu"))
        v, u, sample = cpu(0.05)
        assert v > 0 and u == unit and nbytes > 0 and launches == 1 and "workload" in cfg
