"""World-size-2 run of the sequence-sharded decode path on CPU (gloo): each rank
computes its LPT shard with the oracle, outputs are all-gathered into batch
order, and the result equals the single-process batch."""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, result_dir):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "vllm-apple_b200")]
    from oracle import paged_attention as ref
    from vllm_apple_b200.sharding import ShardPlan, gather_outputs
    from vllm_apple_b200.workloads import make_decode_case

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    full = make_decode_case("qwen_b4", seed=0, batch=9)
    plan = ShardPlan(full.seq_lens.tolist(), world)
    mine = plan.shards[rank]
    case = make_decode_case("qwen_b4", seed=0, batch=9, seq_subset=mine,
                            lengths=full.seq_lens.long())
    # every rank owns only its sequences' pages; no exchange during attention
    kc, vc = case.k_cache.numpy().copy(), case.v_cache.numpy().copy()
    ref.kv_write_decode(kc, vc, case.new_k.numpy(), case.new_v.numpy(), case.block_table.numpy(),
                        case.seq_lens.numpy())
    local = ref.paged_decode(case.q.numpy(), kc, vc, case.block_table.numpy(),
                             case.seq_lens.numpy(), case.scale)
    # timing aggregation as bench.py does it: max over ranks
    t = torch.tensor([float(rank + 1)], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    assert t.item() == world
    gathered = gather_outputs(torch.from_numpy(local), plan, rank)
    np.save(os.path.join(result_dir, f"r{rank}.npy"), gathered.numpy())
    np.save(os.path.join(result_dir, f"q{rank}.npy"), case.q.numpy())
    dist.destroy_process_group()


def test_two_rank_sharded_decode(tmp_path):
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    a = np.load(tmp_path / "r0.npy")
    b = np.load(tmp_path / "r1.npy")
    assert np.array_equal(a, b)
    assert a.shape == (9, 14, 64) and np.isfinite(a).all()
    # each row equals the single-process oracle on that sequence's own inputs
    from oracle import paged_attention as ref
    from vllm_apple_b200.sharding import ShardPlan
    from vllm_apple_b200.workloads import make_decode_case
    full = make_decode_case("qwen_b4", seed=0, batch=9)
    plan = ShardPlan(full.seq_lens.tolist(), world)
    for r, shard in enumerate(plan.shards):
        case = make_decode_case("qwen_b4", seed=0, batch=9, seq_subset=shard,
                                lengths=full.seq_lens.long())
        kc, vc = case.k_cache.numpy().copy(), case.v_cache.numpy().copy()
        ref.kv_write_decode(kc, vc, case.new_k.numpy(), case.new_v.numpy(),
                            case.block_table.numpy(), case.seq_lens.numpy())
        o = ref.paged_decode(case.q.numpy(), kc, vc, case.block_table.numpy(),
                             case.seq_lens.numpy(), case.scale)
        assert np.array_equal(a[shard], o)
