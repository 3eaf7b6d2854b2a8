#!/usr/bin/env python3
"""Benchmark of the paged-attention decode step (fused KV write + attention).

Workload: the 22B-shaped decode of the benchmark configuration -- 32 query /
8 KV heads, head_size 128, block_size 16, context lengths log-normal (median
2048, sigma 0.6) clipped to [512, 8192] -- at batch 1024, sharded by sequence
(greedy LPT on context length) across the N GPUs: total work is fixed, so
scaling is "strong".  A step = one fused decode over the rank's shard, inputs
resident in HBM (KV pool >> L2, so no L2 flush is needed).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  (N > 1: launched by torch.distributed.run, one rank per GPU, NCCL)

value = aggregate algorithmic HBM GB/s over all ranks (bytes a perfect kernel
must move per step / max-over-ranks step time); also reported: seq-tokens/s.
e2e = the same metric through the engine op API (PagedAttentionOp
.encode_decode_fused) with per-step H2D copies of q/new K/new V/block table/
seq_lens from pinned host memory and a D2H copy of the output.
--impl reference times the reference's own CPU path -- the unmodified
MPSAttentionImpl.forward installed in baseline/_ref (KV scatter + per-sequence
gather + GQA repeat + SDPA) -- on the host cores on a bounded sample of the
same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "vllm-apple_b200"))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

WORKLOAD = "devstral_b1024"  # default; --workload selects another decode config
METRIC = "paged-attn decode HBM GB/s (algorithmic bytes)"
GLOBAL_BATCH = 1024
UNIT = "GB/s"


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# DRAM bytes (read + write) per decode launch over its algorithmic bytes, from one
# ncu capture (dram__bytes_read.sum + dram__bytes_write.sum of one launch of the
# devstral_b128 decode, longest first and unsplit: 1.2933 GB read + 3.6 MB written
# for 1.2910 GB algorithmic; 1.3 GB of KV, well above L2); the traffic reported
# for a launch is this ratio times that launch's algorithmic bytes (traffic grows
# with the KV bytes read, which the algorithmic bytes count once).
DECODE_TRAFFIC_RATIO = 1.0046
DECODE_TRAFFIC_CAPTURE = "ncu, devstral_b128 decode, one launch, scaled by algorithmic bytes"


class ClockSampler:
    """nvidia-smi clock/throttle sampling while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,"
         "clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            # nvidia-smi takes a moment to start; samples must cover the timed region,
            # which for short runs (many GPUs, few steps) lasts only tens of ms
            time.sleep(0.5)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()
        return False

    def summary(self):
        rows = []
        for line in (self.out or "").strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 10:
                continue
            try:
                rows.append(dict(sm=float(f[1]), smax=float(f[2]), util=float(f[4]),
                                 hw=f[6], hwt=f[7], swt=f[8], pcap=f[9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        load = [r for r in rows if r["util"] > 0] or rows
        reasons = set()
        for r in load:
            for k, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"),
                            ("swt", "sw_thermal_slowdown"), ("pcap", "sw_power_cap")):
                if r[k].lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in load),
                "sm_max_mhz": max(r["smax"] for r in rows), "reasons": sorted(reasons),
                "samples": len(load)}


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus and world > 1:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    return world, rank, local


def global_lengths():
    from vllm_apple_b200.workloads import DECODE_CONFIGS, draw_lengths
    c = DECODE_CONFIGS[WORKLOAD]
    global GLOBAL_BATCH
    GLOBAL_BATCH = c["batch"]
    gen = torch.Generator().manual_seed(0)
    return draw_lengths(c["dist"], c["batch"], gen)


def run_ours(args, world, rank, local):
    from vllm_apple_b200 import ops
    from vllm_apple_b200.engine import EngineContext, PagedAttentionOp
    from vllm_apple_b200.workloads import lpt_shard, make_decode_case

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
        pg = dist
    L_all = global_lengths()
    shards = lpt_shard(L_all.tolist(), world)
    case = make_decode_case(WORKLOAD, device=dev, seed=0, seq_subset=shards[rank],
                            lengths=L_all)
    B = case.batch
    q, nk, nv = case.q.to(dev), case.new_k.to(dev), case.new_v.to(dev)
    bt, sl = case.block_table.to(dev), case.seq_lens.to(dev)
    out = torch.empty_like(q)
    max_len = case.max_seq_len
    lib_ws = ops._lib.load().va_paged_decode_workspace_size(B, case.Hq, case.Hkv, case.D,
                                                            case.bs, max_len)
    launches_per_step = 2 if lib_ws else 1  # split kernel (+ combine when any can split)

    def step():
        ops.paged_decode(out, q, case.k_cache, case.v_cache, bt, sl, scale=case.scale,
                         max_seq_len=max_len, new_k=nk, new_v=nv, layout="hnd")

    stream = torch.cuda.current_stream(dev)

    def barrier():
        if pg is not None:
            pg.barrier()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    ops.check_device_errors(local)

    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        torch.cuda.synchronize(dev)
        t0.record(stream)
        for _ in range(args.steps):
            step()
        t1.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
    ms_local = t0.elapsed_time(t1)
    ops.check_device_errors(local)

    # ---- NCCL all-gather of the outputs into batch order (not part of the step) ----
    gather = time_gather(args, L_all, world, rank, out, dev, stream, barrier) if pg else None

    # ---- e2e through the engine op API with host buffers ----
    if args.no_e2e:
        e2e_ms_local, h2d, d2h = 0.0, 0, 0
    else:
        e2e_ms_local, h2d, d2h = run_e2e(args, case, local, dev, stream, barrier, q, nk, nv, bt,
                                         sl, out, max_len)
    return finish(args, world, rank, pg, case, ms_local, e2e_ms_local, h2d, d2h,
                  launches_per_step, clk, dev, gather)


def time_gather(args, L_all, world, rank, out, dev, stream, barrier):
    """Device time of ``sharding.OutputGather`` (one NCCL all-gather of every rank's
    [shard, Hq, D] fp16 output + the reorder into batch order), CUDA events on the
    compute stream, max over ranks; checked once against the expected rows."""
    from vllm_apple_b200.sharding import OutputGather, ShardPlan
    plan = ShardPlan(L_all.tolist(), world)
    g = OutputGather(plan, out.shape[1:], out.dtype, dev)
    full = g(out)
    torch.cuda.synchronize(dev)
    mine = torch.as_tensor(plan.shards[rank], device=dev)
    assert torch.equal(full[mine], out), "gathered rows differ from this rank's output"
    n = max(10, min(args.steps, 100))
    for _ in range(3):
        g(out)
    barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(n):
        g(out)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    return {"ms_local": e0.elapsed_time(e1) / n, "bytes_per_rank": g.bytes_per_rank,
            "out_bytes": full.numel() * full.element_size(), "iters": n}


def run_e2e(args, case, local, dev, stream, barrier, q, nk, nv, bt, sl, out, max_len):
    """Steps through the engine op API with host buffers.  Every step copies its
    inputs H2D from pinned memory and its output D2H; the copies run on a copy
    stream, double-buffered, so step i's copies overlap step i-1's kernel (as a
    serving loop does).  Timed on the compute stream from the first H2D to the
    last D2H."""
    from vllm_apple_b200 import ops
    from vllm_apple_b200.engine import EngineContext, PagedAttentionOp
    B = case.batch
    ctx = EngineContext(local)
    op = PagedAttentionOp(ctx, case.Hkv, case.Hq, case.D, case.bs, case.scale)
    host_in = [t.pin_memory() for t in (case.q, case.new_k, case.new_v, case.block_table,
                                         case.seq_lens)]
    host_out = [torch.empty(case.q.shape, dtype=torch.float16).pin_memory() for _ in range(2)]
    dev_in = [[torch.empty_like(t, device=dev) for t in host_in] for _ in range(2)]
    dev_out = [torch.empty_like(out) for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in host_in)
    d2h = host_out[0].numel() * host_out[0].element_size()
    h2d_s, d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    h2d_done = [torch.cuda.Event() for _ in range(2)]
    comp_done = [torch.cuda.Event() for _ in range(2)]
    d2h_done = [torch.cuda.Event() for _ in range(2)]

    def issue_h2d(i):
        b = i & 1
        h2d_s.wait_event(comp_done[b])        # step i-2 no longer reads these inputs
        with torch.cuda.stream(h2d_s):
            for d, h in zip(dev_in[b], host_in):
                d.copy_(h, non_blocking=True)
        h2d_done[b].record(h2d_s)

    def compute(i):
        b = i & 1
        stream.wait_event(h2d_done[b])
        stream.wait_event(d2h_done[b])        # step i-2's output has been read back
        d_q, d_nk, d_nv, d_bt, d_sl = dev_in[b]
        with ctx.new_step(step_kind="decode", num_seqs=B) as sc:
            op.encode_decode_fused(sc, d_q, d_nk, d_nv, case.k_cache, case.v_cache, d_bt, d_sl,
                                   dev_out[b], B, max_len, max_blocks_per_seq=d_bt.shape[1])
        comp_done[b].record(stream)

    def issue_d2h(i):
        b = i & 1
        d2h_s.wait_event(comp_done[b])
        with torch.cuda.stream(d2h_s):
            host_out[b].copy_(dev_out[b], non_blocking=True)
        d2h_done[b].record(d2h_s)

    def run(n):
        issue_h2d(0)
        for i in range(n):
            compute(i)
            if i + 1 < n:
                issue_h2d(i + 1)
            issue_d2h(i)

    run(max(3, args.warmup // 4))
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(dev)
    e2e_steps = max(2, min(args.steps, 100))
    e0.record(stream)
    h2d_s.wait_event(e0)  # the first copy starts inside the timed region
    run(e2e_steps)
    stream.wait_stream(d2h_s)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms_local = e0.elapsed_time(e1) / e2e_steps
    ops.check_device_errors(local)
    # the last step's output really came back
    assert torch.equal(host_out[(e2e_steps - 1) & 1], dev_out[(e2e_steps - 1) & 1].cpu())
    return e2e_ms_local, h2d, d2h


def finish(args, world, rank, pg, case, ms_local, e2e_ms_local, h2d, d2h, launches_per_step,
           clk, dev, gather=None):
    # ---- aggregate over ranks ----
    local_bytes = case.algorithmic_bytes()
    local_tokens = case.context_tokens
    vec = torch.tensor([ms_local / args.steps, e2e_ms_local], dtype=torch.float64, device=dev)
    tot = torch.tensor([float(local_bytes), float(local_tokens)], dtype=torch.float64, device=dev)
    if pg is not None:
        pg.all_reduce(vec, op=pg.ReduceOp.MAX)
        pg.all_reduce(tot, op=pg.ReduceOp.SUM)
    ms_step, e2e_ms = vec.tolist()
    gather_ms = None
    if gather is not None:
        gv = torch.tensor([gather["ms_local"]], dtype=torch.float64, device=dev)
        pg.all_reduce(gv, op=pg.ReduceOp.MAX)
        gather_ms = float(gv.item())
    all_bytes, all_tokens = tot.tolist()
    if rank != 0:
        if pg is not None:
            pg.destroy_process_group()
        return None

    value = all_bytes / (ms_step * 1e-3) / 1e9
    peak, peak_kind = peaks()
    # roofline of the dominant kernel on this rank (the step is that kernel plus a
    # small split combine): algorithmic bytes per launch / mean step time
    achieved = local_bytes / (ms_local / args.steps * 1e-3) / 1e9
    traffic = int(round(local_bytes * DECODE_TRAFFIC_RATIO))
    res = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic (seeded N(0,1) fp16 q/k/v, log-normal lengths)",
        "config": {"workload": WORKLOAD + "_decode", "global_batch": GLOBAL_BATCH,
                   "Hq": case.Hq, "Hkv": case.Hkv, "head_size": case.D, "block_size": case.bs,
                   "ctx": str(case.meta["dist"]),
                   "context_tokens": int(all_tokens), "sharding": "LPT by context length",
                   "layout": "engine [nb,Hkv,bs,D]",
                   "l2": "inputs larger than L2 (no flush)", "parallelism": f"seq-shard x{world}"},
        "seq_tokens_per_s": round(all_tokens / (ms_step * 1e-3), 1),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": traffic, "traffic_source": DECODE_TRAFFIC_CAPTURE,
                     "algorithmic_bytes_per_launch": int(local_bytes)},
        "e2e": None if args.no_e2e else {
            "value": round(all_bytes / (e2e_ms * 1e-3) / 1e9, 1), "unit": UNIT,
            "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h), "api": "engine PagedAttentionOp.encode_decode_fused",
            "copies": "pinned H2D and D2H every step on two copy streams, double-buffered"},
        "gpu_launches": args.steps * launches_per_step,
        "clocks": clk.summary(),
    }
    if gather_ms is not None:
        # bus bandwidth of an all-gather: (world - 1) / world of the gathered bytes
        # cross each rank's links
        out_b = gather["bytes_per_rank"] * world
        res["output_gather"] = {
            "op": "sharding.OutputGather: NCCL all_gather_into_tensor + reorder",
            "ms": round(gather_ms, 4), "bytes_gathered": int(out_b),
            "busbw_GBps": round(out_b * (world - 1) / world / (gather_ms * 1e-3) / 1e9, 1),
            "iters": gather["iters"], "timing": "CUDA events, max over ranks",
            "in_step": False}
    if world == 1 and args.cpu_budget > 0:
        res["cpu_baseline"] = cpu_baseline(budget_s=args.cpu_budget)
    if pg is not None:
        pg.destroy_process_group()
    return res


def cpu_sample_case(n_seqs: int):
    from vllm_apple_b200.workloads import make_decode_case
    L_all = global_lengths()
    return make_decode_case(WORKLOAD, device="cpu", seed=0, layout="nhd",
                            seq_subset=list(range(n_seqs)), lengths=L_all)


def reference_decode_fn(case):
    """One decode step of the reference's own CPU path on ``case`` (vLLM layout).

    Preferred: the UNMODIFIED reference installed in baseline/_ref --
    ``MPSAttentionImpl.forward`` (vllm_apple/v1/attention/backends/mps_attn.py:207-357
    with base_attn.py), imported through oracle/reference_loader.py.  Fallback,
    only when that install is missing: its restatement oracle/mps_port.py
    (golden-pinned to the reference's outputs).  Returns (fn, kind, what)."""
    kv = torch.stack([case.k_cache, case.v_cache])
    B = case.batch
    out = torch.empty_like(case.q)
    try:
        from oracle.reference_loader import load_reference_attention
        mps = load_reference_attention()
    except Exception as e:  # noqa: BLE001  (fallback is labelled in the output)
        mps, why = None, f"{type(e).__name__}: {e}"
    if mps is not None:
        meta = mps.MPSAttentionMetadata(
            num_actual_tokens=B, max_query_len=1,
            query_start_loc=torch.arange(B + 1, dtype=torch.int32), max_seq_len=case.max_seq_len,
            seq_lens=case.seq_lens.clone(), block_table=case.block_table.to(torch.int64),
            slot_mapping=case.slot_mapping, scheduler_metadata=None, causal=True,
            num_decode_tokens=B)
        impl = mps.MPSAttentionImpl(num_heads=case.Hq, head_size=case.D, scale=case.scale,
                                    num_kv_heads=case.Hkv, alibi_slopes=None,
                                    sliding_window=None, kv_cache_dtype="auto")

        def one():
            impl.forward(None, case.q, case.new_k, case.new_v, kv, meta, out)
        return one, "reference", ("unmodified reference MPSAttentionImpl.forward from "
                                  "baseline/_ref (torch CPU, fp16, vLLM layout)")
    from oracle import mps_port
    slots = case.slot_mapping
    qsl = list(range(B + 1))
    bt = case.block_table.to(torch.int64)

    def one():
        mps_port.forward(case.q, case.new_k, case.new_v, kv, bt, case.seq_lens.tolist(), slots,
                         qsl, B, case.scale, case.Hkv, out)
    return one, "port", f"oracle/mps_port.py restatement (baseline/_ref unavailable: {why})"


def cpu_time_sample(case, reps_budget_s: float, fn=None):
    """Time one reference CPU decode step on `case`; returns (seconds per pass, passes)."""
    one = fn or reference_decode_fn(case)[0]
    one()  # warm-up
    times = []
    t_end = time.perf_counter() + reps_budget_s
    while True:
        t = time.perf_counter()
        one()
        times.append(time.perf_counter() - t)
        if time.perf_counter() > t_end or len(times) >= 5:
            break
    return min(times), len(times)


def cpu_baseline(budget_s: float = 15.0, n_seqs: int = 48):
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    case = cpu_sample_case(n_seqs)
    fn, kind, what = reference_decode_fn(case)
    sec, n = cpu_time_sample(case, budget_s, fn)
    return {"value": round(case.algorithmic_bytes() / sec / 1e9, 3), "unit": UNIT,
            "cores": torch.get_num_threads(), "kind": kind,
            "sample": f"first {n_seqs} of the {WORKLOAD} sequences ({case.context_tokens} "
                      f"context tokens), {what}, best of {n} passes",
            "seq_tokens_per_s": round(case.context_tokens / sec, 1)}


def run_reference(args, world, rank):
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    n_seqs = 48
    case = cpu_sample_case(n_seqs)
    fn, kind, what = reference_decode_fn(case)
    for _ in range(args.warmup):
        fn()
    times = []
    for _ in range(args.steps):
        t = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t)
    sec = statistics.median(times)
    value = case.algorithmic_bytes() / sec / 1e9
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": WORKLOAD + "_decode", "global_batch": GLOBAL_BATCH,
                   "sample_seqs": n_seqs, "context_tokens": case.context_tokens},
        "seq_tokens_per_s": round(case.context_tokens / sec, 1),
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT,
                         "cores": torch.get_num_threads(), "kind": kind,
                         "sample": f"first {n_seqs} of {WORKLOAD} sequences per step "
                                   f"(median of {args.steps}), {what}"},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


# ---------------------------------------------------------------------------
# the other hot-path rows (one GPU): --row mixed | rmsnorm | rope | silu_mul | topk
# ---------------------------------------------------------------------------
ROWS = ("decode", "mixed", "rmsnorm", "rope", "silu_mul", "topk")


def tensor_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured (cuBLAS bf16 burst)"
    return 1590.0, "fallback"


L2_BYTES = 126 * 1024 * 1024


def time_rotating(fn, steps, warmup):
    """Device time (ms) of `steps` back-to-back calls of fn (CUDA events around
    the whole loop on the current stream).  fn rotates over input/output sets
    whose total exceeds L2 several times, so every call reads its inputs from
    HBM without an L2 flush between calls."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1)


def rotate(calls):
    """A zero-argument step that runs calls[0], calls[1], ... in turn."""
    state = {"i": 0}

    def step():
        i = state["i"]
        state["i"] = (i + 1) % len(calls)
        calls[i]()
    return step


def n_sets(set_bytes: int) -> int:
    """Input/output sets needed for a working set of >= 3x L2 across calls."""
    return max(1, -(-3 * L2_BYTES // max(set_bytes, 1)))


def cpu_time(fn, budget_s):
    fn()
    times, t_end = [], time.perf_counter() + budget_s
    while True:
        t = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t)
        if time.perf_counter() > t_end or len(times) >= 5:
            return min(times), len(times)


def row_case(row, dev):
    """(step fn, algorithmic bytes, flops or None, launches per step, config, cpu leg)
    of one row at its BASELINE shape; the cpu leg times the oracle restatement of the
    reference on a bounded sample and returns (value, unit, sample text)."""
    from vllm_apple_b200 import ops
    from vllm_apple_b200.workloads import make_elementwise_case, make_mixed_case
    from oracle import paged_attention as ref
    if row == "mixed":
        m = make_mixed_case(device=dev, seed=0)
        q, k, v = m.q.to(dev), m.k.to(dev), m.v.to(dev)
        bt, ts, ps, sm = (m.block_table.to(dev), m.token_to_seq.to(dev), m.positions.to(dev),
                          m.slot_mapping.to(dev))
        out = torch.empty_like(q)

        def step():
            ops.kv_write_slots(m.k_cache, m.v_cache, k, v, sm)
            ops.paged_prefill(out, q, m.k_cache, m.v_cache, bt, ts, ps, scale=m.scale)

        pos = m.positions.long()
        flops = 4 * m.Hq * m.D * int((pos + 1).sum())
        ctx = [int(pos[m.token_to_seq.long() == s].max()) + 1 for s in range(len(m.seq_lens))]
        nbytes = (sum(ctx) * m.Hkv * m.D * 4 + m.num_tokens * (m.Hq + 2 * m.Hkv) * m.D * 2
                  + m.num_tokens * m.Hq * m.D * 2 + m.num_tokens * m.Hkv * m.D * 4)
        cfg = {"workload": "mixed_22b", "tokens": m.num_tokens, "prefill_chunks": "4 x 512",
               "prior": "U[0,4096]", "decode_rows": m.num_decode_tokens, "Hq": m.Hq,
               "Hkv": m.Hkv, "head_size": m.D, "block_size": m.bs}

        def cpu(budget):
            c = make_mixed_case(device="cpu", seed=0, num_chunks=1, chunk=64, prior=(0, 512),
                                num_decode=4, decode_len=(256, 1024))
            kc, vc = c.k_cache.numpy().copy(), c.v_cache.numpy().copy()

            def one():
                ref.kv_write_slots_vectorized(kc, vc, c.k.numpy(), c.v.numpy(),
                                              c.slot_mapping.numpy(), c.layout)
                ref.paged_prefill(c.q.numpy(), kc, vc, c.block_table.numpy(),
                                  c.token_to_seq.numpy(), c.positions.numpy(), c.scale,
                                  layout=c.layout)
            sec, n = cpu_time(one, budget)
            f = 4 * c.Hq * c.D * int((c.positions.long() + 1).sum())
            return f / sec / 1e12, "TFLOP/s", (f"1 chunk of 64 tokens over <=512 prior + 4 decode "
                                               f"rows (numpy float64), best of {n}")
        return step, nbytes, flops, 5, cfg, cpu
    e = make_elementwise_case(device=dev, seed=0)
    T, H = e.x.shape
    if row == "rmsnorm":
        nbytes = 2 * T * H * 2 + H * 2
        sets = [(e.x if i == 0 else e.x.clone(), torch.empty_like(e.x))
                for i in range(n_sets(nbytes))]
        step = rotate([lambda x=x, o=o: ops.rmsnorm(o, x, e.w, e.eps) for x, o in sets])
        cfg = {"workload": "rmsnorm_8192x5120", "eps": e.eps, "sets": len(sets)}

        def cpu(budget):
            n = 512
            x, w = e.x[:n].cpu().numpy(), e.w.cpu().numpy()
            sec, k = cpu_time(lambda: ref.rmsnorm(x, w, e.eps), budget)
            return 2 * n * H * 2 / sec / 1e9, "GB/s", f"first {n} tokens (numpy), best of {k}"
        return step, nbytes, None, 1, cfg, cpu
    if row == "rope":
        c, sn = ref.rope_cos_sin_cache(e.q.shape[2], e.max_position, e.theta)
        cd, sd = torch.from_numpy(c).to(dev), torch.from_numpy(sn).to(dev)
        nel = T * (e.q.shape[1] + e.k.shape[1]) * e.q.shape[2]
        nbytes = 2 * nel * 2 + T * 4
        sets = [(e.q, e.k) if i == 0 else (e.q.clone(), e.k.clone())
                for i in range(n_sets(nbytes))]
        step = rotate([lambda q=q, k=k: ops.rope(q, k, cd, sd, e.positions) for q, k in sets])
        cfg = {"workload": "rope_neox_8192", "theta": e.theta, "Hq": e.q.shape[1],
               "Hkv": e.k.shape[1], "head_size": e.q.shape[2], "sets": len(sets),
               "note": "cos/sin table (L2-resident) excluded from bytes"}

        def cpu(budget):
            n = 256
            q, k, p = e.q[:n].cpu().numpy(), e.k[:n].cpu().numpy(), e.positions[:n].cpu().numpy()
            sec, m = cpu_time(lambda: ref.rope(q, k, c, sn, p), budget)
            b = 2 * n * (e.q.shape[1] + e.k.shape[1]) * e.q.shape[2] * 2
            return b / sec / 1e9, "GB/s", f"first {n} tokens (numpy), best of {m}"
        return step, nbytes, None, 1, cfg, cpu
    if row == "silu_mul":
        out = torch.empty_like(e.gate)
        step = lambda: ops.silu_mul(out, e.gate, e.up)  # noqa: E731
        nbytes = 3 * e.gate.numel() * 2
        cfg = {"workload": "silu_mul_8192x32768"}

        def cpu(budget):
            n = 64
            g, u = e.gate[:n].cpu().numpy(), e.up[:n].cpu().numpy()
            sec, m = cpu_time(lambda: ref.silu_mul(g, u), budget)
            return 3 * g.size * 2 / sec / 1e9, "GB/s", f"first {n} tokens (numpy), best of {m}"
        return step, nbytes, None, 1, cfg, cpu
    if row == "topk":
        g = torch.Generator().manual_seed(0)
        Tk, V, k = 1024, 131072, 50
        x = (torch.randn(Tk, V, generator=g) * 3).half()
        nbytes = Tk * V * 2 + Tk * k * 6
        xds = [x.to(dev) for _ in range(n_sets(nbytes))]
        idx = torch.empty(Tk, k, dtype=torch.int32, device=dev)
        val = torch.empty(Tk, k, dtype=torch.float16, device=dev)
        step = rotate([lambda xd=xd: ops.topk(idx, val, xd, k) for xd in xds])
        cfg = {"workload": "topk_1024x131072", "k": k, "sets": len(xds)}

        def cpu(budget):
            n = 8
            xs = x[:n].numpy()
            sec, m = cpu_time(lambda: ref.topk(xs, k), budget)
            return (n * V * 2 + n * k * 6) / sec / 1e9, "GB/s", f"first {n} rows (numpy), best of {m}"
        return step, nbytes, None, 1, cfg, cpu
    raise ValueError(row)


def run_row(args, rank, local):
    if rank != 0:
        return None
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from vllm_apple_b200 import ops
    step, nbytes, flops, launches, cfg, cpu = row_case(args.row, dev)
    # enough calls that the timed region lasts >= 0.8 s and so spans many clock
    # samples (taken 20 ms apart)
    est = time_rotating(step, 20, args.warmup) / 20
    args.steps = max(args.steps, int(800.0 / max(est, 1e-3)) + 1)
    with ClockSampler(local) as clk:
        ms = time_rotating(step, args.steps, args.warmup)
    ops.check_device_errors(local)
    ms_step = ms / args.steps
    gbs = nbytes / (ms_step * 1e-3) / 1e9
    hbm, hbm_kind = peaks()
    if flops is not None:
        tf = flops / (ms_step * 1e-3) / 1e12
        tpk, tkind = tensor_peak()
        metric, value, unit = "mixed-batch step TFLOP/s (causal prefill FLOPs)", tf, "TFLOP/s"
        # the step's own lower bound: its HBM bytes at the HBM peak and its FLOPs at the
        # tensor peak can overlap at best, so the slower of the two bounds the step
        t_hbm, t_tc = nbytes / (hbm * 1e9) * 1e6, flops / (tpk * 1e12) * 1e6
        roof = {"bound": "tensor", "achieved": round(tf, 2), "peak": tpk, "unit": "TFLOP/s",
                "frac": round(tf / tpk, 4), "peak_kind": tkind, "traffic": None,
                "note": "whole step (KV scatter, planner, tiles and decode rows); the decode "
                        "rows are HBM-bound: GB/s below",
                "step_bound_us": {"hbm": round(t_hbm, 1), "tensor": round(t_tc, 1),
                                  "frac_of_measured": round(max(t_hbm, t_tc) / (ms_step * 1e3),
                                                            4)}}
    else:
        metric, value, unit = f"{args.row} HBM GB/s (algorithmic bytes)", gbs, "GB/s"
        roof = {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(gbs / hbm, 4), "peak_kind": hbm_kind, "traffic": None,
                "algorithmic_bytes_per_launch": int(nbytes)}
    res = {"metric": metric, "value": round(value, 2), "unit": unit, "n_gpus": 1,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
           "data": "synthetic (seeded N(0,1) fp16, BASELINE shapes)",
           "config": dict(cfg, l2="inputs larger than L2: calls rotate over input/output sets "
                                  "totalling >= 3x L2 (no flush)"),
           "GBps": round(gbs, 1), "roofline": roof, "gpu_launches": args.steps * launches,
           "clocks": clk.summary()}
    if args.cpu_budget > 0:
        v, u, sample = cpu(args.cpu_budget)
        res["cpu_baseline"] = {"value": round(v, 4), "unit": u, "cores": 1, "kind": "port",
                               "sample": sample + "; numpy oracle restatement of the "
                                         "reference's CPU formula, one thread"}
    return res


def main():
    global WORKLOAD
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-budget", type=float, default=15.0,
                    help="seconds of CPU-baseline timing (0 skips it)")
    ap.add_argument("--workload", default=WORKLOAD,
                    help="decode config of vllm_apple_b200.workloads (default: %(default)s)")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end leg")
    ap.add_argument("--row", choices=ROWS, default="decode",
                    help="hot-path row to measure (default: the headline decode step)")
    args = ap.parse_args()
    WORKLOAD = args.workload
    if args.warmup < 3:
        args.warmup = 3
    world, rank, local = dist_setup(args.gpus)
    if args.impl == "reference":
        res = run_reference(args, world, rank)
    elif args.row != "decode":
        res = run_row(args, rank, local)
    else:
        res = run_ours(args, world, rank, local)
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
