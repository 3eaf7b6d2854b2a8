"""Per-op device timing of the hot-path kernels on the benchmark shapes.

  python -m vllm_apple_b200.perf --op {decode,mixed,prefill,rmsnorm,rope,silu_mul,topk,all}
                                 [--workload devstral_b128] [--iters 50] [--warmup 5]

Each op runs ``warmup`` untimed then ``iters`` timed launches bracketed by CUDA
events on the launching stream; inputs are larger than L2 (126 MB).  Prints one
JSON line per op: time, algorithmic bytes (and FLOPs for the tensor-core
prefill), achieved GB/s / TFLOP/s and the fraction of the measured HBM peak.
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path

import torch

from . import ops
from .engine.ops import rope_cos_sin_cache
from .workloads import make_decode_case, make_elementwise_case, make_mixed_case


def _peak_gbs() -> float:
    p = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"])
    return 6650.0


def _time(fn, iters, warmup) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(s)
    for _ in range(iters):
        fn()
    b.record(s)
    torch.cuda.synchronize()
    ops.check_device_errors()
    return a.elapsed_time(b) / iters * 1e-3


def _time_graph(fn, iters, warmup) -> float:
    """Device time per call with host launch overhead removed: `iters` calls captured
    in one CUDA graph, replayed."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()  # warm the capture stream (workspaces, side streams)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(iters):
            fn()
    g.replay()
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(s)
    g.replay()
    b.record(s)
    torch.cuda.synchronize()
    ops.check_device_errors()
    return a.elapsed_time(b) / iters * 1e-3


def _report(op, sec, nbytes, flops=None, **extra):
    peak = _peak_gbs()
    r = {"op": op, "us": round(sec * 1e6, 2), "bytes": int(nbytes),
         "GBps": round(nbytes / sec / 1e9, 1), "hbm_frac": round(nbytes / sec / 1e9 / peak, 4)}
    if flops:
        r["flops"] = int(flops)
        r["TFLOPs"] = round(flops / sec / 1e12, 1)
    r.update(extra)
    print(json.dumps(r), flush=True)


def run_decode(workload, iters, warmup, graph=False):
    c = make_decode_case(workload, device="cuda", seed=0)
    q, nk, nv = c.q.cuda(), c.new_k.cuda(), c.new_v.cuda()
    bt, sl = c.block_table.cuda(), c.seq_lens.cuda()
    out = torch.empty_like(q)
    timer = _time_graph if graph else _time
    sec = timer(lambda: ops.paged_decode(out, q, c.k_cache, c.v_cache, bt, sl, scale=c.scale,
                                         max_seq_len=c.max_seq_len, new_k=nk, new_v=nv),
                iters, warmup)
    _report("decode", sec, c.algorithmic_bytes(), workload=workload,
            seq_tokens_per_s=round(c.context_tokens / sec, 1),
            timing="CUDA graph replay" if graph else "back-to-back launches")


def run_mixed(iters, warmup, prefill_only=False, head_size=128):
    kw = {} if head_size == 128 else dict(Hq=14, Hkv=2, D=64)
    if prefill_only:
        kw["num_decode"] = 0
    m = make_mixed_case(device="cuda", seed=0, **kw)
    q, k, v = m.q.cuda(), m.k.cuda(), m.v.cuda()
    bt, ts, ps, sm = (m.block_table.cuda(), m.token_to_seq.cuda(), m.positions.cuda(),
                      m.slot_mapping.cuda())
    out = torch.empty_like(q)

    def step():
        ops.kv_write_slots(m.k_cache, m.v_cache, k, v, sm)
        ops.paged_prefill(out, q, m.k_cache, m.v_cache, bt, ts, ps, scale=m.scale)

    sec = _time(step, iters, warmup)
    pos = m.positions.long()
    Hkv, Hq, D = m.Hkv, m.Hq, m.D
    flops = 4 * Hq * D * int((pos + 1).sum())
    ctx = [int(pos[m.token_to_seq.long() == s].max()) + 1 for s in range(len(m.seq_lens))]
    nbytes = (sum(ctx) * Hkv * D * 4 + m.num_tokens * (Hq + 2 * Hkv) * D * 2
              + m.num_tokens * Hq * D * 2 + m.num_tokens * Hkv * D * 4)
    _report("prefill" if prefill_only else "mixed", sec, nbytes, flops, tokens=m.num_tokens,
            head_size=m.D)


def run_elementwise(which, iters, warmup):
    e = make_elementwise_case(device="cuda", seed=0)
    T, H = e.x.shape
    if which in ("rmsnorm", "all"):
        out = torch.empty_like(e.x)
        sec = _time(lambda: ops.rmsnorm(out, e.x, e.w, e.eps), iters, warmup)
        _report("rmsnorm", sec, 2 * T * H * 2 + H * 2, shape=[T, H])
    if which in ("rope", "all"):
        c, s = rope_cos_sin_cache(e.q.shape[2], e.max_position, e.theta)
        c, s = torch.from_numpy(c).cuda(), torch.from_numpy(s).cuda()
        sec = _time(lambda: ops.rope(e.q, e.k, c, s, e.positions), iters, warmup)
        n = T * (e.q.shape[1] + e.k.shape[1]) * e.q.shape[2]
        _report("rope", sec, 2 * n * 2 + T * 4, note="cos/sin table (16 MB, L2) excluded")
    if which in ("silu_mul", "all"):
        out = torch.empty_like(e.gate)
        sec = _time(lambda: ops.silu_mul(out, e.gate, e.up), iters, warmup)
        _report("silu_mul", sec, 3 * e.gate.numel() * 2, shape=list(e.gate.shape))


def run_topk(iters, warmup):
    """Top-k over a decode batch's logits: 1024 rows x 131072 vocab (268 MB, above
    L2), k = 50 (the reference's default)."""
    g = torch.Generator().manual_seed(0)
    T, V, k = 1024, 131072, 50
    x = (torch.randn(T, V, generator=g) * 3).half().cuda()
    idx = torch.empty(T, k, dtype=torch.int32, device="cuda")
    val = torch.empty(T, k, dtype=torch.float16, device="cuda")
    sec = _time(lambda: ops.topk(idx, val, x, k), iters, warmup)
    _report("topk", sec, T * V * 2 + T * k * 6, shape=[T, V], k=k)
    # a decode batch's worth of rows (fewer rows than SMs, one CTA per row)
    T2 = 64
    x2, i2, v2 = x[:T2].contiguous(), idx[:T2].contiguous(), val[:T2].contiguous()
    sec = _time(lambda: ops.topk(i2, v2, x2, k), iters, warmup)
    _report("topk", sec, T2 * V * 2 + T2 * k * 6, shape=[T2, V], k=k)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", default="all",
                    choices=["decode", "mixed", "prefill", "rmsnorm", "rope", "silu_mul", "topk",
                             "all"])
    ap.add_argument("--head-size", type=int, default=128, choices=[64, 128],
                    help="mixed / prefill: 22B shape (128) or Qwen shape (64)")
    ap.add_argument("--workload", default="devstral_b128")
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--graph", action="store_true",
                    help="decode: time a CUDA graph of the calls (no host launch overhead)")
    a = ap.parse_args()
    torch.cuda.set_device(0)
    if a.op in ("decode", "all"):
        run_decode(a.workload, a.iters, a.warmup, a.graph)
    if a.op in ("mixed", "all"):
        run_mixed(a.iters, a.warmup, head_size=a.head_size)
    if a.op in ("prefill", "all"):
        run_mixed(a.iters, a.warmup, prefill_only=True, head_size=a.head_size)
    if a.op in ("rmsnorm", "rope", "silu_mul", "all"):
        run_elementwise(a.op, a.iters, a.warmup)
    if a.op in ("topk", "all"):
        run_topk(a.iters, a.warmup)


if __name__ == "__main__":
    main()
