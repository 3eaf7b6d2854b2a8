"""Top-k logits on the GPU vs the oracle: indices and values bit-exact."""
import numpy as np
import pytest
import torch

from oracle import paged_attention as ref

pytestmark = pytest.mark.gpu


def _ops():
    from vllm_apple_b200 import ops
    return ops


def _logits(seed, T, V, special):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(T, V, generator=g) * 3).half()
    if special:
        x[0, torch.randint(0, V, (7,), generator=g)] = float("nan")
        x[0, torch.randint(0, V, (7,), generator=g)] = float("-inf")
        x[0, torch.randint(0, V, (2,), generator=g)] = float("inf")
        if T > 1:
            x[1] = 0.25                                  # one long tie
        if T > 2:
            x[2, : V // 2] = float("-inf")               # few valid logits
            x[2, V // 2:] = float("nan")
            x[2, V - 1] = -0.0
            x[2, V - 2] = 0.0
    return x


def _check(x, k, stride=None):
    ops = _ops()
    T, V = x.shape
    if stride is None:
        dx = x.cuda()
    else:
        buf = torch.full((T, stride), float("nan"), dtype=torch.float16)
        buf[:, :V] = x
        dx = buf.cuda()[:, :V]
    idx = torch.empty(T, k, dtype=torch.int32, device="cuda")
    val = torch.empty(T, k, dtype=torch.float16, device="cuda")
    ops.topk(idx, val, dx, k)
    ei, ev = ref.topk(x.numpy(), k)
    np.testing.assert_array_equal(idx.cpu().numpy(), ei)
    np.testing.assert_array_equal(val.cpu().view(torch.int16).numpy(), ev.view(np.int16))


@pytest.mark.parametrize("T,V,k", [(64, 32000, 50), (8, 151936, 8), (3, 131072, 1024),
                                   (5, 1000, 1), (4, 7, 3), (2, 9, 16), (300, 4096, 64)])
@pytest.mark.parametrize("special", [False, True])
def test_topk(T, V, k, special):
    _check(_logits(T * 7 + V + k, T, V, special), k)


@pytest.mark.parametrize("stride", [32003, 32008])
def test_topk_row_stride(stride):
    _check(_logits(stride, 6, 32000, True), 40, stride=stride)


def test_topk_fp16_range_extremes():
    x = torch.tensor([[65504.0, -65504.0, 6e-8, -6e-8, 0.0, -0.0, 1.0, 1.0]]).half()
    _check(x, 8)
    _check(x, 3)


def test_topk_engine_op():
    from vllm_apple_b200.engine import EngineContext, EngineTopK
    ctx = EngineContext()
    op = EngineTopK(ctx, k=50)
    assert op.k == 50 and op.get_stats() == {"k": 50}
    x = _logits(1, 16, 32000, False)
    dx = x.cuda()
    idx = torch.empty(16, 50, dtype=torch.int32, device="cuda")
    val = torch.empty(16, 50, dtype=torch.float16, device="cuda")
    with ctx.new_step() as sc:
        op.encode(sc, dx, idx, val, 16, 32000)
        sc.submit()
        sc.wait_until_completed()
    ei, ev = ref.topk(x.numpy(), 50)
    np.testing.assert_array_equal(idx.cpu().numpy(), ei)
    np.testing.assert_array_equal(val.cpu().numpy(), ev)


def test_topk_rejects():
    from vllm_apple_b200 import _lib
    lib = _lib.load()
    x = torch.zeros(2, 100, dtype=torch.float16, device="cuda")
    i = torch.empty(2, 2048, dtype=torch.int32, device="cuda")
    v = torch.empty(2, 2048, dtype=torch.float16, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert lib.va_topk(i.data_ptr(), v.data_ptr(), x.data_ptr(), 2, 100, 100, 0, s) == 1
    assert lib.va_topk(i.data_ptr(), v.data_ptr(), x.data_ptr(), 2, 100, 99, 5, s) == 1
    assert lib.va_topk(i.data_ptr(), v.data_ptr(), x.data_ptr(), 2, 100, 100, 1025, s) == 2
    assert lib.va_topk(i.data_ptr(), v.data_ptr(), x.data_ptr(), 0, 100, 100, 5, s) == 0


@pytest.mark.parametrize("T,V,k", [(1, 151936, 50), (8, 131072, 50), (16, 32000, 8),
                                   (40, 131072, 256), (3, 4100, 20), (64, 262144, 100)])
@pytest.mark.parametrize("special", [False, True])
def test_topk_few_rows(T, V, k, special):
    """Few rows (a decode batch): one CTA per whole row, no workspace; through the
    workspace entry point with a workspace given anyway, the same results."""
    from vllm_apple_b200 import _lib
    lib = _lib.load()
    assert lib.va_topk_workspace_size(T, V, k) == 0
    x = _logits(T * 11 + V + k, T, V, special)
    _check(x, k)
    dx = x.cuda()
    idx = torch.empty(T, k, dtype=torch.int32, device="cuda")
    val = torch.empty(T, k, dtype=torch.float16, device="cuda")
    junk = torch.empty(1 << 20, dtype=torch.uint8, device="cuda")
    _lib.check(lib.va_topk_ws(idx.data_ptr(), val.data_ptr(), dx.data_ptr(), T, V, V, k,
                              junk.data_ptr(), junk.numel(),
                              torch.cuda.current_stream().cuda_stream), "va_topk_ws")
    ei, ev = ref.topk(x.numpy(), k)
    np.testing.assert_array_equal(idx.cpu().numpy(), ei)
    np.testing.assert_array_equal(val.cpu().view(torch.int16).numpy(), ev.view(np.int16))


@pytest.mark.parametrize("T,V,k", [(32, 32000, 50), (4, 151936, 256), (1024, 131072, 50)])
def test_topk_matches_torch_topk_on_distinct_values(T, V, k):
    """Independent of the oracle: on rows whose values are all distinct (a random
    permutation of distinct fp16 values), the selection is unique, so indices and
    values must equal torch.topk's (sorted, largest first)."""
    ops = _ops()
    g = torch.Generator().manual_seed(T + V + k)
    # 2^15 - 2048 distinct finite fp16 values, each row a random draw without repeats
    pool = torch.arange(-30000, 30000, dtype=torch.int32)
    vals = pool.to(torch.int16).view(torch.float16)
    vals = vals[torch.isfinite(vals)]
    vals = torch.unique(vals.float()).half()
    assert vals.numel() >= min(V, 28000)
    rows = []
    for _ in range(T):
        pick = torch.randperm(vals.numel(), generator=g)[:min(V, vals.numel())]
        r = vals[pick]
        if V > r.numel():  # pad with -inf (never selected)
            r = torch.cat([r, torch.full((V - r.numel(),), float("-inf"), dtype=torch.float16)])
        rows.append(r)
    x = torch.stack(rows)
    dx = x.cuda()
    idx = torch.empty(T, k, dtype=torch.int32, device="cuda")
    val = torch.empty(T, k, dtype=torch.float16, device="cuda")
    ops.topk(idx, val, dx, k)
    tv, ti = torch.topk(dx.float(), k, dim=1, largest=True, sorted=True)
    assert torch.equal(idx.long(), ti)
    assert torch.equal(val.float(), tv)


@pytest.mark.parametrize("V", [131072, 24581, 100000])
def test_topk_many_rows_edge_rows(V):
    """Many rows (more than SMs: one CTA per row) including the rows that leave the
    bound-and-screen path: a row of equal values (candidate overflow), a row whose
    first logits are all -inf, NaN / -inf / +inf, ascending values, and (with a
    padded row stride) a ragged tail of fewer than 8 logits; also through the
    no-workspace entry point."""
    T, k = 200, 64
    x = _logits(V + 5, T, V, special=True)
    x[3] = torch.arange(V, dtype=torch.float32).div(V / 60000.0).sub(30000).half()  # ascending
    x[4, :9000] = float("-inf")                       # a long -inf prefix
    x[5] = 1.5                                        # all equal
    _check(x, k, stride=None if V % 8 == 0 else V + 8 - V % 8)  # aligned rows, ragged tail
    # the no-workspace entry point
    ops = _ops()
    from vllm_apple_b200 import _lib
    xs = x[:7].contiguous()
    dx = xs.cuda()
    idx = torch.empty(7, k, dtype=torch.int32, device="cuda")
    val = torch.empty(7, k, dtype=torch.float16, device="cuda")
    _lib.check(_lib.load().va_topk(idx.data_ptr(), val.data_ptr(), dx.data_ptr(), 7, V, V, k,
                                   torch.cuda.current_stream().cuda_stream), "va_topk")
    ei, ev = ref.topk(xs.numpy(), k)
    np.testing.assert_array_equal(idx.cpu().numpy(), ei)
    np.testing.assert_array_equal(val.cpu().view(torch.int16).numpy(), ev.view(np.int16))


@pytest.mark.parametrize("seed", range(6))
def test_topk_random_tie_heavy(seed):
    """Seeded random shapes (V not a multiple of 8, odd row strides, k up to 512 and
    beyond) over logits drawn from a small set of values, so that ties at the bound,
    candidate lists longer than k and overflows into the exact path all occur; bit
    for bit against the oracle."""
    g = torch.Generator().manual_seed(1234 + seed)
    for _ in range(4):
        T = int(torch.randint(1, 300, (1,), generator=g))
        V = int(torch.randint(9, 40000, (1,), generator=g))
        k = int(torch.randint(1, 600, (1,), generator=g))
        levels = int(torch.randint(2, 200, (1,), generator=g))
        x = (torch.randint(0, levels, (T, V), generator=g).float() / 7 - 3).half()
        if seed % 2:
            x[:, torch.randint(0, V, (V // 50 + 1,), generator=g)] = float("nan")
        stride = None if seed % 3 else V + int(torch.randint(0, 16, (1,), generator=g))
        _check(x, k, stride=stride)
