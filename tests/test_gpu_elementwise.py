"""RMSNorm, RoPE and SiLU-mul on the GPU vs the oracle (config-5 shapes)."""
import numpy as np
import pytest
import torch

from _util import ATOL, max_abs, np16, ulp_distance_fp16
from oracle import paged_attention as ref

pytestmark = pytest.mark.gpu


def _ops():
    from vllm_apple_b200 import ops
    return ops


@pytest.mark.parametrize("T,H", [(8192, 5120), (7, 896), (5, 130), (3, 9000)])
@pytest.mark.parametrize("residual", [False, True])
def test_rmsnorm(T, H, residual):
    ops = _ops()
    g = torch.Generator().manual_seed(T + H)
    x = torch.randn(T, H, generator=g).half()
    w = (1 + 0.02 * torch.randn(H, generator=g)).half()
    r = torch.randn(T, H, generator=g).half() if residual else None
    out = torch.empty(T, H, dtype=torch.float16, device="cuda")
    ops.rmsnorm(out, x.cuda(), w.cuda(), 1e-5, residual=None if r is None else r.cuda())
    exp = ref.rmsnorm(x.numpy(), w.numpy(), 1e-5, None if r is None else r.numpy())
    assert max_abs(np16(out), exp) <= ATOL


@pytest.mark.parametrize("neox", [True, False])
@pytest.mark.parametrize("T,Hq,Hkv,D,rot,theta,maxpos",
                         [(8192, 32, 8, 128, 128, 1e6, 32768), (16, 14, 2, 64, 64, 1e4, 64),
                          (33, 4, 1, 128, 64, 1e4, 2048), (9, 3, 1, 40, 40, 1e4, 512)])
def test_rope(neox, T, Hq, Hkv, D, rot, theta, maxpos):
    ops = _ops()
    g = torch.Generator().manual_seed(T + D)
    q = torch.randn(T, Hq, D, generator=g).half()
    k = torch.randn(T, Hkv, D, generator=g).half()
    pos = torch.randint(0, maxpos, (T,), generator=g).to(torch.int32)
    cos, sin = ref.rope_cos_sin_cache(rot, maxpos, theta)
    dq, dk = q.cuda(), k.cuda()
    ops.rope(dq, dk, torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda(), pos.cuda(),
             rotary_dim=rot, is_neox=neox)
    eq, ek = ref.rope(q.numpy(), k.numpy(), cos, sin, pos.numpy(), rot, is_neox=neox)
    # same fp32 operations as the oracle: the fp16 results are the oracle's fp32 rounded once
    np.testing.assert_array_equal(np16(dq), eq.astype(np.float32).astype(np.float16))
    np.testing.assert_array_equal(np16(dk), ek.astype(np.float32).astype(np.float16))
    assert max_abs(np16(dq), eq) <= ATOL


def test_rope_bad_position_flagged_and_untouched():
    ops = _ops()
    q = torch.randn(4, 2, 64).half().cuda()
    k = torch.randn(4, 1, 64).half().cuda()
    q0, k0 = q.clone(), k.clone()
    cos, sin = ref.rope_cos_sin_cache(64, 16, 1e4)
    pos = torch.tensor([0, 16, -1, 3], dtype=torch.int32, device="cuda")
    ops.rope(q, k, torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda(), pos)
    assert ops.check_device_errors(raise_on_error=False) & 0x10
    assert torch.equal(q[1], q0[1]) and torch.equal(q[2], q0[2]) and torch.equal(k[1], k0[1])


@pytest.mark.parametrize("n", [8192 * 4096, 1000, 13])
def test_silu_mul(n):
    ops = _ops()
    g = torch.Generator().manual_seed(n % 1000)
    gate = torch.randn(n, generator=g).half()
    up = torch.randn(n, generator=g).half()
    out = torch.empty(n, dtype=torch.float16, device="cuda")
    ops.silu_mul(out, gate.cuda(), up.cuda())
    got = np16(out)
    exp = ref.silu_mul(gate.numpy(), up.numpy())
    ulps = ulp_distance_fp16(got, exp)
    assert int(ulps.max()) <= 1
    small = np.abs(exp) < 4
    assert max_abs(got[small], exp[small]) <= ATOL
