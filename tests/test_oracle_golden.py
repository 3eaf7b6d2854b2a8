"""Pin the CPU oracle to the reference: golden vectors produced by running the
reference's own code (tests/golden/make_golden.py) must be reproduced."""
import ctypes
import hashlib
import os
import subprocess

import numpy as np
import pytest
import torch

from oracle import mps_port
from oracle import paged_attention as ref

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def load(name):
    return dict(np.load(os.path.join(GOLD, name)))


def test_decode_kv_scatter_bit_exact_to_reference():
    g = load("decode_qwen_b4.npz")
    kc, vc = g["cache_in"][0].copy(), g["cache_in"][1].copy()
    ref.kv_write_slots(kc, vc, g["k"], g["v"], g["slot_mapping"], layout="nhd")
    assert np.array_equal(kc.view(np.int16), g["cache_out"][0].view(np.int16))
    assert np.array_equal(vc.view(np.int16), g["cache_out"][1].view(np.int16))
    # the decode-position writer lands on the same bytes
    kc2, vc2 = g["cache_in"][0].copy(), g["cache_in"][1].copy()
    ref.kv_write_decode(kc2, vc2, g["k"], g["v"], g["block_table"], g["seq_lens"], layout="nhd")
    assert np.array_equal(kc2.view(np.int16), g["cache_out"][0].view(np.int16))


def test_decode_attention_matches_reference():
    g = load("decode_qwen_b4.npz")
    kc, vc = g["cache_out"][0], g["cache_out"][1]
    o = ref.paged_decode(g["q"], kc, vc, g["block_table"], g["seq_lens"], 1 / np.sqrt(64),
                         layout="nhd")
    assert np.max(np.abs(o - g["out"])) < 2e-5


def test_mixed_batch_decode_rows_match_reference():
    """Decode rows of a mixed batch (the reference misaligns the prefill rows of a
    mixed batch: mps_attn.py:263 with base_attn.py:249 -- see make_golden.py)."""
    g = load("mixed_noprior.npz")
    kc, vc = g["cache_in"][0].copy(), g["cache_in"][1].copy()
    ref.kv_write_slots(kc, vc, g["k"], g["v"], g["slot_mapping"], layout="nhd")
    o = ref.paged_prefill(g["q"], kc, vc, g["block_table"], g["token_to_seq"], g["positions"],
                          1 / np.sqrt(64), layout="nhd")
    nd = 2
    assert np.max(np.abs(o[:nd] - g["out"][:nd])) < 2e-5


def test_prefill_matches_reference_when_no_prior_context():
    g = load("prefill_noprior.npz")
    kc, vc = g["cache_in"][0].copy(), g["cache_in"][1].copy()
    ref.kv_write_slots(kc, vc, g["k"], g["v"], g["slot_mapping"], layout="nhd")
    assert np.array_equal(kc.view(np.int16), g["cache_out"][0].view(np.int16))
    o = ref.paged_prefill(g["q"], kc, vc, g["block_table"], g["token_to_seq"], g["positions"],
                          1 / np.sqrt(64), layout="nhd")
    assert np.max(np.abs(o - g["out"])) < 2e-5


def test_cpu_baseline_port_matches_reference():
    """The timed CPU baseline (oracle/mps_port.py) reproduces the reference output."""
    g = load("decode_qwen_b4.npz")
    kv = torch.from_numpy(g["cache_in"]).float()
    out = torch.zeros(g["q"].shape)
    B = g["q"].shape[0]
    mps_port.forward(torch.from_numpy(g["q"]).float(), torch.from_numpy(g["k"]).float(),
                     torch.from_numpy(g["v"]).float(), kv,
                     torch.from_numpy(g["block_table"]).long(), g["seq_lens"].tolist(),
                     torch.from_numpy(g["slot_mapping"]), list(range(B + 1)), B,
                     1 / np.sqrt(64), 2, out)
    assert torch.max(torch.abs(out - torch.from_numpy(g["out"]))) < 1e-6
    m = load("prefill_noprior.npz")
    kv = torch.from_numpy(m["cache_in"]).float()
    out = torch.zeros(m["q"].shape)
    mps_port.forward(torch.from_numpy(m["q"]).float(), torch.from_numpy(m["k"]).float(),
                     torch.from_numpy(m["v"]).float(), kv,
                     torch.from_numpy(m["block_table"]).long(), m["seq_lens"].tolist(),
                     torch.from_numpy(m["slot_mapping"]), m["query_start_loc"].tolist(), 0,
                     1 / np.sqrt(64), 4, out)
    assert torch.max(torch.abs(out - torch.from_numpy(m["out"]))) < 1e-6


def test_rope_tables_bit_exact_to_reference():
    g = load("rope_tables.npz")
    c, s = ref.rope_cos_sin_cache(64, 64, 1e4)
    assert np.array_equal(c, g["cos_64_64_1e4"]) and np.array_equal(s, g["sin_64_64_1e4"])
    c, s = ref.rope_cos_sin_cache(128, 32768, 1e6)
    assert hashlib.sha256(c.tobytes()).digest() == g["sha256_cos_128_32768_1e6"].tobytes()
    assert hashlib.sha256(s.tobytes()).digest() == g["sha256_sin_128_32768_1e6"].tobytes()


def test_product_rope_table_equals_reference():
    """The engine op uploads the same fp32 table as the reference engine."""
    from vllm_apple_b200.engine.ops import rope_cos_sin_cache
    g = load("rope_tables.npz")
    c, s = rope_cos_sin_cache(128, 32768, 1e6)
    assert hashlib.sha256(c.tobytes()).digest() == g["sha256_cos_128_32768_1e6"].tobytes()
    assert np.array_equal(s[[0, 1, 4095, 32767]], g["rows_sin_128_32768_1e6"])


def _kv_gold():
    g = load("kv_write_c.npz")
    nb, H, bs, D, T = (int(x) for x in g["dims"])
    return g, nb, H, bs, D, T


def test_write_kv_batch_restatement_matches_reference_c():
    g, nb, H, bs, D, T = _kv_gold()
    ko, vo = g["key_dst"].copy(), g["value_dst"].copy()
    ref.write_kv_batch(ko, vo, g["key_src"], g["value_src"], g["block_ids"], g["token_offsets"],
                       T, H, D, H * bs * D, bs * D, D)
    assert np.array_equal(ko, g["key_out"]) and np.array_equal(vo, g["value_out"])


def _oracle_c():
    so = os.path.join(ROOT, "oracle/_build/libkv_scatter_oracle.so")
    if not os.path.exists(so):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "all"], check=True)
    return ctypes.CDLL(so)


def test_c_oracle_matches_reference_c():
    g, nb, H, bs, D, T = _kv_gold()
    lib = _oracle_c()
    ko, vo = g["key_dst"].copy(), g["value_dst"].copy()
    slots = (g["block_ids"] * bs + g["token_offsets"]).astype(np.int64)
    P = ctypes.c_void_p
    I64 = ctypes.c_int64
    lib.oracle_kv_write_slots(P(ko.ctypes.data), P(vo.ctypes.data), P(g["key_src"].ctypes.data),
                              P(g["value_src"].ctypes.data), P(slots.ctypes.data), I64(T), H, D,
                              bs, I64(nb), I64(H * bs * D), I64(bs * D), I64(D), I64(H * D),
                              I64(D))
    assert np.array_equal(ko, g["key_out"]) and np.array_equal(vo, g["value_out"])


def test_live_reference_c_when_built():
    """When oracle/_ref holds the reference's compiled kv_write.c, run it live
    against the numpy restatement on fresh random inputs."""
    so = os.path.join(ROOT, "oracle/_ref/libkv_write_ref.so")
    if not os.path.exists(so):
        pytest.skip("reference kv_write.c not built here")
    lib = ctypes.CDLL(so)
    rng = np.random.default_rng(7)
    nb, H, bs, D, T = 9, 2, 16, 64, 31
    kd = rng.integers(0, 65535, nb * H * bs * D, dtype=np.uint16)
    vd = kd[::-1].copy()
    ks = rng.integers(0, 65535, T * H * D, dtype=np.uint16)
    vs = ks[::-1].copy()
    sl = rng.permutation(nb * bs)[:T]
    blk, off = (sl // bs).astype(np.int64), (sl % bs).astype(np.int64)
    a_k, a_v, b_k, b_v = kd.copy(), vd.copy(), kd.copy(), vd.copy()
    P = ctypes.c_void_p
    lib.metal_write_kv_batch(P(a_k.ctypes.data), P(a_v.ctypes.data), P(ks.ctypes.data),
                             P(vs.ctypes.data), P(blk.ctypes.data), P(off.ctypes.data), T, H, D,
                             H * bs * D, bs * D, D)
    ref.write_kv_batch(b_k, b_v, ks, vs, blk, off, T, H, D, H * bs * D, bs * D, D)
    assert np.array_equal(a_k, b_k) and np.array_equal(a_v, b_v)


def test_rmsnorm_and_silu_match_reference_tests():
    g = load("norm_silu.npz")
    y = ref.rmsnorm(g["x"], g["w"], 1e-6)
    assert np.max(np.abs(y - g["rms"])) < 1e-5
    s = ref.silu_mul(g["gate"], g["up"])
    assert np.max(np.abs(s - g["silu_mul"])) < 1e-5


def test_oracle_self_check_against_plain_softmax():
    """float64 oracle vs an independent plain softmax(QK^T)V in torch fp64."""
    rng = np.random.default_rng(3)
    nb, H, bs, D, G = 20, 2, 16, 32, 3
    kc = rng.standard_normal((nb, H, bs, D)).astype(np.float16)
    vc = rng.standard_normal((nb, H, bs, D)).astype(np.float16)
    bt = rng.permutation(nb)[:12].reshape(2, 6).astype(np.int32)
    L = np.array([90, 41], np.int32)
    q = rng.standard_normal((2, H * G, D)).astype(np.float16)
    o = ref.paged_decode(q, kc, vc, bt, L, 0.2)
    for i in range(2):
        for h in range(H * G):
            kh = h // G
            k = torch.from_numpy(kc[bt[i], kh].reshape(-1, D)[:L[i]].astype(np.float64))
            v = torch.from_numpy(vc[bt[i], kh].reshape(-1, D)[:L[i]].astype(np.float64))
            p = torch.softmax(torch.from_numpy(q[i, h].astype(np.float64)) @ k.T * 0.2, 0)
            assert np.max(np.abs((p @ v).numpy() - o[i, h])) < 1e-12


def test_known_answer_layout_roundtrip():
    """Write at block 3 offset 5 with a 1.5/2.5 fill and read back through the
    layout (reference tests/metal/test_kv_cache_layout.py:68-131)."""
    nb, H, bs, D = 8, 4, 16, 64
    for layout in ("hnd", "nhd"):
        shape = (nb, H, bs, D) if layout == "hnd" else (nb, bs, H, D)
        kc = np.zeros(shape, np.float16)
        vc = np.zeros(shape, np.float16)
        nk = np.full((1, H, D), 1.5, np.float16)
        nv = np.full((1, H, D), 2.5, np.float16)
        ref.kv_write_slots(kc, vc, nk, nv, np.array([3 * bs + 5]), layout)
        if layout == "hnd":
            assert np.all(kc[3, :, 5] == 1.5) and np.all(vc[3, :, 5] == 2.5)
        else:
            assert np.all(kc[3, 5] == 1.5) and np.all(vc[3, 5] == 2.5)
        assert kc.sum() == 1.5 * H * D and vc.sum() == 2.5 * H * D


def _expected_cache(g):
    """cache_in with the rows the reference wrote at the new tokens' slots."""
    c = g["cache_in"].copy()
    bs = c.shape[2]
    sl = g["slot_mapping"]
    c[:, sl // bs, sl % bs] = g["written_rows"]
    return c


@pytest.mark.parametrize("name,D", [("decode_config1.npz", 64), ("decode_22b_600.npz", 128)])
def test_decode_config_goldens(name, D):
    """Config 1 exactly (qwen_b4, seed 0) and a 22B-shaped 600-token sequence, as the
    reference's MPSAttentionImpl.forward computed them: the oracle's KV write lands on
    the same bytes and its attention matches the reference's fp32 output."""
    g = load(name)
    kc, vc = g["cache_in"][0].copy(), g["cache_in"][1].copy()
    ref.kv_write_decode(kc, vc, g["k"], g["v"], g["block_table"], g["seq_lens"], layout="nhd")
    exp = _expected_cache(g)
    assert np.array_equal(kc.view(np.int16), exp[0].view(np.int16))
    assert np.array_equal(vc.view(np.int16), exp[1].view(np.int16))
    o = ref.paged_decode(g["q"], kc, vc, g["block_table"], g["seq_lens"], 1 / np.sqrt(D),
                         layout="nhd")
    assert np.max(np.abs(o - g["out"])) < 2e-5
