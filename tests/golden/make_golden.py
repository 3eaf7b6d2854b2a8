"""Generate the golden fixtures of this directory by running the REFERENCE.

Run where the reference's source tree is available (VA_REFERENCE_ROOT, or the
tree that baseline/_ref was pip-installed from); the outputs are committed
and the tests read only them, so nothing at test time needs the reference.

What runs (all reference code, unmodified):
  * MPSAttentionImpl.forward (vllm_apple/v1/attention/backends/mps_attn.py:207-282)
    with its base class (base_attn.py), loaded through an import shim for
    vLLM 0.22 (the reference targets an older vLLM layout):
      - decode batch (config-1 shape, smaller pool): KV scatter + decode SDPA;
      - mixed batch whose prefill sequences have no prior context (the only
        case where the reference's plugin prefill, which ignores cached
        context, equals the engine semantics).
    Attention runs on fp32 upcasts of the fp16 inputs (fp32-accumulated
    reference); the KV scatter runs on the fp16 cache (bit-exact bytes).
  * EngineRoPE._precompute_cache (vllm_apple/engine/ops/elementwise.py:680-697)
    with a stand-in context that captures the uploaded bytes.
  * metal_write_kv_batch from vllm_apple/metal/native/kv_write.c, compiled by
    oracle/Makefile into oracle/_ref.
  * RMSNorm / SiLU expected values exactly as the reference's own tests compute
    them (tests/metal/test_transformer_block.py:158-162, :205-255).

Usage:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import ctypes
import hashlib
import importlib.util
import os
import subprocess
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
from oracle.reference_loader import reference_source_tree  # noqa: E402

# the reference SOURCE tree: VA_REFERENCE_ROOT, else the tree baseline/_ref was installed from
REF = reference_source_tree()


def load_reference_attention():
    """Import base_attn.py / mps_attn.py of the reference against vLLM 0.22."""
    from oracle.reference_loader import load_reference_attention as _load
    return _load(REF)


def make_meta(mps, T, query_start_loc, seq_lens, block_table, slot_mapping, num_decode):
    return mps.MPSAttentionMetadata(
        num_actual_tokens=T, max_query_len=int(np.diff(query_start_loc).max()),
        query_start_loc=torch.tensor(query_start_loc, dtype=torch.int32),
        max_seq_len=int(max(seq_lens)), seq_lens=torch.tensor(seq_lens, dtype=torch.int32),
        block_table=block_table, slot_mapping=slot_mapping, scheduler_metadata=None,
        causal=True, num_decode_tokens=num_decode)


def run_forward(mps, Hq, Hkv, D, q, k, v, kv_cache, meta):
    impl = mps.MPSAttentionImpl(num_heads=Hq, head_size=D, scale=1.0 / np.sqrt(D),
                                num_kv_heads=Hkv, alibi_slopes=None, sliding_window=None,
                                kv_cache_dtype="auto")
    out = torch.zeros_like(q)
    impl.forward(None, q, k, v, kv_cache, meta, out)
    return out


def disjoint_blocks(lengths, bs, pool, gen):
    perm = torch.randperm(pool, generator=gen)
    need = [(L + bs - 1) // bs for L in lengths]
    bt = torch.full((len(lengths), max(need)), -1, dtype=torch.int64)
    at = 0
    for i, n in enumerate(need):
        bt[i, :n] = perm[at:at + n]
        at += n
    return bt


def golden_decode(mps):
    gen = torch.Generator().manual_seed(0)
    Hq, Hkv, D, bs, pool, B = 14, 2, 64, 16, 80, 4
    L = torch.randint(32, 301, (B,), generator=gen).tolist()
    bt = disjoint_blocks(L, bs, pool, gen)
    slots = torch.tensor([int(bt[i, (L[i] - 1) // bs]) * bs + (L[i] - 1) % bs for i in range(B)])
    q = torch.randn(B, Hq, D, generator=gen).half()
    k = torch.randn(B, Hkv, D, generator=gen).half()
    v = torch.randn(B, Hkv, D, generator=gen).half()
    cache = torch.randn(2, pool, bs, Hkv, D, generator=gen).half()
    meta = make_meta(mps, B, list(range(B + 1)), L, bt, slots, B)
    c16 = cache.clone()
    run_forward(mps, Hq, Hkv, D, q, k, v, c16, meta)          # fp16: KV bytes
    c32 = cache.float()
    out = run_forward(mps, Hq, Hkv, D, q.float(), k.float(), v.float(), c32, meta)
    np.savez_compressed(os.path.join(HERE, "decode_qwen_b4.npz"), q=q.numpy(), k=k.numpy(),
                        v=v.numpy(), cache_in=cache.numpy(), cache_out=c16.numpy(),
                        block_table=bt.numpy().astype(np.int32),
                        seq_lens=np.array(L, np.int32), slot_mapping=slots.numpy(),
                        out=out.numpy().astype(np.float32))


def golden_mixed(mps):
    """2 decode rows (cached context) + 2 prefill sequences with no prior context.

    Only the decode rows of this fixture are meaningful: in a mixed batch the
    reference's prefill branch (mps_attn.py:263) slices the query to the prefill
    tokens but _compute_attention_sdpa (base_attn.py:249) walks the UNshifted
    query_start_loc of the whole batch, so its prefill rows are misaligned.
    The prefill semantics are pinned by golden_prefill below."""
    gen = torch.Generator().manual_seed(1)
    Hq, Hkv, D, bs, pool = 8, 2, 64, 16, 64
    Ld = torch.randint(20, 200, (2,), generator=gen).tolist()
    P = [37, 50]  # new tokens of the prefill sequences (prior context 0)
    L = Ld + P
    bt = disjoint_blocks(L, bs, pool, gen)
    qlen = [1, 1] + P
    qsl = np.concatenate([[0], np.cumsum(qlen)]).tolist()
    tok_seq, pos = [], []
    for s, n in enumerate(qlen):
        tok_seq += [s] * n
        pos += list(range(L[s] - n, L[s]))
    T = len(pos)
    slots = torch.tensor([int(bt[tok_seq[t], pos[t] // bs]) * bs + pos[t] % bs
                          for t in range(T)])
    q = torch.randn(T, Hq, D, generator=gen).half()
    k = torch.randn(T, Hkv, D, generator=gen).half()
    v = torch.randn(T, Hkv, D, generator=gen).half()
    cache = torch.randn(2, pool, bs, Hkv, D, generator=gen).half()
    meta = make_meta(mps, T, qsl, L, bt, slots, 2)
    c32 = cache.float()
    out = run_forward(mps, Hq, Hkv, D, q.float(), k.float(), v.float(), c32, meta)
    np.savez_compressed(os.path.join(HERE, "mixed_noprior.npz"), q=q.numpy(), k=k.numpy(),
                        v=v.numpy(), cache_in=cache.numpy(),
                        block_table=bt.numpy().astype(np.int32), seq_lens=np.array(L, np.int32),
                        token_to_seq=np.array(tok_seq, np.int32),
                        positions=np.array(pos, np.int32), slot_mapping=slots.numpy(),
                        query_start_loc=np.array(qsl, np.int32),
                        out=out.numpy().astype(np.float32))


def golden_prefill(mps):
    """Prefill-only batch, no prior context: the reference's per-sequence causal
    SDPA over the new tokens equals the engine's paged prefill semantics."""
    gen = torch.Generator().manual_seed(5)
    Hq, Hkv, D, bs, pool = 12, 4, 64, 16, 48
    L = [45, 70, 1]
    bt = disjoint_blocks(L, bs, pool, gen)
    qsl = np.concatenate([[0], np.cumsum(L)]).tolist()
    tok_seq = sum(([s] * n for s, n in enumerate(L)), [])
    pos = sum((list(range(n)) for n in L), [])
    T = len(pos)
    slots = torch.tensor([int(bt[tok_seq[t], pos[t] // bs]) * bs + pos[t] % bs
                          for t in range(T)])
    q = torch.randn(T, Hq, D, generator=gen).half()
    k = torch.randn(T, Hkv, D, generator=gen).half()
    v = torch.randn(T, Hkv, D, generator=gen).half()
    cache = torch.randn(2, pool, bs, Hkv, D, generator=gen).half()
    meta = make_meta(mps, T, qsl, L, bt, slots, 0)
    c16 = cache.clone()
    run_forward(mps, Hq, Hkv, D, q, k, v, c16, meta)
    out = run_forward(mps, Hq, Hkv, D, q.float(), k.float(), v.float(), cache.float(), meta)
    np.savez_compressed(os.path.join(HERE, "prefill_noprior.npz"), q=q.numpy(), k=k.numpy(),
                        v=v.numpy(), cache_in=cache.numpy(), cache_out=c16.numpy(),
                        block_table=bt.numpy().astype(np.int32), seq_lens=np.array(L, np.int32),
                        token_to_seq=np.array(tok_seq, np.int32),
                        positions=np.array(pos, np.int32), slot_mapping=slots.numpy(),
                        query_start_loc=np.array(qsl, np.int32),
                        out=out.numpy().astype(np.float32))


def reference_rope_tables(rotary_dim, max_position, base):
    mod = importlib.import_module("vllm_apple.engine.ops.elementwise")
    captured = []

    class Ctx:
        def create_buffer_from_bytes(self, b):
            captured.append(bytes(b))
            return b

    obj = types.SimpleNamespace(rotary_dim=rotary_dim, max_position=max_position, base=base,
                                _context=Ctx())
    mod.EngineRoPE._precompute_cache(obj)
    half = rotary_dim // 2
    cos = np.frombuffer(captured[0], np.float32).reshape(max_position, half)
    sin = np.frombuffer(captured[1], np.float32).reshape(max_position, half)
    return cos, sin


def golden_rope():
    cos, sin = reference_rope_tables(64, 64, 1e4)
    big_c, big_s = reference_rope_tables(128, 32768, 1e6)
    np.savez_compressed(
        os.path.join(HERE, "rope_tables.npz"), cos_64_64_1e4=cos, sin_64_64_1e4=sin,
        sha256_cos_128_32768_1e6=np.frombuffer(hashlib.sha256(big_c.tobytes()).digest(), np.uint8),
        sha256_sin_128_32768_1e6=np.frombuffer(hashlib.sha256(big_s.tobytes()).digest(), np.uint8),
        rows_cos_128_32768_1e6=big_c[[0, 1, 4095, 32767]],
        rows_sin_128_32768_1e6=big_s[[0, 1, 4095, 32767]])


def golden_kv_write_c():
    subprocess.run(["make", "-s", "-C", os.path.join(REPO, "oracle"), "ref",
                    f"REF_ROOT={REF}"], check=True)
    lib = ctypes.CDLL(os.path.join(REPO, "oracle/_ref/libkv_write_ref.so"))
    gen = np.random.default_rng(2)
    nb, H, bs, D, T = 12, 3, 16, 32, 40
    kd = gen.integers(0, 65535, nb * H * bs * D, dtype=np.uint16)
    vd = gen.integers(0, 65535, nb * H * bs * D, dtype=np.uint16)
    ks = gen.integers(0, 65535, T * H * D, dtype=np.uint16)
    vs = gen.integers(0, 65535, T * H * D, dtype=np.uint16)
    slots = gen.permutation(nb * bs)[:T]
    blk, off = (slots // bs).astype(np.int64), (slots % bs).astype(np.int64)
    ko, vo = kd.copy(), vd.copy()
    P = ctypes.c_void_p
    lib.metal_write_kv_batch(P(ko.ctypes.data), P(vo.ctypes.data), P(ks.ctypes.data),
                             P(vs.ctypes.data), P(blk.ctypes.data), P(off.ctypes.data),
                             T, H, D, H * bs * D, bs * D, D)
    np.savez_compressed(os.path.join(HERE, "kv_write_c.npz"), key_dst=kd, value_dst=vd,
                        key_src=ks, value_src=vs, block_ids=blk, token_offsets=off,
                        key_out=ko, value_out=vo, dims=np.array([nb, H, bs, D, T]))


def golden_norm_silu():
    """Expected values computed exactly as the reference's tests do."""
    np.random.seed(42)
    x = np.random.randn(4, 128).astype(np.float16)
    w = np.random.randn(128).astype(np.float16)
    xt, wt = torch.from_numpy(x.astype(np.float32)), torch.from_numpy(w.astype(np.float32))
    var = xt.pow(2).mean(-1, keepdim=True)
    rms = (xt * torch.rsqrt(var + 1e-6) * wt).numpy()
    g = np.random.randn(1000).astype(np.float16)
    u = np.random.randn(1000).astype(np.float16)
    gt = torch.from_numpy(g.astype(np.float32))
    silu = (torch.nn.functional.silu(gt) * torch.from_numpy(u.astype(np.float32))).numpy()
    np.savez_compressed(os.path.join(HERE, "norm_silu.npz"), x=x, w=w, rms=rms, gate=g, up=u,
                        silu_mul=silu)


def golden_decode_configs(mps):
    """The reference's decode on the exact config-1 step (qwen_b4, seed 0, as
    vllm_apple_b200.workloads builds it) and on one 22B-shaped sequence of 600 tokens
    (32q/8kv heads, D = 128, GQA 4:1; the config-3 shape, one sequence to keep the
    fixture small)."""
    sys.path.insert(0, os.path.join(REPO, "vllm-apple_b200"))
    from vllm_apple_b200.workloads import DecodeCase, assign_blocks, make_decode_case
    cases = {"decode_config1.npz": make_decode_case("qwen_b4", seed=0, layout="nhd")}
    gen = torch.Generator().manual_seed(3)
    L = torch.tensor([600])
    bt, nb = assign_blocks(L.tolist(), 16, 0, gen)
    slot = bt[0, 599 // 16].to(torch.int64).reshape(1) * 16 + 599 % 16
    cases["decode_22b_600.npz"] = DecodeCase(
        "22b", 32, 8, 128, 16, "nhd", nb, L.to(torch.int32), bt, slot,
        torch.randn(1, 32, 128, generator=gen).half(), torch.randn(1, 8, 128, generator=gen).half(),
        torch.randn(1, 8, 128, generator=gen).half(),
        torch.randn(nb, 16, 8, 128, generator=gen).half(),
        torch.randn(nb, 16, 8, 128, generator=gen).half())
    for name, c in cases.items():
        B = c.batch
        cache = torch.stack([c.k_cache, c.v_cache])
        L = c.seq_lens.tolist()
        bt = c.block_table.to(torch.int64)
        meta = make_meta(mps, B, list(range(B + 1)), L, bt, c.slot_mapping, B)
        c16 = cache.clone()
        run_forward(mps, c.Hq, c.Hkv, c.D, c.q, c.new_k, c.new_v, c16, meta)  # KV bytes
        c32 = cache.float()
        out = run_forward(mps, c.Hq, c.Hkv, c.D, c.q.float(), c.new_k.float(), c.new_v.float(),
                          c32, meta)
        # the reference wrote exactly the B slots; keep the rows it wrote (not the
        # whole second cache) to keep the fixture small
        ci, co = cache.numpy(), c16.numpy()
        sl = c.slot_mapping.numpy()
        blk, off = sl // c.bs, sl % c.bs
        diff = np.zeros(ci.shape[1:3], bool)
        diff[blk, off] = True
        assert np.array_equal(ci.view(np.int16)[:, ~diff], co.view(np.int16)[:, ~diff])
        np.savez_compressed(os.path.join(HERE, name), q=c.q.numpy(), k=c.new_k.numpy(),
                            v=c.new_v.numpy(), cache_in=ci, written_rows=co[:, blk, off],
                            block_table=c.block_table.numpy(), seq_lens=c.seq_lens.numpy(),
                            slot_mapping=sl, out=out.numpy().astype(np.float32))


def main():
    mps = load_reference_attention()
    golden_decode_configs(mps)
    golden_decode(mps)
    golden_mixed(mps)
    golden_prefill(mps)
    golden_rope()
    golden_kv_write_c()
    golden_norm_silu()
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
