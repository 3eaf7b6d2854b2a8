"""Seeded synthetic inputs with the shapes of the benchmark configurations.

The reference measures this path on no public dataset; these generators stand
in for real traffic with the configured shapes, length distributions and
N(0,1) fp16 activations.  Small per-sequence metadata (lengths, block tables,
slots) is drawn on the CPU from ``torch.Generator().manual_seed(seed)``; large
tensors (the KV pool) are drawn on ``device``.

Configurations (head counts Hq/Hkv, head_size D, block_size 16):
  ``qwen_b4``        Qwen2-0.5B shape 14/2/64, batch 4, L ~ U[32, 512], pool 256
  ``qwen_b64``       same shape, batch 64, L ~ U[1, 4096], pool max(8192, demand)
  ``devstral_b128``  22B shape 32/8/128, batch 128, L log-normal(median 2048,
                     sigma 0.6) clipped to [512, 8192]
  ``devstral_b1024`` same, batch 1024 (sharded by sequence across GPUs)
  ``mixed_22b``      22B shape: 4 prefill chunks of 512 tokens with prior
                     context U[0, 4096] + 60 decode sequences with L ~ U[256, 8192]
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

DECODE_CONFIGS = {
    "qwen_b4": dict(Hq=14, Hkv=2, D=64, bs=16, batch=4, dist=("uniform", 32, 512), pool=256),
    "qwen_b64": dict(Hq=14, Hkv=2, D=64, bs=16, batch=64, dist=("uniform", 1, 4096), pool=8192),
    "devstral_b128": dict(Hq=32, Hkv=8, D=128, bs=16, batch=128,
                          dist=("lognormal", 2048, 0.6, 512, 8192), pool=0),
    "devstral_b1024": dict(Hq=32, Hkv=8, D=128, bs=16, batch=1024,
                           dist=("lognormal", 2048, 0.6, 512, 8192), pool=0),
}


def draw_lengths(dist, n: int, gen: torch.Generator) -> torch.Tensor:
    """Context lengths (including the new token) as int64 [n]."""
    kind = dist[0]
    if kind == "uniform":
        lo, hi = dist[1], dist[2]
        return torch.randint(lo, hi + 1, (n,), generator=gen, dtype=torch.int64)
    if kind == "lognormal":
        median, sigma, lo, hi = dist[1:]
        z = torch.randn(n, generator=gen, dtype=torch.float64)
        L = torch.exp(math.log(median) + sigma * z).round().to(torch.int64)
        return L.clamp(lo, hi)
    raise ValueError(kind)


def lpt_shard(lengths, world: int) -> list[list[int]]:
    """Sequences of each rank (greedy LPT on context length; see sharding.py)."""
    from .sharding import lpt_partition
    return lpt_partition(lengths, world)


def assign_blocks(lengths, bs: int, pool_min: int, gen: torch.Generator):
    """Disjoint random (shuffled-pool) blocks per sequence.

    Returns (block_table int32 [B, max_blocks] padded with -1, num_blocks)."""
    need = [(int(L) + bs - 1) // bs for L in lengths]
    pool = max(pool_min, sum(need), 1)
    perm = torch.randperm(pool, generator=gen).to(torch.int32)
    width = max(need) if need else 1
    bt = torch.full((len(need), max(width, 1)), -1, dtype=torch.int32)
    at = 0
    for i, n in enumerate(need):
        bt[i, :n] = perm[at:at + n]
        at += n
    return bt, pool


def _randn(shape, gen_cpu, device, seed):
    if torch.device(device).type == "cuda":
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        return torch.randn(shape, generator=g, device=device, dtype=torch.float16)
    return torch.randn(shape, generator=gen_cpu, dtype=torch.float32).to(torch.float16)


def alloc_cache(num_blocks, Hkv, bs, D, layout, device, seed, gen_cpu):
    shape = (num_blocks, Hkv, bs, D) if layout == "hnd" else (num_blocks, bs, Hkv, D)
    return _randn(shape, gen_cpu, device, seed)


@dataclass
class DecodeCase:
    name: str
    Hq: int
    Hkv: int
    D: int
    bs: int
    layout: str
    num_blocks: int
    seq_lens: torch.Tensor      # int32 [B] (cpu)
    block_table: torch.Tensor   # int32 [B, max_blocks] (cpu)
    slot_mapping: torch.Tensor  # int64 [B] (cpu): slot of the new token
    q: torch.Tensor             # fp16 [B, Hq, D]
    new_k: torch.Tensor         # fp16 [B, Hkv, D]
    new_v: torch.Tensor
    k_cache: torch.Tensor       # fp16, layout
    v_cache: torch.Tensor
    meta: dict = field(default_factory=dict)

    @property
    def batch(self) -> int:
        return int(self.seq_lens.numel())

    @property
    def scale(self) -> float:
        return 1.0 / math.sqrt(self.D)

    @property
    def max_seq_len(self) -> int:
        return int(self.seq_lens.max()) if self.batch else 0

    @property
    def context_tokens(self) -> int:
        return int(self.seq_lens.to(torch.int64).sum())

    def algorithmic_bytes(self) -> int:
        """HBM bytes one fused decode step must move at minimum: every context
        K/V row once per kv head, q read + out write, new K/V read + write,
        block-table entries and seq_lens."""
        B, Hq, Hkv, D, bs = self.batch, self.Hq, self.Hkv, self.D, self.bs
        pages = int(((self.seq_lens.to(torch.int64) + bs - 1) // bs).sum())
        return (self.context_tokens * Hkv * D * 2 * 2 + B * Hq * D * 2 * 2
                + B * Hkv * D * 2 * 2 * 2 + pages * 4 + B * 4)


def make_decode_case(config: str, *, device="cpu", seed: int = 0, layout: str = "hnd",
                     batch: int | None = None, seq_subset: list[int] | None = None,
                     lengths: torch.Tensor | None = None) -> DecodeCase:
    """Build one decode step of ``config``.  ``seq_subset`` keeps only those
    sequences (a rank's shard); ``lengths`` overrides the drawn lengths."""
    c = DECODE_CONFIGS[config]
    gen = torch.Generator().manual_seed(seed)
    B = batch or c["batch"]
    L = draw_lengths(c["dist"], B, gen) if lengths is None else lengths.to(torch.int64)
    if seq_subset is not None:
        L = L[torch.as_tensor(seq_subset, dtype=torch.int64)]
        gen = torch.Generator().manual_seed(seed * 7919 + 17 + len(seq_subset))
    bt, nb = assign_blocks(L.tolist(), c["bs"], c["pool"], gen)
    bs = c["bs"]
    Lm1 = L - 1
    slot = bt[torch.arange(len(L)), (Lm1 // bs)].to(torch.int64) * bs + Lm1 % bs
    Hq, Hkv, D = c["Hq"], c["Hkv"], c["D"]
    q = _randn((len(L), Hq, D), gen, "cpu", 0)
    nk = _randn((len(L), Hkv, D), gen, "cpu", 0)
    nv = _randn((len(L), Hkv, D), gen, "cpu", 0)
    kc = alloc_cache(nb, Hkv, bs, D, layout, device, seed + 101, gen)
    vc = alloc_cache(nb, Hkv, bs, D, layout, device, seed + 202, gen)
    return DecodeCase(config, Hq, Hkv, D, bs, layout, nb, L.to(torch.int32), bt, slot,
                      q, nk, nv, kc, vc, meta=dict(seed=seed, dist=c["dist"]))


@dataclass
class MixedCase:
    """Chunked-prefill mixed batch: decode rows first, then prefill chunks."""
    Hq: int
    Hkv: int
    D: int
    bs: int
    layout: str
    num_blocks: int
    seq_lens: torch.Tensor       # int32 [S] full length after this step
    block_table: torch.Tensor    # int32 [S, max_blocks]
    query_start_loc: torch.Tensor  # int32 [S+1]
    token_to_seq: torch.Tensor   # int32 [T]
    positions: torch.Tensor      # int32 [T]
    slot_mapping: torch.Tensor   # int64 [T]
    q: torch.Tensor              # fp16 [T, Hq, D]
    k: torch.Tensor              # fp16 [T, Hkv, D] new rows
    v: torch.Tensor
    k_cache: torch.Tensor
    v_cache: torch.Tensor
    num_decode_tokens: int

    @property
    def scale(self) -> float:
        return 1.0 / math.sqrt(self.D)

    @property
    def num_tokens(self) -> int:
        return int(self.positions.numel())


def make_mixed_case(*, device="cpu", seed: int = 0, layout: str = "hnd", Hq=32, Hkv=8, D=128,
                    bs=16, num_chunks=4, chunk=512, prior=(0, 4096), num_decode=60,
                    decode_len=(256, 8192)) -> MixedCase:
    gen = torch.Generator().manual_seed(seed)
    Ld = torch.randint(decode_len[0], decode_len[1] + 1, (num_decode,), generator=gen)
    P = torch.randint(prior[0], prior[1] + 1, (num_chunks,), generator=gen)
    full = torch.cat([Ld, P + chunk]).to(torch.int64)
    bt, nb = assign_blocks(full.tolist(), bs, 0, gen)
    qlen = torch.cat([torch.ones(num_decode, dtype=torch.int64),
                      torch.full((num_chunks,), chunk, dtype=torch.int64)])
    qsl = torch.zeros(len(full) + 1, dtype=torch.int64)
    qsl[1:] = torch.cumsum(qlen, 0)
    tok_seq, pos = [], []
    for s in range(len(full)):
        n = int(qlen[s])
        tok_seq.append(torch.full((n,), s, dtype=torch.int64))
        pos.append(torch.arange(int(full[s]) - n, int(full[s]), dtype=torch.int64))
    tok_seq = torch.cat(tok_seq)
    pos = torch.cat(pos)
    slot = bt[tok_seq, pos // bs].to(torch.int64) * bs + pos % bs
    T = len(pos)
    q = _randn((T, Hq, D), gen, "cpu", 0)
    k = _randn((T, Hkv, D), gen, "cpu", 0)
    v = _randn((T, Hkv, D), gen, "cpu", 0)
    kc = alloc_cache(nb, Hkv, bs, D, layout, device, seed + 101, gen)
    vc = alloc_cache(nb, Hkv, bs, D, layout, device, seed + 202, gen)
    return MixedCase(Hq, Hkv, D, bs, layout, nb, full.to(torch.int32), bt, qsl.to(torch.int32),
                     tok_seq.to(torch.int32), pos.to(torch.int32), slot, q, k, v, kc, vc,
                     num_decode)


@dataclass
class ElementwiseCase:
    x: torch.Tensor        # fp16 [T, hidden]
    w: torch.Tensor        # fp16 [hidden] ~ N(1, 0.02)
    eps: float
    q: torch.Tensor        # fp16 [T, Hq, D]
    k: torch.Tensor        # fp16 [T, Hkv, D]
    positions: torch.Tensor  # int32 [T]
    theta: float
    max_position: int
    gate: torch.Tensor     # fp16 [T, I]
    up: torch.Tensor


def make_elementwise_case(*, device="cpu", seed=0, T=8192, hidden=5120, Hq=32, Hkv=8, D=128,
                          theta=1e6, max_position=32768, inter=32768) -> ElementwiseCase:
    gen = torch.Generator().manual_seed(seed)
    x = _randn((T, hidden), gen, device, seed + 1)
    w = (1.0 + 0.02 * torch.randn(hidden, generator=gen)).to(torch.float16).to(device)
    q = _randn((T, Hq, D), gen, device, seed + 2)
    k = _randn((T, Hkv, D), gen, device, seed + 3)
    pos = torch.randint(0, max_position, (T,), generator=gen, dtype=torch.int64)
    gate = _randn((T, inter), gen, device, seed + 4)
    up = _randn((T, inter), gen, device, seed + 5)
    return ElementwiseCase(x, w, 1e-5, q, k, pos.to(torch.int32).to(device), theta,
                           max_position, gate, up)
