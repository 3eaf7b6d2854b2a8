"""torch-facing wrappers of the C ABI (one call = one or two kernel launches).

Every function takes CUDA tensors, derives pointers and element strides, and
enqueues the sm_100a kernels on the current CUDA stream of the tensors'
device.  Nothing here synchronises; device-side data problems (bad slots,
blocks or positions) set bits in a per-device error word that
:func:`check_device_errors` reads.  There is no CPU fallback: non-CUDA inputs
raise.

Cache layouts (element strides; head_size contiguous):
  ``"hnd"`` engine layout ``[num_blocks, num_kv_heads, block_size, head_size]``
  ``"nhd"`` vLLM layout   ``[num_blocks, block_size, num_kv_heads, head_size]``
"""
from __future__ import annotations

import threading
from dataclasses import dataclass

import torch

from . import _lib

_state_lock = threading.Lock()
_err_flags: dict[int, torch.Tensor] = {}
_workspaces: dict[tuple[int, str, int], torch.Tensor] = {}


# ---------------------------------------------------------------------------
# per-device state
# ---------------------------------------------------------------------------
def _dev_index(t: torch.Tensor) -> int:
    if not t.is_cuda:
        raise RuntimeError("vllm_apple_b200 ops run on CUDA tensors only (no CPU fallback); "
                           f"got a tensor on {t.device}")
    return t.device.index if t.device.index is not None else torch.cuda.current_device()


def err_flag(device: int) -> torch.Tensor:
    """The device's int32 error word (allocated zeroed on first use)."""
    with _state_lock:
        f = _err_flags.get(device)
        if f is None:
            f = torch.zeros(1, dtype=torch.int32, device=f"cuda:{device}")
            _err_flags[device] = f
        return f


def check_device_errors(device: int | None = None, raise_on_error: bool = True) -> int:
    """Synchronise ``device``, read and clear its error word; raise if set."""
    dev = torch.cuda.current_device() if device is None else device
    f = err_flag(dev)
    bits = int(f.item())
    if bits:
        f.zero_()
        if raise_on_error:
            raise _lib.VAError("device reported: " + "; ".join(_lib.describe_flags(bits)))
    return bits


def workspace(device: int, kind: str, nbytes: int,
              stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """A device scratch buffer of at least ``nbytes`` for calls enqueued on
    ``stream`` (default: the device's current stream), grown on demand.

    One buffer per (device, kind, stream): calls on one stream are ordered, so
    they may share it; calls on different streams get different buffers and
    cannot race.  A grown buffer is allocated while ``stream`` is current, so the
    caching allocator reuses the old one only behind the work already queued
    on that stream."""
    st = torch.cuda.current_stream(device) if stream is None else stream
    key = (device, kind, st.cuda_stream)
    with _state_lock:
        ws = _workspaces.get(key)
        if ws is None or ws.numel() < nbytes:
            size = max(nbytes, 1 << 16)
            if ws is not None:
                size = max(size, 2 * ws.numel())
            with torch.cuda.stream(st):
                ws = torch.empty(size, dtype=torch.uint8, device=f"cuda:{device}")
            _workspaces[key] = ws
        return ws


def _stream(device: int) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


# ---------------------------------------------------------------------------
# cache geometry
# ---------------------------------------------------------------------------
@dataclass(frozen=True)
class CacheGeom:
    num_blocks: int
    num_kv_heads: int
    block_size: int
    head_size: int
    s_block: int
    s_head: int
    s_token: int


def cache_geom(cache: torch.Tensor, layout: str) -> CacheGeom:
    if cache.dtype != torch.float16:
        raise TypeError(f"KV cache must be float16, got {cache.dtype}")
    if cache.dim() != 4 or cache.stride(3) != 1:
        raise ValueError("KV cache must be 4-D with a contiguous head_size axis")
    st = cache.stride()
    if layout == "hnd":
        nb, h, bs, d = cache.shape
        return CacheGeom(nb, h, bs, d, st[0], st[1], st[2])
    if layout == "nhd":
        nb, bs, h, d = cache.shape
        return CacheGeom(nb, h, bs, d, st[0], st[2], st[1])
    raise ValueError(f"unknown cache layout {layout!r}")


def _rows3(t: torch.Tensor, name: str) -> tuple[int, int]:
    if t.dtype != torch.float16:
        raise TypeError(f"{name} must be float16, got {t.dtype}")
    if t.dim() != 3 or t.stride(2) != 1:
        raise ValueError(f"{name} must be [tokens, heads, head_size] with contiguous head_size")
    return t.stride(0), t.stride(1)


def _i32(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dtype != torch.int32:
        raise TypeError(f"{name} must be int32, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t


# ---------------------------------------------------------------------------
# KV-cache writes
# ---------------------------------------------------------------------------
def kv_write_slots(k_cache, v_cache, new_k, new_v, slot_mapping, layout="hnd"):
    """Scatter ``new_k/new_v`` [T, Hkv, D] into the caches by slot (-1 = skip)."""
    dev = _dev_index(k_cache)
    g = cache_geom(k_cache, layout)
    if cache_geom(v_cache, layout) != g:
        raise ValueError("K and V caches differ in shape or strides")
    n_tok, n_head = _rows3(new_k, "new_k")
    if _rows3(new_v, "new_v") != (n_tok, n_head) or new_k.shape != new_v.shape:
        raise ValueError("new_k and new_v differ in shape or strides")
    if slot_mapping.dtype not in (torch.int32, torch.int64) or not slot_mapping.is_contiguous():
        raise TypeError("slot_mapping must be a contiguous int32 or int64 tensor")
    T = new_k.shape[0]
    if slot_mapping.numel() < T:
        raise ValueError("slot_mapping shorter than the number of tokens")
    _lib.check(_lib.load().va_kv_write_slots(
        k_cache.data_ptr(), v_cache.data_ptr(), new_k.data_ptr(), new_v.data_ptr(),
        slot_mapping.data_ptr(), int(slot_mapping.dtype == torch.int64), T, g.num_kv_heads,
        g.head_size, g.block_size, g.num_blocks, g.s_block, g.s_head, g.s_token, n_tok, n_head,
        err_flag(dev).data_ptr(), _stream(dev)), "va_kv_write_slots")


def kv_write_decode(k_cache, v_cache, new_k, new_v, block_table, seq_lens, layout="hnd",
                    max_blocks_per_seq=None, num_seqs=None):
    """Write row i of ``new_k/new_v`` at position seq_lens[i]-1 through the block table."""
    dev = _dev_index(k_cache)
    g = cache_geom(k_cache, layout)
    n_tok, n_head = _rows3(new_k, "new_k")
    _rows3(new_v, "new_v")
    _i32(block_table, "block_table")
    _i32(seq_lens, "seq_lens")
    B = new_k.shape[0] if num_seqs is None else num_seqs
    mb = block_table.shape[1] if max_blocks_per_seq is None else max_blocks_per_seq
    _lib.check(_lib.load().va_kv_write_decode(
        k_cache.data_ptr(), v_cache.data_ptr(), new_k.data_ptr(), new_v.data_ptr(),
        block_table.data_ptr(), seq_lens.data_ptr(), B, mb, g.num_kv_heads, g.head_size,
        g.block_size, g.num_blocks, g.s_block, g.s_head, g.s_token, n_tok, n_head,
        err_flag(dev).data_ptr(), _stream(dev)), "va_kv_write_decode")


def write_kv_batch(key_dst, value_dst, key_src, value_src, block_ids, token_offsets,
                   num_tokens, num_kv_heads, head_size, stride_block, stride_head, stride_token):
    """Device twin of the reference's ``metal_write_kv_batch`` (same arguments)."""
    dev = _dev_index(key_dst)
    for t, n in ((block_ids, "block_ids"), (token_offsets, "token_offsets")):
        if t.dtype != torch.int64 or not t.is_contiguous():
            raise TypeError(f"{n} must be a contiguous int64 tensor")
    _lib.check(_lib.load().va_write_kv_batch(
        key_dst.data_ptr(), value_dst.data_ptr(), key_src.data_ptr(), value_src.data_ptr(),
        block_ids.data_ptr(), token_offsets.data_ptr(), num_tokens, num_kv_heads, head_size,
        stride_block, stride_head, stride_token, _stream(dev)), "va_write_kv_batch")


# ---------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------
def paged_decode(out, q, k_cache, v_cache, block_table, seq_lens, *, scale, max_seq_len,
                 new_k=None, new_v=None, layout="hnd", num_seqs=None,
                 max_blocks_per_seq=None):
    """Decode attention (+ fused KV write when ``new_k``/``new_v`` are given).

    out/q [B, Hq, D]; block_table int32 [B, max_blocks]; seq_lens int32 [B]
    (including the new token); ``max_seq_len`` >= every seq_len.
    """
    dev = _dev_index(q)
    g = cache_geom(k_cache, layout)
    if cache_geom(v_cache, layout) != g:
        raise ValueError("K and V caches differ in shape or strides")
    q_st, q_sh = _rows3(q, "q")
    o_st, o_sh = _rows3(out, "out")
    _i32(block_table, "block_table")
    _i32(seq_lens, "seq_lens")
    B = q.shape[0] if num_seqs is None else num_seqs
    Hq, D = q.shape[1], q.shape[2]
    if D != g.head_size:
        raise ValueError(f"q head_size {D} != cache head_size {g.head_size}")
    n_st = n_sh = 0
    if new_k is not None:
        n_st, n_sh = _rows3(new_k, "new_k")
        if _rows3(new_v, "new_v") != (n_st, n_sh):
            raise ValueError("new_k and new_v differ in strides")
    mb = block_table.shape[1] if max_blocks_per_seq is None else max_blocks_per_seq
    lib = _lib.load()
    nbytes = lib.va_paged_decode_workspace_size(B, Hq, g.num_kv_heads, D, g.block_size,
                                                max_seq_len)
    ws = workspace(dev, "decode", nbytes) if nbytes else None
    _lib.check(lib.va_paged_decode(
        out.data_ptr(), q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
        block_table.data_ptr(), seq_lens.data_ptr(), _ptr(new_k), _ptr(new_v), B, Hq,
        g.num_kv_heads, D, g.block_size, mb, max_seq_len, g.num_blocks, float(scale), g.s_block,
        g.s_head, g.s_token, q_st, q_sh, o_st, o_sh, n_st, n_sh, _ptr(ws),
        0 if ws is None else ws.numel(), err_flag(dev).data_ptr(), _stream(dev)),
        "va_paged_decode")


def paged_prefill(out, q, k_cache, v_cache, block_table, token_to_seq, positions, *, scale,
                  layout="hnd", num_tokens=None, num_seqs=None, max_blocks_per_seq=None):
    """Token-parallel causal attention: token t attends to positions 0..positions[t]
    of sequence token_to_seq[t] (K/V of the new tokens already in the cache)."""
    dev = _dev_index(q)
    g = cache_geom(k_cache, layout)
    q_st, q_sh = _rows3(q, "q")
    o_st, o_sh = _rows3(out, "out")
    _i32(block_table, "block_table")
    _i32(token_to_seq, "token_to_seq")
    _i32(positions, "positions")
    T = q.shape[0] if num_tokens is None else num_tokens
    S = block_table.shape[0] if num_seqs is None else num_seqs
    mb = block_table.shape[1] if max_blocks_per_seq is None else max_blocks_per_seq
    lib = _lib.load()
    nbytes = lib.va_paged_prefill_workspace_size(T, S, q.shape[1], g.num_kv_heads, q.shape[2],
                                                 g.block_size, mb)
    ws = workspace(dev, "prefill", nbytes)
    _lib.check(lib.va_paged_prefill(
        out.data_ptr(), q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
        block_table.data_ptr(), token_to_seq.data_ptr(), positions.data_ptr(), T, S, q.shape[1],
        g.num_kv_heads, q.shape[2], g.block_size, mb, g.num_blocks, float(scale), g.s_block,
        g.s_head, g.s_token, q_st, q_sh, o_st, o_sh, ws.data_ptr(), ws.numel(),
        err_flag(dev).data_ptr(), _stream(dev)), "va_paged_prefill")


# ---------------------------------------------------------------------------
# elementwise
# ---------------------------------------------------------------------------
def _rows2(t: torch.Tensor, name: str) -> int:
    if t.dtype != torch.float16:
        raise TypeError(f"{name} must be float16, got {t.dtype}")
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be [tokens, hidden] with a contiguous hidden axis")
    return t.stride(0)


def rmsnorm(out, x, weight, eps, residual=None, num_tokens=None):
    """out = x * rsqrt(mean(x^2) + eps) * weight (+ residual), rows of [T, H]."""
    dev = _dev_index(x)
    xs, os_ = _rows2(x, "x"), _rows2(out, "out")
    rs = _rows2(residual, "residual") if residual is not None else 0
    T = x.shape[0] if num_tokens is None else num_tokens
    _lib.check(_lib.load().va_rmsnorm(
        out.data_ptr(), x.data_ptr(), weight.data_ptr(), _ptr(residual), T, x.shape[1],
        float(eps), xs, os_, rs, _stream(dev)), "va_rmsnorm")


def rope(q, k, cos_cache, sin_cache, positions, rotary_dim=None, is_neox=True,
         num_tokens=None):
    """In-place rotary embedding of q [T, Hq, D] and k [T, Hkv, D]."""
    dev = _dev_index(q)
    q_st, _ = _rows3(q, "q")
    k_st, _ = _rows3(k, "k")
    if q.stride(1) != q.shape[2] or k.stride(1) != k.shape[2]:
        raise ValueError("q/k heads must be packed (head stride == head_size)")
    for t, n in ((cos_cache, "cos_cache"), (sin_cache, "sin_cache")):
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise TypeError(f"{n} must be a contiguous float32 tensor")
    _i32(positions, "positions")
    T = q.shape[0] if num_tokens is None else num_tokens
    D = q.shape[2]
    rot = D if rotary_dim is None else rotary_dim
    _lib.check(_lib.load().va_rope(
        q.data_ptr(), k.data_ptr(), cos_cache.data_ptr(), sin_cache.data_ptr(),
        positions.data_ptr(), T, q.shape[1], k.shape[1], D, rot, cos_cache.shape[0], q_st, k_st,
        int(bool(is_neox)), err_flag(dev).data_ptr(), _stream(dev)), "va_rope")


def silu_mul(out, gate, up, num_elements=None):
    """out = silu(gate) * up, elementwise over contiguous fp16 buffers."""
    dev = _dev_index(gate)
    for t, n in ((out, "out"), (gate, "gate"), (up, "up")):
        if t.dtype != torch.float16 or not t.is_contiguous():
            raise TypeError(f"{n} must be a contiguous float16 tensor")
    n = gate.numel() if num_elements is None else num_elements
    _lib.check(_lib.load().va_silu_mul(out.data_ptr(), gate.data_ptr(), up.data_ptr(), n,
                                       _stream(dev)), "va_silu_mul")


def topk(indices, values, logits, k, num_tokens=None):
    """Top-k of each row of fp16 ``logits [T, V]`` (row stride may exceed V):
    ``indices [T, k]`` int32 and ``values [T, k]`` fp16, largest first, ties by the
    lower index; NaN / -inf are never selected and short rows are padded with
    (-1, -inf)."""
    dev = _dev_index(logits)
    if logits.dtype != torch.float16 or logits.dim() != 2 or logits.stride(1) != 1:
        raise TypeError("logits must be a float16 [T, V] tensor with unit inner stride")
    if indices.dtype != torch.int32 or values.dtype != torch.float16:
        raise TypeError("indices must be int32 and values float16")
    for t, n in ((indices, "indices"), (values, "values")):
        if not t.is_contiguous():
            raise TypeError(f"{n} must be contiguous")
    T = logits.shape[0] if num_tokens is None else num_tokens
    if indices.numel() < T * k or values.numel() < T * k:
        raise ValueError("indices / values hold fewer than num_tokens * k entries")
    lib = _lib.load()
    V = logits.shape[1]
    nbytes = lib.va_topk_workspace_size(T, V, int(k))
    ws = workspace(dev, "topk", nbytes) if nbytes else None
    _lib.check(lib.va_topk_ws(indices.data_ptr(), values.data_ptr(), logits.data_ptr(), T, V,
                              logits.stride(0), int(k), 0 if ws is None else ws.data_ptr(),
                              nbytes, _stream(dev)), "va_topk_ws")


# ---------------------------------------------------------------------------
# step-level ops
# ---------------------------------------------------------------------------
def rope_kv_write_slots(q, k, v, k_cache, v_cache, cos_cache, sin_cache, positions,
                        slot_mapping, layout="hnd"):
    """Neox RoPE of q/k in place + scatter of rotated k and v into the cache by slot."""
    dev = _dev_index(q)
    g = cache_geom(k_cache, layout)
    q_st, _ = _rows3(q, "q")
    k_st, _ = _rows3(k, "k")
    v_st, _ = _rows3(v, "v")
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        if t.stride(1) != t.shape[2]:
            raise ValueError(f"{n} heads must be packed (head stride == head_size)")
    _i32(positions, "positions")
    if slot_mapping.dtype not in (torch.int32, torch.int64) or not slot_mapping.is_contiguous():
        raise TypeError("slot_mapping must be a contiguous int32 or int64 tensor")
    _lib.check(_lib.load().va_rope_kv_write_slots(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
        cos_cache.data_ptr(), sin_cache.data_ptr(), positions.data_ptr(), slot_mapping.data_ptr(),
        int(slot_mapping.dtype == torch.int64), q.shape[0], q.shape[1], k.shape[1], q.shape[2],
        g.block_size, g.num_blocks, cos_cache.shape[0], q_st, k_st, v_st, g.s_block, g.s_head,
        g.s_token, err_flag(dev).data_ptr(), _stream(dev)), "va_rope_kv_write_slots")


def build_prefill_metadata(query_start_loc, seq_lens, block_table, num_tokens, first_token=0,
                           block_size=16, with_slots=True):
    """(token_to_seq int32, positions int32, slot_mapping int64 | None) on the device."""
    dev = _dev_index(seq_lens)
    _i32(query_start_loc, "query_start_loc")
    _i32(seq_lens, "seq_lens")
    _i32(block_table, "block_table")
    d = seq_lens.device
    ts = torch.empty(num_tokens, dtype=torch.int32, device=d)
    ps = torch.empty(num_tokens, dtype=torch.int32, device=d)
    sm = torch.empty(num_tokens, dtype=torch.int64, device=d) if with_slots else None
    _lib.check(_lib.load().va_build_prefill_metadata(
        query_start_loc.data_ptr(), seq_lens.data_ptr(), block_table.data_ptr(),
        seq_lens.numel(), first_token, num_tokens, block_table.shape[1], block_size,
        ts.data_ptr(), ps.data_ptr(), _ptr(sm), _stream(dev)), "va_build_prefill_metadata")
    return ts, ps, sm


def kv_sync_blocks(src_k, src_v, dst_k, dst_v, block_table, seq_lens, src_layout="nhd",
                   dst_layout="hnd"):
    """Copy the active blocks of every sequence between cache layouts (bit-exact)."""
    dev = _dev_index(src_k)
    s = cache_geom(src_k, src_layout)
    d = cache_geom(dst_k, dst_layout)
    if (s.num_blocks, s.num_kv_heads, s.block_size, s.head_size) != (
            d.num_blocks, d.num_kv_heads, d.block_size, d.head_size):
        raise ValueError("source and destination caches differ in geometry")
    _i32(block_table, "block_table")
    _i32(seq_lens, "seq_lens")
    _lib.check(_lib.load().va_kv_sync_blocks(
        src_k.data_ptr(), src_v.data_ptr(), dst_k.data_ptr(), dst_v.data_ptr(),
        block_table.data_ptr(), seq_lens.data_ptr(), seq_lens.numel(), block_table.shape[1],
        s.num_kv_heads, s.head_size, s.block_size, s.num_blocks, s.s_block, s.s_head, s.s_token,
        d.s_block, d.s_head, d.s_token, _stream(dev)), "va_kv_sync_blocks")
