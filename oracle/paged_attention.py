"""numpy restatement of the vllm_apple paged-attention hot path (TEST ORACLE).

Test infrastructure only -- never imported by the product package.

Cache layouts (element strides, last dim contiguous):
  * ``"hnd"``: engine / Metal layout ``[num_blocks, num_kv_heads, block_size, head_size]``
    (vllm_apple/engine/kv_cache.py:136-151, engine/ops/attention.py:206-209)
  * ``"nhd"``: vLLM tensor layout ``[num_blocks, block_size, num_kv_heads, head_size]``
    (vllm_apple/v1/attention/backends/base_attn.py:113-125; one half of the
    ``(2, nb, bs, H, D)`` kv_cache tensor)

All floating-point attention/norm math runs in float64 (an fp32-or-better
accumulated reference); callers compare the fp16 kernel output against it.
"""
from __future__ import annotations

import numpy as np

# --------------------------------------------------------------------------
# layout helpers
# --------------------------------------------------------------------------


def _row(cache: np.ndarray, layout: str, block: int, head: int, off: int) -> np.ndarray:
    if layout == "hnd":
        return cache[block, head, off]
    if layout == "nhd":
        return cache[block, off, head]
    raise ValueError(f"unknown layout {layout!r}")


def cache_geometry(cache: np.ndarray, layout: str):
    """Return (num_blocks, num_kv_heads, block_size, head_size)."""
    if layout == "hnd":
        nb, h, bs, d = cache.shape
    elif layout == "nhd":
        nb, bs, h, d = cache.shape
    else:
        raise ValueError(layout)
    return nb, h, bs, d


# --------------------------------------------------------------------------
# KV-cache writes (bit-exact byte copies)
# --------------------------------------------------------------------------


def kv_write_slots(k_cache, v_cache, new_k, new_v, slot_mapping, layout="hnd"):
    """Scatter new K/V rows by ``slot_mapping``; slots < 0 are padding and skipped.

    Follows ``kv_write_prefill`` (vllm_apple/engine/ops/kv_write.py:118-156):
    slot -> (block = slot // bs, offset = slot % bs), one row per (token, head);
    and the vLLM-layout scatter ``_update_kv_cache_scatter``
    (vllm_apple/v1/attention/backends/base_attn.py:308-342).
    Slots beyond the cache are rejected on the host by the reference
    (engine/kv_cache.py:363-420); here they raise.
    Modifies the caches in place and returns them.
    """
    nb, h, bs, d = cache_geometry(k_cache, layout)
    slots = np.asarray(slot_mapping).astype(np.int64).reshape(-1)
    for t, s in enumerate(slots):
        if s < 0:
            continue
        if s >= nb * bs:
            raise ValueError(f"slot {s} out of range")
        blk, off = divmod(int(s), bs)
        for hh in range(h):
            _row(k_cache, layout, blk, hh, off)[...] = new_k[t, hh]
            _row(v_cache, layout, blk, hh, off)[...] = new_v[t, hh]
    return k_cache, v_cache


def kv_write_slots_vectorized(k_cache, v_cache, new_k, new_v, slot_mapping, layout="hnd"):
    """Same result as :func:`kv_write_slots`, vectorised for large inputs."""
    nb, h, bs, d = cache_geometry(k_cache, layout)
    slots = np.asarray(slot_mapping).astype(np.int64).reshape(-1)
    keep = slots >= 0
    if np.any(slots[keep] >= nb * bs):
        raise ValueError("slot out of range")
    idx = np.nonzero(keep)[0]
    blk, off = slots[idx] // bs, slots[idx] % bs
    if layout == "hnd":
        for hh in range(h):
            k_cache[blk, hh, off] = new_k[idx, hh]
            v_cache[blk, hh, off] = new_v[idx, hh]
    else:
        k_cache[blk, off] = new_k[idx]
        v_cache[blk, off] = new_v[idx]
    return k_cache, v_cache


def kv_write_decode(k_cache, v_cache, new_k, new_v, block_table, seq_lens,
                    max_blocks_per_seq=None, layout="hnd"):
    """Decode KV write: the new token of sequence i sits at position seq_lens[i]-1.

    Follows ``kv_write_decode`` (vllm_apple/engine/ops/kv_write.py:66-114 and
    vllm_apple/metal/kernels/paged_attention_fused.metal:55-101): skip when
    seq_len <= 0, when the block index reaches ``max_blocks_per_seq`` or when
    the physical block is negative.
    """
    nb, h, bs, d = cache_geometry(k_cache, layout)
    bt = np.asarray(block_table)
    mb = bt.shape[1] if max_blocks_per_seq is None else max_blocks_per_seq
    for i, L in enumerate(np.asarray(seq_lens).reshape(-1)):
        L = int(L)
        if L <= 0:
            continue
        pos = L - 1
        bi, off = divmod(pos, bs)
        if bi >= mb:
            continue
        blk = int(bt[i, bi])
        if blk < 0 or blk >= nb:
            continue
        for hh in range(h):
            _row(k_cache, layout, blk, hh, off)[...] = new_k[i, hh]
            _row(v_cache, layout, blk, hh, off)[...] = new_v[i, hh]
    return k_cache, v_cache


def write_kv_batch(key_dst, value_dst, key_src, value_src, block_ids, token_offsets,
                   num_tokens, num_kv_heads, head_size, stride_block, stride_head,
                   stride_token):
    """Flat-buffer KV writer with the reference's native signature.

    Follows ``metal_write_kv_batch`` (vllm_apple/metal/native/kv_write.c:33-78):
    for token t and head h, copy ``head_size`` elements of
    ``src[t*H*D + h*D]`` to ``dst[block*stride_block + h*stride_head + off*stride_token]``.
    ``key_dst``/``value_dst`` are flat uint16/float16 arrays, modified in place.
    """
    src_tok = num_kv_heads * head_size
    ks = key_src.reshape(-1)
    vs = value_src.reshape(-1)
    for t in range(num_tokens):
        base = int(block_ids[t]) * stride_block + int(token_offsets[t]) * stride_token
        for hh in range(num_kv_heads):
            dst = base + hh * stride_head
            src = t * src_tok + hh * head_size
            key_dst[dst:dst + head_size] = ks[src:src + head_size]
            value_dst[dst:dst + head_size] = vs[src:src + head_size]


# --------------------------------------------------------------------------
# attention
# --------------------------------------------------------------------------


def _gather_context(k_cache, v_cache, bt_row, ctx_len, head, layout):
    """Rows 0..ctx_len-1 of one sequence's kv head, through its block-table row."""
    nb, h, bs, d = cache_geometry(k_cache, layout)
    nblk = (ctx_len + bs - 1) // bs
    blocks = np.asarray(bt_row[:nblk]).astype(np.int64)
    if np.any(blocks < 0) or np.any(blocks >= nb):
        raise ValueError("invalid block id inside the context")
    if layout == "hnd":
        k = k_cache[blocks, head].reshape(-1, d)[:ctx_len]
        v = v_cache[blocks, head].reshape(-1, d)[:ctx_len]
    else:
        k = k_cache[blocks, :, head].reshape(-1, d)[:ctx_len]
        v = v_cache[blocks, :, head].reshape(-1, d)[:ctx_len]
    return k.astype(np.float64), v.astype(np.float64)


def _softmax_attend(q, k, v, scale):
    """q [G, D], k/v [L, D] -> [G, D]; the reduction of
    ``paged_attention_fused_h128`` (paged_attention_fused.metal:107-201):
    softmax(q k^T * scale) v, with an empty context giving zeros (``l > 0``
    else 0, :190-193)."""
    if k.shape[0] == 0:
        return np.zeros_like(q)
    s = (q @ k.T) * scale
    s = s - s.max(axis=1, keepdims=True)
    p = np.exp(s)
    return (p @ v) / p.sum(axis=1, keepdims=True)


def paged_decode(q, k_cache, v_cache, block_table, seq_lens, scale, layout="hnd",
                 out=None):
    """Single-token decode attention over the paged cache.

    q: [B, Hq, D] (fp16 or fp32); returns float64 [B, Hq, D].
    Sequence i attends to cache positions 0..seq_lens[i]-1 (seq_lens include
    the new token, whose K/V must already be in the cache).  Query head h
    reads kv head h // (Hq/Hkv) (GQA mapping, paged_attention_fused.metal:127).
    Rows with seq_len <= 0 are left as in ``out`` (zeros by default), as the
    reference kernels return without writing (:123-124).
    Follows also MPSAttentionImpl._compute_decode_sdpa
    (vllm_apple/v1/attention/backends/mps_attn.py:284-357).
    """
    q = np.asarray(q)
    B, Hq, D = q.shape
    nb, Hkv, bs, d = cache_geometry(k_cache, layout)
    G = Hq // Hkv
    res = np.zeros((B, Hq, D), np.float64) if out is None else out
    for i in range(B):
        L = int(seq_lens[i])
        if L <= 0:
            continue
        for kh in range(Hkv):
            k, v = _gather_context(k_cache, v_cache, block_table[i], L, kh, layout)
            qq = q[i, kh * G:(kh + 1) * G].astype(np.float64)
            res[i, kh * G:(kh + 1) * G] = _softmax_attend(qq, k, v, scale)
    return res


def paged_prefill(q, k_cache, v_cache, block_table, token_to_seq, positions, scale,
                  layout="hnd", max_blocks_per_seq=None, out=None):
    """Token-parallel causal paged attention (engine prefill semantics).

    Follows ``paged_attention_v2_prefill`` (vllm_apple/metal/kernels/
    paged_attention_v2.metal:375-478): token t of sequence token_to_seq[t]
    attends to cache positions 0..positions[t] through the block table; the
    new tokens' K/V were scattered into the cache beforehand
    (engine/runner.py:1006-1055).  Tokens with an invalid sequence index,
    a negative position, a context longer than the block table or a negative
    block inside the context are skipped (output left untouched, :391-428).
    Returns float64 [T, Hq, D].
    """
    q = np.asarray(q)
    T, Hq, D = q.shape
    nb, Hkv, bs, d = cache_geometry(k_cache, layout)
    G = Hq // Hkv
    bt = np.asarray(block_table)
    mb = bt.shape[1] if max_blocks_per_seq is None else max_blocks_per_seq
    res = np.zeros((T, Hq, D), np.float64) if out is None else out
    tseq = np.asarray(token_to_seq).astype(np.int64)
    tpos = np.asarray(positions).astype(np.int64)
    # per-token validity (paged_attention_v2.metal:391-401, :428)
    ok = (tseq >= 0) & (tseq < bt.shape[0]) & (tpos >= 0)
    ok &= (tpos + bs) // bs <= mb
    for t in np.nonzero(ok)[0]:
        nblk = (tpos[t] + bs) // bs
        if np.any(bt[tseq[t], :nblk] < 0):
            ok[t] = False
    # all tokens of one sequence share its context: one masked softmax per sequence
    for s in np.unique(tseq[ok]):
        toks = np.nonzero(ok & (tseq == s))[0]
        ctx = int(tpos[toks].max()) + 1
        mask = np.arange(ctx)[None, :] <= tpos[toks][:, None]          # [n, ctx]
        for kh in range(Hkv):
            k, v = _gather_context(k_cache, v_cache, bt[s], ctx, kh, layout)
            qq = q[toks, kh * G:(kh + 1) * G].astype(np.float64)        # [n, G, D]
            sc = np.einsum("ngd,cd->ngc", qq, k) * scale
            sc = np.where(mask[:, None, :], sc, -np.inf)
            sc = sc - sc.max(axis=2, keepdims=True)
            p = np.exp(sc)
            res[toks, kh * G:(kh + 1) * G] = np.einsum("ngc,cd->ngd", p, v) / p.sum(
                axis=2, keepdims=True)
    return res


# --------------------------------------------------------------------------
# elementwise ops around the attention step
# --------------------------------------------------------------------------


def rmsnorm(x, weight, eps, residual=None):
    """``y = x * rsqrt(mean(x^2) + eps) * w (+ residual)`` in float64.

    Follows ``rmsnorm_kernel`` / ``rmsnorm_residual_kernel``
    (vllm_apple/engine/ops/rmsnorm.py:78-124, :128-173) and the reference's
    own CPU check (tests/metal/test_transformer_block.py:158-162).
    """
    xf = np.asarray(x).astype(np.float64)
    r = 1.0 / np.sqrt((xf * xf).mean(axis=-1, keepdims=True) + eps)
    y = xf * r * np.asarray(weight).astype(np.float64)
    if residual is not None:
        y = y + np.asarray(residual).astype(np.float64)
    return y


def rope_cos_sin_cache(rotary_dim, max_position, base):
    """fp32 cos/sin tables ``[max_position, rotary_dim // 2]``.

    Restates EngineRoPE._precompute_cache (vllm_apple/engine/ops/
    elementwise.py:680-697) step for step: fp32 ``inv_freq = 1/base**(i/half)``,
    fp32 ``outer(positions, inv_freq)``, then fp32 cos/sin.
    """
    half = rotary_dim // 2
    inv_freq = 1.0 / (base ** (np.arange(0, half, dtype=np.float32) / half))
    pos = np.arange(max_position, dtype=np.float32)
    freqs = np.outer(pos, inv_freq)
    return np.cos(freqs).astype(np.float32), np.sin(freqs).astype(np.float32)


def rope(q, k, cos_cache, sin_cache, positions, rotary_dim=None, is_neox=True):
    """Rotate q [T, Hq, D] and k [T, Hkv, D]; returns float64 copies.

    Neox (split-half) follows ``rope_neox_kernel`` (elementwise.py:185-239):
    pairs (x[i], x[i + rot/2]); GPT-J follows ``rope_kernel`` (:129-180):
    pairs (x[2i], x[2i+1]).  Products and the difference are taken in fp32 as
    the kernels do (``q0*c - q1*s`` and ``q0*s + q1*c``) and returned as
    float64 for comparison.  Dimensions beyond ``rotary_dim`` pass through.
    """
    D = q.shape[-1]
    rot = rotary_dim or D
    half = rot // 2
    pos = np.asarray(positions).astype(np.int64)
    c = cos_cache[pos][:, None, :].astype(np.float32)
    s = sin_cache[pos][:, None, :].astype(np.float32)

    def apply(x):
        x = np.asarray(x).astype(np.float32)
        y = x.copy()
        if is_neox:
            a, b = x[..., :half], x[..., half:rot]
            y[..., :half] = a * c - b * s
            y[..., half:rot] = a * s + b * c
        else:
            a, b = x[..., 0:rot:2], x[..., 1:rot:2]
            y[..., 0:rot:2] = a * c - b * s
            y[..., 1:rot:2] = a * s + b * c
        return y.astype(np.float64)

    return apply(q), apply(k)


def silu_mul(gate, up):
    """``silu(g) * u = g / (1 + exp(-g)) * u`` in float64.

    Follows ``silu_mul_kernel`` (vllm_apple/engine/ops/elementwise.py:114-124).
    """
    g = np.asarray(gate).astype(np.float64)
    u = np.asarray(up).astype(np.float64)
    return g / (1.0 + np.exp(-g)) * u


# --------------------------------------------------------------------------
# step-level helpers
# --------------------------------------------------------------------------


def prefill_metadata(query_start_loc, seq_lens, block_table, block_size):
    """(token_to_seq, positions, slot_mapping) of a batch laid out by query_start_loc.

    token_to_seq follows the reference runner (vllm_apple/engine/runner.py:526-546,
    :642-683: repeat_interleave of sequence ids by query length); the i-th new
    token of sequence s sits at position seq_lens[s] - query_len + i and its slot
    is block_table[s][pos // bs] * bs + pos % bs (-1 when the block is unused).
    """
    qsl = np.asarray(query_start_loc).astype(np.int64)
    L = np.asarray(seq_lens).astype(np.int64)
    bt = np.asarray(block_table).astype(np.int64)
    lens = qsl[1:] - qsl[:-1]
    if np.any(lens < 0):
        raise ValueError("query_start_locs must be non-decreasing")
    tok = np.repeat(np.arange(len(lens)), lens)
    pos = np.concatenate([np.arange(L[s] - n, L[s]) for s, n in enumerate(lens)]) \
        if len(tok) else np.zeros(0, np.int64)
    slots = np.full(len(tok), -1, np.int64)
    for t, (s, p) in enumerate(zip(tok, pos)):
        if p >= 0 and p // block_size < bt.shape[1] and bt[s, p // block_size] >= 0:
            slots[t] = bt[s, p // block_size] * block_size + p % block_size
    return tok.astype(np.int32), pos.astype(np.int32), slots


def kv_sync_blocks(src_k, src_v, dst_k, dst_v, block_table, seq_lens, src_layout="nhd",
                   dst_layout="hnd"):
    """Copy every active block from one cache layout to the other, in place.

    Follows EngineKVCache.sync_from_torch_cache (vllm_apple/engine/kv_cache.py:
    518-684): the active blocks are block_table[s][i] for i < ceil(seq_len/bs)
    (capped at the table width), ids >= 0; ids beyond the cache are skipped; each
    copied block is the (bs, H, D) -> (H, bs, D) permutation of the source.
    """
    nb, H, bs, D = cache_geometry(src_k, src_layout)
    bt = np.asarray(block_table)
    active = set()
    for s, L in enumerate(np.asarray(seq_lens).reshape(-1)):
        n = (int(L) + bs - 1) // bs
        for i in range(min(n, bt.shape[1])):
            b = int(bt[s, i])
            if b >= 0:
                active.add(b)
    for b in active:
        if b >= nb:
            continue
        for hh in range(H):
            for t in range(bs):
                _row(dst_k, dst_layout, b, hh, t)[...] = _row(src_k, src_layout, b, hh, t)
                _row(dst_v, dst_layout, b, hh, t)[...] = _row(src_v, src_layout, b, hh, t)
    return dst_k, dst_v


# --------------------------------------------------------------------------
# top-k logits
# --------------------------------------------------------------------------


def _topk_keys(bits: np.ndarray) -> np.ndarray:
    """Order-preserving integer key of fp16 bit patterns; 0 for NaN and -inf."""
    b = bits.astype(np.int64)
    key = np.where(b & 0x8000, (~b) & 0xFFFF, b | 0x8000)
    bad = ((b & 0x7FFF) > 0x7C00) | (b == 0xFC00)
    return np.where(bad, 0, key)


def topk(logits, k):
    """Top-k per row of fp16 ``logits [T, V]`` -> (int32 indices, fp16 values), each
    ``[T, k]``, largest first.

    Follows EngineTopK's selection (vllm_apple/engine/ops/topk.py:80-151, the
    insertion list of the k best values initialised to -inf, and its merge
    :153-216): a logit is kept only if it is greater than -inf (so NaN and -inf never
    are), rows with fewer than k kept logits are padded with index -1 and value
    -inf (the list's initial entries, written out at :218-226).  Order between equal
    values is by the lower index, and +0 ranks above -0 (the bit-level order);
    the reference leaves both to its thread layout.
    """
    x = np.ascontiguousarray(np.asarray(logits, dtype=np.float16))
    T, V = x.shape
    keys = _topk_keys(x.view(np.uint16))
    idx = np.full((T, k), -1, dtype=np.int32)
    val = np.full((T, k), -np.inf, dtype=np.float16)
    cols = np.arange(V)
    for t in range(T):
        order = np.lexsort((cols, -keys[t]))  # key desc, index asc
        order = order[keys[t][order] > 0][:k]
        idx[t, :len(order)] = order
        val[t, :len(order)] = x[t, order]
    return idx, val


def topk_insertion_lists(logits, k, threads=64):
    """Pure-Python restatement of the reference kernel's own two stages (per-thread
    insertion lists over a strided slice of the row, then a pairwise tree merge,
    vllm_apple/engine/ops/topk.py:80-216) for small cases; returns the values in
    the reference's output order (used to pin ``topk`` by value)."""
    x = np.asarray(logits, dtype=np.float16)
    T, V = x.shape
    out_v = np.full((T, k), -np.inf, dtype=np.float32)
    out_i = np.full((T, k), -1, dtype=np.int64)

    def insert(vals, idxs, v, i):
        if v > vals[k - 1]:
            pos = next(j for j in range(k) if v > vals[j])
            vals.insert(pos, v)
            idxs.insert(pos, i)
            del vals[k:], idxs[k:]

    for t in range(T):
        lists = []
        for th in range(threads):
            vals, idxs = [-np.inf] * k, [-1] * k
            for i in range(th, V, threads):
                insert(vals, idxs, float(x[t, i]), i)
            lists.append((vals, idxs))
        stride = threads // 2
        while stride > 0:
            for th in range(stride):
                vals, idxs = lists[th]
                ov, oi = lists[th + stride]
                for v, i in zip(ov, oi):
                    insert(vals, idxs, v, i)
            stride //= 2
        out_v[t], out_i[t] = lists[0][0], lists[0][1]
    return out_i, out_v.astype(np.float16)
