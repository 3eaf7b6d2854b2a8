"""torch-CPU restatement of the reference's pure-PyTorch attention path (TEST ORACLE).

Test infrastructure only.  This is the code path the reference itself runs
when no Metal kernel is used (backend "MPS_ATTN"), restated so that it runs
without the reference tree (which is absent on the GPU box).  ``bench.py``
times it on the host cores as the reference CPU baseline.

Follows:
  * ``BaseAppleAttentionImpl._update_kv_cache_scatter``
    (vllm_apple/v1/attention/backends/base_attn.py:308-342)
  * ``MPSAttentionImpl.forward`` (vllm_apple/v1/attention/backends/mps_attn.py:207-282)
  * ``MPSAttentionImpl._compute_decode_sdpa`` (mps_attn.py:284-357)
  * ``BaseAppleAttentionImpl._compute_attention_sdpa`` (base_attn.py:223-306)

Cache tensors use the vLLM layout ``[num_blocks, block_size, num_kv_heads, head_size]``.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def update_kv_cache_scatter(key, value, key_cache, value_cache, slot_mapping):
    """Vectorised scatter of [T, H, D] rows into the flattened slot axis."""
    T, H, D = key.shape
    kf = key_cache.view(-1, key_cache.shape[2], key_cache.shape[3])
    vf = value_cache.view(-1, value_cache.shape[2], value_cache.shape[3])
    idx = slot_mapping.to(torch.int64).view(-1, 1, 1).expand(T, H, D)
    kf.scatter_(0, idx, key)
    vf.scatter_(0, idx, value)


def compute_decode_sdpa(query, key_cache, value_cache, block_table, seq_lens, scale,
                        num_queries_per_kv, output):
    """Per-sequence gather + GQA repeat + SDPA, one decode token per sequence."""
    nb, bs, H, D = key_cache.shape
    for i in range(query.shape[0]):
        L = int(seq_lens[i])
        nblk = (L + bs - 1) // bs
        blocks = block_table[i, :nblk]
        k = key_cache[blocks].view(-1, H, D)[:L].transpose(0, 1)
        v = value_cache[blocks].view(-1, H, D)[:L].transpose(0, 1)
        if num_queries_per_kv != 1:
            k = k.repeat_interleave(num_queries_per_kv, dim=0)
            v = v.repeat_interleave(num_queries_per_kv, dim=0)
        q = query[i:i + 1].transpose(0, 1)
        o = F.scaled_dot_product_attention(q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0),
                                           attn_mask=None, dropout_p=0.0, is_causal=False,
                                           scale=scale)
        output[i] = o.squeeze(0).transpose(0, 1).squeeze(0)
    return output


def compute_prefill_sdpa(query, key, value, query_start_loc, scale, num_queries_per_kv,
                         output):
    """Causal SDPA over the new tokens of each sequence only (the reference's
    plugin prefill; it ignores any prior cached context)."""
    locs = [int(x) for x in query_start_loc]
    for s in range(len(locs) - 1):
        a, b = locs[s], locs[s + 1]
        if b == a:
            continue
        q = query[a:b].transpose(0, 1)
        k = key[a:b].transpose(0, 1)
        v = value[a:b].transpose(0, 1)
        if num_queries_per_kv != 1:
            k = k.repeat_interleave(num_queries_per_kv, dim=0)
            v = v.repeat_interleave(num_queries_per_kv, dim=0)
        o = F.scaled_dot_product_attention(q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0),
                                           attn_mask=None, dropout_p=0.0, is_causal=True,
                                           scale=scale)
        output[a:b] = o.squeeze(0).transpose(0, 1)
    return output


def forward(query, key, value, kv_cache, block_table, seq_lens, slot_mapping,
            query_start_loc, num_decode_tokens, scale, num_kv_heads, output):
    """MPSAttentionImpl.forward for a batch with decodes first."""
    T = query.shape[0]
    G = query.shape[1] // num_kv_heads
    update_kv_cache_scatter(key[:T], value[:T], kv_cache[0], kv_cache[1], slot_mapping[:T])
    if T > num_decode_tokens:
        compute_prefill_sdpa(query[num_decode_tokens:], key[num_decode_tokens:],
                             value[num_decode_tokens:],
                             [x - num_decode_tokens for x in query_start_loc[num_decode_tokens:]],
                             scale, G, output[num_decode_tokens:])
    if num_decode_tokens:
        compute_decode_sdpa(query[:num_decode_tokens], kv_cache[0], kv_cache[1], block_table,
                            seq_lens, scale, G, output[:num_decode_tokens])
    return output


def engine_prefill_sdpa(query, key_cache, value_cache, block_table, token_to_seq, positions,
                        scale, num_queries_per_kv, output):
    """Engine-semantics token-parallel prefill on CPU: each run of tokens of
    one sequence attends to its cached context 0..position through the block
    table (paged_attention_v2.metal:375-478), done as gather + SDPA with an
    absolute-position causal mask."""
    nb, bs, H, D = key_cache.shape
    T = query.shape[0]
    t = 0
    while t < T:
        s = int(token_to_seq[t])
        e = t
        while e < T and int(token_to_seq[e]) == s:
            e += 1
        pos = positions[t:e].to(torch.int64)
        ctx = int(pos.max()) + 1
        nblk = (ctx + bs - 1) // bs
        blocks = block_table[s, :nblk].to(torch.int64)
        k = key_cache[blocks].view(-1, H, D)[:ctx].transpose(0, 1)
        v = value_cache[blocks].view(-1, H, D)[:ctx].transpose(0, 1)
        if num_queries_per_kv != 1:
            k = k.repeat_interleave(num_queries_per_kv, dim=0)
            v = v.repeat_interleave(num_queries_per_kv, dim=0)
        mask = torch.arange(ctx)[None, :] <= pos[:, None]
        q = query[t:e].transpose(0, 1)
        o = F.scaled_dot_product_attention(q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0),
                                           attn_mask=mask, dropout_p=0.0, scale=scale)
        output[t:e] = o.squeeze(0).transpose(0, 1)
        t = e
    return output
