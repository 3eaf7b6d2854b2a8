/*
 * vllm_apple_b200 -- C ABI of the B200 (sm_100a) paged-attention hot path.
 *
 * One shared library, libvllm_apple_b200.so, exports the entry points below.
 * They take plain device pointers, 64-bit sizes and element strides and a
 * cudaStream_t passed as `void *` (NULL = legacy default stream); nothing in
 * the signatures is a torch or CUDA C++ type.  Every call only enqueues work
 * on `stream` (never synchronises) and returns an int status:
 *
 *   VA_OK                0  launched
 *   VA_ERR_INVALID_ARG   1  bad size / stride / pointer alignment (nothing launched)
 *   VA_ERR_UNSUPPORTED   2  shape outside the compiled variants (nothing launched)
 *   VA_ERR_LAUNCH        3  the CUDA launch itself failed
 *   VA_ERR_WORKSPACE     4  workspace missing or too small
 *   VA_ERR_SCRATCH_LIMIT 5  shape needs more than the built-in scratch (nothing launched)
 *
 * Data-dependent problems found on the device (a slot or block id outside the
 * cache, a context longer than the block table, a bounded wait that ran out)
 * never fault: the offending row is skipped and a bit is OR-ed into the
 * optional device word `err_flag` (VA_FLAG_*), which the host reads when it
 * chooses to synchronise.
 *
 * All K/V/Q/O tensors are IEEE fp16 stored as 2-byte elements.  A paged KV
 * cache is addressed by (block, kv_head, offset-in-block) through three
 * element strides; the head_size axis is contiguous.  The two layouts of the
 * reference are both expressible:
 *   engine layout [num_blocks, num_kv_heads, block_size, head_size]
 *       (vllm_apple/engine/kv_cache.py:136-151):
 *       s_block = H*bs*D, s_head = bs*D, s_token = D
 *   vLLM layout   [num_blocks, block_size, num_kv_heads, head_size]
 *       (vllm_apple/v1/attention/backends/base_attn.py:113-125):
 *       s_block = bs*H*D, s_head = D, s_token = H*D
 */
#ifndef VLLM_APPLE_B200_H
#define VLLM_APPLE_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define VA_API __attribute__((visibility("default")))
#else
#define VA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define VA_OK 0
#define VA_ERR_INVALID_ARG 1
#define VA_ERR_UNSUPPORTED 2
#define VA_ERR_LAUNCH 3
#define VA_ERR_WORKSPACE 4
#define VA_ERR_SCRATCH_LIMIT 5

#define VA_FLAG_BAD_SLOT 0x1        /* slot >= num_blocks*block_size, or < -1 */
#define VA_FLAG_BAD_BLOCK 0x2       /* block id < 0 or >= num_blocks inside a context */
#define VA_FLAG_CTX_OVERFLOW 0x4    /* context longer than max_blocks_per_seq*block_size
                                       or than the max_seq_len the grid was sized for */
#define VA_FLAG_WAIT_TIMEOUT 0x8    /* a bounded barrier wait gave up */
#define VA_FLAG_BAD_POSITION 0x10   /* RoPE position outside [0, max_position) */

/* Library version string, e.g. "vllm_apple_b200 0.1.0 sm_100a". */
VA_API const char *va_version(void);

/* ---------------------------------------------------------------------------
 * KV-cache writes (bit-exact copies)
 * ------------------------------------------------------------------------- */

/* Scatter new K/V rows [num_tokens, num_kv_heads, head_size] into the cache by
 * slot = block*block_size + offset.  slot == -1 (any negative) is padding and
 * skipped.  slot_mapping is int32 (slot_is_i64 = 0) or int64 (slot_is_i64 = 1).
 * Replaces KVWriteOp.encode_prefill / kv_write_prefill
 * (vllm_apple/engine/ops/kv_write.py:336-402, :118-156) and the vLLM-layout
 * scatter BaseAppleAttentionImpl._update_kv_cache_scatter
 * (vllm_apple/v1/attention/backends/base_attn.py:308-342).
 * new_s_token/new_s_head are element strides of the new K/V rows (rows may be
 * views into a planar QKV buffer, vllm_apple/engine/runner.py:919-934). */
VA_API int va_kv_write_slots(void *k_cache, void *v_cache, const void *new_k, const void *new_v,
                      const void *slot_mapping, int slot_is_i64, int64_t num_tokens,
                      int num_kv_heads, int head_size, int block_size, int64_t num_blocks,
                      int64_t s_block, int64_t s_head, int64_t s_token,
                      int64_t new_s_token, int64_t new_s_head, int32_t *err_flag,
                      void *stream);

/* Decode KV write: the new row of sequence i goes to position seq_lens[i]-1
 * through block_table (int32 [num_seqs, max_blocks_per_seq]).  Skips rows with
 * seq_len <= 0, a block index >= max_blocks_per_seq or a negative block.
 * Replaces KVWriteOp.encode_decode / kv_write_decode
 * (vllm_apple/engine/ops/kv_write.py:261-334, :66-114;
 *  vllm_apple/metal/kernels/paged_attention_fused.metal:55-101). */
VA_API int va_kv_write_decode(void *k_cache, void *v_cache, const void *new_k, const void *new_v,
                       const int32_t *block_table, const int32_t *seq_lens, int64_t num_seqs,
                       int64_t max_blocks_per_seq, int num_kv_heads, int head_size,
                       int block_size, int64_t num_blocks, int64_t s_block, int64_t s_head,
                       int64_t s_token, int64_t new_s_token, int64_t new_s_head,
                       int32_t *err_flag, void *stream);

/* Device-side twin of the reference's native writer, same argument list and
 * meaning as metal_write_kv_batch (vllm_apple/metal/native/kv_write.c:33-46;
 * ctypes binding vllm_apple/metal/bridge/metal_paged_attention_v2.py:563-607)
 * plus a stream: key/value_dst are device cache pointers, key/value_src device
 * rows [num_tokens, num_kv_heads, head_size], block_ids/token_offsets device
 * int64 [num_tokens], strides in elements.  Pairs with a negative block id are
 * skipped. */
VA_API int va_write_kv_batch(uint16_t *key_dst, uint16_t *value_dst, const uint16_t *key_src,
                      const uint16_t *value_src, const int64_t *block_ids,
                      const int64_t *token_offsets, int num_tokens, int num_kv_heads,
                      int head_size, int stride_block, int stride_head, int stride_token,
                      void *stream);

/* ---------------------------------------------------------------------------
 * Paged attention
 * ------------------------------------------------------------------------- */

/* Bytes of workspace va_paged_decode needs for this shape (0 when no sequence
 * needs neither split-KV partials nor an ordering).  The workspace holds fp32
 * split partials and, for large batches (at least 1024 sequence x kv-head CTAs),
 * the longest-first order of the sequences (written
 * by the call itself); it needs no initialisation.  Calls that share a workspace
 * must not overlap on the GPU (stream order is enough). */
VA_API size_t va_paged_decode_workspace_size(int64_t num_seqs, int num_query_heads, int num_kv_heads,
                                      int head_size, int block_size, int64_t max_seq_len);

/* Single-token decode attention over the paged cache, with the fused KV write.
 *   out  [num_seqs, Hq, D] at (o_s_token, o_s_head); q likewise (q_s_*).
 *   seq_lens include the new token; sequence i attends to positions
 *   0..seq_lens[i]-1.  Rows with seq_len <= 0 are skipped (out untouched).
 *   new_k/new_v: when non-NULL, row i ([num_seqs, Hkv, D] at new_s_*) is
 *   written to position seq_lens[i]-1 of the cache and used as that position's
 *   K/V (fused write); when NULL the cache must already hold it.
 *   max_seq_len bounds every seq_len (it sizes the split-KV grid).
 * Replaces PagedAttentionOp.encode_decode_fused
 * (vllm_apple/engine/ops/attention.py:369-537) -- kernels kv_write_decode +
 * paged_attention_fused_h128 / paged_attention_fused_generic
 * (vllm_apple/metal/kernels/paged_attention_fused.metal:55-328) -- and the
 * decode branch of MetalAttentionImpl.forward
 * (vllm_apple/v1/attention/backends/metal_attn.py:766-845). */
VA_API int va_paged_decode(void *out, const void *q, void *k_cache, void *v_cache,
                    const int32_t *block_table, const int32_t *seq_lens,
                    const void *new_k, const void *new_v, int64_t num_seqs,
                    int num_query_heads, int num_kv_heads, int head_size, int block_size,
                    int64_t max_blocks_per_seq, int64_t max_seq_len, int64_t num_blocks,
                    float scale, int64_t s_block, int64_t s_head, int64_t s_token,
                    int64_t q_s_token, int64_t q_s_head, int64_t o_s_token,
                    int64_t o_s_head, int64_t new_s_token, int64_t new_s_head,
                    void *workspace, size_t workspace_bytes, int32_t *err_flag,
                    void *stream);

/* va_paged_decode for callers that cannot allocate device memory: a host that
 * only reaches this library through the C ABI and has no CUDA allocator of its
 * own, or a serving loop whose memory is fixed up front and must not call
 * cudaMalloc/cudaFree while running.  Same arguments and results as
 * va_paged_decode minus the workspace: the split-KV partials go to a scratch
 * array built into the library, VA_DECODE_STATIC_SCRATCH_BYTES per GPU, held by
 * every GPU that loads the library until the process exits.  Shapes whose
 * va_paged_decode_workspace_size exceeds it return VA_ERR_SCRATCH_LIMIT and
 * launch nothing; a shape va_paged_decode rejects gets the same status here.
 * The first call on a device (with that device current) looks up the array's
 * device address; make that first call before any stream capture.  The address
 * is kept for the life of the process's CUDA context on that device: after a
 * cudaDeviceReset of that device, do not call this entry point again in the
 * same process.  All calls share the one array, so calls that overlap on the GPU
 * (different streams, no ordering between them) race; calls ordered on one
 * stream do not.  Allocates nothing.  It has no counterpart in the reference. */
#define VA_DECODE_STATIC_SCRATCH_BYTES (32u << 20)
VA_API int va_paged_decode_noalloc(void *out, const void *q, void *k_cache, void *v_cache,
                                   const int32_t *block_table, const int32_t *seq_lens,
                                   const void *new_k, const void *new_v, int64_t num_seqs,
                                   int num_query_heads, int num_kv_heads, int head_size,
                                   int block_size, int64_t max_blocks_per_seq,
                                   int64_t max_seq_len, int64_t num_blocks, float scale,
                                   int64_t s_block, int64_t s_head, int64_t s_token,
                                   int64_t q_s_token, int64_t q_s_head, int64_t o_s_token,
                                   int64_t o_s_head, int64_t new_s_token, int64_t new_s_head,
                                   int32_t *err_flag, void *stream);

/* Bytes of workspace va_paged_prefill needs: the tile plan and the split-KV
 * partials of the one-token rows (decode rows of a mixed batch), which are
 * routed to the decode kernel.  No initialisation needed. */
VA_API size_t va_paged_prefill_workspace_size(int64_t num_tokens, int64_t num_seqs,
                                              int num_query_heads, int num_kv_heads,
                                              int head_size, int block_size,
                                              int64_t max_blocks_per_seq);

/* Token-parallel causal paged attention (prefill / chunked-prefill mixed batch).
 * Token t of sequence token_to_seq[t] attends to cache positions
 * 0..positions[t] (the new tokens' K/V already written, e.g. by
 * va_kv_write_slots).  Tokens with an invalid sequence, a negative position, a
 * context longer than the block table or a negative block inside the context
 * are skipped (out untouched).  Runs of consecutive tokens of one sequence are
 * processed as tensor-core tiles (tcgen05 UMMA for head_size 64/128); one-token
 * runs go to the split-KV decode kernel.  With tensor-core tiles, those rows
 * run on one library-owned side stream per device, forked from and joined back
 * to `stream` with events (so the call stays stream-ordered and capturable);
 * calls on one device take that side stream in turn (a mutex), so eager calls
 * from several threads serialise on it, and a stream capture that includes a
 * prefill call must not overlap an eager prefill call on the same device.
 * Replaces PagedAttentionOp.encode_prefill
 * (vllm_apple/engine/ops/attention.py:290-367) -- kernel
 * paged_attention_v2_prefill (vllm_apple/metal/kernels/paged_attention_v2.metal:375-478). */
VA_API int va_paged_prefill(void *out, const void *q, const void *k_cache, const void *v_cache,
                     const int32_t *block_table, const int32_t *token_to_seq,
                     const int32_t *positions, int64_t num_tokens, int64_t num_seqs,
                     int num_query_heads, int num_kv_heads, int head_size, int block_size,
                     int64_t max_blocks_per_seq, int64_t num_blocks, float scale,
                     int64_t s_block, int64_t s_head, int64_t s_token, int64_t q_s_token,
                     int64_t q_s_head, int64_t o_s_token, int64_t o_s_head,
                     void *workspace, size_t workspace_bytes, int32_t *err_flag,
                     void *stream);

/* ---------------------------------------------------------------------------
 * Step-level ops around the attention call
 * ------------------------------------------------------------------------- */

/* Neox rotary embedding of q [T, Hq, D] and k [T, Hkv, D] (in place, rot = D)
 * fused with the scatter of the rotated k and of v [T, Hkv, D] into the paged
 * cache by slot (-1 = padding, skipped): one pass over k and v instead of a
 * RoPE pass and a KV-write pass.  Tokens with a position outside
 * [0, max_position) are left untouched (VA_FLAG_BAD_POSITION).
 * Replaces the sequence EngineRoPE.encode + KVWriteOp.encode_prefill of the
 * reference runner (vllm_apple/engine/runner.py:942-1055; kernels
 * rope_neox_kernel, vllm_apple/engine/ops/elementwise.py:185-239, and
 * kv_write_prefill, vllm_apple/engine/ops/kv_write.py:118-156). */
VA_API int va_rope_kv_write_slots(void *q, void *k, const void *v, void *k_cache, void *v_cache,
                                  const float *cos_cache, const float *sin_cache,
                                  const int32_t *positions, const void *slot_mapping,
                                  int slot_is_i64, int64_t num_tokens, int num_heads,
                                  int num_kv_heads, int head_size, int block_size,
                                  int64_t num_blocks, int64_t max_position, int64_t q_s_token,
                                  int64_t k_s_token, int64_t v_s_token, int64_t s_block,
                                  int64_t s_head, int64_t s_token, int32_t *err_flag,
                                  void *stream);

/* Per-token prefill metadata on the device: for tokens first_token ..
 * first_token+num_tokens-1 of a batch laid out by query_start_loc
 * (int32 [num_seqs+1]), token_to_seq[t] = its sequence and positions[t] =
 * seq_lens[s] - query_len(s) + (index within the sequence's new tokens);
 * slot_mapping (optional, int64) = block_table[s][pos/bs]*bs + pos%bs or -1.
 * Replaces the host-side derivation in the reference runner
 * (vllm_apple/engine/runner.py:526-546, :642-683). */
VA_API int va_build_prefill_metadata(const int32_t *query_start_loc, const int32_t *seq_lens,
                                     const int32_t *block_table, int64_t num_seqs,
                                     int64_t first_token, int64_t num_tokens,
                                     int64_t max_blocks_per_seq, int block_size,
                                     int32_t *token_to_seq, int32_t *positions,
                                     int64_t *slot_mapping, void *stream);

/* Copy every active block -- block_table[s][i] for i < ceil(seq_lens[s]/bs),
 * ids in [0, num_blocks) -- of K and V from one cache layout to another
 * (strides in elements, e.g. vLLM (nb, bs, H, D) -> engine [nb, H, bs, D]).
 * Bit-exact.  Replaces EngineKVCache.sync_from_torch_cache
 * (vllm_apple/engine/kv_cache.py:518-684). */
VA_API int va_kv_sync_blocks(const void *src_k, const void *src_v, void *dst_k, void *dst_v,
                             const int32_t *block_table, const int32_t *seq_lens,
                             int64_t num_seqs, int64_t max_blocks_per_seq, int num_kv_heads,
                             int head_size, int block_size, int64_t num_blocks,
                             int64_t src_s_block, int64_t src_s_head, int64_t src_s_token,
                             int64_t dst_s_block, int64_t dst_s_head, int64_t dst_s_token,
                             void *stream);

/* ---------------------------------------------------------------------------
 * Elementwise ops around the attention step
 * ------------------------------------------------------------------------- */

/* out[t,:] = half(x[t,:] * rsqrt(mean(x[t,:]^2) + eps) * w [+ residual[t,:]]), fp32 math.
 * residual may be NULL.  Row strides in elements (x_s_token, out_s_token,
 * res_s_token).  Replaces EngineRMSNorm.encode -- rmsnorm_kernel /
 * rmsnorm_residual_kernel (vllm_apple/engine/ops/rmsnorm.py:226-321, :78-173). */
VA_API int va_rmsnorm(void *out, const void *x, const void *weight, const void *residual,
               int64_t num_tokens, int64_t hidden_size, float eps, int64_t x_s_token,
               int64_t out_s_token, int64_t res_s_token, void *stream);

/* In-place rotary embedding of q [T, Hq, D] (row stride q_s_token) and
 * k [T, Hkv, D] (k_s_token) with fp32 tables cos/sin [max_position, rot/2] and
 * int32 positions [T].  is_neox = 1: split-half pairs (x[i], x[i+rot/2]);
 * 0: interleaved pairs (x[2i], x[2i+1]).  Positions outside
 * [0, max_position) leave the token untouched and set VA_FLAG_BAD_POSITION.
 * Replaces EngineRoPE.encode -- rope_neox_kernel / rope_kernel
 * (vllm_apple/engine/ops/elementwise.py:700-766, :185-239, :129-180). */
VA_API int va_rope(void *q, void *k, const float *cos_cache, const float *sin_cache,
            const int32_t *positions, int64_t num_tokens, int num_heads, int num_kv_heads,
            int head_size, int rotary_dim, int64_t max_position, int64_t q_s_token,
            int64_t k_s_token, int is_neox, int32_t *err_flag, void *stream);

/* out[i] = half(silu(gate[i]) * up[i]) = half(g / (1 + exp(-g)) * u), fp32 math.
 * Replaces EngineElementwiseOps.encode_silu_mul -- silu_mul_kernel
 * (vllm_apple/engine/ops/elementwise.py:496-532, :114-124). */
VA_API int va_silu_mul(void *out, const void *gate, const void *up, int64_t num_elements,
                void *stream);

/* Top-k logits per token: indices[T][k] (int32) and values[T][k] (fp16), largest
 * first, ties by the lower index.  logits is fp16 [T][row_stride] (row_stride >=
 * vocab_size elements).  NaN and -inf are never selected; rows with fewer than
 * k other logits are padded with index -1 and value -inf.  1 <= k <= 1024.
 * Replaces EngineTopK.encode -- topk_select / topk_select_small_k
 * (vllm_apple/engine/ops/topk.py:57-283, :317-399). */
VA_API int va_topk(int32_t *indices, void *values, const void *logits, int64_t num_tokens,
                   int64_t vocab_size, int64_t row_stride, int k, void *stream);

/* The same selection with a caller workspace (kept for callers that pass one): every
 * row is selected whole by one CTA, so va_topk_workspace_size returns 0 and any
 * workspace (also none) works; results equal va_topk's. */
VA_API size_t va_topk_workspace_size(int64_t num_tokens, int64_t vocab_size, int k);
VA_API int va_topk_ws(int32_t *indices, void *values, const void *logits, int64_t num_tokens,
                      int64_t vocab_size, int64_t row_stride, int k, void *workspace,
                      size_t workspace_bytes, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* VLLM_APPLE_B200_H */
