/*
 * Plain-C restatement of the reference's KV-cache writers (TEST ORACLE).
 *
 * Test infrastructure only: built by oracle/Makefile into oracle/_build and
 * loaded by tests through ctypes as a byte-exact checker of the CUDA
 * scatter kernels.
 *
 * oracle_kv_write_slots follows kv_write_prefill
 *   (vllm_apple/engine/ops/kv_write.py:118-156): slot < 0 is padding.
 * oracle_kv_write_decode follows kv_write_decode
 *   (vllm_apple/engine/ops/kv_write.py:66-114).
 * Strides are in 2-byte elements; the innermost (head_size) axis is contiguous.
 */
#include <stdint.h>
#include <string.h>

void oracle_kv_write_slots(uint16_t *k_cache, uint16_t *v_cache,
                           const uint16_t *new_k, const uint16_t *new_v,
                           const int64_t *slots, int64_t num_tokens,
                           int num_kv_heads, int head_size, int block_size,
                           int64_t num_blocks, int64_t s_block, int64_t s_head,
                           int64_t s_token, int64_t n_token, int64_t n_head) {
    for (int64_t t = 0; t < num_tokens; ++t) {
        int64_t slot = slots[t];
        if (slot < 0 || slot >= num_blocks * block_size) continue;
        int64_t blk = slot / block_size, off = slot % block_size;
        for (int h = 0; h < num_kv_heads; ++h) {
            int64_t dst = blk * s_block + h * s_head + off * s_token;
            int64_t src = t * n_token + h * n_head;
            memcpy(k_cache + dst, new_k + src, (size_t)head_size * 2);
            memcpy(v_cache + dst, new_v + src, (size_t)head_size * 2);
        }
    }
}

void oracle_kv_write_decode(uint16_t *k_cache, uint16_t *v_cache,
                            const uint16_t *new_k, const uint16_t *new_v,
                            const int32_t *block_table, const int32_t *seq_lens,
                            int64_t num_seqs, int64_t max_blocks_per_seq,
                            int num_kv_heads, int head_size, int block_size,
                            int64_t num_blocks, int64_t s_block, int64_t s_head,
                            int64_t s_token, int64_t n_token, int64_t n_head) {
    for (int64_t i = 0; i < num_seqs; ++i) {
        int32_t L = seq_lens[i];
        if (L <= 0) continue;
        int64_t pos = L - 1, bi = pos / block_size, off = pos % block_size;
        if (bi >= max_blocks_per_seq) continue;
        int64_t blk = block_table[i * max_blocks_per_seq + bi];
        if (blk < 0 || blk >= num_blocks) continue;
        for (int h = 0; h < num_kv_heads; ++h) {
            int64_t dst = blk * s_block + h * s_head + off * s_token;
            int64_t src = i * n_token + h * n_head;
            memcpy(k_cache + dst, new_k + src, (size_t)head_size * 2);
            memcpy(v_cache + dst, new_v + src, (size_t)head_size * 2);
        }
    }
}
