// KV-cache write kernels: bit-exact scatter of new K/V rows into paged blocks.
//
// Memory-bound byte movement: one thread moves one 16-byte chunk of a K row
// and the matching chunk of the V row (coalesced: consecutive threads walk a
// row, then the next head, then the next token).  When pointers or strides are
// not 16-byte aligned the same kernel runs with 4- or 2-byte chunks.
#include "common.cuh"

namespace {

template <int VEC>  // elements (2-byte) per chunk: 8, 2 or 1
struct Chunk;
template <>
struct Chunk<8> {
  using T = uint4;
};
template <>
struct Chunk<2> {
  using T = uint32_t;
};
template <>
struct Chunk<1> {
  using T = uint16_t;
};

struct KVWriteArgs {
  uint16_t *kc, *vc;
  const uint16_t *nk, *nv;
  int64_t rows;  // tokens (or sequences) * heads
  int heads, head_size, block_size;
  int64_t num_blocks;
  int64_t s_block, s_head, s_token, n_token, n_head;
  int32_t *err;
};

// mode 0: slot_mapping int32, 1: slot_mapping int64,
// mode 2: decode (block_table + seq_lens), 3: (block_ids, token_offsets) int64 pairs.
template <int VEC, int MODE>
__global__ void __launch_bounds__(256) kv_write_kernel(KVWriteArgs a, const void *idx0,
                                                       const void *idx1, int64_t max_blocks) {
  using T = typename Chunk<VEC>::T;
  const int cpr = a.head_size / VEC;  // chunks per row
  const int64_t total = a.rows * cpr;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / cpr;
    const int c = static_cast<int>(i - row * cpr);
    const int64_t tok = row / a.heads;
    const int h = static_cast<int>(row - tok * a.heads);
    int64_t blk, off;
    if (MODE == 0 || MODE == 1) {
      const int64_t slot = MODE == 0 ? (int64_t) static_cast<const int32_t *>(idx0)[tok]
                                     : static_cast<const int64_t *>(idx0)[tok];
      if (slot < 0) {  // -1 is padding; anything below is an invalid slot
        if (slot < -1 && h == 0 && c == 0) va::raise_flag(a.err, VA_FLAG_BAD_SLOT);
        continue;
      }
      if (slot >= a.num_blocks * a.block_size) {
        if (h == 0 && c == 0) va::raise_flag(a.err, VA_FLAG_BAD_SLOT);
        continue;
      }
      blk = slot / a.block_size;
      off = slot - blk * a.block_size;
    } else if (MODE == 2) {
      const int32_t L = static_cast<const int32_t *>(idx1)[tok];
      if (L <= 0) continue;
      const int64_t bi = (L - 1) / a.block_size;
      off = (L - 1) - bi * a.block_size;
      if (bi >= max_blocks) {
        if (h == 0 && c == 0) va::raise_flag(a.err, VA_FLAG_CTX_OVERFLOW);
        continue;
      }
      blk = static_cast<const int32_t *>(idx0)[tok * max_blocks + bi];
      if (blk < 0 || blk >= a.num_blocks) {
        if (h == 0 && c == 0) va::raise_flag(a.err, VA_FLAG_BAD_BLOCK);
        continue;
      }
    } else {
      blk = static_cast<const int64_t *>(idx0)[tok];
      off = static_cast<const int64_t *>(idx1)[tok];
      if (blk < 0) continue;
    }
    const int64_t dst = blk * a.s_block + h * a.s_head + off * a.s_token + (int64_t)c * VEC;
    const int64_t src = tok * a.n_token + h * a.n_head + (int64_t)c * VEC;
    const T kv = va::ldg_stream(reinterpret_cast<const T *>(a.nk + src));
    const T vv = va::ldg_stream(reinterpret_cast<const T *>(a.nv + src));
    *reinterpret_cast<T *>(a.kc + dst) = kv;
    *reinterpret_cast<T *>(a.vc + dst) = vv;
  }
}

int pick_vec(const KVWriteArgs &a) {
  auto ok = [&](int v) {
    const uintptr_t m = static_cast<uintptr_t>(v * 2 - 1);
    return (a.head_size % v == 0) && !(reinterpret_cast<uintptr_t>(a.kc) & m) &&
           !(reinterpret_cast<uintptr_t>(a.vc) & m) && !(reinterpret_cast<uintptr_t>(a.nk) & m) &&
           !(reinterpret_cast<uintptr_t>(a.nv) & m) && a.s_block % v == 0 && a.s_head % v == 0 &&
           a.s_token % v == 0 && a.n_token % v == 0 && a.n_head % v == 0;
  };
  if (ok(8)) return 8;
  if (ok(2)) return 2;
  return 1;
}

template <int MODE>
int launch(const KVWriteArgs &a, const void *i0, const void *i1, int64_t max_blocks,
           cudaStream_t st) {
  if (a.rows <= 0) return VA_OK;
  const int vec = pick_vec(a);
  const int64_t total = a.rows * (a.head_size / vec);
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(va_host::sm_count()) * 16;
  if (blocks > cap) blocks = cap;
  switch (vec) {
    case 8:
      kv_write_kernel<8, MODE><<<(unsigned)blocks, threads, 0, st>>>(a, i0, i1, max_blocks);
      break;
    case 2:
      kv_write_kernel<2, MODE><<<(unsigned)blocks, threads, 0, st>>>(a, i0, i1, max_blocks);
      break;
    default:
      kv_write_kernel<1, MODE><<<(unsigned)blocks, threads, 0, st>>>(a, i0, i1, max_blocks);
  }
  return va_host::launch_status();
}

bool basic_ok(const void *kc, const void *vc, const void *nk, const void *nv, int heads, int d,
              int bs) {
  return kc && vc && nk && nv && heads > 0 && d > 0 && bs > 0;
}

}  // namespace

extern "C" int va_kv_write_slots(void *k_cache, void *v_cache, const void *new_k,
                                 const void *new_v, const void *slot_mapping, int slot_is_i64,
                                 int64_t num_tokens, int num_kv_heads, int head_size,
                                 int block_size, int64_t num_blocks, int64_t s_block,
                                 int64_t s_head, int64_t s_token, int64_t new_s_token,
                                 int64_t new_s_head, int32_t *err_flag, void *stream) {
  if (num_tokens < 0 || num_blocks < 0) return VA_ERR_INVALID_ARG;
  if (num_tokens == 0) return VA_OK;
  if (!basic_ok(k_cache, v_cache, new_k, new_v, num_kv_heads, head_size, block_size) ||
      !slot_mapping)
    return VA_ERR_INVALID_ARG;
  KVWriteArgs a{(uint16_t *)k_cache, (uint16_t *)v_cache, (const uint16_t *)new_k,
                (const uint16_t *)new_v, num_tokens * num_kv_heads, num_kv_heads, head_size,
                block_size, num_blocks, s_block, s_head, s_token, new_s_token, new_s_head,
                err_flag};
  auto st = static_cast<cudaStream_t>(stream);
  return slot_is_i64 ? launch<1>(a, slot_mapping, nullptr, 0, st)
                     : launch<0>(a, slot_mapping, nullptr, 0, st);
}

extern "C" int va_kv_write_decode(void *k_cache, void *v_cache, const void *new_k,
                                  const void *new_v, const int32_t *block_table,
                                  const int32_t *seq_lens, int64_t num_seqs,
                                  int64_t max_blocks_per_seq, int num_kv_heads, int head_size,
                                  int block_size, int64_t num_blocks, int64_t s_block,
                                  int64_t s_head, int64_t s_token, int64_t new_s_token,
                                  int64_t new_s_head, int32_t *err_flag, void *stream) {
  if (num_seqs < 0 || max_blocks_per_seq < 0) return VA_ERR_INVALID_ARG;
  if (num_seqs == 0) return VA_OK;
  if (!basic_ok(k_cache, v_cache, new_k, new_v, num_kv_heads, head_size, block_size) ||
      !block_table || !seq_lens)
    return VA_ERR_INVALID_ARG;
  KVWriteArgs a{(uint16_t *)k_cache, (uint16_t *)v_cache, (const uint16_t *)new_k,
                (const uint16_t *)new_v, num_seqs * num_kv_heads, num_kv_heads, head_size,
                block_size, num_blocks, s_block, s_head, s_token, new_s_token, new_s_head,
                err_flag};
  return launch<2>(a, block_table, seq_lens, max_blocks_per_seq, static_cast<cudaStream_t>(stream));
}

extern "C" int va_write_kv_batch(uint16_t *key_dst, uint16_t *value_dst, const uint16_t *key_src,
                                 const uint16_t *value_src, const int64_t *block_ids,
                                 const int64_t *token_offsets, int num_tokens, int num_kv_heads,
                                 int head_size, int stride_block, int stride_head,
                                 int stride_token, void *stream) {
  if (num_tokens < 0) return VA_ERR_INVALID_ARG;
  if (num_tokens == 0) return VA_OK;
  if (!basic_ok(key_dst, value_dst, key_src, value_src, num_kv_heads, head_size, 1) ||
      !block_ids || !token_offsets)
    return VA_ERR_INVALID_ARG;
  KVWriteArgs a{key_dst, value_dst, key_src, value_src, (int64_t)num_tokens * num_kv_heads,
                num_kv_heads, head_size, 1, INT64_MAX, stride_block, stride_head, stride_token,
                (int64_t)num_kv_heads * head_size, head_size, nullptr};
  return launch<3>(a, block_ids, token_offsets, 0, static_cast<cudaStream_t>(stream));
}
