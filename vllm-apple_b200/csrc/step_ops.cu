// Step-level kernels around the attention call:
//   * va_rope_kv_write_slots  -- rotary embedding of q and k fused with the
//                                K/V scatter into the paged cache (one pass);
//   * va_build_prefill_metadata -- per-token sequence index, position and slot,
//                                built on the device from query_start_loc,
//                                seq_lens and the block table;
//   * va_kv_sync_blocks       -- copy every active block of the listed
//                                sequences from one cache layout to another.
#include "common.cuh"

namespace {

VA_DEVINL void unpack8(const uint4 &v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = va::h2_to_f2(w[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
VA_DEVINL uint4 pack8(const float (&f)[8]) {
  return make_uint4(va::pack_h2(f[0], f[1]), va::pack_h2(f[2], f[3]), va::pack_h2(f[4], f[5]),
                    va::pack_h2(f[6], f[7]));
}
VA_DEVINL void rot_pair(float x0, float x1, float c, float s, float &y0, float &y1) {
  y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
  y1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
}

// ---------------------------------------------------------------------------
// RoPE (Neox, rot == D) + K/V scatter.  One thread per (token, head slot,
// group of 8 rotation pairs); head slots: Hq query heads, Hkv key heads
// (rotated, stored back and scattered), Hkv value heads (scattered only).
// ---------------------------------------------------------------------------
struct RopeKV {
  __half *q, *k;
  const __half *v;
  __half *kc, *vc;
  const float *cs, *sn;
  const int32_t *pos;
  const void *slots;
  int slot64;
  int64_t T, max_pos, qs, ks, vs, num_blocks, s_block, s_head, s_token;
  int Hq, Hkv, D, bs;
  int32_t *err;
};

__global__ void __launch_bounds__(256) rope_kv_write_kernel(const RopeKV a) {
  const int half = a.D / 2, groups = half / 8;
  const int slots_per_tok = a.Hq + 2 * a.Hkv;
  const int64_t total = a.T * slots_per_tok * groups;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t tok = i / (slots_per_tok * groups);
    const int rem = (int)(i - tok * slots_per_tok * groups);
    const int h = rem / groups, gi = rem - (rem / groups) * groups;
    const int p = a.pos[tok];
    const bool is_q = h < a.Hq, is_k = !is_q && h < a.Hq + a.Hkv;
    const int kvh = is_q ? 0 : (is_k ? h - a.Hq : h - a.Hq - a.Hkv);
    __half *x = is_q ? a.q + tok * a.qs + (int64_t)h * a.D
                     : (is_k ? a.k + tok * a.ks + (int64_t)kvh * a.D
                             : const_cast<__half *>(a.v) + tok * a.vs + (int64_t)kvh * a.D);
    uint4 *pa = reinterpret_cast<uint4 *>(x + gi * 8);
    uint4 *pb = reinterpret_cast<uint4 *>(x + half + gi * 8);
    uint4 ra = *pa, rb = *pb;
    if ((is_q || is_k) && (p < 0 || p >= a.max_pos)) {  // token left untouched
      if (h == 0 && gi == 0) va::raise_flag(a.err, VA_FLAG_BAD_POSITION);
      continue;
    }
    if (is_q || is_k) {
      const float4 *cp = reinterpret_cast<const float4 *>(a.cs + (int64_t)p * half + gi * 8);
      const float4 *sp = reinterpret_cast<const float4 *>(a.sn + (int64_t)p * half + gi * 8);
      const float4 c0 = __ldg(cp), c1 = __ldg(cp + 1), s0 = __ldg(sp), s1 = __ldg(sp + 1);
      const float c[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
      const float s[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
      float fa[8], fb[8], ya[8], yb[8];
      unpack8(ra, fa);
      unpack8(rb, fb);
#pragma unroll
      for (int j = 0; j < 8; ++j) rot_pair(fa[j], fb[j], c[j], s[j], ya[j], yb[j]);
      ra = pack8(ya);
      rb = pack8(yb);
      *pa = ra;
      *pb = rb;
    }
    if (is_q) continue;
    int64_t slot = a.slot64 ? static_cast<const int64_t *>(a.slots)[tok]
                            : (int64_t) static_cast<const int32_t *>(a.slots)[tok];
    if (slot < 0) {
      if (slot < -1 && kvh == 0 && gi == 0) va::raise_flag(a.err, VA_FLAG_BAD_SLOT);
      continue;
    }
    if (slot >= a.num_blocks * a.bs) {
      if (kvh == 0 && gi == 0) va::raise_flag(a.err, VA_FLAG_BAD_SLOT);
      continue;
    }
    const int64_t blk = slot / a.bs, off = slot - blk * a.bs;
    __half *dst = (is_k ? a.kc : a.vc) + blk * a.s_block + (int64_t)kvh * a.s_head +
                  off * a.s_token;
    *reinterpret_cast<uint4 *>(dst + gi * 8) = ra;
    *reinterpret_cast<uint4 *>(dst + half + gi * 8) = rb;
  }
}

// ---------------------------------------------------------------------------
// Per-token metadata: token t of sequence s (query_start_loc[s] <= t <
// query_start_loc[s+1]) sits at position seq_lens[s] - query_len + i.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) prefill_metadata_kernel(
    const int32_t *qsl, const int32_t *seq_lens, const int32_t *bt, int64_t S, int64_t T,
    int64_t max_blocks, int bs, int64_t first_token, int32_t *tok_seq, int32_t *pos,
    int64_t *slots) {
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < T;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t gt = first_token + t;  // token index in the whole batch
    // last sequence whose start is <= gt (binary search over query_start_loc)
    int64_t lo = 0, hi = S - 1;
    while (lo < hi) {
      const int64_t mid = (lo + hi + 1) >> 1;
      if (qsl[mid] <= gt) lo = mid; else hi = mid - 1;
    }
    const int64_t s = lo;
    const int64_t qlen = (int64_t)qsl[s + 1] - qsl[s];
    const int64_t p = (int64_t)seq_lens[s] - qlen + (gt - qsl[s]);
    tok_seq[t] = (int32_t)s;
    pos[t] = (int32_t)p;
    if (slots) {
      int64_t sl = -1;
      if (p >= 0 && p / bs < max_blocks) {
        const int32_t b = bt[s * max_blocks + p / bs];
        if (b >= 0) sl = (int64_t)b * bs + p % bs;
      }
      slots[t] = sl;
    }
  }
}

// ---------------------------------------------------------------------------
// Active-block copy between cache layouts: CTA per (sequence, block index).
// ---------------------------------------------------------------------------
struct SyncArgs {
  const __half *sk, *sv;
  __half *dk, *dv;
  const int32_t *bt, *seq_lens;
  int64_t max_blocks, num_blocks;
  int H, bs, D;
  int64_t ss_block, ss_head, ss_token, ds_block, ds_head, ds_token;
};

__global__ void __launch_bounds__(256) kv_sync_kernel(const SyncArgs a) {
  const int64_t s = blockIdx.y;
  const int64_t bi = blockIdx.x;
  const int L = a.seq_lens[s];
  if (L <= 0 || bi * a.bs >= L || bi >= a.max_blocks) return;
  const int32_t blk = a.bt[s * a.max_blocks + bi];
  if (blk < 0 || blk >= a.num_blocks) return;  // unused / out-of-range ids are skipped
  const int cpr = a.D / 8;
  const int items = a.H * a.bs * cpr;
  for (int i = threadIdx.x; i < items; i += blockDim.x) {
    const int c = i % cpr, r = i / cpr;
    const int tok = r % a.bs, h = r / a.bs;
    const int64_t so = (int64_t)blk * a.ss_block + h * a.ss_head + tok * a.ss_token + c * 8;
    const int64_t d = (int64_t)blk * a.ds_block + h * a.ds_head + tok * a.ds_token + c * 8;
    *reinterpret_cast<uint4 *>(a.dk + d) = __ldg(reinterpret_cast<const uint4 *>(a.sk + so));
    *reinterpret_cast<uint4 *>(a.dv + d) = __ldg(reinterpret_cast<const uint4 *>(a.sv + so));
  }
}

unsigned grid_for(int64_t work, int threads) {
  int64_t b = (work + threads - 1) / threads;
  const int64_t cap = (int64_t)va_host::sm_count() * 32;
  if (b > cap) b = cap;
  return (unsigned)(b < 1 ? 1 : b);
}

bool m8(int64_t x) { return x % 8 == 0; }

}  // namespace

extern "C" int va_rope_kv_write_slots(void *q, void *k, const void *v, void *k_cache,
                                      void *v_cache, const float *cos_cache,
                                      const float *sin_cache, const int32_t *positions,
                                      const void *slot_mapping, int slot_is_i64,
                                      int64_t num_tokens, int num_heads, int num_kv_heads,
                                      int head_size, int block_size, int64_t num_blocks,
                                      int64_t max_position, int64_t q_s_token, int64_t k_s_token,
                                      int64_t v_s_token, int64_t s_block, int64_t s_head,
                                      int64_t s_token, int32_t *err_flag, void *stream) {
  if (num_tokens < 0 || num_heads < 0 || num_kv_heads <= 0 || block_size <= 0)
    return VA_ERR_INVALID_ARG;
  if (num_tokens == 0) return VA_OK;
  if (!q || !k || !v || !k_cache || !v_cache || !cos_cache || !sin_cache || !positions ||
      !slot_mapping)
    return VA_ERR_INVALID_ARG;
  if (head_size % 16) return VA_ERR_UNSUPPORTED;  // 8-pair groups of a split-half rotation
  if (!va_host::aligned16(q) || !va_host::aligned16(k) || !va_host::aligned16(v) ||
      !va_host::aligned16(k_cache) || !va_host::aligned16(v_cache) ||
      !va_host::aligned16(cos_cache) || !va_host::aligned16(sin_cache) || !m8(q_s_token) ||
      !m8(k_s_token) || !m8(v_s_token) || !m8(s_block) || !m8(s_head) || !m8(s_token))
    return VA_ERR_INVALID_ARG;
  RopeKV a{static_cast<__half *>(q), static_cast<__half *>(k), static_cast<const __half *>(v),
           static_cast<__half *>(k_cache), static_cast<__half *>(v_cache), cos_cache, sin_cache,
           positions, slot_mapping, slot_is_i64, num_tokens, max_position, q_s_token,
           k_s_token, v_s_token, num_blocks, s_block, s_head, s_token, num_heads, num_kv_heads,
           head_size, block_size, err_flag};
  const int64_t work = num_tokens * (num_heads + 2 * num_kv_heads) * (head_size / 16);
  rope_kv_write_kernel<<<grid_for(work, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return va_host::launch_status();
}

extern "C" int va_build_prefill_metadata(const int32_t *query_start_loc, const int32_t *seq_lens,
                                         const int32_t *block_table, int64_t num_seqs,
                                         int64_t first_token, int64_t num_tokens,
                                         int64_t max_blocks_per_seq, int block_size,
                                         int32_t *token_to_seq, int32_t *positions,
                                         int64_t *slot_mapping, void *stream) {
  if (num_tokens < 0 || num_seqs < 0 || first_token < 0 || block_size <= 0)
    return VA_ERR_INVALID_ARG;
  if (num_tokens == 0) return VA_OK;
  if (num_seqs == 0 || !query_start_loc || !seq_lens || !token_to_seq || !positions ||
      (slot_mapping && !block_table))
    return VA_ERR_INVALID_ARG;
  prefill_metadata_kernel<<<grid_for(num_tokens, 256), 256, 0,
                            static_cast<cudaStream_t>(stream)>>>(
      query_start_loc, seq_lens, block_table, num_seqs, num_tokens, max_blocks_per_seq,
      block_size, first_token, token_to_seq, positions, slot_mapping);
  return va_host::launch_status();
}

extern "C" int va_kv_sync_blocks(const void *src_k, const void *src_v, void *dst_k, void *dst_v,
                                 const int32_t *block_table, const int32_t *seq_lens,
                                 int64_t num_seqs, int64_t max_blocks_per_seq, int num_kv_heads,
                                 int head_size, int block_size, int64_t num_blocks,
                                 int64_t src_s_block, int64_t src_s_head, int64_t src_s_token,
                                 int64_t dst_s_block, int64_t dst_s_head, int64_t dst_s_token,
                                 void *stream) {
  if (num_seqs < 0 || max_blocks_per_seq < 0 || num_kv_heads <= 0 || block_size <= 0)
    return VA_ERR_INVALID_ARG;
  if (num_seqs == 0 || max_blocks_per_seq == 0) return VA_OK;
  if (!src_k || !src_v || !dst_k || !dst_v || !block_table || !seq_lens)
    return VA_ERR_INVALID_ARG;
  if (head_size % 8 || !va_host::aligned16(src_k) || !va_host::aligned16(src_v) ||
      !va_host::aligned16(dst_k) || !va_host::aligned16(dst_v) || !m8(src_s_block) ||
      !m8(src_s_head) || !m8(src_s_token) || !m8(dst_s_block) || !m8(dst_s_head) ||
      !m8(dst_s_token))
    return VA_ERR_INVALID_ARG;
  if (num_seqs > 65535 || max_blocks_per_seq > 0x7fffffff) return VA_ERR_UNSUPPORTED;
  SyncArgs a{static_cast<const __half *>(src_k), static_cast<const __half *>(src_v),
             static_cast<__half *>(dst_k), static_cast<__half *>(dst_v), block_table, seq_lens,
             max_blocks_per_seq, num_blocks, num_kv_heads, block_size, head_size, src_s_block,
             src_s_head, src_s_token, dst_s_block, dst_s_head, dst_s_token};
  kv_sync_kernel<<<dim3((unsigned)max_blocks_per_seq, (unsigned)num_seqs), 256, 0,
                   static_cast<cudaStream_t>(stream)>>>(a);
  return va_host::launch_status();
}
