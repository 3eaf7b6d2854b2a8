// Top-k logits selection per token (the step after the model's output side):
// indices int32 [T, k] and values fp16 [T, k], largest first.
//
// Replaces EngineTopK.encode -- topk_select / topk_select_small_k
// (vllm_apple/engine/ops/topk.py:57-283, :340-399).  Same selection rule as the
// reference's insertion lists, which keep a logit only if it is greater than
// the current k-th value initialised to -inf: NaN and -inf are never selected,
// and rows with fewer than k such logits are padded with index -1 and value
// -inf.  Ties are resolved by the lower index (the reference's order between
// equal values depends on its thread layout; values are identical either way).
//
// Design (HBM-bound: one read of the row from DRAM, two more from L2): one CTA
// per row runs a 16-bit radix select on an order-preserving key of the fp16
// bits -- a 256-bin histogram of the high byte (per-warp private bins), the
// bin holding the k-th largest, a 256-bin histogram of the low byte inside
// that bin -- which yields the exact k-th key.  A third pass compacts the keys
// above it (any order) and the lowest-index ties equal to it (block-wide
// ordered scan), then a shared-memory bitonic sort orders the <= 1024
// candidates by (key desc, index asc).
#include "common.cuh"
#include "vllm_apple_b200.h"

namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxK = 1024;

// Order-preserving 16-bit key of an fp16 bit pattern, 0 for NaN and -inf
// (never selected).  Valid keys lie in [0x0400, 0xFC00].
VA_DEVINL uint32_t key_of(uint32_t h) {
  if ((h & 0x7FFFu) > 0x7C00u || h == 0xFC00u) return 0u;
  return (h & 0x8000u) ? (~h & 0xFFFFu) : (h | 0x8000u);
}
VA_DEVINL uint16_t half_bits_of(uint32_t key) {
  return (uint16_t)((key & 0x8000u) ? (key & 0x7FFFu) : (~key & 0xFFFFu));
}

// Calls f(index, fp16 bits) for every element of the row; 16-byte loads when
// the row is aligned.  Order of calls is unspecified.
template <typename F>
VA_DEVINL void for_each(const uint16_t *row, int64_t n, bool vec, F &&f) {
  const int tid = threadIdx.x;
  int64_t done = 0;
  if (vec) {
    const int64_t nv = n / 8;
    const uint4 *rv = reinterpret_cast<const uint4 *>(row);
    for (int64_t i = tid; i < nv; i += kThreads) {
      const uint4 v = __ldg(rv + i);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        f(i * 8 + 2 * j, w[j] & 0xFFFFu);
        f(i * 8 + 2 * j + 1, w[j] >> 16);
      }
    }
    done = nv * 8;
  }
  for (int64_t i = done + tid; i < n; i += kThreads) f(i, (uint32_t)__ldg(row + i));
}

// Block-wide exclusive scan of one int per thread; returns the exclusive
// prefix, *total receives the sum.
VA_DEVINL int block_scan(int v, int *warp_sums, int *total) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[wid] = x;
  __syncthreads();
  if (wid == 0) {
    int w = lane < kWarps ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < kWarps) warp_sums[lane] = w;
  }
  __syncthreads();
  const int excl = x - v + (wid > 0 ? warp_sums[wid - 1] : 0);
  *total = warp_sums[kWarps - 1];
  __syncthreads();
  return excl;
}

// Histogram of (key >> shift) & 0xFF over keys whose bits above `shift + 8`
// equal `prefix` (all valid keys when shift == 8), then the bin b holding the
// r-th largest key (1-based) of that population: *bin = b, *above = number of
// keys in bins > b.  Returns the population size.
VA_DEVINL int radix_step(const uint16_t *row, int64_t n, bool vec, int shift, uint32_t prefix,
                         int r, int (*whist)[256], int *hist, int *warp_sums, int *bin,
                         int *above) {
  const int tid = threadIdx.x, wid = tid >> 5;
  for (int i = tid; i < kWarps * 256; i += kThreads) (&whist[0][0])[i] = 0;
  __syncthreads();
  int *mine = whist[wid];
  for_each(row, n, vec, [&](int64_t, uint32_t h) {
    const uint32_t key = key_of(h);
    if (key != 0u && (shift == 8 || (key >> 8) == prefix)) atomicAdd(&mine[(key >> shift) & 0xFFu], 1);
  });
  __syncthreads();
  if (tid < 256) {
    int s = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += whist[w][tid];
    hist[tid] = s;
  }
  __syncthreads();
  // suffix sums: bins are scanned from the top (bin 255 first)
  const int b = 255 - tid;
  const int c = tid < 256 ? hist[b] : 0;
  int total;
  const int gt = block_scan(c, warp_sums, &total);  // keys in bins above b
  if (tid < 256 && gt < r && r <= gt + c) {
    *bin = b;
    *above = gt;
  }
  __syncthreads();
  return total;
}

__global__ void __launch_bounds__(kThreads) topk_kernel(int32_t *out_idx, uint16_t *out_val,
                                                        const uint16_t *logits, int64_t n,
                                                        int64_t row_stride, int k, int vec) {
  __shared__ int whist[kWarps][256];
  __shared__ int hist[256];
  __shared__ int warp_sums[kWarps];
  __shared__ int s_bin, s_above, s_gt, s_ties;
  __shared__ unsigned long long cand[kMaxK];
  const int tid = threadIdx.x;
  const uint16_t *row = logits + (int64_t)blockIdx.x * row_stride;
  const bool v = vec != 0;

  // ---- radix select of the k-th largest key ----
  uint32_t thr = 0;
  int n_gt = 0, need = 0;
  const int valid = radix_step(row, n, v, 8, 0u, k, whist, hist, warp_sums, &s_bin, &s_above);
  if (valid <= k) {
    n_gt = valid;  // every valid key; the rest of the row is padding
  } else {
    const uint32_t b1 = (uint32_t)s_bin;
    const int above1 = s_above;
    radix_step(row, n, v, 0, b1, k - above1, whist, hist, warp_sums, &s_bin, &s_above);
    thr = (b1 << 8) | (uint32_t)s_bin;
    n_gt = above1 + s_above;
    need = k - n_gt;
  }

  // ---- compaction: keys > thr (any order), then the first `need` ties by index ----
  if (tid == 0) { s_gt = 0; s_ties = 0; }
  __syncthreads();
  for (int64_t base = 0; base < n; base += (int64_t)kThreads * 8) {
    const int64_t i0 = base + (int64_t)tid * 8;
    uint32_t h[8];
    if (v && i0 + 8 <= n) {
      const uint4 q = __ldg(reinterpret_cast<const uint4 *>(row + i0));
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        h[2 * j] = w[j] & 0xFFFFu;
        h[2 * j + 1] = w[j] >> 16;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) h[j] = i0 + j < n ? (uint32_t)__ldg(row + i0 + j) : 0x7FFFu;
    }
    int ties = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t key = key_of(h[j]);
      if (key > thr) {
        const int slot = atomicAdd(&s_gt, 1);
        if (slot < kMaxK)
          cand[slot] = ((unsigned long long)key << 32) | (0xFFFFFFFFu - (uint32_t)(i0 + j));
      }
      ties += (need > 0 && key == thr) ? 1 : 0;
    }
    if (need > 0) {
      int total;
      const int before = s_ties;  // read before the scan's barriers
      int pos = before + block_scan(ties, warp_sums, &total);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (key_of(h[j]) == thr && pos < need) {
          cand[n_gt + pos] = ((unsigned long long)thr << 32) | (0xFFFFFFFFu - (uint32_t)(i0 + j));
          ++pos;
        }
      }
      if (tid == 0) s_ties = before + total;
    }
    __syncthreads();
    if (s_gt >= n_gt && (need == 0 || s_ties >= need)) break;  // uniform
  }
  // padding (rows with fewer than k valid logits)
  for (int i = n_gt + need + tid; i < kMaxK; i += kThreads) cand[i] = 0ull;
  __syncthreads();

  // ---- bitonic sort, descending, over the next power of two >= k ----
  int m = 1;
  while (m < k) m <<= 1;
  for (int size = 2; size <= m; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < m / 2; i += kThreads) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool desc = (lo & size) == 0;
        const unsigned long long a = cand[lo], b = cand[hi];
        if ((a < b) == desc) {
          cand[lo] = b;
          cand[hi] = a;
        }
      }
      __syncthreads();
    }
  }
  for (int i = tid; i < k; i += kThreads) {
    const unsigned long long c = cand[i];
    const int64_t o = (int64_t)blockIdx.x * k + i;
    if (c == 0ull) {
      out_idx[o] = -1;
      out_val[o] = 0xFC00u;  // -inf
    } else {
      out_idx[o] = (int32_t)(0xFFFFFFFFu - (uint32_t)(c & 0xFFFFFFFFull));
      out_val[o] = half_bits_of((uint32_t)(c >> 32));
    }
  }
}

}  // namespace

extern "C" int va_topk(int32_t *indices, void *values, const void *logits, int64_t num_tokens,
                       int64_t vocab_size, int64_t row_stride, int k, void *stream) {
  if (num_tokens < 0 || vocab_size < 0 || k < 1 || row_stride < vocab_size)
    return VA_ERR_INVALID_ARG;
  if (k > kMaxK || vocab_size > INT32_MAX - 1 || num_tokens > INT32_MAX) return VA_ERR_UNSUPPORTED;
  if (num_tokens == 0) return VA_OK;
  if (!indices || !values || !logits) return VA_ERR_INVALID_ARG;
  const int vec = (va_host::aligned16(logits) && row_stride % 8 == 0) ? 1 : 0;
  topk_kernel<<<(unsigned)num_tokens, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      indices, static_cast<uint16_t *>(values), static_cast<const uint16_t *>(logits),
      vocab_size, row_stride, k, vec);
  return va_host::launch_status();
}
