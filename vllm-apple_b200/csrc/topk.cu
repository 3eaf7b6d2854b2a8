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
// Design (HBM-bound: one read of the row from DRAM, ~3 % of it read again), one CTA
// per row, on an order-preserving 16-bit key of the fp16 bits:
//   * fast path (k <= 512): every thread takes the maxima of 4 sub-regions of
//     its share of the row (fp16 max over 16-byte vectors); the k-th largest of
//     those maxima -- found from 256-bin shared-memory histograms of their high,
//     then low byte -- is a lower bound of the row's k-th largest key (the k
//     maxima above it are k distinct logits), so the logits at or above it
//     contain the answer, ties included.  Only the ~k sub-regions whose maximum
//     reaches the bound can hold such logits: a second pass re-reads just their
//     vectors, 8 logits at a time with an fp16 compare against the bound, and
//     appends the few that pass to shared memory (warp-aggregated slots).  Each
//     candidate's rank in (key desc, index asc) order is the count of larger
//     candidates (one thread per candidate; a bitonic sort for long lists), and
//     the first k are written at their ranks.
//   * exact path (k > 512, fewer than k valid sub-region maxima, or more
//     than kCap logits passing the bound, e.g. a row of equal logits): a radix
//     select -- 256-bin histograms of the high, then the low byte (per-warp
//     private bins) -- finds the exact k-th key; the keys above it (any order)
//     and the lowest-index ties equal to it (block-wide ordered scan) are
//     compacted and sorted the same way.
#include "common.cuh"
#include "vllm_apple_b200.h"

namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxK = 1024;
constexpr int kCap = 2048;  // candidates of the fast path

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
    constexpr int kU = 4;  // independent 16-byte loads in flight per thread
    const int64_t nv = n / 8;
    const uint4 *rv = reinterpret_cast<const uint4 *>(row);
    for (int64_t i0 = tid; i0 < nv; i0 += (int64_t)kThreads * kU) {
      uint4 v[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t i = i0 + (int64_t)u * kThreads;
        if (i < nv) v[u] = __ldg(rv + i);
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t i = i0 + (int64_t)u * kThreads;
        if (i >= nv) continue;
        const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          f(i * 8 + 2 * j, w[j] & 0xFFFFu);
          f(i * 8 + 2 * j + 1, w[j] >> 16);
        }
      }
    }
    done = nv * 8;
  }
  for (int64_t i = done + tid; i < n; i += kThreads) f(i, (uint32_t)__ldg(row + i));
}

// Calls f8(first index, 8 fp16 as uint4) for the 16-byte vectors of an aligned
// row (kU loads in flight per thread) and f1(index, fp16 bits) for the
// remaining elements.
// 16-byte read-only load with an L2 eviction-priority policy.
VA_DEVINL uint4 ldg_policy(const uint4 *p, uint64_t pol) {
  uint4 v;
  asm volatile("ld.global.nc.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(pol));
  return v;
}

template <typename F8, typename F1>
VA_DEVINL void for_each8(const uint16_t *row, int64_t n, bool vec, uint64_t pol, F8 &&f8,
                         F1 &&f1) {
  const int tid = threadIdx.x;
  int64_t done = 0;
  if (vec) {
    constexpr int kU = 4;
    const int64_t nv = n / 8;
    const uint4 *rv = reinterpret_cast<const uint4 *>(row);
    for (int64_t i0 = tid; i0 < nv; i0 += (int64_t)kThreads * kU) {
      uint4 v[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t i = i0 + (int64_t)u * kThreads;
        if (i < nv) v[u] = ldg_policy(rv + i, pol);
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t i = i0 + (int64_t)u * kThreads;
        if (i < nv) f8(i * 8, v[u]);
      }
    }
    done = nv * 8;
  }
  for (int64_t i = done + tid; i < n; i += kThreads) f1(i, (uint32_t)__ldg(row + i));
}

VA_DEVINL __half2 as_h2(uint32_t w) { return *reinterpret_cast<__half2 *>(&w); }
VA_DEVINL uint32_t as_u32(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }

// Bitonic sort of cand[0, m) (m a power of two), descending, by the block or
// (WARP) by warp 0 alone.
template <bool WARP>
VA_DEVINL void sort_desc(unsigned long long *cand, int m) {
  const int t = WARP ? (threadIdx.x & 31) : threadIdx.x;
  const int nt = WARP ? 32 : kThreads;
  for (int size = 2; size <= m; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = t; i < m / 2; i += nt) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool desc = (lo & size) == 0;
        const unsigned long long a = cand[lo], b = cand[hi];
        if ((a < b) == desc) {
          cand[lo] = b;
          cand[hi] = a;
        }
      }
      if (WARP) __syncwarp(); else __syncthreads();
    }
  }
}

// Candidate: key in the high word, complemented index in the low word, so that
// the descending order is (key desc, index asc); 0 = empty.
VA_DEVINL unsigned long long pack_cand(uint32_t key, int64_t i) {
  return ((unsigned long long)key << 32) | (0xFFFFFFFFu - (uint32_t)i);
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

// Warp 0: the bin b of hist[256] holding the r-th largest entry (1-based,
// counting from bin 255 down): *bin = b (-1 when the total is below r),
// *above = the count in bins above b.
VA_DEVINL void find_bin(const int *hist, int r, int *bin, int *above) {
  const int lane = threadIdx.x & 31;
  int c[8], s = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    c[j] = hist[255 - 8 * lane - j];
    s += c[j];
  }
  int incl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  int run = incl - s;
  if (lane == 31 && incl < r) *bin = -1;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (run < r && run + c[j] >= r) {
      *bin = 255 - 8 * lane - j;
      *above = run;
    }
    run += c[j];
  }
}

// One CTA per row: CTA r selects the top k of row r into output row r.
__global__ void __launch_bounds__(kThreads, 3) topk_kernel(int32_t *out_idx, uint16_t *out_val,
                                                        const uint16_t *logits, int64_t n_row,
                                                        int64_t row_stride, int k, int vec) {
  __shared__ int whist[kWarps][256];
  __shared__ int hist[256];
  __shared__ int warp_sums[kWarps];
  __shared__ int s_bin, s_above, s_gt, s_ties;
  __shared__ unsigned long long cand[kCap];
  __shared__ int s_cnt, s_na;
  __shared__ int s_list[4 * kThreads];  // sub-regions whose maximum reaches the bound
  va::pdl_enter();
  const int tid = threadIdx.x, lane = tid & 31;
  const int64_t n = n_row;
  const uint16_t *row = logits + (int64_t)blockIdx.x * row_stride;
  const bool v = vec != 0;
  const int64_t orow = blockIdx.x;  // output row
  if (k <= kThreads)
    for (int i = tid; i < 512; i += kThreads) (&whist[0][0])[i] = 0;

  // ---- fast path: bound from the per-thread maxima, screen, sort ----
  if (k <= kThreads) {
    // Maxima of 4 sub-regions per thread (sub-region u: vectors tid + u * kThreads
    // + m * 4 * kThreads; fp16 max, NaN ignored; whether -0 or +0 wins a tie only
    // lowers the bound, which stays valid) and of the scalar logits (the tail of a
    // vectorised row, every logit of an unaligned one).
    uint32_t sm[4] = {0u, 0u, 0u, 0u};
    uint32_t mx = 0;
    // the first read keeps the row in L2 for the second (evict_last), which
    // releases it (evict_first)
    uint64_t keep, drop;
    asm("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(keep));
    asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(drop));
    const int64_t nv = v ? n / 8 : 0;
    {
      const uint4 *rv = reinterpret_cast<const uint4 *>(row);
      __half2 m2[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) m2[u] = as_h2(0xFC00FC00u);  // (-inf, -inf)
      for (int64_t i0 = tid; i0 < nv; i0 += (int64_t)kThreads * 4) {
        uint4 q[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (i0 + u * kThreads < nv) q[u] = ldg_policy(rv + i0 + u * kThreads, keep);
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (i0 + u * kThreads < nv)
            m2[u] = __hmax2(m2[u], __hmax2(__hmax2(as_h2(q[u].x), as_h2(q[u].y)),
                                           __hmax2(as_h2(q[u].z), as_h2(q[u].w))));
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        sm[u] = max(key_of(as_u32(m2[u]) & 0xFFFFu), key_of(as_u32(m2[u]) >> 16));
    }
    for (int64_t i = nv * 8 + tid; i < n; i += kThreads) mx = max(mx, key_of(__ldg(row + i)));
    if (tid == 0) {
      s_cnt = 0;
      s_na = 0;
    }
    // the k-th largest of these maxima (0 when fewer than k are valid): 256-bin
    // histograms of their high byte, then of the low bytes in its bin
    __syncthreads();  // the histograms' zeroing is complete
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (sm[u] != 0u) atomicAdd(&whist[0][sm[u] >> 8], 1);
    if (mx != 0u) atomicAdd(&whist[0][mx >> 8], 1);
    __syncthreads();
    if (tid < 32) find_bin(whist[0], k, &s_bin, &s_above);
    __syncthreads();
    const int hb = s_bin;
    uint32_t bound = 0;
    if (hb >= 0) {  // uniform
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (sm[u] != 0u && (int)(sm[u] >> 8) == hb) atomicAdd(&whist[1][sm[u] & 0xFFu], 1);
      if (mx != 0u && (int)(mx >> 8) == hb) atomicAdd(&whist[1][mx & 0xFFu], 1);
      __syncthreads();
      if (tid < 32) find_bin(whist[1], k - s_above, &s_gt, &s_ties);
      __syncthreads();
      bound = ((uint32_t)hb << 8) | (uint32_t)s_gt;
    }
    if (bound != 0u) {  // at least k valid logits: the answer is inside the bound
      // screen 8 at a time against the bound's value (a superset of the keys >=
      // bound: -0 and +0 compare equal), then one warp round per pending logit
      const __half2 b2 = as_h2(half_bits_of(bound) * 0x10001u);
      auto append = [&](unsigned act, uint32_t pend, const uint32_t (&w)[4], int64_t i0) {
        while (__any_sync(act, pend != 0u)) {
          const bool take = pend != 0u;
          const int j = __ffs(pend) - 1;
          pend &= pend - 1u;
          const unsigned ball = __ballot_sync(act, take);
          const int leader = __ffs(ball) - 1;
          int base = 0;
          if (lane == leader) base = atomicAdd(&s_cnt, __popc(ball));
          base = __shfl_sync(act, base, leader);
          if (take) {
            const uint32_t wj = j < 2 ? w[0] : j < 4 ? w[1] : j < 6 ? w[2] : w[3];
            const int slot = base + __popc(ball & ((1u << lane) - 1u));
            if (slot < kCap) cand[slot] = pack_cand(key_of((wj >> ((j & 1) * 16)) & 0xFFFFu), i0 + j);
          }
        }
      };
      auto screen8 = [&](int64_t i0, const uint4 &q) {
        const unsigned act = __activemask();
        const unsigned hit = __hge2_mask(as_h2(q.x), b2) | __hge2_mask(as_h2(q.y), b2) |
                             __hge2_mask(as_h2(q.z), b2) | __hge2_mask(as_h2(q.w), b2);
        if (__any_sync(act, hit != 0u)) {
          const uint32_t w[4] = {q.x, q.y, q.z, q.w};
          uint32_t pend = 0;
          if (hit) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
              if (key_of((w[j >> 1] >> ((j & 1) * 16)) & 0xFFFFu) >= bound) pend |= 1u << j;
          }
          append(act, pend, w, i0);
        }
      };
      auto screen1 = [&](int64_t i, uint32_t h) {
        const uint32_t w[4] = {h, 0u, 0u, 0u};
        append(__activemask(), key_of(h) >= bound ? 1u : 0u, w, i);
      };
      if (v) {
        // only sub-regions whose maximum reaches the bound hold vector logits >=
        // bound: the block re-reads just those; the scalar tail is screened whole
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (sm[u] >= bound) s_list[atomicAdd(&s_na, 1)] = tid + u * kThreads;
        __syncthreads();
        const int64_t stride = (int64_t)kThreads * 4;
        const int per = (int)((nv + stride - 1) / stride);
        const int total = s_na * per;
        const uint4 *rv = reinterpret_cast<const uint4 *>(row);
        for (int w0 = tid; w0 < total; w0 += kThreads * 4) {
          uint4 qv[4];
          int64_t iv[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int w = w0 + u * kThreads;
            iv[u] = -1;
            if (w < total) {
              const int a = w / per;
              const int64_t i = s_list[a] + (int64_t)(w - a * per) * stride;
              if (i < nv) {
                iv[u] = i;
                qv[u] = ldg_policy(rv + i, drop);
              }
            }
          }
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (iv[u] >= 0) screen8(iv[u] * 8, qv[u]);
        }
        for (int64_t i = nv * 8 + tid; i < n; i += kThreads) screen1(i, (uint32_t)__ldg(row + i));
      } else {
        for_each8(row, n, v, drop, screen8, screen1);
      }
      __syncthreads();
      const int cnt = s_cnt;
      if (cnt <= kThreads) {  // uniform; candidates are distinct: rank = number larger
        if (tid < cnt) {
          const unsigned long long mine = cand[tid];
          int rank = 0;
#pragma unroll 4
          for (int j = 0; j < cnt; ++j) rank += cand[j] > mine ? 1 : 0;
          if (rank < k) {
            const int64_t o = orow * k + rank;
            out_idx[o] = (int32_t)(0xFFFFFFFFu - (uint32_t)(mine & 0xFFFFFFFFull));
            out_val[o] = half_bits_of((uint32_t)(mine >> 32));
          }
        }
        return;
      }
      if (cnt <= kCap) {  // uniform
        int mc = 1;
        while (mc < cnt) mc <<= 1;
        for (int i = cnt + tid; i < mc; i += kThreads) cand[i] = 0ull;
        __syncthreads();
        if (mc <= 256) {  // small: warp 0 alone, no block barriers
          if (tid < 32) sort_desc<true>(cand, mc);
          __syncthreads();
        } else {
          sort_desc<false>(cand, mc);
        }
        for (int i = tid; i < k; i += kThreads) {
          const unsigned long long c = cand[i];
          const int64_t o = orow * k + i;
          out_idx[o] = (int32_t)(0xFFFFFFFFu - (uint32_t)(c & 0xFFFFFFFFull));
          out_val[o] = half_bits_of((uint32_t)(c >> 32));
        }
        return;
      }
    }
    __syncthreads();
  }

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
          cand[slot] = pack_cand(key, i0 + j);
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
          cand[n_gt + pos] = pack_cand(thr, i0 + j);
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
  sort_desc<false>(cand, m);
  for (int i = tid; i < k; i += kThreads) {
    const unsigned long long c = cand[i];
    const int64_t o = orow * k + i;
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

// Every row runs whole on one CTA: cutting the rows of small batches into slices
// on separate CTAs plus a merge kernel measured 2-3x slower under graph replay
// (8 x 131072: 17.8 us against 7.0), so no workspace is needed.
extern "C" size_t va_topk_workspace_size(int64_t, int64_t, int) { return 0; }

extern "C" int va_topk_ws(int32_t *indices, void *values, const void *logits,
                          int64_t num_tokens, int64_t vocab_size, int64_t row_stride, int k,
                          void *, size_t, void *stream) {
  return va_topk(indices, values, logits, num_tokens, vocab_size, row_stride, k, stream);
}

extern "C" int va_topk(int32_t *indices, void *values, const void *logits, int64_t num_tokens,
                       int64_t vocab_size, int64_t row_stride, int k, void *stream) {
  if (num_tokens < 0 || vocab_size < 0 || k < 1 || row_stride < vocab_size)
    return VA_ERR_INVALID_ARG;
  if (k > kMaxK || vocab_size > INT32_MAX - 1 || num_tokens > INT32_MAX) return VA_ERR_UNSUPPORTED;
  if (num_tokens == 0) return VA_OK;
  if (!indices || !values || !logits) return VA_ERR_INVALID_ARG;
  const int vec = (va_host::aligned16(logits) && row_stride % 8 == 0) ? 1 : 0;
  va_host::launch_pdl(topk_kernel, (unsigned)num_tokens, kThreads,
                      static_cast<cudaStream_t>(stream), indices, static_cast<uint16_t *>(values),
                      static_cast<const uint16_t *>(logits), vocab_size, row_stride, k, vec);
  return va_host::launch_status();
}
