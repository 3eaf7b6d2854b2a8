// Token-parallel causal paged attention (prefill / chunked-prefill mixed batch).
//
// Semantics of the reference's paged_attention_v2_prefill: token t of
// sequence token_to_seq[t] attends to cache positions 0..positions[t].
//
// Design:
//   * a one-CTA planner kernel cuts the token list into tiles: a tile is at
//     most TQ consecutive tokens of one sequence (run boundaries found with a
//     block-wide max-scan, tile slots with a sum-scan).  Decode rows of a mixed
//     batch become one-token tiles.
//   * one CTA (4 warps) per (tile, kv head [, q-head group]).  Its 64 MMA rows
//     are (token, q head) pairs of the GQA group, so every K/V tile staged in
//     shared memory serves all heads of the group.
//   * K/V move HBM -> shared memory in chunks of 64 keys (4 pages) with
//     16-byte cp.async into padded rows (conflict-free ldmatrix), double
//     buffered; unwritten positions and invalid pages are zero-filled.
//   * S = Q K^T and O += P V on tensor cores (mma.sync m16n8k16, fp16 in, fp32
//     accumulate), online softmax in registers, per-row causal mask by
//     absolute position.
#include <math.h>

#include <mutex>

#include "common.cuh"
#include <cudaTypedefs.h>

#include "prefill_tc.cuh"

namespace va_internal {  // split-KV decode of one-token rows (paged_decode.cu)
size_t decode_rows_workspace(int64_t rows_bound, int Hq, int Hkv, int D, int bs,
                             int64_t max_blocks);
int decode_rows(void *out, const void *q, const void *kc, const void *vc, const int32_t *bt,
                const int32_t *rows, const int32_t *rows_n, const int32_t *tok_seq,
                const int32_t *pos, int64_t rows_bound, int64_t num_seqs, int Hq, int Hkv, int D,
                int bs, int64_t max_blocks, int64_t num_blocks, float scale, int64_t s_block,
                int64_t s_head, int64_t s_token, int64_t q_s_token, int64_t q_s_head,
                int64_t o_s_token, int64_t o_s_head, void *ws, size_t ws_bytes, int32_t *err,
                cudaStream_t st);
}  // namespace va_internal

namespace {

constexpr int kRows = 64;   // MMA rows per CTA (4 warps x 16)
constexpr int kKeys = 64;   // keys per staged chunk (4 pages of 16)
constexpr int kThreads = 128;

// ---------------------------------------------------------------------------
// planner: tiles[i] = {first token, token count}; tiles_n = number of tiles;
// optionally order[] = tile indices by descending context of their last token
// (counting sort over 64-key buckets), so the longest tiles launch first.
// ---------------------------------------------------------------------------
constexpr int kOrderBuckets = 2048;

// Key-range parts of the tensor-core items (filled when `units` is given).
struct UnitPlan {
  int4 *units;        // [max_units] {tile, part | parts << 16, planned chunks, slot base}
  int32_t *tickets;   // [max_tiles * ny] arrival counters, zeroed here
  int ny;             // items per unit (kv heads x q-head groups)
  int nsm;            // SMs of the device
  int slot_cap;       // partial-result slots available
  int max_units;
};

// Exclusive block-wide scan (1024 threads) of v; returns the prefix, *total the sum.
VA_DEVINL int block_excl_scan(int v, int *warp_buf, int *total) {
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  int x = v;
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += n;
  }
  if (lane == 31) warp_buf[wid] = x;
  __syncthreads();
  if (wid == 0) {
    int w = warp_buf[lane];
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += n;
    }
    warp_buf[lane] = w;
  }
  __syncthreads();
  const int excl = x - v + (wid > 0 ? warp_buf[wid - 1] : 0);
  *total = warp_buf[31];
  __syncthreads();
  return excl;
}

__global__ void __launch_bounds__(1024) plan_tiles_kernel(const int32_t *token_to_seq,
                                                          const int32_t *positions,
                                                          int64_t T, int TQ, int2 *tiles,
                                                          int32_t *tiles_n, int64_t max_tiles,
                                                          int32_t *singles, int32_t *singles_n,
                                                          int32_t *order, int32_t *err,
                                                          UnitPlan up) {
  __shared__ int warp_buf[32];
  __shared__ int carry_max, carry_sum, n_single;
  __shared__ int bucket[kOrderBuckets];
  va::pdl_enter();
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  if (tid == 0) { carry_max = 0; carry_sum = 0; n_single = 0; }
  __syncthreads();
  for (int64_t base = 0; base < T; base += 1024) {
    const int64_t t = base + tid;
    const bool in = t < T;
    const int s = in ? token_to_seq[t] : 0;
    const bool run_start = in && (t == 0 || token_to_seq[t - 1] != s);
    // inclusive max-scan of run starts
    int v = run_start ? (int)t : -1;
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v = max(v, n);
    }
    if (lane == 31) warp_buf[wid] = v;
    __syncthreads();
    if (wid == 0) {
      int w = warp_buf[lane];
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w = max(w, n);
      }
      warp_buf[lane] = w;
    }
    __syncthreads();
    int rs = v;
    if (wid > 0) rs = max(rs, warp_buf[wid - 1]);
    rs = max(rs, carry_max);
    const bool tstart = in && ((t - rs) % TQ == 0);
    __syncthreads();
    if (tid == 1023) carry_max = rs;
    // exclusive sum-scan of tile starts
    int c = tstart ? 1 : 0;
    int x = c;
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += n;
    }
    if (lane == 31) warp_buf[wid] = x;
    __syncthreads();
    if (wid == 0) {
      int w = warp_buf[lane];
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += n;
      }
      warp_buf[lane] = w;
    }
    __syncthreads();
    const int excl = x - c + (wid > 0 ? warp_buf[wid - 1] : 0) + carry_sum;
    if (tstart) {
      if (excl < max_tiles) tiles[excl] = make_int2((int)t, 0);
      else va::raise_flag(err, VA_FLAG_CTX_OVERFLOW);
    }
    __syncthreads();
    if (tid == 1023) carry_sum = excl + c;
    __syncthreads();
  }
  __syncthreads();
  const int n = carry_sum < max_tiles ? carry_sum : (int)max_tiles;
  for (int i = tid; i < n; i += 1024) {
    const int next = (i + 1 < n) ? tiles[i + 1].x : (int)T;
    const int cnt = next - tiles[i].x;
    tiles[i].y = cnt;
    // one-token tiles (decode rows of a mixed batch) go to the split-KV decode kernel
    if (singles && cnt == 1) singles[atomicAdd(&n_single, 1)] = tiles[i].x;
  }
  __syncthreads();
  if (tid == 0) {
    *tiles_n = n;
    if (singles_n) *singles_n = n_single;
    tiles_n[2] = 0;  // item counter of the persistent tile kernel
  }
  if (!order) return;
  // bucket b holds tiles whose last token sees about 64 * (kOrderBuckets - 1 - b) keys
  auto bucket_of = [&](int i) {
    const int2 t = tiles[i];
    const int p = positions[t.x + t.y - 1];
    const int w = (p < 0 || (singles && t.y == 1)) ? 0 : (p >> 6) + 1;
    return kOrderBuckets - 1 - min(w, kOrderBuckets - 1);
  };
  for (int b = tid; b < kOrderBuckets; b += 1024) bucket[b] = 0;
  __syncthreads();
  for (int i = tid; i < n; i += 1024) atomicAdd(&bucket[bucket_of(i)], 1);
  __syncthreads();
  // exclusive scan of the bucket counts (two buckets per thread)
  {
    const int b0 = 2 * tid;
    const int c0 = bucket[b0], c1 = bucket[b0 + 1];
    int x = c0 + c1;
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_buf[wid] = x;
    __syncthreads();
    if (wid == 0) {
      int w = warp_buf[lane];
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      warp_buf[lane] = w;
    }
    __syncthreads();
    const int excl = x - (c0 + c1) + (wid > 0 ? warp_buf[wid - 1] : 0);
    bucket[b0] = excl;
    bucket[b0 + 1] = excl + c0;
  }
  __syncthreads();
  for (int i = tid; i < n; i += 1024) order[atomicAdd(&bucket[bucket_of(i)], 1)] = i;
  if (!up.units) return;
  __syncthreads();
  // ---- key-range parts: long tiles are cut into parts of about KP chunks of 64
  // keys, so the persistent grid's last items are short.  KP is half the
  // per-SM share of all the work (>= 16 chunks); the longest tiles are cut first,
  // as long as partial-result slots last.  Units follow the tile order (longest
  // first), the parts of a tile consecutively. ----
  auto chunks_of = [&](int i) {
    const int2 t = tiles[i];
    const int p = positions[t.x + t.y - 1];
    return (p < 0 || (singles && t.y == 1)) ? 0 : (p + 64) / 64;
  };
  __shared__ unsigned long long work_sum;
  __shared__ int carry_slot, carry_unit;
  if (tid == 0) { work_sum = 0ull; carry_slot = 0; carry_unit = 0; }
  __syncthreads();
  __shared__ int busy_tiles;
  if (tid == 0) busy_tiles = 0;
  __syncthreads();
  unsigned long long wloc = 0;
  int bloc = 0;
  for (int i = tid; i < n; i += 1024) {
    const int c = chunks_of(i);
    wloc += (unsigned long long)c;
    bloc += c > 0;
  }
  for (int o = 16; o > 0; o >>= 1) {
    wloc += __shfl_xor_sync(0xffffffffu, wloc, o);
    bloc += __shfl_xor_sync(0xffffffffu, bloc, o);
  }
  if (lane == 0 && wloc) atomicAdd(&work_sum, wloc);
  if (lane == 0 && bloc) atomicAdd(&busy_tiles, bloc);
  __syncthreads();
  // Cutting costs each part a pipeline fill, a partial write and (last part) a
  // merge; measured on B200 it pays only when there are fewer items than SMs
  // (config-4 shapes: 120 items at head_size 64 gained 11 %, 256 at head_size 128
  // lost 15 %), so tiles are cut only then.
  const bool cut = (long long)busy_tiles * up.ny < up.nsm;
  if (!cut) {  // one unit per tile, in the tile order
    for (int i = tid; i < n; i += 1024) {
      const int tile = order[i];
      up.units[i] = make_int4(tile, 1 << 16, chunks_of(tile), -1);
    }
    if (tid == 0) tiles_n[3] = n;
    return;
  }
  for (int i = tid; i < n * up.ny; i += 1024) up.tickets[i] = 0;
  const unsigned long long per_sm = work_sum * (unsigned long long)up.ny / (2ull * up.nsm);
  const int KP = (int)max(16ull, min(per_sm, 1ull << 20));
  for (int base = 0; base < n; base += 1024) {
    const int i = base + tid;
    const bool in = i < n;
    const int tile = in ? order[i] : 0;
    const int nch = in ? chunks_of(tile) : 0;
    int np = nch > KP ? (nch + KP - 1) / KP : 1;
    int tot;
    const int need = (in && np > 1) ? np * up.ny : 0;
    const int sbase = block_excl_scan(need, warp_buf, &tot) + carry_slot;
    int slot = -1;
    if (np > 1) {
      if (sbase + need <= up.slot_cap) slot = sbase;
      else np = 1;
    }
    const int ubase = block_excl_scan(in ? np : 0, warp_buf, &tot) + carry_unit;
    if (in)
      for (int p = 0; p < np; ++p)
        if (ubase + p < up.max_units)
          up.units[ubase + p] = make_int4(tile, p | (np << 16), nch, slot);
    __syncthreads();
    if (tid == 1023) {
      carry_slot = sbase + need;
      carry_unit = ubase + (in ? np : 0);
    }
    __syncthreads();
  }
  if (tid == 0) tiles_n[3] = min(carry_unit, up.max_units);
}

// ---------------------------------------------------------------------------
// attention
// ---------------------------------------------------------------------------
struct PrefillArgs {
  __half *out;
  const __half *q, *kc, *vc;
  const int32_t *bt, *tok_seq, *pos;
  const int2 *tiles;
  const int32_t *tiles_n;
  int32_t *err;
  int64_t num_seqs, max_blocks, num_blocks;
  int Hq, Hkv, G, hgroups, TQ, bs, skip_singles;
  float scale_log2;
  int64_t s_block, s_head, s_token, q_s_token, q_s_head, o_s_token, o_s_head;
};

VA_DEVINL void cp_async16(void *smem, const void *g) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(va::smem_addr(smem)), "l"(g)
               : "memory");
}
VA_DEVINL void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
VA_DEVINL void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

VA_DEVINL void ldsm_x4(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3, const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(va::smem_addr(p)));
}
VA_DEVINL void ldsm_x4_t(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3, const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(va::smem_addr(p)));
}
VA_DEVINL void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
VA_DEVINL uint32_t pack_h2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&h);
}

template <int D>
struct PShape {
  static constexpr int CPR = D / 8;        // 16-byte chunks per row
  static constexpr int LD = D + 8;         // padded row (halves): odd chunk count
  static constexpr size_t kTile = size_t(kKeys) * LD;  // halves per K or V chunk tile
  static constexpr size_t kSmem = (size_t(kRows) * LD + 4 * kTile) * 2;
};

template <int D, int GC>
__global__ void __launch_bounds__(kThreads) paged_prefill_kernel(const PrefillArgs a) {
  using S = PShape<D>;
  constexpr int LD = S::LD, CPR = S::CPR;
  extern __shared__ __align__(128) unsigned char smem[];
  __half *Qs = reinterpret_cast<__half *>(smem);
  __half *Ks = Qs + kRows * LD;       // [2][kKeys][LD]
  __half *Vs = Ks + 2 * S::kTile;     // [2][kKeys][LD]
  __shared__ int s_pos[kRows];        // per-token position (-1: token skipped)
  __shared__ int s_ctx, s_bad_from;

  const int tile = blockIdx.x;
  if (tile >= *a.tiles_n) return;
  const int2 td = a.tiles[tile];
  const int t0 = td.x, nq = td.y;
  if (nq == 1 && a.skip_singles) return;  // handled by the split-KV decode kernel
  const int seq = a.tok_seq[t0];
  const int kvh = blockIdx.y / a.hgroups, hg = blockIdx.y - (blockIdx.y / a.hgroups) * a.hgroups;
  const int head0 = kvh * a.G + hg * GC;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int BS = a.bs;

  if (tid == 0) { s_ctx = 0; s_bad_from = INT_MAX; }
  __syncthreads();
  if (tid < a.TQ) {
    int p = -1;
    if (tid < nq && seq >= 0 && seq < a.num_seqs) {
      p = a.pos[t0 + tid];
      if (p >= 0 && (int64_t)((p + BS) / BS) > a.max_blocks) {
        va::raise_flag(a.err, VA_FLAG_CTX_OVERFLOW);
        p = -1;
      }
      if (p < 0) p = -1;
    }
    s_pos[tid] = p;
    if (p >= 0) atomicMax(&s_ctx, p + 1);
  }
  __syncthreads();
  const int ctx = s_ctx;
  if (ctx == 0) return;
  const int32_t *bt_row = a.bt + (int64_t)seq * a.max_blocks;
  const int nchunks = (ctx + kKeys - 1) / kKeys;

  // ---- stage Q rows (token-major, head-minor) ----
  for (int i = tid; i < kRows * CPR; i += kThreads) {
    const int r = i / CPR, c = i - r * CPR;
    const int tk = r / GC, g = r - tk * GC;
    __half *dst = Qs + r * LD + c * 8;
    if (tk < nq && r < a.TQ * GC) {
      cp_async16(dst, a.q + (int64_t)(t0 + tk) * a.q_s_token + (int64_t)(head0 + g) * a.q_s_head +
                          c * 8);
    } else {
      *reinterpret_cast<uint4 *>(dst) = make_uint4(0, 0, 0, 0);
    }
  }

  auto load_chunk = [&](int ch, int buf) {
    __half *kd = Ks + buf * S::kTile, *vd = Vs + buf * S::kTile;
    for (int i = tid; i < kKeys * CPR; i += kThreads) {
      const int r = i / CPR, c = i - r * CPR;
      const int key = ch * kKeys + r;
      const int page = key / BS, off = key - page * BS;
      bool ok = key < ctx;
      int32_t blk = -1;
      if (ok) {
        blk = bt_row[page];
        if (blk < 0 || blk >= a.num_blocks) {
          ok = false;
          atomicMin(&s_bad_from, page * BS);
        }
      }
      __half *kdst = kd + r * LD + c * 8, *vdst = vd + r * LD + c * 8;
      if (ok) {
        const int64_t src = (int64_t)blk * a.s_block + (int64_t)kvh * a.s_head +
                            (int64_t)off * a.s_token + c * 8;
        cp_async16(kdst, a.kc + src);
        cp_async16(vdst, a.vc + src);
      } else {
        *reinterpret_cast<uint4 *>(kdst) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4 *>(vdst) = make_uint4(0, 0, 0, 0);
      }
    }
  };

  load_chunk(0, 0);
  cp_async_commit();

  // per-lane row bookkeeping: rows r0 = warp*16 + lane/4 and r0 + 8
  const int rA = warp * 16 + (lane >> 2), rB = rA + 8;
  const int tkA = rA / GC, tkB = rB / GC;
  const int posA = (rA < a.TQ * GC && tkA < a.TQ) ? s_pos[tkA] : -1;
  const int posB = (rB < a.TQ * GC && tkB < a.TQ) ? s_pos[tkB] : -1;

  uint32_t qf[D / 16][4];
  float o[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;

#pragma unroll 1
  for (int ch = 0; ch < nchunks; ++ch) {
    const int buf = ch & 1;
    if (ch + 1 < nchunks) {
      load_chunk(ch + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (ch == 0) {  // Q fragments (A operand), kept in registers for the whole loop
      const int lr = warp * 16 + (lane & 15), lc = (lane >> 4) * 8;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk)
        ldsm_x4(qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], Qs + lr * LD + kk * 16 + lc);
    }
    const __half *kt = Ks + buf * S::kTile, *vt = Vs + buf * S::kTile;
    // ---- S = Q K^T (16 rows x 64 keys per warp) ----
    float s[kKeys / 8][4];
#pragma unroll
    for (int n = 0; n < kKeys / 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int n = 0; n < kKeys / 8; n += 2) {
        // matrices: (n, k lo), (n, k hi), (n+1, k lo), (n+1, k hi)
        const int key = n * 8 + (lane & 7) + ((lane >> 4) << 3);
        const int col = kk * 16 + ((lane >> 3) & 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(b0, b1, b2, b3, kt + key * LD + col);
        mma16816(s[n], qf[kk], b0, b1);
        mma16816(s[n + 1], qf[kk], b2, b3);
      }
    }
    // ---- mask + online softmax ----
    float mxA = -INFINITY, mxB = -INFINITY;
#pragma unroll
    for (int n = 0; n < kKeys / 8; ++n) {
      const int j = ch * kKeys + n * 8 + 2 * (lane & 3);
      s[n][0] = (j <= posA) ? s[n][0] * a.scale_log2 : -INFINITY;
      s[n][1] = (j + 1 <= posA) ? s[n][1] * a.scale_log2 : -INFINITY;
      s[n][2] = (j <= posB) ? s[n][2] * a.scale_log2 : -INFINITY;
      s[n][3] = (j + 1 <= posB) ? s[n][3] * a.scale_log2 : -INFINITY;
      mxA = fmaxf(mxA, fmaxf(s[n][0], s[n][1]));
      mxB = fmaxf(mxB, fmaxf(s[n][2], s[n][3]));
    }
#pragma unroll
    for (int o2 = 1; o2 < 4; o2 <<= 1) {
      mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, o2));
      mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, o2));
    }
    const float mnA = fmaxf(mA, mxA), mnB = fmaxf(mB, mxB);
    const bool noneA = mnA == -INFINITY, noneB = mnB == -INFINITY;
    const float alA = noneA ? 1.f : va::fast_exp2(mA - mnA);
    const float alB = noneB ? 1.f : va::fast_exp2(mB - mnB);
    mA = mnA;
    mB = mnB;
    float sumA = 0.f, sumB = 0.f;
#pragma unroll
    for (int n = 0; n < kKeys / 8; ++n) {
      s[n][0] = noneA ? 0.f : va::fast_exp2(s[n][0] - mnA);
      s[n][1] = noneA ? 0.f : va::fast_exp2(s[n][1] - mnA);
      s[n][2] = noneB ? 0.f : va::fast_exp2(s[n][2] - mnB);
      s[n][3] = noneB ? 0.f : va::fast_exp2(s[n][3] - mnB);
      sumA += s[n][0] + s[n][1];
      sumB += s[n][2] + s[n][3];
    }
    lA = lA * alA + sumA;
    lB = lB * alB + sumB;
#pragma unroll
    for (int n = 0; n < D / 8; ++n) {
      o[n][0] *= alA; o[n][1] *= alA;
      o[n][2] *= alB; o[n][3] *= alB;
    }
    // ---- O += P V ----
#pragma unroll
    for (int kk = 0; kk < kKeys / 16; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_h2(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack_h2(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack_h2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack_h2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int n = 0; n < D / 8; n += 2) {
        const int key = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int col = n * 8 + (lane >> 4) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(b0, b1, b2, b3, vt + key * LD + col);
        mma16816(o[n], pa, b0, b1);
        mma16816(o[n + 1], pa, b2, b3);
      }
    }
    __syncthreads();  // buffer `buf` is refilled by the next iteration's prefetch
  }

  // ---- normalise + store ----
#pragma unroll
  for (int o2 = 1; o2 < 4; o2 <<= 1) {
    lA += __shfl_xor_sync(0xffffffffu, lA, o2);
    lB += __shfl_xor_sync(0xffffffffu, lB, o2);
  }
  const int bad_from = s_bad_from;
  if (bad_from != INT_MAX && tid == 0) va::raise_flag(a.err, VA_FLAG_BAD_BLOCK);
  const float invA = lA > 0.f ? 1.f / lA : 0.f, invB = lB > 0.f ? 1.f / lB : 0.f;
  const bool wA = posA >= 0 && posA < bad_from && tkA < nq;
  const bool wB = posB >= 0 && posB < bad_from && tkB < nq;
  const int gA = rA - tkA * GC, gB = rB - tkB * GC;
  __half *oA = a.out + (int64_t)(t0 + tkA) * a.o_s_token + (int64_t)(head0 + gA) * a.o_s_head;
  __half *oB = a.out + (int64_t)(t0 + tkB) * a.o_s_token + (int64_t)(head0 + gB) * a.o_s_head;
#pragma unroll
  for (int n = 0; n < D / 8; ++n) {
    const int c = n * 8 + 2 * (lane & 3);
    if (wA) *reinterpret_cast<uint32_t *>(oA + c) = pack_h2(o[n][0] * invA, o[n][1] * invA);
    if (wB) *reinterpret_cast<uint32_t *>(oB + c) = pack_h2(o[n][2] * invB, o[n][3] * invB);
  }
}

template <int D, int GC>
int launch_t(const PrefillArgs &a, dim3 grid, cudaStream_t st) {
  using S = PShape<D>;
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(paged_prefill_kernel<D, GC>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)S::kSmem) != cudaSuccess)
      return VA_ERR_LAUNCH;
    configured[dev] = 1;
  }
  paged_prefill_kernel<D, GC><<<grid, kThreads, S::kSmem, st>>>(a);
  return va_host::launch_status();
}

template <int D>
int launch_g(int gc, const PrefillArgs &a, dim3 grid, cudaStream_t st) {
  switch (gc) {
    case 1: return launch_t<D, 1>(a, grid, st);
    case 2: return launch_t<D, 2>(a, grid, st);
    case 3: return launch_t<D, 3>(a, grid, st);
    case 4: return launch_t<D, 4>(a, grid, st);
    case 5: return launch_t<D, 5>(a, grid, st);
    case 6: return launch_t<D, 6>(a, grid, st);
    case 7: return launch_t<D, 7>(a, grid, st);
    case 8: return launch_t<D, 8>(a, grid, st);
  }
  return VA_ERR_UNSUPPORTED;
}

template <int D, int GC>
int launch_tc_t(const tc::Args &a, const CUtensorMap &mk, const CUtensorMap &mv, dim3 grid,
                cudaStream_t st) {
  using S = tc::Smem<D>;
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(tc::paged_prefill_tc_kernel<D, GC>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)S::kBytes) != cudaSuccess)
      return VA_ERR_LAUNCH;
    configured[dev] = 1;
  }
  va_host::launch_pdl_smem(tc::paged_prefill_tc_kernel<D, GC>, grid, tc::kThreads, S::kBytes,
                           st, a, mk, mv);
  return va_host::launch_status();
}

template <int D>
int launch_tc_g(int gc, const tc::Args &a, const CUtensorMap &mk, const CUtensorMap &mv,
                dim3 grid, cudaStream_t st) {
  switch (gc) {
    case 1: return launch_tc_t<D, 1>(a, mk, mv, grid, st);
    case 2: return launch_tc_t<D, 2>(a, mk, mv, grid, st);
    case 3: return launch_tc_t<D, 3>(a, mk, mv, grid, st);
    case 4: return launch_tc_t<D, 4>(a, mk, mv, grid, st);
    case 5: return launch_tc_t<D, 5>(a, mk, mv, grid, st);
    case 6: return launch_tc_t<D, 6>(a, mk, mv, grid, st);
    case 7: return launch_tc_t<D, 7>(a, mk, mv, grid, st);
    case 8: return launch_tc_t<D, 8>(a, mk, mv, grid, st);
  }
  return VA_ERR_UNSUPPORTED;
}

// Cache layout the TMA path understands: 0 = [nb, H, bs, D], 1 = [nb, bs, H, D], -1 = other.
int tma_layout(int64_t sb, int64_t sh, int64_t st, int H, int bs, int D) {
  if (sb == (int64_t)H * bs * D && sh == (int64_t)bs * D && st == D) return 0;
  if (sb == (int64_t)bs * H * D && st == (int64_t)H * D && sh == D) return 1;
  return -1;
}

// 3-D tensor map over one cache tensor whose box is one page x 64 head dims,
// 128-byte swizzled.  The encoder comes from the driver through the runtime.
bool encode_page_map(CUtensorMap *m, const void *base, int nhd, int64_t nb, int H, int bs,
                     int D) {
  static PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
  if (!enc) {
    cudaDriverEntryPointQueryResult q;
    void *fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return false;
    enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  cuuint64_t dims[3], strides[2];
  cuuint32_t box[3], estr[3] = {1, 1, 1};
  dims[0] = (cuuint64_t)D;
  if (nhd) {  // (D, H, nb*bs): one head, bs token rows
    dims[1] = (cuuint64_t)H;
    dims[2] = (cuuint64_t)(nb * bs);
    strides[0] = (cuuint64_t)D * 2;
    strides[1] = (cuuint64_t)H * D * 2;
    box[0] = 64; box[1] = 1; box[2] = (cuuint32_t)bs;
  } else {  // (D, bs, nb*H): one (block, head) page
    dims[1] = (cuuint64_t)bs;
    dims[2] = (cuuint64_t)(nb * H);
    strides[0] = (cuuint64_t)D * 2;
    strides[1] = (cuuint64_t)bs * D * 2;
    box[0] = 64; box[1] = (cuuint32_t)bs; box[2] = 1;
  }
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(base), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Side stream of the one-token rows: they are HBM-bound split-KV decode work
// and run beside the compute-bound tile kernel (they fill the SMs the tiles'
// last wave leaves idle).  Forked from and joined to the caller's stream with
// events, so stream capture sees an ordinary fork / join.  One set per device;
// the mutex orders concurrent callers' use of the shared events.
struct SideStream {
  cudaStream_t s = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};
std::mutex g_side_mu;
SideStream g_side[64];

bool side_concurrency_enabled() {
  static int on = -1;
  if (on < 0) {
    const char *e = getenv("VA_PREFILL_CONCURRENT");
    on = (e && atoi(e) == 0) ? 0 : 1;
  }
  return on == 1;
}

int group_chunk(int g) {
  for (int c = 8; c >= 1; --c)
    if (g % c == 0) return c;
  return 1;
}

int64_t max_tiles_for(int64_t T, int64_t num_seqs, int TQ) {
  int64_t m = (T + TQ - 1) / TQ + num_seqs;
  return m < T ? m : T;
}

bool use_tc_kernel(int head_size) {
  static int force_legacy = -1;
  if (force_legacy < 0) {
    const char *e = getenv("VA_PREFILL_MMA_SYNC");
    force_legacy = (e && atoi(e) != 0) ? 1 : 0;
  }
  return !force_legacy && (head_size == 64 || head_size == 128);
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Workspace layout of one prefill call: [counters | tiles | one-token rows | decode partials].
struct PrefillPlan {
  int TQ, gc, ny, slot_cap, max_units;
  bool tc, route;
  int64_t mt, rows_bound;
  size_t o_tiles, o_singles, o_order, o_units, o_tickets, o_part_o, o_part_ml, o_part_bad,
      o_dec, dec_bytes, total;
};

// Bytes of partial results the tensor-core kernel may use for key-range parts.
constexpr size_t kPartBudget = size_t(64) << 20;

// `tc_layout` >= 0 when the tcgen05/TMA tile kernel can take this cache.  Buffer
// sizes use the smaller tile (more tiles) so they do not depend on the choice.
PrefillPlan prefill_plan(int64_t T, int64_t S, int Hq, int Hkv, int D, int bs, int64_t maxb,
                         int tc_layout) {
  PrefillPlan p{};
  p.gc = group_chunk(Hq / Hkv);
  p.tc = use_tc_kernel(D) && bs >= 8 && tc_layout >= 0;
  // the tcgen05 kernel takes a pair of tiles of kRows / gc tokens per CTA
  p.TQ = p.tc ? tc::kTiles * (tc::kRows / p.gc) : kRows / p.gc;
  p.mt = max_tiles_for(T, S, p.TQ);
  const int64_t bound = max_tiles_for(T, S, kRows / p.gc);
  p.route = bs == 16 && bound <= 65535;
  p.rows_bound = bound;
  p.o_tiles = 256;
  p.o_singles = p.o_tiles + align256((size_t)bound * sizeof(int2));
  p.o_order = p.o_singles + align256((size_t)bound * sizeof(int32_t));
  size_t at = p.o_order + align256((size_t)bound * sizeof(int32_t));
  if (p.tc) {
    // key-range parts of long tiles: unit list, per-(tile, item) tickets, and
    // partial (O, m, l) slots -- at most kPartBudget, and no more than every tile
    // cut into parts of 16 chunks could use
    p.ny = Hkv * ((Hq / Hkv) / p.gc);
    const size_t slot_bytes = (size_t)tc::kTiles * tc::kRows * ((size_t)D + 2) * 4 + 4;
    const int64_t max_nch = (maxb * bs + tc::kKeys - 1) / tc::kKeys;
    const int64_t maxp = (max_nch + 15) / 16;
    int64_t cap = (int64_t)(kPartBudget / slot_bytes);
    const int64_t want = maxp > 1 ? p.mt * p.ny * maxp : 0;
    cap = cap < want ? cap : want;
    p.slot_cap = (int)(cap < (1 << 24) ? cap : (1 << 24));
    p.max_units = (int)(p.mt + p.slot_cap);
    p.o_units = at;
    at += align256((size_t)p.max_units * sizeof(int4));
    p.o_tickets = at;
    at += align256((size_t)p.mt * p.ny * sizeof(int32_t));
    p.o_part_o = at;
    at += align256((size_t)p.slot_cap * tc::kTiles * tc::kRows * D * 4);
    p.o_part_ml = at;
    at += align256((size_t)p.slot_cap * tc::kTiles * tc::kRows * 8);
    p.o_part_bad = at;
    at += align256((size_t)p.slot_cap * 4);
  }
  p.o_dec = at;
  p.dec_bytes = p.route ? va_internal::decode_rows_workspace(bound, Hq, Hkv, D, bs, maxb) : 0;
  p.total = p.o_dec + p.dec_bytes;
  return p;
}

}  // namespace

extern "C" size_t va_paged_prefill_workspace_size(int64_t num_tokens, int64_t num_seqs,
                                                  int num_query_heads, int num_kv_heads,
                                                  int head_size, int block_size,
                                                  int64_t max_blocks_per_seq) {
  if (num_tokens <= 0 || num_kv_heads <= 0 || num_query_heads <= 0 ||
      num_query_heads % num_kv_heads)
    return 0;
  return prefill_plan(num_tokens, num_seqs, num_query_heads, num_kv_heads, head_size,
                      block_size, max_blocks_per_seq, 0)
      .total;
}

extern "C" int va_paged_prefill(void *out, const void *q, const void *k_cache,
                                const void *v_cache, const int32_t *block_table,
                                const int32_t *token_to_seq, const int32_t *positions,
                                int64_t num_tokens, int64_t num_seqs, int num_query_heads,
                                int num_kv_heads, int head_size, int block_size,
                                int64_t max_blocks_per_seq, int64_t num_blocks, float scale,
                                int64_t s_block, int64_t s_head, int64_t s_token,
                                int64_t q_s_token, int64_t q_s_head, int64_t o_s_token,
                                int64_t o_s_head, void *workspace, size_t workspace_bytes,
                                int32_t *err_flag, void *stream) {
  if (num_tokens < 0 || num_seqs < 0 || max_blocks_per_seq < 0 || num_blocks < 0)
    return VA_ERR_INVALID_ARG;
  if (num_tokens == 0) return VA_OK;
  if (!out || !q || !k_cache || !v_cache || !block_table || !token_to_seq || !positions)
    return VA_ERR_INVALID_ARG;
  if (num_kv_heads <= 0 || num_query_heads <= 0 || num_query_heads % num_kv_heads)
    return VA_ERR_INVALID_ARG;
  if (head_size != 32 && head_size != 64 && head_size != 96 && head_size != 128)
    return VA_ERR_UNSUPPORTED;
  if (block_size <= 0 || block_size > kKeys || kKeys % block_size) return VA_ERR_UNSUPPORTED;
  if (num_tokens > INT32_MAX / 2) return VA_ERR_UNSUPPORTED;
  auto m8 = [](int64_t s) { return s % 8 == 0; };
  if (!va_host::aligned16(q) || !va_host::aligned16(k_cache) || !va_host::aligned16(v_cache) ||
      !va_host::aligned16(out) || !m8(s_block) || !m8(s_head) || !m8(s_token) ||
      !m8(q_s_token) || !m8(q_s_head) || o_s_token % 2 || o_s_head % 2)
    return VA_ERR_INVALID_ARG;
  // the tensor-core kernel folds the scale into its exponent and needs it > 0
  const int layout = scale > 0.f
                         ? tma_layout(s_block, s_head, s_token, num_kv_heads, block_size, head_size)
                         : -1;
  const PrefillPlan pl = prefill_plan(num_tokens, num_seqs, num_query_heads, num_kv_heads,
                                      head_size, block_size, max_blocks_per_seq, layout);
  if (!workspace || workspace_bytes < pl.total) return VA_ERR_WORKSPACE;
  const int G = num_query_heads / num_kv_heads;
  const int gc = pl.gc;
  const bool use_tc = pl.tc;
  const int TQ = pl.TQ;
  const int64_t mt = pl.mt;
  if (mt > INT32_MAX) return VA_ERR_UNSUPPORTED;

  unsigned char *ws = static_cast<unsigned char *>(workspace);
  int32_t *tiles_n = reinterpret_cast<int32_t *>(ws);
  int32_t *singles_n = tiles_n + 1;
  int2 *tiles = reinterpret_cast<int2 *>(ws + pl.o_tiles);
  int32_t *singles = reinterpret_cast<int32_t *>(ws + pl.o_singles);
  auto st = static_cast<cudaStream_t>(stream);
  int32_t *order = reinterpret_cast<int32_t *>(ws + pl.o_order);
  UnitPlan up{};
  if (use_tc) {
    up.units = reinterpret_cast<int4 *>(ws + pl.o_units);
    up.tickets = reinterpret_cast<int32_t *>(ws + pl.o_tickets);
    up.ny = pl.ny;
    up.nsm = va_host::sm_count();
    up.slot_cap = pl.slot_cap;
    up.max_units = pl.max_units;
  }
  va_host::launch_pdl(plan_tiles_kernel, 1, 1024, st, token_to_seq, positions, num_tokens, TQ,
                      tiles, tiles_n, mt, pl.route ? singles : nullptr,
                      pl.route ? singles_n : nullptr, use_tc ? order : nullptr, err_flag, up);
  if (va_host::launch_status() != VA_OK) return VA_ERR_LAUNCH;
  auto launch_rows = [&](cudaStream_t rs) {
    return va_internal::decode_rows(
        out, q, k_cache, v_cache, block_table, singles, singles_n, token_to_seq, positions,
        pl.rows_bound,
        num_seqs, num_query_heads, num_kv_heads, head_size, block_size, max_blocks_per_seq,
        num_blocks, scale, s_block, s_head, s_token, q_s_token, q_s_head, o_s_token, o_s_head,
        ws + pl.o_dec, pl.dec_bytes, err_flag, rs);
  };
  // the rows go beside the tile kernel on the side stream when the tiles run on
  // the tensor-core kernel; otherwise (and if the side stream cannot be set up)
  // in order on the caller's stream
  SideStream *side = nullptr;
  std::unique_lock<std::mutex> side_lock(g_side_mu, std::defer_lock);
  if (pl.route && use_tc && side_concurrency_enabled()) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64) {
      side_lock.lock();
      SideStream &ss = g_side[dev];
      cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
      cudaStreamIsCapturing(st, &cap);
      // created outside stream capture only (the first eager call does it)
      if (!ss.s && cap == cudaStreamCaptureStatusNone) {
        if (cudaStreamCreateWithFlags(&ss.s, cudaStreamNonBlocking) != cudaSuccess ||
            cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&ss.join, cudaEventDisableTiming) != cudaSuccess) {
          cudaGetLastError();
          ss = SideStream{};
        }
      }
      if (ss.s) side = &ss;
      else side_lock.unlock();
    }
  }
  if (pl.route && !side) {
    const int rc = launch_rows(st);
    if (rc != VA_OK) return rc;
  }

  PrefillArgs a{};
  a.out = static_cast<__half *>(out);
  a.q = static_cast<const __half *>(q);
  a.kc = static_cast<const __half *>(k_cache);
  a.vc = static_cast<const __half *>(v_cache);
  a.bt = block_table;
  a.tok_seq = token_to_seq;
  a.pos = positions;
  a.tiles = tiles;
  a.tiles_n = tiles_n;
  a.err = err_flag;
  a.num_seqs = num_seqs;
  a.max_blocks = max_blocks_per_seq;
  a.num_blocks = num_blocks;
  a.Hq = num_query_heads;
  a.Hkv = num_kv_heads;
  a.G = G;
  a.hgroups = G / gc;
  a.TQ = TQ;
  a.bs = block_size;
  a.skip_singles = pl.route ? 1 : 0;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.s_block = s_block; a.s_head = s_head; a.s_token = s_token;
  a.q_s_token = q_s_token; a.q_s_head = q_s_head;
  a.o_s_token = o_s_token; a.o_s_head = o_s_head;
  const dim3 grid((unsigned)mt, (unsigned)(num_kv_heads * a.hgroups));
  if (use_tc) {
    tc::Args t{};
    t.out = a.out; t.q = a.q; t.kc = a.kc; t.vc = a.vc; t.bt = a.bt; t.tok_seq = a.tok_seq;
    t.pos = a.pos; t.tiles = a.tiles; t.err = a.err;
    t.units = up.units; t.units_n = tiles_n + 3; t.tickets = up.tickets;
    t.part_o = reinterpret_cast<float *>(ws + pl.o_part_o);
    t.part_ml = reinterpret_cast<float2 *>(ws + pl.o_part_ml);
    t.part_bad = reinterpret_cast<int32_t *>(ws + pl.o_part_bad);
    t.work = tiles_n + 2;
    t.num_seqs = a.num_seqs; t.max_blocks = a.max_blocks; t.num_blocks = a.num_blocks;
    t.Hq = a.Hq; t.Hkv = a.Hkv; t.G = a.G; t.hgroups = a.hgroups; t.TQ = a.TQ / tc::kTiles;
    t.bs = a.bs;
    t.skip_singles = a.skip_singles;
    t.nhd = layout;
    t.scale_log2 = a.scale_log2; t.s_block = a.s_block; t.s_head = a.s_head;
    t.s_token = a.s_token; t.q_s_token = a.q_s_token; t.q_s_head = a.q_s_head;
    t.o_s_token = a.o_s_token; t.o_s_head = a.o_s_head;
    CUtensorMap mk, mv;
    if (!encode_page_map(&mk, k_cache, layout, num_blocks, num_kv_heads, block_size, head_size) ||
        !encode_page_map(&mv, v_cache, layout, num_blocks, num_kv_heads, block_size, head_size))
      return VA_ERR_LAUNCH;
    // persistent: one CTA per SM (shared memory and TMEM allow no more), items
    // taken in the planner's longest-first order (bounded by its unit capacity)
    const int64_t nitems = (int64_t)pl.max_units * grid.y;
    if (nitems > INT32_MAX) return VA_ERR_UNSUPPORTED;
    const int64_t nsm = va_host::sm_count();
    const dim3 grid1((unsigned)(nitems < nsm ? nitems : nsm));
    if (side && cudaEventRecord(side->fork, st) != cudaSuccess) return VA_ERR_LAUNCH;
    const int rc = head_size == 64 ? launch_tc_g<64>(gc, t, mk, mv, grid1, st)
                                   : launch_tc_g<128>(gc, t, mk, mv, grid1, st);
    if (!side) return rc;
    // join even when the tile launch failed, so the caller's stream never
    // runs ahead of the rows
    if (cudaStreamWaitEvent(side->s, side->fork, 0) != cudaSuccess) return VA_ERR_LAUNCH;
    const int rr = launch_rows(side->s);
    if (cudaEventRecord(side->join, side->s) != cudaSuccess ||
        cudaStreamWaitEvent(st, side->join, 0) != cudaSuccess)
      return VA_ERR_LAUNCH;
    return rc != VA_OK ? rc : rr;
  }
  switch (head_size) {
    case 32: return launch_g<32>(gc, a, grid, st);
    case 64: return launch_g<64>(gc, a, grid, st);
    case 96: return launch_g<96>(gc, a, grid, st);
    case 128: return launch_g<128>(gc, a, grid, st);
  }
  return VA_ERR_UNSUPPORTED;
}
