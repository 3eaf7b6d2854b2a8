// Token-parallel causal paged attention on the 5th-generation tensor cores
// (tcgen05 UMMA, TMEM accumulators), head_size 64 or 128.  Included by
// paged_prefill.cu, which owns the tile planner and the C-ABI entry point.
//
// Persistent CTAs (one per SM: shared memory and TMEM allow no more) take
// items = (tile pair, kv head [, q-head group]) from a counter in the planner's
// order, longest context first; 11 warps with fixed roles per item.
//   * A tile = 128 MMA rows = (token, q head) pairs of up to 128/G consecutive
//     tokens of one sequence; a CTA owns two consecutive tiles of the same
//     sequence, so every staged K/V chunk serves both tiles and every head of
//     the group.  Warpgroup h (warps 4h..4h+3) runs the softmax of tile h, one
//     thread per row (TMEM lane = row).
//   * Warp 8 (producer) streams K and V in chunks of 64 keys by TMA
//     (cp.async.bulk.tensor.3d, one box per page and 64 head dims, hardware
//     128-byte swizzle, no multicast) into kStages stages; a stage is reused
//     once the tensor core has finished with it (tcgen05.commit on the
//     stage's "empty" barrier).  Block ids are read a warp-group of pages
//     ahead; invalid pages and pages past the context are zero-filled, and
//     the page holding the end of the context is copied row by row with its
//     tail zeroed (V rows past the context must not hold NaN: P = 0 there).
//   * Warp 9 + h (MMA for tile h) issues S_h = Q_h K^T (M=128, N=64, K=D) two
//     chunks ahead into one of two TMEM buffers, and O_h += P_h V once warpgroup
//     h has written P_h (fp16) over the first 32 columns of that chunk's S
//     buffer: A is read from TMEM (the tcgen05.mma [a_tmem] form), B = V as an
//     MN-major operand (the same shared-memory image as K).  Keeping P out of
//     shared memory matters: the UMMA operand reads, the TMA writes and the P
//     stores all share the SM's 128 B/clk of shared-memory bandwidth.  One
//     issuing warp per tile: neither tile waits for the other's softmax; a
//     stage is free when both warps committed it.
//   * Softmax: log2-domain online softmax; the max only moves when it grows by
//     more than 2^8, so O is rarely rescaled in TMEM (only then does the
//     softmax wait for the previous PV).
//   * Q is staged once per item by cp.async from the softmax and MMA warps, while
//     the producer already streams the first chunks.  TMEM is allocated once per
//     CTA; the mbarriers are re-initialised between items, after every arrival
//     of the previous item has landed.
//   * Every wait on an mbarrier is bounded and reports VA_FLAG_WAIT_TIMEOUT;
//     after a timeout the CTA runs to the end without waiting or issuing,
//     waits (bounded) for its copies and MMAs in flight and frees TMEM.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace tc {

constexpr int kRows = 128;  // MMA M
constexpr int kKeys = 64;   // keys per chunk (MMA N of S, MMA K of PV)
constexpr int kTiles = 2;   // tiles (softmax warpgroups) per CTA
constexpr int kSoftmax = kTiles * kRows;  // softmax threads, one per row
constexpr int kProducerWarp = kSoftmax / 32, kMmaWarp = kProducerWarp + 1;  // MMA: 9, 10
constexpr int kMath = kSoftmax + 32 * kTiles;  // softmax + MMA threads
constexpr int kThreads = kMath + 32;           // + producer warp
constexpr uint32_t kTmemCols = 512;  // S: 2 tiles x 2 buffers x 64; O: 2 tiles x D (<= 128)
constexpr uint32_t kWaitLimit = 1u << 22;
constexpr int kStages = 5;  // K/V chunks in flight (a chunk = 64 keys of K and of V)

// ---- PTX wrappers (tcgen05 family, sm_100a) --------------------------------
VA_DEVINL void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   va::smem_addr(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
VA_DEVINL void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
VA_DEVINL void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
VA_DEVINL void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16, fp32 accumulate.
VA_DEVINL void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]: A (M x K fp16, K-major) read from TMEM, one
// row per lane, two fp16 per 32-bit column (K = 16 per instruction: 8 columns).
VA_DEVINL void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once every MMA issued so far by this thread has completed.
VA_DEVINL void umma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          va::smem_addr(bar))
      : "memory");
}

#define VA_R8(i) "=r"(v[i]), "=r"(v[i + 1]), "=r"(v[i + 2]), "=r"(v[i + 3]), "=r"(v[i + 4]), \
                 "=r"(v[i + 5]), "=r"(v[i + 6]), "=r"(v[i + 7])
// 32 consecutive fp32 columns of this thread's TMEM lane.
VA_DEVINL void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : VA_R8(0), VA_R8(8), VA_R8(16), VA_R8(24)
      : "r"(taddr));
}
#undef VA_R8
#define VA_W8(i) "r"(v[i]), "r"(v[i + 1]), "r"(v[i + 2]), "r"(v[i + 3]), "r"(v[i + 4]), \
                 "r"(v[i + 5]), "r"(v[i + 6]), "r"(v[i + 7])
VA_DEVINL void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
      "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(
          taddr),
      VA_W8(0), VA_W8(8), VA_W8(16), VA_W8(24)
      : "memory");
}
#undef VA_W8
VA_DEVINL void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
VA_DEVINL void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

VA_DEVINL void cp_async16(void *smem, const void *g) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(va::smem_addr(smem)), "l"(g)
               : "memory");
}
VA_DEVINL void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
VA_DEVINL void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// 3-D tiled TMA load global -> shared, completion as tx bytes on `bar`.
VA_DEVINL void tma_load_3d(void *dst, const CUtensorMap *map, int c0, int c1, int c2,
                           uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(va::smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(va::smem_addr(bar))
      : "memory");
}

// ---- packed fp32 pairs (sm_100 f32x2 arithmetic) -----------------------------
VA_DEVINL uint64_t pk2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
VA_DEVINL void upk2(uint64_t v, float &lo, float &hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
VA_DEVINL uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
VA_DEVINL uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
VA_DEVINL float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// ---- descriptors ------------------------------------------------------------
// Shared-memory matrix descriptor, 128-byte swizzle (canonical 8-row x 128 B
// atoms, atoms 1024-byte aligned).  lbo/sbo in bytes.
VA_DEVINL uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
}
// Instruction descriptor, kind::f16: fp16 A/B, fp32 accumulate, M x N.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool b_mn_major) {
  return (1u << 4) | ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

// Byte offset of element (row, col) of a [rows x cols] fp16 tile stored as
// cols/64 blocks of [rows x 128 B], each 128-byte-swizzled.
__host__ __device__ constexpr uint32_t sw128_off(int row, int col, int rows) {
  return (uint32_t)((col >> 6) * rows * 128 + row * 128 +
                    ((((col & 63) >> 3) ^ (row & 7)) << 4) + (col & 7) * 2);
}

struct Args {
  __half *out;
  const __half *q, *kc, *vc;
  const int32_t *bt, *tok_seq, *pos;
  const int2 *tiles;
  const int4 *units;      // {tile, part | parts << 16, planned chunks, slot base}, longest first
  const int32_t *units_n;
  int32_t *tickets;       // [tile * ny + yb] parts finished (zeroed by the planner)
  float *part_o;          // [slot][tile h][D][kRows] un-normalised O of a key-range part
  float2 *part_ml;        // [slot][tile h][kRows] (m, l) of that part
  int32_t *part_bad;      // [slot] first context position behind a bad block (INT_MAX: none)
  int32_t *work;  // item counter (zeroed by the planner)
  int32_t *err;
  int64_t num_seqs, max_blocks, num_blocks;
  int Hq, Hkv, G, hgroups;
  int TQ;  // tokens per tile (a CTA owns up to 2 * TQ)
  int bs, skip_singles;
  int nhd;  // cache layout of the tensor maps: 0 = [nb, H, bs, D], 1 = [nb, bs, H, D]
  float scale_log2;
  int64_t s_block, s_head, s_token, q_s_token, q_s_head, o_s_token, o_s_head;
};

template <int D>
struct Smem {
  static constexpr uint32_t kQ = kRows * D * 2;      // 16/32 KB per tile
  static constexpr uint32_t kKV = kKeys * D * 2;     // 8/16 KB per chunk
  static constexpr uint32_t oQ = 0, oK = kTiles * kQ, oV = oK + kStages * kKV,
                            oBar = oV + kStages * kKV;  // mbarriers + tmem slot
  static constexpr uint32_t oPos = oBar + 256;        // int [kTiles][kRows]
  static constexpr uint32_t kBytes = oPos + kTiles * kRows * 4 + 1024;  // + 1 KB alignment slack
};

// Named barrier over the softmax and MMA warps (the producer warp runs free).
VA_DEVINL void math_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kMath) : "memory"); }
// The softmax warpgroups (both tiles), for the key-range part epilogue.
VA_DEVINL void softmax_sync() { asm volatile("bar.sync 3, %0;" ::"n"(kSoftmax) : "memory"); }
// Every warp of the CTA, met from different places in the role code.
VA_DEVINL void all_sync() { asm volatile("bar.sync 2, %0;" ::"n"(kThreads) : "memory"); }

template <int D, int GC>
__global__ void __launch_bounds__(kThreads, 1)
    paged_prefill_tc_kernel(const Args a, const __grid_constant__ CUtensorMap tmk,
                            const __grid_constant__ CUtensorMap tmv) {
  using S = Smem<D>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  // 128-byte swizzle atoms must sit on 1024-byte boundaries of the shared window
  unsigned char *smem = smem_raw + ((1024u - (va::smem_addr(smem_raw) & 1023u)) & 1023u);
  uint64_t *bar_full = reinterpret_cast<uint64_t *>(smem + S::oBar);  // [kStages] chunk landed
  uint64_t *bar_empty = bar_full + kStages;  // [kStages] both MMA warps done with the stage
  uint64_t *bar_s = bar_empty + kStages;     // [kTiles][2] S buffer written
  uint64_t *bar_p = bar_s + 2 * kTiles;      // [kTiles] P published (kRows arrivals)
  uint64_t *bar_pv = bar_p + kTiles;         // [kTiles] PV done
  uint64_t *bar_done = bar_pv + kTiles;      // [kTiles] every MMA of the tile retired
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bar_done + kTiles);
  int *s_pos = reinterpret_cast<int *>(smem + S::oPos);  // [kTiles][kRows]
  __shared__ int s_ctx[kTiles], s_bad_from, s_dead, s_item[2], s_last;

  // the planner's tiles, units and counter are read below: wait for it
  va::pdl_enter();
  const int ny = a.Hkv * a.hgroups;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int BS = a.bs, TQ = a.TQ;
  const int nitems = *a.units_n * ny;
  if ((int)blockIdx.x >= nitems) return;
  if (tid == 0) s_dead = 0;
  if (warp == kMmaWarp) tmem_alloc(tmem_slot, kTmemCols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  constexpr int CPR = D / 8;  // 16-byte pieces per row

  auto dead = [&]() { return *(volatile int *)&s_dead != 0; };
  // A build with -DVA_DIAG_SITES also sets bit 8 + site of the error word, naming
  // the wait that gave up: 0 producer / stage free, 1-2 producer teardown, 3 MMA /
  // chunk landed, 4 MMA / P published, 5 MMA teardown, 6 softmax / S written,
  // 7 softmax / PV before a rescale, 8 softmax / last PV.
  auto timeout = [&](int site = 15) {
#ifdef VA_DIAG_SITES
    va::raise_flag(a.err, 0x100 << site);
#endif
    if (atomicExch(&s_dead, 1) == 0) va::raise_flag(a.err, VA_FLAG_WAIT_TIMEOUT);
  };
  auto wait_bar = [&](uint64_t *bar, uint32_t parity, int site = 15) {
    if (dead()) return;
    if (!va::mbar_wait_bounded(bar, parity, kWaitLimit)) timeout(site);
  };
  bool inited = false;  // thread 0: the mbarriers hold an earlier item's state

  // Persistent: each CTA takes (tile pair, kv head) items from a counter in the
  // planner's order (longest context first) until none is left.
#pragma unroll 1
  for (int iter = 0;; ++iter) {
    if (tid == 0) s_item[iter & 1] = atomicAdd(a.work, 1);
    __syncthreads();
    const int it = s_item[iter & 1];
    if (it >= nitems || dead()) break;  // uniform
    const int item = it / ny, yb = it - item * ny;
    const int4 unit = a.units[item];
    const int tile = unit.x, kpart = unit.y & 0xFFFF, nparts = unit.y >> 16;
    const int2 td = a.tiles[tile];
    const int t0 = td.x, nq = td.y;
    if (nq == 1 && a.skip_singles) continue;  // handled by the split-KV decode kernel
    const int seq = a.tok_seq[t0];
    const int kvh = yb / a.hgroups;
    const int hg = yb - kvh * a.hgroups;
    const int head0 = kvh * a.G + hg * GC;

    if (tid < kTiles) s_ctx[tid] = 0;
    if (tid == 0) s_bad_from = INT_MAX;
    __syncthreads();
    if (tid < kSoftmax) {
      const int h = tid / kRows, tk = tid % kRows;
      int p = -1;
      const int ti = h * TQ + tk;
      if (tk < TQ && ti < nq && seq >= 0 && seq < a.num_seqs) {
        p = a.pos[t0 + ti];
        if (p >= 0 && (int64_t)((p + BS) / BS) > a.max_blocks) {
          va::raise_flag(a.err, VA_FLAG_CTX_OVERFLOW);
          p = -1;
        }
        if (p < 0) p = -1;
      }
      s_pos[tid] = p;
      if (p >= 0) atomicMax(&s_ctx[h], p + 1);
    }
    if (tid == 0) {
      // every phase of the previous item has completed (its roles met at the end)
      uint64_t *bars = bar_full;
      constexpr int kBars = 2 * kStages + 5 * kTiles;
      if (inited)
        for (int i = 0; i < kBars; ++i) va::mbar_inval(&bars[i]);
      for (int i = 0; i < kStages; ++i) {
        va::mbar_init(&bar_full[i], 1);
        va::mbar_init(&bar_empty[i], kTiles);
      }
      for (int i = 0; i < 2 * kTiles; ++i) va::mbar_init(&bar_s[i], 1);
      for (int i = 0; i < kTiles; ++i) {
        va::mbar_init(&bar_p[i], kRows);
        va::mbar_init(&bar_pv[i], 1);
        va::mbar_init(&bar_done[i], 1);
      }
      va::fence_barrier_init();
      inited = true;
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const int ctx = max(s_ctx[0], s_ctx[1]);
    if (ctx == 0) continue;  // nothing to attend (all tokens skipped): in every part
    const int nch_all = (ctx + kKeys - 1) / kKeys;
    // this unit's key range: chunks [cb, cb + nch) of the context (all of it when
    // the tile is not cut into parts)
    const int cb = nparts > 1 ? kpart * unit.z / nparts : 0;
    const int ce = nparts > 1 ? min((kpart + 1) * unit.z / nparts, nch_all) : nch_all;
    const int nch = ce > cb ? ce - cb : 0;
    const int32_t *bt_row = a.bt + (int64_t)seq * a.max_blocks;

    if (warp == kProducerWarp) {
      // =================== producer: K/V chunks into the stages ===================
      const int npc = kKeys / BS;  // a power of two <= 8: a chunk never straddles a group
      const int pages = (ctx + BS - 1) / BS;  // <= max_blocks (checked above)
      const int tail_rows = ctx - (pages - 1) * BS;  // rows of the last page inside the context
      // block ids are read 32 pages (one per lane) at a time, one group ahead
      auto load_group = [&](int g) -> int32_t {
        const int page = g * 32 + lane;
        return page < pages ? __ldg(bt_row + page) : -1;
      };
      int gi = (cb * npc) >> 5;
      int32_t g_cur = load_group(gi), g_next = load_group(gi + 1);
#pragma unroll 1
      for (int i = 0; i < nch; ++i) {  // i: local chunk index, c: chunk of the context
        const int c = cb + i;
        const int buf = i % kStages;
        const int first = c * npc;
        if ((first >> 5) != gi) {
          gi = first >> 5;
          g_cur = g_next;
          g_next = load_group(gi + 1);
        }
        const int32_t gid = __shfl_sync(0xffffffffu, g_cur, (first & 31) + (lane & (npc - 1)));
        if (i >= kStages) wait_bar(&bar_empty[buf], (uint32_t)(((i / kStages) - 1) & 1), 0);
        // page ids of this chunk (lane p holds page p)
        int32_t id = -1;
        const int page = first + lane;
        if (lane < npc && page < pages) {
          id = gid;
          if (id < 0 || id >= a.num_blocks) {
            atomicMin(&s_bad_from, page * BS);
            id = -2;
          }
        }
        unsigned char *kb = smem + S::oK + buf * S::kKV, *vb = smem + S::oV + buf * S::kKV;
        // by TMA: valid whole pages; by the warp: the partial last page (copied, tail
        // zeroed) and invalid / past-context pages (zeroed)
        const bool part = page == pages - 1 && tail_rows < BS;
        const unsigned valid = __ballot_sync(0xffffffffu, lane < npc && id >= 0 && !part);
        const unsigned partial = __ballot_sync(0xffffffffu, lane < npc && id >= 0 && part);
        if (valid != (1u << npc) - 1u) {  // only near the end of the context
          const int ppage = partial ? __ffs(partial) - 1 : -1;
          const int32_t pid = __shfl_sync(0xffffffffu, id, ppage < 0 ? 0 : ppage);
          for (int i = lane; i < kKeys * CPR; i += 32) {
            const int r = i / CPR, ch16 = i - r * CPR;
            const int p = r / BS;
            if ((valid >> p) & 1u) continue;
            const uint32_t o = sw128_off(r, ch16 * 8, kKeys);
            uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
            if (p == ppage && r - p * BS < tail_rows) {
              const int64_t off = (int64_t)pid * a.s_block + (int64_t)kvh * a.s_head +
                                  (int64_t)(r - p * BS) * a.s_token + ch16 * 8;
              kv = __ldg(reinterpret_cast<const uint4 *>(a.kc + off));
              vv = __ldg(reinterpret_cast<const uint4 *>(a.vc + off));
            }
            *reinterpret_cast<uint4 *>(kb + o) = kv;
            *reinterpret_cast<uint4 *>(vb + o) = vv;
          }
          va::fence_proxy_async_smem();
          __syncwarp();
        }
        if (lane == 0) va::mbar_arrive_expect_tx(&bar_full[buf], __popc(valid) * (2u * BS * D * 2u));
        __syncwarp();
        {  // one box per lane: lane = (page, 64-column block, K or V)
          constexpr int kBoxes = D / 64 * 2;
          const int p = lane / kBoxes, rem = lane - p * kBoxes;
          const int kbk = rem >> 1;
          const int pidl = __shfl_sync(0xffffffffu, id, p & 31);
          if (p < npc && ((valid >> p) & 1u)) {
            const uint32_t off = kbk * kKeys * 128 + p * BS * 128;
            const int c1 = a.nhd ? kvh : 0;
            const int c2 = a.nhd ? pidl * BS : pidl * a.Hkv + kvh;
            if (rem & 1)
              tma_load_3d(vb + off, &tmv, kbk * 64, c1, c2, &bar_full[buf]);
            else
              tma_load_3d(kb + off, &tmk, kbk * 64, c1, c2, &bar_full[buf]);
          }
        }
        __syncwarp();
        if (dead()) break;
      }
      // Before the barriers are re-initialised for the next item, nothing may still
      // arrive on them: no copy may still be landing (normally none is: the MMA
      // warps consumed every chunk), and the stage releases the MMA warps commit
      // for the last chunks -- which nobody else waits for -- must have arrived.
      // Bounded, reported like any other wait.
      if (lane == 0) {
        for (int c = nch - kStages < 0 ? 0 : nch - kStages; c < nch; ++c) {
          const uint32_t par = (uint32_t)((c / kStages) & 1);
          if (!va::mbar_wait_bounded(&bar_full[c % kStages], par, kWaitLimit)) timeout(1);
          if (!dead() && !va::mbar_wait_bounded(&bar_empty[c % kStages], par, kWaitLimit))
            timeout(2);
        }
      }
      __syncwarp();
      all_sync();
    } else {
      // ---- Q of both tiles: cp.async by the softmax and MMA warps ----
      const int mtid = warp > kProducerWarp ? tid - 32 : tid;  // 0 .. kMath - 1
      for (int i = mtid; i < kTiles * kRows * CPR; i += kMath) {
        const int r2 = i / CPR, c = i - r2 * CPR;
        const int h = r2 / kRows, r = r2 - h * kRows;
        const int tk = r / GC, g = r - tk * GC;
        const int ti = h * TQ + tk;
        unsigned char *dst = smem + S::oQ + h * S::kQ + sw128_off(r, c * 8, kRows);
        if (tk < TQ && ti < nq)
          cp_async16(dst, a.q + (int64_t)(t0 + ti) * a.q_s_token + (int64_t)(head0 + g) * a.q_s_head +
                              c * 8);
        else
          *reinterpret_cast<uint4 *>(dst) = make_uint4(0, 0, 0, 0);
      }
      cp_async_commit();
      cp_async_wait<0>();
      va::fence_proxy_async_smem();
      math_sync();

      if (warp > kProducerWarp) {
        // =================== MMA issue for tile h (lane 0) ===================
        const int h = warp - kMmaWarp;
        // local chunks of this unit that hold keys of tile h
        const int nj = min(max((s_ctx[h] + kKeys - 1) / kKeys - cb, 0), nch);
        const uint32_t sQ = va::smem_addr(smem + S::oQ) + h * S::kQ;
        const uint32_t sK = va::smem_addr(smem + S::oK);
        const uint32_t sV = va::smem_addr(smem + S::oV);
        const uint32_t tS = tmem + 2 * h * kKeys;        // two S buffers of this tile
        const uint32_t tO = tmem + 4 * kKeys + h * D;    // O of this tile
        constexpr uint32_t IDESC_S = idesc_f16(kRows, kKeys, false);
        constexpr uint32_t IDESC_O = idesc_f16(kRows, D, true);
        auto wait_chunk = [&](int c) {
          wait_bar(&bar_full[c % kStages], (uint32_t)((c / kStages) & 1), 3);
        };
        // S_h(j) = Q_h K_j^T: A = Q_h [128 x D] K-major, B = K chunk [64 x D] K-major.
        auto issue_s = [&](int j) {
          if (lane == 0 && !dead()) {
            fence_after_sync();
            const uint32_t kbase = sK + (j % kStages) * S::kKV;
#pragma unroll
            for (int ks = 0; ks < D / 16; ++ks) {
              const uint32_t kblk = ks >> 2, kin = (ks & 3) * 32;
              umma_f16(tS + (j & 1) * kKeys, sdesc(sQ + kblk * kRows * 128 + kin, 16, 1024),
                       sdesc(kbase + kblk * kKeys * 128 + kin, 16, 1024), IDESC_S, ks > 0);
            }
            umma_commit(&bar_s[2 * h + (j & 1)]);
          }
          __syncwarp();
        };
        // O_h (+)= P_h V_j: A = P_h [128 x 64] from TMEM (written by the softmax over the
        // first 32 columns of S_h(j)'s buffer), B = V chunk [64 keys x D] MN-major
        // (LBO = next 64 columns, SBO = next 8 keys).  S_h(j+2), issued later by this
        // thread into the same buffer, executes after this MMA has read P (one
        // thread's tcgen05.mma operations run in issue order).
        auto issue_pv = [&](int j) {
          wait_bar(&bar_p[h], (uint32_t)(j & 1), 4);
          if (lane == 0 && !dead()) {
            fence_after_sync();
            const uint32_t vbase = sV + (j % kStages) * S::kKV;
#pragma unroll
            for (int ks = 0; ks < kKeys / 16; ++ks)
              umma_f16_ts(tO, tmem + (2 * h + (j & 1)) * kKeys + ks * 8,
                          sdesc(vbase + ks * 2048, kKeys * 128, 1024), IDESC_O,
                          (j > 0 || ks > 0) ? 1u : 0u);
            umma_commit(&bar_pv[h]);
          }
          __syncwarp();
        };
        // S runs two chunks ahead of PV: S_h(j+2) reuses the buffer of S_h(j), read
        // before P_h(j) was published.  Every chunk is waited for (and released) by
        // both MMA warps, also past this tile's context, so the stage barriers stay
        // in step.
#pragma unroll 1
        for (int c = 0; c < 2 && c < nch; ++c) {
          wait_chunk(c);
          if (c < nj) issue_s(c);
        }
#pragma unroll 1
        for (int j = 0; j < nch; ++j) {
          if (j < nj) issue_pv(j);
          // stage j is free once PV(j) (and S(j), issued earlier) completes: release it
          // before S(j+2) goes in, so the producer's refill is not held behind it
          if (lane == 0 && !dead()) umma_commit(&bar_empty[j % kStages]);
          __syncwarp();
          if (j + 2 < nch) {
            wait_chunk(j + 2);
            if (j + 2 < nj) issue_s(j + 2);
          }
        }
        // teardown: every MMA issued by this thread has retired
        if (lane == 0) {
          umma_commit(&bar_done[h]);
          if (!va::mbar_wait_bounded(&bar_done[h], 0, kWaitLimit)) timeout(5);
        }
        __syncwarp();
        all_sync();
      } else {
        // =================== softmax of tile h, one thread per row ===================
        const int h = warp >> 2;
        const int row = tid & (kRows - 1);
        const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t tO = tmem + 4 * kKeys + h * D + lane_base;
        const int tk = row / GC;
        const int my_pos = (tk < TQ) ? s_pos[h * kRows + tk] : -1;
        const int nj = min(max((s_ctx[h] + kKeys - 1) / kKeys - cb, 0), nch);
        // m: the max the probabilities are taken against.  It only moves when the row
        // max exceeds it by more than 2^8 (P stays <= 256, exact enough in fp16, and
        // O / l at the end cancels it), so O is rescaled in TMEM rarely.
        float m = -INFINITY, l = 0.f;
#pragma unroll 1
        for (int j = 0; j < nj; ++j) {
          float p[kKeys];
          {
            wait_bar(&bar_s[2 * h + (j & 1)], (uint32_t)((j >> 1) & 1), 6);
            fence_after_sync();
            // both halves of the row's 64 scores in flight, then one wait
            uint32_t sr[32], sr2[32];
            const uint32_t tS = tmem + (2 * h + (j & 1)) * kKeys + lane_base;
            tmem_ld32(tS, sr);
            tmem_ld32(tS + 32, sr2);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) {
              p[c] = __uint_as_float(sr[c]);
              p[32 + c] = __uint_as_float(sr2[c]);
            }
          }
          float alpha;
          {
            // raw scores: the scale (> 0) is applied in the exponent's FMA
            const int vis = my_pos - (cb + j) * kKeys;  // keys 0..vis of this chunk are visible
            if (vis < kKeys - 1) {
#pragma unroll
              for (int c = 0; c < kKeys; ++c) p[c] = c <= vis ? p[c] : -INFINITY;
            }
            float mx4[4] = {p[0], p[1], p[2], p[3]};
#pragma unroll
            for (int c = 4; c < kKeys; c += 8) {
              mx4[0] = fmax3(mx4[0], p[c + 0], p[c + 1]);
              mx4[1] = fmax3(mx4[1], p[c + 2], p[c + 3]);
              mx4[2] = fmax3(mx4[2], p[c + 4], p[c + 5]);
              if (c + 7 < kKeys) mx4[3] = fmax3(mx4[3], p[c + 6], p[c + 7]);
              else mx4[3] = fmaxf(mx4[3], p[c + 6]);
            }
            const float rmax = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * a.scale_log2;
            const float mn = (m == -INFINITY || rmax > m + 8.f) ? fmaxf(m, rmax) : m;
            const bool none = mn == -INFINITY;
            alpha = (none || mn == m) ? 1.f : va::fast_exp2(m - mn);
            const float nmn = none ? 0.f : -mn;
            // p = 2^(s * scale - m) in pairs: the exponent argument by a packed FMA, the
            // power by the special-function unit (measured on B200: evaluating a third
            // of them by a polynomial on the FMA pipe instead cost 1.5 %: the softmax
            // is bound by issue and latency, not by that unit)
            const uint64_t sc2 = pk2(a.scale_log2, a.scale_log2), nm2 = pk2(nmn, nmn);
            uint64_t sum2[2] = {pk2(0.f, 0.f), pk2(0.f, 0.f)};
#pragma unroll
            for (int c = 0; c < kKeys / 2; ++c) {
              const uint64_t x = ffma2(pk2(p[2 * c], p[2 * c + 1]), sc2, nm2);
              float x0, x1;
              upk2(x, x0, x1);
              const uint64_t e = pk2(va::fast_exp2(x0), va::fast_exp2(x1));
              upk2(e, p[2 * c], p[2 * c + 1]);
              sum2[c & 1] = fadd2(sum2[c & 1], e);
            }
            float s0, s1, s2, s3;
            upk2(sum2[0], s0, s1);
            upk2(sum2[1], s2, s3);
            l = l * alpha + ((s0 + s1) + (s2 + s3));
            m = mn;
          }
          // rescale this row of O where the max moved (warp-collective TMEM access),
          // once PV_h(j-1) is done with O.  P_h(j) goes to S_h(j)'s own buffer, which
          // no pending MMA reads, so without a rescale there is nothing to wait for.
          if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
            wait_bar(&bar_pv[h], (uint32_t)((j - 1) & 1), 7);
            fence_after_sync();
#pragma unroll 1
            for (int c = 0; c < D; c += 32) {
              uint32_t o[32];
              tmem_ld32(tO + c, o);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
              tmem_st32(tO + c, o);
            }
            tmem_wait_st();
          }
          // P row (fp16 pairs) into the first 32 columns of S_h(j)'s TMEM buffer (already
          // read above), then publish it to the MMA warp
          {
            uint32_t pw[32];
#pragma unroll
            for (int c = 0; c < 32; ++c) pw[c] = va::pack_h2(p[2 * c], p[2 * c + 1]);
            tmem_st32(tmem + (2 * h + (j & 1)) * kKeys + lane_base, pw);
            tmem_wait_st();
          }
          fence_before_sync();
          va::mbar_arrive(&bar_p[h]);
        }
        if (nj > 0) {
          wait_bar(&bar_pv[h], (uint32_t)((nj - 1) & 1), 8);
          fence_after_sync();
        }
        // ---- epilogue: O / l -> fp16 rows, once every role is done ----
        all_sync();  // s_bad_from / s_dead are final
        const bool ok = !dead();  // uniform across the CTA after the barrier
        const int bad_from = s_bad_from;
        if (bad_from != INT_MAX && tid == 0) va::raise_flag(a.err, VA_FLAG_BAD_BLOCK);
        const int ti = h * TQ + tk;
        const bool row_ok = my_pos >= 0 && tk < TQ && ti < nq && row < TQ * GC;
        const int g = row - tk * GC;
        __half *orow = a.out + (int64_t)(t0 + ti) * a.o_s_token + (int64_t)(head0 + g) * a.o_s_head;
        auto store32 = [&](int c, const float (&v)[32], float inv) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 w;
            w.x = va::pack_h2(v[i + 0] * inv, v[i + 1] * inv);
            w.y = va::pack_h2(v[i + 2] * inv, v[i + 3] * inv);
            w.z = va::pack_h2(v[i + 4] * inv, v[i + 5] * inv);
            w.w = va::pack_h2(v[i + 6] * inv, v[i + 7] * inv);
            *reinterpret_cast<uint4 *>(orow + c + i) = w;
          }
        };
        if (nparts == 1) {
          const bool write = ok && nj > 0 && row_ok && my_pos < bad_from;
          const float inv = l > 0.f ? 1.f / l : 0.f;
          if (ok && nj > 0) {
#pragma unroll 1
            for (int c = 0; c < D; c += 32) {
              uint32_t o[32];
              tmem_ld32(tO + c, o);
              tmem_wait_ld();
              if (write) {
                float v[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(o[i]);
                store32(c, v, inv);
              }
            }
          }
        } else {
          // A key-range part: publish (O, m, l) of every row, take a ticket; the
          // part that finishes last merges all parts in part order and writes
          // the rows (no CTA waits for another).
          const int slot0 = unit.w + yb * nparts;
          const size_t sp = (size_t)(slot0 + kpart) * kTiles + h;
          float *po = a.part_o + sp * D * kRows + row;  // column-major: coalesced per d
          const bool have = ok && nj > 0;
          if (have) {
#pragma unroll 1
            for (int c = 0; c < D; c += 32) {
              uint32_t o[32];
              tmem_ld32(tO + c, o);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i) __stcg(po + (size_t)(c + i) * kRows, __uint_as_float(o[i]));
            }
          }
          __stcg(a.part_ml + sp * kRows + row, have ? make_float2(m, l) : make_float2(-INFINITY, 0.f));
          if (tid == 0) __stcg(a.part_bad + slot0 + kpart, bad_from);
          __threadfence();
          softmax_sync();
          if (tid == 0) s_last = atomicAdd(a.tickets + tile * ny + yb, 1) == nparts - 1;
          softmax_sync();
          if (s_last) {
            __threadfence();
            int bad = INT_MAX;
            float M = -INFINITY;
            for (int p = 0; p < nparts; ++p) {
              bad = min(bad, __ldcg(a.part_bad + slot0 + p));
              M = fmaxf(M, __ldcg(a.part_ml + ((size_t)(slot0 + p) * kTiles + h) * kRows + row).x);
            }
            const bool write = ok && row_ok && my_pos < bad && M != -INFINITY;
            float L = 0.f;
            for (int p = 0; p < nparts; ++p) {
              const float2 v = __ldcg(a.part_ml + ((size_t)(slot0 + p) * kTiles + h) * kRows + row);
              if (v.x != -INFINITY) L = fmaf(v.y, va::fast_exp2(v.x - M), L);
            }
            const float inv = L > 0.f ? 1.f / L : 0.f;
            if (write) {
#pragma unroll 1
              for (int c = 0; c < D; c += 32) {
                float acc[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) acc[i] = 0.f;
                for (int p = 0; p < nparts; ++p) {
                  const size_t q = (size_t)(slot0 + p) * kTiles + h;
                  const float mp = __ldcg(a.part_ml + q * kRows + row).x;
                  if (mp == -INFINITY) continue;
                  const float e = va::fast_exp2(mp - M);
                  const float *src = a.part_o + q * D * kRows + row + (size_t)c * kRows;
#pragma unroll
                  for (int i = 0; i < 32; ++i) acc[i] = fmaf(__ldcg(src + (size_t)i * kRows), e, acc[i]);
                }
                store32(c, acc, inv);
              }
            }
          }
        }
      }
    }
    // all roles meet here before the next item re-initialises the barriers
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
  }
  // the first MMA warp releases TMEM
  fence_before_sync();
  __syncthreads();
  if (warp == kMmaWarp) {
    fence_after_sync();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace tc
