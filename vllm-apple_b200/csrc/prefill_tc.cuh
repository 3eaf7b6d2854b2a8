// Token-parallel causal paged attention on the 5th-generation tensor cores
// (tcgen05 UMMA, TMEM accumulators), head_size 64 or 128.  Included by
// paged_prefill.cu, which owns the tile planner and the C-ABI entry point.
//
// One CTA (4 warps, 128 threads) per (tile, kv head [, q-head group]):
//   * 128 MMA rows = (token, q head) pairs of up to 128/G consecutive tokens of
//     one sequence, so each staged K/V chunk serves every head of the group;
//     thread t owns row t (TMEM lane t) for the whole softmax.
//   * Q, K and V tiles live in shared memory in the 128-byte-swizzled
//     canonical layout (8-row x 128-byte atoms).  K and V chunks of 64 keys
//     arrive by TMA (cp.async.bulk.tensor.3d, one box per page and 64 head
//     dims, hardware 128-byte swizzle, no multicast), issued by one thread and
//     completed on a per-stage mbarrier, kStages deep (chunk j+3 is requested
//     as soon as chunk j-1 retires).  Invalid pages and pages past the context
//     are zero-filled by the threads; V rows past the context in the last page
//     are zeroed after their page lands.  Q is staged once by cp.async.
//   * S = Q K^T (M=128, N=64, K=D) goes to one of two TMEM buffers, so the MMA
//     of chunk j+1 runs while the rows of chunk j are in softmax; O (M=128,
//     N=D) accumulates in TMEM: rows whose running max grew are rescaled in
//     TMEM before the next PV MMA.  P (fp16) is written to shared memory in
//     the same swizzled layout and consumed by O += P V (V as an MN-major
//     operand: the same shared-memory image as K).
//   * Warp roles: one producer warp runs ahead of the math, fetching block ids
//     and issuing the TMA boxes of chunk c into stage c % kStages as soon as
//     the tensor core has finished with that stage (a tcgen05.commit after the
//     chunk's PV MMA arrives on the stage's "empty" barrier); eight softmax
//     warps own the rows, and one of their threads issues every MMA.  Every
//     wait on an mbarrier is bounded and reports VA_FLAG_WAIT_TIMEOUT.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace tc {

constexpr int kRows = 128;  // MMA M
constexpr int kKeys = 64;   // keys per chunk (MMA N of S, MMA K of PV)
constexpr int kConsumers = 256;          // 8 softmax warps: two threads per MMA row
constexpr int kThreads = kConsumers + 32;  // + 1 producer warp (TMA)
constexpr uint32_t kTmemCols = 256;  // S x2 (2 x 64) + O (<= 128)
constexpr uint32_t kWaitLimit = 1u << 22;
constexpr int kStages = 4;  // K/V chunks in flight (a chunk = 64 keys of K and of V)

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
  const int32_t *tiles_n;
  int32_t *err;
  int64_t num_seqs, max_blocks, num_blocks;
  int Hq, Hkv, G, hgroups, TQ, bs, skip_singles;
  int nhd;  // cache layout of the tensor maps: 0 = [nb, H, bs, D], 1 = [nb, bs, H, D]
  float scale_log2;
  int64_t s_block, s_head, s_token, q_s_token, q_s_head, o_s_token, o_s_head;
};

template <int D>
struct Smem {
  static constexpr uint32_t kQ = kRows * D * 2;    // 16/32 KB
  static constexpr uint32_t kKV = kKeys * D * 2;   // 8/16 KB per chunk
  static constexpr uint32_t kP = kRows * kKeys * 2;  // 16 KB
  static constexpr uint32_t oQ = 0, oK = kQ, oV = oK + kStages * kKV, oP = oV + kStages * kKV;
  static constexpr uint32_t oBar = oP + kP;  // S, PV, full[kStages], empty[kStages] + tmem slot
  // + slack to align the base to 1 KB; D=64 is padded so at most 2 CTAs share
  // an SM (2 x 256 TMEM columns = the whole TMEM)
  static constexpr uint32_t kNeed = oBar + 128 + 1024;
  static constexpr uint32_t kBytes = (D == 64 && kNeed < 80u * 1024) ? 80u * 1024 : kNeed;
};

// Named barrier over the 8 softmax warps only (the producer warp runs free).
VA_DEVINL void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory");
}

template <int D, int GC>
__global__ void __launch_bounds__(kThreads)
    paged_prefill_tc_kernel(const Args a, const __grid_constant__ CUtensorMap tmk,
                            const __grid_constant__ CUtensorMap tmv) {
  using S = Smem<D>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  // 128-byte swizzle atoms must sit on 1024-byte boundaries of the shared window
  unsigned char *smem = smem_raw + ((1024u - (va::smem_addr(smem_raw) & 1023u)) & 1023u);
  uint64_t *bar_s = reinterpret_cast<uint64_t *>(smem + S::oBar);
  uint64_t *bar_pv = bar_s + 1;
  uint64_t *bar_full = bar_s + 2;              // [kStages]: chunk landed
  uint64_t *bar_empty = bar_full + kStages;    // [kStages]: tensor core done with the stage
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bar_empty + kStages);
  __shared__ int s_pos[kRows];
  __shared__ float s_red[2][kRows];  // per-half row max (per chunk) / row sum (at the end)
  __shared__ int s_ctx, s_bad_from, s_dead;

  const int tile = blockIdx.x;
  if (tile >= *a.tiles_n) return;
  const int2 td = a.tiles[tile];
  const int t0 = td.x, nq = td.y;
  if (nq == 1 && a.skip_singles) return;  // handled by the split-KV decode kernel
  const int seq = a.tok_seq[t0];
  const int kvh = blockIdx.y / a.hgroups;
  const int hg = blockIdx.y - kvh * a.hgroups;
  const int head0 = kvh * a.G + hg * GC;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int BS = a.bs;

  if (tid == 0) { s_ctx = 0; s_bad_from = INT_MAX; s_dead = 0; }
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
  const int nch = (ctx + kKeys - 1) / kKeys;
  const int32_t *bt_row = a.bt + (int64_t)seq * a.max_blocks;

  // ---- barriers + TMEM ----
  if (tid == 0) {
    va::mbar_init(bar_s, 1);
    va::mbar_init(bar_pv, 1);
    for (int i = 0; i < kStages; ++i) {
      va::mbar_init(&bar_full[i], 1);
      va::mbar_init(&bar_empty[i], 1);
    }
    va::fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, kTmemCols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  constexpr int CPR = D / 8;
  // Q: every thread, 16-byte cp.async into the swizzled layout (once)
  for (int i = tid; i < kRows * CPR; i += kThreads) {
    const int r = i / CPR, c = i - r * CPR;
    const int tk = r / GC, g = r - tk * GC;
    unsigned char *dst = smem + S::oQ + sw128_off(r, c * 8, kRows);
    if (tk < nq && tk < a.TQ)
      cp_async16(dst, a.q + (int64_t)(t0 + tk) * a.q_s_token + (int64_t)(head0 + g) * a.q_s_head +
                          c * 8);
    else
      *reinterpret_cast<uint4 *>(dst) = make_uint4(0, 0, 0, 0);
  }
  cp_async_commit();

  auto dead = [&]() { return *(volatile int *)&s_dead != 0; };
  auto timeout = [&]() {
    if (atomicExch(&s_dead, 1) == 0) va::raise_flag(a.err, VA_FLAG_WAIT_TIMEOUT);
  };
  auto wait_bar = [&](uint64_t *bar, uint32_t parity) {
    if (dead()) return;
    if (!va::mbar_wait_bounded(bar, parity, kWaitLimit)) timeout();
  };

  if (warp == kConsumers / 32) {
    // =================== producer warp: TMA staging of K/V chunks ===================
    const int npc = kKeys / BS;  // a power of two <= 8: a chunk never straddles a group
    const int pages = (ctx + BS - 1) / BS;  // <= max_blocks (checked above)
    // block ids are read 32 pages (one per lane) at a time, one group ahead
    auto load_group = [&](int g) -> int32_t {
      const int page = g * 32 + lane;
      return page < pages ? __ldg(bt_row + page) : -1;
    };
    int gi = 0;
    int32_t g_cur = load_group(0), g_next = load_group(1);
#pragma unroll 1
    for (int c = 0; c < nch; ++c) {
      const int buf = c % kStages;
      const int first = c * npc;
      if ((first >> 5) != gi) {
        gi = first >> 5;
        g_cur = g_next;
        g_next = load_group(gi + 1);
      }
      const int32_t gid = __shfl_sync(0xffffffffu, g_cur, (first & 31) + (lane & (npc - 1)));
      if (c >= kStages) wait_bar(&bar_empty[buf], (uint32_t)(((c / kStages) - 1) & 1));
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
      // zero the stage rows of pages that will not be loaded (past context / invalid)
      unsigned char *kb = smem + S::oK + buf * S::kKV, *vb = smem + S::oV + buf * S::kKV;
      const unsigned valid = __ballot_sync(0xffffffffu, lane < npc && id >= 0);
      if (valid != (1u << npc) - 1u) {  // a hole: only near the end of the context
        for (int i = lane; i < kKeys * CPR; i += 32) {
          const int r = i / CPR, ch16 = i - r * CPR;
          if (!((valid >> (r / BS)) & 1u)) {
            const uint32_t o = sw128_off(r, ch16 * 8, kKeys);
            *reinterpret_cast<uint4 *>(kb + o) = make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4 *>(vb + o) = make_uint4(0, 0, 0, 0);
          }
        }
        va::fence_proxy_async_smem();
        __syncwarp();
      }
      if (lane == 0) va::mbar_arrive_expect_tx(&bar_full[buf], __popc(valid) * (2u * BS * D * 2u));
      __syncwarp();
      // one box per lane: lane = (page, 64-column block, K or V)
      {
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
    // no copy may still be landing when the CTA exits (normally all have: the
    // softmax warps consumed every chunk); bounded, reports like any other wait
    if (lane == 0) {
      for (int c = nch - kStages < 0 ? 0 : nch - kStages; c < nch; ++c)
        if (!va::mbar_wait_bounded(&bar_full[c % kStages], (uint32_t)((c / kStages) & 1), kWaitLimit))
          timeout();
    }
    __syncwarp();
  } else {
    // =================== softmax warps (+ MMA issue by thread 0) ===================
    const int row = tid & (kRows - 1);
    const int half = tid >> 7;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t tO = tmem + 2 * kKeys;
    const uint32_t sQ = va::smem_addr(smem + S::oQ);
    const uint32_t sK = va::smem_addr(smem + S::oK);
    const uint32_t sV = va::smem_addr(smem + S::oV);
    const uint32_t sP = va::smem_addr(smem + S::oP);
    constexpr uint32_t IDESC_S = idesc_f16(kRows, kKeys, false);
    constexpr uint32_t IDESC_O = idesc_f16(kRows, D, true);

    // S_j = Q K_j^T: A = Q [128 x D] K-major, B = K chunk [64 x D] K-major.
    auto issue_s = [&](int j) {
      if (tid == 0 && !dead()) {
        fence_after_sync();
        const uint32_t kbase = sK + (j % kStages) * S::kKV;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t kblk = ks >> 2, kin = (ks & 3) * 32;
          umma_f16(tmem + (j & 1) * kKeys, sdesc(sQ + kblk * kRows * 128 + kin, 16, 1024),
                   sdesc(kbase + kblk * kKeys * 128 + kin, 16, 1024), IDESC_S, ks > 0);
        }
        umma_commit(bar_s);
      }
    };
    // O (+)= P_j V_j: A = P [128 x 64] K-major, B = V chunk [64 keys x D] MN-major (the
    // same swizzled image as a K tile: LBO = next 64 columns, SBO = next 8 keys); then the
    // stage is released to the producer once both MMAs of chunk j are done.
    auto issue_pv = [&](int j) {
      if (tid == 0 && !dead()) {
        fence_after_sync();
        const uint32_t vbase = sV + (j % kStages) * S::kKV;
#pragma unroll
        for (int ks = 0; ks < kKeys / 16; ++ks)
          umma_f16(tO, sdesc(sP + ks * 32, 16, 1024), sdesc(vbase + ks * 2048, kKeys * 128, 1024),
                   IDESC_O, (j > 0 || ks > 0) ? 1u : 0u);
        umma_commit(bar_pv);
        umma_commit(&bar_empty[j % kStages]);
      }
    };
    // chunk ch landed; V rows past the context inside the last page are zeroed
    // (p = 0 there, but 0 * garbage could be NaN)
    auto wait_chunk = [&](int ch) {
      const int buf = ch % kStages;
      wait_bar(&bar_full[buf], (uint32_t)((ch / kStages) & 1));
      if (ch == nch - 1 && ctx % kKeys != 0) {
        for (int i = tid; i < kKeys * CPR; i += kConsumers) {
          const int r = i / CPR, c = i - r * CPR;
          if (ch * kKeys + r >= ctx)
            *reinterpret_cast<uint4 *>(smem + S::oV + buf * S::kKV + sw128_off(r, c * 8, kKeys)) =
                make_uint4(0, 0, 0, 0);
        }
      }
    };

    cp_async_wait<0>();
    wait_chunk(0);
    va::fence_proxy_async_smem();
    consumer_sync();
    issue_s(0);

    const int tk = row / GC;
    const int my_pos = (tk < a.TQ) ? s_pos[tk] : -1;
    // m: the max the probabilities are taken against.  It only moves when the row
    // max exceeds it by more than 2^8 (P stays <= 256, exact enough in fp16, and
    // O / l at the end cancels it), so O is rescaled in TMEM rarely.
    float m = -INFINITY, l = 0.f;  // l: this thread's half of the row sum

#pragma unroll 1
    for (int j = 0; j < nch; ++j) {
      // (1) this thread's 32 scores of chunk j, masked, and their max
      wait_bar(bar_s, (uint32_t)(j & 1));
      fence_after_sync();
      uint32_t sr[32];
      tmem_ld32(tmem + (j & 1) * kKeys + half * 32 + lane_base, sr);
      tmem_wait_ld();
      fence_before_sync();
      float p[32];
      const int kbase = j * kKeys + half * 32;
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const float s = __uint_as_float(sr[c]) * a.scale_log2;
        p[c] = (kbase + c <= my_pos) ? s : -INFINITY;
        mx4[c & 3] = fmaxf(mx4[c & 3], p[c]);
      }
      s_red[half][row] = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      // (2) chunk j+1 landed -> (3) S_{j+1} on the tensor core
      if (j + 1 < nch) wait_chunk(j + 1);
      va::fence_proxy_async_smem();
      consumer_sync();
      if (j + 1 < nch) issue_s(j + 1);
      // (4) online softmax against the (lazily moved) max of both halves of the row
      const float rmax = fmaxf(s_red[0][row], s_red[1][row]);
      const float mn = (m == -INFINITY || rmax > m + 8.f) ? fmaxf(m, rmax) : m;
      const bool none = mn == -INFINITY;
      const float alpha = (none || mn == m) ? 1.f : va::fast_exp2(m - mn);
      float sum4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        p[c] = none ? 0.f : va::fast_exp2(p[c] - mn);
        sum4[c & 3] += p[c];
      }
      l = l * alpha + ((sum4[0] + sum4[1]) + (sum4[2] + sum4[3]));
      m = mn;
      // (5) PV_{j-1} done: P buffer and O are free
      if (j > 0) {
        wait_bar(bar_pv, (uint32_t)((j - 1) & 1));
        fence_after_sync();
      }
      // (6) rescale this thread's half of O where the max moved (warp-collective)
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
        for (int c = half * (D / 2); c < (half + 1) * (D / 2); c += 32) {
          uint32_t o[32];
          tmem_ld32(tO + lane_base + c, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(tO + lane_base + c, o);
        }
        tmem_wait_st();
      }
      // (7) this thread's 32 probabilities -> P (fp16, swizzled)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint4 w;
        w.x = va::pack_h2(p[8 * c + 0], p[8 * c + 1]);
        w.y = va::pack_h2(p[8 * c + 2], p[8 * c + 3]);
        w.z = va::pack_h2(p[8 * c + 4], p[8 * c + 5]);
        w.w = va::pack_h2(p[8 * c + 6], p[8 * c + 7]);
        *reinterpret_cast<uint4 *>(smem + S::oP + sw128_off(row, half * 32 + c * 8, kRows)) = w;
      }
      va::fence_proxy_async_smem();
      fence_before_sync();
      consumer_sync();
      issue_pv(j);
    }

    // ---- epilogue: O / l -> fp16 rows ----
    wait_bar(bar_pv, (uint32_t)((nch - 1) & 1));
    s_red[half][row] = l;
    consumer_sync();
    const bool ok = !dead();  // uniform across the softmax warps after the barrier
    const float lt = s_red[0][row] + s_red[1][row];
    const int bad_from = s_bad_from;
    if (bad_from != INT_MAX && tid == 0) va::raise_flag(a.err, VA_FLAG_BAD_BLOCK);
    const bool write = ok && my_pos >= 0 && my_pos < bad_from && tk < nq && row < a.TQ * GC;
    const float inv = lt > 0.f ? 1.f / lt : 0.f;
    const int g = row - tk * GC;
    __half *orow = a.out + (int64_t)(t0 + tk) * a.o_s_token + (int64_t)(head0 + g) * a.o_s_head;
    if (ok) {
      fence_after_sync();
#pragma unroll 1
      for (int c = half * (D / 2); c < (half + 1) * (D / 2); c += 32) {
        uint32_t o[32];
        tmem_ld32(tO + lane_base + c, o);
        tmem_wait_ld();
        if (write) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 w;
            w.x = va::pack_h2(__uint_as_float(o[i + 0]) * inv, __uint_as_float(o[i + 1]) * inv);
            w.y = va::pack_h2(__uint_as_float(o[i + 2]) * inv, __uint_as_float(o[i + 3]) * inv);
            w.z = va::pack_h2(__uint_as_float(o[i + 4]) * inv, __uint_as_float(o[i + 5]) * inv);
            w.w = va::pack_h2(__uint_as_float(o[i + 6]) * inv, __uint_as_float(o[i + 7]) * inv);
            *reinterpret_cast<uint4 *>(orow + c + i) = w;
          }
        }
      }
    }
  }
  // producer and softmax warps meet here; warp 0 releases TMEM
  fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    fence_after_sync();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace tc
