// Single-token decode paged attention with the fused KV-cache write (sm_100a).
//
// Design (HBM-bound, CUDA cores only):
//   * one CTA per (split of a sequence's pages, kv head [, q-head group], seq);
//     every q head of the GQA group is served from ONE read of each K/V page.
//   * each of the CTA's NW warps owns every NW-th page of the split and runs
//     its own STAGES-deep pipeline: lane 0 arms an mbarrier and the page's K
//     and V tiles arrive in shared memory by 1-D bulk copies (TMA engine, no
//     multicast); the copy for page k+STAGES is issued once page k is consumed.
//   * QK^T: TPT lanes share one token, each holding DPL dims of every q head in
//     registers as packed fp16; products use the sm_100 mixed-precision FMA
//     (fp16 x fp16 + fp32); partial dot products are reduce-scattered across
//     the TPT lanes so each lane ends with whole scores of distinct heads.
//   * online softmax per page in the log2 domain, probabilities staged in a
//     per-warp shared buffer; PV accumulates fp32 with each lane owning D/32
//     output dims of every head.
//   * warps merge through shared memory; a sequence with several splits
//     writes fp32 partials (m, l, acc) to the workspace and a small combine
//     kernel (launched only when some sequence can have several splits) merges
//     them in split order -- deterministic, and the workspace needs no
//     initialisation.
//   * fused KV write: the CTA whose split holds position seq_len-1 patches the
//     new K/V row into its staged page and (first q-head group only) stores it
//     to the cache; no other CTA reads that slot.
#include <math.h>

#include <atomic>
#include <mutex>

#include "common.cuh"

namespace {

// Tuning knobs (defaults are the measured best on B200).
#ifndef VA_DECODE_STAGES
#define VA_DECODE_STAGES 2
#endif
#ifndef VA_DECODE_DPL128
#define VA_DECODE_DPL128 32
#endif

constexpr int kNW = 4;                     // warps per CTA
constexpr int kStages = VA_DECODE_STAGES;  // pages in flight per warp
constexpr uint32_t kWaitLimit = 1u << 22;  // bounded mbarrier polls

struct DecodeArgs {
  __half *out;
  const __half *q;
  __half *kc, *vc;
  const int32_t *bt, *seq_lens;
  const __half *nk, *nv;
  float *ws_acc, *ws_ml;
  int32_t *err;
  const int32_t *order;  // grid row z -> sequence, longest first (null: z itself)
  int64_t max_blocks, num_blocks;
  int Hq, Hkv, G, hgroups, pps, max_splits;
  float scale_log2;
  int64_t s_block, s_head, s_token, q_s_token, q_s_head, o_s_token, o_s_head, n_s_token,
      n_s_head;
  // Row mode (one-token rows of a prefill batch): grid row r is token rows[r];
  // its sequence is row_tok_seq[t] and its context positions 0..row_pos[t].
  const int32_t *rows, *rows_n, *row_tok_seq, *row_pos;
  int64_t row_num_seqs;
};

// Block-table row, context length and q/out row of grid row r; false = skip.
VA_DEVINL bool decode_row(const DecodeArgs &a, int r, int bs, int &bt_seq, int &L_in,
                          int64_t &qo) {
  if (a.rows == nullptr) {
    bt_seq = r;
    L_in = a.seq_lens[r];
    qo = r;
    return L_in > 0;
  }
  if (r >= *a.rows_n) return false;
  const int t = a.rows[r];
  const int s = a.row_tok_seq[t];
  const int p = a.row_pos[t];
  if (s < 0 || s >= a.row_num_seqs || p < 0) return false;
  if ((int64_t)((p + bs) / bs) > a.max_blocks) {  // prefill rule: such a token is skipped
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0)
      va::raise_flag(a.err, VA_FLAG_CTX_OVERFLOW);
    return false;
  }
  bt_seq = s;
  L_in = p + 1;
  qo = t;
  return true;
}

constexpr int pow2ceil(int x) { return x <= 1 ? 1 : 2 * pow2ceil((x + 1) / 2); }

// a[0..1] *= s as one packed f32x2 multiply (each lane rounded like a fp32 multiply).
VA_DEVINL void fmul2_bcast(float &a0, float &a1, float sc) {
  uint64_t acc, ss;
  asm("mov.b64 %0, {%1, %2};" : "=l"(acc) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %1};" : "=l"(ss) : "f"(sc));
  asm("mul.rn.f32x2 %0, %0, %1;" : "+l"(acc) : "l"(ss));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a0), "=f"(a1) : "l"(acc));
}

// acc[0..1] = fma(p, v[0..1], acc[0..1]) as one packed sm_100 f32x2 FMA (each lane
// rounded exactly like fmaf).
VA_DEVINL void ffma2_bcast(float &a0, float &a1, float p, float v0, float v1) {
  uint64_t acc, vv, pp;
  asm("mov.b64 %0, {%1, %2};" : "=l"(acc) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(vv) : "f"(v0), "f"(v1));
  asm("mov.b64 %0, {%1, %1};" : "=l"(pp) : "f"(p));
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(pp), "l"(vv));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a0), "=f"(a1) : "l"(acc));
}

template <int D>
struct Shape {
  static constexpr int DPL = (D == 96) ? 24 : (D == 128 ? VA_DECODE_DPL128 : 16);  // dims per lane in QK^T
  static constexpr int TPT = D / DPL;              // lanes sharing a token
  static constexpr int TOK = 32 / TPT;             // tokens per pass
  static constexpr int DV = (D == 96) ? 3 : D / 32;  // output dims per lane in PV
};

// Output dim owned by `lane` as its j-th PV dim.
template <int D>
VA_DEVINL int pv_dim(int lane, int j) {
  if constexpr (D == 96) return j < 2 ? 2 * lane + j : 64 + lane;
  else return lane * (D / 32) + j;
}

template <int D>
VA_DEVINL void load_v(const __half *row, int lane, float (&v)[Shape<D>::DV]) {
  if constexpr (D == 128) {
    const uint2 r = *reinterpret_cast<const uint2 *>(row + 4 * lane);
    const float2 a = va::h2_to_f2(r.x), b = va::h2_to_f2(r.y);
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
  } else if constexpr (D == 64) {
    const float2 a = va::h2_to_f2(*reinterpret_cast<const uint32_t *>(row + 2 * lane));
    v[0] = a.x; v[1] = a.y;
  } else if constexpr (D == 96) {
    const float2 a = va::h2_to_f2(*reinterpret_cast<const uint32_t *>(row + 2 * lane));
    v[0] = a.x; v[1] = a.y;
    v[2] = __half2float(row[64 + lane]);
  } else {
    v[0] = __half2float(row[lane]);
  }
}

// Per-lane rotation of the order in which a lane walks its 16-byte chunks of a
// K row (and, identically, of its q registers) so that the 8 lanes of each
// shared-memory wavefront hit 8 distinct 16-byte bank groups.
template <int D>
VA_DEVINL int chunk_rot(int lane) {
  constexpr int DPL = Shape<D>::DPL, TPT = Shape<D>::TPT;
  const int cq = lane % TPT, tq = lane / TPT;
  if constexpr (D == 96) return 0;                      // 12 chunks/row: already distinct
  else if constexpr (DPL == 32) return ((cq >> 1) + 2 * (tq & 1)) & 3;  // D=128, 4 lanes/token
  else if constexpr (TPT == 8) return (cq >> 2) & 1;    // D=128, 8 lanes/token
  else if constexpr (TPT == 4) return tq & 1;           // D=64
  else return (tq >> 1) & 1;                            // D=32
}

// Reduce-scatter N partial sums across the lanes that differ in bits
// MASK, MASK/2, ..., 1; afterwards lane keeps max(N/ (2*MASK), 1) full sums.
template <int N, int MASK>
VA_DEVINL void reduce_scatter(float *v, int lane) {
  if constexpr (MASK >= 1) {
    if constexpr (N >= 2) {
      const bool up = (lane & MASK) != 0;
#pragma unroll
      for (int i = 0; i < N / 2; ++i) {
        const float send = up ? v[i] : v[i + N / 2];
        const float keep = up ? v[i + N / 2] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, MASK);
      }
      reduce_scatter<N / 2, MASK / 2>(v, lane);
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], MASK);
      reduce_scatter<1, MASK / 2>(v, lane);
    }
  }
}

// Index of the first head a lane holds after reduce_scatter<N, MASK>.
template <int N, int MASK>
VA_DEVINL int rs_head_base(int lane) {
  if constexpr (MASK >= 1 && N >= 2)
    return ((lane & MASK) ? N / 2 : 0) + rs_head_base<N / 2, MASK / 2>(lane);
  else
    return 0;
}

template <int D, int GC, int BS>
struct Cfg {
  using S = Shape<D>;
  static constexpr int GP = pow2ceil(GC);
  static constexpr int TPT = S::TPT, TOK = S::TOK, DPL = S::DPL, DV = S::DV;
  static constexpr int NPASS = BS / TOK;
  static constexpr int R = GP >= TPT ? GP / TPT : 1;
  static constexpr int PAGE = BS * D;  // halves in one K (or V) page tile
  static constexpr size_t kStageBytes = size_t(kNW) * kStages * 2 * PAGE * 2;
  static constexpr size_t kBarBytes = size_t(kNW) * kStages * 8;
  static constexpr size_t kPBytes = size_t(kNW) * BS * GP * 4;
  static constexpr size_t kABytes = size_t(kNW) * GP * 4;
  static constexpr size_t kSmem = kStageBytes + kBarBytes + kPBytes + kABytes;
  static_assert(BS % TOK == 0, "block size must be a multiple of tokens per pass");
  static_assert(size_t(kNW) * GC * D * 4 + 2 * size_t(kNW) * GP * 4 <= kStageBytes,
                "merge buffers must fit in the stage area");
};

// Small heads with a large GQA group (D <= 64, GC >= 5: the Qwen shape) do ~3x the
// arithmetic per KV byte of the 22B shape; their register demand (q of every head
// in registers) would cap them at 3 CTAs per SM, so they are held to 4.
template <int D, int GC>
constexpr int decode_min_blocks() { return (D <= 64 && GC >= 5) ? 4 : 1; }

template <int D, int GC, int BS>
__global__ void __launch_bounds__(kNW * 32, decode_min_blocks<D, GC>())
    paged_decode_kernel(const DecodeArgs a) {
  using C = Cfg<D, GC, BS>;
  constexpr int GP = C::GP, TPT = C::TPT, TOK = C::TOK, DPL = C::DPL, DV = C::DV;
  constexpr int NPASS = C::NPASS, R = C::R, PAGE = C::PAGE;
  extern __shared__ __align__(128) unsigned char smem[];
  __half *stage = reinterpret_cast<__half *>(smem);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kStageBytes);
  float *pbuf = reinterpret_cast<float *>(smem + C::kStageBytes + C::kBarBytes);
  float *abuf = pbuf + kNW * BS * GP;

  // the combine kernel (launched with programmatic dependency) may be scheduled now;
  // it waits for this grid's completion before reading any partial
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // with an order, this grid is a programmatic dependent of the ordering kernel:
  // wait until that grid has completed and its order is visible
  if (a.order) asm volatile("griddepcontrol.wait;" ::: "memory");
  // index of the partials; the sequence outside row mode, taken longest first when
  // an order is given (long CTAs first: the grid's tail is made of short ones)
  const int seq = a.order ? a.order[blockIdx.z] : (int)blockIdx.z;
  int bt_seq, L_in;
  int64_t qo;
  if (!decode_row(a, seq, BS, bt_seq, L_in, qo)) return;
  int64_t L = L_in;
  int64_t npages = (L + BS - 1) / BS;
  bool clamped = false;
  if (npages > a.max_blocks) {
    npages = a.max_blocks;
    clamped = true;
  }
  int64_t nsplit = (npages + a.pps - 1) / a.pps;
  if (nsplit > (int64_t)gridDim.x) {
    nsplit = gridDim.x;
    npages = nsplit * a.pps;
    clamped = true;
  }
  if (clamped) {
    L = npages * BS < L ? npages * BS : L;
    if (blockIdx.x == 0 && threadIdx.x == 0) va::raise_flag(a.err, VA_FLAG_CTX_OVERFLOW);
  }
  const int split = blockIdx.x;
  if (split >= nsplit) return;

  const int kvh = blockIdx.y / a.hgroups;
  const int hg = blockIdx.y - kvh * a.hgroups;
  const int head0 = kvh * a.G + hg * GC;
  const int64_t pbeg = (int64_t)split * a.pps;
  const int64_t pend = pbeg + a.pps < npages ? pbeg + a.pps : npages;
  const int64_t new_pos = (int64_t)L_in - 1;
  const int64_t pnew = new_pos / BS;
  const bool fuse = a.nk != nullptr && !clamped;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x < kNW * kStages) va::mbar_init(&bars[threadIdx.x], 1);
  va::fence_barrier_init();
  __syncthreads();

  const int64_t span = pend - pbeg;
  const int nloc = span > warp ? (int)((span - warp + kNW - 1) / kNW) : 0;
  const int32_t *bt_row = a.bt + (int64_t)bt_seq * a.max_blocks;
  const uint64_t policy = va::l2_policy_evict_first();
  const bool contiguous = (a.s_token == D);

  auto stage_k = [&](int slot) { return stage + (size_t)((warp * kStages + slot) * 2) * PAGE; };

  // Issue the K and V tile copies of local page k (warp-uniform call).
  auto issue = [&](int k) {
    const int64_t page = pbeg + warp + (int64_t)k * kNW;
    const int slot = k % kStages;
    uint64_t *bar = &bars[warp * kStages + slot];
    const int32_t blk = bt_row[page];
    if (blk < 0 || blk >= a.num_blocks) {
      if (lane == 0) va::mbar_arrive(bar);
      return;
    }
    __half *dk = stage_k(slot);
    __half *dv = dk + PAGE;
    const __half *sk = a.kc + (int64_t)blk * a.s_block + (int64_t)kvh * a.s_head;
    const __half *sv = a.vc + (int64_t)blk * a.s_block + (int64_t)kvh * a.s_head;
    if (contiguous) {
      if (lane == 0) {
        va::mbar_arrive_expect_tx(bar, 2 * PAGE * 2);
        va::bulk_copy_g2s(dk, sk, PAGE * 2, bar, policy);
        va::bulk_copy_g2s(dv, sv, PAGE * 2, bar, policy);
      }
    } else {
      if (lane == 0) va::mbar_arrive_expect_tx(bar, 2 * PAGE * 2);
      __syncwarp();
      if (lane < BS) {
        va::bulk_copy_g2s(dk + lane * D, sk + (int64_t)lane * a.s_token, D * 2, bar, policy);
        va::bulk_copy_g2s(dv + lane * D, sv + (int64_t)lane * a.s_token, D * 2, bar, policy);
      }
    }
  };

#pragma unroll 1
  for (int k = 0; k < kStages && k < nloc; ++k) issue(k);

  // q of every head of the group, DPL dims of this lane's chunk, packed fp16.
  const int tq = lane / TPT, cq = lane % TPT;
  constexpr int NCH = DPL / 8;  // 16-byte chunks per lane
  const int rot = chunk_rot<D>(lane);
  uint32_t qr[GC][DPL / 2];
#pragma unroll
  for (int h = 0; h < GC; ++h) {
    const uint4 *qp = reinterpret_cast<const uint4 *>(a.q + qo * a.q_s_token +
                                                      (int64_t)(head0 + h) * a.q_s_head +
                                                      cq * DPL);
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      int c = j + rot;
      if (c >= NCH) c -= NCH;
      const uint4 v = __ldg(qp + c);
      qr[h][4 * j + 0] = v.x; qr[h][4 * j + 1] = v.y;
      qr[h][4 * j + 2] = v.z; qr[h][4 * j + 3] = v.w;
    }
  }
  const int hb = rs_head_base<GP, TPT / 2>(lane);

  float m[R], lsum[R];
#pragma unroll
  for (int r = 0; r < R; ++r) { m[r] = -INFINITY; lsum[r] = 0.f; }
  float acc[GC][DV];
#pragma unroll
  for (int h = 0; h < GC; ++h)
#pragma unroll
    for (int j = 0; j < DV; ++j) acc[h][j] = 0.f;

  float *pw = pbuf + warp * BS * GP;
  float *aw = abuf + warp * GP;
  bool dead = false;

#pragma unroll 1
  for (int k = 0; k < nloc; ++k) {
    const int slot = k % kStages;
    const uint32_t parity = (uint32_t)(k / kStages) & 1u;
    if (!va::mbar_wait_bounded(&bars[warp * kStages + slot], parity, dead ? 64u : kWaitLimit)) {
      if (!dead && lane == 0) {
        va::raise_flag(a.err, VA_FLAG_WAIT_TIMEOUT);
#ifdef VA_DIAG_SITES  // diagnostic builds: bit 20 decode, bit 21 one-token prefill rows
        va::raise_flag(a.err, 0x100 << (a.rows ? 13 : 12));
#endif
      }
      dead = true;
    }
    const int64_t page = pbeg + warp + (int64_t)k * kNW;
    const int32_t blk = bt_row[page];
    const bool ok = !dead && blk >= 0 && blk < a.num_blocks;
    if (!ok && !dead && lane == 0) va::raise_flag(a.err, VA_FLAG_BAD_BLOCK);
    const int64_t left = L - page * BS;
    const int ntok = ok ? (left < BS ? (int)left : BS) : 0;
    __half *sk = stage_k(slot);
    __half *sv = sk + PAGE;

    if (fuse && ok && page == pnew) {  // fused KV write of the new token
      const int row = (int)(new_pos - pnew * BS);
      constexpr int CPR = D / 8;  // 16-byte chunks per row
      for (int c = lane; c < 2 * CPR; c += 32) {
        const int which = c / CPR, cc = c - which * CPR;
        const __half *src = (which ? a.nv : a.nk) + (int64_t)seq * a.n_s_token +
                            (int64_t)kvh * a.n_s_head + cc * 8;
        const uint4 val = __ldg(reinterpret_cast<const uint4 *>(src));
        *reinterpret_cast<uint4 *>((which ? sv : sk) + row * D + cc * 8) = val;
        if (hg == 0) {
          __half *dst = (which ? a.vc : a.kc) + (int64_t)blk * a.s_block +
                        (int64_t)kvh * a.s_head + (int64_t)row * a.s_token + cc * 8;
          *reinterpret_cast<uint4 *>(dst) = val;
        }
      }
      __syncwarp();
    }

    if (ntok > 0) {
      // ---- scores ----
      float sc[NPASS][R];
#pragma unroll
      for (int P = 0; P < NPASS; ++P) {
        const int t = P * TOK + tq;
        const __half *krow = sk + t * D + cq * DPL;
        uint32_t kr[DPL / 2];
#pragma unroll
        for (int j = 0; j < NCH; ++j) {
          int c = j + rot;
          if (c >= NCH) c -= NCH;
          const uint4 x = *reinterpret_cast<const uint4 *>(krow + 8 * c);
          kr[4 * j + 0] = x.x; kr[4 * j + 1] = x.y; kr[4 * j + 2] = x.z; kr[4 * j + 3] = x.w;
        }
        // two independent FMA chains per head, summed at the end
        float part[GP], part2[GP];
#pragma unroll
        for (int h = 0; h < GP; ++h) { part[h] = 0.f; part2[h] = 0.f; }
#pragma unroll
        for (int h = 0; h < GC; ++h)
#pragma unroll
          for (int j = 0; j < DPL / 2; j += 2) {
            va::fma2_f16_f32(part[h], qr[h][j], kr[j]);
            va::fma2_f16_f32(part2[h], qr[h][j + 1], kr[j + 1]);
          }
#pragma unroll
        for (int h = 0; h < GC; ++h) part[h] += part2[h];
        reduce_scatter<GP, TPT / 2>(part, lane);
        const bool valid = t < ntok;
#pragma unroll
        for (int r = 0; r < R; ++r) sc[P][r] = valid ? part[r] * a.scale_log2 : -INFINITY;
      }
      // ---- online softmax (per head, over this page) ----
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float mx = sc[0][r];
#pragma unroll
        for (int P = 1; P < NPASS; ++P) mx = fmaxf(mx, sc[P][r]);
#pragma unroll
        for (int mk = TPT; mk < 32; mk <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, mk));
        const float mn = fmaxf(m[r], mx);
        const bool none = (mn == -INFINITY);
        const float alpha = none ? 1.f : va::fast_exp2(m[r] - mn);
        float ps = 0.f;
        const int h = hb + r;
#pragma unroll
        for (int P = 0; P < NPASS; ++P) {
          const float p = none ? 0.f : va::fast_exp2(sc[P][r] - mn);
          ps += p;
          if (h < GC) pw[(P * TOK + tq) * GP + h] = p;
        }
        lsum[r] = lsum[r] * alpha + ps;
        m[r] = mn;
        if (tq == 0 && h < GC) aw[h] = alpha;
      }
      __syncwarp();
      // ---- PV ----
      float al[GC];
#pragma unroll
      for (int h = 0; h < GC; ++h) al[h] = aw[h];
#pragma unroll
      for (int h = 0; h < GC; ++h) {
        if constexpr (DV % 2 == 0) {
#pragma unroll
          for (int j = 0; j < DV; j += 2) fmul2_bcast(acc[h][j], acc[h][j + 1], al[h]);
        } else {
#pragma unroll
          for (int j = 0; j < DV; ++j) acc[h][j] *= al[h];
        }
      }
      auto pv_token = [&](int t) {
        float v[DV];
        load_v<D>(sv + t * D, lane, v);
        const float *pr = pw + t * GP;
        float p[GP];
        if constexpr (GP >= 4) {
#pragma unroll
          for (int i = 0; i < GP; i += 4) {
            const float4 x = *reinterpret_cast<const float4 *>(pr + i);
            p[i] = x.x; p[i + 1] = x.y; p[i + 2] = x.z; p[i + 3] = x.w;
          }
        } else if constexpr (GP == 2) {
          const float2 x = *reinterpret_cast<const float2 *>(pr);
          p[0] = x.x; p[1] = x.y;
        } else {
          p[0] = pr[0];
        }
#pragma unroll
        for (int h = 0; h < GC; ++h) {
          if constexpr (DV % 2 == 0) {
#pragma unroll
            for (int j = 0; j < DV; j += 2)
              ffma2_bcast(acc[h][j], acc[h][j + 1], p[h], v[j], v[j + 1]);
          } else {
#pragma unroll
            for (int j = 0; j < DV; ++j) acc[h][j] = fmaf(p[h], v[j], acc[h][j]);
          }
        }
      };
      if (ntok == BS) {
#pragma unroll
        for (int t = 0; t < BS; ++t) pv_token(t);
      } else {
#pragma unroll 1
        for (int t = 0; t < ntok; ++t) pv_token(t);
      }
    }
    va::fence_proxy_async_smem();
    __syncwarp();
    if (k + kStages < nloc && !dead) issue(k + kStages);
  }

  // final per-head denominators: sum the per-lane partials over token lanes
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int mk = TPT; mk < 32; mk <<= 1)
      lsum[r] += __shfl_xor_sync(0xffffffffu, lsum[r], mk);

  // ---- merge the warps through shared memory (stage area reused) ----
  __syncthreads();
  float *wacc = reinterpret_cast<float *>(smem);  // [NW][GC][D]
  float *wm = wacc + kNW * GC * D;                  // [NW][GP]
  float *wl = wm + kNW * GP;                        // [NW][GP]
#pragma unroll
  for (int h = 0; h < GC; ++h)
#pragma unroll
    for (int j = 0; j < DV; ++j) wacc[(warp * GC + h) * D + pv_dim<D>(lane, j)] = acc[h][j];
  if (tq == 0) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int h = hb + r;
      if (h < GC) { wm[warp * GP + h] = m[r]; wl[warp * GP + h] = lsum[r]; }
    }
  }
  __syncthreads();

  const bool single = (nsplit == 1);
  const int64_t part_base = ((int64_t)seq * a.Hq + head0) * a.max_splits;
  for (int idx = threadIdx.x; idx < GC * D; idx += kNW * 32) {
    const int h = idx / D, d = idx - (idx / D) * D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kNW; ++w) M = fmaxf(M, wm[w * GP + h]);
    float Ls = 0.f, A = 0.f;
#pragma unroll
    for (int w = 0; w < kNW; ++w) {
      const float mw = wm[w * GP + h];
      if (mw != -INFINITY) {
        const float e = va::fast_exp2(mw - M);
        Ls = fmaf(wl[w * GP + h], e, Ls);
        A = fmaf(wacc[(w * GC + h) * D + d], e, A);
      }
    }
    if (single) {
      const float inv = Ls > 0.f ? 1.f / Ls : 0.f;
      a.out[qo * a.o_s_token + (int64_t)(head0 + h) * a.o_s_head + d] =
          __float2half_rn(A * inv);
    } else {
      const int64_t pidx = part_base + (int64_t)h * a.max_splits + split;
      a.ws_acc[pidx * D + d] = A;
      if (d == 0) { a.ws_ml[2 * pidx] = M; a.ws_ml[2 * pidx + 1] = Ls; }
    }
  }
}


// Number of pages and splits of one sequence, clamped exactly as the main kernel.
VA_DEVINL int64_t seq_splits(const DecodeArgs &a, int L_in, int bs, int grid_splits) {
  int64_t npages = ((int64_t)L_in + bs - 1) / bs;
  if (npages > a.max_blocks) npages = a.max_blocks;
  int64_t nsplit = (npages + a.pps - 1) / a.pps;
  return nsplit > grid_splits ? grid_splits : nsplit;
}

// Merge the split partials of one (sequence, q-head group) in split order:
// one thread per output element (block = group heads x head_size threads).
template <int D>
__global__ void __launch_bounds__(1024) paged_decode_combine_kernel(const DecodeArgs a, int gc,
                                                                    int bs) {
  // launched as a programmatic dependent of the split kernel: wait until that grid
  // has completed and its partials are visible
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int seq = blockIdx.x;
  int bt_seq, L_in;
  int64_t qo;
  if (!decode_row(a, seq, bs, bt_seq, L_in, qo)) return;
  const int64_t nsplit = seq_splits(a, L_in, bs, a.max_splits);
  if (nsplit <= 1) return;  // written directly by the main kernel
  const int kvh = blockIdx.y / a.hgroups;
  const int hg = blockIdx.y - kvh * a.hgroups;
  const int h = threadIdx.x / D, d = threadIdx.x - (threadIdx.x / D) * D;
  if (h >= gc) return;
  const int head = kvh * a.G + hg * gc + h;
  const int64_t pb = ((int64_t)seq * a.Hq + head) * a.max_splits;
  const float2 *ml = reinterpret_cast<const float2 *>(a.ws_ml) + pb;
  const float *acc = a.ws_acc + pb * D + d;
  // all loads of up to kU splits issued before any use: one memory latency
  constexpr int kU = 16;
  float mv[kU], lv[kU], av[kU];
#pragma unroll
  for (int s = 0; s < kU; ++s) {
    if (s < nsplit) {
      const float2 v = __ldcs(ml + s);
      mv[s] = v.x;
      lv[s] = v.y;
      av[s] = __ldcs(acc + (int64_t)s * D);
    } else {
      mv[s] = -INFINITY;
      lv[s] = 0.f;
      av[s] = 0.f;
    }
  }
  float M = -INFINITY;
#pragma unroll
  for (int s = 0; s < kU; ++s) M = fmaxf(M, mv[s]);
  for (int s = kU; s < nsplit; ++s) M = fmaxf(M, ml[s].x);
  float Ls = 0.f, A = 0.f;
#pragma unroll
  for (int s = 0; s < kU; ++s) {
    if (mv[s] != -INFINITY) {
      const float e = va::fast_exp2(mv[s] - M);
      Ls = fmaf(lv[s], e, Ls);
      A = fmaf(av[s], e, A);
    }
  }
  for (int s = kU; s < nsplit; ++s) {
    const float2 v = ml[s];
    if (v.x != -INFINITY) {
      const float e = va::fast_exp2(v.x - M);
      Ls = fmaf(v.y, e, Ls);
      A = fmaf(acc[(int64_t)s * D], e, A);
    }
  }
  const float inv = Ls > 0.f ? 1.f / Ls : 0.f;
  a.out[qo * a.o_s_token + (int64_t)head * a.o_s_head + d] = __float2half_rn(A * inv);
}

// Sequences by descending page count (counting sort over page-count buckets, one
// CTA): order[i] = the sequence of grid row i.  Sequences of >= kOrderBuckets - 1
// pages share the top bucket.
constexpr int kOrderBuckets = 1024;
__global__ void __launch_bounds__(1024) order_by_length_kernel(const int32_t *seq_lens,
                                                              int64_t num_seqs, int bs,
                                                              int32_t *order) {
  // the decode grid may launch now; it waits for this grid's completion
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __shared__ int hist[kOrderBuckets];
  __shared__ int warp_buf[32];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  hist[tid] = 0;
  __syncthreads();
  auto bucket = [&](int64_t i) {
    const int L = seq_lens[i];
    const int np = L > 0 ? (L + bs - 1) / bs : 0;
    return kOrderBuckets - 1 - min(np, kOrderBuckets - 1);  // longest -> bucket 0
  };
  for (int64_t i = tid; i < num_seqs; i += 1024) atomicAdd(&hist[bucket(i)], 1);
  __syncthreads();
  // exclusive scan of the bucket counts
  const int c = hist[tid];
  int x = c;
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
  hist[tid] = x - c + (wid > 0 ? warp_buf[wid - 1] : 0);
  __syncthreads();
  for (int64_t i = tid; i < num_seqs; i += 1024) order[atomicAdd(&hist[bucket(i)], 1)] = (int32_t)i;
}

// Whether a grid of `units` (sequence, kv head, q-head group) CTAs runs longest first
// (VA_DECODE_ORDER=0 / 1 forces never / always).  With enough units the ordered grid is
// an LPT schedule (at head_size > 64 it then needs no splitting, see make_plan); below
// that the order does not pay for its extra launch (measured: Qwen shape batch 64
// 28.5 -> 32.2 us, 22B batch 64 124 -> 131 us with it; Qwen batch 512, 1024 units,
// 155 -> 141 us).
bool order_enabled(int64_t units, int head_size) {
  static int env = -2;
  if (env == -2) {
    const char *e = getenv("VA_DECODE_ORDER");
    env = e ? atoi(e) : -1;
  }
  if (env >= 0) return env != 0;
  return units >= 1024;
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct Plan {
  int gc, hgroups, pps, max_splits;
  bool ordered;  // grid rows taken longest first
};

int largest_group_divisor(int g) {
  for (int c = 8; c >= 1; --c)
    if (g % c == 0) return c;
  return 1;
}

// allow_order: false for the one-token rows of a prefill batch, whose grid is sized
// by an upper bound of the rows (most grid rows may be empty).
Plan make_plan(int64_t num_seqs, int Hq, int Hkv, int head_size, int block_size,
               int64_t max_seq_len, bool allow_order = true) {
  Plan p{};
  const int G = Hq / Hkv;
  p.gc = largest_group_divisor(G);
  p.hgroups = G / p.gc;
  const int64_t npmax = (max_seq_len + block_size - 1) / block_size;
  const int64_t base = num_seqs * Hkv * p.hgroups;
  static int env_pps = -1;
  if (env_pps < 0) {
    const char *e = getenv("VA_DECODE_PAGES_PER_SPLIT");
    env_pps = e ? atoi(e) : 0;
  }
  int pps = env_pps;
  p.ordered = allow_order && order_enabled(base, head_size);
  if (pps <= 0 && p.ordered && head_size > 64) {
    // Longest first with at least ~2 waves of CTAs: an LPT schedule of whole sequences
    // balances the SMs by itself; splitting only adds partials, a combine and more
    // CTAs.  Measured on B200 (22B shape, us): 128 sequences 230 -> 200, the 128-, 256-
    // and 512-sequence shards of the batch of 1024 232 -> 203, 418 -> 392, 812 -> 783;
    // pages per split 128 / 256 gave 216 / 214 at 128 sequences.  At head_size <= 64
    // (many q heads per kv head, compute-heavy pages) splitting still pays: Qwen shape
    // batch 256 unsplit 101 us against 83 us split.
    pps = 512;
  } else if (pps <= 0) {
    // Largest split (fewest partials, fewest idle CTAs) whose worst-case CTA count
    // still reaches 2048, and at head_size <= 64 at least 8 pages per split unless the
    // grid is tiny (fewer than 32 sequence x kv-head units: Qwen batch 4 runs best at 4).
    // Measured on B200 (graph replay, us; the earlier floors 8192 at head_size 128,
    // 2048 at 64, no minimum -> this rule): 22B shape batch 16 88.4 -> 44.3, batch 32
    // 96.8 -> 62.2 (32 / 64 pages per split instead of 4 / 8); Qwen shape batch 16
    // 20.5 -> 14.6 (8 instead of 4); unchanged at Qwen batch 64 and 256.
    // The one-token rows of a prefill batch keep the earlier, higher floors: their
    // grid is sized by an upper bound of the rows, so `base` overstates the CTAs
    // (config-4 mixed step: 321 us with them, 350 us with 2048).
    const int64_t floor_units =
        allow_order ? 2048 : (head_size >= 128 ? 8192 : (head_size >= 96 ? 4096 : 2048));
    const int min_pps = (allow_order && head_size <= 64 && base >= 32) ? 8 : 4;
    const int choices[] = {512, 256, 128, 64, 32, 16, 8, 4};
    pps = min_pps;
    for (int c : choices)
      if (c >= min_pps && base * ((npmax + c - 1) / c) >= floor_units) { pps = c; break; }
  }
  p.pps = pps;
  const int64_t ms = npmax > 0 ? (npmax + pps - 1) / pps : 1;
  p.max_splits = (int)(ms < 1 ? 1 : ms);
  return p;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct WsLayout {
  size_t acc, ml, order, total;
  bool ordered;
};

// [split partials: acc, (m, l)] [sequence order]; empty when neither is needed.
WsLayout ws_layout(int64_t num_seqs, int Hq, int Hkv, int D, const Plan &p,
                   bool with_order = false) {
  WsLayout w{};
  if (p.max_splits > 1) {
    const size_t parts = (size_t)num_seqs * Hq * p.max_splits;
    w.acc = 0;
    w.ml = align256(parts * D * 4);
    w.total = w.ml + align256(parts * 2 * 4);
  }
  if (with_order) {
    w.ordered = true;
    w.order = w.total;
    w.total += align256((size_t)num_seqs * 4);
  }
  return w;
}

template <int D, int GC, int BS>
int launch_t(const DecodeArgs &a, dim3 grid, cudaStream_t st) {
  using C = Cfg<D, GC, BS>;
  // per-device opt-in to the kernel's dynamic shared memory (setting it twice from
  // two threads is harmless; the flag only saves the call)
  static std::atomic<int> configured[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(paged_decode_kernel<D, GC, BS>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)C::kSmem) != cudaSuccess)
      return VA_ERR_LAUNCH;
    configured[dev].store(1, std::memory_order_release);
  }
  if (a.order) {
    // launched as a programmatic dependent of the ordering kernel, so its launch
    // overlaps that kernel (it waits for the order before reading it)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kNW * 32);
    cfg.dynamicSmemBytes = C::kSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, paged_decode_kernel<D, GC, BS>, a) != cudaSuccess)
      return VA_ERR_LAUNCH;
  } else {
    paged_decode_kernel<D, GC, BS><<<grid, kNW * 32, C::kSmem, st>>>(a);
  }
  if (grid.x > 1) {
    const int st0 = va_host::launch_status();
    if (st0 != VA_OK) return st0;
    // programmatic dependent launch: the combine grid's launch overlaps the split
    // kernel's tail instead of following its completion
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid.z, grid.y);
    cfg.blockDim = dim3(GC * D);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, paged_decode_combine_kernel<D>, a, GC, BS) != cudaSuccess)
      return VA_ERR_LAUNCH;
  }
  return va_host::launch_status();
}

template <int D, int BS>
int launch_g(int gc, const DecodeArgs &a, dim3 grid, cudaStream_t st) {
  switch (gc) {
    case 1: return launch_t<D, 1, BS>(a, grid, st);
    case 2: return launch_t<D, 2, BS>(a, grid, st);
    case 3: return launch_t<D, 3, BS>(a, grid, st);
    case 4: return launch_t<D, 4, BS>(a, grid, st);
    case 5: return launch_t<D, 5, BS>(a, grid, st);
    case 6: return launch_t<D, 6, BS>(a, grid, st);
    case 7: return launch_t<D, 7, BS>(a, grid, st);
    case 8: return launch_t<D, 8, BS>(a, grid, st);
  }
  return VA_ERR_UNSUPPORTED;
}

}  // namespace

namespace va_internal {

// Workspace bytes of decode_rows for up to rows_bound rows.
size_t decode_rows_workspace(int64_t rows_bound, int Hq, int Hkv, int D, int bs,
                             int64_t max_blocks) {
  if (rows_bound <= 0 || Hkv <= 0 || Hq % Hkv) return 0;
  const Plan p = make_plan(rows_bound, Hq, Hkv, D, bs, max_blocks * bs, false);
  return ws_layout(rows_bound, Hq, Hkv, D, p).total;
}

// Split-KV decode attention of one-token prefill rows (row mode).  The row list
// and its length live on the device (written by the prefill planner).
int decode_rows(void *out, const void *q, const void *kc, const void *vc, const int32_t *bt,
                const int32_t *rows, const int32_t *rows_n, const int32_t *tok_seq,
                const int32_t *pos, int64_t rows_bound, int64_t num_seqs, int Hq, int Hkv, int D,
                int bs, int64_t max_blocks, int64_t num_blocks, float scale, int64_t s_block,
                int64_t s_head, int64_t s_token, int64_t q_s_token, int64_t q_s_head,
                int64_t o_s_token, int64_t o_s_head, void *ws, size_t ws_bytes, int32_t *err,
                cudaStream_t st) {
  if (rows_bound <= 0) return VA_OK;
  if (rows_bound > 65535 || bs != 16) return VA_ERR_UNSUPPORTED;
  const Plan p = make_plan(rows_bound, Hq, Hkv, D, bs, max_blocks * bs, false);
  const WsLayout w = ws_layout(rows_bound, Hq, Hkv, D, p);
  if (w.total && (!ws || ws_bytes < w.total)) return VA_ERR_WORKSPACE;
  DecodeArgs a{};
  a.out = static_cast<__half *>(out);
  a.q = static_cast<const __half *>(q);
  a.kc = const_cast<__half *>(static_cast<const __half *>(kc));
  a.vc = const_cast<__half *>(static_cast<const __half *>(vc));
  a.bt = bt;
  unsigned char *wsb = static_cast<unsigned char *>(ws);
  a.ws_acc = w.total ? reinterpret_cast<float *>(wsb + w.acc) : nullptr;
  a.ws_ml = w.total ? reinterpret_cast<float *>(wsb + w.ml) : nullptr;
  a.err = err;
  a.max_blocks = max_blocks;
  a.num_blocks = num_blocks;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.G = Hq / Hkv;
  a.hgroups = p.hgroups;
  a.pps = p.pps;
  a.max_splits = p.max_splits;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.s_block = s_block; a.s_head = s_head; a.s_token = s_token;
  a.q_s_token = q_s_token; a.q_s_head = q_s_head;
  a.o_s_token = o_s_token; a.o_s_head = o_s_head;
  a.rows = rows; a.rows_n = rows_n; a.row_tok_seq = tok_seq; a.row_pos = pos;
  a.row_num_seqs = num_seqs;
  const dim3 grid((unsigned)p.max_splits, (unsigned)(Hkv * p.hgroups), (unsigned)rows_bound);
  switch (D) {
    case 32: return launch_g<32, 16>(p.gc, a, grid, st);
    case 64: return launch_g<64, 16>(p.gc, a, grid, st);
    case 96: return launch_g<96, 16>(p.gc, a, grid, st);
    case 128: return launch_g<128, 16>(p.gc, a, grid, st);
  }
  return VA_ERR_UNSUPPORTED;
}

}  // namespace va_internal

extern "C" size_t va_paged_decode_workspace_size(int64_t num_seqs, int num_query_heads,
                                                 int num_kv_heads, int head_size,
                                                 int block_size, int64_t max_seq_len) {
  if (num_seqs <= 0 || num_kv_heads <= 0 || num_query_heads % num_kv_heads || block_size <= 0)
    return 0;
  const Plan p = make_plan(num_seqs, num_query_heads, num_kv_heads, head_size, block_size, max_seq_len);
  return ws_layout(num_seqs, num_query_heads, num_kv_heads, head_size, p, p.ordered).total;
}

extern "C" int va_paged_decode(void *out, const void *q, void *k_cache, void *v_cache,
                               const int32_t *block_table, const int32_t *seq_lens,
                               const void *new_k, const void *new_v, int64_t num_seqs,
                               int num_query_heads, int num_kv_heads, int head_size,
                               int block_size, int64_t max_blocks_per_seq, int64_t max_seq_len,
                               int64_t num_blocks, float scale, int64_t s_block, int64_t s_head,
                               int64_t s_token, int64_t q_s_token, int64_t q_s_head,
                               int64_t o_s_token, int64_t o_s_head, int64_t new_s_token,
                               int64_t new_s_head, void *workspace, size_t workspace_bytes,
                               int32_t *err_flag, void *stream) {
  if (num_seqs < 0 || max_seq_len < 0 || num_blocks < 0 || max_blocks_per_seq < 0)
    return VA_ERR_INVALID_ARG;
  if (num_seqs == 0 || max_seq_len == 0) return VA_OK;
  if (!out || !q || !k_cache || !v_cache || !block_table || !seq_lens) return VA_ERR_INVALID_ARG;
  if (num_kv_heads <= 0 || num_query_heads <= 0 || num_query_heads % num_kv_heads)
    return VA_ERR_INVALID_ARG;
  if ((new_k == nullptr) != (new_v == nullptr)) return VA_ERR_INVALID_ARG;
  if (num_seqs > 65535) return VA_ERR_UNSUPPORTED;
  if (block_size != 16) return VA_ERR_UNSUPPORTED;
  if (head_size != 32 && head_size != 64 && head_size != 96 && head_size != 128)
    return VA_ERR_UNSUPPORTED;
  // 16-byte alignment of every row the kernel moves with vector or bulk copies
  auto m8 = [](int64_t s) { return s % 8 == 0; };
  if (!va_host::aligned16(q) || !va_host::aligned16(k_cache) || !va_host::aligned16(v_cache) ||
      !m8(s_block) || !m8(s_head) || !m8(s_token) || !m8(q_s_token) || !m8(q_s_head))
    return VA_ERR_INVALID_ARG;
  if (new_k && (!va_host::aligned16(new_k) || !va_host::aligned16(new_v) || !m8(new_s_token) ||
                !m8(new_s_head)))
    return VA_ERR_INVALID_ARG;

  const Plan p = make_plan(num_seqs, num_query_heads, num_kv_heads, head_size, block_size, max_seq_len);
  const WsLayout w = ws_layout(num_seqs, num_query_heads, num_kv_heads, head_size, p,
                               p.ordered);
  if (w.total && (!workspace || workspace_bytes < w.total)) return VA_ERR_WORKSPACE;

  DecodeArgs a{};
  a.out = static_cast<__half *>(out);
  a.q = static_cast<const __half *>(q);
  a.kc = static_cast<__half *>(k_cache);
  a.vc = static_cast<__half *>(v_cache);
  a.bt = block_table;
  a.seq_lens = seq_lens;
  a.nk = static_cast<const __half *>(new_k);
  a.nv = static_cast<const __half *>(new_v);
  unsigned char *ws = static_cast<unsigned char *>(workspace);
  a.ws_acc = p.max_splits > 1 ? reinterpret_cast<float *>(ws + w.acc) : nullptr;
  a.ws_ml = p.max_splits > 1 ? reinterpret_cast<float *>(ws + w.ml) : nullptr;
  a.err = err_flag;
  a.max_blocks = max_blocks_per_seq;
  a.num_blocks = num_blocks;
  a.Hq = num_query_heads;
  a.Hkv = num_kv_heads;
  a.G = num_query_heads / num_kv_heads;
  a.hgroups = p.hgroups;
  a.pps = p.pps;
  a.max_splits = p.max_splits;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.s_block = s_block; a.s_head = s_head; a.s_token = s_token;
  a.q_s_token = q_s_token; a.q_s_head = q_s_head;
  a.o_s_token = o_s_token; a.o_s_head = o_s_head;
  a.n_s_token = new_s_token; a.n_s_head = new_s_head;

  const dim3 grid((unsigned)p.max_splits, (unsigned)(num_kv_heads * p.hgroups),
                  (unsigned)num_seqs);
  auto st = static_cast<cudaStream_t>(stream);
  if (w.ordered) {
    int32_t *ord = reinterpret_cast<int32_t *>(ws + w.order);
    order_by_length_kernel<<<1, 1024, 0, st>>>(seq_lens, num_seqs, block_size, ord);
    if (va_host::launch_status() != VA_OK) return VA_ERR_LAUNCH;
    a.order = ord;
  }
  switch (head_size) {
    case 32: return launch_g<32, 16>(p.gc, a, grid, st);
    case 64: return launch_g<64, 16>(p.gc, a, grid, st);
    case 96: return launch_g<96, 16>(p.gc, a, grid, st);
    case 128: return launch_g<128, 16>(p.gc, a, grid, st);
  }
  return VA_ERR_UNSUPPORTED;
}

// ---------------------------------------------------------------------------
// Decode without caller-provided scratch.
//
// For callers that cannot allocate device memory themselves -- a host that
// reaches this library only through its C ABI (an FFI binding with no CUDA
// allocator of its own), or a serving loop whose device memory is fixed up
// front by another runtime and must not call cudaMalloc/cudaFree (which can
// synchronise the device) once it is running.  The split-KV partials live in
// the file-scope array below instead of a workspace argument.  Every GPU that
// loads this library reserves VA_DECODE_STATIC_SCRATCH_BYTES for it until the
// process exits.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_decode_scratch[VA_DECODE_STATIC_SCRATCH_BYTES];

namespace {
std::mutex g_scratch_mu;
void *g_scratch_ptr[64] = {nullptr};
}  // namespace

extern "C" int va_paged_decode_noalloc(void *out, const void *q, void *k_cache, void *v_cache,
                                       const int32_t *block_table, const int32_t *seq_lens,
                                       const void *new_k, const void *new_v, int64_t num_seqs,
                                       int num_query_heads, int num_kv_heads, int head_size,
                                       int block_size, int64_t max_blocks_per_seq,
                                       int64_t max_seq_len, int64_t num_blocks, float scale,
                                       int64_t s_block, int64_t s_head, int64_t s_token,
                                       int64_t q_s_token, int64_t q_s_head, int64_t o_s_token,
                                       int64_t o_s_head, int64_t new_s_token,
                                       int64_t new_s_head, int32_t *err_flag, void *stream) {
  // the shape checks of va_paged_decode come first, so a shape it would reject
  // reports the same status here, whatever its scratch need
  if (num_seqs < 0 || max_seq_len < 0 || num_blocks < 0 || max_blocks_per_seq < 0 ||
      num_kv_heads <= 0 || num_query_heads <= 0 || num_query_heads % num_kv_heads)
    return VA_ERR_INVALID_ARG;
  if (num_seqs > 65535 || block_size != 16 ||
      (head_size != 32 && head_size != 64 && head_size != 96 && head_size != 128))
    return VA_ERR_UNSUPPORTED;
  const size_t need = va_paged_decode_workspace_size(num_seqs, num_query_heads, num_kv_heads,
                                                     head_size, block_size, max_seq_len);
  if (need > (size_t)VA_DECODE_STATIC_SCRATCH_BYTES) return VA_ERR_SCRATCH_LIMIT;
  void *ws = nullptr;
  if (need) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return VA_ERR_LAUNCH;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
      // The array's host-side name is only a handle; its device address comes
      // from the runtime, once per device, with that device current.
      void *p = nullptr;
      if (cudaGetSymbolAddress(&p, g_decode_scratch) != cudaSuccess || !p) {
        cudaGetLastError();
        return VA_ERR_LAUNCH;
      }
      g_scratch_ptr[dev] = p;
    }
    ws = g_scratch_ptr[dev];
  }
  // The split partials need no initial value: the combine reads only what the
  // main kernel of the same call wrote.
  return va_paged_decode(out, q, k_cache, v_cache, block_table, seq_lens, new_k, new_v,
                         num_seqs, num_query_heads, num_kv_heads, head_size, block_size,
                         max_blocks_per_seq, max_seq_len, num_blocks, scale, s_block, s_head,
                         s_token, q_s_token, q_s_head, o_s_token, o_s_head, new_s_token,
                         new_s_head, ws, need, err_flag, stream);
}
