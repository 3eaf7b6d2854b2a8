// Memory-bound per-token ops around the attention step: RMSNorm (+ residual),
// rotary embedding (Neox split-half and GPT-J interleaved) and SiLU-mul.
//
// All three move 16-byte vectors (8 fp16) per thread with coalesced access and
// compute in fp32 with explicitly rounded operations (no FMA contraction), so
// the fp32 intermediate equals the operation-by-operation fp32 formula of the
// reference kernels; the result is rounded to fp16 once.
#include <math.h>

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
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t *>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// ---------------------------------------------------------------------------
// RMSNorm: one CTA per row; the row is read once into registers (VPT vectors
// per thread), reduced with warp shuffles + shared memory, normalised and
// written.
// ---------------------------------------------------------------------------
constexpr int kNormThreads = 128;

template <int THREADS>
VA_DEVINL float block_sum(float v, float *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < THREADS / 32; ++i) t += red[i];
  return t;
}

// Rows are processed grid-stride; the next row's loads are issued before the
// current row is reduced, normalised and stored, so every CTA keeps a row in
// flight from HBM while it works on the previous one.
template <int VPT, bool RES>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_vec_kernel(
    __half *out, const __half *x, const __half *w, const __half *res, int64_t T, int64_t hidden,
    float eps, int64_t xs, int64_t os, int64_t rs) {
  __shared__ float red[2][kNormThreads / 32];  // alternating rows: one barrier per row
  va::pdl_enter();
  const int nvec = (int)(hidden / 8);
  const uint4 *wr = reinterpret_cast<const uint4 *>(w);
  auto load = [&](int64_t row, uint4 (&v)[VPT]) {
    const uint4 *xr = reinterpret_cast<const uint4 *>(x + row * xs);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = threadIdx.x + i * kNormThreads;
      if (c < nvec) v[i] = va::ldg_stream(xr + c);
    }
  };
  uint4 cur[VPT], nxt[VPT];
  int64_t row = blockIdx.x;
  if (row < T) load(row, cur);
  for (int it = 0; row < T; row += gridDim.x, ++it) {
    const int64_t next = row + gridDim.x;
    if (next < T) load(next, nxt);
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = threadIdx.x + i * kNormThreads;
      if (c < nvec) {
        float f[8];
        unpack8(cur[i], f);
#pragma unroll
        for (int j = 0; j < 8; ++j) ss = __fadd_rn(ss, __fmul_rn(f[j], f[j]));
      }
    }
    const float tot = block_sum<kNormThreads>(ss, red[it & 1]);
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)hidden), eps)));
    uint4 *orow = reinterpret_cast<uint4 *>(out + row * os);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = threadIdx.x + i * kNormThreads;
      if (c < nvec) {
        float f[8], g[8];
        unpack8(cur[i], f);
        unpack8(__ldg(wr + c), g);
        float y[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) y[j] = __fmul_rn(__fmul_rn(f[j], r), g[j]);
        if (RES) {
          float q[8];
          unpack8(va::ldg_stream(reinterpret_cast<const uint4 *>(res + row * rs) + c), q);
#pragma unroll
          for (int j = 0; j < 8; ++j) y[j] = __fadd_rn(y[j], q[j]);
        }
        orow[c] = pack8(y);
      }
    }
#pragma unroll
    for (int i = 0; i < VPT; ++i) cur[i] = nxt[i];
  }
}

// Generic path (any hidden size / alignment): two passes over the row, the
// second served from L1/L2.
template <bool RES>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_any_kernel(
    __half *out, const __half *x, const __half *w, const __half *res, int64_t hidden, float eps,
    int64_t xs, int64_t os, int64_t rs) {
  __shared__ float red[kNormThreads / 32];
  const int64_t row = blockIdx.x;
  const __half *xr = x + row * xs;
  float ss = 0.f;
  for (int64_t i = threadIdx.x; i < hidden; i += kNormThreads) {
    const float f = __half2float(xr[i]);
    ss = __fadd_rn(ss, __fmul_rn(f, f));
  }
  const float tot = block_sum<kNormThreads>(ss, red);
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)hidden), eps)));
  for (int64_t i = threadIdx.x; i < hidden; i += kNormThreads) {
    float y = __fmul_rn(__fmul_rn(__half2float(xr[i]), r), __half2float(w[i]));
    if (RES) y = __fadd_rn(y, __half2float(res[row * rs + i]));
    out[row * os + i] = __float2half_rn(y);
  }
}

// Grid: as many CTAs as fit on the GPU at once (rows are walked grid-stride).
template <int VPT, bool RES>
unsigned norm_grid(int64_t T) {
  static int per_sm = 0;
  if (!per_sm) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rmsnorm_vec_kernel<VPT, RES>,
                                                      kNormThreads, 0) != cudaSuccess ||
        per_sm < 1)
      per_sm = 1;
  }
  const int64_t cap = (int64_t)va_host::sm_count() * per_sm;
  return (unsigned)(T < cap ? T : cap);
}

template <int VPT>
void launch_norm_vec(bool r, int64_t T, cudaStream_t st, __half *o, const __half *x,
                     const __half *w, const __half *res, int64_t h, float eps, int64_t xs,
                     int64_t os, int64_t rs) {
  if (r)
    va_host::launch_pdl(rmsnorm_vec_kernel<VPT, true>, norm_grid<VPT, true>(T), kNormThreads, st, o, x,
               w, res, T, h, eps, xs, os, rs);
  else
    va_host::launch_pdl(rmsnorm_vec_kernel<VPT, false>, norm_grid<VPT, false>(T), kNormThreads, st, o,
               x, w, res, T, h, eps, xs, os, rs);
}

// ---------------------------------------------------------------------------
// RoPE: one thread per (token, head, group of 8 rotation pairs).
// ---------------------------------------------------------------------------
struct RopeArgs {
  __half *q, *k;
  const float *cs, *sn;
  const int32_t *pos;
  int64_t T, max_pos, qs, ks;
  int Hq, Hkv, D, rot;
  int32_t *err;
};

VA_DEVINL void rot_pair(float x0, float x1, float c, float s, float &y0, float &y1) {
  y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
  y1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
}

template <bool NEOX>
__global__ void __launch_bounds__(256) rope_vec_kernel(const RopeArgs a) {
  va::pdl_enter();
  const int half = a.rot / 2;
  const int groups = half / 8;
  const int heads = a.Hq + a.Hkv;
  const int64_t total = a.T * heads * groups;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t tok = i / (heads * groups);
    const int rem = (int)(i - tok * heads * groups);
    const int h = rem / groups, gidx = rem - (rem / groups) * groups;
    const int p = a.pos[tok];
    if (p < 0 || p >= a.max_pos) {
      if (h == 0 && gidx == 0) va::raise_flag(a.err, VA_FLAG_BAD_POSITION);
      continue;
    }
    __half *x = h < a.Hq ? a.q + tok * a.qs + (int64_t)h * a.D
                         : a.k + tok * a.ks + (int64_t)(h - a.Hq) * a.D;
    const float4 *cp = reinterpret_cast<const float4 *>(a.cs + (int64_t)p * half + gidx * 8);
    const float4 *sp = reinterpret_cast<const float4 *>(a.sn + (int64_t)p * half + gidx * 8);
    const float4 c0 = __ldg(cp), c1 = __ldg(cp + 1), s0 = __ldg(sp), s1 = __ldg(sp + 1);
    const float c[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float s[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    if (NEOX) {
      uint4 *pa = reinterpret_cast<uint4 *>(x + gidx * 8);
      uint4 *pb = reinterpret_cast<uint4 *>(x + half + gidx * 8);
      float fa[8], fb[8], ya[8], yb[8];
      unpack8(*pa, fa);
      unpack8(*pb, fb);
#pragma unroll
      for (int j = 0; j < 8; ++j) rot_pair(fa[j], fb[j], c[j], s[j], ya[j], yb[j]);
      *pa = pack8(ya);
      *pb = pack8(yb);
    } else {
      uint4 *pa = reinterpret_cast<uint4 *>(x + gidx * 16);
      float f[16], y[16];
      float t0[8], t1[8];
      unpack8(pa[0], t0);
      unpack8(pa[1], t1);
#pragma unroll
      for (int j = 0; j < 8; ++j) { f[j] = t0[j]; f[8 + j] = t1[j]; }
#pragma unroll
      for (int j = 0; j < 8; ++j) rot_pair(f[2 * j], f[2 * j + 1], c[j], s[j], y[2 * j], y[2 * j + 1]);
#pragma unroll
      for (int j = 0; j < 8; ++j) { t0[j] = y[j]; t1[j] = y[8 + j]; }
      pa[0] = pack8(t0);
      pa[1] = pack8(t1);
    }
  }
}

template <bool NEOX>
__global__ void __launch_bounds__(256) rope_any_kernel(const RopeArgs a) {
  const int half = a.rot / 2;
  const int heads = a.Hq + a.Hkv;
  const int64_t total = a.T * heads * half;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t tok = i / (heads * half);
    const int rem = (int)(i - tok * heads * half);
    const int h = rem / half, j = rem - (rem / half) * half;
    const int p = a.pos[tok];
    if (p < 0 || p >= a.max_pos) {
      if (h == 0 && j == 0) va::raise_flag(a.err, VA_FLAG_BAD_POSITION);
      continue;
    }
    __half *x = h < a.Hq ? a.q + tok * a.qs + (int64_t)h * a.D
                         : a.k + tok * a.ks + (int64_t)(h - a.Hq) * a.D;
    const float c = a.cs[(int64_t)p * half + j], s = a.sn[(int64_t)p * half + j];
    const int i0 = NEOX ? j : 2 * j, i1 = NEOX ? j + half : 2 * j + 1;
    float y0, y1;
    rot_pair(__half2float(x[i0]), __half2float(x[i1]), c, s, y0, y1);
    x[i0] = __float2half_rn(y0);
    x[i1] = __float2half_rn(y1);
  }
}

// ---------------------------------------------------------------------------
// SiLU-mul
// ---------------------------------------------------------------------------
// fp32 silu(g) * u rounded to fp16 once.  The quotient uses the fast division
// (<= 2 fp32 ulp; the IEEE divide costs ~4x the instructions on this
// instruction-heavy, HBM-bound loop): both sit ~2^13 fp32 ulps below the fp16
// rounding step, so the fp16 result stays within 1 ulp of the exact value.
VA_DEVINL float silu_mul1(float g, float u) {
  return __fmul_rn(__fdividef(g, __fadd_rn(1.0f, expf(-g))), u);
}
VA_DEVINL float silu_mul1_exact(float g, float u) {
  return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

// Grid-stride over 16-byte vectors, two vectors of each input in flight per
// thread per iteration.
__global__ void __launch_bounds__(256) silu_mul_vec_kernel(uint4 *out, const uint4 *g,
                                                           const uint4 *u, int64_t nvec) {
  va::pdl_enter();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nvec; i += 2 * stride) {
    const int64_t i2 = i + stride;
    const bool two = i2 < nvec;
    const uint4 g0 = va::ldg_stream(g + i), u0 = va::ldg_stream(u + i);
    uint4 g1 = make_uint4(0, 0, 0, 0), u1 = g1;
    if (two) {
      g1 = va::ldg_stream(g + i2);
      u1 = va::ldg_stream(u + i2);
    }
    float fg[8], fu[8], y[8];
    unpack8(g0, fg);
    unpack8(u0, fu);
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = silu_mul1(fg[j], fu[j]);
    __stcs(out + i, pack8(y));
    if (two) {
      unpack8(g1, fg);
      unpack8(u1, fu);
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = silu_mul1(fg[j], fu[j]);
      __stcs(out + i2, pack8(y));
    }
  }
}

__global__ void __launch_bounds__(256) silu_mul_any_kernel(__half *out, const __half *g,
                                                           const __half *u, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = __float2half_rn(silu_mul1_exact(__half2float(g[i]), __half2float(u[i])));
}

unsigned grid_for(int64_t work, int threads) {
  int64_t b = (work + threads - 1) / threads;
  const int64_t cap = (int64_t)va_host::sm_count() * 32;
  if (b > cap) b = cap;
  return (unsigned)(b < 1 ? 1 : b);
}

}  // namespace

extern "C" const char *va_version(void) { return "vllm_apple_b200 0.1.0 sm_100a"; }

extern "C" int va_rmsnorm(void *out, const void *x, const void *weight, const void *residual,
                          int64_t num_tokens, int64_t hidden_size, float eps, int64_t x_s_token,
                          int64_t out_s_token, int64_t res_s_token, void *stream) {
  if (num_tokens < 0 || hidden_size <= 0) return VA_ERR_INVALID_ARG;
  if (num_tokens == 0) return VA_OK;
  if (!out || !x || !weight) return VA_ERR_INVALID_ARG;
  if (num_tokens > 0x7fffffff) return VA_ERR_UNSUPPORTED;
  auto st = static_cast<cudaStream_t>(stream);
  auto o = static_cast<__half *>(out);
  auto xi = static_cast<const __half *>(x);
  auto w = static_cast<const __half *>(weight);
  auto r = static_cast<const __half *>(residual);
  const bool res = residual != nullptr;
  const dim3 g((unsigned)num_tokens);
  const bool vec = hidden_size % 8 == 0 && va_host::aligned16(out) && va_host::aligned16(x) &&
                   va_host::aligned16(weight) && (!res || va_host::aligned16(residual)) &&
                   x_s_token % 8 == 0 && out_s_token % 8 == 0 && (!res || res_s_token % 8 == 0);
  const int64_t vpt = (hidden_size / 8 + kNormThreads - 1) / kNormThreads;
  if (vec && vpt <= 8) {
    switch (vpt) {
      case 1: launch_norm_vec<1>(res, num_tokens, st, o, xi, w, r, hidden_size, eps, x_s_token, out_s_token, res_s_token); break;
      case 2: launch_norm_vec<2>(res, num_tokens, st, o, xi, w, r, hidden_size, eps, x_s_token, out_s_token, res_s_token); break;
      case 3: launch_norm_vec<3>(res, num_tokens, st, o, xi, w, r, hidden_size, eps, x_s_token, out_s_token, res_s_token); break;
      case 4: launch_norm_vec<4>(res, num_tokens, st, o, xi, w, r, hidden_size, eps, x_s_token, out_s_token, res_s_token); break;
      case 5: launch_norm_vec<5>(res, num_tokens, st, o, xi, w, r, hidden_size, eps, x_s_token, out_s_token, res_s_token); break;
      case 6: launch_norm_vec<6>(res, num_tokens, st, o, xi, w, r, hidden_size, eps, x_s_token, out_s_token, res_s_token); break;
      case 7: launch_norm_vec<7>(res, num_tokens, st, o, xi, w, r, hidden_size, eps, x_s_token, out_s_token, res_s_token); break;
      default: launch_norm_vec<8>(res, num_tokens, st, o, xi, w, r, hidden_size, eps, x_s_token, out_s_token, res_s_token); break;
    }
  } else if (res) {
    rmsnorm_any_kernel<true><<<g, kNormThreads, 0, st>>>(o, xi, w, r, hidden_size, eps, x_s_token,
                                                         out_s_token, res_s_token);
  } else {
    rmsnorm_any_kernel<false><<<g, kNormThreads, 0, st>>>(o, xi, w, r, hidden_size, eps,
                                                          x_s_token, out_s_token, res_s_token);
  }
  return va_host::launch_status();
}

extern "C" int va_rope(void *q, void *k, const float *cos_cache, const float *sin_cache,
                       const int32_t *positions, int64_t num_tokens, int num_heads,
                       int num_kv_heads, int head_size, int rotary_dim, int64_t max_position,
                       int64_t q_s_token, int64_t k_s_token, int is_neox, int32_t *err_flag,
                       void *stream) {
  if (num_tokens < 0 || num_heads < 0 || num_kv_heads < 0 || head_size <= 0)
    return VA_ERR_INVALID_ARG;
  if (rotary_dim <= 0 || rotary_dim > head_size || rotary_dim % 2) return VA_ERR_INVALID_ARG;
  if (num_tokens == 0 || num_heads + num_kv_heads == 0) return VA_OK;
  if ((num_heads && !q) || (num_kv_heads && !k) || !cos_cache || !sin_cache || !positions)
    return VA_ERR_INVALID_ARG;
  RopeArgs a{static_cast<__half *>(q), static_cast<__half *>(k), cos_cache, sin_cache, positions,
             num_tokens, max_position, q_s_token, k_s_token, num_heads, num_kv_heads, head_size,
             rotary_dim, err_flag};
  auto st = static_cast<cudaStream_t>(stream);
  const int half = rotary_dim / 2;
  const bool vec = half % 8 == 0 && head_size % 8 == 0 && va_host::aligned16(cos_cache) &&
                   va_host::aligned16(sin_cache) && (!num_heads || va_host::aligned16(q)) &&
                   (!num_kv_heads || va_host::aligned16(k)) && q_s_token % 8 == 0 &&
                   k_s_token % 8 == 0;
  const int heads = num_heads + num_kv_heads;
  if (vec) {
    const unsigned g = grid_for(num_tokens * heads * (half / 8), 256);
    if (is_neox) va_host::launch_pdl(rope_vec_kernel<true>, g, 256, st, a);
    else va_host::launch_pdl(rope_vec_kernel<false>, g, 256, st, a);
  } else {
    const unsigned g = grid_for(num_tokens * heads * half, 256);
    if (is_neox) rope_any_kernel<true><<<g, 256, 0, st>>>(a);
    else rope_any_kernel<false><<<g, 256, 0, st>>>(a);
  }
  return va_host::launch_status();
}

extern "C" int va_silu_mul(void *out, const void *gate, const void *up, int64_t num_elements,
                           void *stream) {
  if (num_elements < 0) return VA_ERR_INVALID_ARG;
  if (num_elements == 0) return VA_OK;
  if (!out || !gate || !up) return VA_ERR_INVALID_ARG;
  auto st = static_cast<cudaStream_t>(stream);
  if (num_elements % 8 == 0 && va_host::aligned16(out) && va_host::aligned16(gate) &&
      va_host::aligned16(up)) {
    const int64_t nvec = num_elements / 8;
    va_host::launch_pdl(silu_mul_vec_kernel, grid_for(nvec, 256), 256, st,
        static_cast<uint4 *>(out), static_cast<const uint4 *>(gate),
        static_cast<const uint4 *>(up), nvec);
  } else {
    silu_mul_any_kernel<<<grid_for(num_elements, 256), 256, 0, st>>>(
        static_cast<__half *>(out), static_cast<const __half *>(gate),
        static_cast<const __half *>(up), num_elements);
  }
  return va_host::launch_status();
}
