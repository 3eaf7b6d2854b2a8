// Shared device/host helpers for the sm_100a paged-attention kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "vllm_apple_b200.h"

#define VA_DEVINL __device__ __forceinline__

namespace va {

// ---------------------------------------------------------------------------
// error flag
// ---------------------------------------------------------------------------
// Programmatic dependent launch, device side: let the next grid on the stream be
// scheduled now, then wait for the previous grid's completion and memory before
// touching any input (a no-op wait when this grid was launched without the attribute).
VA_DEVINL void pdl_enter() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

VA_DEVINL void raise_flag(int32_t *flag, int32_t bits) {
  if (flag) atomicOr(flag, bits);
}

// ---------------------------------------------------------------------------
// shared-memory / async-proxy PTX wrappers (sm_90+ ISA, used on sm_100a)
// ---------------------------------------------------------------------------
VA_DEVINL uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

VA_DEVINL void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

// Invalidate a barrier whose phases have all completed (before re-initialising it).
VA_DEVINL void mbar_inval(uint64_t *bar) {
  asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Make barrier initialisation visible to the async (bulk-copy) proxy.
VA_DEVINL void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Order this thread's prior generic-proxy shared-memory accesses before later
// async-proxy accesses (a bulk copy that overwrites a buffer just read).
VA_DEVINL void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

VA_DEVINL void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

VA_DEVINL void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

VA_DEVINL void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

VA_DEVINL bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on a barrier phase.  Returns false when `limit` polls (each a
// hardware-suspended try_wait) did not see the phase complete.
VA_DEVINL bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, uint32_t limit) {
  for (uint32_t i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// 1-D bulk copy global -> shared, completion signalled on `bar` as tx bytes.
// dst/src 16-byte aligned, bytes a multiple of 16.  No multicast.
VA_DEVINL void bulk_copy_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                             uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

VA_DEVINL uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// ---------------------------------------------------------------------------
// fp16 helpers
// ---------------------------------------------------------------------------
// acc += a.lo*b.lo + a.hi*b.hi with fp16 operands and an fp32 accumulator
// (sm_100 mixed-precision FMA: the product is exact, one rounding per FMA,
// identical to converting both operands to fp32 first).
VA_DEVINL void fma2_f16_f32(float &acc, uint32_t a, uint32_t b) {
  asm("{\n\t.reg .f16 al, ah, bl, bh;\n\t"
      "mov.b32 {al, ah}, %1;\n\t"
      "mov.b32 {bl, bh}, %2;\n\t"
      "fma.rn.f32.f16 %0, al, bl, %0;\n\t"
      "fma.rn.f32.f16 %0, ah, bh, %0;\n\t}"
      : "+f"(acc)
      : "r"(a), "r"(b));
}

VA_DEVINL float2 h2_to_f2(uint32_t v) {
  __half2 h = *reinterpret_cast<__half2 *>(&v);
  return __half22float2(h);
}

VA_DEVINL uint32_t pack_h2(float lo, float hi) {  // round-to-nearest fp16 pair
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&h);
}

VA_DEVINL float fast_exp2(float x) {  // hardware ex2.approx; exp2(-inf) = 0
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T>
VA_DEVINL T ldg_stream(const T *p) {  // read-once data: do not allocate in L1
  return __ldcs(p);
}

}  // namespace va

// ---------------------------------------------------------------------------
// host helpers
// ---------------------------------------------------------------------------
namespace va_host {

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? VA_OK : VA_ERR_LAUNCH;
}

// <<<grid, block, 0, st>>> with the programmatic-stream-serialization attribute, so
// the launch overlaps the tail of the kernel before it on the stream.
// Every kernel launched this way must execute griddepcontrol.wait in all of its
// CTAs before it exits (va::pdl_enter at entry), so that its completion still
// implies the completion of everything before it on the stream.
template <typename... KArgs, typename... Args>
int launch_pdl_smem(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                    cudaStream_t st, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...) == cudaSuccess ? 0 : 1;
}

template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, cudaStream_t st,
               Args &&...args) {
  return launch_pdl_smem(kernel, grid, block, 0, st, static_cast<Args &&>(args)...);
}

}  // namespace va_host
