// Shared device helpers for the LARA B200 kernels (sm_100a only).
//
// bf16 words are handled as raw uint16 so the C ABI carries no CUDA types;
// the conversions below are exact (bf16 -> fp32 is a 16-bit shift, as in the
// reference's bf16_u16_to_fp32, sw/attn_driver.py:101-103).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "lara_internal.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "lara_b200 kernels are written for sm_100a only"
#endif

namespace lara {

// Upper bound on any single spin-wait, in nanoseconds of %globaltimer.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- programmatic dependent launch ------------------------------------------
// A kernel launched by launch_with_pdl() may start while the kernel before it
// in the stream is still running.  It calls allow_dependent_launch() on entry
// (the next kernel may then be scheduled once every CTA of this grid has
// started) and grid_dependency_wait() before its first global-memory access:
// that wait returns once the previous grid has completed and its writes are
// visible.  Launched without the attribute, both are no-ops.

__device__ __forceinline__ void allow_dependent_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---- mbarrier ---------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
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

// Non-blocking test of phase completion (acquire at CTA scope).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (and never spins forever) if the phase with the
// given parity has not completed within limit_ns (default kWaitLimitNs).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > limit_ns) return false;
  }
}

// ---- bulk async copy (TMA, non-tensor, no multicast) ------------------------

__device__ __forceinline__ uint64_t make_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Copies `bytes` (multiple of 16, both addresses 16-byte aligned) from global
// to this CTA's shared memory; completion is signalled on `bar` as tx bytes.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_addr(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// Asks L2 to fetch `bytes` (multiple of 16, 16-byte aligned address) of global
// memory; no completion is tracked.  L2 is the GPU's point of coherence, so a
// prefetch never makes a later read return stale data, whenever it is issued.
__device__ __forceinline__ void bulk_prefetch_l2(const void* gmem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(gmem_src), "r"(bytes) : "memory");
}

// 2^x by the special-function unit alone: ex2.approx.ftz.f32 (relative error
// about 2^-22; a result below 2^-126 flushes to +0, and -inf gives +0).  A
// probability that small is below the last bit of any output it could enter.
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---- bf16 helpers --------------------------------------------------------------

__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

__device__ __forceinline__ void bf16x8_to_f32(const uint4& u, float f[8]) {
  f[0] = bf16lo(u.x); f[1] = bf16hi(u.x);
  f[2] = bf16lo(u.y); f[3] = bf16hi(u.y);
  f[4] = bf16lo(u.z); f[5] = bf16hi(u.z);
  f[6] = bf16lo(u.w); f[7] = bf16hi(u.w);
}

// fp32 -> bf16 word, round to nearest even, with exactly the integer
// operations of the reference packer (sw/attn_driver.py:88-98): the carry is
// added to the whole 32-bit word, so NaN/Inf patterns behave identically.
__device__ __forceinline__ uint32_t f32_to_bf16_rne_bits(float x) {
  const uint32_t bits = __float_as_uint(x);
  const uint32_t low = bits & 0xFFFFu;
  const uint32_t round_up = ((low >> 15) & 1u) & (((bits >> 16) & 1u) | ((low & 0x7FFFu) != 0u ? 1u : 0u));
  return ((bits + round_up) & 0xFFFF0000u) >> 16;
}

__device__ __forceinline__ uint32_t pack2_bf16(float lo, float hi) {
  return f32_to_bf16_rne_bits(lo) | (f32_to_bf16_rne_bits(hi) << 16);
}

__device__ __forceinline__ void bf16x4_to_f32(const uint2& u, float f[4]) {
  f[0] = bf16lo(u.x); f[1] = bf16hi(u.x);
  f[2] = bf16lo(u.y); f[3] = bf16hi(u.y);
}

// VEC bf16 words -> VEC/2 fp32 pairs (element 2i in .x, 2i+1 in .y)
template <int VEC>
__device__ __forceinline__ void load_bf16_pairs(const uint16_t* p, float2 f[VEC / 2]) {
  if constexpr (VEC == 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    f[0] = make_float2(bf16lo(u.x), bf16hi(u.x));
    f[1] = make_float2(bf16lo(u.y), bf16hi(u.y));
    f[2] = make_float2(bf16lo(u.z), bf16hi(u.z));
    f[3] = make_float2(bf16lo(u.w), bf16hi(u.w));
  } else {
    static_assert(VEC == 4, "VEC must be 4 or 8");
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    f[0] = make_float2(bf16lo(u.x), bf16hi(u.x));
    f[1] = make_float2(bf16lo(u.y), bf16hi(u.y));
  }
}

// VEC (4 or 8) bf16 words -> fp32
template <int VEC>
__device__ __forceinline__ void load_bf16_vec(const uint16_t* p, float f[VEC]) {
  if constexpr (VEC == 8) {
    bf16x8_to_f32(*reinterpret_cast<const uint4*>(p), f);
  } else {
    static_assert(VEC == 4, "VEC must be 4 or 8");
    bf16x4_to_f32(*reinterpret_cast<const uint2*>(p), f);
  }
}

}  // namespace lara
