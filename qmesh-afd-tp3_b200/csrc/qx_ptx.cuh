// Inline-PTX helpers for sm_100a: mbarriers, bulk async copies (TMA engine),
// proxy fences, acquire/release atomics, e2m1/e4m3 converts and the
// mixed-precision FMA. Every bulk copy here lands in the issuing CTA only.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace qx {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- mbarrier ---------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{ .reg .b64 st; mbarrier.arrive.release.cta.shared::cta.b64 st, [%0]; }" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{ .reg .b64 st; mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 st, [%0], %1; }" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: true when the phase completed; false when the deadline passed
// or another thread already raised `abort_bit` in *status (then the caller must
// stop consuming). Never spins without limit. The deadline is checked on the
// clock; *status lives in global memory (an L2 round trip that the waiting
// thread cannot overlap), so it is read only every 1024 failed tries, which a
// wait reaches only when something has already gone wrong.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, volatile uint32_t* status,
                                                  uint32_t abort_bit, uint64_t deadline_ns) {
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 15u) == 15u) {
      if (globaltimer_ns() > deadline_ns) {
        atomicOr(const_cast<uint32_t*>(status), abort_bit);
        return false;
      }
      if ((it & 1023u) == 1023u && (*status & abort_bit)) return false;
    }
  }
}

// ---- bulk async copy global -> shared (TMA engine, no tensor map) ------------
// dst, src 16-byte aligned, bytes a multiple of 16. Completion is signalled on
// `bar` as transaction bytes. CTA-local destination.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Orders this thread's earlier generic-proxy view of global memory before its
// later async-proxy (bulk copy) accesses.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ---- acquire / release on global counters -----------------------------------
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// Fire-and-forget add with release semantics (no value returned, no wait).
__device__ __forceinline__ void red_add_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// ---- programmatic dependent launch --------------------------------------------
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---- NVFP4 / FP8 converts -----------------------------------------------------
// One code byte (two e2m1 nibbles, low nibble = even element) -> f16x2 (even in
// the low half). Exact: every e2m1 value is an f16.
__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t byte) {
  uint32_t r;
  asm("{ .reg .b8 b; cvt.u8.u32 b, %1; cvt.rn.f16x2.e2m1x2 %0, b; }" : "=r"(r) : "r"(byte));
  return r;
}

// Two e4m3 bytes (low byte first) -> f16x2. Exact.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t two) {
  uint32_t r;
  asm("{ .reg .b16 b; cvt.u16.u32 b, %1; cvt.rn.f16x2.e4m3x2 %0, b; }" : "=r"(r) : "r"(two));
  return r;
}

__device__ __forceinline__ float f16lo_to_f32(uint32_t h2) {
  float f;
  asm("{ .reg .b16 lo, hi; mov.b32 {lo, hi}, %1; cvt.f32.f16 %0, lo; }" : "=f"(f) : "r"(h2));
  return f;
}
__device__ __forceinline__ float f16hi_to_f32(uint32_t h2) {
  float f;
  asm("{ .reg .b16 lo, hi; mov.b32 {lo, hi}, %1; cvt.f32.f16 %0, hi; }" : "=f"(f) : "r"(h2));
  return f;
}

// acc + lo(a)*lo(b) + hi(a)*hi(b), f16 operands, FP32 accumulate. Each product
// of two f16 values is exact in FP32, so this equals two FP32 FMAs on the
// widened operands.
__device__ __forceinline__ float fma2_f16_f32(uint32_t a, uint32_t b, float acc) {
  float d;
  asm("{ .reg .b16 al, ah, bl, bh; .reg .f32 t;\n\t"
      "mov.b32 {al, ah}, %1; mov.b32 {bl, bh}, %2;\n\t"
      "fma.rn.f32.f16 t, al, bl, %3;\n\t"
      "fma.rn.f32.f16 %0, ah, bh, t; }"
      : "=f"(d)
      : "r"(a), "r"(b), "f"(acc));
  return d;
}

}  // namespace qx
