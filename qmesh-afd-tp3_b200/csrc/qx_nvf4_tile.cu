// Self-check of the device's block-scaled NVFP4 tensor-core path: one
// 128 x n output tile over nkb 64-wide K blocks, operands in the K-major
// no-swizzle tile layout and 512-byte scale atoms of qx_tc.cuh, accumulated in
// TMEM by tcgen05.mma.kind::mxf4nvf4 and written out as FP32. The decode
// kernels use exactly these layouts, descriptors and instructions; this entry
// point lets a test (or an integrator) confirm them on a given GPU and driver
// against a CPU product.

#include <cuda_runtime.h>
#include <stdint.h>

#include "qmesh_b200.h"
#include "qx_ptx.cuh"
#include "qx_tc.cuh"

namespace qx {
namespace {

constexpr uint32_t A_KB = 128 * tc::ROWB + tc::SF_ATOM;  // 4608 bytes per K block of A
constexpr uint32_t TM_COLS = 512;
constexpr uint32_t TM_SFA = 256, TM_SFB = 288;           // scale columns: 4 per K block for A, 4 per atom for B

__global__ void __launch_bounds__(128, 1)
    nvf4_tile_kernel(const uint8_t* __restrict__ a, const uint8_t* __restrict__ b, int n, int nkb,
                     float* __restrict__ d, uint32_t* status, uint64_t timeout_ns) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t bar_load, bar_mma;
  __shared__ uint32_t tmem_base, grace_status;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t b_atoms = ((uint32_t)n + 127u) / 128u;
  const uint32_t b_kb = (uint32_t)n * tc::ROWB + b_atoms * tc::SF_ATOM;
  const uint32_t a_bytes = (uint32_t)nkb * A_KB, b_bytes = (uint32_t)nkb * b_kb;
  uint8_t* sa = smem;
  uint8_t* sb = smem + a_bytes;
  volatile uint32_t* vstatus = status;

  if (threadIdx.x == 0) {
    mbar_init(&bar_load, 1);
    mbar_init(&bar_mma, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(&tmem_base, TM_COLS);
    tc::tmem_relinquish();
  }
  __syncwarp();   // warp 0 reconverges after its lane 0's set-up: one arrival per warp
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = tmem_base;
  const uint64_t deadline = globaltimer_ns() + timeout_ns;

  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(&bar_load, a_bytes + b_bytes);
    bulk_g2s(sa, a, a_bytes, &bar_load);
    bulk_g2s(sb, b, b_bytes, &bar_load);
  }
  bool loaded = mbar_wait_bounded(&bar_load, 0, vstatus, QX_DEV_TIMEOUT, deadline);
  bool issued = false;
  if (threadIdx.x == 0 && loaded) {
    tc::fence_after_sync();
    const uint32_t idesc = tc::idesc_nvf4((uint32_t)n);
    for (int kb = 0; kb < nkb; ++kb) {
      const uint32_t sa_kb = smem_u32(sa + kb * A_KB), sb_kb = smem_u32(sb + kb * b_kb);
      const uint32_t tsfa = tbase + TM_SFA + 4 * kb, tsfb = tbase + TM_SFB + 4 * b_atoms * kb;
      tc::cp_sf_atom(tsfa, sa_kb + 128 * tc::ROWB);
      for (uint32_t at = 0; at < b_atoms; ++at)
        tc::cp_sf_atom(tsfb + 4 * at, sb_kb + (uint32_t)n * tc::ROWB + at * tc::SF_ATOM);
      tc::mma_nvf4(tbase, tc::sdesc(sa_kb, tc::LBO, tc::SBO), tc::sdesc(sb_kb, tc::LBO, tc::SBO), idesc, tsfa, tsfb,
                   kb > 0 ? 1u : 0u);
    }
    tc::commit(&bar_mma);
    issued = true;
  }
  bool done = mbar_wait_bounded(&bar_mma, 0, vstatus, QX_DEV_TIMEOUT, deadline);
  done = __all_sync(0xffffffffu, done) != 0;
  if (done) {
    tc::fence_after_sync();
    const uint32_t lanes = (uint32_t)(warp * 32) << 16;
    const int m = warp * 32 + lane;
    for (int c = 0; c < n; c += 16) {
      float v[16];
      tc::ld16(tbase + lanes + (uint32_t)c, v);
#pragma unroll
      for (int i = 0; i < 16; ++i) d[(size_t)m * n + c + i] = v[i];
    }
  }
  // After a timeout: let copies and tensor-core work already issued finish
  // (bounded again) before the shared memory and TMEM are released.
  if (threadIdx.x == 0) {
    const uint64_t grace = globaltimer_ns() + timeout_ns;
    grace_status = 0;
    if (!loaded) mbar_wait_bounded(&bar_load, 0, &grace_status, 1u, grace);
    if (issued && !done) mbar_wait_bounded(&bar_mma, 0, &grace_status, 1u, grace);
  }
  __syncwarp();
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tbase, TM_COLS);
}

}  // namespace
}  // namespace qx

extern "C" int qx_diag_nvf4_tile(const uint8_t* a, const uint8_t* b, int32_t n, int32_t nkb, float* d,
                                 uint32_t* status, void* stream) {
  if (!a || !b || !d || !status) return QX_ERR_ARG;
  if (n < 16 || n > 256 || (n % 16) != 0 || nkb < 1 || nkb > 8) return QX_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 15u) return QX_ERR_ALIGN;
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return QX_ERR_DEVICE;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess || major != 10)
    return QX_ERR_DEVICE;
  const size_t b_atoms = ((size_t)n + 127) / 128;
  const size_t smem = (size_t)nkb * qx::A_KB + (size_t)nkb * ((size_t)n * qx::tc::ROWB + b_atoms * qx::tc::SF_ATOM);
  if (cudaFuncSetAttribute(qx::nvf4_tile_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return QX_ERR_LAUNCH;
  const uint64_t timeout_ns = 1000ull * 1000ull * 1000ull;
  qx::nvf4_tile_kernel<<<1, 128, smem, static_cast<cudaStream_t>(stream)>>>(a, b, n, nkb, d, status, timeout_ns);
  return cudaGetLastError() == cudaSuccess ? QX_OK : QX_ERR_LAUNCH;
}
