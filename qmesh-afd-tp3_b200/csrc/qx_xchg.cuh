// Layout of a rank's exchange buffer and the peer-memory primitives of the
// rank-ordered combine (native/qmesh_afd_seam.cu:309-361), shared by the
// stand-alone combine kernel (qx_combine_p2p) and the decode kernel's fused
// combine (qx_slice_decode_tc_xchg).
//
// A buffer (cudaMalloc'd, mapped into the other ranks with CUDA IPC) is
//   header  chunk protocol of qx_combine_p2p:
//             flag[sender][chunk]  written by a sender into the output rank's
//                                  buffer: the call number whose chunk landed;
//             ack[chunk]           written by the output rank into each
//                                  sender's buffer: the last call it consumed;
//             seq[chunk]           this rank's own call counter;
//           unit protocol of the fused combine, the same three arrays per
//           finalize unit (output tile of 128 columns x block of 4 rows);
//   slots   [2][sender][rows_max][5120] BF16 receive slots, alternating by call
//           number, so a sender may run one call ahead of the output rank.
// A buffer serves one of the two protocols: their call counters are separate,
// so calls of both kinds must not interleave on one buffer.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

#include "qmesh_b200.h"
#include "qx_ptx.cuh"

namespace qx {
namespace xb {

constexpr int MAXW = QX_XCHG_MAX_RANKS;
constexpr int NCH = 64;                                 // chunks of qx_combine_p2p
constexpr int MAXU = (QX_HIDDEN / 128) * (QX_MAX_ROWS / 4);   // finalize units of the fused combine

struct Hdr {
  uint32_t flag[MAXW][NCH];
  uint32_t ack[NCH];
  uint32_t seq[NCH];
  uint32_t uflag[MAXW][MAXU];
  uint32_t uack[MAXU];
  uint32_t useq[MAXU];
};
constexpr size_t HDR_BYTES = (sizeof(Hdr) + 255) & ~size_t(255);

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// System-scope fence of one thread. A group's stores to peer memory are ordered
// before one thread's fence and release by a barrier over the group (release is
// cumulative): one fence per group instead of one per thread, which costs
// microseconds when every thread of a CTA fences at system scope.
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// Bounded wait until (int)(*p - need) >= 0; on expiry records QX_DEV_TIMEOUT.
__device__ inline bool wait_at_least(const uint32_t* p, uint32_t need, uint32_t* status, uint64_t deadline) {
  for (uint32_t it = 0;; ++it) {
    if ((int32_t)(ld_acquire_sys(p) - need) >= 0) return true;
    if ((it & 63u) == 63u && globaltimer_ns() > deadline) {
      atomicOr(status, (uint32_t)QX_DEV_TIMEOUT);
      return false;
    }
    if (it > 8) __nanosleep(32);
  }
}

__device__ __forceinline__ __nv_bfloat16* slot_of(uint8_t* buf, uint32_t call, int sender, int rows_max) {
  return reinterpret_cast<__nv_bfloat16*>(buf + HDR_BYTES) +
         ((size_t)(call & 1u) * MAXW + sender) * rows_max * QX_HIDDEN;
}

}  // namespace xb
}  // namespace qx
