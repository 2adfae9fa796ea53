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
//           unit protocol of the fused combine, per finalize unit (output
//           tile of 128 columns x block of 4 rows): ack and seq as above;
//   slots   [2][sender][rows_max][5120] BF16 receive slots of the chunk
//           protocol, alternating by call number, so a sender may run one
//           call ahead of the output rank;
//   words   [2][sender][rows_max][5120 / 4][2] 64-bit receive words of the unit
//           protocol: each holds 4 bytes of BF16 data and, above them, the
//           call number that wrote them, so a word validates itself and the
//           sender needs no fence or flag (the receiver polls the words).
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
// A receiver's acknowledgement that it has read a sender's slot, so the sender
// may overwrite it (two calls later). Issued by one thread after a barrier that
// every reading thread reaches only once its loads of the slot have returned:
// their values feed the sum that thread stored before the barrier. A store
// cannot be seen by the sender before loads that have already returned, so the
// acknowledgement is a relaxed system-scope store, not a release: a release at
// system scope also waits until every earlier store of the thread (the output
// rows) is visible to the whole system, which measured 7.5 us per call at two
// ranks. Should an overwrite ever land first, the receiver would see the words'
// newer call number and run into its bounded wait (an error, not a wrong sum).
__device__ __forceinline__ void ack_after_reads(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
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

__host__ __device__ inline size_t slots_bytes(int rows_max) {
  return (size_t)2 * MAXW * rows_max * QX_HIDDEN * sizeof(uint16_t);
}
__host__ __device__ inline size_t words_bytes(int rows_max) {
  return (size_t)2 * MAXW * rows_max * (QX_HIDDEN / 4) * 2 * sizeof(uint64_t);
}

__device__ __forceinline__ __nv_bfloat16* slot_of(uint8_t* buf, uint32_t call, int sender, int rows_max) {
  return reinterpret_cast<__nv_bfloat16*>(buf + HDR_BYTES) +
         ((size_t)(call & 1u) * MAXW + sender) * rows_max * QX_HIDDEN;
}

// The two receive words of (sender, row, columns k..k+3) for a call's parity.
__device__ __forceinline__ uint64_t* words_of(uint8_t* buf, uint32_t call, int sender, int rows_max, int row,
                                              int k) {
  return reinterpret_cast<uint64_t*>(buf + HDR_BYTES + slots_bytes(rows_max)) +
         ((((size_t)(call & 1u) * MAXW + sender) * rows_max + row) * (QX_HIDDEN / 4) + k / 4) * 2;
}

__device__ __forceinline__ void st_relaxed_sys_b64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_b64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until both receive words carry `call`; their data in v.
__device__ inline bool words_wait(const uint64_t* w, uint32_t call, uint2& v, uint32_t* status, uint64_t deadline) {
  for (uint32_t it = 0;; ++it) {
    const uint64_t a = ld_relaxed_sys_b64(w), b = ld_relaxed_sys_b64(w + 1);
    if ((uint32_t)(a >> 32) == call && (uint32_t)(b >> 32) == call) {
      v = make_uint2((uint32_t)a, (uint32_t)b);
      return true;
    }
    if ((it & 63u) == 63u && globaltimer_ns() > deadline) {
      atomicOr(status, (uint32_t)QX_DEV_TIMEOUT);
      return false;
    }
    if (it > 8) __nanosleep(32);
  }
}

}  // namespace xb
}  // namespace qx
