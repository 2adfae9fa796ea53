// One-shot rank-ordered combine of per-rank BF16 partials over peer memory
// (NVLink / NVSwitch), replacing the reference's RDMA seam: every rank's
// partial reaches the output rank, which sums them in FP32 in rank order with
// one BF16 rounding (native/qmesh_afd_seam.cu:309-361 seam_combine_kernel; the
// fixed NODE-A, NODE-B, NODE-C, shared order of README.md:88-90).
//
// Each rank owns one exchange buffer (layout in qx_xchg.cuh).
// One CTA per chunk of the [rows, 5120] partial. A sender's CTA waits until its
// slot's previous use is acknowledged, stores its chunk straight into the output
// rank's slot with plain 16-byte stores and, after a barrier, one thread fences
// at system scope and releases the chunk's flag. The output rank's CTA acquires every sender's flag for its chunk,
// sums in rank order (its own partial from local memory) and acknowledges. No
// bulk-copy or tensor-memory-access instruction touches peer memory, and nothing
// here maps memory for in-switch reduction. Every wait is bounded
// (QX_TIMEOUT_MS): on expiry the CTA records QX_DEV_TIMEOUT and returns.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "qmesh_b200.h"
#include "qx_ptx.cuh"
#include "qx_xchg.cuh"

namespace qx {
namespace xchg {

using namespace xb;
constexpr int HID = QX_HIDDEN;
constexpr int THR = 256;       // threads per chunk CTA (NCH CTAs per call)

struct Args {
  uint8_t* buf[MAXW];          // every rank's exchange buffer (own included), in this address space
  const __nv_bfloat16* part;   // this rank's partial [rows][part_stride]
  int64_t part_stride;
  const __nv_bfloat16* shared; // optional, output rank only: added after the ranks
  int64_t shared_stride;
  __nv_bfloat16* out;          // output rank only
  int64_t out_stride;
  uint32_t* status;
  int rank, world, dst, rows, rows_max;
  uint64_t timeout_ns;
};

__device__ __forceinline__ void add8(float (&s)[8], uint4 v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    s[2 * i] += __uint_as_float(w[i] << 16);
    s[2 * i + 1] += __uint_as_float(w[i] & 0xffff0000u);
  }
}

__global__ void __launch_bounds__(THR) xchg_kernel(Args a) {
  __shared__ uint32_t s_call;
  __shared__ int s_ok;
  const int c = blockIdx.x, t = threadIdx.x;
  Hdr* me = reinterpret_cast<Hdr*>(a.buf[a.rank]);
  const int n8 = a.rows * (HID / 8);                 // 16-byte units of the partial
  const int u0 = (int)((int64_t)c * n8 / NCH), u1 = (int)((int64_t)(c + 1) * n8 / NCH);
  const uint64_t deadline = globaltimer_ns() + a.timeout_ns;
  if (t == 0) s_call = me->seq[c] + 1u;
  __syncthreads();
  const uint32_t call = s_call;
  if (a.rank != a.dst) {
    // The slot (call & 1) was last used by call - 2: wait for its acknowledgement.
    if (t == 0) s_ok = call <= 2u || wait_at_least(&me->ack[c], call - 2u, a.status, deadline);
    __syncwarp();   // warp 0 reconverges after lane 0's wait: one arrival per warp
    __syncthreads();
    if (!s_ok) return;
    __nv_bfloat16* dst = slot_of(a.buf[a.dst], call, a.rank, a.rows_max);
    for (int u = u0 + t; u < u1; u += THR) {
      const int row = u / (HID / 8), k = (u - row * (HID / 8)) * 8;
      const uint4 v = *reinterpret_cast<const uint4*>(a.part + (size_t)row * a.part_stride + k);
      *reinterpret_cast<uint4*>(dst + (size_t)row * HID + k) = v;
    }
    __syncthreads();   // the CTA's stores, then one system-scope fence and release
    if (t == 0) {
      fence_acq_rel_sys();
      st_release_sys(&reinterpret_cast<Hdr*>(a.buf[a.dst])->flag[a.rank][c], call);
      me->seq[c] = call;
    }
    return;
  }
  // Output rank: every sender's chunk (thread r waits for sender r), then the
  // rank-ordered sum.
  if (t == 0) s_ok = 1;
  __syncthreads();
  if (t < a.world && t != a.dst && !wait_at_least(&me->flag[t][c], call, a.status, deadline)) s_ok = 0;
  __syncwarp();
  __syncthreads();
  if (!s_ok) return;
  for (int u = u0 + t; u < u1; u += THR) {
    const int row = u / (HID / 8), k = (u - row * (HID / 8)) * 8;
    float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int r = 0; r < a.world; ++r) {
      const uint4 v = r == a.dst
                          ? *reinterpret_cast<const uint4*>(a.part + (size_t)row * a.part_stride + k)
                          : __ldcg(reinterpret_cast<const uint4*>(slot_of(a.buf[a.dst], call, r, a.rows_max) +
                                                                  (size_t)row * HID + k));
      add8(s, v);
    }
    if (a.shared) add8(s, *reinterpret_cast<const uint4*>(a.shared + (size_t)row * a.shared_stride + k));
    uint4 o;
    uint32_t* ow = &o.x;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_bfloat162 b = __floats2bfloat162_rn(s[2 * i], s[2 * i + 1]);
      ow[i] = *reinterpret_cast<const uint32_t*>(&b);
    }
    *reinterpret_cast<uint4*>(a.out + (size_t)row * a.out_stride + k) = o;
  }
  __syncthreads();   // every slot read above has returned its value
  if (t < a.world && t != a.dst) ack_after_reads(&reinterpret_cast<Hdr*>(a.buf[t])->ack[c], call);
  if (t == 0) me->seq[c] = call;
}

static uint64_t timeout_ns() {
  const char* e = getenv("QX_TIMEOUT_MS");
  long ms = e ? atol(e) : 1000;
  if (ms < 10) ms = 10;
  return (uint64_t)ms * 1000000ull;
}

}  // namespace xchg
}  // namespace qx

using namespace qx::xchg;

extern "C" {

size_t qx_xchg_bytes(int32_t rows_max) {
  if (rows_max < 1 || rows_max > QX_MAX_ROWS) return 0;
  return HDR_BYTES + slots_bytes(rows_max) + words_bytes(rows_max);
}

int qx_xchg_alloc(int32_t rows_max, void** buf) {
  if (!buf) return QX_ERR_ARG;
  *buf = nullptr;
  const size_t n = qx_xchg_bytes(rows_max);
  if (!n) return QX_ERR_SHAPE;
  void* p = nullptr;
  if (cudaMalloc(&p, n) != cudaSuccess) return QX_ERR_DEVICE;
  if (cudaMemset(p, 0, n) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(p);
    return QX_ERR_DEVICE;
  }
  *buf = p;
  return QX_OK;
}

int qx_xchg_free(void* buf) {
  if (!buf) return QX_ERR_ARG;
  return cudaFree(buf) == cudaSuccess ? QX_OK : QX_ERR_DEVICE;
}

int qx_ipc_handle(const void* buf, void* handle) {
  if (!buf || !handle) return QX_ERR_ARG;
  static_assert(sizeof(cudaIpcMemHandle_t) == QX_IPC_HANDLE_BYTES, "IPC handle size");
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(buf)) != cudaSuccess) return QX_ERR_DEVICE;
  memcpy(handle, &h, sizeof(h));
  return QX_OK;
}

int qx_ipc_open(const void* handle, void** buf) {
  if (!handle || !buf) return QX_ERR_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  *buf = nullptr;
  if (cudaIpcOpenMemHandle(buf, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return QX_ERR_DEVICE;
  return QX_OK;
}

int qx_ipc_close(void* buf) {
  if (!buf) return QX_ERR_ARG;
  return cudaIpcCloseMemHandle(buf) == cudaSuccess ? QX_OK : QX_ERR_DEVICE;
}

int qx_combine_p2p(const QxXchgArgs* x, void* stream) {
  if (!x || !x->part || !x->status) return QX_ERR_ARG;
  if (x->world < 1 || x->world > MAXW || x->rank < 0 || x->rank >= x->world || x->dst < 0 || x->dst >= x->world)
    return QX_ERR_ARG;
  if (x->rows < 1 || x->rows > x->rows_max || x->rows_max > QX_MAX_ROWS) return QX_ERR_SHAPE;
  for (int r = 0; r < x->world; ++r)
    if (!x->bufs[r] || (reinterpret_cast<uintptr_t>(x->bufs[r]) & 255u)) return QX_ERR_ARG;
  if (x->rank == x->dst && !x->out) return QX_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(x->part) & 15u) || (x->part_stride & 7) || x->part_stride < HID)
    return QX_ERR_ALIGN;
  if (x->out && ((reinterpret_cast<uintptr_t>(x->out) & 15u) || (x->out_stride & 7) || x->out_stride < HID))
    return QX_ERR_ALIGN;
  if (x->shared && ((reinterpret_cast<uintptr_t>(x->shared) & 15u) || (x->shared_stride & 7) ||
                    x->shared_stride < HID))
    return QX_ERR_ALIGN;
  Args a = {};
  for (int r = 0; r < x->world; ++r) a.buf[r] = reinterpret_cast<uint8_t*>(x->bufs[r]);
  a.part = reinterpret_cast<const __nv_bfloat16*>(x->part);
  a.part_stride = x->part_stride;
  a.shared = reinterpret_cast<const __nv_bfloat16*>(x->shared);
  a.shared_stride = x->shared_stride;
  a.out = reinterpret_cast<__nv_bfloat16*>(x->out);
  a.out_stride = x->out_stride;
  a.status = reinterpret_cast<uint32_t*>(x->status);
  a.rank = x->rank;
  a.world = x->world;
  a.dst = x->dst;
  a.rows = x->rows;
  a.rows_max = x->rows_max;
  a.timeout_ns = timeout_ns();
  xchg_kernel<<<NCH, THR, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return cudaGetLastError() == cudaSuccess ? QX_OK : QX_ERR_LAUNCH;
}

}  // extern "C"
