// Producer side of the slice on the device: the FP8 activation quantisation the
// attention side applies before posting a layer's activations, and the routing
// front end (softmax, top-k, renormalisation) that produces the ids and weights.
//
// qx_quant_fp8 restates the reference seam's quantiser (native/qmesh_afd_seam.cu:
// 9-16 numerics, seam_amax_kernel :112-146, seam_finish :88-110, seam_pack_kernel
// :152-176), with the per-row scale the slice interface also accepts:
//   m   = max |x| (bf16 values, integer max of the FP32 bit patterns)
//   mc  = max(m, bf16(1e-6));  s = (float)(448 / (double)mc);  inv = (float)(1 / (448 / (double)mc))
//   q   = e4m3_rne_satfinite(clamp(bf16_rn(x * s), +-448))
// over each row (per_post = 0) or over all rows of the post (per_post = 1, the
// reference's form). A non-finite maximum leaves that row's (post's) bytes
// unwritten, sets inv = 1 and records QX_DEV_NONFINITE, as the seam skips its
// pack and counts the post.
//
// qx_route_topk: p = softmax(logits) in FP32, the top-k probabilities (largest
// first, the lower expert id first among equal values), w = p / sum(p_topk),
// one warp per row. The reference receives these from vLLM's router and ships
// them in the routing window (afd_session.py:211-252).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <limits.h>
#include <math.h>
#include <stdint.h>

#include "qmesh_b200.h"

namespace qx {
namespace front {

constexpr int HID = QX_HIDDEN;
constexpr int THR = 256;
constexpr uint32_t INF_BITS = 0x7f800000u;
constexpr float BF16_FLOOR = 9.98377799987793e-07f;   // bf16(1e-6)

__device__ __forceinline__ uint32_t row_amax_bits(const __nv_bfloat16* xr) {
  uint32_t m = 0;
  for (int k = threadIdx.x * 8; k < HID; k += THR * 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + k);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      m = max(m, (w[i] << 16) & 0x7fffffffu);
      m = max(m, w[i] & 0x7fff0000u);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ uint32_t sm[THR / 32];
  if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = m;
  __syncthreads();
  uint32_t r = 0;
#pragma unroll
  for (int i = 0; i < THR / 32; ++i) r = max(r, sm[i]);
  __syncthreads();
  return r;
}

__device__ __forceinline__ uint32_t e4m3x2_rn(float lo, float hi) {
  uint32_t two;
  asm("{ .reg .b16 h; cvt.rn.satfinite.e4m3x2.f32 h, %1, %2; cvt.u32.u16 %0, h; }" : "=r"(two) : "f"(hi), "f"(lo));
  return two & 0xFFFFu;
}

__device__ __forceinline__ float quant_in(float v, float s) {
  const float y = __bfloat162float(__float2bfloat16_rn(__fmul_rn(v, s)));
  return fminf(fmaxf(y, -448.f), 448.f);
}

__device__ void pack_row(const __nv_bfloat16* xr, uint8_t* qr, float s) {
  for (int k = threadIdx.x * 8; k < HID; k += THR * 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + k);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[2] = {0u, 0u};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float lo = __uint_as_float(w[i] << 16), hi = __uint_as_float(w[i] & 0xffff0000u);
      o[i >> 1] |= e4m3x2_rn(quant_in(lo, s), quant_in(hi, s)) << (16 * (i & 1));
    }
    *reinterpret_cast<uint2*>(qr + k) = make_uint2(o[0], o[1]);
  }
}

__device__ __forceinline__ void finish(uint32_t bits, float* s, float* inv) {
  const float mc = fmaxf(__uint_as_float(bits), BF16_FLOOR);
  const double sd = 448.0 / (double)mc;
  *s = (float)sd;
  *inv = (float)(1.0 / sd);
}

// per row: one CTA per row
__global__ void __launch_bounds__(THR) quant_rows_kernel(const __nv_bfloat16* x, int64_t xs, uint8_t* q, int64_t qs,
                                                         float* inv, uint32_t* status) {
  const int r = blockIdx.x;
  const __nv_bfloat16* xr = x + (size_t)r * xs;
  const uint32_t bits = row_amax_bits(xr);
  if (bits >= INF_BITS) {
    if (threadIdx.x == 0) {
      inv[r] = 1.f;
      atomicOr(status, (uint32_t)QX_DEV_NONFINITE);
    }
    return;
  }
  float s, iv;
  finish(bits, &s, &iv);
  if (threadIdx.x == 0) inv[r] = iv;
  pack_row(xr, q + (size_t)r * qs, s);
}

// per post: the maximum over all rows (integer atomicMax into work[0], zeroed by
// the host launch sequence), then the pack with the post's one scale.
__global__ void __launch_bounds__(THR) post_amax_kernel(const __nv_bfloat16* x, int64_t xs, uint32_t* work) {
  const uint32_t bits = row_amax_bits(x + (size_t)blockIdx.x * xs);
  if (threadIdx.x == 0) atomicMax(work, bits);
}

__global__ void __launch_bounds__(THR) post_pack_kernel(const __nv_bfloat16* x, int64_t xs, uint8_t* q, int64_t qs,
                                                        const uint32_t* work, float* inv, uint32_t* status) {
  const uint32_t bits = *work;
  if (bits >= INF_BITS) {
    if (blockIdx.x == 0 && threadIdx.x == 0) {
      inv[0] = 1.f;
      atomicOr(status, (uint32_t)QX_DEV_NONFINITE);
    }
    return;
  }
  float s, iv;
  finish(bits, &s, &iv);
  if (blockIdx.x == 0 && threadIdx.x == 0) inv[0] = iv;
  pack_row(x + (size_t)blockIdx.x * xs, q + (size_t)blockIdx.x * qs, s);
}

// Routing: one warp per row. Selection order: larger probability first, then
// the lower expert id.
__global__ void __launch_bounds__(THR) route_kernel(const float* logits, int64_t ls, int rows, int E, int topk,
                                                    int32_t* ids, float* tw) {
  const int row = blockIdx.x * (THR / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* lr = logits + (size_t)row * ls;
  float mx = -INFINITY;
  for (int e = lane; e < E; e += 32) mx = fmaxf(mx, lr[e]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
  for (int e = lane; e < E; e += 32) sum += expf(lr[e] - mx);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  int prev_e = -1;
  float prev_p = INFINITY;
  float selp[QX_MAX_TOPK];
  int sele[QX_MAX_TOPK];
  float tot = 0.f;
  for (int j = 0; j < topk; ++j) {
    // the best (p, e) strictly after (prev_p, prev_e) in the selection order
    float bp = -1.f;
    int be = INT_MAX;
    for (int e = lane; e < E; e += 32) {
      const float p = expf(lr[e] - mx) / sum;
      const bool after = p < prev_p || (p == prev_p && e > prev_e);
      if (after && (p > bp || (p == bp && e < be))) {
        bp = p;
        be = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float op = __shfl_xor_sync(0xffffffffu, bp, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (op > bp || (op == bp && oe < be)) {
        bp = op;
        be = oe;
      }
    }
    selp[j] = bp;
    sele[j] = be;
    tot += bp;
    prev_p = bp;
    prev_e = be;
  }
  if (lane < topk) {
    float p = 0.f;
    int e = 0;
#pragma unroll
    for (int j = 0; j < QX_MAX_TOPK; ++j)
      if (j == lane) {
        p = selp[j];
        e = sele[j];
      }
    ids[(size_t)row * topk + lane] = e;
    tw[(size_t)row * topk + lane] = p / tot;
  }
}

// Round driver support: one thread waits until the sequence cell (host-mapped
// or device memory, written by whoever publishes the layer's inputs) reaches
// *need_p (read at run time, so a captured graph serves every round), or the
// time limit passes; then records QX_DEV_TIMEOUT and returns, so the stream
// (and a captured round graph) always moves on.
__global__ void wait_cell_kernel(const uint32_t* cell, const uint32_t* need_p, uint64_t timeout_ns, uint32_t* status) {
  const uint32_t need = *need_p;
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (uint32_t it = 0;; ++it) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(cell) : "memory");
    if ((int32_t)(v - need) >= 0) return;
    if ((it & 31u) == 31u) {
      uint64_t t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (t - t0 > timeout_ns) {
        atomicOr(status, (uint32_t)QX_DEV_TIMEOUT);
        return;
      }
    }
    __nanosleep(256);
  }
}

}  // namespace front
}  // namespace qx

using namespace qx::front;

extern "C" {

int qx_quant_fp8(const void* x, int64_t x_stride, int32_t rows, int32_t per_post, void* q, int64_t q_stride,
                 float* inv, uint32_t* work, uint32_t* status, void* stream) {
  if (!x || !q || !inv || !status || (per_post && !work)) return QX_ERR_ARG;
  if (rows < 1 || x_stride < HID || q_stride < HID) return QX_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(x) & 15u) || (x_stride & 7) || (reinterpret_cast<uintptr_t>(q) & 7u) ||
      (q_stride & 7))
    return QX_ERR_ALIGN;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(x);
  uint8_t* qb = reinterpret_cast<uint8_t*>(q);
  if (!per_post) {
    quant_rows_kernel<<<rows, THR, 0, st>>>(xb, x_stride, qb, q_stride, inv, status);
  } else {
    if (cudaMemsetAsync(work, 0, sizeof(uint32_t), st) != cudaSuccess) return QX_ERR_LAUNCH;
    post_amax_kernel<<<rows, THR, 0, st>>>(xb, x_stride, work);
    post_pack_kernel<<<rows, THR, 0, st>>>(xb, x_stride, qb, q_stride, work, inv, status);
  }
  return cudaGetLastError() == cudaSuccess ? QX_OK : QX_ERR_LAUNCH;
}

int qx_wait_cell(const uint32_t* cell, const uint32_t* need, uint64_t timeout_ns, uint32_t* status, void* stream) {
  if (!cell || !need || !status || timeout_ns == 0) return QX_ERR_ARG;
  wait_cell_kernel<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(cell, need, timeout_ns, status);
  return cudaGetLastError() == cudaSuccess ? QX_OK : QX_ERR_LAUNCH;
}

int qx_route_topk(const float* logits, int64_t logits_stride, int32_t rows, int32_t n_experts, int32_t topk,
                  int32_t* ids, float* tw, void* stream) {
  if (!logits || !ids || !tw) return QX_ERR_ARG;
  if (rows < 1 || n_experts < 1 || topk < 1 || topk > QX_MAX_TOPK || topk > n_experts ||
      logits_stride < n_experts)
    return QX_ERR_SHAPE;
  const int per = THR / 32;
  route_kernel<<<(rows + per - 1) / per, THR, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      logits, logits_stride, rows, n_experts, topk, ids, tw);
  return cudaGetLastError() == cudaSuccess ? QX_OK : QX_ERR_LAUNCH;
}

}  // extern "C"
