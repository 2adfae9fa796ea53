// Routed-expert NVFP4 SwiGLU slice for prefill-sized batches (W4A4) on the
// 5th-generation tensor cores of B200 (sm_100a): a grouped block-scaled GEMM
// with `tcgen05.mma.kind::mxf4nvf4` in which both operands are NVFP4 (the arena's
// weights as stored, the activations quantised on the device) and the
// accumulators live in TMEM.
//
// Numerics of the reference's prefill body (gx/gx_ingest.py:190-246, the clamped
// split CUTLASS form): x (the reference's bf16 ingest of the FP8 rows) is
// quantised to NVFP4 with a1g = bf16(6 / max|x|); c1 = bf16((g13 / a1g) x.W13);
// c2 = bf16(silu(min(g, L)) clamp(u, -L, L)); c2 is quantised to NVFP4 with the
// calibrated a2; c3 = bf16((g2 / a2) c2.W2); out = bf16(sum_j bf16(c3_j tw_j)).
// The NVFP4 activation quantiser is vLLM's (`ref_nvfp4_quant`): per 16 elements
// scale = e4m3(min(gs (amax f32(1/6)), 448)), code = e2m1_rne(v / (scale / gs))
// with correctly rounded reciprocals, reproduced bit for bit.
//
// Kernels (stream order):
//   pf_prep_kernel     one CTA per row: max|x| (for a1g) and the routed pairs per
//                      expert (atomic counts);
//   pf_route_kernel    one CTA: expert offsets, groups of <= 96 pairs of one
//                      expert, each group's operand offsets and scales;
//   pf_place_kernel    each pair's position in its expert's range (any order:
//                      a pair's result does not depend on its neighbours);
//   pf_xquant_kernel   one CTA per token row: the row's NVFP4 codes and scales,
//                      quantised once, written straight into the B operand of
//                      each of the row's routed pairs (MMA layout);
//   pf_main_kernel     persistent, one CTA per SM: items gate/up (group,
//                      64-column tile) then down (group, 128-row tile), the same
//                      producer / two MMA issuers / two epilogue warpgroups
//                      pipeline as the decode kernel; both operands' block
//                      scales are copied to TMEM per K block;
//   pf_finalize_kernel out[t] = bf16(sum over slots j in order of y[t, j]).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <limits.h>
#include <stdint.h>
#include <stdlib.h>

#include "qmesh_b200.h"
#include "qx_ptx.cuh"
#include "qx_tc.cuh"

namespace qx {
namespace pf {

constexpr int HID = QX_HIDDEN;
constexpr int KB1 = HID / 64;                  // 80 K blocks of a gate/up item
constexpr int SK = 8;                          // K blocks per stage
constexpr int A_KB = 128 * tc::ROWB + tc::SF_ATOM;   // 4608
constexpr int A_STAGE = SK * A_KB;             // 36864
constexpr int HT = HID / 128;                  // 40 output-row tiles
constexpr int GP = 96;                         // pairs per group at most (accumulator N <= 96)
constexpr int MAXNS = 8;
constexpr int NI = MAXNS + 2;
static_assert(NI % 2 == 0, "epilogue groups alternate meta entries");
constexpr int NTHR = 352;                      // producer, issuers (1, 6), epilogue warps 2-5 and 7-10
constexpr int NEPI = 2;
constexpr int NISS = 2, KB_PER_ISS = SK / NISS;
constexpr int MAXE = 1024;                     // experts the routing kernel handles
constexpr int RT_THR = 1024;
constexpr int XQ_THR = HID / 16;               // 320: one 16-element block per thread
// TMEM: accumulator (buffer b, issuer i) at 256 b + 128 i (96 columns); in the
// four 32-column gaps the scale banks, bank k of issuer i at 96 + 128 (2k + i):
// weight atoms of the stage's 4 K blocks at +0..+15, activation atoms at +16..+31
// (4 columns each, 4-aligned as block-scaled MMAs require).
constexpr uint32_t TM_COLS = 512, TM_SLOT = 128;
__host__ __device__ constexpr uint32_t tm_bank(int iss, int k) { return 96u + 128u * (uint32_t)(2 * k + iss); }

struct Ctl {
  uint32_t work, status, amax_bits, n_groups, n1, n2, b_max, n_valid;
  float a1g;
  uint32_t pad[55];
};
static_assert(sizeof(Ctl) == 256, "ctl block is 256 bytes");

struct Group {      // one group of <= GP routed pairs of one expert
  int32_t expert, gsz, npad, pos_off;
  int32_t sbs, pad0;  // B-operand bytes per stage: npad x 256 codes + 8 x 512 scale atoms
  int64_t xq_off, ab_off;
  float alpha1, alpha2;   // g13 / a1g, g2 / a2
  int32_t pad1[4];
};
static_assert(sizeof(Group) == 64, "group record is 64 bytes");

struct Params {
  const void* x;
  const float* x_scale;
  int64_t x_stride;
  int x_fmt;
  const void* ids;
  int ids64;
  const float* tw;
  const float* a2;
  int rows, topk, P, E;
  int W, NT, tile0, NTA;
  const uint8_t* w13;
  const uint8_t* w2;
  const float* g13;
  const float* g2;
  float limit;
  int has_limit;
  __nv_bfloat16* out;
  int64_t out_stride;
  Ctl* ctl;
  uint32_t* cnt;      // [E] routed pairs per expert
  uint32_t* fill;     // [E] placement counters
  uint32_t* off;      // [E] first position of the expert's pairs
  Group* groups;      // [gmax]
  int32_t* grp_of_pos;// [P] group of a position
  int32_t* pos_pair;  // [P] pair at a position
  int32_t* pos_of;    // [P] position of a pair (routed pairs only)
  uint32_t* cnt1;     // [gmax] gate/up tiles finished per group
  uint8_t* xq;        // per group: 10 stages of sbs bytes
  uint8_t* ab;        // per group: ceil(NT/8) stages of sbs bytes
  __nv_bfloat16* y;   // [P][HID]
  int gmax;
  int x_off, ring_off, ring_bytes;
  int ns, bst, b_off;
  uint64_t timeout_ns;
};

struct ItemMeta {
  int32_t kind, group, tile, nst, nkb_last, n, gsz, pos_off;
  float alpha;
  int32_t pad[3];
};

__host__ __device__ inline size_t al256(size_t v) { return (v + 255) & ~size_t(255); }
__host__ __device__ inline int npad_of(int gsz) { return (gsz + 15) & ~15; }
__host__ __device__ inline int sbs_of(int npad) { return npad * 256 + SK * tc::SF_ATOM; }

// Upper bound of the groups of a call: each expert's pairs split into
// ceil(cnt / GP) groups, so at most P / GP + min(E, P).
__host__ __device__ inline int groups_bound(int P, int E) { return P / GP + (E < P ? E : P) + 1; }

struct WsLayout {
  size_t ctl, cnt, fill, off, groups, grp_of_pos, pos_pair, pos_of, cnt1, xq, ab, y, total;
};

__host__ inline WsLayout ws_layout(int rows, int topk, int W, int E) {
  WsLayout L;
  const int P = rows * topk, NT = (W + 63) / 64, G = groups_bound(P, E);
  const size_t opnd = (size_t)256 * (P + 15 * (size_t)G) + (size_t)SK * tc::SF_ATOM * G;   // sum of sbs
  size_t o = 0;
  L.ctl = o;        o = al256(o + sizeof(Ctl));
  L.cnt = o;        o = al256(o + (size_t)E * 4);
  L.fill = o;       o = al256(o + (size_t)E * 4);
  L.off = o;        o = al256(o + (size_t)E * 4);
  L.groups = o;     o = al256(o + (size_t)G * sizeof(Group));
  L.grp_of_pos = o; o = al256(o + (size_t)P * 4);
  L.pos_pair = o;   o = al256(o + (size_t)P * 4);
  L.pos_of = o;     o = al256(o + (size_t)P * 4);
  L.cnt1 = o;       o = al256(o + (size_t)G * 4);
  L.xq = o;         o = al256(o + (size_t)(KB1 / SK) * opnd);
  L.ab = o;         o = al256(o + (size_t)((NT + SK - 1) / SK) * opnd);
  L.y = o;          o = al256(o + (size_t)P * HID * 2);
  L.total = o;
  return L;
}

__device__ __forceinline__ long long id_of(const Params& p, int q) {
  return p.ids64 ? reinterpret_cast<const long long*>(p.ids)[q] : (long long)reinterpret_cast<const int*>(p.ids)[q];
}

// The reference's bf16 activation values (gx/gx_ingest.py:151-154) of elements
// k0 .. k0 + 15 (k0 % 16 == 0) of a row, from 16-byte loads.
__device__ __forceinline__ void ingest16(const Params& p, const uint8_t* xr, int k0, float inv, float (&v)[16]) {
  if (p.x_fmt == QX_X_BF16) {
    const uint4* src = reinterpret_cast<const uint4*>(xr + (size_t)k0 * 2);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint4 u = src[h];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[8 * h + 2 * i] = __uint_as_float(w[i] << 16);
        v[8 * h + 2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
      }
    }
    return;
  }
  const uint4 u = *reinterpret_cast<const uint4*>(xr + k0);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t f2 = e4m3x2_to_f16x2(w[i] >> (16 * h));
      v[4 * i + 2 * h] = __bfloat162float(__float2bfloat16_rn(__fmul_rn(f16lo_to_f32(f2), inv)));
      v[4 * i + 2 * h + 1] = __bfloat162float(__float2bfloat16_rn(__fmul_rn(f16hi_to_f32(f2), inv)));
    }
  }
}

__device__ __forceinline__ float row_inv(const Params& p, int r) {
  if (p.x_fmt == QX_X_E4M3) return p.x_scale[r];
  if (p.x_fmt == QX_X_E4M3_POST) return p.x_scale[0];
  return 1.f;
}

// e4m3 byte of v >= 0 (round to nearest even, saturating at 448) and its value.
__device__ __forceinline__ uint32_t e4m3_rn(float v) {
  uint32_t two;
  asm("{ .reg .b16 h; cvt.rn.satfinite.e4m3x2.f32 h, %1, %2; cvt.u32.u16 %0, h; }" : "=r"(two) : "f"(0.f), "f"(v));
  return two & 0xFFu;
}

// vLLM's NVFP4 quantiser for one 16-element block (ref_nvfp4_quant): returns the
// scale byte; codes[0..7] = bytes of element pairs (low nibble = even element).
__device__ __forceinline__ uint32_t quant16(const float (&v)[16], float gs, uint32_t (&w)[2]) {
  float vmax = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) vmax = fmaxf(vmax, fabsf(v[i]));
  const float scale = fminf(gs * (vmax * 0.16666667163372040f), 448.f);
  const uint32_t sb = e4m3_rn(scale);
  const float sval = tc::e4m3_val(sb);
  const float os = sval != 0.f ? __frcp_rn(__fmul_rn(sval, __frcp_rn(gs))) : 0.f;
  w[0] = w[1] = 0u;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t byte = tc::e2m1x2_of(__fmul_rn(v[2 * i], os), __fmul_rn(v[2 * i + 1], os));
    w[i >> 2] |= byte << (8 * (i & 3));
  }
  return sb;
}

// ------------------------------------------------------------------ prologue
__global__ void __launch_bounds__(256) pf_prep_kernel(Params p) {
  const int r = blockIdx.x, t = threadIdx.x;
  const float inv = row_inv(p, r);
  const uint8_t* xr = reinterpret_cast<const uint8_t*>(p.x) + (size_t)r * p.x_stride;
  float amax = 0.f;
  for (int k0 = t * 16; k0 < HID; k0 += 256 * 16) {
    float v[16];
    ingest16(p, xr, k0, inv, v);
#pragma unroll
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  // one atomic per row (every row's CTA hits the same word: keep them few)
  __shared__ float wmax[8];
  if ((t & 31) == 0) wmax[t >> 5] = amax;
  __syncthreads();
  if (t == 0) {
    float m = wmax[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) m = fmaxf(m, wmax[i]);
    atomicMax(&p.ctl->amax_bits, __float_as_uint(m));   // amax >= 0: bits order as values
  }
  if (t < p.topk) {
    const long long id = id_of(p, r * p.topk + t);
    if (id >= 0 && id < p.E) atomicAdd(&p.cnt[id], 1u);
    else if (id != -1) atomicOr(&p.ctl->status, (uint32_t)QX_DEV_BAD_ID);
  }
}

// In-place exclusive scan of v[0..n) by the RT_THR-thread block (n <= 4 RT_THR); returns the total.
__device__ int block_scan(int* v, int n, int* wt) {
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  int a[4], s = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int j = 4 * t + i;
    a[i] = j < n ? v[j] : 0;
    s += a[i];
  }
  int inc = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += u;
  }
  if (lane == 31) wt[w] = inc;
  __syncthreads();
  if (w == 0) {
    const int x = wt[lane];
    int xi = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, xi, o);
      if (lane >= o) xi += u;
    }
    wt[lane] = xi - x;
    if (lane == 31) wt[32] = xi;
  }
  __syncthreads();
  int base = wt[w] + inc - s;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int j = 4 * t + i;
    if (j < n) v[j] = base;
    base += a[i];
  }
  const int total = wt[32];
  __syncthreads();
  return total;
}

constexpr int MAXG = 4 * RT_THR;               // groups the routing kernel handles

__global__ void __launch_bounds__(RT_THR) pf_route_kernel(Params p) {
  __shared__ int sc[MAXE], sg[MAXE], sb[MAXG];
  __shared__ int wt[33];
  __shared__ int s_bmax;
  const int t = threadIdx.x;
  if (t == 0) {
    const float amax = fmaxf(__uint_as_float(p.ctl->amax_bits), 9.98377799987793e-07f);   // bf16(1e-6)
    p.ctl->a1g = __bfloat162float(__float2bfloat16_rn(__fdiv_rn(6.f, amax)));
    s_bmax = 0;
  }
  for (int e = t; e < MAXE; e += RT_THR) {
    const int c = e < p.E ? (int)p.cnt[e] : 0;
    sc[e] = c;
    sg[e] = (c + GP - 1) / GP;
  }
  __syncthreads();
  const float a1g = p.ctl->a1g;
  const int nv = block_scan(sc, p.E, wt);      // sc[e] = first position of expert e
  const int G = block_scan(sg, p.E, wt);       // sg[e] = first group of expert e
  for (int e = t; e < p.E; e += RT_THR) {
    p.off[e] = (uint32_t)sc[e];
    p.fill[e] = 0u;
  }
  // groups: an even split of each expert's pairs, in expert order
  int bmax = 0;
  for (int e = t; e < p.E; e += RT_THR) {
    const int c = (int)p.cnt[e];
    if (c == 0) continue;
    const int ng = (c + GP - 1) / GP;
    const float alpha1 = __fdiv_rn(p.g13[e], a1g), alpha2 = __fdiv_rn(p.g2[e], p.a2[e]);
    for (int k = 0; k < ng; ++k) {
      const int lo = k * c / ng, hi = (k + 1) * c / ng;
      Group d = {};
      d.expert = e;
      d.gsz = hi - lo;
      d.npad = npad_of(d.gsz);
      d.pos_off = sc[e] + lo;
      d.sbs = sbs_of(d.npad);
      d.alpha1 = alpha1;
      d.alpha2 = alpha2;
      p.groups[sg[e] + k] = d;
      sb[sg[e] + k] = d.sbs;
      bmax = max(bmax, d.sbs);
      for (int q = lo; q < hi; ++q) p.grp_of_pos[sc[e] + q] = sg[e] + k;
    }
  }
  atomicMax(&s_bmax, bmax);
  __syncthreads();
  // operand offsets: the gate/up operand holds 10 stages per group, the down
  // operand ceil(NT / 8): both are multiples of one prefix sum of stage bytes
  block_scan(sb, G, wt);
  const int nst2 = (p.NT + SK - 1) / SK;
  for (int g = t; g < G; g += RT_THR) {
    p.groups[g].xq_off = (int64_t)sb[g] * (KB1 / SK);
    p.groups[g].ab_off = (int64_t)sb[g] * nst2;
    p.cnt1[g] = 0u;
  }
  if (t == 0) {
    p.ctl->n_groups = (uint32_t)G;
    p.ctl->n1 = (uint32_t)(G * p.NT);
    p.ctl->n2 = (uint32_t)(G * HT);
    p.ctl->b_max = (uint32_t)s_bmax;
    p.ctl->n_valid = (uint32_t)nv;
    p.ctl->work = 0u;
  }
}

__global__ void __launch_bounds__(256) pf_place_kernel(Params p) {
  const int q = blockIdx.x * 256 + threadIdx.x;
  if (q >= p.P) return;
  const long long id = id_of(p, q);
  if (id < 0 || id >= p.E) return;
  const uint32_t pos = p.off[id] + atomicAdd(&p.fill[id], 1u);
  p.pos_pair[pos] = q;
  p.pos_of[q] = (int32_t)pos;
}

// One CTA per token row: the row's NVFP4 codes and scales (x quantised with
// a1g, once), written into the B operand of every routed pair of the row at
// its position r in its group: stage s, codes at (r / 8) 2048 + kb 256 +
// (K half) 128 + (r % 8) 16, scales in the stage's K-block atoms at
// npad 256 + kb 512 + (r % 32) 16 + (r / 32) 4 + j.
__global__ void __launch_bounds__(XQ_THR) pf_xquant_kernel(Params p) {
  // Where the row's routed pairs go: one lane per pair looks it up (id, place,
  // group) while the other threads load and quantise, so the chain of dependent
  // loads is walked once per row, for all pairs at once, not per pair by every thread.
  __shared__ int64_t dst_off[QX_MAX_TOPK];   // the pair's operand block of stage 0, or -1
  __shared__ int32_t dst_sbs[QX_MAX_TOPK], dst_r[QX_MAX_TOPK], dst_npad[QX_MAX_TOPK];
  const int t = blockIdx.x;
  const int b = threadIdx.x;                     // 16-element block
  if (b < p.topk) {
    const int q = t * p.topk + b;
    const long long id = id_of(p, q);
    int64_t off = -1;
    if (id >= 0 && id < p.E) {
      const int pos = p.pos_of[q];
      const Group& g = p.groups[p.grp_of_pos[pos]];
      off = g.xq_off;
      dst_sbs[b] = g.sbs;
      dst_r[b] = pos - g.pos_off;
      dst_npad[b] = g.npad;
    }
    dst_off[b] = off;
  }
  const float inv = row_inv(p, t);
  const uint8_t* xr = reinterpret_cast<const uint8_t*>(p.x) + (size_t)t * p.x_stride;
  float v[16];
  ingest16(p, xr, b * 16, inv, v);
  uint32_t w[2];
  const uint32_t sb = quant16(v, p.ctl->a1g, w);
  const int s = b >> 5, kb = (b >> 2) & (SK - 1), j = b & 3;
  __syncthreads();
  for (int k = 0; k < p.topk; ++k) {
    const int64_t off = dst_off[k];
    if (off < 0) continue;
    const int r = dst_r[k];
    uint8_t* st = p.xq + off + (size_t)s * dst_sbs[k];
    *reinterpret_cast<uint2*>(st + (r >> 3) * 2048 + kb * 256 + (j >> 1) * 128 + (r & 7) * 16 + (j & 1) * 8) =
        make_uint2(w[0], w[1]);
    st[dst_npad[k] * 256 + kb * 512 + (r & 31) * 16 + (r >> 5) * 4 + j] = (uint8_t)sb;
  }
}

// ------------------------------------------------------------------ main kernel
struct Smem {
  uint64_t full[MAXNS], empty[MAXNS], acc_full[2], acc_empty[2], meta_full[NI], meta_empty[NI];
  ItemMeta meta[NI];
  uint64_t drain[NISS];
  uint64_t tm_done;           // every epilogue warp's last TMEM read is complete
  uint32_t tmem_base, prod_scratch, mma_scratch[NISS];
  int32_t pq[NEPI][16];
  float tw[NEPI][16];
};

__device__ __forceinline__ bool bar_and(int id, int n, bool pred) {
  uint32_t r;
  asm volatile("{ .reg .pred p, q; setp.ne.u32 p, %1, 0; bar.red.and.pred q, %2, %3, p; selp.u32 %0, 1, 0, q; }"
               : "=r"(r)
               : "r"((uint32_t)pred), "r"(id), "r"(n)
               : "memory");
  return r != 0u;
}

// Bounded wait until a global counter reaches `need` (acquire); the deadline is
// checked on the clock, the status word (another L2 round trip) every 64 polls.
__device__ bool wait_count(const uint32_t* c, uint32_t need, volatile uint32_t* status, uint64_t deadline) {
  for (uint32_t it = 0;; ++it) {
    if (ld_acquire_gpu(c) >= need) return true;
    if (globaltimer_ns() > deadline) {
      atomicOr(const_cast<uint32_t*>(status), (uint32_t)QX_DEV_TIMEOUT);
      return false;
    }
    if ((it & 63u) == 63u && (*status & QX_DEV_TIMEOUT)) return false;
    __nanosleep(64);
  }
}

__device__ void drain_copies(const Params& p, Smem& S, uint32_t sc) {
  const uint64_t grace = globaltimer_ns() + p.timeout_ns;
  S.prod_scratch = 0;
  const uint32_t first = sc > (uint32_t)p.ns ? sc - (uint32_t)p.ns : 0u;
  for (uint32_t i = first; i < sc; ++i)
    mbar_wait_bounded(&S.full[i % p.ns], (i / p.ns) & 1, &S.prod_scratch, 1u, grace);
}

__device__ void publish(Smem& S, uint32_t& mc, const ItemMeta& m, volatile uint32_t* status, uint64_t deadline,
                        bool& ok) {
  const int mi = (int)(mc % NI);
  if (mc >= (uint32_t)NI &&
      !mbar_wait_bounded(&S.meta_empty[mi], ((mc / NI) - 1) & 1, status, QX_DEV_TIMEOUT, deadline)) {
    ok = false;
    return;
  }
  S.meta[mi] = m;
  mbar_arrive(&S.meta_full[mi]);
  ++mc;
}

__device__ void producer(const Params& p, uint8_t* ring, Smem& S, volatile uint32_t* status, uint64_t deadline) {
  const uint32_t n1 = p.ctl->n1, n2 = p.ctl->n2;
  uint32_t sc = 0, mc = 0;
  bool ok = true;
  uint32_t item = blockIdx.x;
  for (;;) {
    ItemMeta m = {};
    Group g = {};
    if (ok && item < n1 + n2) {
      if (item < n1) {
        m.kind = 1;
        m.group = (int)(item / (uint32_t)p.NT);
        m.tile = (int)(item % (uint32_t)p.NT);
        m.nst = KB1 / SK;
        m.nkb_last = SK;
      } else {
        m.kind = 2;
        m.group = (int)((item - n1) / HT);
        m.tile = (int)((item - n1) % HT);
        m.nst = (p.NT + SK - 1) / SK;
        m.nkb_last = p.NT - (m.nst - 1) * SK;
      }
      g = p.groups[m.group];
      m.n = g.npad;
      m.gsz = g.gsz;
      m.pos_off = g.pos_off;
      m.alpha = m.kind == 1 ? g.alpha1 : g.alpha2;
    }
    publish(S, mc, m, status, deadline, ok);
    if (m.kind == 0 || !ok) {
      if (ok) publish(S, mc, m, status, deadline, ok);   // second end marker: the epilogue groups alternate
      if (!ok) drain_copies(p, S, sc);
      return;
    }
    const uint32_t next = gridDim.x + atomicAdd(&p.ctl->work, 1u);
    const uint8_t* a_src = m.kind == 1 ? p.w13 + ((size_t)g.expert * p.NTA + p.tile0 + m.tile) * (size_t)KB1 * A_KB
                                       : p.w2 + (((size_t)g.expert * HT + m.tile) * p.NTA + p.tile0) * (size_t)A_KB;
    const uint8_t* b_src = m.kind == 1 ? p.xq + g.xq_off : p.ab + g.ab_off;
    if (m.kind == 2 && !wait_count(&p.cnt1[m.group], (uint32_t)p.NT, status, deadline)) ok = false;
    fence_proxy_async_global();
    for (int s = 0; s < m.nst; ++s, ++sc) {
      const int slot = (int)(sc % (uint32_t)p.ns);
      if (sc >= (uint32_t)p.ns &&
          !mbar_wait_bounded(&S.empty[slot], ((sc / p.ns) - 1) & 1, status, QX_DEV_TIMEOUT, deadline)) {
        ok = false;
        break;
      }
      const int nkb = s < m.nst - 1 ? SK : m.nkb_last;
      mbar_arrive_expect_tx(&S.full[slot], (uint32_t)(nkb * A_KB + g.sbs));
      bulk_g2s(ring + (size_t)slot * A_STAGE, a_src + (size_t)s * SK * A_KB, (uint32_t)(nkb * A_KB), &S.full[slot]);
      bulk_g2s(ring + p.b_off + (size_t)slot * p.bst, b_src + (size_t)s * g.sbs, (uint32_t)g.sbs, &S.full[slot]);
    }
    item = next;
  }
}

__device__ void mma_issuer(const Params& p, uint8_t* ring, Smem& S, uint32_t tbase, int iss, volatile uint32_t* status,
                           uint64_t deadline) {
  uint32_t sc = 0, mc = 0, ic = 0;
  for (;;) {
    const int mi = (int)(mc % NI);
    if (!mbar_wait_bounded(&S.meta_full[mi], (mc / NI) & 1, status, QX_DEV_TIMEOUT, deadline)) break;
    const ItemMeta m = S.meta[mi];
    mbar_arrive(&S.meta_empty[mi]);
    ++mc;
    if (m.kind == 0) break;
    const uint32_t n = (uint32_t)m.n;
    const uint32_t idesc = tc::idesc_nvf4(n);
    const int buf = (int)(ic & 1u);
    if (ic >= 2 && !mbar_wait_bounded(&S.acc_empty[buf], ((ic / 2) - 1) & 1, status, QX_DEV_TIMEOUT, deadline))
      break;
    tc::fence_after_sync();
    const uint32_t tacc = tbase + (uint32_t)buf * 2u * TM_SLOT + (uint32_t)iss * TM_SLOT;
    bool ok = true, first = true;
    for (int s = 0; s < m.nst; ++s, ++sc) {
      const int slot = (int)(sc % (uint32_t)p.ns);
      if (!mbar_wait_bounded(&S.full[slot], (sc / p.ns) & 1, status, QX_DEV_TIMEOUT, deadline)) {
        ok = false;
        break;
      }
      const int nkb = s < m.nst - 1 ? SK : m.nkb_last;
      const int k0 = iss * KB_PER_ISS, k1 = min(nkb, k0 + KB_PER_ISS);
      const uint32_t a0 = smem_u32(ring + (size_t)slot * A_STAGE);
      const uint32_t b0 = smem_u32(ring + p.b_off + (size_t)slot * p.bst);
      const uint32_t bank = tbase + tm_bank(iss, (int)(sc & 1u));
      for (int kb = k0; kb < k1; ++kb) {
        const uint32_t j = (uint32_t)(kb - k0);
        tc::cp_sf_atom(bank + 4 * j, a0 + kb * A_KB + 128 * tc::ROWB);
        tc::cp_sf_atom(bank + 16 + 4 * j, b0 + n * 256 + kb * tc::SF_ATOM);
      }
      for (int kb = k0; kb < k1; ++kb) {
        const uint32_t j = (uint32_t)(kb - k0);
        tc::mma_nvf4(tacc, tc::sdesc(a0 + kb * A_KB, tc::LBO, tc::SBO), tc::sdesc(b0 + kb * 256, tc::LBO, 2048),
                     idesc, bank + 4 * j, bank + 16 + 4 * j, first ? 0u : 1u);
        first = false;
      }
      tc::commit(&S.empty[slot]);
    }
    if (!ok) break;
    tc::commit(&S.acc_full[buf]);
    ++ic;
  }
  tc::commit(&S.drain[iss]);
  S.mma_scratch[iss] = 0;
  mbar_wait_bounded(&S.drain[iss], 0, &S.mma_scratch[iss], 1u, globaltimer_ns() + p.timeout_ns);
}

__device__ __forceinline__ bool second_acc(const ItemMeta& m) { return m.nst > 1 || m.nkb_last > KB_PER_ISS; }

__device__ __forceinline__ float bf16r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// Epilogue warpgroup eg: the items of accumulator buffer eg. Pairs go through
// in chunks of 16 accumulator columns.
__device__ void epilogue(const Params& p, Smem& S, float* xg, uint32_t tbase, int eg, volatile uint32_t* status,
                         uint64_t deadline) {
  xg += eg * 2 * 16 * 64;
  float* xu = xg + 16 * 64;                       // [pair of the chunk][column]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int et = threadIdx.x - (eg ? 224 : 64);
  const int B1 = 1 + eg;
  const int quarter = warp & 3;
  const int m = quarter * 32 + lane;
  const uint32_t lanes = (uint32_t)(quarter * 32) << 16;
  for (uint32_t ic = (uint32_t)eg;; ic += NEPI) {
    const uint32_t mc = ic;
    const int mi = (int)(mc % NI);
    const bool got = mbar_wait_bounded(&S.meta_full[mi], (mc / NI) & 1, status, QX_DEV_TIMEOUT, deadline);
    const ItemMeta mt = S.meta[mi];
    if (!bar_and(B1, 128, got)) break;
    if (et == 0) mbar_arrive(&S.meta_empty[mi]);
    if (mt.kind == 0) break;
    const int buf = eg;
    const bool ok = mbar_wait_bounded(&S.acc_full[buf], (ic / 2) & 1, status, QX_DEV_TIMEOUT, deadline);
    if (!bar_and(B1, 128, ok)) break;
    tc::fence_after_sync();
    const uint32_t tacc = tbase + lanes + (uint32_t)buf * 2u * TM_SLOT;
    const bool two = second_acc(mt);
    const Group& gr = p.groups[mt.group];
    if (mt.kind == 1) {
      // ---- gate/up tile: rows 0..63 gate, 64..127 up of columns [64 tile, 64 tile + 64)
      const bool up = m >= 64;
      const int c = m & 63;
      const int kbl = mt.tile % SK;
      uint8_t* st = p.ab + gr.ab_off + (size_t)(mt.tile / SK) * gr.sbs;   // the tile's down stage
      for (int n0 = 0; n0 < mt.gsz; n0 += 16) {
        float v[16], v1[16];
        tc::ld16x2(tacc + n0, tacc + TM_SLOT + n0, v, v1);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float c1 = bf16r(mt.alpha * (v[i] + (two ? v1[i] : 0.f)));
          if (up) xu[i * 64 + c] = c1; else xg[i * 64 + c] = c1;
        }
        if (n0 + 16 >= mt.gsz) {          // the accumulator's last read: hand it back
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&S.acc_empty[buf]);
        }
        asm volatile("bar.sync %0, 128;" ::"r"(B1) : "memory");
        // (pair, 16-column block) units: SwiGLU, NVFP4 with a2, into the down operand
        if (et < 64) {
          const int i = et >> 2, j = et & 3, r = n0 + i;
          if (r < mt.gsz) {
            float a[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const int col = j * 16 + e;
              float gg = xg[i * 64 + col], uu = xu[i * 64 + col];
              if (p.has_limit) {
                gg = fminf(gg, p.limit);
                uu = fminf(fmaxf(uu, -p.limit), p.limit);
              }
              a[e] = (mt.tile * 64 + col < p.W) ? bf16r((gg / (1.f + expf(-gg))) * uu) : 0.f;
            }
            uint32_t w[2];
            const uint32_t sb = quant16(a, p.a2[gr.expert], w);
            *reinterpret_cast<uint2*>(st + (r >> 3) * 2048 + kbl * 256 + (j >> 1) * 128 + (r & 7) * 16 + (j & 1) * 8) =
                make_uint2(w[0], w[1]);
            st[mt.n * 256 + kbl * 512 + (r & 31) * 16 + (r >> 5) * 4 + j] = (uint8_t)sb;
          }
        }
        asm volatile("bar.sync %0, 128;" ::"r"(B1) : "memory");
      }
      // The group's stores are ordered before thread 0's release by the barrier.
      if (et == 0) red_add_release_gpu(&p.cnt1[mt.group], 1u);
    } else {
      // ---- down tile: output rows [128 tile, 128 tile + 128)
      const int h = mt.tile * 128 + m;
      for (int n0 = 0; n0 < mt.gsz; n0 += 16) {
        if (et < 16) {
          const int r = n0 + et;
          const int pq = r < mt.gsz ? p.pos_pair[mt.pos_off + r] : 0;
          S.pq[eg][et] = pq;
          S.tw[eg][et] = r < mt.gsz ? bf16r(p.tw[pq]) : 0.f;
        }
        float v[16], v1[16];
        tc::ld16x2(tacc + n0, tacc + TM_SLOT + n0, v, v1);
        if (n0 + 16 >= mt.gsz) {
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&S.acc_empty[buf]);
        }
        asm volatile("bar.sync %0, 128;" ::"r"(B1) : "memory");
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          if (n0 + i < mt.gsz) {
            const float c3 = bf16r(mt.alpha * (v[i] + (two ? v1[i] : 0.f)));
            p.y[(size_t)S.pq[eg][i] * HID + h] = __float2bfloat16_rn(c3 * S.tw[eg][i]);
          }
        }
        asm volatile("bar.sync %0, 128;" ::"r"(B1) : "memory");
      }
    }
  }
  // This warp reads TMEM no more: TMEM may be released once all epilogue warps say so.
  tc::fence_before_sync();
  __syncwarp();
  if (lane == 0) mbar_arrive(&S.tm_done);
}

__global__ void __launch_bounds__(NTHR, 1) pf_main_kernel(Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  Smem& S = *reinterpret_cast<Smem*>(smem);
  uint8_t* ring = smem + p.ring_off;
  float* xg = reinterpret_cast<float*>(smem + p.x_off);
  const int warp = threadIdx.x >> 5;
  volatile uint32_t* status = &p.ctl->status;
  if (threadIdx.x == 0) {
    for (int s = 0; s < MAXNS; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], NISS);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&S.acc_full[b], NISS);
      mbar_init(&S.acc_empty[b], 4);
    }
    for (int i = 0; i < NI; ++i) {
      mbar_init(&S.meta_full[i], 1);
      mbar_init(&S.meta_empty[i], NISS + 1);
    }
    for (int i = 0; i < NISS; ++i) mbar_init(&S.drain[i], 1);
    mbar_init(&S.tm_done, NEPI * 4);
    fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(&S.tmem_base, TM_COLS);
    tc::tmem_relinquish();
  }
  // Each CTA barrier follows code that one lane of a warp ran alone: the warp
  // reconverges first, so that it arrives at the barrier once.
  __syncwarp();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  {
    const int bmx = (int)p.ctl->b_max;
    p.bst = bmx < 16 ? 16 : bmx;
    int ns = (p.ring_bytes - 512) / (A_STAGE + p.bst);
    p.ns = ns > MAXNS ? MAXNS : ns;
    p.b_off = p.ns * A_STAGE;
  }
  const uint32_t tbase = S.tmem_base;
  const uint64_t deadline = globaltimer_ns() + p.timeout_ns;
  if (p.ns >= 2) {
    if (warp == 0) {
      if ((threadIdx.x & 31) == 0) producer(p, ring, S, status, deadline);
    } else if (warp == 1 || warp == 6) {
      if ((threadIdx.x & 31) == 0) mma_issuer(p, ring, S, tbase, warp == 1 ? 0 : 1, status, deadline);
    } else {
      epilogue(p, S, xg, tbase, warp < 6 ? 0 : 1, status, deadline);
    }
  } else if (threadIdx.x == 0) {
    atomicOr(const_cast<uint32_t*>(status), (uint32_t)QX_DEV_OVERFLOW);   // a group too wide for two ring slots
  }
  __syncwarp();
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    // TMEM is released after the epilogue warps' last reads (bounded wait; none
    // ran when the ring could not hold two stages).
    if ((threadIdx.x & 31) == 0 && p.ns >= 2) {
      S.mma_scratch[0] = 0;
      mbar_wait_bounded(&S.tm_done, 0, &S.mma_scratch[0], 1u, globaltimer_ns() + p.timeout_ns);
    }
    __syncwarp();
    tc::fence_after_sync();
    tc::tmem_dealloc(tbase, TM_COLS);
  }
}

// out[t, k] = bf16(sum over slots j in order of y[t * topk + j, k]).
__global__ void __launch_bounds__(256) pf_finalize_kernel(Params p) {
  const int n8 = p.rows * (HID / 8);
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += gridDim.x * blockDim.x) {
    const int t = i / (HID / 8), k = (i - t * (HID / 8)) * 8;
    float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < p.topk; ++j) {
      const int q = t * p.topk + j;
      const long long id = id_of(p, q);
      if (id < 0 || id >= p.E) continue;
      const uint4 v = __ldcg(reinterpret_cast<const uint4*>(p.y + (size_t)q * HID + k));
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        s[2 * e] += __uint_as_float(w[e] << 16);
        s[2 * e + 1] += __uint_as_float(w[e] & 0xffff0000u);
      }
    }
    uint4 o;
    uint32_t* ow = &o.x;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const __nv_bfloat162 b = __floats2bfloat162_rn(s[2 * e], s[2 * e + 1]);
      ow[e] = *reinterpret_cast<const uint32_t*>(&b);
    }
    *reinterpret_cast<uint4*>(p.out + (size_t)t * p.out_stride + k) = o;
  }
}

constexpr size_t SMEM_LIMIT = 232448;

static uint64_t timeout_ns() {
  const char* e = getenv("QX_TIMEOUT_MS");
  long ms = e ? atol(e) : 1000;
  if (ms < 10) ms = 10;
  return (uint64_t)ms * 1000000ull;
}

}  // namespace pf
}  // namespace qx

using namespace qx::pf;

extern "C" {

size_t qx_prefill_workspace_bytes(int32_t rows, int32_t topk, int32_t c0, int32_t c1, int32_t n_experts) {
  if (rows <= 0 || rows > QX_PREFILL_MAX_ROWS || topk <= 0 || topk > QX_MAX_TOPK || c1 <= c0 || (c1 - c0) % 32 ||
      n_experts <= 0 || n_experts > MAXE)
    return 0;
  return ws_layout(rows, topk, c1 - c0, n_experts).total;
}

int qx_slice_prefill_tc(const QxArena* arena, const QxSliceArgs* a, const float* a2, void* stream) {
  if (!arena || !a || !a2) return QX_ERR_ARG;
  if (!a->x || !a->ids || !a->tw || !a->out || !a->workspace || !arena->w13 || !arena->w2 || !arena->g13 ||
      !arena->g2)
    return QX_ERR_ARG;
  if ((a->x_fmt == QX_X_E4M3 || a->x_fmt == QX_X_E4M3_POST) && !a->x_scale) return QX_ERR_ARG;
  if (a->x_fmt < QX_X_E4M3 || a->x_fmt > QX_X_BF16) return QX_ERR_ARG;
  if (a->rows < 1 || a->rows > QX_PREFILL_MAX_ROWS || a->topk < 1 || a->topk > QX_MAX_TOPK) return QX_ERR_SHAPE;
  if (arena->layout != QX_LAYOUT_TC) return QX_ERR_ARG;
  if (arena->n_experts < 1 || arena->n_experts > MAXE) return QX_ERR_SHAPE;
  if (arena->a0 % 32 || arena->a1 % 32 || arena->a1 <= arena->a0) return QX_ERR_SHAPE;
  if ((a->c0 - arena->a0) % 64 || a->c1 % 32 || a->c0 < arena->a0 || a->c1 > arena->a1 || a->c1 <= a->c0)
    return QX_ERR_SHAPE;
  if (a->c1 - a->c0 > 64 * 64) return QX_ERR_SHAPE;
  const int esz = a->x_fmt == QX_X_BF16 ? 2 : 1;
  if (a->x_stride < (int64_t)HID * esz || a->out_stride < HID) return QX_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(a->x) & 15u) || (a->x_stride & 15) ||
      (reinterpret_cast<uintptr_t>(a->workspace) & 255u) || (reinterpret_cast<uintptr_t>(arena->w13) & 15u) ||
      (reinterpret_cast<uintptr_t>(arena->w2) & 15u) || (reinterpret_cast<uintptr_t>(a->out) & 15u) ||
      (a->out_stride & 7))
    return QX_ERR_ALIGN;
  const int W = a->c1 - a->c0;
  const WsLayout L = ws_layout(a->rows, a->topk, W, arena->n_experts);
  if (a->workspace_bytes < L.total) return QX_ERR_WORKSPACE;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return QX_ERR_DEVICE;
  int major = 0, sms = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess || major != 10)
    return QX_ERR_DEVICE;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return QX_ERR_DEVICE;
  static bool attr_set[64] = {false};
  if (dev < 64 && !attr_set[dev]) {
    if (cudaFuncSetAttribute(pf_main_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_LIMIT) !=
        cudaSuccess)
      return QX_ERR_DEVICE;
    attr_set[dev] = true;
  }
  Params p = {};
  p.x = a->x;
  p.x_scale = a->x_scale;
  p.x_stride = a->x_stride;
  p.x_fmt = a->x_fmt;
  p.ids = a->ids;
  p.ids64 = a->ids_int64 ? 1 : 0;
  p.tw = a->tw;
  p.a2 = a2;
  p.rows = a->rows;
  p.topk = a->topk;
  p.P = a->rows * a->topk;
  p.E = arena->n_experts;
  p.W = W;
  p.NT = (W + 63) / 64;
  p.tile0 = (a->c0 - arena->a0) / 64;
  p.NTA = (arena->a1 - arena->a0 + 63) / 64;
  p.w13 = arena->w13;
  p.w2 = arena->w2;
  p.g13 = arena->g13;
  p.g2 = arena->g2;
  p.limit = a->swiglu_limit;
  p.has_limit = a->has_limit ? 1 : 0;
  p.out = reinterpret_cast<__nv_bfloat16*>(a->out);
  p.out_stride = a->out_stride;
  uint8_t* ws = reinterpret_cast<uint8_t*>(a->workspace);
  p.ctl = reinterpret_cast<Ctl*>(ws + L.ctl);
  p.cnt = reinterpret_cast<uint32_t*>(ws + L.cnt);
  p.fill = reinterpret_cast<uint32_t*>(ws + L.fill);
  p.off = reinterpret_cast<uint32_t*>(ws + L.off);
  p.groups = reinterpret_cast<Group*>(ws + L.groups);
  p.grp_of_pos = reinterpret_cast<int32_t*>(ws + L.grp_of_pos);
  p.pos_pair = reinterpret_cast<int32_t*>(ws + L.pos_pair);
  p.pos_of = reinterpret_cast<int32_t*>(ws + L.pos_of);
  p.cnt1 = reinterpret_cast<uint32_t*>(ws + L.cnt1);
  p.xq = ws + L.xq;
  p.ab = ws + L.ab;
  p.y = reinterpret_cast<__nv_bfloat16*>(ws + L.y);
  p.gmax = groups_bound(p.P, p.E);
  p.x_off = (int)((sizeof(Smem) + 15) & ~size_t(15));
  p.ring_off = (int)(((size_t)p.x_off + (size_t)NEPI * 2 * 16 * 64 * sizeof(float) + 127) & ~size_t(127));
  p.ring_bytes = (int)(SMEM_LIMIT - (size_t)p.ring_off);
  p.timeout_ns = timeout_ns();
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // control block and the per-expert counters start at zero
  if (cudaMemsetAsync(ws + L.ctl, 0, L.groups - L.ctl, st) != cudaSuccess) return QX_ERR_LAUNCH;
  pf_prep_kernel<<<p.rows, 256, 0, st>>>(p);
  pf_route_kernel<<<1, RT_THR, 0, st>>>(p);
  pf_place_kernel<<<(p.P + 255) / 256, 256, 0, st>>>(p);
  pf_xquant_kernel<<<p.rows, XQ_THR, 0, st>>>(p);
  pf_main_kernel<<<sms, NTHR, SMEM_LIMIT, st>>>(p);
  pf_finalize_kernel<<<(p.rows * (HID / 8) + 255) / 256 < 4 * sms ? (p.rows * (HID / 8) + 255) / 256 : 4 * sms, 256,
                       0, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? QX_OK : QX_ERR_LAUNCH;
}

}  // extern "C"
