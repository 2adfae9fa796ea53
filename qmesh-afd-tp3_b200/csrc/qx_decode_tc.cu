// Routed-expert NVFP4 SwiGLU slice for decode rows on the 5th-generation tensor
// cores of B200 (sm_100a): tcgen05.mma.kind::mxf4nvf4 reads the arena's e2m1
// codes and e4m3 block scales straight from shared memory, so no weight is
// dequantised by the SMs and the kernel streams HBM at the copy engines' pace.
//
// Same contract and numerics bar as qx_slice_decode (the reference v7 body,
// gx/kernels/fp4_decode_moe_swz.cu:187-402: x = bf16(e4m3 * inv),
// g, u = g13 * x.W, act = min(g,L)/(1+exp(-min(g,L))) * clamp(u,-L,L),
// y_j = g2 * tw_j * act.W2, out = bf16(sum_j y_j)). The activation side of
// every product enters the MMA as 16 unscaled e2m1 terms on an exponent grid of
// step 2 (v = sum_t 2^(E - 2t) q_t, to 2^-30 of the exponent's range; the
// B-side block scales are a constant 1.0 atom): the gate/up input x with one
// exponent per row, the SwiGLU output with one exponent per pair, fixed at the
// clamp's bound L^2 when the clamp is on (else per tile, moved to the pair's
// largest by the group's last tile). Each term's product with the weights is
// exact in the tensor core and the partial sums meet in FP32 in the epilogue.
//
// Kernels, chained with programmatic dependent launch:
//   tc_prep_kernel     one CTA per (row, 512-element chunk): the reference
//                      ingest, the row's exponent, the chunk's 16 x terms in the
//                      row-major operand layout (one 4,096-byte block per row and
//                      stage); resets the call's counters and checks the ids.
//                      Independent of the routing, so it runs while the decode
//                      kernel starts.
//   tc_decode_kernel   persistent, one CTA per SM, 352 threads (11 warps). Every
//                      CTA first builds the routing tables itself from the ids
//                      (unique experts, groups of <= 6 routed pairs of one
//                      expert, then the shared expert's groups of rows when one
//                      is given; deterministic, so all CTAs agree), then
//                      warp 0      producer: streams each item's weight tile (bulk
//                                  async copy, 8 K blocks = 36,864 bytes per stage)
//                                  and activation operand into a shared-memory
//                                  ring; the first item is the CTA's index and its
//                                  weights are in flight before the prep kernel is
//                                  waited for, later items come from one atomic
//                                  queue;
//                      warps 1, 6  MMA issuers: each copies its K blocks' scale
//                                  atoms into TMEM and issues one M=128 x N x K=64
//                                  block-scaled MMA per K block (the lower / upper
//                                  half of every stage's K blocks) into its own
//                                  accumulator;
//                      warps 2-5, 7-10  two epilogue warpgroups, taking alternate
//                                  items: gate/up -> SwiGLU -> the pair's 16
//                                  activation terms for the down projection; down ->
//                                  y_j = g2 tw_j act.W2 per output row; then
//                                  finalize units.
//                      Items: gate/up (group, 64-column tile: 64 gate + 64 up rows
//                      over K = 5120, split into 2, 5 or 10 K pieces when a call
//                      has too few items to fill the grid, the last piece adding
//                      the pieces' sums in order), then down (group, 128-row output
//                      tile over the slice's columns). A down item waits (bounded)
//                      for its group's activation terms. Every down item counts its
//                      pairs into its 128-row output tile's counter; after its
//                      items each epilogue group finalizes some (output tile,
//                      4-row block) units, out = bf16(sum over slots j in order
//                      of y_j) [+ the shared expert's bf16 output], once their
//                      tile's counter is complete, or hands them to the fused rank
//                      combine (qx_xchg.cuh).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <limits.h>
#include <stdint.h>
#include <stdlib.h>

#include "qmesh_b200.h"
#include "qx_ptx.cuh"
#include "qx_tc.cuh"
#include "qx_xchg.cuh"

namespace qx {
namespace tcd {

constexpr int HID = QX_HIDDEN;                 // 5120
constexpr int KB1 = HID / 64;                  // 80 K blocks in a gate/up item
constexpr int XTERMS = 16;                     // activation terms = B rows per pair (both item kinds)
constexpr int GMAX = 6;                        // routed pairs per group (gate/up N = 16 x 6 = 96)
constexpr int SK = 8;                          // K blocks per stage (36,864-byte weight copies)
constexpr int A_KB = 128 * tc::ROWB + tc::SF_ATOM;  // 4608 weight bytes per K block
constexpr int A_STAGE = SK * A_KB;             // 36864
constexpr int HT = HID / 128;                  // 40 output-row tiles in a down item set
constexpr int MAXP = QX_MAX_ROWS * QX_MAX_TOPK;
constexpr int MAXE = 4096;
constexpr int MAXNS = 12;                      // ring slots
constexpr int NI = MAXNS + 2;                 // even: an epilogue group reuses its own meta entries
static_assert(NI % 2 == 0, "epilogue groups alternate meta entries");
// Warps: 0 producer, 1 and 6 MMA issuers, 2-5 and 7-10 two epilogue warpgroups
// (group g takes the items of accumulator buffer g, so a long gate/up epilogue
// never holds up the next item's accumulator).
constexpr int NTHR = 352;
constexpr int NEPI = 2;                        // epilogue warpgroups
// Two MMA issuer warps split every stage: of its nkb K blocks, the first
// ceil(nkb / 2) go to issuer 0, the rest to issuer 1, each into its own
// accumulator (summed in the epilogue); one thread cannot issue block-scaled
// MMAs as fast as the tensor pipe executes them.
// TMEM columns, in four 128-column slots (accumulators use the first 96):
//   accumulator (buffer b, issuer i) at 256 b + 128 i;
//   in the 32-column gaps: the constant all-1.0 scale atom of every activation
//   operand at 96 (two atoms: operand rows 0..127, 128..255); the weight scale
//   atoms of issuer i's (at most 4) K blocks of a stage (4 columns each), in two banks
//   alternating by stage, at 224 + 128 i + 16 bank. A stage's scale copies are
//   issued before its MMAs into the bank the previous stage's MMAs do not read,
//   so no MMA waits on the copy just before it. Every scale operand starts on a
//   4-column boundary, as block-scaled MMAs require.
constexpr uint32_t TM_COLS = 512, TM_SLOT = 128, TM_ONE = 96, TM_SF = 224, TM_BANK = 16;
constexpr int NISS = 2, KB_PER_ISS = SK / NISS;
static_assert(KB_PER_ISS * 4 <= (int)TM_BANK, "a stage's scale atoms fit one bank");
static_assert(GMAX * XTERMS <= 96, "an accumulator fits its slot");
constexpr int XE_LO = -90, XE_HI = 100;      // x exponents
// K-split of gate/up items: the (group, tile) items that fill whole waves of
// the grid run whole; the remainder, which would leave most CTAs idle in a last
// partial wave (narrow column shards), is split into ks pieces of 10 / ks stages
// (ks in {1, 2, 5, 10}, the largest that keeps the pieces within one wave). A
// piece stores its FP32 sums and the last piece of an item adds the pieces in
// piece order. At most MAXSPLIT pieces per call.
constexpr int MAXSPLIT = 512;      // routed pieces (a split never exceeds the grid)
constexpr int MAXSPLIT_S = MAXSPLIT;   // shared-expert pieces (their own split, after the routed ones;
                                       // the same cap, so they split as a call of their arena alone)
constexpr int MAX_STILES = 64;     // shared-expert column tiles at most (4096 columns)
constexpr int MAXSG = (QX_MAX_ROWS + 5) / 6;   // shared-expert groups at most
constexpr int AE_LO = -90, AE_HI = 100;      // SwiGLU-output exponents (even)

struct Ctl {
  uint32_t work, status;   // dynamic item queue (after the first grid-size items), QX_DEV_* bits
  uint32_t pad[62];
};
static_assert(sizeof(Ctl) == 256, "ctl block is 256 bytes");

struct GroupS {     // one group (<= GMAX routed pairs of one expert), kept in shared memory
  int32_t expert, gsz, pair_off;
  int32_t n, sbs;         // activation operand of either item kind: 16 x gsz rows, bytes per stage
  int32_t ab_off;         // offset of the group's down operand in the activation-term buffer
  int32_t shared;         // 1: rows of the shared expert (its own arena, weight 1)
  int32_t pad;
};
static_assert(sizeof(GroupS) == 32, "shared group record is 32 bytes");

struct RouteHdr {   // call-wide results of the routing, in shared memory
  int32_t n_groups, n1, n2, b_max;   // routed groups, gate/up items (pieces), down items, widest activation stage
  int32_t n_pairs;                   // routed pairs with a valid expert
  int32_t ks, kss;                   // pieces per split gate/up (group, tile) item: routed, shared expert
  int32_t fw, fws;                   // gate/up (group, tile) items that run whole: routed, shared expert
  int32_t n_sgroups;                 // shared-expert groups (gs[n_groups ...])
  int32_t n1s, n2s;                  // the first n1s gate/up and n2s down items are the shared expert's
  int32_t n_fin;                     // pairs whose y every output tile waits for (routed + shared rows)
  int32_t pad[3];
};

struct PairS {      // per group position
  int32_t pq;       // routed pair index (row * topk + slot), or P + row for the shared expert's
  int32_t row;      // the pair's activation row
};
static_assert(sizeof(PairS) == 8, "shared pair record is 8 bytes");

struct Params {
  const void* x;
  const float* x_scale;
  int64_t x_stride;
  int x_fmt;
  const void* ids;
  int ids64;
  const float* tw;
  int rows, topk, P;
  int W, NT, tile0, NTA;      // slice width, its 64-column tiles, first arena tile, arena tiles
  const uint8_t* w13;
  const uint8_t* w2;
  const float* g13;
  const float* g2;
  int E;
  float limit;
  int has_limit;
  __nv_bfloat16* out;
  int64_t out_stride;
  Ctl* ctl;
  uint32_t* cnt1;     // [P + rows] gate/up tiles finished per group
  uint32_t* ready;    // [P + rows] group activation terms complete
  uint32_t* fcnt;     // [HT] routed pairs whose y is written, per 128-row output tile
  uint32_t* pcnt;     // [MAXSPLIT + MAXSG * MAX_STILES] pieces finished per gate/up (group, tile) item
  float* gpart;       // [MAXSPLIT + MAXSPLIT_S][GMAX][128] FP32 sums of each gate/up piece
  int32_t* emax;      // [P + rows] per group position: common activation exponent
  int32_t* eloc;      // [P + rows][MAX_STILES] per group position and tile: tile exponent
  int32_t* xexp;      // [rows]
  uint8_t* xt;        // [rows][10 stages][4096 bytes]: x terms, row-major
  uint8_t* ab;        // per group: ceil(NT / SK) stages of sbs bytes (SwiGLU-output terms)
  float* y;           // [P + rows][HID]: routed pairs, then the shared expert's rows
  int x_off;          // shared-memory offset of the SwiGLU exchanges (per epilogue group 2 x gmax x 64 floats)
  int tab_off;        // shared-memory offset of the group and pair tables
  int ring_off, ring_bytes;  // shared-memory span of the stage rings
  int gmax;           // pairs per group at most
  int ns, bst, b_off; // set on the device from the largest group: ring slots, activation
                      // bytes per slot, offset of the activation ring
  uint64_t timeout_ns;
  uint32_t dep_extra; // test hook: extra arrivals a down item waits for (0 in service)
  int ae_fixed;       // 1: every SwiGLU-output tile uses exponent ae_val (a clamped SwiGLU's
  int ae_val;         //    bound); 0: per-tile exponents, fixed up by the group's last tile
  // shared expert (the output rank's dense SwiGLU of config 2): a one-expert
  // arena over its intermediate columns [0, sW); every row is routed to it with
  // weight 1 and its BF16 output is added after the routed partials
  const uint8_t* sw13;
  const uint8_t* sw2;
  const float* sg13;
  const float* sg2;
  int sW, sNT;        // sNT == 0: no shared expert
  // fused rank combine (qx_slice_decode_tc_xchg; xworld == 0 otherwise): every
  // rank's exchange buffer, the optional shared-expert partial of the output rank
  uint8_t* xbuf[QX_XCHG_MAX_RANKS];
  const __nv_bfloat16* xshared;
  int64_t xshared_stride;
  int xrank, xworld, xdst, xrows_max;
};

struct ItemMeta {
  int32_t kind;       // 1 gate/up, 2 down, 0 end
  int32_t group, tile, nst, nkb_last;
  int32_t piece;      // gate/up: the item's K piece (stages piece * nst ...)
  int32_t ks;         // gate/up: pieces of its (group, tile) item (1: whole)
  int32_t gi;         // gate/up piece: index of its (group, tile) item among the split ones
};

__host__ __device__ inline size_t al256(size_t v) { return (v + 255) & ~size_t(255); }

// Activation operands (16 x gsz rows of e2m1 terms, codes only; the B-side
// scales are the constant 1.0 atom). x terms are kept row-major, one 4,096-byte
// block per row and stage laid out [row group 2][K block 8][K half 2][8 terms]
// [16 bytes]. A group's stage is its pairs' blocks side by side (pair q at
// 4,096 q), so operand row group j sits at 2,048 j: one MMA per K block with
// leading offset 128 and stride 2,048 reads all of the group's rows, and the
// gate/up stage is gsz copies of 4,096 bytes. The SwiGLU-output terms of a group
// (down items) use the same stage layout, one copy of gsz x 4,096 bytes.
constexpr int XT_STAGE = SK * 512;             // term bytes per pair (row) and stage
constexpr uint32_t XT_SBO = SK * 256;          // row group to row group
constexpr uint32_t XT_KB = 256;                // K block to K block

struct WsLayout {
  size_t ctl, cnt1, ready, fcnt, pcnt, emax, eloc, xexp, xt, ab, y, gpart, total;
};

// The workspace always has room for a shared expert of up to MAX_STILES tiles
// over the call's rows (about 52 KB per row).
__host__ inline WsLayout ws_layout(int rows, int topk, int W) {
  WsLayout L;
  const int P = rows * topk, NT = (W + 63) / 64, PS = P + rows;
  size_t o = 0;
  L.ctl = o;      o = al256(o + sizeof(Ctl));
  L.cnt1 = o;     o = al256(o + (size_t)PS * 4);
  L.ready = o;    o = al256(o + (size_t)PS * 4);
  L.fcnt = o;     o = al256(o + (size_t)HT * 4);
  L.pcnt = o;     o = al256(o + (size_t)(MAXSPLIT + MAXSG * MAX_STILES) * 4);
  L.emax = o;     o = al256(o + (size_t)PS * 4);
  L.eloc = o;     o = al256(o + (size_t)PS * MAX_STILES * 4);
  L.xexp = o;     o = al256(o + (size_t)rows * 4);
  L.xt = o;       o = al256(o + (size_t)rows * (KB1 / SK) * XT_STAGE);
  L.ab = o;       o = al256(o + ((size_t)P * ((NT + SK - 1) / SK) + (size_t)rows * (MAX_STILES / SK)) * XT_STAGE);
  L.y = o;        o = al256(o + (size_t)PS * HID * 4);
  L.gpart = o;    o = al256(o + (size_t)(MAXSPLIT + MAXSPLIT_S) * GMAX * 128 * 4);
  L.total = o;
  return L;
}

// Weights and geometry of a group's expert: the call's arena and column range,
// or the shared expert's one-expert arena over all its columns.
struct Geo {
  const uint8_t* w13;
  const uint8_t* w2;
  int NT, NTA, tile0, W;
};
__device__ __forceinline__ Geo geo_of(const Params& p, const GroupS& g) {
  Geo r;
  if (g.shared) {
    r.w13 = p.sw13; r.w2 = p.sw2; r.NT = p.sNT; r.NTA = p.sNT; r.tile0 = 0; r.W = p.sW;
  } else {
    r.w13 = p.w13; r.w2 = p.w2; r.NT = p.NT; r.NTA = p.NTA; r.tile0 = p.tile0; r.W = p.W;
  }
  return r;
}



// ------------------------------------------------------------------ prologue
// SwiGLU-output exponent of one pair over one 64-column tile: the smallest EVEN
// E with 6 * 2^E >= amax, clamped to [-90, 100] (-90 for amax == 0, so an
// all-zero tile never raises the pair's common exponent). Even, so that moving
// a tile to a larger common exponent is a shift of whole terms.
__device__ __forceinline__ int act_exponent(float amax) {
  if (!(amax > 0.f)) return AE_LO;
  int ex;
  frexpf(amax, &ex);
  int e = ex - 3;
  while (e > AE_LO && ldexpf(6.f, e - 1) >= amax) --e;
  while (e < AE_HI && ldexpf(6.f, e) < amax) ++e;
  e += e & 1;
  return e > AE_HI ? AE_HI : e;
}

// Smallest E with 6 * 2^E >= amax (0 for amax == 0), clamped to [-90, 100]:
// the first unscaled x term then lies within the e2m1 range.
__device__ __forceinline__ int x_exponent(float amax) {
  if (!(amax > 0.f)) return 0;
  int ex;
  frexpf(amax, &ex);
  int e = ex - 3;
  while (e > XE_LO && ldexpf(6.f, e - 1) >= amax) --e;
  while (e < XE_HI && ldexpf(6.f, e) < amax) ++e;
  return e;
}

constexpr int XCH = SK * 64;             // activation elements per x-term unit (one stage)
constexpr int NXCH = HID / XCH;          // 10 units per row
constexpr int PREP_THR = XCH / 2;        // prep threads per unit: two elements each

// The reference's bf16 activation value of element k (gx/gx_ingest.py:151-154).
__device__ __forceinline__ float ingest_one(const Params& p, const uint8_t* xr, int k, float inv) {
  if (p.x_fmt == QX_X_BF16) return __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(xr)[k] << 16);
  const uint32_t f2 = e4m3x2_to_f16x2(xr[k]);
  return __bfloat162float(__float2bfloat16_rn(__fmul_rn(f16lo_to_f32(f2), inv)));
}

// max |x| over one row (5 KB of L2 reads) by the PREP_THR threads of a prep
// CTA; red: PREP_THR / 32 floats of shared memory. Every thread gets the result.
__device__ float row_amax(const Params& p, const uint8_t* xr, float inv, float* red, int tid) {
  float amax = 0.f;
  if (p.x_fmt == QX_X_BF16) {
    for (int u = tid; u < HID / 8; u += PREP_THR) {
      const uint4 w = *reinterpret_cast<const uint4*>(xr + (size_t)u * 16);
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        amax = fmaxf(amax, fabsf(__uint_as_float(ww[k] << 16)));
        amax = fmaxf(amax, fabsf(__uint_as_float(ww[k] & 0xffff0000u)));
      }
    }
  } else {
    constexpr int NW = (HID / 16 + PREP_THR - 1) / PREP_THR;
    uint4 wv[NW];                           // all loads first
#pragma unroll
    for (int i = 0; i < NW; ++i) {
      const int u = tid + PREP_THR * i;
      wv[i] = u < HID / 16 ? *reinterpret_cast<const uint4*>(xr + (size_t)u * 16) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int i = 0; i < NW; ++i) {
      const uint32_t ww[4] = {wv[i].x, wv[i].y, wv[i].z, wv[i].w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const uint32_t f2 = e4m3x2_to_f16x2(ww[k] >> (16 * hh));
          amax = fmaxf(amax, fabsf(__bfloat162float(__float2bfloat16_rn(__fmul_rn(f16lo_to_f32(f2), inv)))));
          amax = fmaxf(amax, fabsf(__bfloat162float(__float2bfloat16_rn(__fmul_rn(f16hi_to_f32(f2), inv)))));
        }
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((tid & 31) == 0) red[tid >> 5] = amax;
  __syncthreads();
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < PREP_THR / 32; ++i) m = fmaxf(m, red[i]);
  return m;
}

constexpr int IDR = MAXP / 32;   // expert ids per lane of the routing warp

// Lane `lane`'s expert ids (pairs lane + 32 i); ids outside [0, E) (the -1
// sentinel, or bad ids that the prep kernel flags) become -1 and are skipped.
__device__ __forceinline__ void load_ids(const Params& p, int lane, int (&idr)[IDR]) {
#pragma unroll
  for (int i = 0; i < IDR; ++i) {
    const int q = lane + 32 * i;
    long long id = -1;
    if (q < p.P)
      id = p.ids64 ? __ldg(reinterpret_cast<const long long*>(p.ids) + q)
                   : (long long)__ldg(reinterpret_cast<const int*>(p.ids) + q);
    idr[i] = (id >= 0 && id < p.E) ? (int)id : -1;
  }
}

// The routing tables of a call, built by one warp of every CTA from the ids
// (the reference groups the routed pairs by expert the same way for its
// grouped launch, gx/gx_decode_swz.py:148-179): unique experts in ascending
// order; an expert's pairs in (row, slot) order, split evenly into groups of at
// most gmax; per group its operand geometry and the offset of its down operand;
// gs[g], ps[group position], hdr. Every CTA computes the same tables.
//
// The warp sorts the keys (expert << 9 | pair) of its 32 K slots (pair
// lane + 32 j, no pair = all ones, sorted last) with a bitonic network, element
// i = K lane + j after the sort; an expert's pairs are then a run of the sorted
// order, and scans over the order give each pair its run's start and end, its
// rank in the run and its group. A group's pairs are contiguous in the order,
// so its down operand sits at (its first position) x (bytes per pair).
// Compare-exchange of this lane's slots j and j | S (S < K) towards ascending
// order where bit k of the element index K lane + j is clear.
template <int K, int S>
__device__ __forceinline__ void cx_lane(uint32_t (&v)[K], int k, int lane) {
#pragma unroll
  for (int j = 0; j < K; ++j) {
    if ((j & S) == 0) {
      const bool asc = ((K * lane + j) & k) == 0;
      const uint32_t a = v[j], b = v[j | S];
      v[j] = asc ? min(a, b) : max(a, b);
      v[j | S] = asc ? max(a, b) : min(a, b);
    }
  }
}

// floor(a / b) for 0 <= a < 2^22, 1 <= b < 2^22: a float quotient corrected by one step.
__device__ __forceinline__ int div_small(int a, int b) {
  int q = __float2int_rz(__fdividef((float)a, (float)b));
  if (q * b > a) --q;
  else if ((q + 1) * b <= a) ++q;
  return q;
}

template <int K>
__device__ void route_sort(const Params& p, const int (&idr)[IDR], GroupS* gs, PairS* ps, RouteHdr* hdr) {
  static_assert(K <= IDR && (K & (K - 1)) == 0, "keys per lane");
  constexpr uint32_t FULL = 0xffffffffu, NONE = 0xffffffffu;
  constexpr int N = 32 * K;
  const int lane = threadIdx.x & 31;
  const int gmax = min(GMAX, p.rows);
  uint32_t v[K];
#pragma unroll
  for (int j = 0; j < K; ++j) {
    const int q = lane + 32 * j;
    v[j] = (q < p.P && idr[j] >= 0) ? ((uint32_t)idr[j] << 9) | (uint32_t)q : NONE;
  }
  if constexpr (K == 2) {
    // Up to 64 keys: a rank sort. A key's place is the number of smaller keys
    // (the valid keys are distinct: the pair index is in their low bits; the
    // equal NONE keys sort after them and are not placed); one short loop of
    // shuffles, which the SM fetches once (the sort runs at every CTA's start,
    // when each instruction fetched is a miss).
    uint32_t* sb = reinterpret_cast<uint32_t*>(gs);   // scratch: the tables are written after
    int r0 = 0, r1 = 0;
#pragma unroll 4
    for (int src = 0; src < 32; ++src) {
      const uint32_t a = __shfl_sync(FULL, v[0], src), b = __shfl_sync(FULL, v[1], src);
      r0 += (int)(a < v[0]) + (int)(b < v[0]);
      r1 += (int)(a < v[1]) + (int)(b < v[1]);
    }
    const int nv = __popc(__ballot_sync(FULL, v[0] != NONE)) + __popc(__ballot_sync(FULL, v[1] != NONE));
    if (v[0] != NONE) sb[r0] = v[0];
    if (v[1] != NONE) sb[r1] = v[1];
    __syncwarp();
    v[0] = 2 * lane < nv ? sb[2 * lane] : NONE;
    v[1] = 2 * lane + 1 < nv ? sb[2 * lane + 1] : NONE;
    __syncwarp();
  } else {
  // The network's stages run as loops: a fully unrolled network of 512 keys is
  // thousands of instructions that every SM fetches once at its start.
#pragma unroll 1
  for (int k = 2; k <= N; k <<= 1) {
#pragma unroll 1
    for (int s = k >> 1; s > 0; s >>= 1) {
      if (s >= K) {                        // partner in lane ^ (s / K), same slot
        const bool keep_min = ((lane & (k / K)) == 0) == ((lane & (s / K)) == 0);
#pragma unroll
        for (int j = 0; j < K; ++j) {
          const uint32_t o = __shfl_xor_sync(FULL, v[j], s / K);
          v[j] = keep_min ? min(v[j], o) : max(v[j], o);
        }
      } else if (s == 1) {                 // partner in this lane's slot j ^ s
        cx_lane<K, 1>(v, k, lane);
      } else if (s == 2) {
        if constexpr (K > 2) cx_lane<K, 2>(v, k, lane);
      } else if (s == 4) {
        if constexpr (K > 4) cx_lane<K, 4>(v, k, lane);
      } else {
        if constexpr (K > 8) cx_lane<K, 8>(v, k, lane);
      }
    }
  }
  }
  // runs: f = first pair of an expert; st = run start (inclusive max scan of
  // the starts), en = next run's start (suffix min), or the valid-pair count
  int Pv = 0, e[K];
  bool f[K];
#pragma unroll
  for (int j = 0; j < K; ++j) {
    e[j] = v[j] == NONE ? -1 : (int)(v[j] >> 9);
    Pv += __popc(__ballot_sync(FULL, v[j] != NONE));
  }
  const int prev = __shfl_up_sync(FULL, e[K - 1], 1);
#pragma unroll
  for (int j = 0; j < K; ++j) f[j] = e[j] >= 0 && (j ? e[j - 1] != e[j] : (lane == 0 || prev != e[0]));
  int st[K], en[K], run = -1, nx = INT_MAX;
#pragma unroll
  for (int j = 0; j < K; ++j) {
    if (f[j]) run = K * lane + j;
    st[j] = run;
  }
#pragma unroll
  for (int j = K - 1; j >= 0; --j) {
    en[j] = nx;
    if (f[j]) nx = K * lane + j;
  }
  int lmax = run, lmin = nx;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int a = __shfl_up_sync(FULL, lmax, o), b = __shfl_down_sync(FULL, lmin, o);
    if (lane >= o) lmax = max(lmax, a);
    if (lane + o < 32) lmin = min(lmin, b);
  }
  // (every lane takes part in each shuffle; the edge lanes' values are replaced after)
  int before = __shfl_up_sync(FULL, lmax, 1), after = __shfl_down_sync(FULL, lmin, 1);
  if (lane == 0) before = -1;
  if (lane == 31) after = INT_MAX;
  // per pair: run length c, rank r, groups of the run ng, own group k; the
  // inclusive sum of ng over run starts numbers the groups
  int c[K], r[K], ng[K], gk[K], sum = 0;
#pragma unroll
  for (int j = 0; j < K; ++j) {
    st[j] = max(st[j], before);
    const int end = min(min(en[j], after), Pv);
    c[j] = e[j] >= 0 ? end - st[j] : 1;
    r[j] = K * lane + j - st[j];
    ng[j] = div_small(c[j] + gmax - 1, gmax);
    gk[j] = div_small((r[j] + 1) * ng[j] - 1, c[j]);   // the k with k c / ng <= r < (k + 1) c / ng
    if (f[j]) sum += ng[j];
    st[j] = sum;                               // from here: inclusive group count
  }
  int lsum = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int a = __shfl_up_sync(FULL, lsum, o);
    if (lane >= o) lsum += a;
  }
  const int G = __shfl_sync(FULL, lsum, 31), base = lsum - sum;
  const int abs = ((p.NT + SK - 1) / SK) * XT_STAGE;   // down-operand bytes per pair
  int bmx = 0;
#pragma unroll
  for (int j = 0; j < K; ++j) {
    if (e[j] < 0) continue;
    const int i = K * lane + j;
    ps[i].pq = (int)(v[j] & 511u);
    ps[i].row = div_small(ps[i].pq, p.topk);
    const int lo = div_small(gk[j] * c[j], ng[j]);
    if (r[j] == lo) {                          // the group's first pair writes its record
      const int gsz = div_small((gk[j] + 1) * c[j], ng[j]) - lo;
      GroupS d;
      d.expert = e[j];
      d.gsz = gsz;
      d.pair_off = i;
      d.n = XTERMS * gsz;
      d.sbs = gsz * XT_STAGE;
      d.ab_off = i * abs;
      d.shared = 0;
      d.pad = 0;
      gs[base + st[j] - ng[j] + gk[j]] = d;
      bmx = max(bmx, d.sbs);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) bmx = max(bmx, __shfl_xor_sync(FULL, bmx, o));
  if (lane == 0) {
    hdr->n_groups = G;
    hdr->b_max = bmx;
    hdr->n_pairs = Pv;
  }
  __syncwarp();
}

// Split of `items` gate/up (group, tile) items over the grid: the first *whole
// (a multiple of the grid) run whole; the rest, fewer than the grid, run as ks
// pieces each, ks the largest of 1, 2, 5, 10 with rest x ks <= grid (and
// <= cap). Depends only on the item count and the grid, so a call's routed
// items split the same with or without a shared expert, and a shared expert the
// same as a call of its arena alone.
__device__ __forceinline__ int split_of(int items, int cap, int* whole) {
  const int grid = (int)gridDim.x;
  *whole = items - items % grid;
  const int rest = items - *whole;
  int ks = 1;
  const int opt[3] = {2, 5, 10};
#pragma unroll
  for (int i = 0; i < 3; ++i)
    if (rest * opt[i] <= grid && rest * opt[i] <= cap) ks = opt[i];
  return ks;
}

// After the routed tables: the shared expert's groups (every row, in row order,
// split evenly into groups of at most gmax, as the routing splits one expert's
// pairs) at gs[G ...], their pairs at ps[Pv ...] (code P + row), and the item
// counts of the call. One warp.
__device__ void route_finish(const Params& p, GroupS* gs, PairS* ps, RouteHdr* hdr) {
  const int lane = threadIdx.x & 31;
  const int G = hdr->n_groups, Pv = hdr->n_pairs;
  const int gmax = min(GMAX, p.rows);
  int Gs = 0;
  if (p.sNT > 0) {
    Gs = (p.rows + gmax - 1) / gmax;
    for (int r = lane; r < p.rows; r += 32) {
      ps[Pv + r].pq = p.P + r;
      ps[Pv + r].row = r;
    }
    const int abs_r = ((p.NT + SK - 1) / SK) * XT_STAGE, abs_s = ((p.sNT + SK - 1) / SK) * XT_STAGE;
    if (lane < Gs) {
      const int lo = div_small(lane * p.rows, Gs), hi = div_small((lane + 1) * p.rows, Gs);
      GroupS d;
      d.expert = 0;
      d.gsz = hi - lo;
      d.pair_off = Pv + lo;
      d.n = XTERMS * d.gsz;
      d.sbs = d.gsz * XT_STAGE;
      d.ab_off = p.P * abs_r + lo * abs_s;
      d.shared = 1;
      d.pad = 0;
      gs[G + lane] = d;
    }
  }
  __syncwarp();
  if (lane == 0) {
    int fw = 0, fws = 0;
    const int ks = split_of(G * p.NT, MAXSPLIT, &fw);
    const int kss = Gs ? split_of(Gs * p.sNT, MAXSPLIT_S, &fws) : 1;
    hdr->ks = ks;
    hdr->kss = kss;
    hdr->fw = fw;
    hdr->fws = fws;
    hdr->n_sgroups = Gs;
    hdr->n1s = fws + (Gs * p.sNT - fws) * kss;
    hdr->n1 = hdr->n1s + fw + (G * p.NT - fw) * ks;
    hdr->n2s = Gs * HT;
    hdr->n2 = (G + Gs) * HT;
    hdr->n_fin = Pv + (Gs ? p.rows : 0);
    if (Gs) hdr->b_max = max(hdr->b_max, gmax * XT_STAGE);
  }
  __syncwarp();
}

__device__ void route_local(const Params& p, const int (&idr)[IDR], GroupS* gs, PairS* ps, RouteHdr* hdr) {
  if (p.P <= 64) route_sort<2>(p, idr, gs, ps, hdr);
  else if (p.P <= 128) route_sort<4>(p, idr, gs, ps, hdr);
  else if (p.P <= 256) route_sort<8>(p, idr, gs, ps, hdr);
  else route_sort<16>(p, idr, gs, ps, hdr);
  route_finish(p, gs, ps, hdr);
}

// One CTA per unit (row r, 512-element chunk c = stage c of the gate/up
// operand): the reference ingest of row r, its exponent E (every unit of the
// row computes the same), and the chunk's 16 unscaled x terms
// q_t = rne(r_t / 2^(E - 2t)) (two elements per thread) into the row's stage
// block. CTA 0 also resets the call's counters and records bad ids.
__global__ void __launch_bounds__(PREP_THR) tc_prep_kernel(Params p) {
  __shared__ float red[PREP_THR / 32];
  pdl_launch_dependents();
  const int tid = threadIdx.x, lane = tid & 31;
  if (blockIdx.x == 0) {
    bool bad = false;
    for (int q = tid; q < p.P + p.rows; q += PREP_THR) {
      if (q < p.P) {
        const long long id = p.ids64 ? reinterpret_cast<const long long*>(p.ids)[q]
                                     : (long long)reinterpret_cast<const int*>(p.ids)[q];
        bad |= !(id == -1 || (id >= 0 && id < p.E));
      }
      p.cnt1[q] = 0;
      p.ready[q] = 0;
      p.emax[q] = INT_MIN;
    }
    for (int i = tid; i < HT; i += PREP_THR) p.fcnt[i] = 0;
    bad = __syncthreads_or(bad);
    uint32_t* c = reinterpret_cast<uint32_t*>(p.ctl);
    for (int i = tid; i < (int)(sizeof(Ctl) / 4); i += PREP_THR) c[i] = 0;
    __syncthreads();
    if (tid == 0 && bad) p.ctl->status = (uint32_t)QX_DEV_BAD_ID;
  }
  for (int i = blockIdx.x * PREP_THR + tid; i < MAXSPLIT + MAXSG * MAX_STILES; i += gridDim.x * PREP_THR)
    p.pcnt[i] = 0;
  const int r = blockIdx.x / NXCH, c = blockIdx.x - r * NXCH;
  float inv = 1.f;
  if (p.x_fmt == QX_X_E4M3) inv = p.x_scale[r];
  else if (p.x_fmt == QX_X_E4M3_POST) inv = p.x_scale[0];
  const uint8_t* xr = reinterpret_cast<const uint8_t*>(p.x) + (size_t)r * p.x_stride;
  // Thread tid owns elements k, k + 1 (k = XCH c + 2 tid): warp w is K block w
  // of the stage, lane l its columns 2l, 2l + 1.
  const int k = c * XCH + 2 * tid;
  float v0 = ingest_one(p, xr, k, inv), v1 = ingest_one(p, xr, k + 1, inv);
  const int e = x_exponent(row_amax(p, xr, inv, red, tid));
  if (c == 0 && tid == 0) p.xexp[r] = e;
  uint8_t* blk = p.xt + ((size_t)r * NXCH + c) * XT_STAGE + (tid >> 5) * XT_KB + (lane >> 4) * 128 + (lane & 12);
  float g = tc::exp2i(e), ig = tc::exp2i(-e);
#pragma unroll 1
  for (int tt = 0; tt < XTERMS; ++tt) {
    const uint32_t w = tc::pack4(tc::digit2(v0, v1, g, ig), lane);
    if ((lane & 3) == 0) *reinterpret_cast<uint32_t*>(blk + (tt >> 3) * XT_SBO + (tt & 7) * 16) = w;
    g *= 0.25f;
    ig *= 4.f;
  }
}

__device__ __forceinline__ void st_release_gpu(uint32_t* ptr, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}

// Named barrier over `n` threads that also ANDs a predicate across them, so a
// decision taken after a bounded wait is the same in every participating warp.
__device__ __forceinline__ bool bar_and(int id, int n, bool pred) {
  uint32_t r;
  asm volatile("{ .reg .pred p, q; setp.ne.u32 p, %1, 0; bar.red.and.pred q, %2, %3, p; selp.u32 %0, 1, 0, q; }"
               : "=r"(r)
               : "r"((uint32_t)pred), "r"(id), "r"(n)
               : "memory");
  return r != 0u;
}

// Bounded wait until a global flag set by other CTAs reaches `need` (acquire).
// The deadline is checked on the clock; the status word (another L2 round
// trip) only every 64 polls.
__device__ bool wait_flag(const uint32_t* flag, uint32_t need, volatile uint32_t* status, uint64_t deadline) {
  for (uint32_t it = 0;; ++it) {
    if (ld_acquire_gpu(flag) >= need) return true;
    if (globaltimer_ns() > deadline) {
      atomicOr(const_cast<uint32_t*>(status), (uint32_t)QX_DEV_TIMEOUT);
      return false;
    }
    if ((it & 63u) == 63u && (*status & QX_DEV_TIMEOUT)) return false;
    __nanosleep(64);
  }
}

struct Smem {       // fixed part of the dynamic shared memory, before the rings
  alignas(16) uint8_t one_atom[512];   // e4m3 1.0 scale atom (gate/up activation scales)
  uint64_t full[MAXNS], empty[MAXNS], acc_full[2], acc_empty[2], meta_full[NI], meta_empty[NI];
  ItemMeta meta[NI];
  uint64_t drain[NISS];
  uint64_t init_bar;
  uint64_t tm_done;           // every epilogue warp's last TMEM read is complete
  uint32_t tmem_base, prod_scratch, mma_scratch[NISS];   // scratch: status words of drain waits
  uint32_t last_flag[NEPI];
  float amx[NEPI][GMAX][2];   // per epilogue group, pair, half: |act| maximum
  int32_t em[NEPI][GMAX];     // down item: the group's common activation exponents
  int32_t xe[NEPI][GMAX];     // gate/up item: the group's rows' x exponents
  float tws[NEPI][GMAX];      // down item: the group's routing weights
  uint32_t xcall[NEPI];       // fused combine: the call number of the unit in hand
  RouteHdr hdr;
};

// After an abort: wait (bounded) until the copies of the last ring round have
// landed, so none writes into shared memory after the CTA has left.
__device__ void drain_copies(const Params& p, Smem& S, uint32_t sc) {
  const uint64_t grace = globaltimer_ns() + p.timeout_ns;
  S.prod_scratch = 0;
  const uint32_t first = sc > (uint32_t)p.ns ? sc - (uint32_t)p.ns : 0u;
  for (uint32_t i = first; i < sc; ++i)
    mbar_wait_bounded(&S.full[i % p.ns], (i / p.ns) & 1, &S.prod_scratch, 1u, grace);
}

__device__ void producer(const Params& p, uint8_t* ring, Smem& S, const GroupS* gs, const PairS* ps,
                         const RouteHdr& hdr, volatile uint32_t* status, uint64_t deadline) {
  const uint32_t n1 = (uint32_t)hdr.n1, n2 = (uint32_t)hdr.n2, n1s = (uint32_t)hdr.n1s, n2s = (uint32_t)hdr.n2s;
  const int G = hdr.n_groups;
  uint32_t sc = 0, mc = 0;
  // ring position of stage sc, kept incrementally: slot = sc % ns, and the
  // parity of the slot's previous use, ((sc / ns) - 1) & 1, for sc >= ns
  int slot = 0;
  uint32_t prev_phase = 1u;
  int seen_a = -1;                    // last group whose activation flag was seen set
  bool ok = true, prep_seen = false;  // prep_seen: the prep kernel's results are visible
  uint32_t item = blockIdx.x;         // the first item is static, the rest come from the queue
  uint32_t cl_next = 0, cl_end = 0;   // items claimed and not yet started: [cl_next, cl_end)
  // Routed down items of one or two stages are claimed in batches (of 4 or 2),
  // so the queue's round trip is paid once per batch, except near the queue's
  // end; longer items (and the shared expert's, which come first) one at a time.
  const int nst2 = (p.NT + SK - 1) / SK;
  const uint32_t dclaim = nst2 == 1 ? 4u : nst2 == 2 ? 2u : 1u;
  for (;;) {
    ItemMeta m = {};
    if (!ok || item >= n1 + n2) {
      m.kind = 0;
    } else if (item < n1) {
      // Gate/up items: the shared expert's first, then the routed groups'; of
      // each, the whole items, then the pieces of the split ones (pieces of one
      // (group, tile) are consecutive, so they run side by side).
      const bool sh = item < n1s;
      const uint32_t nt = (uint32_t)(sh ? p.sNT : p.NT), fw = (uint32_t)(sh ? hdr.fws : hdr.fw);
      const uint32_t loc = sh ? item : item - n1s;
      uint32_t it = loc, ks = 1, piece = 0;
      if (loc >= fw) {
        ks = (uint32_t)(sh ? hdr.kss : hdr.ks);
        it = fw + (loc - fw) / ks;
        piece = (loc - fw) % ks;
      }
      m.kind = 1;
      m.group = (int)(it / nt) + (sh ? G : 0);
      m.tile = (int)(it % nt);
      m.piece = (int)piece;
      m.ks = (int)ks;
      m.gi = (int)(it - fw) + (sh ? MAXSPLIT : 0);
      m.nst = (KB1 / SK) / (int)ks;
      m.nkb_last = SK;
    } else {
      // Down items: the shared expert's groups first, then the routed groups.
      const bool sh = item - n1 < n2s;
      const uint32_t loc = sh ? item - n1 : item - n1 - n2s;
      const int nt = sh ? p.sNT : p.NT;
      m.kind = 2;
      m.group = (int)(loc / HT) + (sh ? G : 0);
      m.tile = (int)(loc % HT);
      m.nst = (nt + SK - 1) / SK;
      m.nkb_last = nt - (m.nst - 1) * SK;
    }
    const int mi = (int)(mc % NI);
    if (mc >= (uint32_t)NI &&
        !mbar_wait_bounded(&S.meta_empty[mi], ((mc / NI) - 1) & 1, status, QX_DEV_TIMEOUT, deadline)) {
      drain_copies(p, S, sc);
      return;
    }
    S.meta[mi] = m;
    mbar_arrive(&S.meta_full[mi]);
    ++mc;
    if (m.kind == 0) {
      // A second end marker: the epilogue groups take alternate entries.
      const int mi2 = (int)(mc % NI);
      if (mc < (uint32_t)NI ||
          mbar_wait_bounded(&S.meta_empty[mi2], ((mc / NI) - 1) & 1, status, QX_DEV_TIMEOUT, deadline)) {
        S.meta[mi2] = m;
        mbar_arrive(&S.meta_full[mi2]);
      }
      if (!prep_seen) pdl_wait();
      if (!ok) drain_copies(p, S, sc);
      return;
    }
    const GroupS& gr = gs[m.group];
    const Geo geo = geo_of(p, gr);
    const int sbs = gr.sbs;
    const uint8_t* a_src = m.kind == 1
                               ? geo.w13 + ((size_t)gr.expert * geo.NTA + geo.tile0 + m.tile) * (size_t)KB1 * A_KB +
                                     (size_t)m.piece * m.nst * SK * A_KB
                               : geo.w2 + (((size_t)gr.expert * HT + m.tile) * geo.NTA + geo.tile0) * (size_t)A_KB;
    // Weights of the CTA's first stages go out before the prep kernel is waited
    // for: they depend on the routing only (the ring is empty, so every slot is free).
    const int pre = prep_seen ? 0 : min(m.nst, p.ns);
    for (int s = 0; s < pre; ++s) {
      const int nkb = s < m.nst - 1 ? SK : m.nkb_last;
      mbar_arrive_expect_tx(&S.full[s], (uint32_t)(nkb * A_KB + sbs));
      bulk_g2s(ring + (size_t)s * A_STAGE, a_src + (size_t)s * SK * A_KB, (uint32_t)(nkb * A_KB), &S.full[s]);
    }
    if (!prep_seen) {
      pdl_wait();
      fence_proxy_async_global();
      prep_seen = true;
    }
    // The following item: the next of the batch in hand, or claimed from the
    // queue now. The queue's answer is first used after this item's copies are
    // issued, so its round trip overlaps them.
    uint32_t next = 0, claim_k = 0, claimed = 0;
    if (cl_next < cl_end) {
      next = cl_next++;
    } else {
      // batches while more than one batch per CTA is left, then single items,
      // so the last items spread over the CTAs (a batch would leave up to
      // dclaim - 1 items of tail on one CTA)
      claim_k = item >= n1 + n2s && (n1 + n2) - item > dclaim * gridDim.x ? dclaim : 1u;
      claimed = atomicAdd(&p.ctl->work, claim_k);
    }
    bool check = m.kind == 2 && seen_a != m.group;
    // gate/up: the pairs' x-term rows, the item's first stage (the per-stage
    // loop below issues their copies with no table reads)
    const uint8_t* xsrc[GMAX];
#pragma unroll
    for (int q = 0; q < GMAX; ++q)
      xsrc[q] = m.kind == 1 && q < gr.gsz
                    ? p.xt + ((size_t)ps[gr.pair_off + q].row * NXCH + m.piece * m.nst) * XT_STAGE
                    : p.xt;
    const int ns = p.ns;
    // every exit of a stage (end, continue, break) advances sc and its slot together
    for (int s = 0; s < m.nst; ++s, ++sc, (++slot == ns ? (slot = 0, prev_phase ^= 1u) : 0u)) {
      if (s >= pre) {
        // slot (weights + activation operand) free once stage sc - ns completed
        if (sc >= (uint32_t)p.ns &&
            !mbar_wait_bounded(&S.empty[slot], prev_phase, status, QX_DEV_TIMEOUT, deadline)) {
          ok = false;
          break;
        }
        const int nkb = s < m.nst - 1 ? SK : m.nkb_last;
        mbar_arrive_expect_tx(&S.full[slot], (uint32_t)(nkb * A_KB + sbs));
        bulk_g2s(ring + (size_t)slot * A_STAGE, a_src + (size_t)s * SK * A_KB, (uint32_t)(nkb * A_KB),
                 &S.full[slot]);
      }
      uint8_t* bdst = ring + p.b_off + (size_t)slot * p.bst;
      if (m.kind == 1) {
        // gate/up: each pair's row-major x-term block of this stage
#pragma unroll
        for (int q = 0; q < GMAX; ++q)
          if (q < gr.gsz)
            bulk_g2s(bdst + q * XT_STAGE, xsrc[q] + (size_t)s * XT_STAGE, (uint32_t)XT_STAGE, &S.full[slot]);
        continue;
      }
      if (check) {
        // The weights of this stage are already in flight; the activation
        // operand waits for its producer. On a timeout the copy is still issued
        // (of stale bytes) so the stage completes and nothing is left pending.
        // fixed exponent: the group's terms are final once all its tiles are
        // counted; else its last tile's fixup releases the ready flag
        const bool got = p.ae_fixed ? wait_flag(&p.cnt1[m.group], (uint32_t)geo.NT + p.dep_extra, status, deadline)
                                    : wait_flag(&p.ready[m.group], 1u + p.dep_extra, status, deadline);
        if (!got) ok = false;
        fence_proxy_async_global();
        check = false;
        if (ok) seen_a = m.group;
      }
      bulk_g2s(bdst, p.ab + gr.ab_off + (size_t)s * sbs, (uint32_t)sbs, &S.full[slot]);
      if (!ok) {
        ++sc;   // this stage's copies are issued: drain_copies waits for them
        break;
      }
    }
    if (claim_k) {
      next = gridDim.x + claimed;
      cl_next = next + 1;
      cl_end = next + claim_k;
    }
    item = next;
  }
}

// Issuer `iss` of its half of every stage's K blocks into accumulator (buffer,
// iss). Both issuers consume every stage and item in the same order.
__device__ void mma_issuer(const Params& p, uint8_t* ring, Smem& S, const GroupS* gs, uint32_t tbase, int iss,
                           volatile uint32_t* status, uint64_t deadline) {
  uint32_t sc = 0, mc = 0, ic = 0;
  // ring position of stage sc, kept incrementally: slot = sc % ns, phase = (sc / ns) & 1
  int slot = 0;
  uint32_t phase = 0;
  const uint32_t ns = (uint32_t)p.ns;
  const uint32_t sfbase = tbase + TM_SF + (uint32_t)iss * TM_SLOT;
  for (;;) {
    const int mi = (int)(mc % NI);
    if (!mbar_wait_bounded(&S.meta_full[mi], (mc / NI) & 1, status, QX_DEV_TIMEOUT, deadline)) break;
    const ItemMeta m = S.meta[mi];
    mbar_arrive(&S.meta_empty[mi]);
    ++mc;
    if (m.kind == 0) break;
    const GroupS& gr = gs[m.group];
    const uint32_t idesc = tc::idesc_nvf4((uint32_t)gr.n);
    const int buf = (int)(ic & 1u);
    if (ic >= 2 && !mbar_wait_bounded(&S.acc_empty[buf], ((ic / 2) - 1) & 1, status, QX_DEV_TIMEOUT, deadline))
      break;
    tc::fence_after_sync();
    const uint32_t tacc = tbase + (uint32_t)buf * 2u * TM_SLOT + (uint32_t)iss * TM_SLOT;
    bool ok = true, first = true;
    for (int s = 0; s < m.nst; ++s, ++sc) {
      // The stage's operands were written by the bulk copies (async proxy) the
      // barrier tracks; the MMAs read them through the same proxy, so the wait
      // alone orders them (no thread-sync fence, as for any TMA-fed stage).
      if (!mbar_wait_bounded(&S.full[slot], phase, status, QX_DEV_TIMEOUT, deadline)) {
        ok = false;
        break;
      }
      const int nkb = s < m.nst - 1 ? SK : m.nkb_last;
      const int k0 = iss ? (nkb + 1) >> 1 : 0, k1 = iss ? nkb : (nkb + 1) >> 1;   // <= KB_PER_ISS each
      const uint32_t a0 = smem_u32(ring + (size_t)slot * A_STAGE);
      const uint32_t b0 = smem_u32(ring + p.b_off + (size_t)slot * p.bst);
      const uint32_t bank = sfbase + (sc & 1u) * TM_BANK;
      for (int kb = k0; kb < k1; ++kb)     // this issuer's weight scale atoms of the stage first ...
        tc::cp_sf_atom(bank + 4 * (uint32_t)(kb - k0), a0 + kb * A_KB + 128 * tc::ROWB);
      for (int kb = k0; kb < k1; ++kb) {   // ... then its MMAs (activation scales: the constant atom)
        const uint32_t sa = a0 + kb * A_KB, sbb = b0 + kb * XT_KB;
        tc::mma_nvf4(tacc, tc::sdesc(sa, tc::LBO, tc::SBO), tc::sdesc(sbb, tc::LBO, XT_SBO), idesc,
                     bank + 4 * (uint32_t)(kb - k0), tbase + TM_ONE, first ? 0u : 1u);
        first = false;
      }
      tc::commit(&S.empty[slot]);          // arrives when this issuer's work on the stage is done
      if (++slot == (int)ns) {
        slot = 0;
        phase ^= 1u;
      }
    }
    if (!ok) break;
    tc::commit(&S.acc_full[buf]);
    ++ic;
  }
  // Let every tensor-core operation this thread issued complete before TMEM is freed.
  tc::commit(&S.drain[iss]);
  S.mma_scratch[iss] = 0;
  mbar_wait_bounded(&S.drain[iss], 0, &S.mma_scratch[iss], 1u, globaltimer_ns() + p.timeout_ns);
}

// Whether issuer 1 wrote its accumulator for an item (it owns the upper half,
// ceil(nkb / 2) onwards, of the K blocks of each stage).
__device__ __forceinline__ bool second_acc(const ItemMeta& m) { return m.nst > 1 || m.nkb_last > 1; }


// One finalize unit: output columns [128 tile, 128 tile + 128) of rows
// [4 rb, 4 rb + 4), by one epilogue group (et = 0..127), once every routed
// pair's y covers the tile. Thread et takes 4 consecutive outputs (column k) of
// row 4 rb + et / 32: bf16(sum over slots j in order of y[row * topk + j][k]),
// a slot without a valid expert adding 0. Returns the 4 BF16 values (zeros for a
// row past the post's last).
__device__ uint2 unit_partial(const Params& p, int tile, int rb, int et, int& row, int& k) {
  k = tile * 128 + 4 * (et & 31);
  row = 4 * rb + (et >> 5);
  if (row >= p.rows) return make_uint2(0u, 0u);
  float4 v[QX_MAX_TOPK];
  bool val[QX_MAX_TOPK];
#pragma unroll
  for (int j = 0; j < QX_MAX_TOPK; ++j) {   // ids and y loads issued together
    val[j] = false;
    v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (j < p.topk) {
      const int q = row * p.topk + j;
      const long long id = p.ids64 ? __ldg(reinterpret_cast<const long long*>(p.ids) + q)
                                   : (long long)__ldg(reinterpret_cast<const int*>(p.ids) + q);
      val[j] = id >= 0 && id < p.E;
      v[j] = __ldcg(reinterpret_cast<const float4*>(p.y + (size_t)q * HID + k));
    }
  }
  float4 s = val[0] ? v[0] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int j = 1; j < QX_MAX_TOPK; ++j) {
    const float4 z = val[j] ? v[j] : make_float4(0.f, 0.f, 0.f, 0.f);
    s.x += z.x;
    s.y += z.y;
    s.z += z.z;
    s.w += z.w;
  }
  const __nv_bfloat162 lo = __floats2bfloat162_rn(s.x, s.y), hi = __floats2bfloat162_rn(s.z, s.w);
  return make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
}

// Rank r's exchange buffer, chosen without indexing the parameter array at run
// time (which would copy the parameters to local memory).
__device__ __forceinline__ uint8_t* xbuf_at(const Params& p, int r) {
  uint8_t* b = p.xbuf[0];
#pragma unroll
  for (int i = 1; i < QX_XCHG_MAX_RANKS; ++i)
    if (r == i) b = p.xbuf[i];
  return b;
}

__device__ __forceinline__ void add4(float (&s)[4], uint2 v) {
  s[0] += __uint_as_float(v.x << 16);
  s[1] += __uint_as_float(v.x & 0xffff0000u);
  s[2] += __uint_as_float(v.y << 16);
  s[3] += __uint_as_float(v.y & 0xffff0000u);
}

__device__ __forceinline__ uint2 pack_bf16x4(const float (&s)[4]) {
  const __nv_bfloat162 lo = __floats2bfloat162_rn(s[0], s[1]), hi = __floats2bfloat162_rn(s[2], s[3]);
  return make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
}

// The shared expert's BF16 output at (row, k..k+3): its one slot, weight 1,
// rounded once, as a call of its arena alone would write it.
__device__ __forceinline__ uint2 shared_partial(const Params& p, int row, int k) {
  const float4 v = __ldcg(reinterpret_cast<const float4*>(p.y + (size_t)(p.P + row) * HID + k));
  const float s[4] = {v.x, v.y, v.z, v.w};
  return pack_bf16x4(s);
}

// Finalize unit u (tile, rb). Alone, it writes the output. In the fused rank
// combine a sender, once the output rank has acknowledged its use of the same
// receive words two calls ago, stores each thread's 8 BF16 bytes as two 64-bit
// words {data, call} straight into the output rank's buffer (plain stores over
// NVLink; a word validates itself, so no fence and no flag); the output rank
// polls every sender's words for the call, sums the ranks' BF16 partials in
// FP32 in rank order (then the shared-expert partial) with one BF16 rounding
// (native/qmesh_afd_seam.cu:309-361) and acknowledges. Every wait is bounded;
// false when one ran out (QX_DEV_TIMEOUT recorded).
__device__ bool finalize_unit(const Params& p, Smem& S, int u, int tile, int rb, int et, int eg, int B1,
                              uint32_t* status, uint64_t deadline) {
  using namespace xb;
  int row, k;
  const uint2 mine = unit_partial(p, tile, rb, et, row, k);
  const bool has = row < p.rows;
  if (p.xworld == 0) {
    if (has) {
      uint2 o = mine;
      if (p.sNT > 0) {   // bf16(routed + shared) in FP32, the combine's order
        float s[4] = {0.f, 0.f, 0.f, 0.f};
        add4(s, mine);
        add4(s, shared_partial(p, row, k));
        o = pack_bf16x4(s);
      }
      *reinterpret_cast<uint2*>(p.out + (size_t)row * p.out_stride + k) = o;
    }
    return true;
  }
  Hdr* me = reinterpret_cast<Hdr*>(xbuf_at(p, p.xrank));
  bool ok = true;
  if (et == 0) S.xcall[eg] = __ldcg(&me->useq[u]) + 1u;
  if (p.xrank != p.xdst) {
    if (et == 0) {
      const uint32_t call = S.xcall[eg];
      ok = call <= 2u || wait_at_least(&me->uack[u], call - 2u, status, deadline);
    }
    if (!bar_and(B1, 128, ok)) return false;
    const uint32_t call = S.xcall[eg];
    if (has) {
      uint64_t* w = words_of(xbuf_at(p, p.xdst), call, p.xrank, p.xrows_max, row, k);
      st_relaxed_sys_b64(w, (uint64_t)call << 32 | mine.x);
      st_relaxed_sys_b64(w + 1, (uint64_t)call << 32 | mine.y);
    }
    if (et == 0) me->useq[u] = call;
    return true;
  }
  asm volatile("bar.sync %0, 128;" ::"r"(B1) : "memory");
  const uint32_t call = S.xcall[eg];
  if (has) {
    uint8_t* own = xbuf_at(p, p.xrank);
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    // Every sender's words are requested at once (one round trip for all ranks);
    // those not yet carrying this call are then polled, in rank order.
    uint64_t wa[QX_XCHG_MAX_RANKS], wb[QX_XCHG_MAX_RANKS];
#pragma unroll
    for (int r = 0; r < QX_XCHG_MAX_RANKS; ++r) {
      if (r < p.xworld && r != p.xdst) {
        const uint64_t* w = words_of(own, call, r, p.xrows_max, row, k);
        wa[r] = ld_relaxed_sys_b64(w);
        wb[r] = ld_relaxed_sys_b64(w + 1);
      }
    }
#pragma unroll
    for (int r = 0; r < QX_XCHG_MAX_RANKS; ++r) {
      if (r >= p.xworld || !ok) continue;
      uint2 v = mine;
      if (r != p.xdst) {
        if ((uint32_t)(wa[r] >> 32) == call && (uint32_t)(wb[r] >> 32) == call)
          v = make_uint2((uint32_t)wa[r], (uint32_t)wb[r]);
        else
          ok = words_wait(words_of(own, call, r, p.xrows_max, row, k), call, v, status, deadline);
      }
      add4(s, v);
    }
    if (p.xshared) add4(s, *reinterpret_cast<const uint2*>(p.xshared + (size_t)row * p.xshared_stride + k));
    else if (p.sNT > 0) add4(s, shared_partial(p, row, k));
    const __nv_bfloat162 lo = __floats2bfloat162_rn(s[0], s[1]), hi = __floats2bfloat162_rn(s[2], s[3]);
    if (ok)
      *reinterpret_cast<uint2*>(p.out + (size_t)row * p.out_stride + k) =
          make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
  }
  // Every word read above has returned its value: the senders may reuse them.
  if (!bar_and(B1, 128, ok)) return false;
  if (et < p.xworld && et != p.xdst) ack_after_reads(&reinterpret_cast<Hdr*>(xbuf_at(p, et))->uack[u], call);
  if (et == 0) me->useq[u] = call;
  return true;
}

// Epilogue warpgroup eg (warps 2-5 or 7-10): the items of accumulator buffer
// eg, i.e. every other item. Named barriers 1 + 2 eg (its 128 threads) and
// 2 + 2 eg (its gate half).
__device__ void epilogue(const Params& p, Smem& S, float* xg, const GroupS* gs, const PairS* ps, uint32_t tbase,
                         int eg, volatile uint32_t* status, uint64_t deadline) {
  xg += eg * 2 * p.gmax * 64;
  float* xu = xg + p.gmax * 64;                  // gate and up values of a gate/up item, [pair][column]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int et = threadIdx.x - (eg ? 224 : 64);    // 0..127
  const int B1 = 1 + 2 * eg;                       // this group's 128-thread barrier
  const int quarter = warp & 3;                    // TMEM lane quarter this warp may read
  const int m = quarter * 32 + lane;               // accumulator row
  const uint32_t lanes = (uint32_t)(quarter * 32) << 16;

  pdl_wait();                                       // x exponents, reset counters

  uint32_t* last_flag = &S.last_flag[eg];
  float(*amx)[2] = S.amx[eg];
  int32_t* em = S.em[eg];
  int32_t* xe_s = S.xe[eg];
  float* tws = S.tws[eg];
  // The group whose down-item values (routing weights, common exponents, g2) this
  // warpgroup holds: consecutive down items of one group fetch them once.
  int dgrp = -1;
  float g2c = 0.f;
  for (uint32_t ic = (uint32_t)eg;; ic += NEPI) {   // item ic = meta entry ic
    const uint32_t mc = ic;
    const int mi = (int)(mc % NI);
    const bool got = mbar_wait_bounded(&S.meta_full[mi], (mc / NI) & 1, status, QX_DEV_TIMEOUT, deadline);
    const ItemMeta mt = S.meta[mi];
    if (!bar_and(B1, 128, got)) break;
    if (et == 0) mbar_arrive(&S.meta_empty[mi]);
    if (mt.kind == 0) break;
    const GroupS& gr = gs[mt.group];
    const Geo geo = geo_of(p, gr);
    bool ok = true;
    if (mt.kind == 1 && et < gr.gsz)   // the rows' x exponents, fetched while the MMAs run
      xe_s[et] = __ldcg(&p.xexp[ps[gr.pair_off + et].row]);
    if (mt.kind == 2 && mt.group != dgrp) {
      // A new group's g2, routing weights (1 for the shared expert) and common
      // exponents, fetched while the MMAs run.
      g2c = __ldg(gr.shared ? p.sg2 : &p.g2[gr.expert]);
      if (et < gr.gsz) {
        const int pq = ps[gr.pair_off + et].pq;
        tws[et] = pq < p.P ? __ldg(&p.tw[pq]) : 1.f;
        if (p.ae_fixed) {
          em[et] = p.ae_val;           // every tile's exponent; the producer waited for the terms
        } else {
          ok = wait_flag(&p.ready[mt.group], 1u + p.dep_extra, status, deadline);
          em[et] = __ldcg(&p.emax[gr.pair_off + et]);
        }
      }
      dgrp = mt.group;                 // on a failed wait the loop ends below
    }
    // The expert's global scale: g13 for a gate/up item (fetched while its MMAs run), g2 for a down item.
    const float gsc = mt.kind == 1 ? __ldg(gr.shared ? p.sg13 : &p.g13[gr.expert]) : g2c;
    const int buf = eg;
    ok = mbar_wait_bounded(&S.acc_full[buf], (ic / 2) & 1, status, QX_DEV_TIMEOUT, deadline) && ok;
    if (!bar_and(B1, 128, ok)) break;
    tc::fence_after_sync();
    const uint32_t tacc = tbase + lanes + (uint32_t)buf * 2u * TM_SLOT;   // issuer 1's at + TM_SLOT
    const bool two = second_acc(mt);
    if (mt.kind == 1) {
      // ---- gate/up tile: rows 0..63 gate, 64..127 up of columns [64 tile, 64 tile + 64)
      const bool up = m >= 64;
      const int c = m & 63;
      const int ks = mt.ks;
      // a split item's counter, and its pieces' sums: routed items from 0, the shared expert's after MAXSPLIT
      const size_t gi = (size_t)mt.gi;
      const size_t gp0 = gi >= (size_t)MAXSPLIT ? (size_t)MAXSPLIT + (gi - MAXSPLIT) * ks : gi * ks;
      for (int q = 0; q < gr.gsz; ++q) {
        float v[16], v1[16];
        tc::ld16x2(tacc + XTERMS * q, tacc + TM_SLOT + XTERMS * q, v, v1);   // v1 holds data only if two
#pragma unroll
        for (int t = 0; t < XTERMS; ++t) v[t] += two ? v1[t] : 0.f;
        const float s = tc::term_sum16(v, xe_s[q]);
        if (ks > 1) __stcg(p.gpart + ((gp0 + mt.piece) * GMAX + q) * 128 + m, s);
        else if (up) xu[q * 64 + c] = s * gsc;
        else xg[q * 64 + c] = s * gsc;
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.acc_empty[buf]);
      if (ks > 1) {
        // A piece of a K-split item: its sums are stored (ordered before thread
        // 0's acq_rel count by the barrier); the item's last piece adds every
        // piece's sums in piece order and goes on with the tile.
        asm volatile("bar.sync %0, 128;" ::"r"(B1) : "memory");
        if (et == 0) *last_flag = atom_add_acq_rel_gpu(&p.pcnt[gi], 1u) == (uint32_t)ks - 1u ? 1u : 0u;
        asm volatile("bar.sync %0, 128;" ::"r"(B1) : "memory");
        if (!*last_flag) continue;
        const float* g0 = p.gpart + gp0 * GMAX * 128 + m;
        for (int q = 0; q < gr.gsz; ++q) {
          float s = 0.f;
          for (int pc = 0; pc < ks; ++pc) s += __ldcg(g0 + ((size_t)pc * GMAX + q) * 128);
          if (up) xu[q * 64 + c] = s * gsc; else xg[q * 64 + c] = s * gsc;
        }
      }
      asm volatile("bar.sync %0, 128;" ::"r"(B1) : "memory");
      const int col0 = mt.tile * 64;
      const int kbl = mt.tile % SK;                   // the tile is K block kbl of down stage tile / SK
      uint8_t* ab = p.ab + gr.ab_off + (size_t)(mt.tile / SK) * gr.sbs;
      if (!up) {
        // SwiGLU per pair, |act| maxima per half tile
        const int half = warp & 1;   // quarters 0, 1 <-> columns 0..31, 32..63
        for (int q = 0; q < gr.gsz; ++q) {
          float g = xg[q * 64 + c], u = xu[q * 64 + c];
          if (p.has_limit) {
            g = fminf(g, p.limit);
            u = fminf(fmaxf(u, -p.limit), p.limit);
          }
          float a = (g / (1.f + expf(-g))) * u;
          if (col0 + c >= geo.W) a = 0.f;
          xg[q * 64 + c] = a;
          if (p.ae_fixed) continue;          // the exponent is known: no maximum needed
          float mx = fabsf(a);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
          if (lane == 0) amx[q][half] = mx;
        }
      }
      asm volatile("bar.sync %0, 128;" ::"r"(B1) : "memory");
      // 16 unscaled e2m1 terms per pair with the tile's exponent el (fixed, or
      // the tile's own even one): act = sum_t 2^(el - 2t) q_t (the digit rule of
      // the x terms). Warp w of the group takes pairs w, w + 4; lane l the
      // columns 2l, 2l + 1.
      for (int q = et >> 5; q < gr.gsz; q += 4) {
        const int el = p.ae_fixed ? p.ae_val : act_exponent(fmaxf(amx[q][0], amx[q][1]));
        float r0 = xg[q * 64 + 2 * lane], r1 = xg[q * 64 + 2 * lane + 1];
        uint8_t* blk = ab + (size_t)q * XT_STAGE + kbl * XT_KB + (lane >> 4) * 128 + (lane & 12);
        float g = tc::exp2i(el), ig = tc::exp2i(-el);
#pragma unroll
        for (int t = 0; t < XTERMS; ++t) {
          const uint32_t w = tc::pack4(tc::digit2(r0, r1, g, ig), lane);
          if ((lane & 3) == 0) *reinterpret_cast<uint32_t*>(blk + (t >> 3) * XT_SBO + (t & 7) * 16) = w;
          g *= 0.25f;
          ig *= 4.f;
        }
        if (lane == 0) {
          p.eloc[(size_t)(gr.pair_off + q) * MAX_STILES + mt.tile] = el;
          atomicMax(&p.emax[gr.pair_off + q], el);
        }
      }
      // The group's stores are ordered before thread 0's release by the barrier.
      asm volatile("bar.sync %0, 128;" ::"r"(B1) : "memory");
      if (p.ae_fixed) {
        // Every tile is on the one exponent: count the tile (release, no reply
        // awaited); the group's down items wait until every tile is counted.
        if (et == 0) red_add_release_gpu(&p.cnt1[mt.group], 1u);
        continue;
      }
      // Per-tile exponents: the group's last tile (found by the count, acq_rel)
      // fixes the group's terms up to a common exponent and releases them.
      if (et == 0) {
        const uint32_t old = atom_add_acq_rel_gpu(&p.cnt1[mt.group], 1u);
        *last_flag = (old == (uint32_t)geo.NT - 1u) ? 1u : 0u;
      }
      asm volatile("bar.sync %0, 128;" ::"r"(B1) : "memory");
      if (*last_flag) {
        // Last tile of the group: bring every tile to the pair's common exponent
        // em by moving its terms d = (em - el) / 2 places down (term t becomes
        // term t + d; the last d terms, below the common precision, drop out).
        // Shifts of all (tile, pair) items first (into the exchange area, free
        // now; NT x gsz <= 64 gmax), then one item per warp and lane = (K half,
        // term) owning 16 code bytes, four items in flight per warp.
        int* dsh = reinterpret_cast<int*>(xg);
        const int nit = geo.NT * gr.gsz;
        for (int i = et; i < nit; i += 128) {
          const int tile = i / gr.gsz, q = i - tile * gr.gsz;
          dsh[i] = (__ldcg(&p.emax[gr.pair_off + q]) -
                    __ldcg(&p.eloc[(size_t)(gr.pair_off + q) * MAX_STILES + tile])) >> 1;
        }
        asm volatile("bar.sync %0, 128;" ::"r"(B1) : "memory");
        const int ew = et >> 5, t = lane & 15, kh = lane >> 4;
        for (int i0 = 4 * ew; i0 < nit; i0 += 16) {
          int dd[4];
          uint4* wp[4];
          uint4 v[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int i = i0 + j;
            dd[j] = i < nit ? dsh[i] : 0;
            const int tile = i / gr.gsz, q = i - tile * gr.gsz;
            wp[j] = reinterpret_cast<uint4*>(p.ab + gr.ab_off + (size_t)(tile / SK) * gr.sbs + (size_t)q * XT_STAGE +
                                             (t >> 3) * XT_SBO + (tile % SK) * XT_KB + kh * 128 + (t & 7) * 16);
            if (dd[j] > 0) v[j] = __ldcg(wp[j]);
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (dd[j] <= 0) continue;          // warp-uniform
            const int d = dd[j];
            uint4 nv;
            nv.x = __shfl_up_sync(0xffffffffu, v[j].x, d & 15, 16);
            nv.y = __shfl_up_sync(0xffffffffu, v[j].y, d & 15, 16);
            nv.z = __shfl_up_sync(0xffffffffu, v[j].z, d & 15, 16);
            nv.w = __shfl_up_sync(0xffffffffu, v[j].w, d & 15, 16);
            if (t < d) nv = make_uint4(0u, 0u, 0u, 0u);
            __stcg(wp[j], nv);
          }
        }
        asm volatile("bar.sync %0, 128;" ::"r"(B1) : "memory");
        if (et == 0) st_release_gpu(&p.ready[mt.group], 1u);
      }
    } else {
      // ---- down tile: output rows [128 tile, 128 tile + 128)
      const int h = mt.tile * 128 + m;
      for (int q = 0; q < gr.gsz; ++q) {
        float v[16], v1[16];
        tc::ld16x2(tacc + XTERMS * q, tacc + TM_SLOT + XTERMS * q, v, v1);   // v1 holds data only if two
#pragma unroll
        for (int t = 0; t < XTERMS; ++t) v[t] += two ? v1[t] : 0.f;
        p.y[(size_t)ps[gr.pair_off + q].pq * HID + h] = tc::term_sum16(v, em[q]) * (gsc * tws[q]);
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.acc_empty[buf]);
      // The group's y stores are ordered before thread 0's release by the barrier:
      // the tile's counter counts the routed pairs whose y covers it.
      asm volatile("bar.sync %0, 128;" ::"r"(B1) : "memory");
      if (et == 0) red_add_release_gpu(&p.fcnt[mt.tile], (uint32_t)gr.gsz);
    }
  }
  // This warp reads TMEM no more: TMEM may be released once all epilogue warps say so.
  tc::fence_before_sync();
  __syncwarp();
  if (lane == 0) mbar_arrive(&S.tm_done);
  // Finalize units (output tile, block of 4 rows), dealt round robin over every
  // CTA's epilogue groups: each waits (bounded) until its tile's counter holds
  // every routed pair, then sums its rows. A post without a valid pair needs no
  // wait and writes zeros.
  const int rbn = (p.rows + 3) >> 2;
  for (int u = blockIdx.x * NEPI + eg; u < HT * rbn; u += gridDim.x * NEPI) {
    const int tile = u / rbn;
    bool ok = true;
    if (et == 0) ok = wait_flag(&p.fcnt[tile], (uint32_t)S.hdr.n_fin, status, deadline);
    if (!bar_and(B1, 128, ok)) break;   // every thread's y reads follow thread 0's acquire
    if (!finalize_unit(p, S, u, tile, u - tile * rbn, et, eg, B1, const_cast<uint32_t*>(status), deadline)) break;
  }
}

__global__ void __launch_bounds__(NTHR, 1) tc_decode_kernel(Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  Smem& S = *reinterpret_cast<Smem*>(smem);
  uint8_t* ring = smem + p.ring_off;
  float* xg = reinterpret_cast<float*>(smem + p.x_off);
  GroupS* gs = reinterpret_cast<GroupS*>(smem + p.tab_off);
  PairS* ps = reinterpret_cast<PairS*>(smem + p.tab_off + (size_t)(p.P + p.rows) * sizeof(GroupS));
  const int warp = threadIdx.x >> 5;
  volatile uint32_t* status = &p.ctl->status;
  // Warp 0 loads the call's expert ids while other warps set up the CTA.
  int idr[IDR];
  if (warp == 0) load_ids(p, threadIdx.x & 31, idr);
  if (threadIdx.x == 64) {
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
    mbar_init(&S.init_bar, 1);
    mbar_init(&S.tm_done, NEPI * 4);
    fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(&S.tmem_base, TM_COLS);
    tc::tmem_relinquish();
  }
  // Every CTA barrier below follows code that one lane of a warp ran alone: the
  // warp reconverges first, so that it arrives at the barrier once.
  __syncwarp();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (threadIdx.x == 32) {
    // The gate/up MMAs' activation scales: a constant atom of e4m3 1.0, copied
    // into TMEM before any issuer starts (bounded wait for the copy).
    for (int i = 0; i < 512 / 4; ++i) reinterpret_cast<uint32_t*>(S.one_atom)[i] = 0x38383838u;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc::cp_sf_atom(S.tmem_base + TM_ONE, smem_u32(S.one_atom));       // operand rows 0..127
    tc::cp_sf_atom(S.tmem_base + TM_ONE + 4, smem_u32(S.one_atom));   // rows 128..255
    tc::commit(&S.init_bar);
    S.mma_scratch[0] = 0;
    mbar_wait_bounded(&S.init_bar, 0, &S.mma_scratch[0], 1u, globaltimer_ns() + p.timeout_ns);
  }
  // The ids come from work before the prep kernel (which is launched without
  // early start), so the routing needs no wait; the prep kernel's results are
  // waited for by the threads that read them (producer, epilogue).
  if (warp == 0) route_local(p, idr, gs, ps, &S.hdr);
  pdl_launch_dependents();
  __syncwarp();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  {
    // Ring geometry from the largest group of this call: every slot holds one
    // weight stage and one activation stage of the widest operand.
    const int bmx = S.hdr.b_max;
    p.bst = bmx < 16 ? 16 : bmx;
    int ns = (p.ring_bytes - 512) / (A_STAGE + p.bst);   // 512: slack for the last scale-atom read
    p.ns = ns > MAXNS ? MAXNS : ns;
    p.b_off = p.ns * A_STAGE;
  }
  const uint32_t tbase = S.tmem_base;
  const uint64_t deadline = globaltimer_ns() + p.timeout_ns;
  if (warp == 0) {
    if ((threadIdx.x & 31) == 0) producer(p, ring, S, gs, ps, S.hdr, status, deadline);
  } else if (warp == 1 || warp == 6) {
    if ((threadIdx.x & 31) == 0) mma_issuer(p, ring, S, gs, tbase, warp == 1 ? 0 : 1, status, deadline);
  } else {
    epilogue(p, S, xg, gs, ps, tbase, warp < 6 ? 0 : 1, status, deadline);
  }
  // The producer drained its copies and the issuers their tensor-core work (all
  // bounded) before returning; the epilogue's last TMEM reads are complete.
  __syncwarp();
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    // TMEM is released after the epilogue warps' last reads (bounded wait).
    if ((threadIdx.x & 31) == 0) {
      S.mma_scratch[0] = 0;
      mbar_wait_bounded(&S.tm_done, 0, &S.mma_scratch[0], 1u, globaltimer_ns() + p.timeout_ns);
    }
    __syncwarp();
    tc::fence_after_sync();
    tc::tmem_dealloc(tbase, TM_COLS);
  }
}

// ------------------------------------------------------------------ host side
constexpr size_t SMEM_LIMIT = 232448;    // 227 KB per CTA

static int device_sms(int* dev_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  static int cached[64] = {0};
  static bool attr_set[64] = {false};
  if (dev < 0 || dev >= 64) return -1;
  if (cached[dev] == 0) {
    int major = 0, sms = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return -1;
    if (major != 10) return -1;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
    cached[dev] = sms;
  }
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(tc_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_LIMIT) !=
        cudaSuccess)
      return -1;
    attr_set[dev] = true;
  }
  *dev_out = dev;
  return cached[dev];
}

static uint64_t timeout_ns() {
  const char* e = getenv("QX_TIMEOUT_MS");
  long ms = e ? atol(e) : 1000;
  if (ms < 10) ms = 10;
  return (uint64_t)ms * 1000000ull;
}

// Test hook QX_TEST_DEP_EXTRA=n: every down item waits for a group flag value
// that is never reached, so the bounded wait runs out and QX_DEV_TIMEOUT is
// recorded.
static uint32_t dep_extra() {
  const char* e = getenv("QX_TEST_DEP_EXTRA");
  return e ? (uint32_t)atol(e) : 0u;
}

}  // namespace tcd
}  // namespace qx

using namespace qx::tcd;

extern "C" {

size_t qx_arena_tc_w13_bytes(int32_t n_experts, int32_t width) {
  if (n_experts <= 0 || width <= 0 || width % 32) return 0;
  return (size_t)n_experts * ((width + 63) / 64) * (size_t)KB1 * A_KB;
}

size_t qx_arena_tc_w2_bytes(int32_t n_experts, int32_t width) {
  if (n_experts <= 0 || width <= 0 || width % 32) return 0;
  return (size_t)n_experts * HT * (size_t)((width + 63) / 64) * A_KB;
}

size_t qx_slice_workspace_tc_bytes(int32_t rows, int32_t topk, int32_t c0, int32_t c1) {
  if (rows <= 0 || rows > QX_MAX_ROWS || topk <= 0 || topk > QX_MAX_TOPK || c1 <= c0 || (c1 - c0) % 32) return 0;
  return ws_layout(rows, topk, c1 - c0).total;
}

}  // extern "C"

// The slice call, alone (x == nullptr) or with the fused rank combine, and with
// the shared expert's arena (sh) on the output rank.
static int tc_launch(const QxArena* arena, const QxSliceArgs* a, const QxXchgArgs* x, const QxArena* sh,
                     void* stream) {
  if (!arena || !a) return QX_ERR_ARG;
  if (!a->x || !a->ids || !a->tw || !a->out || !a->workspace || !arena->w13 || !arena->w2 || !arena->g13 ||
      !arena->g2)
    return QX_ERR_ARG;
  if ((a->x_fmt == QX_X_E4M3 || a->x_fmt == QX_X_E4M3_POST) && !a->x_scale) return QX_ERR_ARG;
  if (a->x_fmt < QX_X_E4M3 || a->x_fmt > QX_X_BF16) return QX_ERR_ARG;
  if (a->rows < 1 || a->rows > QX_MAX_ROWS || a->topk < 1 || a->topk > QX_MAX_TOPK) return QX_ERR_SHAPE;
  if (arena->layout != QX_LAYOUT_TC) return QX_ERR_ARG;
  if (arena->n_experts < 1 || arena->n_experts > MAXE) return QX_ERR_SHAPE;
  if (a->c1 - a->c0 > 64 * 64) return QX_ERR_SHAPE;   // at most 64 column tiles per slice
  if (arena->a0 % 32 || arena->a1 % 32 || arena->a1 <= arena->a0) return QX_ERR_SHAPE;
  if ((a->c0 - arena->a0) % 64 || a->c1 % 32 || a->c0 < arena->a0 || a->c1 > arena->a1 || a->c1 <= a->c0)
    return QX_ERR_SHAPE;
  const int esz = a->x_fmt == QX_X_BF16 ? 2 : 1;
  if (a->x_stride < (int64_t)HID * esz || a->out_stride < HID) return QX_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(a->x) & 15u) || (a->x_stride & 15) ||
      (reinterpret_cast<uintptr_t>(a->workspace) & 255u) || (reinterpret_cast<uintptr_t>(arena->w13) & 15u) ||
      (reinterpret_cast<uintptr_t>(arena->w2) & 15u) || (reinterpret_cast<uintptr_t>(a->out) & 7u) ||
      (a->out_stride & 3))
    return QX_ERR_ALIGN;
  const int W = a->c1 - a->c0;
  const WsLayout L = ws_layout(a->rows, a->topk, W);
  if (a->workspace_bytes < L.total) return QX_ERR_WORKSPACE;
  int dev = 0;
  const int sms = device_sms(&dev);
  if (sms <= 0) return QX_ERR_DEVICE;

  Params p;
  p.x = a->x;
  p.x_scale = a->x_scale;
  p.x_stride = a->x_stride;
  p.x_fmt = a->x_fmt;
  p.ids = a->ids;
  p.ids64 = a->ids_int64 ? 1 : 0;
  p.tw = a->tw;
  p.rows = a->rows;
  p.topk = a->topk;
  p.P = a->rows * a->topk;
  p.W = W;
  p.NT = (W + 63) / 64;
  p.tile0 = (a->c0 - arena->a0) / 64;
  p.NTA = (arena->a1 - arena->a0 + 63) / 64;
  p.w13 = arena->w13;
  p.w2 = arena->w2;
  p.g13 = arena->g13;
  p.g2 = arena->g2;
  p.E = arena->n_experts;
  p.limit = a->swiglu_limit;
  p.has_limit = a->has_limit ? 1 : 0;
  p.out = reinterpret_cast<__nv_bfloat16*>(a->out);
  p.out_stride = a->out_stride;
  uint8_t* ws = reinterpret_cast<uint8_t*>(a->workspace);
  p.ctl = reinterpret_cast<Ctl*>(ws + L.ctl);
  p.cnt1 = reinterpret_cast<uint32_t*>(ws + L.cnt1);
  p.ready = reinterpret_cast<uint32_t*>(ws + L.ready);
  p.fcnt = reinterpret_cast<uint32_t*>(ws + L.fcnt);
  p.pcnt = reinterpret_cast<uint32_t*>(ws + L.pcnt);
  p.gpart = reinterpret_cast<float*>(ws + L.gpart);
  p.emax = reinterpret_cast<int32_t*>(ws + L.emax);
  p.eloc = reinterpret_cast<int32_t*>(ws + L.eloc);
  p.xexp = reinterpret_cast<int32_t*>(ws + L.xexp);
  p.xt = ws + L.xt;
  p.ab = ws + L.ab;
  p.y = reinterpret_cast<float*>(ws + L.y);
  p.gmax = a->rows < GMAX ? a->rows : GMAX;
  {
    p.bst = p.gmax * XT_STAGE;   // the widest possible group, for the shape check
  }
  // shared memory: [Smem][exchange][tables][rings: ns weight stages | ns activation stages]
  const size_t tables = (size_t)(p.P + p.rows) * (sizeof(GroupS) + sizeof(PairS));
  const size_t xchg = (size_t)NEPI * 2 * p.gmax * 64 * sizeof(float);
  p.x_off = (int)((sizeof(Smem) + 15) & ~size_t(15));
  p.tab_off = (int)(((size_t)p.x_off + xchg + 15) & ~size_t(15));
  p.ring_off = (int)(((size_t)p.tab_off + tables + 127) & ~size_t(127));
  p.ring_bytes = (int)(SMEM_LIMIT - (size_t)p.ring_off);
  if (p.ring_bytes - 512 < 2 * (A_STAGE + p.bst)) return QX_ERR_SHAPE;   // two slots of the widest group
  p.ns = p.b_off = 0;
  p.timeout_ns = timeout_ns();
  p.dep_extra = dep_extra();
  // With the clamp, |act| = |silu(min(g, L)) * clamp(u, -L, L)| <= L^2: one
  // exponent E with 6 * 2^E >= L^2 covers every tile, so the tiles' terms need
  // no common-exponent fixup. For L <= 16 the 16 terms then still resolve act
  // to 2^(E - 31) <= 2^-24, far below the BF16 rounding of the output.
  p.ae_fixed = 0;
  p.ae_val = 0;
  if (p.has_limit && p.limit > 0.f && p.limit <= 16.f) {
    const double bound = (double)p.limit * (double)p.limit * 1.001;
    int e = XE_LO;
    while (6.0 * ldexp(1.0, e) < bound) ++e;
    p.ae_fixed = 1;
    p.ae_val = e;
  }
  p.xworld = 0;
  p.xshared = nullptr;
  p.xshared_stride = 0;
  p.xrank = p.xdst = p.xrows_max = 0;
  for (int r = 0; r < QX_XCHG_MAX_RANKS; ++r) p.xbuf[r] = nullptr;
  if (x && x->world > 1) {
    if (x->world > QX_XCHG_MAX_RANKS || x->rank < 0 || x->rank >= x->world || x->dst < 0 || x->dst >= x->world)
      return QX_ERR_ARG;
    if (x->rows_max < a->rows || x->rows_max > QX_MAX_ROWS) return QX_ERR_SHAPE;
    for (int r = 0; r < x->world; ++r) {
      if (!x->bufs[r] || (reinterpret_cast<uintptr_t>(x->bufs[r]) & 255u)) return QX_ERR_ARG;
      p.xbuf[r] = reinterpret_cast<uint8_t*>(x->bufs[r]);
    }
    if (x->rank == x->dst && x->shared) {
      if ((reinterpret_cast<uintptr_t>(x->shared) & 7u) || (x->shared_stride & 3) || x->shared_stride < HID)
        return QX_ERR_ALIGN;
      p.xshared = reinterpret_cast<const __nv_bfloat16*>(x->shared);
      p.xshared_stride = x->shared_stride;
    }
    p.xworld = x->world;
    p.xrank = x->rank;
    p.xdst = x->dst;
    p.xrows_max = x->rows_max;
  }
  p.sw13 = p.sw2 = nullptr;
  p.sg13 = p.sg2 = nullptr;
  p.sW = p.sNT = 0;
  if (sh) {
    if (sh->layout != QX_LAYOUT_TC || sh->n_experts != 1 || !sh->w13 || !sh->w2 || !sh->g13 || !sh->g2)
      return QX_ERR_ARG;
    if (sh->a0 % 32 || sh->a1 % 32 || sh->a1 <= sh->a0 || sh->a1 - sh->a0 > MAX_STILES * 64) return QX_ERR_SHAPE;
    if ((reinterpret_cast<uintptr_t>(sh->w13) & 15u) || (reinterpret_cast<uintptr_t>(sh->w2) & 15u))
      return QX_ERR_ALIGN;
    // only the rank that writes the output adds the shared expert, and not twice
    if (p.xworld > 1 && (p.xrank != p.xdst || p.xshared)) return QX_ERR_ARG;
    p.sw13 = sh->w13;
    p.sw2 = sh->w2;
    p.sg13 = sh->g13;
    p.sg2 = sh->g2;
    p.sW = sh->a1 - sh->a0;
    p.sNT = (p.sW + 63) / 64;
  }
  const size_t smem_bytes = SMEM_LIMIT;

  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  tc_prep_kernel<<<a->rows * NXCH, PREP_THR, 0, st>>>(p);
  if (cudaGetLastError() != cudaSuccess) return QX_ERR_LAUNCH;

  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sms, 1, 1);
  cfg.blockDim = dim3(NTHR, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, tc_decode_kernel, p) != cudaSuccess) return QX_ERR_LAUNCH;
  return QX_OK;
}

extern "C" {

int qx_slice_decode_tc(const QxArena* arena, const QxSliceArgs* a, void* stream) {
  return tc_launch(arena, a, nullptr, nullptr, stream);
}

int qx_slice_decode_tc_xchg(const QxArena* arena, const QxSliceArgs* a, const QxXchgArgs* x, void* stream) {
  if (!x) return QX_ERR_ARG;
  return tc_launch(arena, a, x, nullptr, stream);
}

int qx_slice_decode_tc_shared(const QxArena* arena, const QxSliceArgs* a, const QxArena* shared,
                              const QxXchgArgs* x, void* stream) {
  if (!shared) return QX_ERR_ARG;
  return tc_launch(arena, a, x, shared, stream);
}

}  // extern "C"
