// tcgen05 (5th-generation tensor core) helpers for sm_100a: TMEM allocation,
// shared-memory matrix descriptors, the block-scaled NVFP4 MMA
// (kind::mxf4nvf4, e2m1 x e2m1 with one UE4M3 scale per 16 elements along K),
// scale-factor copies into TMEM, commits and accumulator loads.
//
// Operand layout used throughout (K-major, no swizzle): one MMA consumes K = 64
// e2m1 values per row = 32 bytes = two 16-byte "core matrix" columns. A tile of
// R rows (R % 8 == 0) for one 64-wide K block is stored as
//     [R/8 row groups][2 K halves][8 rows][16 bytes]
// so the core matrix of (row group g, half h) starts at g*256 + h*128 bytes:
// leading (K) byte offset 128, stride (row-group) byte offset 256. Inside the
// 16 bytes, element 2i is the low nibble of byte i.
//
// Scale factors of one 64-wide K block for up to 128 rows form a 512-byte atom:
// byte (row % 32) * 16 + (row / 32) * 4 + j holds the scale of elements
// [16j, 16j + 16) of `row`. `tcgen05.cp.32x128b.warpx4` places the atom's 32
// sixteen-byte lines in TMEM lanes 0..31 and copies them to the other three lane
// quarters, four 32-bit columns wide: the arrangement the MMA reads its scales
// from (lane = row % 32, byte = (row / 32) * 4 + j). For a B operand of more
// than 128 rows, rows [128a, 128a + 128) form atom a, copied to the next four
// columns (byte (row / 32) * 4 + j still holds for the 8-column span).
#pragma once

#include <stdint.h>

#include "qx_ptx.cuh"

namespace qx {
namespace tc {

constexpr uint32_t KBLK = 64;             // e2m1 elements per MMA along K
constexpr uint32_t ROWB = KBLK / 2;       // bytes per row per K block
constexpr uint32_t SF_ATOM = 512;         // scale bytes per K block (<= 128 rows)
constexpr uint32_t LBO = 128;             // K-half to K-half
constexpr uint32_t SBO = 256;             // row group to row group

// Byte offset of (row, k) inside one K block's operand tile (k in [0, 64)); the
// nibble is k & 1.
__host__ __device__ constexpr uint32_t opnd_off(uint32_t row, uint32_t k) {
  return (row >> 3) * SBO + (k >> 5) * LBO + (row & 7) * 16 + ((k & 31) >> 1);
}
// Byte offset of the scale of (row, 16-block j) inside one K block's atom.
__host__ __device__ constexpr uint32_t sf_off(uint32_t row, uint32_t j) {
  return (row & 31) * 16 + (row >> 5) * 4 + j;
}

// ---- TMEM allocation (warp-wide, .sync.aligned) --------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// ---- ordering between thread syncs and tcgen05 operations ----------------------
__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// ---- descriptors ---------------------------------------------------------------
// Shared-memory matrix descriptor, K-major, no swizzle (layout type 0),
// descriptor version 1, base offset 0.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  return d;
}

// Instruction descriptor of kind::mxf4nvf4: A and B e2m1 (format 1), UE4M3
// scales (bit 23 clear), both K-major, dense, M = 128, N = n (multiple of 16,
// 16..256), K = 64, scale-factor byte ids 0.
__host__ __device__ constexpr uint32_t idesc_nvf4(uint32_t n) {
  return (1u << 7) | (1u << 10) | ((n >> 3) << 17) | ((128u >> 4) << 24);
}

// ---- tensor-core operations (issued by one thread) -----------------------------
// D[tmem_d] (+)= (A * SFA) x (B * SFB)^T for one 64-wide K block.
__device__ __forceinline__ void mma_nvf4(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t tsfa, uint32_t tsfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n" ::"r"(
          tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb)
      : "memory");
}

// One 512-byte scale atom (32 lines x 16 bytes) from shared memory into TMEM
// lanes 0..127 (copied to all four lane quarters), 4 columns at `taddr`.
__device__ __forceinline__ void cp_sf_atom(uint32_t taddr, uint32_t saddr) {
  const uint64_t d = sdesc(saddr, 0, 128);
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(d) : "memory");
}

// Arrive once on `bar` when every tcgen05 operation this thread issued so far
// has completed (the operands in shared memory may then be overwritten and the
// accumulator read).
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ---- accumulator loads ----------------------------------------------------------
// Lane i of the calling warp receives TMEM lane (taddr.lane + i), 16
// consecutive 32-bit columns starting at taddr.col. The wait sits in the same
// asm statement so no use of the registers can be scheduled before it.
__device__ __forceinline__ void ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];\n\ttcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Two ld16 loads (e.g. the two issuers' accumulators) behind one wait.
__device__ __forceinline__ void ld16x2(uint32_t ta, uint32_t tb, float (&v)[16], float (&w)[16]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%32];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31}, [%33];\n\ttcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(ta), "r"(tb)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    v[i] = __uint_as_float(r[i]);
    w[i] = __uint_as_float(r[16 + i]);
  }
}

// As ld16, 8 columns.
__device__ __forceinline__ void ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// ---- NVFP4 encoders for operands built on the device ---------------------------
// Value of an e2m1 code (exact).
__device__ __forceinline__ float e2m1_val(uint32_t code) { return f16lo_to_f32(e2m1x2_to_f16x2(code & 15u)); }
// Value of an e4m3 byte (exact).
__device__ __forceinline__ float e4m3_val(uint32_t b) { return f16lo_to_f32(e4m3x2_to_f16x2(b & 0xFFu)); }

// Smallest e4m3 byte b with val(b) * g6 >= a (a >= 0; g6 = 6 * 2^k, inv_g6 its
// reciprocal); 0 for a == 0; 448 caps. The hardware round-to-nearest of the
// quotient estimate is at most one e4m3 step below the answer, and
// val(b) * g6 is exact, so one exact comparison settles it.
__device__ __forceinline__ uint32_t e4m3_ceil(float a, float g6, float inv_g6) {
  if (!(a > 0.f)) return 0u;
  uint32_t two;
  asm("{ .reg .b16 h; cvt.rn.satfinite.e4m3x2.f32 h, %1, %2; cvt.u32.u16 %0, h; }"
      : "=r"(two)
      : "f"(0.f), "f"(a * inv_g6));
  uint32_t b = two & 0xFFu;
  if (b < 0x7Eu && e4m3_val(b) * g6 < a) ++b;
  return b;
}

// e2m1 code of the exact quotient r / sg (|r| <= 6 sg), round to nearest with
// ties to the even code, by comparing |r| with the seven midpoints times sg
// (each product is exact). 0 when sg == 0.
__device__ __forceinline__ uint32_t e2m1_of(float r, float sg) {
  if (!(sg > 0.f)) return 0u;
  const float a = fabsf(r);
  uint32_t i = (a > 0.25f * sg) ? 1u : 0u;
  i += (a >= 0.75f * sg) ? 1u : 0u;
  i += (a > 1.25f * sg) ? 1u : 0u;
  i += (a >= 1.75f * sg) ? 1u : 0u;
  i += (a > 2.5f * sg) ? 1u : 0u;
  i += (a >= 3.5f * sg) ? 1u : 0u;
  i += (a > 5.f * sg) ? 1u : 0u;
  return i | ((__float_as_uint(r) >> 28) & 8u);
}

// One residual NVFP4 term of a 16-element block spread one element per lane over
// 16 consecutive lanes (lane groups 0-15 and 16-31 are independent blocks): the
// block scale byte (returned in *sb), the lane's e2m1 code (returned), and the
// residual update r -= code * scale * g, exact. g = 2^k.
__device__ __forceinline__ uint32_t term_step(float& r, float g, uint32_t* sb) {
  float a = fabsf(r);
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
  const float g6 = 6.f * g;
  const uint32_t b = e4m3_ceil(a, g6, __frcp_rn(g6));
  const float sg = e4m3_val(b) * g;
  const uint32_t code = e2m1_of(r, sg);
  r = fmaf(-e2m1_val(code), sg, r);
  *sb = b;
  return code;
}

// e2m1 codes of two values (|v| <= 6), round to nearest with ties to the even
// code (the hardware conversion), packed as one byte: lo in bits 0-3, hi in 4-7.
__device__ __forceinline__ uint32_t e2m1x2_of(float lo, float hi) {
  uint32_t r;
  asm("{ .reg .b8 b; cvt.rn.satfinite.e2m1x2.f32 b, %1, %2; cvt.u32.u8 %0, b; }" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// 2^e as a float for -126 <= e <= 127 (exact, no library call).
__device__ __forceinline__ float exp2i(int e) { return __int_as_float((e + 127) << 23); }

// One digit step of the unscaled term decomposition for two values held by one
// thread: the byte of their e2m1 codes at scale g (ig = 1/g, both powers of two,
// so r * ig is exact) and the exact residual update r -= code * g.
__device__ __forceinline__ uint32_t digit2(float& r0, float& r1, float g, float ig) {
  const uint32_t byte = e2m1x2_of(r0 * ig, r1 * ig);
  const uint32_t h2 = e2m1x2_to_f16x2(byte);
  r0 = fmaf(-f16lo_to_f32(h2), g, r0);
  r1 = fmaf(-f16hi_to_f32(h2), g, r1);
  return byte;
}

// Packs the bytes of 4 consecutive lanes into one word (lane 4j + i -> byte i);
// the word is valid in every lane of the group.
__device__ __forceinline__ uint32_t pack4(uint32_t byte, int lane) {
  uint32_t w = byte << (8 * (lane & 3));
  w |= __shfl_xor_sync(0xffffffffu, w, 1);
  w |= __shfl_xor_sync(0xffffffffu, w, 2);
  return w;
}

// Sum of 16 term accumulators, sum_t v[t] 2^(e - 2t), smallest term first
// (-90 <= e <= 100, so every scale is a normal float).
__device__ __forceinline__ float term_sum16(const float (&v)[16], int e) {
  float g = exp2i(e - 30), s = 0.f;
#pragma unroll
  for (int t = 15; t >= 0; --t) {
    s = fmaf(v[t], g, s);
    g *= 4.f;
  }
  return s;
}

// Packs the codes of 8 consecutive lanes into one word (lane 8j + i -> nibble i);
// the word is valid in every lane of the group.
__device__ __forceinline__ uint32_t pack8(uint32_t code, int lane) {
  uint32_t w = code << (4 * (lane & 7));
  w |= __shfl_xor_sync(0xffffffffu, w, 1);
  w |= __shfl_xor_sync(0xffffffffu, w, 2);
  w |= __shfl_xor_sync(0xffffffffu, w, 4);
  return w;
}

// e4m3 byte divided by 2^sh (sh >= 0), rounded to nearest even on the e4m3 grid.
__device__ __forceinline__ uint32_t e4m3_shift(uint32_t b, int sh) {
  b &= 0xFFu;
  if (sh <= 0 || b == 0u) return b;
  const int e = (int)((b >> 3) & 15u);
  if (e - sh >= 1) return (uint32_t)((e - sh) << 3) | (b & 7u);   // stays normal: exact
  const float v = ldexpf(e4m3_val(b), -sh);                       // < 2^-6: subnormal grid 2^-9
  return (uint32_t)__float2int_rn(v * 512.f);
}

}  // namespace tc
}  // namespace qx
