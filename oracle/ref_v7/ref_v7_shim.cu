// Test-only C ABI around the reference's unmodified v7 decode kernel.
//
// The kernel source is NOT copied here: it is #included at build time from the
// reference tree (REF_KERNEL_FILE = gx/kernels/fp4_decode_moe_swz.cu) by
// oracle/ref_v7/build.py, which writes the library to oracle/_ref/. The three
// instantiations are the slice widths the reference kernel's static asserts
// admit (C <= 1024, CP a multiple of 128): 864/896 (a GX rank), 576/640 (the
// NODE-A width) and 288/384 (an 8-way split of 2304).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include REF_KERNEL_FILE

#define REF_ENTRY(C, CP)                                                                                    \
  extern "C" int ref_v7_decode_##C(const void* x, const int* ids, const float* tw, const uint8_t* w13,    \
                                   const uint8_t* s13, const float* g13, const uint8_t* w2,               \
                                   const uint8_t* s2, const float* g2, float* act, void* out, int rows,    \
                                   float limit, int has_limit, void* stream) {                             \
    decode_moe<5120, CP, C>(reinterpret_cast<const __nv_bfloat16*>(x), ids, tw, w13, s13, g13, w2, s2, g2, \
                            act, reinterpret_cast<__nv_bfloat16*>(out), rows, limit, has_limit,           \
                            reinterpret_cast<cudaStream_t>(stream));                                      \
    return cudaGetLastError() == cudaSuccess ? 0 : 1;                                                      \
  }

REF_ENTRY(864, 896)
REF_ENTRY(576, 640)
REF_ENTRY(288, 384)
