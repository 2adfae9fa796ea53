// Test-only C ABI around the reference's unmodified seam kernels (the FP8 post
// quantiser and the ordered combine of native/qmesh_afd_seam.cu).
//
// The kernel source is NOT copied here: oracle/ref_seam/build.py #includes it
// at build time from the reference tree (REF_SEAM_FILE) into
// oracle/_ref/libref_seam.so. In the reference that file is compiled as the
// tail of native/qmesh_afd_peer.cpp, whose wire constants it uses; the two it
// needs are restated below with the peer file's values (K_HIDDEN 5120,
// ROUT_HDR 16, qmesh_afd_peer.cpp:57, :99). The launch shapes follow the
// reference's own launchers (seam_blocks: 256 threads, at most 1024 blocks,
// native/qmesh_afd_seam_host.inc:152-159) and its quant_test harness
// (native/qmesh_afd_seam_py.inc:8-45): amax with the finish folded in, then the
// byte pack; the combine is seam_combine(_vec)_kernel as seam_launch_collect
// picks it (native/qmesh_afd_seam_api.inc:48-72), without the collect wait.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

static constexpr int K_HIDDEN = 5120;
static constexpr size_t ROUT_HDR = 16;

#include REF_SEAM_FILE

static int ref_blocks(size_t work) {
  size_t b = (work + 255) / 256;
  if (b < 1) b = 1;
  return (int)(b > 1024 ? 1024 : b);
}

extern "C" {

size_t ref_seam_status_bytes(void) { return sizeof(SeamStatus); }

// The seam's post quantiser over n bf16 rows of stride xs elements: q [n, 5120]
// e4m3, scale[0] = s, scale[1] = inv. work: 2 device words (amax, fin);
// status: ref_seam_status_bytes() of device memory, zeroed by the caller.
int ref_seam_quant_post(const void* x, size_t xs, int n, uint8_t* q, float* scale, uint32_t* work,
                        void* status, void* stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  SeamDev d{};
  d.np = 1;
  d.amax = work;
  d.fin = work + 1;
  d.scale = scale;
  d.in[0] = q;
  d.st = reinterpret_cast<SeamStatus*>(status);
  if (cudaMemsetAsync(work, 0, 2 * sizeof(uint32_t), st) != cudaSuccess) return 1;
  seam_amax_kernel<<<ref_blocks((size_t)n * K_HIDDEN), 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), xs, n, d, __bfloat162float(__float2bfloat16_rn(1e-6f)));
  seam_pack_kernel<<<ref_blocks((size_t)n * K_HIDDEN), 256, 0, st>>>(
      d, reinterpret_cast<const __nv_bfloat16*>(x), xs, nullptr, 0, nullptr, n);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

// The seam's combine: out[:n] = bf16(fp32(out) + fp32(p0) + ... ) in peer
// order (np <= 4 contiguous [n, 5120] bf16 partials), in place on out (row
// stride os elements); vec selects seam_combine_vec_kernel. status as above.
int ref_seam_combine(void* out, size_t os, const void* const* parts, int np, int n, int vec, void* status,
                     void* stream) {
  if (np < 0 || np > SEAM_MAXP) return 1;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  SeamDev d{};
  d.np = np;
  for (int p = 0; p < np; ++p) d.out[p] = reinterpret_cast<const __nv_bfloat16*>(parts[p]);
  d.st = reinterpret_cast<SeamStatus*>(status);
  const size_t total = (size_t)n * K_HIDDEN;
  if (vec)
    seam_combine_vec_kernel<false><<<ref_blocks(total / 8), 256, 0, st>>>(d, out, os, n);
  else
    seam_combine_kernel<false><<<ref_blocks(total), 256, 0, st>>>(d, out, os, n);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

}  // extern "C"
