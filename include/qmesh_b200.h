/* qmesh_b200 -- C ABI of the B200 routed-expert NVFP4 slice.
 *
 * One shared library, libqmesh_b200.so, built for sm_100a. Every entry point
 * takes plain pointers and sizes, launches on the caller's stream, allocates
 * nothing, never synchronises the host and never exits the process: it returns
 * a status code (QX_OK on success). Device-side problems found while running
 * (bad expert ids, a wait that ran out of time) are recorded in the status
 * words of the caller's workspace; qx_status_read decodes them.
 *
 * Reference interfaces these replace (paths inside QMesh AFD-TP3):
 *   qx_slice_decode    gx/kernels/ext_variant.cu:11-24  run(out, x, ids, tw,
 *                      w13, s13, g13, w2, s2, g2, act, swiglu_limit, has_limit)
 *                      -> decode_moe<5120,896,864> (fp4_decode_moe_swz.cu:390-402),
 *                      reached through gx/gx_decode_swz.py:163-178 body().
 *   qx_combine_ordered native/qmesh_afd_seam.cu:310-484 seam_combine(_vec)_kernel,
 *                      launched by Seam.collect (native/qmesh_afd_seam_py.inc:69-106).
 */
#ifndef QMESH_B200_H
#define QMESH_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
enum {
  QX_OK = 0,
  QX_ERR_ARG = 1,        /* null pointer or inconsistent argument */
  QX_ERR_SHAPE = 2,      /* size outside what the kernel supports */
  QX_ERR_ALIGN = 3,      /* pointer or stride not aligned as required */
  QX_ERR_WORKSPACE = 4,  /* workspace smaller than qx_slice_workspace_bytes */
  QX_ERR_LAUNCH = 5,     /* the CUDA launch itself failed */
  QX_ERR_DEVICE = 6      /* no usable sm_100 device */
};

/* Device status bits written into the workspace by the kernels. */
enum {
  QX_DEV_BAD_ID = 1,       /* an id outside {-1} U [0, E): that slot was skipped */
  QX_DEV_TIMEOUT = 2,      /* a bounded device wait ran out; the output is invalid */
  QX_DEV_OVERFLOW = 4,     /* more routed pairs than the workspace was sized for */
  QX_DEV_NONFINITE = 8     /* qx_quant_fp8: a non-finite maximum; those bytes were not written */
};

/* Activation formats. */
enum {
  QX_X_E4M3 = 0,   /* e4m3 [rows, hidden] + one FP32 dequant scale per row (inv) */
  QX_X_E4M3_POST = 1, /* e4m3 [rows, hidden] + one FP32 dequant scale for all rows */
  QX_X_BF16 = 2    /* bf16 [rows, hidden] (the reference body's input) */
};

/* Arena layouts: which kernel family the tiles were stored for. The two
 * layouts have the same byte counts, so the tag is the only thing that tells
 * them apart; every slice entry point refuses an arena whose tag is not its own
 * with QX_ERR_ARG (an untagged arena, layout 0, included). */
enum {
  QX_LAYOUT_TC = 0x54430001,   /* tensor-core tiles: qx_slice_decode_tc(_xchg), qx_slice_prefill_tc */
  QX_LAYOUT_FRAG = 0x46520002  /* register-fed fragment tiles: qx_slice_decode, qx_slice_decode_static */
};

/* Geometry of the build's NVFP4 arena (one MoE layer on one GPU).
 *
 * The arena holds intermediate columns [a0, a1) of every expert. Codes and
 * scales are stored in tiles so that any 32-column-aligned column range of
 * one expert streams as contiguous bulk copies (see qx_arena_bytes). */
typedef struct {
  const uint8_t* w13;      /* gate/up tiles, qx_arena_w13_bytes(E, a1-a0) bytes */
  const uint8_t* w2;       /* down tiles,    qx_arena_w2_bytes(E, a1-a0) bytes */
  const float*   g13;      /* [E] w13 weight_scale_2 (w1 and w3 share it) */
  const float*   g2;       /* [E] w2 weight_scale_2 */
  int32_t        n_experts;
  int32_t        a0, a1;   /* arena column range, multiples of 32 */
  int32_t        layout;   /* QX_LAYOUT_TC or QX_LAYOUT_FRAG */
} QxArena;

/* One call of the routed-expert slice over columns [c0, c1). */
typedef struct {
  const void*  x;          /* activations, format x_fmt, row stride x_stride bytes */
  const float* x_scale;    /* QX_X_E4M3: [rows]; QX_X_E4M3_POST: [1]; else unused */
  int64_t      x_stride;   /* bytes between rows of x (>= hidden * element size) */
  int32_t      x_fmt;
  const void*  ids;        /* int32 or int64 [rows, topk]; -1 = padding slot */
  int32_t      ids_int64;
  const float* tw;         /* FP32 [rows, topk] routing weights */
  int32_t      rows;       /* 1 .. QX_MAX_ROWS */
  int32_t      topk;       /* 1 .. QX_MAX_TOPK */
  int32_t      c0, c1;     /* column range, 32-aligned, inside [a0, a1) */
  float        swiglu_limit;
  int32_t      has_limit;
  uint16_t*    out;        /* BF16 [rows, hidden] partial, row stride out_stride elements */
  int64_t      out_stride;
  void*        workspace;  /* qx_slice_workspace_bytes(rows, topk, c0, c1) bytes, 256-aligned */
  size_t       workspace_bytes;
} QxSliceArgs;

#define QX_HIDDEN 5120
#define QX_MAX_ROWS 64
#define QX_MAX_TOPK 8

/* Arena sizes in bytes for E experts and `width` = a1 - a0 columns. */
size_t qx_arena_w13_bytes(int32_t n_experts, int32_t width);
size_t qx_arena_w2_bytes(int32_t n_experts, int32_t width);

/* Workspace bytes one qx_slice_decode call needs. */
size_t qx_slice_workspace_bytes(int32_t rows, int32_t topk, int32_t c0, int32_t c1);

/* Routed-expert NVFP4 SwiGLU slice (decode, rows <= QX_MAX_ROWS) over an
 * arena in the fragment layout (QX_LAYOUT_FRAG).
 * Replaces gx/kernels/ext_variant.cu:11-24 run(). Three launches on `stream`
 * (a routing/activation prologue, the persistent weight-streaming kernel and
 * the slot-order finalize); capture-safe. */
int qx_slice_decode(const QxArena* arena, const QxSliceArgs* args, void* stream);

/* Limits of qx_slice_decode_static. */
#define QX_STATIC_MAX_ROWS 8
#define QX_STATIC_MAX_TOPK 8
#define QX_STATIC_MAX_WIDTH 2304

/* The slice of qx_slice_decode for callers that cannot allocate device memory.
 * No counterpart in the reference: its worker always owns its scratch.
 *
 * Some callers can't call cudaMalloc: a serving process whose device memory is
 * fully claimed by its own arena and pools at start-up (the reference's GX worker
 * sizes its expert arena to the free memory and refuses to start otherwise), or
 * a host runtime embedding this library through an FFI without a device
 * allocator of its own. This entry point needs no workspace from the caller: its
 * scratch is one static array in the library (about 3.2 MiB per GPU that loads
 * the library, held until the process exits), large enough for
 * QX_STATIC_MAX_ROWS rows, QX_STATIC_MAX_TOPK slots and QX_STATIC_MAX_WIDTH
 * columns; larger calls return QX_ERR_SHAPE. args->workspace and
 * args->workspace_bytes are ignored; inputs and outputs are the caller's, as in
 * qx_slice_decode, and the arena must be in the fragment layout
 * (QX_LAYOUT_FRAG). It allocates nothing and calls no allocating routine.
 *
 * The first call on a device looks up the array's device address (with that
 * device current); make that first call before any stream capture. Every call
 * on a device shares the one array, and the kernels reinitialise what must
 * start at zero on each call: calls that overlap on the GPU (two streams, or
 * two host threads) race on the array and must be serialised by the caller.
 * Device-side conditions of the last call (QX_DEV_BAD_ID, QX_DEV_TIMEOUT, ...)
 * sit in the array's status word: read them with qx_slice_decode_static_status. */
int qx_slice_decode_static(const QxArena* arena, const QxSliceArgs* args, void* stream);

/* The QX_DEV_* bits that the last qx_slice_decode_static call on the current
 * device recorded (a host copy, synchronous on `stream`; queue it after that
 * call). QX_ERR_DEVICE if no call has run on this device yet. */
int qx_slice_decode_static_status(uint32_t* status, void* stream);

/* Fixed-order combine: out = bf16(fp32(parts[0]) + ... + fp32(parts[n-1])), in
 * that order, one rounding (out_f32: keep FP32). parts[i] are BF16 [rows, hidden]
 * rows of stride part_stride elements; they may live on peer GPUs (P2P-mapped
 * pointers). Replaces native/qmesh_afd_seam.cu:310-484. */
int qx_combine_ordered(const uint16_t* const* parts, int32_t n_parts, int64_t part_stride,
                       void* out, int64_t out_stride, int32_t out_f32, int32_t rows,
                       void* stream);

/* ---- prefill slice (W4A4 grouped tcgen05 block-scaled GEMM) -------------------
 * The reference's prefill body (gx/gx_ingest.py:190-246, cutlass_body_clamped:
 * scaled_fp4_experts_quant + cutlass_fp4_moe_mm + silu_and_mul_with_clamp):
 * x (FP8 rows + scale, or BF16) is quantised to NVFP4 with a1g = bf16(6 / max|x|),
 * both GEMMs run as `tcgen05.mma.kind::mxf4nvf4` over the tensor-core arena,
 * the clamp SwiGLU output is quantised to NVFP4 with the caller's calibrated
 * a2 (device FP32 [n_experts], gx/gx_expert_worker.py:250-283), and
 * out = bf16(sum_j bf16(c3_j * bf16(tw_j))). Arena in the tensor-core layout;
 * rows up to QX_PREFILL_MAX_ROWS, n_experts up to 1024; workspace from
 * qx_prefill_workspace_bytes (256-byte aligned). Same column-range rules and
 * status codes as qx_slice_decode_tc. */
#define QX_PREFILL_MAX_ROWS 8192
size_t qx_prefill_workspace_bytes(int32_t rows, int32_t topk, int32_t c0, int32_t c1, int32_t n_experts);
int qx_slice_prefill_tc(const QxArena* arena, const QxSliceArgs* args, const float* a2, void* stream);

/* ---- producer side: FP8 activation quantisation and the routing front end ----
 * qx_quant_fp8 replaces the seam's post quantiser (native/qmesh_afd_seam.cu:9-16,
 * seam_amax_kernel / seam_finish / seam_pack_kernel :88-176): BF16 x [rows, 5120]
 * -> e4m3 q with m = max|x|, mc = max(m, bf16(1e-6)), s = (float)(448 / (double)mc),
 * inv = (float)(1 / (448 / (double)mc)), q = e4m3_rne_satfinite(clamp(bf16_rn(x s),
 * +-448)); per row (inv [rows], per_post = 0) or per post (inv [1], the
 * reference's form; `work` is one device word of scratch). A non-finite maximum
 * leaves those bytes unwritten, sets inv = 1 and QX_DEV_NONFINITE in *status.
 * qx_route_topk: softmax of FP32 logits [rows, n_experts], the top-k experts
 * (larger probability first, lower id first among equals), weights renormalised
 * to sum 1 (the router output the reference posts with each layer,
 * afd_session.py:211-252). */
int qx_quant_fp8(const void* x, int64_t x_stride, int32_t rows, int32_t per_post, void* q, int64_t q_stride,
                 float* inv, uint32_t* work, uint32_t* status, void* stream);
int qx_route_topk(const float* logits, int64_t logits_stride, int32_t rows, int32_t n_experts, int32_t topk,
                  int32_t* ids, float* tw, void* stream);

/* Bounded device wait for a round driver (the counterpart of gx/gx_spin.py's
 * spin kernel): one thread waits until the 32-bit sequence cell (host-mapped or
 * device memory) reaches *need (a device word read when the wait runs, so one
 * captured round graph serves every round; wrap-around order), or until
 * timeout_ns passes, then sets QX_DEV_TIMEOUT in *status; work queued after it
 * on the stream runs either way. */
int qx_wait_cell(const uint32_t* cell, const uint32_t* need, uint64_t timeout_ns, uint32_t* status, void* stream);

/* ---- one-shot combine over peer memory (NVLink) ------------------------------
 * Replaces the reference's RDMA seam (native/qmesh_afd_seam.cu:309-361,
 * qmesh_afd_edge/peer transport) inside one box: every rank's BF16 partial is
 * stored straight into the output rank's receive slot over NVLink, and the
 * output rank sums the partials in FP32 in rank order (then `shared`, if given)
 * with one BF16 rounding. Setup: each rank allocates its exchange buffer
 * (qx_xchg_alloc, zero-filled), exports it (qx_ipc_handle), the ranks swap the
 * 64-byte handles (e.g. torch.distributed.all_gather_object) and open the
 * others' buffers (qx_ipc_open). Every rank then calls qx_combine_p2p once per
 * step with the same rank order, on its own stream; calls are graph-capturable.
 * Waits on peers are bounded (QX_TIMEOUT_MS); a timeout sets QX_DEV_TIMEOUT in
 * *status and leaves the exchange unusable (recreate it). */
#define QX_XCHG_MAX_RANKS 8
#define QX_IPC_HANDLE_BYTES 64

typedef struct QxXchgArgs {
  void*        bufs[QX_XCHG_MAX_RANKS]; /* every rank's exchange buffer in this process (own included) */
  const void*  part;        /* this rank's BF16 partial [rows, 5120] */
  int64_t      part_stride; /* elements */
  const void*  shared;      /* output rank only, optional: BF16 [rows, 5120] added after the ranks */
  int64_t      shared_stride;
  void*        out;         /* output rank only: BF16 [rows, 5120] */
  int64_t      out_stride;
  uint32_t*    status;      /* device word: QX_DEV_TIMEOUT on a wait that ran out */
  int32_t      rank, world, dst, rows, rows_max;
} QxXchgArgs;

size_t qx_xchg_bytes(int32_t rows_max);
int qx_xchg_alloc(int32_t rows_max, void** buf);
int qx_xchg_free(void* buf);
int qx_ipc_handle(const void* buf, void* handle);   /* handle: QX_IPC_HANDLE_BYTES bytes */
int qx_ipc_open(const void* handle, void** buf);
int qx_ipc_close(void* buf);
int qx_combine_p2p(const QxXchgArgs* args, void* stream);

/* Read the device status words of a workspace (host copy, synchronous on
 * `stream`): bit set of QX_DEV_*. */
int qx_status_read(const void* workspace, uint32_t* status, void* stream);

/* ---- tensor-core slice (tcgen05 block-scaled NVFP4 MMA) ----------------------
 * Same call contract as qx_slice_decode over an arena in the tensor-core tile
 * layout: w13 [E][ceil(W/64)][80][4608 B], w2 [E][40][ceil(W/64)][4608 B] for
 * arena width W = a1 - a0 (each 4608-byte K block = a 128-row x 64-element
 * operand tile, then its 512-byte scale atom; columns past a1 are zero). The
 * activations enter the MMA as 16 residual e2m1 terms (to 2^-30 of their
 * maximum), so results stay within the same tolerance of the reference's FP32
 * arithmetic. Requires
 * (c0 - a0) % 64 == 0 and c1 % 32 == 0. Replaces the same reference body as
 * qx_slice_decode (gx/kernels/ext_variant.cu:11-24). */
size_t qx_arena_tc_w13_bytes(int32_t n_experts, int32_t width);
size_t qx_arena_tc_w2_bytes(int32_t n_experts, int32_t width);
size_t qx_slice_workspace_tc_bytes(int32_t rows, int32_t topk, int32_t c0, int32_t c1);
int qx_slice_decode_tc(const QxArena* arena, const QxSliceArgs* args, void* stream);

/* The tensor-core slice with the rank combine fused into its finalize, one
 * kernel per rank and call: each rank's BF16 partial goes straight from the
 * finalize into the output rank's receive words (64-bit words that carry the
 * call number beside 4 data bytes, in the buffers of qx_xchg_alloc mapped with
 * qx_ipc_open; x->bufs, rank, world, dst, rows_max as for qx_combine_p2p), and
 * the output rank writes bf16(sum over ranks in order of the partials
 * [+ x->shared]) to args->out, as qx_combine_p2p would. Sender
 * ranks do not write args->out; x->part, x->out and x->status are not used (a
 * wait that runs out sets QX_DEV_TIMEOUT in the workspace status). A buffer
 * serves either this call or qx_combine_p2p, not both interleaved. Replaces the
 * slice + seam pair (gx/kernels/ext_variant.cu:11-24, then
 * native/qmesh_afd_seam.cu:309-361). */
int qx_slice_decode_tc_xchg(const QxArena* arena, const QxSliceArgs* args, const QxXchgArgs* x, void* stream);

/* The tensor-core slice plus a shared expert: the dense NVFP4 SwiGLU that the
 * reference runs beside the routed experts on the node that writes the layer
 * output, added after the routed partials in the reference's fixed order
 * (README.md:88-90: NODE-A, NODE-B, NODE-C, shared; native/qmesh_afd_seam.cu:309-361).
 * `shared` is a one-expert arena in the tensor-core layout over its whole
 * intermediate range [a0, a1) (at most 4096 columns); every row of the call
 * goes through it with weight 1, as extra work items of the same kernel. The
 * output is bf16(fp32(routed partial) + fp32(shared)) for x == NULL, and
 * bf16(p_0 + ... + p_{N-1} + shared) on the output rank of a fused rank combine
 * (x as for qx_slice_decode_tc_xchg; only the output rank passes `shared`, and
 * x->shared must be NULL). The shared expert's BF16 output and the routed
 * partial are each bit-identical to separate qx_slice_decode_tc calls (the
 * shared one with ids 0, weights 1, topk 1). Same workspace as
 * qx_slice_decode_tc (qx_slice_workspace_tc_bytes has room for it). */
int qx_slice_decode_tc_shared(const QxArena* arena, const QxSliceArgs* args, const QxArena* shared,
                              const QxXchgArgs* x, void* stream);

/* Self-check of the block-scaled NVFP4 tensor-core path (no counterpart in the
 * reference): d[128][n] (FP32, row-major) = sum over nkb 64-wide K blocks of
 * (A * SFA) x (B * SFB)^T, computed by tcgen05.mma.kind::mxf4nvf4 with the
 * operand layouts the decode kernels stream. `a` holds nkb K blocks of 4608
 * bytes (a 128-row tile of 4096 bytes, then its 512-byte scale atom); `b` holds
 * nkb K blocks of n*32 + 512*ceil(n/128) bytes (tile, then one atom per 128 rows). n in {16, 32, ..., 256}, nkb in 1..8, a and b
 * 16-byte aligned, status a device word (QX_DEV_TIMEOUT on a wait that ran out). */
int qx_diag_nvf4_tile(const uint8_t* a, const uint8_t* b, int32_t n, int32_t nkb, float* d,
                      uint32_t* status, void* stream);

/* Library version string. */
const char* qx_version(void);

#ifdef __cplusplus
}
#endif
#endif /* QMESH_B200_H */
