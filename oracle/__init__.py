"""CPU oracle for the routed-expert NVFP4 slice -- TEST INFRASTRUCTURE ONLY.

Nothing in the product imports this package. Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` use it, and only as the checker (or the timed CPU
baseline), never as the thing measured or shipped.

What it restates (paths relative to the QMesh AFD-TP3 reference tree):

* NVFP4 unpack and scale decode: gx/kernels/fp4_decode_moe_swz.cu:58, :82-96
  (low nibble = even k; value = e2m1 * e4m3(block scale) * weight_scale_2).
* Decode-row MoE body (W4A16, FP32 intermediate):
  gx/kernels/fp4_decode_moe_swz.cu:287-299 (stage 1: g13 after the dot,
  clamp gate <= L and -L <= up <= L, silu(gate) * up) and :356-385
  (stage 2: g2[e] * tw folded per expert, FP32 sum over top-6, one BF16
  round).
* Gate-first split: gx/gx_expert_worker.py:96-108.
* FP8 activation transport: native/qmesh_afd_seam.cu:9-16 (producer) and
  gx/gx_ingest.py:151-154 (consumer: x = bf16(float(e4m3) * inv)).
* Fixed-order combine: native/qmesh_afd_seam.cu:310-361 (FP32 sum in peer
  order, one BF16 round).
* Scale swizzle byte map: gx/kernels/fp4_decode_moe_swz.cu:19-24.

Parity pins (see tests/test_oracle_pins.py and tests/golden/):

* the swizzle byte map against vLLM's own ``swizzle_blockscale`` run on CPU;
* host routing policy and row buckets against gx/gx_ingest.py run on CPU;
* the reference SwiGLU form against gx/gx_expert_worker.py:swiglu run on CPU;
* e4m3 decode of all 256 bytes against torch's float8_e4m3fn;
* the decode arithmetic against the reference's own v7 CUDA kernel, built
  from its unmodified source by ``oracle/ref_v7`` into ``oracle/_ref`` and run
  on the GPU by ``tests/test_ref_v7_pin.py``.
"""
