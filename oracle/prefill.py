"""W4A4 prefill slice on the CPU -- test infrastructure.

Restates the reference's prefill body (gx/gx_ingest.py:190-246, the clamped
split CUTLASS form `cutlass_body_clamped`), whose arithmetic differs from the
W4A16 decode body: the activations themselves are quantised to NVFP4.

  a1g = bf16(6 / max(max|x|, bf16(1e-6)))          (gx_ingest.py:223; x is bf16)
  xq  = nvfp4(x, a1g)                               (scaled_fp4_experts_quant)
  c1  = bf16((g13 / a1g) * sum_k xq * w13q)         (cutlass_fp4_moe_mm, bf16 out)
  c2  = bf16(silu(min(g, L)) * clamp(u, -L, L))     (silu_and_mul_with_clamp)
  c2q = nvfp4(c2, a2)                               (a2: calibrated per layer,
                                                     gx_expert_worker.py:250-283)
  c3  = bf16((g2 / a2) * sum_c c2q * w2q)
  out = bf16(sum_j bf16(c3_j * bf16(tw_j)))         (gx_ingest.py:244-245, FP32 sum)

nvfp4(v, gs) is vLLM's reference NVFP4 activation quantiser
(`ref_nvfp4_quant`, vllm/model_executor/layers/quantization/utils/
nvfp4_emulation_utils.py, vLLM 0.22.0 in this image; the reference ran
0.24.0): per 16 elements scale = e4m3(min(gs * (amax * f32(1/6)), 448)),
code = e2m1_rne(clamp(v * 1/(scale * 1/gs), -6, 6)), every step in FP32 with
correctly rounded reciprocals. Pinned by tests/golden/prefill_quant.npz.

The GEMM products code*scale are exact; the oracle sums them in float64 and
rounds the scaled result once to FP32 then BF16, so it differs from any FP32
tensor-core accumulation only in the last FP32 bits of c1 / c3.
"""

from __future__ import annotations

import torch

from . import nvfp4 as q4

SIXTH = torch.tensor(1.0 / 6.0, dtype=torch.float32)


def _recip(x: torch.Tensor) -> torch.Tensor:
    return torch.where(x != 0, torch.reciprocal(torch.where(x != 0, x, torch.ones_like(x))), torch.zeros_like(x))


def act_quant(v: torch.Tensor, gs) -> tuple[torch.Tensor, torch.Tensor]:
    """float32 [m, n] (n % 16 == 0) -> (nibbles uint8 [m, n], e4m3 scale bytes uint8 [m, n/16])."""
    v = v.to(torch.float32)
    m, n = v.shape
    gs = torch.as_tensor(gs, dtype=torch.float32)
    blk = v.reshape(m, n // 16, 16)
    vmax = blk.abs().amax(dim=-1, keepdim=True)
    scale = gs * (vmax * SIXTH)
    scale = torch.clamp(scale, min=-448.0, max=448.0)
    sbyte = scale.to(torch.float8_e4m3fn).view(torch.uint8)
    sval = q4.e4m3_decode(sbyte)
    out_scale = _recip(sval * _recip(gs))
    scaled = torch.clamp(blk * out_scale, -6.0, 6.0)
    return q4.e2m1_encode(scaled).reshape(m, n), sbyte.reshape(m, n // 16)


def act_dequant_unscaled(nib: torch.Tensor, sbyte: torch.Tensor) -> torch.Tensor:
    """code * block scale (exact in float32), without the global scale."""
    return q4.e2m1_decode(nib) * q4.e4m3_decode(sbyte).repeat_interleave(16, dim=-1)


def a1_scale(x: torch.Tensor) -> torch.Tensor:
    """bf16(6 / max(max|x|, bf16(1e-6))) for bf16-valued x (gx_ingest.py:223)."""
    amax = x.abs().amax().to(torch.float32)
    amax = torch.clamp(amax, min=q4.BF16_FLOOR)
    return q4.bf16_round(torch.tensor(6.0, dtype=torch.float32) / amax)


def silu_clamp(c1g: torch.Tensor, c1u: torch.Tensor, limit: float, has_limit: bool = True) -> torch.Tensor:
    """bf16(silu(min(g, L)) * clamp(u, -L, L)) in FP32 from bf16 inputs."""
    g = c1g.to(torch.float32)
    u = c1u.to(torch.float32)
    if has_limit:
        g = torch.clamp(g, max=limit)
        u = torch.clamp(u, min=-limit, max=limit)
    return q4.bf16_round(g / (1.0 + torch.exp(-g)) * u)


def slice_w4a4(x: torch.Tensor, ids: torch.Tensor, tw: torch.Tensor, layer: dict, c0: int, c1: int,
               a2, limit: float = 10.0, has_limit: bool = True, stats: dict | None = None) -> torch.Tensor:
    """BF16 partial [T, H] of the W4A4 prefill body over intermediate columns [c0, c1).

    x: bf16-valued float32 [T, H]; ids int [T, k] (-1 = no expert); tw float32
    [T, k]; a2: FP32 per-expert [E] or a scalar; layer: pack tensors over the
    full intermediate (c13 [E, 2I, H/2] ...).
    """
    t, k = ids.shape
    hid = x.shape[1]
    inter = layer["c13"].shape[1] // 2
    a1g = a1_scale(x)
    xn, xs = act_quant(x, a1g)
    xq = act_dequant_unscaled(xn, xs).to(torch.float64)
    a2 = torch.as_tensor(a2, dtype=torch.float32)
    y = torch.zeros(t, k, hid, dtype=torch.float32)
    c2max = 0.0
    for e in torch.unique(ids[ids >= 0]).tolist():
        sel = (ids == e).nonzero().tolist()
        rows = [p[0] for p in sel]
        a2e = a2[e] if a2.dim() else a2
        w13 = q4.dequant(layer["c13"][e], layer["s13"][e], 1.0).to(torch.float64)
        wg, wu = w13[c0:c1], w13[inter + c0:inter + c1]
        alpha1 = (layer["g13"][e].to(torch.float32) / a1g).to(torch.float32)
        xr = xq[rows]
        cg = q4.bf16_round((alpha1.double() * (xr @ wg.T)).to(torch.float32))
        cu = q4.bf16_round((alpha1.double() * (xr @ wu.T)).to(torch.float32))
        c2 = silu_clamp(cg, cu, limit, has_limit)
        c2max = max(c2max, float(c2.abs().max()))
        an, as_ = act_quant(c2, a2e)
        aq = act_dequant_unscaled(an, as_).to(torch.float64)
        w2 = q4.dequant(layer["c2"][e][:, c0 // 2:c1 // 2], layer["s2"][e][:, c0 // 16:c1 // 16], 1.0)
        alpha2 = (layer["g2"][e].to(torch.float32) / a2e).to(torch.float32)
        c3 = q4.bf16_round((alpha2.double() * (aq @ w2.to(torch.float64).T)).to(torch.float32))
        for i, (row, j) in enumerate(sel):
            twb = q4.bf16_round(tw[row, j].to(torch.float32))
            y[row, j] = q4.bf16_round(c3[i] * twb)
    out = y[:, 0].clone()
    for j in range(1, k):
        out = out + y[:, j]
    if stats is not None:
        stats["c2_amax"] = c2max      # what the reference's a2 calibration estimates (gx_expert_worker.py:250-283)
    return q4.bf16_round(out)
