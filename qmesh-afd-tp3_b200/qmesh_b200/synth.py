"""Seeded synthetic inputs for the slice (benchmark and examples), any device.

Routing: FP32 logits -> softmax -> top-k distinct ids -> weights renormalised to
sum 1. Activations: RMSNorm-like N(0,1) rows in BF16, quantised to FP8 e4m3 with
one FP32 scale per row using the reference seam's arithmetic
(native/qmesh_afd_seam.cu:9-16): s = float(448 / max(amax, bf16(1e-6))),
q = e4m3_rne(clamp(bf16_rn(x * s), +-448)), inv = float(1 / (448 / mc)).
"""

from __future__ import annotations

import torch

_BF16_FLOOR = float(torch.tensor(1e-6, dtype=torch.bfloat16).float())


def routing(logits: torch.Tensor, topk: int = 6) -> tuple[torch.Tensor, torch.Tensor]:
    p = torch.softmax(logits.float(), dim=-1)
    w, ids = torch.topk(p, topk, dim=-1)
    return ids.to(torch.int32), (w / w.sum(dim=-1, keepdim=True)).float()


def zipf_bias(n_experts: int, s: float, gen: torch.Generator) -> torch.Tensor:
    """Per-expert logit bias -s*ln(rank), ranks a seeded permutation of 1..E."""
    rank = torch.randperm(n_experts, generator=gen).float() + 1.0
    return -s * torch.log(rank)


def fp8_quant_rows(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """BF16-valued rows -> (e4m3 bytes uint8 [R, K], dequant scale inv f32 [R])."""
    x = x.float()
    mc = torch.clamp(x.abs().amax(dim=-1).double(), min=_BF16_FLOOR)
    sd = 448.0 / mc
    y = (x * sd.float().unsqueeze(-1)).to(torch.bfloat16).float()
    q = torch.clamp(y, -448.0, 448.0).to(torch.float8_e4m3fn).view(torch.uint8)
    return q, (1.0 / sd).float()


def make_activation(rows: int, gen: torch.Generator, hidden: int = 5120):
    x = torch.randn(rows, hidden, generator=gen).to(torch.bfloat16).float()
    return fp8_quant_rows(x)
