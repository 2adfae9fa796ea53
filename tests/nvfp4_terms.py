"""CPU model of the residual NVFP4 term decomposition the tensor-core decode path
feeds to `tcgen05.mma.kind::mxf4nvf4` (test infrastructure).

A vector v (one activation row, or one routed pair's SwiGLU output) becomes T
NVFP4 terms, v ~= sum_t G_t * s_{t,b} * q_{t,k}:

  * G_t = 2^(E - 2t), E = ceil(log2(amax(v) / (6 * 448))), a per-vector power of
    two (applied to the accumulator column in the epilogue);
  * s_{t,b} = the smallest e4m3 value >= amax_b(r_t) / (6 G_t), one per 16 elements
    (the MMA's block scale; rounding up keeps |r / (s G)| <= 6);
  * q_{t,k} = e2m1 round-to-nearest-even of r_t,k / (s_{t,b} G_t);
  * r_{t+1} = r_t - G_t s q (exact: every factor is a short power-of-two product).

Each term shrinks a block's residual by about 6x, and the 4x step between
consecutive G_t keeps every block scale at or below the one before it, so the
scales never overflow e4m3.
"""

from __future__ import annotations

import torch

from oracle import nvfp4 as q4

E4M3_MAX = 448.0


def _e4m3_positive_table() -> torch.Tensor:
    b = torch.arange(1, 0x7F, dtype=torch.int64)
    return q4.e4m3_decode(b.to(torch.uint8)).to(torch.float64)


_E4M3_POS = _e4m3_positive_table()          # ascending, 2^-9 .. 448


def e4m3_round_up(v: torch.Tensor) -> torch.Tensor:
    """Smallest positive e4m3 value >= v (v in [0, 448]); 0 stays 0. Returns bytes."""
    v64 = v.to(torch.float64).contiguous()
    i = torch.searchsorted(_E4M3_POS, v64, right=False).clamp(max=_E4M3_POS.numel() - 1)
    byte = (i + 1).to(torch.uint8)
    return torch.where(v64 > 0, byte, torch.zeros_like(byte))


def exponent_for(amax: torch.Tensor) -> torch.Tensor:
    """E with 2^E >= amax / 2688 (int32); amax == 0 gives a harmless E."""
    a = amax.to(torch.float64) / (6.0 * E4M3_MAX)
    e = torch.ceil(torch.log2(torch.where(a > 0, a, torch.ones_like(a))))
    return torch.where(a > 0, e, torch.full_like(e, -126.0)).to(torch.int32)


def decompose(v: torch.Tensor, terms: int, exp: torch.Tensor | None = None):
    """v float32 [n, K] (K % 16 == 0) -> (codes uint8 [n, T, K] nibbles,
    scales uint8 [n, T, K/16] e4m3 bytes, E int32 [n]); exp overrides E."""
    n, k = v.shape
    r = v.to(torch.float64).clone()
    e = exponent_for(v.abs().amax(dim=1)) if exp is None else exp.to(torch.int32)
    codes = torch.zeros(n, terms, k, dtype=torch.uint8)
    scales = torch.zeros(n, terms, k // 16, dtype=torch.uint8)
    for t in range(terms):
        g = torch.pow(2.0, (e - 2 * t).to(torch.float64)).view(n, 1)
        amax_b = r.view(n, k // 16, 16).abs().amax(dim=2)
        sb = e4m3_round_up(amax_b / (6.0 * g))
        s = q4.e4m3_decode(sb).to(torch.float64)
        sg = (s * g).repeat_interleave(16, dim=1)
        ratio = torch.where(sg > 0, r / torch.where(sg > 0, sg, torch.ones_like(sg)), torch.zeros_like(r))
        c = q4.e2m1_encode(ratio.to(torch.float32))
        codes[:, t] = c
        scales[:, t] = sb
        r = r - q4.e2m1_decode(c).to(torch.float64) * sg
    return codes, scales, e


def reconstruct(codes: torch.Tensor, scales: torch.Tensor, e: torch.Tensor) -> torch.Tensor:
    """Sum of the terms in float64 [n, K]."""
    n, t_, k = codes.shape
    out = torch.zeros(n, k, dtype=torch.float64)
    for t in range(t_):
        g = torch.pow(2.0, (e - 2 * t).to(torch.float64)).view(n, 1)
        s = q4.e4m3_decode(scales[:, t]).to(torch.float64).repeat_interleave(16, dim=1)
        out += q4.e2m1_decode(codes[:, t]).to(torch.float64) * s * g
    return out
