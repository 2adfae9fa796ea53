"""CPU model of the residual NVFP4 term decomposition the tensor-core decode path
feeds to `tcgen05.mma.kind::mxf4nvf4` (test infrastructure; the kernel's own
arithmetic, so tests can compare its buffers bit for bit).

A vector v (one activation row, or one routed pair's SwiGLU output over a
64-column tile) becomes T = 8 NVFP4 terms, v ~= sum_t G_t * s_{t,b} * q_{t,k}:

  * E = the smallest integer with 2688 * 2^E >= amax(v) (0 when v == 0), clamped to
    [-100, 100]; G_t = 2^(E - 2t), applied to the accumulator column in the epilogue;
  * s_{t,b} = the smallest e4m3 value s with s * 6 * G_t >= amax_b(r_t) (exact
    comparison), one per 16 elements (the MMA's block scale); 0 when the block's
    residual is 0;
  * q_{t,k} = e2m1 round-to-nearest-even (ties to the even code) of the exact
    quotient r_t,k / (s_{t,b} G_t), which lies in [-6, 6];
  * r_{t+1} = r_t - G_t s q, exact in fp32 (q s has at most 6 significant bits and
    lies within a factor 2 of r when q != 0).

Each term shrinks a block's residual about 6x; the 4x step between consecutive
G_t keeps each block scale at or below the previous one, so none overflows e4m3.
A tile decomposed with its own exponent E_loc is brought to a common exponent
E >= E_loc by dividing every scale byte by 2^(E - E_loc) (exact while the result
stays a normal e4m3 number, else rounded to nearest even on the subnormal grid).
"""

from __future__ import annotations

import torch

from oracle import nvfp4 as q4

TERMS = 8
E4M3_MAX = 448.0
E_MIN, E_MAX = -100, 100


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
    """Smallest E with 2688 * 2^E >= amax, clamped to [-100, 100]; 0 for amax == 0."""
    a = amax.to(torch.float64)
    pos = a > 0
    e = torch.ceil(torch.log2(torch.where(pos, a, torch.ones_like(a)) / 2688.0))
    e = torch.where(2688.0 * torch.pow(2.0, e - 1) >= a, e - 1, e)
    e = torch.where(2688.0 * torch.pow(2.0, e) < a, e + 1, e)
    e = torch.where(pos, e.clamp(E_MIN, E_MAX), torch.zeros_like(e))
    return e.to(torch.int32)


_MIDS = (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0)    # between e2m1 magnitudes i and i + 1


def e2m1_exact(ratio: torch.Tensor) -> torch.Tensor:
    """e2m1 code of a float64 quotient, round to nearest, ties to the even code."""
    a = ratio.abs()
    i = torch.zeros_like(a, dtype=torch.int64)
    for j, m in enumerate(_MIDS):
        i += (a >= m).to(torch.int64) if j % 2 else (a > m).to(torch.int64)
    sign = torch.signbit(ratio).to(torch.int64) << 3
    return (i | sign).to(torch.uint8)


def decompose(v: torch.Tensor, terms: int = TERMS, exp: torch.Tensor | None = None):
    """v float32 [n, K] (K % 16 == 0) -> (codes uint8 [n, T, K] nibbles,
    scales uint8 [n, T, K/16] e4m3 bytes, E int32 [n]); exp overrides E."""
    n, k = v.shape
    r = v.to(torch.float32).to(torch.float64).clone()
    e = exponent_for(v.abs().amax(dim=1)) if exp is None else exp.to(torch.int32)
    codes = torch.zeros(n, terms, k, dtype=torch.uint8)
    scales = torch.zeros(n, terms, k // 16, dtype=torch.uint8)
    for t in range(terms):
        g = torch.pow(2.0, (e - 2 * t).to(torch.float64)).view(n, 1)
        amax_b = r.view(n, k // 16, 16).abs().amax(dim=2)
        sb = e4m3_round_up(amax_b / (6.0 * g))
        s = q4.e4m3_decode(sb).to(torch.float64)
        sg = (s * g).repeat_interleave(16, dim=1)
        ratio = r / torch.where(sg > 0, sg, torch.ones_like(sg))
        c = torch.where(sg > 0, e2m1_exact(ratio), torch.zeros_like(r, dtype=torch.uint8))
        codes[:, t] = c
        scales[:, t] = sb
        r = r - q4.e2m1_decode(c).to(torch.float64) * sg
    return codes, scales, e


def shift_scales(scales: torch.Tensor, shift: torch.Tensor) -> torch.Tensor:
    """e4m3 bytes divided by 2^shift (shift >= 0, broadcast), rounded to nearest even."""
    val = q4.e4m3_decode(scales).to(torch.float64) * torch.pow(2.0, -shift.to(torch.float64))
    return q4.e4m3_encode(val.to(torch.float32))


def decompose_tiles(v: torch.Tensor, tile: int = 64, terms: int = TERMS):
    """Tile-local decomposition (each `tile` columns with their own exponent), then
    every tile's scales shifted to the largest exponent. Returns (codes, scales, E)."""
    n, k = v.shape
    parts = [decompose(v[:, i:i + tile], terms) for i in range(0, k, tile)]
    eloc = torch.stack([p[2] for p in parts], dim=1)                 # [n, tiles]
    emax = eloc.max(dim=1).values
    codes = torch.cat([p[0] for p in parts], dim=2)
    scales = torch.cat([shift_scales(p[1], (emax - eloc[:, i]).view(n, 1, 1)) for i, p in enumerate(parts)], dim=2)
    return codes, scales, emax


def reconstruct(codes: torch.Tensor, scales: torch.Tensor, e: torch.Tensor) -> torch.Tensor:
    """Sum of the terms in float64 [n, K]."""
    n, t_, k = codes.shape
    out = torch.zeros(n, k, dtype=torch.float64)
    for t in range(t_):
        g = torch.pow(2.0, (e - 2 * t).to(torch.float64)).view(n, 1)
        s = q4.e4m3_decode(scales[:, t]).to(torch.float64).repeat_interleave(16, dim=1)
        out += q4.e2m1_decode(codes[:, t]).to(torch.float64) * s * g
    return out


# ---------------------------------------------------------------- unscaled x terms
# The activation row x of the gate/up products enters the MMA as 16 residual
# e2m1 terms with no block scale (the MMA's B scales are all 1.0):
#   E = the smallest integer with 6 * 2^E >= amax(x) (0 when x == 0), clamped to
#       [-90, 100]; G_t = 2^(E - 2t);
#   q_t = e2m1 round-to-nearest-even (ties to the even code) of r_t / G_t (exact:
#       G_t is a power of two; |r_t / G_t| <= 6 always);
#   r_{t+1} = r_t - G_t q_t (exact). |r_T| <= G_{T-1}.
X_TERMS = 16
XE_MIN, XE_MAX = -90, 100


def x_exponent(amax: torch.Tensor) -> torch.Tensor:
    a = amax.to(torch.float64)
    pos = a > 0
    e = torch.ceil(torch.log2(torch.where(pos, a, torch.ones_like(a)) / 6.0))
    e = torch.where(6.0 * torch.pow(2.0, e - 1) >= a, e - 1, e)
    e = torch.where(6.0 * torch.pow(2.0, e) < a, e + 1, e)
    e = torch.where(pos, e.clamp(XE_MIN, XE_MAX), torch.zeros_like(e))
    return e.to(torch.int32)


def decompose_x(v: torch.Tensor, terms: int = X_TERMS):
    """v float32 [n, K] -> (codes uint8 [n, T, K] nibbles, E int32 [n])."""
    n, k = v.shape
    r = v.to(torch.float32).to(torch.float64).clone()
    e = x_exponent(v.abs().amax(dim=1))
    codes = torch.zeros(n, terms, k, dtype=torch.uint8)
    for t in range(terms):
        g = torch.pow(2.0, (e - 2 * t).to(torch.float64)).view(n, 1)
        c = e2m1_exact(r / g)
        codes[:, t] = c
        r = r - q4.e2m1_decode(c).to(torch.float64) * g
    return codes, e


def reconstruct_x(codes: torch.Tensor, e: torch.Tensor) -> torch.Tensor:
    n, t_, k = codes.shape
    out = torch.zeros(n, k, dtype=torch.float64)
    for t in range(t_):
        g = torch.pow(2.0, (e - 2 * t).to(torch.float64)).view(n, 1)
        out += q4.e2m1_decode(codes[:, t]).to(torch.float64) * g
    return out
