"""CPU model of the residual e2m1 term decomposition the tensor-core decode path
feeds to `tcgen05.mma.kind::mxf4nvf4` as its activation operands (test
infrastructure; the kernel's own arithmetic, so tests can compare its buffers
bit for bit).

Both activation operands enter the MMA as 16 residual e2m1 terms with no block
scale (the MMA's B-side scales are all 1.0), one exponent per vector:

  * x (one activation row of the gate/up products): E = the smallest integer
    with 6 * 2^E >= amax(x) (0 when x == 0), clamped to [-90, 100];
  * the SwiGLU output of one routed pair (down products): each 64-column tile
    first gets its own E_loc = the smallest EVEN integer with 6 * 2^E_loc >=
    amax(tile) (-90 when the tile is zero), clamped to [-90, 100]; then every
    tile is moved to the pair's largest exponent E by d = (E - E_loc) / 2 whole
    terms (term t becomes term t + d, the last d terms drop out);
  * G_t = 2^(E - 2t); q_t = e2m1 round-to-nearest, ties to the even code, of the
    exact quotient r_t / G_t (|r_t / G_t| <= 6 always); r_{t+1} = r_t - G_t q_t
    (exact in fp32). |r_T| <= G_{T-1}.
"""

from __future__ import annotations

import torch

from oracle import nvfp4 as q4

_MIDS = (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0)    # between e2m1 magnitudes i and i + 1


def e2m1_exact(ratio: torch.Tensor) -> torch.Tensor:
    """e2m1 code of a float64 quotient, round to nearest, ties to the even code."""
    a = ratio.abs()
    i = torch.zeros_like(a, dtype=torch.int64)
    for j, m in enumerate(_MIDS):
        i += (a >= m).to(torch.int64) if j % 2 else (a > m).to(torch.int64)
    sign = torch.signbit(ratio).to(torch.int64) << 3
    return (i | sign).to(torch.uint8)


X_TERMS = 16
XE_MIN, XE_MAX = -90, 100
AE_MIN, AE_MAX = -90, 100


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


def act_exponent(amax: torch.Tensor) -> torch.Tensor:
    """Smallest even E with 6 * 2^E >= amax, clamped to [-90, 100]; -90 for amax == 0."""
    e = x_exponent(amax).to(torch.int64)
    e = e + (e & 1)
    e = torch.where(amax.to(torch.float64) > 0, e.clamp(AE_MIN, AE_MAX), torch.full_like(e, AE_MIN))
    return e.to(torch.int32)


def _digits(v: torch.Tensor, e: torch.Tensor, terms: int) -> torch.Tensor:
    n, k = v.shape
    r = v.to(torch.float32).to(torch.float64).clone()
    codes = torch.zeros(n, terms, k, dtype=torch.uint8)
    for t in range(terms):
        g = torch.pow(2.0, (e - 2 * t).to(torch.float64)).view(n, 1)
        c = e2m1_exact(r / g)
        codes[:, t] = c
        r = r - q4.e2m1_decode(c).to(torch.float64) * g
    return codes


def decompose_act(v: torch.Tensor, tile: int = 64, terms: int = X_TERMS):
    """SwiGLU output v float32 [n, W] -> (codes uint8 [n, T, W] at the common
    exponent, E int32 [n], per-tile E_loc int32 [n, tiles])."""
    n, w = v.shape
    starts = list(range(0, w, tile))
    eloc = torch.stack([act_exponent(v[:, i:i + tile].abs().amax(dim=1)) for i in starts], dim=1)
    e = eloc.max(dim=1).values
    out = []
    for j, i in enumerate(starts):
        c = _digits(v[:, i:i + tile], eloc[:, j], terms)
        d = ((e - eloc[:, j]) // 2).tolist()
        sh = torch.zeros_like(c)
        for row, dr in enumerate(d):
            if dr < terms:
                sh[row, dr:] = c[row, :terms - dr]
        out.append(sh)
    return torch.cat(out, dim=2), e, eloc
